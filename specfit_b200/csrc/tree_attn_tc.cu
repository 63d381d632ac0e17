// K6 on tensor cores: tree-masked GQA attention with tcgen05/TMEM.
//
// Same contract as tree_attn.cu (SDPA under the verification mask,
// transformers/models/qwen3_moe/modeling_qwen3_moe.py:172-186 with the mask of
// src/specfit/runtime/eagle3_types.py:450-473), for head_dim 128 and key
// ranges up to 8192.  One CTA = one query head x 128 query rows x one range of
// 256 keys ("split"); splits are merged by tree_attn_merge_kernel.
//
//   1. TMA loads the Q tile [128 rows x 128 d] and the K range [256 keys x
//      128 d] as two 64-wide K-major chunks each (128-byte swizzle); all
//      threads meanwhile load V [256 keys x 128 d] and store it transposed
//      (V^T: d rows x key columns) in the same K-major swizzled layout.
//   2. One thread issues S = Q K^T (M 128, N <= 256, K 128) into TMEM.
//   3. Four warps, one query row per thread, read S from TMEM twice: row max
//      over visible keys, then p = exp(scale*s - max) written as bf16 into the
//      K buffer (no longer needed), row sum kept in fp32.
//   4. One thread issues O = P V (M 128, N 128, K = keys) into TMEM.
//   5. The four warps write the unnormalised O row, max and sum (the split
//      partials the merge kernel combines).
//
// Every barrier wait is bounded; on a timeout the CTA records the error in
// the library's device status word and skips the rest.  No TMA multicast.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "sm100_ptx.cuh"
#include "tree_attn.h"

namespace sf {

extern __device__ int g_device_status;

namespace {

constexpr int kD = 128;
constexpr int kRowsTile = 128;
constexpr int kKeysSplit = 256;
constexpr int kThreads = 192;
constexpr int kQChunk = kRowsTile * 64 * 2;    // 16 KB
constexpr int kKChunk = kKeysSplit * 64 * 2;   // 32 KB
constexpr int kVtChunk = kD * 64 * 2;          // 16 KB: 128 d rows x 64 keys
constexpr int kPChunk = kRowsTile * 64 * 2;    // 16 KB: 128 q rows x 64 keys
constexpr int kTmemCols = 512;                 // S: [0, 256), O: [256, 384)

struct __align__(8) TailSmem {
  uint64_t tma_bar, s_bar, p_bar, o_bar;
  uint32_t tmem_base;
  int abort_flag;
  int go;
};

constexpr size_t kSmemBytes = 1024 + 2 * kQChunk + 2 * kKChunk + 4 * kVtChunk + sizeof(TailSmem);

__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Byte offset of 16-byte unit `u` (0..7) of row `r` in a K-major 128B-swizzled
// chunk whose rows are 128 bytes.
__device__ __forceinline__ uint32_t sw128(uint32_t r, uint32_t u) {
  return r * 128u + ((u ^ (r & 7u)) << 4);
}

__global__ void __launch_bounds__(kThreads, 1)
tree_attn_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* q_s = base;                          // 2 chunks
  uint8_t* kp_s = q_s + 2 * kQChunk;            // K: 2 chunks of 32 KB; later P: 4 chunks of 16 KB
  uint8_t* vt_s = kp_s + 2 * kKChunk;           // 4 chunks
  TailSmem* tail = reinterpret_cast<TailSmem*>(vt_s + 4 * kVtChunk);
  volatile int* abort_flag = &tail->abort_flag;

  const int head = blockIdx.x;
  const int kvh = head / p.group;
  const int t0 = blockIdx.y * kRowsTile;
  const int split = blockIdx.z;
  const int key_lo = split * kKeysSplit;
  const int nkeys = min(kKeysSplit, p.kv_len - key_lo);
  const int npad = (nkeys + 15) & ~15;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    ptx::mbar_init(&tail->tma_bar, 1);
    ptx::mbar_init(&tail->s_bar, 1);
    ptx::mbar_init(&tail->p_bar, 128);
    ptx::mbar_init(&tail->o_bar, 1);
    tail->abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc(&tail->tmem_base, kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = tail->tmem_base;
  const uint32_t tmem_s = tmem, tmem_o = tmem + 256;

  if (threadIdx.x == 0) {
    ptx::mbar_arrive_expect_tx(&tail->tma_bar, 2 * kQChunk + 2 * kKChunk);
    for (int c = 0; c < 2; ++c) {
      ptx::tma_load_3d(q_s + c * kQChunk, &tm_q, &tail->tma_bar, c * 64, t0, head);
      ptx::tma_load_3d(kp_s + c * kKChunk, &tm_k, &tail->tma_bar, c * 64, key_lo, kvh);
    }
  }

  // V^T: 8x8 blocks (8 keys x 8 d), loaded as 8 rows of 16 bytes, transposed
  // in registers, stored as 8 rows (d) of 8 keys.  Keys past kv_len are zero.
  {
    const __nv_bfloat16* vbase = p.v + (int64_t)kvh * p.kv_hs;
    for (int unit = threadIdx.x; unit < (kKeysSplit / 8) * (kD / 8); unit += kThreads) {
      const int kb = unit % (kKeysSplit / 8);   // key block (8 keys)
      const int db = unit / (kKeysSplit / 8);   // d block (8 dims)
      uint32_t in[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int key = key_lo + kb * 8 + i;
        uint4 v4 = make_uint4(0, 0, 0, 0);
        if (key < p.kv_len)
          v4 = *reinterpret_cast<const uint4*>(vbase + (int64_t)key * p.kv_rs + db * 8);
        in[i][0] = v4.x; in[i][1] = v4.y; in[i][2] = v4.z; in[i][3] = v4.w;
      }
      const int chunk = kb / 8, u = kb % 8;
#pragma unroll
      for (int j = 0; j < 8; ++j) {   // d = db*8 + j
        const uint32_t sel = (j & 1) ? 0x7632u : 0x5410u;
        uint4 out;
        out.x = __byte_perm(in[0][j >> 1], in[1][j >> 1], sel);
        out.y = __byte_perm(in[2][j >> 1], in[3][j >> 1], sel);
        out.z = __byte_perm(in[4][j >> 1], in[5][j >> 1], sel);
        out.w = __byte_perm(in[6][j >> 1], in[7][j >> 1], sel);
        const uint32_t d = db * 8 + j;
        *reinterpret_cast<uint4*>(vt_s + chunk * kVtChunk + sw128(d, u)) = out;
      }
    }
  }
  fence_async_smem();
  __syncthreads();

  if (warp == 1 && lane == 0) {
    // S = Q K^T
    bool ok = ptx::mbar_wait(&tail->tma_bar, 0, abort_flag);
    if (ok) {
      ptx::tc_fence_after();
      const uint32_t idesc = ptx::idesc_bf16_f32(kRowsTile, npad);
      for (int c = 0; c < 2; ++c) {
        const uint64_t ad = ptx::smem_desc_k_sw128(ptx::smem_u32(q_s + c * kQChunk));
        const uint64_t bd = ptx::smem_desc_k_sw128(ptx::smem_u32(kp_s + c * kKChunk));
#pragma unroll
        for (int k = 0; k < 4; ++k)
          ptx::umma_f16(tmem_s, ad + 2 * k, bd + 2 * k, idesc, (c | k) != 0);
      }
    }
    ptx::umma_commit(&tail->s_bar);  // fires even when nothing was issued
    // O = P V
    ok = ok && ptx::mbar_wait(&tail->p_bar, 0, abort_flag);
    if (ok) {
      ptx::tc_fence_after();
      const uint32_t idesc = ptx::idesc_bf16_f32(kRowsTile, kD);
      const int kchunks = (nkeys + 63) / 64;
      for (int c = 0; c < kchunks; ++c) {
        const uint64_t ad = ptx::smem_desc_k_sw128(ptx::smem_u32(kp_s + c * kPChunk));
        const uint64_t bd = ptx::smem_desc_k_sw128(ptx::smem_u32(vt_s + c * kVtChunk));
#pragma unroll
        for (int k = 0; k < 4; ++k)
          ptx::umma_f16(tmem_o, ad + 2 * k, bd + 2 * k, idesc, (c | k) != 0);
      }
    }
    ptx::umma_commit(&tail->o_bar);
  } else if (warp >= 2) {
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // query row within the tile = TMEM lane
    const int t = t0 + r;
    const bool row_ok = t < p.q_len;
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    ptx::mbar_wait(&tail->s_bar, 0, abort_flag);
    ptx::named_bar_sync(1, 128);
    if (threadIdx.x == 64) tail->go = !*abort_flag;
    ptx::named_bar_sync(1, 128);
    const bool go = tail->go;
    float m = -INFINITY, l = 0.f;
    if (go) {
      ptx::tc_fence_after();
      const uint32_t* bits = p.bits + (int64_t)(row_ok ? t : 0) * p.bit_words;
      auto visible = [&](int key) -> bool {
        if (!row_ok || key >= p.kv_len) return false;
        if (key < p.prefix_len) return true;
        const int j = key - p.prefix_len;
        return (bits[j >> 5] >> (j & 31)) & 1u;
      };
      // Pass 1: row max of the visible scaled scores.
      for (int c0 = 0; c0 < npad; c0 += 16) {
        float v[16];
        ptx::tmem_ld_16(tmem_s + lane_off + c0, v);
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if (visible(key_lo + c0 + i)) m = fmaxf(m, v[i] * p.scale);
      }
      // Pass 2: probabilities (bf16 into the P chunks), fp32 row sum.
      for (int c0 = 0; c0 < kKeysSplit; c0 += 16) {
        float v[16];
        if (c0 < npad) ptx::tmem_ld_16(tmem_s + lane_off + c0, v);
        uint32_t packed[8];
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          float a = 0.f, b = 0.f;
          if (c0 < npad && m != -INFINITY) {
            if (visible(key_lo + c0 + i)) a = __expf(v[i] * p.scale - m);
            if (visible(key_lo + c0 + i + 1)) b = __expf(v[i + 1] * p.scale - m);
          }
          l += a + b;
          __nv_bfloat162 h2 = __floats2bfloat162_rn(a, b);
          packed[i / 2] = *reinterpret_cast<uint32_t*>(&h2);
        }
        const int chunk = c0 / 64, u = (c0 % 64) / 8;
        uint8_t* dst = kp_s + chunk * kPChunk;
        *reinterpret_cast<uint4*>(dst + sw128(r, u)) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
        *reinterpret_cast<uint4*>(dst + sw128(r, u + 1)) = make_uint4(packed[4], packed[5], packed[6], packed[7]);
      }
      fence_async_smem();
      ptx::tc_fence_before();
    }
    ptx::mbar_arrive(&tail->p_bar);
    if (go && ptx::mbar_wait(&tail->o_bar, 0, abort_flag)) {
      ptx::tc_fence_after();
      if (row_ok) {
        const int64_t idx = ((int64_t)split * p.num_heads + head) * p.q_len + t;
        float* dst = p.part_o + idx * kD;
        for (int c0 = 0; c0 < kD; c0 += 16) {
          float v[16];
          ptx::tmem_ld_16(tmem_o + lane_off + c0, v);
#pragma unroll
          for (int i = 0; i < 16; i += 4)
            *reinterpret_cast<float4*>(dst + c0 + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
        }
        p.part_ml[idx * 2] = m;
        p.part_ml[idx * 2 + 1] = l;
      } else {
        // Keep the warp converged for the TMEM loads of the other rows.
        for (int c0 = 0; c0 < kD; c0 += 16) {
          float v[16];
          ptx::tmem_ld_16(tmem_o + lane_off + c0, v);
        }
      }
    }
  }

  // Teardown: every TMA load and MMA issued above has completed once the
  // barriers below have fired (the MMA thread committed both), so TMEM can go.
  if (threadIdx.x == 0) {
    volatile int never = 0;
    ptx::mbar_wait(&tail->tma_bar, 0, &never);
  }
  if (warp == 1 && lane == 0) {
    volatile int never = 0;
    ptx::mbar_wait(&tail->o_bar, 0, &never);
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, kTmemCols);
  }
  if (threadIdx.x == 0 && tail->abort_flag) atomicExch(&g_device_status, 2);
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

int encode3d(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
             uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box1) {
  auto fn = encode_fn();
  if (!fn) return set_error(SF_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  cuuint32_t box[3] = {64, box1, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                  es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(SF_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return SF_OK;
}

}  // namespace

bool tree_attention_tc_supports(const AttnParams& p, int head_dim) {
  return head_dim == kD && p.kv_len <= 32 * kKeysSplit && p.q_rs % 8 == 0 && p.q_hs % 8 == 0 &&
         p.kv_rs % 8 == 0 && p.kv_hs % 8 == 0 && aligned16(p.q) && aligned16(p.k) && aligned16(p.v) &&
         p.q_len > 0 && p.kv_len > 0;
}

int tree_attention_tc(const AttnParams& p_in, cudaStream_t stream, int* splits_out) {
  AttnParams p = p_in;
  static std::atomic<unsigned long long> configured{0};
  if (int rc = once_per_device(configured, [] {
        SF_CHECK_CUDA(cudaFuncSetAttribute(tree_attn_tc_kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes));
        return SF_OK;
      }))
    return rc;
  CUtensorMap tm_q, tm_k;
  if (int rc = encode3d(&tm_q, p.q, kD, (uint64_t)p.q_len, (uint64_t)p.num_heads, (uint64_t)p.q_rs * 2,
                        (uint64_t)p.q_hs * 2, kRowsTile))
    return rc;
  if (int rc = encode3d(&tm_k, p.k, kD, (uint64_t)p.kv_len, (uint64_t)p.num_kv_heads,
                        (uint64_t)p.kv_rs * 2, (uint64_t)p.kv_hs * 2, kKeysSplit))
    return rc;
  p.splits = (p.kv_len + kKeysSplit - 1) / kKeysSplit;
  p.keys_per_split = kKeysSplit;
  p.part_ml = p.part_o + (size_t)p.splits * p.num_heads * p.q_len * kD;
  dim3 grid((unsigned)p.num_heads, (unsigned)((p.q_len + kRowsTile - 1) / kRowsTile), (unsigned)p.splits);
  tree_attn_tc_kernel<<<grid, kThreads, kSmemBytes, stream>>>(tm_q, tm_k, p);
  SF_CHECK_LAUNCH();
  *splits_out = p.splits;
  return SF_OK;
}

}  // namespace sf
