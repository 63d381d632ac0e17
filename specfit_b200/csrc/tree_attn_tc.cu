// K6 on tcgen05: tree-masked GQA attention with the score and output tiles
// in TMEM and K/V staged by TMA.
//
// Same contract as tree_attn.cu / tree_attn_mma.cu (SDPA under the
// verification mask; transformers/models/qwen3_moe/modeling_qwen3_moe.py:
// 172-186 with src/specfit/runtime/eagle3_types.py:450-473), head_dim 128,
// for passes with many query rows (a 64-node tree has 65 rows; its 8 query
// heads per KV head give 520 packed rows), where the attention FLOPs, not the
// K/V bytes, bound the warp-level kernel.
//
// A CTA owns one KV head, 128 packed query rows (the MMA's M; row =
// head_in_group * Tq + t, as in tree_attn_mma.cu) and one key range (a
// split), which it walks in blocks of 128 keys:
//   warp 0      TMA producer (one lane): K and V blocks of 128 keys x 128 d,
//               two 64-d regions each with 128-byte swizzling, 2 stages;
//   warp 1      TMEM allocator and MMA issuer (one lane):
//                 S = Q K^T    (M 128, N 128 keys, K 128 d; Q and K K-major)
//                 O_j = P V    (M 128, N 128 d, K 128 keys; P K-major, V
//                               MN-major: V rows are keys with d contiguous);
//   warps 2..9  two threads per packed row (the TMEM lane; warps w and
//               w + 4 share a lane quadrant), each owning half of the row's
//               key columns and half of its output dims: Q half-row ->
//               shared memory; per block, S half-row from TMEM, tree mask,
//               online softmax in fp32 (the two halves' row max and row sum
//               exchanged through shared memory, the sum added in half
//               order), P half-row (bf16) -> shared memory; then
//               O = O * exp(m_old - m_new) + O_j over its 64 dims in registers.
// TMEM: S_j in columns [0, 128) or [128, 256) by the parity of j, O_j in
// [256, 384).  The MMA warp issues S_{j+1} = Q K_{j+1}^T before O_j = P_j V_j,
// so the next block's scores are computed while the softmax warps finish
// block j.  S_{j+1} reuses S_{j-1}'s columns, read before P_{j-1} was
// published; P_{j+1} is written after O_j has been read back (so after the
// O_j MMA read P_j); O_j is read back before P_{j+1} is published.
//
// Output: with one split the CTA normalises and writes bf16 [Tq, Hq, D];
// otherwise it writes unnormalised O and (row max, row sum) per split for
// tree_attn_merge_kernel, in tree_attn_mma.cu's format.  Every barrier wait
// is bounded (sm100_ptx.cuh); a wait that gives up records its site in this
// file's status word and the CTA drains its own copies and MMAs and returns.
// Every TMA load here is issued by one CTA for its own shared memory.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>

#include "common.cuh"
#include "sm100_ptx.cuh"
#include "swiglu.h"
#include "tree_attn.h"

namespace sf {
namespace {

__device__ int g_attn_tc_status;

constexpr int kD = 128;
constexpr int kBM = 128;                       // packed query rows per CTA (MMA M)
constexpr int kKB = 128;                       // keys per block
constexpr int kStages = 2;
constexpr int kThreads = 320;                  // 2 + 8 warps
constexpr int kMaxSplits = 32;                 // the workspace of sf_tree_attention covers 32
constexpr int kRegion = 128 * 128;             // one 64-element column region of a 128-row tile (B)
constexpr int kQBytes = 2 * kRegion;           // Q: 128 rows x 128 d
constexpr int kPBytes = 2 * kRegion;           // P: 128 rows x 128 keys
constexpr int kKBytes = 2 * kRegion;           // one K block: 128 keys x 128 d
constexpr int kStageBytes = 2 * kKBytes;       // K and V
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kSCol = 0, kOCol = 256;  // S_j at kSCol + (j & 1) * 128

struct __align__(8) Tail {
  uint64_t kv_full[kStages];
  uint64_t kv_empty[kStages];
  uint64_t q_ready;
  uint64_t s_full[2];
  uint64_t p_full;
  uint64_t o_full;
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort_flag;
  float red_max[2][kBM];  // per half: the half-row's max of visible scaled scores
  float red_sum[2][kBM];  // per half: the half-row's sum of probabilities
  int pair_ok[3][2][4];   // per exchange point, half and lane quadrant: the warp's wait succeeded
};

constexpr size_t kSmemBytes =
    1024 /*alignment slack*/ + kQBytes + kPBytes + (size_t)kStages * kStageBytes + sizeof(Tail);

// Byte offset of 16-byte chunk c (0..15 along the row) of row r in a
// [128 rows x 128 bf16] K-major tile kept as two 64-element column regions
// of 128-byte rows with the 128-byte swizzle (the layout TMA writes, and the
// one smem_desc_k_sw128 describes): chunk c & 7 of row r lands at chunk
// (c & 7) ^ (r & 7) of the row.
__device__ __forceinline__ uint32_t sw128_offset(int r, int c) {
  return (uint32_t)((c >> 3) * kRegion + (r >> 3) * 1024 + (r & 7) * 128 + (((c & 7) ^ (r & 7)) << 4));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Descriptor offsets (16-byte units) of the 16-wide K step k (0..7) inside a
// K-major two-region tile: region k / 4, then 32 bytes per step in its rows.
__device__ __forceinline__ uint64_t kstep_offset(int k) {
  return (uint64_t)(((k >> 2) * kRegion + (k & 3) * 32) >> 4);
}

__global__ void __launch_bounds__(kThreads, 1)
tree_attn_tc_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                    AttnParams p, __nv_bfloat16* __restrict__ out, int direct) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* q_s = smem;
  uint8_t* p_s = q_s + kQBytes;
  uint8_t* kv_s = p_s + kPBytes;
  Tail* tail = reinterpret_cast<Tail*>(kv_s + (size_t)kStages * kStageBytes);
  volatile int* abort_flag = &tail->abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kvh = blockIdx.x, tile = blockIdx.y;
  const int req = blockIdx.z / p.splits, split = blockIdx.z % p.splits;  // request, key range
  const int packed_rows = p.group * p.q_len;
  const int key_lo = split * p.keys_per_split;
  const int key_hi = min(p.kv_len, key_lo + p.keys_per_split);
  const int nblocks = key_hi > key_lo ? (key_hi - key_lo + kKB - 1) / kKB : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      ptx::mbar_init(&tail->kv_full[s], 1);
      ptx::mbar_init(&tail->kv_empty[s], 1);
    }
    ptx::mbar_init(&tail->q_ready, 256);
    ptx::mbar_init(&tail->s_full[0], 1);
    ptx::mbar_init(&tail->s_full[1], 1);
    ptx::mbar_init(&tail->p_full, 256);
    ptx::mbar_init(&tail->o_full, 1);
    ptx::mbar_init(&tail->mma_done, 1);
    tail->abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tensormap(&tm_k);
    ptx::prefetch_tensormap(&tm_v);
  }
  if (warp == 1) {
    ptx::tmem_alloc(&tail->tmem_base, kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = tail->tmem_base;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int j = 0;
      for (; j < nblocks; ++j) {
        const int s = j % kStages;
        const uint32_t ph = (j / kStages) & 1;
        if (!ptx::mbar_wait(&tail->kv_empty[s], ph ^ 1, abort_flag, &g_attn_tc_status, 1)) break;
        ptx::mbar_arrive_expect_tx(&tail->kv_full[s], kStageBytes);
        uint8_t* st = kv_s + (size_t)s * kStageBytes;
        const int key0 = key_lo + j * kKB;
        ptx::tma_load_4d(st, &tm_k, &tail->kv_full[s], 0, key0, kvh, req);
        ptx::tma_load_4d(st + kRegion, &tm_k, &tail->kv_full[s], 64, key0, kvh, req);
        ptx::tma_load_4d(st + kKBytes, &tm_v, &tail->kv_full[s], 0, key0, kvh, req);
        ptx::tma_load_4d(st + kKBytes + kRegion, &tm_v, &tail->kv_full[s], 64, key0, kvh, req);
      }
      // Let every load this thread issued land before the CTA can exit.
      volatile int never = 0;
      for (int i = max(0, j - kStages); i < j; ++i)
        ptx::mbar_wait(&tail->kv_full[i % kStages], (i / kStages) & 1, &never, &g_attn_tc_status, 2);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc_s = ptx::idesc_bf16_f32(kBM, kKB);
      const uint32_t idesc_o = ptx::idesc_bf16_f32(kBM, kD) | ptx::kIdescBMajorMN;
      const uint64_t qdesc = ptx::smem_desc_k_sw128(ptx::smem_u32(q_s));
      const uint64_t pdesc = ptx::smem_desc_k_sw128(ptx::smem_u32(p_s));
      bool ok = nblocks == 0 || ptx::mbar_wait(&tail->q_ready, 0, abort_flag, &g_attn_tc_status, 3);
      // S_j = Q K_j^T into the S buffer of j's parity.
      auto issue_s = [&](int j) -> bool {
        const int s = j % kStages;
        if (!ptx::mbar_wait(&tail->kv_full[s], (j / kStages) & 1, abort_flag, &g_attn_tc_status, 4)) return false;
        ptx::tc_fence_after();
        const uint64_t kdesc = ptx::smem_desc_k_sw128(ptx::smem_u32(kv_s + (size_t)s * kStageBytes));
        const uint32_t scol = kSCol + (uint32_t)(j & 1) * 128;
#pragma unroll
        for (int k = 0; k < kD / 16; ++k)
          ptx::umma_f16(tmem + scol, qdesc + kstep_offset(k), kdesc + kstep_offset(k), idesc_s, k != 0);
        ptx::umma_commit(&tail->s_full[j & 1]);
        return true;
      };
      if (ok && nblocks > 0) ok = issue_s(0);
      for (int j = 0; ok && j < nblocks; ++j) {
        const int s = j % kStages;
        const uint32_t st = ptx::smem_u32(kv_s + (size_t)s * kStageBytes);
        // The next block's scores first (its buffer's last reader, the
        // softmax of block j - 1, published P_{j-1} before O_{j-1} was issued).
        if (j + 1 < nblocks && !issue_s(j + 1)) break;
        if (!ptx::mbar_wait(&tail->p_full, j & 1, abort_flag, &g_attn_tc_status, 5)) break;
        ptx::tc_fence_after();
        // V block as the MN-major B operand: 16 keys (two 8-key atoms,
        // 2,048 B) per K step; its second 64-d region is kRegion further on.
        const uint64_t vdesc = ptx::smem_desc_mn_sw128(st + kKBytes, kRegion);
#pragma unroll
        for (int k = 0; k < kKB / 16; ++k)
          ptx::umma_f16(tmem + kOCol, pdesc + kstep_offset(k), vdesc + (uint64_t)((k * 16 * 128) >> 4),
                        idesc_o, k != 0);
        ptx::umma_commit(&tail->o_full);
        ptx::umma_commit(&tail->kv_empty[s]);
      }
      // Drain: the barrier fires once every MMA issued above has completed.
      ptx::umma_commit(&tail->mma_done);
      volatile int never = 0;
      ptx::mbar_wait(&tail->mma_done, 0, &never, &g_attn_tc_status, 6);
    }
  } else {
    // ---------------- softmax / epilogue (warps 2..9) ----------------
    const int quad = warp & 3;          // TMEM lane quadrant this warp may access
    const int half = (warp - 2) >> 2;   // 0: keys / dims 0..63 of the row, 1: 64..127
    const int r = quad * 32 + lane;     // tile row == TMEM lane
    const int pr = tile * kBM + r;      // packed row
    const bool rok = pr < packed_rows;
    const int t = rok ? pr % p.q_len : 0;
    const int head = kvh * p.group + (rok ? pr / p.q_len : 0);
    const uint32_t pair_bar = 1 + quad;  // named barrier of the two warps of this quadrant
    // Both warps of a quadrant take the same go / stop decision at each
    // exchange point (a warp that stopped alone would leave its partner
    // waiting at the named barrier).
    auto pair_agree = [&](int point, bool mine) -> bool {
      if (lane == 0) tail->pair_ok[point][half][quad] = mine ? 1 : 0;
      ptx::named_bar_sync(pair_bar, 64);
      return tail->pair_ok[point][0][quad] && tail->pair_ok[point][1][quad];
    };

    // Q half-row -> shared memory in the swizzled K-major layout (zeros past the rows).
    {
      const __nv_bfloat16* qrow = p.q + (int64_t)req * p.q_bs + (int64_t)head * p.q_hs + (int64_t)t * p.q_rs;
#pragma unroll 4
      for (int c = half * (kD / 16); c < (half + 1) * (kD / 16); ++c) {
        const uint4 v = rok ? *reinterpret_cast<const uint4*>(qrow + c * 8) : make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(q_s + sw128_offset(r, c)) = v;
      }
      ptx::fence_proxy_async_smem();
      ptx::mbar_arrive(&tail->q_ready);
    }

    const uint32_t trow = tmem + ((uint32_t)(quad * 32) << 16);
    const uint32_t* rbits = p.bits ? p.bits + (int64_t)req * p.bits_bs + (int64_t)t * p.bit_words : nullptr;
    constexpr int kHalf = kD / 2;
    float o[kHalf];
#pragma unroll
    for (int i = 0; i < kHalf; ++i) o[i] = 0.f;
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nblocks; ++j) {
      // Visibility of this half's 64 keys of the block for this row.
      uint64_t win;
      {
        const int kb = key_lo + j * kKB + 64 * half;
        uint64_t w;
        if (rbits) {
          w = tree_mask_window(rbits, p.bit_words, kb - p.prefix_len);
        } else {
          w = kb + 64 <= p.prefix_len ? ~0ull
                                      : (kb >= p.prefix_len ? 0ull : (1ull << (p.prefix_len - kb)) - 1);
        }
        const int valid = key_hi - kb;  // keys of this window inside the split
        if (valid < 64) w &= valid <= 0 ? 0ull : ((1ull << valid) - 1);
        win = rok ? w : 0ull;
      }

      ok = __all_sync(0xffffffffu, ptx::mbar_wait(&tail->s_full[j & 1], (j >> 1) & 1, abort_flag,
                                                  &g_attn_tc_status, 7));
      if (ok) ptx::tc_fence_after();
      const uint32_t scol = kSCol + (uint32_t)(j & 1) * 128;

      // Pass 1: the half-row max of the visible scaled scores, then the row's.
      float mx = -INFINITY;
      if (ok) {
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          float sv[16];
          ptx::tmem_ld_16(trow + scol + half * 64 + c * 16, sv);
          const uint32_t bits16 = (uint32_t)(win >> (c * 16)) & 0xFFFFu;
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if ((bits16 >> i) & 1u) mx = fmaxf(mx, sv[i] * p.scale);
        }
      }
      tail->red_max[half][r] = mx;
      if (!pair_agree(0, ok)) {
        ok = false;
        break;
      }
      const float mnew = fmaxf(m, fmaxf(tail->red_max[0][r], tail->red_max[1][r]));
      const float alpha = (m == -INFINITY) ? 0.f : __expf(m - mnew);

      // Pass 2: probabilities, their fp32 half-row sum, and the bf16 P half-row.
      float sum = 0.f;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float sv[16];
        ptx::tmem_ld_16(trow + scol + half * 64 + c * 16, sv);
        const uint32_t bits16 = (uint32_t)(win >> (c * 16)) & 0xFFFFu;
        uint32_t pk[8];
#pragma unroll
        for (int i = 0; i < 16; i += 2) {
          const float p0 = ((bits16 >> i) & 1u) ? __expf(sv[i] * p.scale - mnew) : 0.f;
          const float p1 = ((bits16 >> (i + 1)) & 1u) ? __expf(sv[i + 1] * p.scale - mnew) : 0.f;
          sum += p0 + p1;
          pk[i / 2] = pack_bf16x2(p0, p1);
        }
        const int cc = half * 8 + 2 * c;  // 16-byte chunk of the P row
        *reinterpret_cast<uint4*>(p_s + sw128_offset(r, cc)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        *reinterpret_cast<uint4*>(p_s + sw128_offset(r, cc + 1)) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
      }
      tail->red_sum[half][r] = sum;
      ptx::fence_proxy_async_smem();
      ptx::tc_fence_before();
      ptx::mbar_arrive(&tail->p_full);
      ptx::named_bar_sync(pair_bar, 64);  // both halves' sums are in shared memory
      l = l * alpha + (tail->red_sum[0][r] + tail->red_sum[1][r]);
      m = mnew;

      ok = __all_sync(0xffffffffu, ptx::mbar_wait(&tail->o_full, j & 1, abort_flag, &g_attn_tc_status, 8));
      if (!pair_agree(1, ok)) {
        ok = false;
        break;
      }
      ptx::tc_fence_after();
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float ov[16];
        ptx::tmem_ld_16(trow + kOCol + half * 64 + c * 16, ov);
#pragma unroll
        for (int i = 0; i < 16; ++i) o[c * 16 + i] = o[c * 16 + i] * alpha + ov[i];
      }
      ptx::tc_fence_before();
    }

    if (ok && rok) {
      if (direct) {
        const float inv = l > 0.f ? 1.f / l : 0.f;
        __nv_bfloat16* dst = out + (int64_t)req * p.out_bs + ((int64_t)t * p.num_heads + head) * kD + half * kHalf;
#pragma unroll
        for (int c = 0; c < kHalf / 8; ++c) {
          uint4 v;
          v.x = pack_bf16x2(o[c * 8 + 0] * inv, o[c * 8 + 1] * inv);
          v.y = pack_bf16x2(o[c * 8 + 2] * inv, o[c * 8 + 3] * inv);
          v.z = pack_bf16x2(o[c * 8 + 4] * inv, o[c * 8 + 5] * inv);
          v.w = pack_bf16x2(o[c * 8 + 6] * inv, o[c * 8 + 7] * inv);
          *reinterpret_cast<uint4*>(dst + c * 8) = v;
        }
      } else {
        const int64_t idx = (((int64_t)req * p.splits + split) * p.num_heads + head) * p.q_len + t;
        float* dst = p.part_o + idx * kD + half * kHalf;
#pragma unroll
        for (int c = 0; c < kHalf / 4; ++c)
          *reinterpret_cast<float4*>(dst + c * 4) = make_float4(o[c * 4], o[c * 4 + 1], o[c * 4 + 2], o[c * 4 + 3]);
        if (half == 0) {
          p.part_ml[idx * 2] = m;
          p.part_ml[idx * 2 + 1] = l;
        }
      }
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

bool tree_attention_tc_supports(const AttnParams& p, int head_dim) {
  return head_dim == kD && p.group >= 1 && p.group <= 8 && p.q_len > 0 && p.kv_len > 0 &&
         p.q_rs % 8 == 0 && p.q_hs % 8 == 0 && p.kv_rs % 8 == 0 && p.kv_hs % 8 == 0 &&
         aligned16(p.q) && aligned16(p.k) && aligned16(p.v) && p.part_o != nullptr;
}

int tree_attention_tc(AttnParams& p, void* out, bool* merged, cudaStream_t stream) {
  *merged = false;
  if (!tree_attention_tc_supports(p, kD))
    return set_error(SF_ERR_UNSUPPORTED,
                     "tcgen05 tree attention needs D=128, <= 8 query heads per KV head, and 16-byte "
                     "aligned q/k/v rows");
  static std::atomic<unsigned long long> configured{0};
  if (int rc = once_per_device(configured, [] {
        int dev = 0, major = 0;
        SF_CHECK_CUDA(cudaGetDevice(&dev));
        SF_CHECK_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
        if (major != 10) return set_error(SF_ERR_UNSUPPORTED, "tcgen05 tree attention needs an sm_100 device");
        SF_CHECK_CUDA(cudaFuncSetAttribute(tree_attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)kSmemBytes));
        return SF_OK;
      }))
    return rc;

  CUtensorMap tm_k, tm_v;
  {
    // [batch][kv heads][keys][d]: a request is one more coordinate.
    const int64_t kv_bs = p.batch > 1 ? p.kv_bs : (int64_t)p.num_kv_heads * p.kv_hs;
    cuuint64_t dims[4] = {(cuuint64_t)kD, (cuuint64_t)p.kv_len, (cuuint64_t)p.num_kv_heads,
                          (cuuint64_t)p.batch};
    cuuint64_t strides[3] = {(cuuint64_t)p.kv_rs * 2, (cuuint64_t)p.kv_hs * 2, (cuuint64_t)kv_bs * 2};
    cuuint32_t box[4] = {64, kKB, 1, 1};
    if (int rc = tma_encode_bf16(&tm_k, p.k, 4, dims, strides, box)) return rc;
    if (int rc = tma_encode_bf16(&tm_v, p.v, 4, dims, strides, box)) return rc;
  }
  const int64_t row_tiles = ((int64_t)p.group * p.q_len + kBM - 1) / kBM;
  const int64_t blocks = ((int64_t)p.kv_len + kKB - 1) / kKB;
  // Splits of the key range: the count that minimises (waves of CTAs) x
  // (key blocks per CTA + a CTA's fixed cost, about two blocks: set-up, the
  // Q tile, pipeline fill, the partial write), plus a small charge per split
  // for the merge.
  const int64_t units = (int64_t)p.batch * p.num_kv_heads * row_tiles;
  const int64_t sms = num_sms();
  int64_t best = 1;
  double best_cost = 1e30;
  for (int64_t s = 1; s <= std::min<int64_t>(blocks, kMaxSplits); ++s) {
    const int64_t per = (blocks + s - 1) / s;
    const int64_t used = (blocks + per - 1) / per;  // splits that get keys
    const double cost = (double)((units * used + sms - 1) / sms) * ((double)per + 2.0) + 0.05 * (double)used;
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = s;
    }
  }
  p.keys_per_split = (int)(((blocks + best - 1) / best) * kKB);
  p.splits = (int)((p.kv_len + p.keys_per_split - 1) / p.keys_per_split);
  p.part_ml = p.part_o + (size_t)p.batch * p.splits * p.num_heads * p.q_len * kD;
  const int direct = p.splits == 1 ? 1 : 0;
  SF_CHECK_ARG(row_tiles < 65536, "too many query rows");
  SF_CHECK_ARG((int64_t)p.splits * p.batch < 65536, "too many requests for one launch");
  dim3 grid((unsigned)p.num_kv_heads, (unsigned)row_tiles, (unsigned)(p.splits * p.batch));
  SF_CHECK_CUDA(launch_pdl(tree_attn_tc_kernel, grid, dim3(kThreads), kSmemBytes, stream, tm_k, tm_v, p,
                           static_cast<__nv_bfloat16*>(out), direct));
  SF_CHECK_LAUNCH();
  *merged = direct != 0;
  return SF_OK;
}

int tree_attention_tc_status(int* status, int reset) {
  SF_CHECK_CUDA(cudaMemcpyFromSymbol(status, g_attn_tc_status, sizeof(int)));
  if (reset) {
    const int zero = 0;
    SF_CHECK_CUDA(cudaMemcpyToSymbol(g_attn_tc_status, &zero, sizeof(int)));
  }
  return SF_OK;
}

}  // namespace sf
