// K6 on warp-level tensor cores: tree-masked GQA attention, split-KV.
//
// Same contract as the CUDA-core kernel in tree_attn.cu (SDPA under the
// verification mask; transformers/models/qwen3_moe/modeling_qwen3_moe.py:
// 172-186 with src/specfit/runtime/eagle3_types.py:450-473), head_dim 128.
//
// Work decomposition: the Hq/Hkv query heads of one KV head are packed into
// one row space (row = head_in_group * Tq + t), so every staged K/V tile is
// used by all of them.  A CTA owns one KV head, 64 packed rows (4 warps x 16)
// and one key range (a "split"); it walks that range in blocks of 64 keys:
//   * K and V blocks are staged in shared memory with cp.async (rows padded
//     to 272 bytes so ldmatrix reads are bank-conflict free);
//   * S = Q K^T with mma.sync m16n8k16 (bf16 in, fp32 out); Q fragments stay
//     in registers for the whole range;
//   * the tree mask and an online softmax run on the S fragments (each row
//     is spread over the 4 lanes of a quad);
//   * P (bf16) is reused in registers as the A operand of O += P V, with V
//     fragments read transposed by ldmatrix.trans.
// The CTA writes unnormalised O plus (row max, row sum) per split; the merge
// kernel in tree_attn.cu combines the splits.  No barriers other than
// __syncthreads, no TMEM, no TMA.
#include <cooperative_groups.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "tree_attn.h"

namespace sf {
namespace {

constexpr int kD = 128;
constexpr int kWarps = 4;
constexpr int kRowsCta = 16 * kWarps;  // packed query rows per CTA
constexpr int kKeys = 64;              // keys per staged block
constexpr int kPitch = kD + 8;         // bf16 elements per staged row (272 bytes)
constexpr int kMaxSplitsMma = 32;

__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Stages keys [b0, b0 + 64) of one KV head into one K/V buffer pair with
// cp.async (one commit group); rows at or past key_hi are zero-filled.
__device__ __forceinline__ void stage_block(__nv_bfloat16* ks, __nv_bfloat16* vs,
                                            const __nv_bfloat16* kbase,
                                            const __nv_bfloat16* vbase, int64_t kv_rs, int b0,
                                            int key_hi) {
  for (int i = threadIdx.x; i < kKeys * (kD / 8); i += kWarps * 32) {
    const int r = i / (kD / 8), col = (i % (kD / 8)) * 8;
    const int key = b0 + r;
    __nv_bfloat16* kd = ks + r * kPitch + col;
    __nv_bfloat16* vd = vs + r * kPitch + col;
    if (key < key_hi) {
      const uint32_t ka = static_cast<uint32_t>(__cvta_generic_to_shared(kd));
      const uint32_t va = static_cast<uint32_t>(__cvta_generic_to_shared(vd));
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(ka),
                   "l"(kbase + (int64_t)key * kv_rs + col)
                   : "memory");
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(va),
                   "l"(vbase + (int64_t)key * kv_rs + col)
                   : "memory");
    } else {
      *reinterpret_cast<uint4*>(kd) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(vd) = make_uint4(0, 0, 0, 0);
    }
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
}

constexpr int kStageElems = kKeys * kPitch;  // one K (or V) buffer
constexpr size_t kSmemBytes = 4 * kStageElems * sizeof(__nv_bfloat16);  // 2 stages x (K, V)
// In-kernel merge: the splits of a row block form one cluster (at most 16
// CTAs); each CTA owns ceil(64 / S) of the 64 packed rows and receives every
// split's unnormalised row output and (max, sum) for them.
constexpr int kMaxFusedSplits = 16;
constexpr int kRecvRows = kRowsCta + kMaxFusedSplits;  // >= S * ceil(64 / S)
constexpr size_t kFusedSmemBytes = kSmemBytes + (size_t)kRecvRows * (kD + 2) * sizeof(float);

template <bool kFused>
__global__ void __launch_bounds__(kWarps * 32)
tree_attn_mma_kernel(AttnParams p, __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) __nv_bfloat16 smem[];

  const int kvh = blockIdx.x;
  const int split = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int packed_rows = p.group * p.q_len;
  const int key_lo = split * p.keys_per_split;
  const int key_hi = min(p.kv_len, key_lo + p.keys_per_split);

  // The two rows this thread holds: packed row -> (head, t).
  int head[2], trow[2];
  bool rok[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int pr = blockIdx.y * kRowsCta + warp * 16 + g + 8 * h;
    rok[h] = pr < packed_rows;
    const int hg = rok[h] ? pr / p.q_len : 0;
    trow[h] = rok[h] ? pr % p.q_len : 0;
    head[h] = kvh * p.group + hg;
  }

  // Q fragments for the 8 k-steps of d (16 each), kept in registers.
  uint32_t qa[8][4];
#pragma unroll
  for (int ks8 = 0; ks8 < 8; ++ks8) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const __nv_bfloat16* qrow = p.q + (int64_t)head[h] * p.q_hs + (int64_t)trow[h] * p.q_rs;
      const int d0 = ks8 * 16 + 2 * c;
      qa[ks8][h] = rok[h] ? *reinterpret_cast<const uint32_t*>(qrow + d0) : 0u;
      qa[ks8][2 + h] = rok[h] ? *reinterpret_cast<const uint32_t*>(qrow + d0 + 8) : 0u;
    }
  }

  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};

  const __nv_bfloat16* kbase = p.k + (int64_t)kvh * p.kv_hs;
  const __nv_bfloat16* vbase = p.v + (int64_t)kvh * p.kv_hs;

  const uint32_t* rbits[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) rbits[h] = p.bits ? p.bits + (int64_t)trow[h] * p.bit_words : nullptr;

  // Two-stage pipeline: block i+1 streams in while block i is computed.
  if (key_lo < key_hi) stage_block(smem, smem + kStageElems, kbase, vbase, p.kv_rs, key_lo, key_hi);
  int it = 0;
  for (int b0 = key_lo; b0 < key_hi; b0 += kKeys, ++it) {
    const __nv_bfloat16* ks = smem + (it & 1) * 2 * kStageElems;
    const __nv_bfloat16* vs = ks + kStageElems;
    if (b0 + kKeys < key_hi) {
      __nv_bfloat16* nk = smem + ((it + 1) & 1) * 2 * kStageElems;
      stage_block(nk, nk + kStageElems, kbase, vbase, p.kv_rs, b0 + kKeys, key_hi);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();

    uint64_t win[2];
#pragma unroll
    for (int h = 0; h < 2; ++h)
      win[h] = rbits[h] ? tree_mask_window(rbits[h], p.bit_words, b0 - p.prefix_len)
                        : (b0 + kKeys <= p.prefix_len ? ~0ull
                                                      : (b0 >= p.prefix_len ? 0ull
                                                                            : (1ull << (p.prefix_len - b0)) - 1));

    // S = Q K^T for this warp's 16 rows x 64 keys (8 n-tiles of 8 keys).
    float s[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
      for (int kp = 0; kp < 4; ++kp) {  // pairs of 16-wide d steps
        uint32_t kb[4];
        const int krow = nt * 8 + (lane & 7);
        const int kcol = kp * 32 + (lane >> 3) * 8;
        ldsm_x4(kb, ks + krow * kPitch + kcol);
        mma_bf16(s[nt], qa[2 * kp], kb[0], kb[1]);
        mma_bf16(s[nt], qa[2 * kp + 1], kb[2], kb[3]);
      }
    }

    // Mask, online softmax (a row lives on the 4 lanes of a quad).
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float mx = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int kb = nt * 8 + 2 * c + e;
          const bool vis = rok[h] && b0 + kb < key_hi && ((win[h] >> kb) & 1ull);
          const float a = vis ? s[nt][2 * h + e] * p.scale : -INFINITY;
          s[nt][2 * h + e] = a;
          mx = fmaxf(mx, a);
        }
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mnew = fmaxf(m[h], mx);
      if (mnew == -INFINITY) {
        // Nothing visible yet for this row: probabilities are all zero.
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) s[nt][2 * h] = s[nt][2 * h + 1] = 0.f;
        continue;
      }
      const float corr = (m[h] == -INFINITY) ? 0.f : __expf(m[h] - mnew);
      float sum = 0.f;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float a = s[nt][2 * h + e];
          const float pv = (a == -INFINITY) ? 0.f : __expf(a - mnew);
          s[nt][2 * h + e] = pv;
          sum += pv;
        }
      }
      l[h] = l[h] * corr + sum;
      m[h] = mnew;
#pragma unroll
      for (int dt = 0; dt < 16; ++dt) {
        o[dt][2 * h] *= corr;
        o[dt][2 * h + 1] *= corr;
      }
    }

    // O += P V: P from the S fragments (bf16), V^T fragments via ldmatrix.trans.
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {  // 16 keys per step
      uint32_t pa[4];
      pa[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {  // pairs of 8-wide d tiles
        uint32_t vb[4];
        const int mtx = lane >> 3;
        const int vrow = kk * 16 + (mtx & 1) * 8 + (lane & 7);
        const int vcol = dp * 16 + (mtx >> 1) * 8;
        ldsm_x4_t(vb, vs + vrow * kPitch + vcol);
        mma_bf16(o[2 * dp], pa, vb[0], vb[1]);
        mma_bf16(o[2 * dp + 1], pa, vb[2], vb[3]);
      }
    }
    __syncthreads();  // this stage is consumed before it is refilled
  }

  // Row sums across the quad.
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    l[h] += __shfl_xor_sync(0xffffffffu, l[h], 1);
    l[h] += __shfl_xor_sync(0xffffffffu, l[h], 2);
  }
  if constexpr (!kFused) {
    // The split partials, merged by tree_attn_merge_kernel.
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (!rok[h]) continue;
      const int64_t idx = ((int64_t)split * p.num_heads + head[h]) * p.q_len + trow[h];
      float* dst = p.part_o + idx * kD;
#pragma unroll
      for (int dt = 0; dt < 16; ++dt)
        *reinterpret_cast<float2*>(dst + dt * 8 + 2 * c) = make_float2(o[dt][2 * h], o[dt][2 * h + 1]);
      if (c == 0) {
        p.part_ml[idx * 2] = m[h];
        p.part_ml[idx * 2 + 1] = l[h];
      }
    }
  } else {
    // Each packed row goes to the CTA of the cluster that owns it (stores
    // into its shared memory); after the cluster barrier every CTA merges
    // its own rows over the S splits in split order and writes them.
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    const int S = (int)cluster.num_blocks();  // == gridDim.z: one cluster per (head, row block)
    const int rpo = (kRowsCta + S - 1) / S;
    float* recv_o = reinterpret_cast<float*>(smem + 4 * kStageElems);  // [kRecvRows][kD]
    float* recv_ml = recv_o + (size_t)kRecvRows * kD;                 // [kRecvRows][2]
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int prow = warp * 16 + g + 8 * h;
      const int owner = prow / rpo;
      const int slot = split * rpo + (prow - owner * rpo);
      float* dsto = cluster.map_shared_rank(recv_o, owner) + (size_t)slot * kD;
#pragma unroll
      for (int dt = 0; dt < 16; ++dt)
        *reinterpret_cast<float2*>(dsto + dt * 8 + 2 * c) = make_float2(o[dt][2 * h], o[dt][2 * h + 1]);
      if (c == 0) {
        float* dml = cluster.map_shared_rank(recv_ml, owner) + (size_t)slot * 2;
        dml[0] = m[h];
        dml[1] = l[h];
      }
    }
    cluster.sync();
    for (int lr = warp; lr < rpo; lr += kWarps) {
      const int prow = split * rpo + lr;  // this CTA's rank in the cluster is its split
      const int pr = blockIdx.y * kRowsCta + prow;
      if (prow >= kRowsCta || pr >= packed_rows) break;
      float gm = -INFINITY;
      for (int sp = 0; sp < S; ++sp) gm = fmaxf(gm, recv_ml[(sp * rpo + lr) * 2]);
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      float denom = 0.f;
      if (gm != -INFINITY) {
        for (int sp = 0; sp < S; ++sp) {
          const float ms = recv_ml[(sp * rpo + lr) * 2];
          if (ms == -INFINITY) continue;
          const float w = expf(ms - gm);
          denom += w * recv_ml[(sp * rpo + lr) * 2 + 1];
          const float4 ov = *reinterpret_cast<const float4*>(recv_o + (size_t)(sp * rpo + lr) * kD + lane * 4);
          acc[0] += w * ov.x;
          acc[1] += w * ov.y;
          acc[2] += w * ov.z;
          acc[3] += w * ov.w;
        }
      }
      const float inv = denom > 0.f ? 1.f / denom : 0.f;
      const int hd = kvh * p.group + pr / p.q_len, t = pr % p.q_len;
      __nv_bfloat16* dst = out + ((int64_t)t * p.num_heads + hd) * kD + lane * 4;
      __nv_bfloat162 lo = __floats2bfloat162_rn(acc[0] * inv, acc[1] * inv);
      __nv_bfloat162 hi = __floats2bfloat162_rn(acc[2] * inv, acc[3] * inv);
      uint2 packed;
      packed.x = *reinterpret_cast<uint32_t*>(&lo);
      packed.y = *reinterpret_cast<uint32_t*>(&hi);
      *reinterpret_cast<uint2*>(dst) = packed;
    }
  }
}

}  // namespace

bool tree_attention_mma_supports(const AttnParams& p, int head_dim) {
  return head_dim == kD && p.q_rs % 2 == 0 && p.q_hs % 2 == 0 && p.kv_rs % 8 == 0 &&
         p.kv_hs % 8 == 0 && aligned16(p.k) && aligned16(p.v) &&
         (reinterpret_cast<uintptr_t>(p.q) & 3u) == 0 && p.q_len > 0 && p.kv_len > 0;
}

namespace {

// Whether clusters of `size` CTAs of the fused kernel can be placed (16 is
// above the portable limit of 8), checked once per device and size.
bool fused_clusters_ok(int size) {
  static std::mutex mu;
  static int known[64][kMaxFusedSplits + 1] = {};  // 0 unknown, 1 yes, 2 no
  int dev = 0;
  if (size < 1 || size > kMaxFusedSplits || cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return false;
  std::lock_guard<std::mutex> lock(mu);
  int& k = known[dev][size];
  if (k == 0) {
    bool ok = cudaFuncSetAttribute(tree_attn_mma_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)kFusedSmemBytes) == cudaSuccess &&
              cudaFuncSetAttribute(tree_attn_mma_kernel<true>,
                                   cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess;
    if (ok) {
      cudaLaunchConfig_t probe = {};
      probe.gridDim = dim3(1, 1, (unsigned)size);
      probe.blockDim = dim3(kWarps * 32, 1, 1);
      probe.dynamicSmemBytes = kFusedSmemBytes;
      cudaLaunchAttribute a[1];
      a[0].id = cudaLaunchAttributeClusterDimension;
      a[0].val.clusterDim.x = 1;
      a[0].val.clusterDim.y = 1;
      a[0].val.clusterDim.z = (unsigned)size;
      probe.attrs = a;
      probe.numAttrs = 1;
      int clusters = 0;
      ok = cudaOccupancyMaxActiveClusters(&clusters, tree_attn_mma_kernel<true>, &probe) == cudaSuccess &&
           clusters > 0;
    }
    (void)cudaGetLastError();
    k = ok ? 1 : 2;
  }
  return k == 1;
}

}  // namespace

int tree_attention_mma(AttnParams& p, void* out, bool* merged, cudaStream_t stream) {
  const int64_t row_blocks = ((int64_t)p.group * p.q_len + kRowsCta - 1) / kRowsCta;
  const int64_t blocks = (p.kv_len + kKeys - 1) / kKeys;
  int64_t want = (2 * (int64_t)num_sms() + p.num_kv_heads * row_blocks - 1) /
                 (p.num_kv_heads * row_blocks);
  *merged = false;
  // In-kernel merge when the splits fit one cluster without giving a CTA
  // more key blocks than the separate-merge launch would (a longer serial
  // chain per CTA costs more than the merge launch saves: measured at 2,320
  // keys and 6 query rows).
  {
    const int64_t fw = std::max<int64_t>(1, std::min<int64_t>(want, std::min<int64_t>(blocks, kMaxFusedSplits)));
    const int64_t sw = std::max<int64_t>(1, std::min<int64_t>(want, std::min<int64_t>(blocks, kMaxSplitsMma)));
    const int kps = (int)(((blocks + fw - 1) / fw) * kKeys);
    const int splits = (int)((p.kv_len + kps - 1) / kps);
    if (out && (blocks + fw - 1) / fw <= (blocks + sw - 1) / sw && fused_clusters_ok(splits)) {
      p.keys_per_split = kps;
      p.splits = splits;
      dim3 grid((unsigned)p.num_kv_heads, (unsigned)row_blocks, (unsigned)splits);
      SF_CHECK_CUDA(launch_pdl_cluster3(tree_attn_mma_kernel<true>, grid, dim3(kWarps * 32),
                                        kFusedSmemBytes, stream, dim3(1, 1, (unsigned)splits), p,
                                        static_cast<__nv_bfloat16*>(out)));
      *merged = true;
      return SF_OK;
    }
  }
  want = std::max<int64_t>(1, std::min<int64_t>(want, std::min<int64_t>(blocks, kMaxSplitsMma)));
  p.keys_per_split = (int)(((blocks + want - 1) / want) * kKeys);
  p.splits = (int)((p.kv_len + p.keys_per_split - 1) / p.keys_per_split);
  p.part_ml = p.part_o + (size_t)p.splits * p.num_heads * p.q_len * kD;
  dim3 grid((unsigned)p.num_kv_heads, (unsigned)row_blocks, (unsigned)p.splits);
  static std::atomic<unsigned long long> attr_done{0};
  const int rc = once_per_device(attr_done, [] {
    SF_CHECK_CUDA(cudaFuncSetAttribute(tree_attn_mma_kernel<false>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes));
    return SF_OK;
  });
  if (rc != SF_OK) return rc;
  SF_CHECK_CUDA(launch_pdl(tree_attn_mma_kernel<false>, dim3(grid), dim3(kWarps * 32), kSmemBytes,
                           stream, p, static_cast<__nv_bfloat16*>(nullptr)));
  SF_CHECK_LAUNCH();
  return SF_OK;
}

}  // namespace sf
