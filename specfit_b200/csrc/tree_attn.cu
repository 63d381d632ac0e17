// K6: tree-masked GQA attention of the verification pass.
//
// Restates the attention of Qwen3MoeAttention.forward after the KV-cache
// update (transformers/models/qwen3_moe/modeling_qwen3_moe.py:172-186: SDPA,
// scale head_dim**-0.5, GQA) under the verification mask of
// Eagle3DraftTree.verification_attention_mask (src/specfit/runtime/
// eagle3_types.py:450-473): every query sees the committed prefix and, inside
// the tree block, itself and its ancestors.  The mask arrives as one bit per
// tree column (little-endian uint32 words per query row); prefix keys need no
// bits.
//
// Split-KV ("flash-decoding") on CUDA cores: a CTA owns one KV head, a block
// of 8 query rows and one KV range; its 8 warps are the 8 query heads that
// share the KV head, so each K/V tile is staged in shared memory once for all
// of them.  Scores use an online softmax in fp32; a second kernel merges the
// per-split partial results and writes bf16 [Tq, Hq, D].
//
// The tiles are laid out for head_dim 128 (the Qwen3-30B-A3B shape).  Smaller
// head dims (a multiple of 4, e.g. the 8- and 16-wide heads of the tiny test
// configurations) are staged with zeros past head_dim: the extra products are
// exact zeros, so scores and outputs equal those of a D-wide kernel, and the
// merge writes only the first head_dim dims of each output row.
#include <math.h>

#include <algorithm>

#include "common.cuh"
#include "tree_attn.h"

namespace sf {
namespace {

constexpr int kD = 128;        // tile width of head_dim (head_dim <= kD)
constexpr int kRows = 8;       // query rows per CTA
constexpr int kTile = 64;      // keys per shared-memory tile
constexpr int kKPitch = kD + 2;  // bf16 pitch of the K tile (bank-conflict free)
constexpr int kMaxGroup = 8;   // query heads per KV head handled by one CTA
constexpr int kMaxSplits = 32;

using Params = AttnParams;

__device__ __forceinline__ bool visible(const Params& p, int row, int key) {
  if (key < p.prefix_len) return true;
  const int j = key - p.prefix_len;
  return (p.bits[(int64_t)row * p.bit_words + (j >> 5)] >> (j & 31)) & 1u;
}

__global__ void __launch_bounds__(kMaxGroup * 32)
tree_attn_split_kernel(Params p) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __nv_bfloat16* vs = reinterpret_cast<__nv_bfloat16*>(smem_raw);          // [kTile][kD]
  __nv_bfloat16* ks = vs + kTile * kD;                                      // [kTile][kKPitch]
  __nv_bfloat16* qs = ks + kTile * kKPitch;                                 // [group][kRows][kD]

  const int kvh = blockIdx.x;
  const int row0 = blockIdx.y * kRows;
  const int split = blockIdx.z;
  const int warp = threadIdx.x >> 5;  // query head within the group
  const int lane = threadIdx.x & 31;
  const int head = kvh * p.group + warp;
  const bool head_ok = warp < p.group;
  const int key_lo = split * p.keys_per_split;
  const int key_hi = min(p.kv_len, key_lo + p.keys_per_split);

  // Stage this warp's query rows (bf16, exact copies; the scale is applied
  // to the fp32 scores).
  __nv_bfloat16* qw = qs + warp * kRows * kD;
  for (int r = 0; r < kRows; ++r) {
    const int row = row0 + r;
    for (int d = lane; d < kD; d += 32) {
      __nv_bfloat16 qv = __float2bfloat16_rn(0.f);
      if (head_ok && row < p.q_len && d < p.head_dim)
        qv = p.q[(int64_t)head * p.q_hs + (int64_t)row * p.q_rs + d];
      qw[r * kD + d] = qv;
    }
  }

  float m[kRows], l[kRows], o[kRows][4];
#pragma unroll
  for (int r = 0; r < kRows; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) o[r][c] = 0.f;
  }

  for (int t0 = key_lo; t0 < key_hi; t0 += kTile) {
    const int nk = min(kTile, key_hi - t0);
    __syncthreads();
    // Stage K (padded pitch) and V tiles: 64 keys x 128 dims, 8 bytes/thread.
    for (int i = threadIdx.x; i < kTile * (kD / 4); i += blockDim.x) {
      const int key = i / (kD / 4);
      const int d4 = (i % (kD / 4)) * 4;
      uint2 kv = make_uint2(0, 0), vv = make_uint2(0, 0);
      if (key < nk && d4 < p.head_dim) {
        const int64_t off = (int64_t)kvh * p.kv_hs + (int64_t)(t0 + key) * p.kv_rs + d4;
        kv = *reinterpret_cast<const uint2*>(p.k + off);
        vv = *reinterpret_cast<const uint2*>(p.v + off);
      }
      *reinterpret_cast<uint32_t*>(&ks[key * kKPitch + d4]) = kv.x;
      *reinterpret_cast<uint32_t*>(&ks[key * kKPitch + d4 + 2]) = kv.y;
      *reinterpret_cast<uint2*>(&vs[key * kD + d4]) = vv;
    }
    __syncthreads();
    if (!head_ok) continue;

    // Scores: lane owns keys lane and lane+32 of the tile, all rows.
    float s[kRows][2];
#pragma unroll
    for (int r = 0; r < kRows; ++r) s[r][0] = s[r][1] = 0.f;
#pragma unroll 4
    for (int d = 0; d < kD; d += 2) {
      const float2 k0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ks[lane * kKPitch + d]));
      const float2 k1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ks[(lane + 32) * kKPitch + d]));
#pragma unroll
      for (int r = 0; r < kRows; ++r) {
        const float2 qv = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&qw[r * kD + d]));
        s[r][0] = fmaf(qv.x, k0.x, fmaf(qv.y, k0.y, s[r][0]));
        s[r][1] = fmaf(qv.x, k1.x, fmaf(qv.y, k1.y, s[r][1]));
      }
    }
    // Mask, online softmax, and P.V (lane owns dims 4*lane .. 4*lane+3).
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      const int row = row0 + r;
      const bool rok = row < p.q_len;
      const bool v0 = rok && lane < nk && visible(p, row, t0 + lane);
      const bool v1 = rok && lane + 32 < nk && visible(p, row, t0 + lane + 32);
      const float a0 = v0 ? s[r][0] * p.scale : -INFINITY;
      const float a1 = v1 ? s[r][1] * p.scale : -INFINITY;
      float tmax = fmaxf(a0, a1);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
      if (tmax == -INFINITY) continue;  // nothing visible in this tile for this row
      const float mnew = fmaxf(m[r], tmax);
      const float corr = (m[r] == -INFINITY) ? 0.f : expf(m[r] - mnew);
      const float p0 = v0 ? expf(a0 - mnew) : 0.f;
      const float p1 = v1 ? expf(a1 - mnew) : 0.f;
      float psum = p0 + p1;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, off);
      l[r] = l[r] * corr + psum;
      m[r] = mnew;
#pragma unroll
      for (int c = 0; c < 4; ++c) o[r][c] *= corr;
      for (int j = 0; j < 32; ++j) {
        const float pj0 = __shfl_sync(0xffffffffu, p0, j);
        const float pj1 = __shfl_sync(0xffffffffu, p1, j);
        if (pj0 != 0.f) {
          const uint2 vv = *reinterpret_cast<const uint2*>(&vs[j * kD + lane * 4]);
          const float2 va = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&vv.x));
          const float2 vb = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&vv.y));
          o[r][0] = fmaf(pj0, va.x, o[r][0]);
          o[r][1] = fmaf(pj0, va.y, o[r][1]);
          o[r][2] = fmaf(pj0, vb.x, o[r][2]);
          o[r][3] = fmaf(pj0, vb.y, o[r][3]);
        }
        if (pj1 != 0.f) {
          const uint2 vv = *reinterpret_cast<const uint2*>(&vs[(j + 32) * kD + lane * 4]);
          const float2 va = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&vv.x));
          const float2 vb = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&vv.y));
          o[r][0] = fmaf(pj1, va.x, o[r][0]);
          o[r][1] = fmaf(pj1, va.y, o[r][1]);
          o[r][2] = fmaf(pj1, vb.x, o[r][2]);
          o[r][3] = fmaf(pj1, vb.y, o[r][3]);
        }
      }
    }
  }

  if (!head_ok) return;
#pragma unroll
  for (int r = 0; r < kRows; ++r) {
    const int row = row0 + r;
    if (row >= p.q_len) break;
    const int64_t idx = ((int64_t)split * p.num_heads + head) * p.q_len + row;
    float4 ov = make_float4(o[r][0], o[r][1], o[r][2], o[r][3]);
    *reinterpret_cast<float4*>(p.part_o + idx * kD + lane * 4) = ov;
    if (lane == 0) {
      p.part_ml[idx * 2] = m[r];
      p.part_ml[idx * 2 + 1] = l[r];
    }
  }
}

// Merge the splits of one (head, row) per warp; lane owns 4 dims.
__global__ void tree_attn_merge_kernel(Params p, __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int64_t pair = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int64_t per_req = (int64_t)p.num_heads * p.q_len;  // also the stride between splits
  if (pair >= per_req * p.batch) return;
  const int req = (int)(pair / per_req);
  const int head = (int)((pair % per_req) / p.q_len);
  const int row = (int)(pair % p.q_len);
  const int64_t stride = per_req;
  const int64_t base = (int64_t)req * p.splits * per_req + (int64_t)head * p.q_len + row;
  // Lanes read the splits' (max, sum) pairs in parallel (split lane + 32 k).
  float gm = -INFINITY;
  for (int s = lane; s < p.splits; s += 32) gm = fmaxf(gm, p.part_ml[(base + s * stride) * 2]);
#pragma unroll
  for (int off = 16; off; off >>= 1) gm = fmaxf(gm, __shfl_xor_sync(0xffffffffu, gm, off));
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  float denom = 0.f;
  if (gm != -INFINITY) {
    for (int s = lane; s < p.splits; s += 32) {
      const float ms = p.part_ml[(base + s * stride) * 2];
      if (ms != -INFINITY) denom += expf(ms - gm) * p.part_ml[(base + s * stride) * 2 + 1];
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) denom += __shfl_xor_sync(0xffffffffu, denom, off);
    // Weighted outputs, four splits' loads in flight at a time.
    for (int s0 = 0; s0 < p.splits; s0 += 32) {
      const int s = s0 + lane;
      float w = 0.f;
      if (s < p.splits) {
        const float ms = p.part_ml[(base + s * stride) * 2];
        w = (ms == -INFINITY) ? 0.f : expf(ms - gm);
      }
      const int n = min(32, p.splits - s0);
      for (int j = 0; j < n; j += 4) {
        float4 ov[4];
        float wj[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          wj[u] = __shfl_sync(0xffffffffu, w, (j + u) & 31);
          ov[u] = (j + u < n && wj[u] != 0.f)
                      ? *reinterpret_cast<const float4*>(p.part_o + (base + (int64_t)(s0 + j + u) * stride) * kD + lane * 4)
                      : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (j + u < n) {
            acc[0] += wj[u] * ov[u].x;
            acc[1] += wj[u] * ov[u].y;
            acc[2] += wj[u] * ov[u].z;
            acc[3] += wj[u] * ov[u].w;
          }
        }
      }
    }
  }
  const float inv = denom > 0.f ? 1.f / denom : 0.f;
  if (lane * 4 >= p.head_dim) return;
  __nv_bfloat16* dst = out + (int64_t)req * p.out_bs + ((int64_t)row * p.num_heads + head) * p.head_dim + lane * 4;
  __nv_bfloat162 lo = __floats2bfloat162_rn(acc[0] * inv, acc[1] * inv);
  __nv_bfloat162 hi = __floats2bfloat162_rn(acc[2] * inv, acc[3] * inv);
  uint2 packed;
  packed.x = *reinterpret_cast<uint32_t*>(&lo);
  packed.y = *reinterpret_cast<uint32_t*>(&hi);
  *reinterpret_cast<uint2*>(dst) = packed;
}

int choose_splits(int num_kv_heads, int64_t q_len, int64_t kv_len) {
  const int64_t row_blocks = (q_len + kRows - 1) / kRows;
  const int64_t tiles = (kv_len + kTile - 1) / kTile;
  int64_t want = (2 * (int64_t)num_sms() + num_kv_heads * row_blocks - 1) / (num_kv_heads * row_blocks);
  want = std::max<int64_t>(1, std::min<int64_t>(want, std::min<int64_t>(tiles, kMaxSplits)));
  return (int)want;
}

}  // namespace
}  // namespace sf

extern "C" size_t sf_tree_attention_workspace_bytes(int num_heads, int64_t q_len, int64_t kv_len) {
  if (num_heads <= 0 || q_len <= 0 || kv_len <= 0) return 0;
  return (size_t)sf::kMaxSplits * num_heads * q_len * (sf::kD + 2) * sizeof(float);
}

extern "C" int sf_tree_attention_ex(const void* q, const void* k, const void* v,
                                    const uint32_t* tree_bits, int bit_words, int64_t q_len,
                                    int64_t kv_len, int64_t prefix_len, int num_heads,
                                    int num_kv_heads, int head_dim, int64_t q_head_stride,
                                    int64_t q_row_stride, int64_t kv_head_stride,
                                    int64_t kv_row_stride, float scale, void* out, void* workspace,
                                    size_t workspace_bytes, int impl, void* stream) {
  using namespace sf;
  SF_CHECK_ARG(head_dim > 0 && head_dim <= kD && head_dim % 4 == 0,
               "head_dim must be a multiple of 4 in [4, 128]");
  SF_CHECK_ARG(num_heads > 0 && num_kv_heads > 0 && num_heads % num_kv_heads == 0,
               "num_heads must be a positive multiple of num_kv_heads");
  SF_CHECK_ARG(num_heads / num_kv_heads <= kMaxGroup, "at most 8 query heads per KV head");
  SF_CHECK_ARG(q_len >= 0 && kv_len >= 0 && prefix_len >= 0 && prefix_len <= kv_len,
               "invalid lengths");
  SF_CHECK_ARG(q_len < (1 << 30) && kv_len < (1 << 30), "sequence too long");
  if (q_len == 0) return SF_OK;
  SF_CHECK_ARG(q && k && v && out && workspace, "null pointer argument");
  SF_CHECK_ARG(kv_len == prefix_len || (tree_bits && (int64_t)bit_words * 32 >= kv_len - prefix_len),
               "tree_bits must cover kv_len - prefix_len columns");
  SF_CHECK_ARG(q_row_stride % 2 == 0 && q_head_stride % 2 == 0, "q strides must be even");
  SF_CHECK_ARG(kv_row_stride % 4 == 0 && kv_head_stride % 4 == 0 &&
                   (reinterpret_cast<uintptr_t>(k) & 7u) == 0 &&
                   (reinterpret_cast<uintptr_t>(v) & 7u) == 0,
               "k/v rows must be 8-byte aligned");
  if (workspace_bytes < sf_tree_attention_workspace_bytes(num_heads, q_len, kv_len))
    return set_error(SF_ERR_WORKSPACE, "tree attention workspace needs %zu bytes",
                     sf_tree_attention_workspace_bytes(num_heads, q_len, kv_len));
  Params p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.bits = tree_bits;
  p.bit_words = bit_words;
  p.q_len = (int)q_len;
  p.kv_len = (int)kv_len;
  p.prefix_len = (int)prefix_len;
  p.num_heads = num_heads;
  p.num_kv_heads = num_kv_heads;
  p.group = num_heads / num_kv_heads;
  p.head_dim = head_dim;
  p.q_hs = q_head_stride;
  p.q_rs = q_row_stride;
  p.kv_hs = kv_head_stride;
  p.kv_rs = kv_row_stride;
  p.scale = scale;
  p.splits = choose_splits(num_kv_heads, q_len, kv_len);
  const int64_t tiles = (kv_len + kTile - 1) / kTile;
  p.keys_per_split = (int)(((tiles + p.splits - 1) / p.splits) * kTile);
  p.splits = (int)((kv_len + p.keys_per_split - 1) / p.keys_per_split);
  if (p.splits < 1) p.splits = 1;
  p.part_o = static_cast<float*>(workspace);
  p.part_ml = p.part_o + (size_t)p.splits * num_heads * q_len * kD;
  cudaStream_t s = as_stream(stream);
  const int64_t pairs = (int64_t)num_heads * q_len;
  SF_CHECK_ARG(impl == SF_ATTN_AUTO || impl == SF_ATTN_SIMT || impl == SF_ATTN_MMA ||
                   impl == SF_ATTN_TCGEN05,
               "unknown attention implementation %d", impl);
  // AUTO takes the tcgen05 kernel where it measured faster than the
  // warp-level one on the B200: many packed rows over a long context
  // (65 rows x 8 heads over 4,161 keys: 43.8 vs 64.5 us); short contexts
  // and few rows stay on mma.sync (65 x 8 over 577 keys: 18.7 vs 23.6 us).
  if (impl == SF_ATTN_AUTO && (int64_t)p.group * p.q_len >= 256 && p.kv_len >= 2048 &&
      tree_attention_tc_supports(p, head_dim))
    impl = SF_ATTN_TCGEN05;
  if (impl == SF_ATTN_TCGEN05) {
    SF_CHECK_ARG(tree_attention_tc_supports(p, head_dim),
                 "the tcgen05 tree attention needs D=128 and 16-byte aligned q/k/v rows");
    bool merged = false;
    if (int rc = tree_attention_tc(p, out, &merged, s)) return rc;
    if (merged) return SF_OK;
    SF_CHECK_CUDA(launch_pdl(tree_attn_merge_kernel, dim3((unsigned)((pairs + 7) / 8)), dim3(256),
                             0, s, p, static_cast<__nv_bfloat16*>(out)));
    SF_CHECK_LAUNCH();
    return SF_OK;
  }
  if (impl != SF_ATTN_SIMT && tree_attention_mma_supports(p, head_dim)) {
    bool merged = false;
    if (int rc = tree_attention_mma(p, out, &merged, s)) return rc;
    if (merged) return SF_OK;
    SF_CHECK_CUDA(launch_pdl(tree_attn_merge_kernel, dim3((unsigned)((pairs + 7) / 8)), dim3(256),
                             0, s, p, static_cast<__nv_bfloat16*>(out)));
    SF_CHECK_LAUNCH();
    return SF_OK;
  }
  SF_CHECK_ARG(impl != SF_ATTN_MMA, "the tensor-core tree attention does not support this layout");
  SF_CHECK_ARG((reinterpret_cast<uintptr_t>(out) & 7u) == 0, "out must be 8-byte aligned");
  dim3 grid((unsigned)num_kv_heads, (unsigned)((q_len + kRows - 1) / kRows), (unsigned)p.splits);
  const size_t smem = (size_t)(kTile * kD + kTile * kKPitch + kMaxGroup * kRows * kD) * 2;
  static std::atomic<unsigned long long> configured{0};
  if (int rc = once_per_device(configured, [&] {
        SF_CHECK_CUDA(cudaFuncSetAttribute(tree_attn_split_kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        return SF_OK;
      }))
    return rc;
  SF_CHECK_CUDA(launch_pdl(tree_attn_split_kernel, dim3(grid), dim3(kMaxGroup * 32), smem, s, p));
  SF_CHECK_LAUNCH();
  SF_CHECK_CUDA(launch_pdl(tree_attn_merge_kernel, dim3((unsigned)((pairs + 7) / 8)), dim3(256), 0,
                           s, p, static_cast<__nv_bfloat16*>(out)));
  SF_CHECK_LAUNCH();
  return SF_OK;
}

extern "C" size_t sf_tree_attention_batched_workspace_bytes(int batch, int num_heads, int64_t q_len,
                                                           int64_t kv_len) {
  if (batch <= 0) return 0;
  return (size_t)batch * sf_tree_attention_workspace_bytes(num_heads, q_len, kv_len);
}

extern "C" int sf_tree_attention_batched(const void* q, const void* k, const void* v,
                                         const uint32_t* tree_bits, int bit_words, int batch,
                                         int64_t q_batch_stride, int64_t kv_batch_stride,
                                         int64_t bits_batch_stride, int64_t out_batch_stride,
                                         int64_t q_len, int64_t kv_len, int64_t prefix_len, int num_heads,
                                         int num_kv_heads, int head_dim, int64_t q_head_stride,
                                         int64_t q_row_stride, int64_t kv_head_stride,
                                         int64_t kv_row_stride, float scale, void* out, void* workspace,
                                         size_t workspace_bytes, void* stream) {
  using namespace sf;
  SF_CHECK_ARG(batch > 0 && batch < 65536, "batch must be in [1, 65535]");
  SF_CHECK_ARG(num_heads > 0 && num_kv_heads > 0 && num_heads % num_kv_heads == 0 &&
                   num_heads / num_kv_heads <= kMaxGroup,
               "num_heads must be a multiple of num_kv_heads, at most 8 per KV head");
  SF_CHECK_ARG(q_len >= 0 && kv_len >= 0 && prefix_len >= 0 && prefix_len <= kv_len &&
                   q_len < (1 << 30) && kv_len < (1 << 30),
               "invalid lengths");
  if (q_len == 0) return SF_OK;
  SF_CHECK_ARG(q && k && v && out && workspace, "null pointer argument");
  SF_CHECK_ARG(kv_len == prefix_len || (tree_bits && (int64_t)bit_words * 32 >= kv_len - prefix_len),
               "tree_bits must cover kv_len - prefix_len columns");
  SF_CHECK_ARG(q_batch_stride >= 0 && kv_batch_stride >= 0 && bits_batch_stride >= 0 && out_batch_stride >= 0,
               "batch strides must be non-negative");
  if (workspace_bytes < sf_tree_attention_batched_workspace_bytes(batch, num_heads, q_len, kv_len))
    return set_error(SF_ERR_WORKSPACE, "batched tree attention workspace needs %zu bytes",
                     sf_tree_attention_batched_workspace_bytes(batch, num_heads, q_len, kv_len));
  Params p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.bits = tree_bits;
  p.bit_words = bit_words;
  p.q_len = (int)q_len;
  p.kv_len = (int)kv_len;
  p.prefix_len = (int)prefix_len;
  p.num_heads = num_heads;
  p.num_kv_heads = num_kv_heads;
  p.group = num_heads / num_kv_heads;
  p.head_dim = head_dim;
  p.q_hs = q_head_stride;
  p.q_rs = q_row_stride;
  p.kv_hs = kv_head_stride;
  p.kv_rs = kv_row_stride;
  p.scale = scale;
  p.part_o = static_cast<float*>(workspace);
  p.batch = batch;
  p.q_bs = q_batch_stride;
  p.kv_bs = kv_batch_stride;
  p.bits_bs = bits_batch_stride;
  p.out_bs = out_batch_stride;
  if (!tree_attention_tc_supports(p, head_dim) || kv_batch_stride % 8 != 0 || q_batch_stride % 8 != 0 ||
      out_batch_stride % 8 != 0)
    return SF_ERR_UNSUPPORTED;  // no message: callers run one request per call
  cudaStream_t s = as_stream(stream);
  bool merged = false;
  if (int rc = tree_attention_tc(p, out, &merged, s)) return rc;
  if (merged) return SF_OK;
  const int64_t pairs = (int64_t)batch * num_heads * q_len;
  SF_CHECK_CUDA(launch_pdl(tree_attn_merge_kernel, dim3((unsigned)((pairs + 7) / 8)), dim3(256), 0, s, p,
                           static_cast<__nv_bfloat16*>(out)));
  SF_CHECK_LAUNCH();
  return SF_OK;
}

extern "C" int sf_tree_attention(const void* q, const void* k, const void* v,
                                 const uint32_t* tree_bits, int bit_words, int64_t q_len,
                                 int64_t kv_len, int64_t prefix_len, int num_heads,
                                 int num_kv_heads, int head_dim, int64_t q_head_stride,
                                 int64_t q_row_stride, int64_t kv_head_stride,
                                 int64_t kv_row_stride, float scale, void* out, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  return sf_tree_attention_ex(q, k, v, tree_bits, bit_words, q_len, kv_len, prefix_len, num_heads,
                              num_kv_heads, head_dim, q_head_stride, q_row_stride, kv_head_stride,
                              kv_row_stride, scale, out, workspace, workspace_bytes, SF_ATTN_AUTO,
                              stream);
}
