// Fused elementwise steps of a Qwen3-MoE decoder layer for the verify pass.
//
// The Hugging Face layer (transformers/models/qwen3_moe/modeling_qwen3_moe.py)
// runs each RMSNorm, residual add, per-head q/k norm and rotary embedding as
// a chain of small torch kernels (about 50 per layer); at a few verify rows
// those launches cost more than the layer's arithmetic.  Two kernels replace
// them, keeping the bf16 rounding points of the torch code:
//
//   sf_add_rmsnorm   h = residual + x (bf16 add), out = bf16(w * bf16(h * rsqrt(mean(h^2) + eps)))
//                    (Qwen3MoeRMSNorm.forward, and the residual adds of
//                    Qwen3MoeDecoderLayer.forward)
//   sf_qk_norm_rope  per head of a fused q|k|v projection row: q and k get the
//                    head RMSNorm (q_norm / k_norm) and the rotary embedding
//                    q*cos + rotate_half(q)*sin, each product and the sum
//                    rounded to bf16 (apply_rotary_pos_emb); q is written
//                    head-major for the attention kernel, k and v straight
//                    into the KV cache rows (the cache update), at a row
//                    offset given on the host or read from device memory.
//
// Sums of squares are fp32 in a fixed order (per-thread, then a butterfly),
// which may differ from torch's reduction order in the last bit of the
// variance; outputs agree with the torch chain to bf16 rounding.
//
// Further down, the per-cycle steps around the verify pass: all-layer KV
// compaction of the accepted rows (sf_kv_compact), visibility words of a
// device-resident tree block (sf_tree_mask_words), and the drafter's fused
// log-softmax + top-k over the vocabulary (sf_logsoftmax_topk).
#include <cooperative_groups.h>

#include "common.cuh"

namespace sf {
namespace {

constexpr int kNormThreads = 256;  // 8 bf16 per thread covers H = 2048

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ __nv_bfloat16 bf(float v) { return __float2bfloat16_rn(v); }
__device__ __forceinline__ float fl(__nv_bfloat16 v) { return __bfloat162float(v); }

// One CTA per row; H % 8 == 0, rows 16-byte aligned.
__global__ void __launch_bounds__(kNormThreads)
add_rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ res_in,
                   __nv_bfloat16* __restrict__ res_out, const __nv_bfloat16* __restrict__ w,
                   float eps, int H, __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  __shared__ float part[kNormThreads / 32];
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * H;
  float h[8 * 4];  // up to 4 chunks of 8 per thread (H <= 8192)
  float ss = 0.f;
  int nch = 0;
  for (int c0 = threadIdx.x * 8; c0 < H; c0 += kNormThreads * 8, ++nch) {
    __nv_bfloat16 xv[8];
    *reinterpret_cast<uint4*>(xv) = *reinterpret_cast<const uint4*>(xr + c0);
    __nv_bfloat16 hv[8];
    if (res_in) {
      __nv_bfloat16 rv[8];
      *reinterpret_cast<uint4*>(rv) = *reinterpret_cast<const uint4*>(res_in + row * H + c0);
#pragma unroll
      for (int v = 0; v < 8; ++v) hv[v] = bf(fl(rv[v]) + fl(xv[v]));
    } else {
#pragma unroll
      for (int v = 0; v < 8; ++v) hv[v] = xv[v];
    }
    if (res_out) *reinterpret_cast<uint4*>(res_out + row * H + c0) = *reinterpret_cast<uint4*>(hv);
#pragma unroll
    for (int v = 0; v < 8; ++v) {
      const float f = fl(hv[v]);
      h[nch * 8 + v] = f;
      ss += f * f;
    }
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) tot += part[i];
  const float r = rsqrtf(tot / (float)H + eps);
  int ch = 0;
  for (int c0 = threadIdx.x * 8; c0 < H; c0 += kNormThreads * 8, ++ch) {
    __nv_bfloat16 wv[8], ov[8];
    *reinterpret_cast<uint4*>(wv) = *reinterpret_cast<const uint4*>(w + c0);
#pragma unroll
    for (int v = 0; v < 8; ++v) ov[v] = bf(fl(wv[v]) * fl(bf(h[ch * 8 + v] * r)));
    *reinterpret_cast<uint4*>(out + row * H + c0) = *reinterpret_cast<uint4*>(ov);
  }
}

// One warp per (token, head) of the q|k|v row; D == 128 (4 values per lane).
__global__ void qk_norm_rope_kernel(const __nv_bfloat16* __restrict__ qkv, int64_t n_tokens, int T,
                                    int hq, int hkv, const __nv_bfloat16* __restrict__ qw,
                                    const __nv_bfloat16* __restrict__ kw,
                                    const __nv_bfloat16* __restrict__ cos,
                                    const __nv_bfloat16* __restrict__ sin, float eps,
                                    __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ kbuf,
                                    __nv_bfloat16* __restrict__ vbuf, int64_t kv_batch_stride,
                                    int64_t kv_head_stride, int64_t row0_host,
                                    const int64_t* __restrict__ row0_dev) {
  pdl_wait();
  pdl_trigger();
  constexpr int D = 128;
  const int heads = hq + 2 * hkv;
  const int64_t item = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (item >= n_tokens * heads) return;
  const int lane = threadIdx.x & 31;
  const int64_t n = item / heads;
  const int head = (int)(item - n * heads);
  const int b = (int)(n / T), t = (int)(n - (int64_t)b * T);
  const __nv_bfloat16* src = qkv + n * (int64_t)heads * D + (int64_t)head * D + lane * 4;
  __nv_bfloat16 xv[4];
  *reinterpret_cast<uint2*>(xv) = *reinterpret_cast<const uint2*>(src);
  const int64_t row = (row0_dev ? *row0_dev : row0_host) + t;
  if (head >= hq + hkv) {  // v: straight into the cache
    __nv_bfloat16* dst = vbuf + b * kv_batch_stride + (int64_t)(head - hq - hkv) * kv_head_stride + row * D;
    *reinterpret_cast<uint2*>(dst + lane * 4) = *reinterpret_cast<uint2*>(xv);
    return;
  }
  const __nv_bfloat16* w = head < hq ? qw : kw;
  float y[4];
  if (w) {
    float ss = 0.f;
#pragma unroll
    for (int v = 0; v < 4; ++v) ss += fl(xv[v]) * fl(xv[v]);
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / (float)D + eps);
#pragma unroll
    for (int v = 0; v < 4; ++v) y[v] = fl(bf(fl(w[lane * 4 + v]) * fl(bf(fl(xv[v]) * r))));
  } else {  // no head norm
#pragma unroll
    for (int v = 0; v < 4; ++v) y[v] = fl(xv[v]);
  }
  // rotate_half: dims d < 64 take -x[d + 64], dims d >= 64 take x[d - 64] (lane +- 16).
  float other[4];
#pragma unroll
  for (int v = 0; v < 4; ++v) other[v] = __shfl_xor_sync(0xffffffffu, y[v], 16);
  const bool low = lane < 16;
  const __nv_bfloat16* cr = cos + n * D + lane * 4;
  const __nv_bfloat16* sr = sin + n * D + lane * 4;
  __nv_bfloat16 o[4];
#pragma unroll
  for (int v = 0; v < 4; ++v) {
    const float rot = low ? -other[v] : other[v];
    o[v] = bf(fl(bf(y[v] * fl(cr[v]))) + fl(bf(rot * fl(sr[v]))));
  }
  if (head < hq) {
    __nv_bfloat16* dst = q_out + (((int64_t)b * hq + head) * T + t) * D + lane * 4;
    *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<uint2*>(o);
  } else {
    __nv_bfloat16* dst = kbuf + b * kv_batch_stride + (int64_t)(head - hq) * kv_head_stride + row * D;
    *reinterpret_cast<uint2*>(dst + lane * 4) = *reinterpret_cast<uint2*>(o);
  }
}

}  // namespace
}  // namespace sf

extern "C" int sf_add_rmsnorm(const void* x, const void* residual_in, void* residual_out,
                              const void* weight, float eps, int64_t rows, int hidden_size,
                              void* out, void* stream) {
  using namespace sf;
  SF_CHECK_ARG(rows >= 0 && hidden_size > 0, "invalid sizes");
  SF_CHECK_ARG(hidden_size % 8 == 0 && hidden_size <= 8 * 4 * kNormThreads,
               "hidden_size must be a multiple of 8 and at most %d", 8 * 4 * kNormThreads);
  if (rows == 0) return SF_OK;
  SF_CHECK_ARG(x && weight && out, "null pointer argument");
  SF_CHECK_ARG(aligned16(x) && aligned16(out) && aligned16(weight) &&
               (!residual_in || aligned16(residual_in)) && (!residual_out || aligned16(residual_out)),
               "tensors must be 16-byte aligned");
  SF_CHECK_CUDA(launch_pdl(add_rmsnorm_kernel, dim3((unsigned)rows), dim3(kNormThreads), 0,
                           as_stream(stream), static_cast<const __nv_bfloat16*>(x),
                           static_cast<const __nv_bfloat16*>(residual_in),
                           static_cast<__nv_bfloat16*>(residual_out),
                           static_cast<const __nv_bfloat16*>(weight), eps, hidden_size,
                           static_cast<__nv_bfloat16*>(out)));
  SF_CHECK_LAUNCH();
  return SF_OK;
}

extern "C" int sf_qk_norm_rope(const void* qkv, int64_t batch, int64_t tokens, int num_heads,
                               int num_kv_heads, int head_dim, const void* q_norm_weight,
                               const void* k_norm_weight, const void* cos, const void* sin,
                               float eps, void* q_out, void* k_cache, void* v_cache,
                               int64_t kv_batch_stride, int64_t kv_head_stride, int64_t row0,
                               const int64_t* row0_device, void* stream) {
  using namespace sf;
  SF_CHECK_ARG(head_dim == 128, "head_dim must be 128");
  SF_CHECK_ARG(batch >= 0 && tokens >= 0 && num_heads > 0 && num_kv_heads > 0, "invalid sizes");
  const int64_t n = batch * tokens;
  if (n == 0) return SF_OK;
  SF_CHECK_ARG(qkv && cos && sin && q_out && k_cache && v_cache, "null pointer argument");
  SF_CHECK_ARG((q_norm_weight == nullptr) == (k_norm_weight == nullptr),
               "pass both head-norm weights or neither");
  SF_CHECK_ARG(aligned16(qkv) && aligned16(q_out) && aligned16(k_cache) && aligned16(v_cache),
               "tensors must be 16-byte aligned");
  SF_CHECK_ARG(kv_batch_stride % 8 == 0 && kv_head_stride % 8 == 0, "cache strides must be multiples of 8");
  const int64_t items = n * (num_heads + 2 * num_kv_heads);
  SF_CHECK_CUDA(launch_pdl(qk_norm_rope_kernel, dim3((unsigned)((items + 7) / 8)), dim3(256), 0,
                           as_stream(stream), static_cast<const __nv_bfloat16*>(qkv), n,
                           (int)tokens, num_heads, num_kv_heads,
                           static_cast<const __nv_bfloat16*>(q_norm_weight),
                           static_cast<const __nv_bfloat16*>(k_norm_weight),
                           static_cast<const __nv_bfloat16*>(cos),
                           static_cast<const __nv_bfloat16*>(sin), eps,
                           static_cast<__nv_bfloat16*>(q_out), static_cast<__nv_bfloat16*>(k_cache),
                           static_cast<__nv_bfloat16*>(v_cache), kv_batch_stride, kv_head_stride,
                           row0, row0_device));
  SF_CHECK_LAUNCH();
  return SF_OK;
}

namespace sf {
namespace {

// KV compaction of a verify pass over every layer at once: row base + src[i]
// of each K and V buffer moves to base + i.  The kept rows are first
// gathered into a caller-provided stage and then written back, in two
// launches, so moves whose source and destination overlap are safe.  One CTA
// per (buffer, kept row); a row is `heads` runs of D contiguous elements,
// head_stride apart.
__global__ void kv_gather_kernel(const uint64_t* __restrict__ bufs, int layers, int heads,
                                 int64_t head_stride, int64_t base, const int32_t* __restrict__ src,
                                 int n, int D, __nv_bfloat16* __restrict__ stage) {
  pdl_wait();
  pdl_trigger();
  const int i = blockIdx.x % n;
  const int l2 = blockIdx.x / n;  // layer * 2 + (k or v)
  const __nv_bfloat16* buf = reinterpret_cast<const __nv_bfloat16*>(bufs[l2]);
  __nv_bfloat16* st = stage + ((int64_t)l2 * n + i) * heads * D;
  for (int e = threadIdx.x * 8; e < heads * D; e += blockDim.x * 8) {
    const int h = e / D, d = e % D;
    *reinterpret_cast<uint4*>(st + e) =
        *reinterpret_cast<const uint4*>(buf + h * head_stride + (base + src[i]) * D + d);
  }
}

__global__ void kv_scatter_kernel(const uint64_t* __restrict__ bufs, int layers, int heads,
                                  int64_t head_stride, int64_t base, int n, int D,
                                  const __nv_bfloat16* __restrict__ stage) {
  pdl_wait();
  pdl_trigger();
  const int i = blockIdx.x % n;
  const int l2 = blockIdx.x / n;
  __nv_bfloat16* buf = reinterpret_cast<__nv_bfloat16*>(bufs[l2]);
  const __nv_bfloat16* st = stage + ((int64_t)l2 * n + i) * heads * D;
  for (int e = threadIdx.x * 8; e < heads * D; e += blockDim.x * 8) {
    const int h = e / D, d = e % D;
    *reinterpret_cast<uint4*>(buf + h * head_stride + (base + i) * D + d) =
        *reinterpret_cast<const uint4*>(st + e);
  }
}

}  // namespace
}  // namespace sf

extern "C" int sf_kv_compact(const uint64_t* buffers, int layers, int heads, int head_dim,
                             int64_t head_stride, int64_t base, const int32_t* src_rows, int n,
                             void* stage, void* stream) {
  using namespace sf;
  SF_CHECK_ARG(layers > 0 && heads > 0 && head_dim % 8 == 0 && n >= 0, "invalid sizes");
  SF_CHECK_ARG(head_stride % 8 == 0 && base >= 0, "invalid strides");
  if (n == 0) return SF_OK;
  SF_CHECK_ARG(buffers && src_rows && stage, "null pointer argument");
  SF_CHECK_ARG(aligned16(stage), "stage must be 16-byte aligned");
  cudaStream_t s = as_stream(stream);
  const unsigned grid = (unsigned)(2 * layers * n);
  SF_CHECK_CUDA(launch_pdl(kv_gather_kernel, dim3(grid), dim3(128), 0, s, buffers, layers, heads,
                           head_stride, base, src_rows, n, head_dim,
                           static_cast<__nv_bfloat16*>(stage)));
  SF_CHECK_LAUNCH();
  SF_CHECK_CUDA(launch_pdl(kv_scatter_kernel, dim3(grid), dim3(128), 0, s, buffers, layers, heads,
                           head_stride, base, n, head_dim,
                           static_cast<const __nv_bfloat16*>(stage)));
  SF_CHECK_LAUNCH();
  return SF_OK;
}

namespace sf {
namespace {

// Word w of row r: column c = 32 w + bit is visible when c < start, or when
// 0 <= c - start < 64 and bit (c - start) of the row's ancestor set is set.
__global__ void tree_mask_words_kernel(const int64_t* __restrict__ vis, int n,
                                       const int64_t* __restrict__ start_dev, int words,
                                       int32_t* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)n * words) return;
  const int r = (int)(i / words), w = (int)(i - (int64_t)r * words);
  const int64_t start = *start_dev;
  const uint64_t set = (uint64_t)vis[r];
  uint32_t word = 0;
  for (int bit = 0; bit < 32; ++bit) {
    const int64_t rel = (int64_t)w * 32 + bit - start;
    const bool on = rel < 0 || (rel < 64 && ((set >> rel) & 1ull));
    word |= (uint32_t)on << bit;
  }
  out[i] = (int32_t)word;
}

}  // namespace
}  // namespace sf

extern "C" int sf_tree_mask_words(const int64_t* ancestor_sets, int rows, const int64_t* start_device,
                                  int words, int32_t* out, void* stream) {
  using namespace sf;
  SF_CHECK_ARG(rows >= 0 && words > 0, "invalid sizes");
  if (rows == 0) return SF_OK;
  SF_CHECK_ARG(ancestor_sets && start_device && out, "null pointer argument");
  const int64_t total = (int64_t)rows * words;
  SF_CHECK_CUDA(launch_pdl(tree_mask_words_kernel, dim3((unsigned)((total + 255) / 256)), dim3(256),
                           0, as_stream(stream), ancestor_sets, rows, start_device, words, out));
  SF_CHECK_LAUNCH();
  return SF_OK;
}

namespace sf {
namespace {

namespace cg = cooperative_groups;

constexpr int kTopkThreads = 512;
constexpr int kTopkWarps = kTopkThreads / 32;
constexpr int kTopkVecs = 4;          // 16-byte vectors (32 values) per thread per batch
constexpr int kTopkSlots = kTopkVecs * 8;
constexpr int kTopkMaxCluster = 16;   // CTAs per row (8 where 16 is not available)
constexpr int kMaxTopk = 8;
constexpr int kNoIndex = 0x7fffffff;

// (value, index) order of the result: larger value first, lower index first
// among equal values.
__device__ __forceinline__ bool topk_better(float a, int ai, float b, int bi) {
  return a > b || (a == b && ai < bi);
}

// Every lane gets the warp's best (value, index).
__device__ __forceinline__ void warp_best(float& v, int& i) {
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (topk_better(ov, oi, v, i)) {
      v = ov;
      i = oi;
    }
  }
}

// Online (max, sum of exponentials) merge of two partial states.
__device__ __forceinline__ void lse_merge(float& m, float& s, float m2, float s2) {
  const float mm = fmaxf(m, m2);
  if (mm == -INFINITY) return;
  s = (m == -INFINITY ? 0.f : s * __expf(m - mm)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - mm));
  m = mm;
}

// A sorted list of K (value, index) pairs held by every lane of a warp.
template <int K>
struct WarpList {
  float v[K];
  int i[K];
  __device__ void clear() {
#pragma unroll
    for (int j = 0; j < K; ++j) {
      v[j] = -INFINITY;
      i[j] = kNoIndex;
    }
  }
  __device__ void pop() {
#pragma unroll
    for (int j = 0; j + 1 < K; ++j) {
      v[j] = v[j + 1];
      i[j] = i[j + 1];
    }
    v[K - 1] = -INFINITY;
    i[K - 1] = kNoIndex;
  }
};

// Sorted lists held one per lane (lanes without one hold padding) merged
// into the warp's best k, handed to emit(r, value, index) on every lane.
template <int K, typename Emit>
__device__ __forceinline__ void merge_lane_lists(WarpList<K>& mine, int k, Emit emit) {
  for (int r = 0; r < k; ++r) {
    float bv = mine.v[0];
    int bi = mine.i[0];
    warp_best(bv, bi);
    emit(r, bv, bi);
    if (mine.i[0] == bi && bi != kNoIndex) mine.pop();
  }
}

// Log-softmax of scale * logits (bf16 rows) and its top-k.  A cluster of
// 16 (or 8) CTAs shares one row, each streaming a contiguous part of it.
// A thread takes 32 values per batch (four 16-byte loads in flight), adds
// their exponentials against the running maximum (rescaled once per batch),
// and its warp selects the batch's k best together with the k best so far
// in k rounds of a warp-wide argmax over each lane's best remaining value;
// only the lane that supplied a round's winner rescans its values.  The 16
// warps' lists are merged per CTA, and CTA 0 of the cluster merges the
// CTAs' lists and (max, sum) pairs through distributed shared memory and
// writes (y - max) - log(sum), y = scale * logit in fp32.
template <int K>
__global__ void __launch_bounds__(kTopkThreads)
logsoftmax_topk_kernel(const __nv_bfloat16* __restrict__ logits, int64_t vocab, float scale, int k,
                       float* __restrict__ top_v, int64_t* __restrict__ top_i) {
  pdl_wait();
  pdl_trigger();
  __shared__ float s_m[kTopkWarps], s_s[kTopkWarps];
  __shared__ float w_v[kTopkWarps][K];
  __shared__ int w_i[kTopkWarps][K];
  __shared__ float p_ms[2];  // this CTA's (max, sum)
  __shared__ float p_v[K];
  __shared__ int p_i[K];
  cg::cluster_group cluster = cg::this_cluster();
  const int crank = (int)cluster.block_rank();
  const int csize = (int)cluster.num_blocks();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t row = blockIdx.y;
  const __nv_bfloat16* x = logits + row * vocab;
  const int64_t chunk = ((vocab + 7) / 8 + csize - 1) / csize * 8;
  const int64_t lo = min(vocab, crank * chunk), hi = min(vocab, lo + chunk);
  const bool vec = (vocab % 8 == 0) && ((reinterpret_cast<uintptr_t>(logits) & 15) == 0);
  // One batch covers kTopkThreads * kTopkSlots consecutive values of [lo, hi).
  constexpr int64_t kBatch = (int64_t)kTopkThreads * kTopkSlots;

  float m = -INFINITY, sum = 0.f;
  WarpList<K> best;
  best.clear();
  for (int64_t b0 = lo; b0 < hi; b0 += kBatch) {
    float y[kTopkSlots];
    // Index of slot s: vec: (c + v T) * 8 + j with c = b0 / 8 + tid (s = 8 v + j);
    // scalar: b0 + s T + tid.  Both grow with s.
    if (vec) {
      const uint4* x8 = reinterpret_cast<const uint4*>(x);
      uint4 u[kTopkVecs];
#pragma unroll
      for (int v = 0; v < kTopkVecs; ++v) {
        const int64_t c = b0 / 8 + threadIdx.x + (int64_t)v * kTopkThreads;
        u[v] = c * 8 < hi ? __ldg(x8 + c) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int v = 0; v < kTopkVecs; ++v) {
        const bool ok = (b0 / 8 + threadIdx.x + (int64_t)v * kTopkThreads) * 8 < hi;
        const __nv_bfloat162* e = reinterpret_cast<const __nv_bfloat162*>(&u[v]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(e[j]);
          y[v * 8 + 2 * j] = ok ? f.x * scale : -INFINITY;
          y[v * 8 + 2 * j + 1] = ok ? f.y * scale : -INFINITY;
        }
      }
    } else {
#pragma unroll
      for (int sl = 0; sl < kTopkSlots; ++sl) {
        const int64_t e = b0 + (int64_t)sl * kTopkThreads + threadIdx.x;
        y[sl] = e < hi ? __bfloat162float(x[e]) * scale : -INFINITY;
      }
    }
    auto index_of = [&](int sl) -> int {
      return vec ? (int)((b0 / 8 + threadIdx.x + (int64_t)(sl >> 3) * kTopkThreads) * 8 + (sl & 7))
                 : (int)(b0 + (int64_t)sl * kTopkThreads + threadIdx.x);
    };
    // Sum of exponentials against the new running maximum.
    float bm = -INFINITY;
#pragma unroll
    for (int sl = 0; sl < kTopkSlots; ++sl) bm = fmaxf(bm, y[sl]);
    const float mn = fmaxf(m, bm);
    if (mn != -INFINITY) {
      float a[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int sl = 0; sl < kTopkSlots; ++sl) a[sl & 3] += __expf(y[sl] - mn);
      sum = (m == -INFINITY ? 0.f : sum * __expf(m - mn)) + ((a[0] + a[1]) + (a[2] + a[3]));
      m = mn;
    }
    // This lane's best remaining slot (the first on ties: the lower index;
    // -inf slots, including those past the row, are never taken).
    float lv = -INFINITY;
    int ls = -1;
#pragma unroll
    for (int sl = 0; sl < kTopkSlots; ++sl)
      if (y[sl] > lv) {
        lv = y[sl];
        ls = sl;
      }
    WarpList<K> next;
#pragma unroll
    for (int r = 0; r < K; ++r) {
      next.v[r] = -INFINITY;
      next.i[r] = kNoIndex;
      if (r >= k) continue;
      int li = ls >= 0 ? index_of(ls) : kNoIndex;
      float wv = lv;
      int wi = li;
      warp_best(wv, wi);
      if (topk_better(best.v[0], best.i[0], wv, wi)) {  // the list so far wins this round
        next.v[r] = best.v[0];
        next.i[r] = best.i[0];
        best.pop();
      } else {
        next.v[r] = wv;
        next.i[r] = wi;
        if (wi == li && wi != kNoIndex) {  // this lane supplied the winner: rescan
#pragma unroll
          for (int sl = 0; sl < kTopkSlots; ++sl)
            if (sl == ls) y[sl] = -INFINITY;
          lv = -INFINITY;
          ls = -1;
#pragma unroll
          for (int sl = 0; sl < kTopkSlots; ++sl)
            if (y[sl] > lv) {
              lv = y[sl];
              ls = sl;
            }
        }
      }
    }
    best = next;
  }
  // Warp and CTA partials.
#pragma unroll
  for (int o = 16; o; o >>= 1)
    lse_merge(m, sum, __shfl_xor_sync(0xffffffffu, m, o), __shfl_xor_sync(0xffffffffu, sum, o));
  if (lane == 0) {
    s_m[warp] = m;
    s_s[warp] = sum;
#pragma unroll
    for (int r = 0; r < K; ++r) {
      w_v[warp][r] = best.v[r];
      w_i[warp][r] = best.i[r];
    }
  }
  __syncthreads();
  if (warp == 0) {
    float M = lane < kTopkWarps ? s_m[lane] : -INFINITY;
    float S = lane < kTopkWarps ? s_s[lane] : 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1)
      lse_merge(M, S, __shfl_xor_sync(0xffffffffu, M, o), __shfl_xor_sync(0xffffffffu, S, o));
    WarpList<K> mine;
    mine.clear();
    if (lane < kTopkWarps) {
#pragma unroll
      for (int r = 0; r < K; ++r) {
        mine.v[r] = w_v[lane][r];
        mine.i[r] = w_i[lane][r];
      }
    }
    merge_lane_lists<K>(mine, k, [&](int r, float bv, int bi) {
      if (lane == 0) {
        p_v[r] = bv;
        p_i[r] = bi;
      }
    });
    if (lane == 0) {
      p_ms[0] = M;
      p_ms[1] = S;
    }
  }
  cluster.sync();  // every CTA's partial is in its shared memory
  if (crank == 0 && warp == 0) {
    float M = -INFINITY, S = 0.f;
    WarpList<K> mine;
    mine.clear();
    if (lane < csize) {
      const float* ms = cluster.map_shared_rank(p_ms, lane);
      const float* pv = cluster.map_shared_rank(p_v, lane);
      const int* pi = cluster.map_shared_rank(p_i, lane);
      M = ms[0];
      S = ms[1];
#pragma unroll
      for (int r = 0; r < K; ++r) {
        mine.v[r] = r < k ? pv[r] : -INFINITY;
        mine.i[r] = r < k ? pi[r] : kNoIndex;
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1)
      lse_merge(M, S, __shfl_xor_sync(0xffffffffu, M, o), __shfl_xor_sync(0xffffffffu, S, o));
    const float log_s = logf(S);
    merge_lane_lists<K>(mine, k, [&](int r, float bv, int bi) {
      if (lane == 0) {
        top_v[row * k + r] = (bv - M) - log_s;
        top_i[row * k + r] = bi;
      }
    });
  }
  cluster.sync();  // peers keep their shared memory until CTA 0 has read it
}

static_assert(kTopkWarps <= 32 && kTopkMaxCluster <= 32, "one list per lane in the merges");

template <int K>
int launch_topk_rows(const __nv_bfloat16* x, int64_t rows, int64_t vocab, float scale, int k,
                     float* top_v, int64_t* top_i, cudaStream_t stream) {
  static std::atomic<unsigned long long> configured{0};
  static int cluster_size[64] = {};
  int dev = 0;
  SF_CHECK_CUDA(cudaGetDevice(&dev));
  if (int rc = once_per_device(configured, [] {
        SF_CHECK_CUDA(cudaFuncSetAttribute(logsoftmax_topk_kernel<K>,
                                           cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
        int d = 0;
        SF_CHECK_CUDA(cudaGetDevice(&d));
        // 16 CTAs per row where the device can co-schedule such clusters, else 8.
        cudaLaunchConfig_t probe = {};
        probe.gridDim = dim3(kTopkMaxCluster, 1, 1);
        probe.blockDim = dim3(kTopkThreads, 1, 1);
        cudaLaunchAttribute a[1];
        a[0].id = cudaLaunchAttributeClusterDimension;
        a[0].val.clusterDim.x = kTopkMaxCluster;
        a[0].val.clusterDim.y = 1;
        a[0].val.clusterDim.z = 1;
        probe.attrs = a;
        probe.numAttrs = 1;
        int clusters = 0;
        const cudaError_t e = cudaOccupancyMaxActiveClusters(&clusters, logsoftmax_topk_kernel<K>, &probe);
        if (e != cudaSuccess) (void)cudaGetLastError();
        if (d >= 0 && d < 64) cluster_size[d] = (e == cudaSuccess && clusters > 0) ? kTopkMaxCluster : 8;
        return SF_OK;
      }))
    return rc;
  const int cs = (dev >= 0 && dev < 64 && cluster_size[dev]) ? cluster_size[dev] : 8;
  SF_CHECK_CUDA(launch_pdl_cluster(logsoftmax_topk_kernel<K>, dim3((unsigned)cs, (unsigned)rows, 1),
                                   dim3(kTopkThreads), 0, stream, (unsigned)cs, 1u, x, vocab, scale,
                                   k, top_v, top_i));
  return SF_OK;
}

}  // namespace
}  // namespace sf

extern "C" int sf_logsoftmax_topk(const void* logits, int64_t rows, int64_t vocab, float scale, int k,
                                  float* top_values, int64_t* top_indices, void* stream) {
  using namespace sf;
  SF_CHECK_ARG(rows >= 0 && rows <= 65535 && vocab > 0 && vocab < (1LL << 31) - 1, "invalid sizes");
  SF_CHECK_ARG(k >= 1 && k <= kMaxTopk && k <= vocab, "k must be in [1, %d] and at most vocab", kMaxTopk);
  if (rows == 0) return SF_OK;
  SF_CHECK_ARG(logits && top_values && top_indices, "null pointer argument");
  auto* x = static_cast<const __nv_bfloat16*>(logits);
  cudaStream_t s = as_stream(stream);
  if (k <= 1) return launch_topk_rows<1>(x, rows, vocab, scale, k, top_values, top_indices, s);
  if (k <= 2) return launch_topk_rows<2>(x, rows, vocab, scale, k, top_values, top_indices, s);
  if (k <= 4) return launch_topk_rows<4>(x, rows, vocab, scale, k, top_values, top_indices, s);
  return launch_topk_rows<8>(x, rows, vocab, scale, k, top_values, top_indices, s);
}
