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
  add_rmsnorm_kernel<<<(unsigned)rows, kNormThreads, 0, as_stream(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(residual_in),
      static_cast<__nv_bfloat16*>(residual_out), static_cast<const __nv_bfloat16*>(weight), eps,
      hidden_size, static_cast<__nv_bfloat16*>(out));
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
  qk_norm_rope_kernel<<<(unsigned)((items + 7) / 8), 256, 0, as_stream(stream)>>>(
      static_cast<const __nv_bfloat16*>(qkv), n, (int)tokens, num_heads, num_kv_heads,
      static_cast<const __nv_bfloat16*>(q_norm_weight), static_cast<const __nv_bfloat16*>(k_norm_weight),
      static_cast<const __nv_bfloat16*>(cos), static_cast<const __nv_bfloat16*>(sin), eps,
      static_cast<__nv_bfloat16*>(q_out), static_cast<__nv_bfloat16*>(k_cache),
      static_cast<__nv_bfloat16*>(v_cache), kv_batch_stride, kv_head_stride, row0, row0_device);
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
  kv_gather_kernel<<<grid, 128, 0, s>>>(buffers, layers, heads, head_stride, base, src_rows, n,
                                         head_dim, static_cast<__nv_bfloat16*>(stage));
  SF_CHECK_LAUNCH();
  kv_scatter_kernel<<<grid, 128, 0, s>>>(buffers, layers, heads, head_stride, base, n, head_dim,
                                          static_cast<const __nv_bfloat16*>(stage));
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
  tree_mask_words_kernel<<<(unsigned)((total + 255) / 256), 256, 0, as_stream(stream)>>>(
      ancestor_sets, rows, start_device, words, out);
  SF_CHECK_LAUNCH();
  return SF_OK;
}

namespace sf {
namespace {

namespace cg = cooperative_groups;

constexpr int kTopkThreads = 512;
constexpr int kTopkWarps = kTopkThreads / 32;
constexpr int kTopkCluster = 8;  // CTAs per row, merged through distributed shared memory
constexpr int kMaxTopk = 8;

__device__ __forceinline__ bool topk_better(float a, int ai, float b, int bi) {
  return a > b || (a == b && ai < bi);
}

// The K largest (value, index) pairs seen, larger value first and lower index
// first among equal values; held in registers (fully unrolled insertion).
template <int K>
struct TopK {
  float v[K];
  int i[K];
  __device__ void init() {
#pragma unroll
    for (int j = 0; j < K; ++j) {
      v[j] = -INFINITY;
      i[j] = 0x7fffffff;
    }
  }
  __device__ void push(float x, int xi) {
    if (!topk_better(x, xi, v[K - 1], i[K - 1])) return;
#pragma unroll
    for (int j = 0; j < K; ++j) {
      if (topk_better(x, xi, v[j], i[j])) {
        const float tv = v[j];
        const int ti = i[j];
        v[j] = x;
        i[j] = xi;
        x = tv;
        xi = ti;
      }
    }
  }
  __device__ void pop_front() {
#pragma unroll
    for (int j = 0; j + 1 < K; ++j) {
      v[j] = v[j + 1];
      i[j] = i[j + 1];
    }
    v[K - 1] = -INFINITY;
    i[K - 1] = 0x7fffffff;
  }
  // The warp's k best over every lane's list; round r's winner (bv, bi) is
  // handed to emit(r, bv, bi) on every lane.
  template <typename Emit>
  __device__ void warp_merge(int k, Emit emit) {
    for (int r = 0; r < k; ++r) {
      float bv = v[0];
      int bi = i[0];
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (topk_better(ov, oi, bv, bi)) {
          bv = ov;
          bi = oi;
        }
      }
      emit(r, bv, bi);
      if (i[0] == bi && v[0] == bv) pop_front();  // real indices are unique: only the owner pops
    }
  }
};

// Online (max, sum of exponentials) merge of two partial states.
__device__ __forceinline__ void lse_merge(float& m, float& s, float m2, float s2) {
  const float mm = fmaxf(m, m2);
  if (mm == -INFINITY) return;
  s = (m == -INFINITY ? 0.f : s * __expf(m - mm)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - mm));
  m = mm;
}

// Log-softmax of scale * logits (bf16 rows) and its top-k.  A cluster of 8
// CTAs shares one row: each CTA streams one eighth of it (16-byte loads, two
// in flight per thread), keeping an online max / sum of exponentials and a
// register top-k per thread, merged per warp and then per CTA; CTA 0 of the
// cluster merges the eight partials through distributed shared memory and
// writes (y - max) - log(sum), y = scale * logit in fp32.
template <int K>
__global__ void __cluster_dims__(kTopkCluster, 1, 1) __launch_bounds__(kTopkThreads)
logsoftmax_topk_kernel(const __nv_bfloat16* __restrict__ logits, int64_t vocab, float scale, int k,
                       float* __restrict__ top_v, int64_t* __restrict__ top_i) {
  __shared__ float s_m[kTopkWarps], s_s[kTopkWarps];
  __shared__ float c_v[kTopkWarps * K];
  __shared__ int c_i[kTopkWarps * K];
  __shared__ float p_ms[2];  // this CTA's (max, sum)
  __shared__ float p_v[K];
  __shared__ int p_i[K];
  cg::cluster_group cluster = cg::this_cluster();
  const int crank = (int)cluster.block_rank();
  const int64_t row = blockIdx.y;
  const __nv_bfloat16* x = logits + row * vocab;
  const int64_t chunk = ((vocab + 7) / 8 + kTopkCluster - 1) / kTopkCluster * 8;
  const int64_t lo = min(vocab, crank * chunk), hi = min(vocab, lo + chunk);
  float m = -INFINITY, sum = 0.f;
  TopK<K> t;
  t.init();
  auto take = [&](float y, int c) {
    if (y > m) {
      sum = sum * __expf(m - y) + 1.f;
      m = y;
    } else if (y != -INFINITY) {
      sum += __expf(y - m);
    }
    t.push(y, c);
  };
  auto take8 = [&](const uint4& u, int64_t c8) {
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
    for (int j = 0; j < 8; ++j) take(__bfloat162float(e[j]) * scale, (int)(c8 * 8 + j));
  };
  const bool vec = (vocab % 8 == 0) && ((reinterpret_cast<uintptr_t>(logits) & 15) == 0);
  if (vec) {  // lo and hi are multiples of 8 here
    const uint4* x8 = reinterpret_cast<const uint4*>(x);
    const int64_t hi8 = hi / 8;
    for (int64_t c = lo / 8 + threadIdx.x; c < hi8; c += 2 * kTopkThreads) {
      const uint4 u0 = __ldg(x8 + c);
      const bool two = c + kTopkThreads < hi8;
      uint4 u1 = make_uint4(0, 0, 0, 0);
      if (two) u1 = __ldg(x8 + c + kTopkThreads);
      take8(u0, c);
      if (two) take8(u1, c + kTopkThreads);
    }
  } else {
    for (int64_t c = lo + threadIdx.x; c < hi; c += kTopkThreads) take(__bfloat162float(x[c]) * scale, (int)c);
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o; o >>= 1)
    lse_merge(m, sum, __shfl_xor_sync(0xffffffffu, m, o), __shfl_xor_sync(0xffffffffu, sum, o));
  if (lane == 0) {
    s_m[warp] = m;
    s_s[warp] = sum;
  }
  t.warp_merge(k, [&](int r, float bv, int bi) {
    if (lane == 0) {
      c_v[warp * K + r] = bv;
      c_i[warp * K + r] = bi;
    }
  });
  __syncthreads();
  if (warp == 0) {  // this CTA's partial
    float M = lane < kTopkWarps ? s_m[lane] : -INFINITY;
    float S = lane < kTopkWarps ? s_s[lane] : 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1)
      lse_merge(M, S, __shfl_xor_sync(0xffffffffu, M, o), __shfl_xor_sync(0xffffffffu, S, o));
    TopK<K> f;
    f.init();
    if (lane < kTopkWarps)
      for (int r = 0; r < k; ++r) f.push(c_v[lane * K + r], c_i[lane * K + r]);
    f.warp_merge(k, [&](int r, float bv, int bi) {
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
    TopK<K> f;
    f.init();
    if (lane < kTopkCluster) {
      const float* ms = cluster.map_shared_rank(p_ms, lane);
      const float* pv = cluster.map_shared_rank(p_v, lane);
      const int* pi = cluster.map_shared_rank(p_i, lane);
      M = ms[0];
      S = ms[1];
      for (int r = 0; r < k; ++r) f.push(pv[r], pi[r]);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1)
      lse_merge(M, S, __shfl_xor_sync(0xffffffffu, M, o), __shfl_xor_sync(0xffffffffu, S, o));
    const float log_s = logf(S);
    f.warp_merge(k, [&](int r, float bv, int bi) {
      if (lane == 0) {
        top_v[row * k + r] = (bv - M) - log_s;
        top_i[row * k + r] = bi;
      }
    });
  }
  cluster.sync();  // peers keep their shared memory until CTA 0 has read it
}

}  // namespace
}  // namespace sf

extern "C" int sf_logsoftmax_topk(const void* logits, int64_t rows, int64_t vocab, float scale, int k,
                                  float* top_values, int64_t* top_indices, void* stream) {
  using namespace sf;
  SF_CHECK_ARG(rows >= 0 && rows <= 65535 && vocab > 0 && vocab < (1LL << 31), "invalid sizes");
  SF_CHECK_ARG(k >= 1 && k <= kMaxTopk && k <= vocab, "k must be in [1, %d] and at most vocab", kMaxTopk);
  if (rows == 0) return SF_OK;
  SF_CHECK_ARG(logits && top_values && top_indices, "null pointer argument");
  auto* x = static_cast<const __nv_bfloat16*>(logits);
  const dim3 grid(kTopkCluster, (unsigned)rows);
  cudaStream_t s = as_stream(stream);
  if (k <= 1) logsoftmax_topk_kernel<1><<<grid, kTopkThreads, 0, s>>>(x, vocab, scale, k, top_values, top_indices);
  else if (k <= 2) logsoftmax_topk_kernel<2><<<grid, kTopkThreads, 0, s>>>(x, vocab, scale, k, top_values, top_indices);
  else if (k <= 4) logsoftmax_topk_kernel<4><<<grid, kTopkThreads, 0, s>>>(x, vocab, scale, k, top_values, top_indices);
  else logsoftmax_topk_kernel<8><<<grid, kTopkThreads, 0, s>>>(x, vocab, scale, k, top_values, top_indices);
  SF_CHECK_LAUNCH();
  return SF_OK;
}
