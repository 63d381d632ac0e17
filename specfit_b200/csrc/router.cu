// K1: MoE router — logits, fp32 softmax, top-k, renormalisation.
//
// Restates Qwen3MoeTopKRouter.forward (transformers/models/qwen3_moe/
// modeling_qwen3_moe.py:263-272):
//   logits = F.linear(h, W)            -> model dtype
//   probs  = softmax(logits, fp32)
//   top    = topk(probs, k)            -> (values, indices)
//   top   /= top.sum() if norm_topk_prob
//
// Numerics: each logit is an exact fp64 dot product (bf16*bf16 and f32*f32
// products are exact in fp64) rounded ONCE to the model dtype, so the result
// is the correctly rounded logit and does not depend on a reduction order.
// Top-k runs on the logits ordered by (value desc, expert id asc); softmax is
// monotone, so this equals topk(probs) with the tie rule "lower id wins".
//
// Two launches: a logits kernel that spreads T*E*H fp64 FMAs over the whole
// GPU (a CTA per 8 tokens x 16 experts), and a warp-per-token top-k kernel.
#include <math.h>

#include <mutex>

#include "common.cuh"

namespace sf {
namespace {

constexpr int kTokTile = 8;    // tokens per logits CTA
constexpr int kExpTile = 16;   // experts per logits CTA (2 per warp)
constexpr int kWarps = 8;
constexpr int kNone = 0x7fffffff;  // "no expert" marker in the top-k reduction

// Correctly rounded double -> bf16 (as float): keep 8 significant bits,
// round half to even.  frexp/rint/ldexp are exact.
__device__ __forceinline__ float round_f64_to_bf16(double d) {
  if (d == 0.0 || !isfinite(d)) return (float)d;
  int e;
  double m = frexp(d, &e);           // d = m * 2^e, 0.5 <= |m| < 1
  double r = rint(m * 256.0);        // round to 8 significant bits (RNE)
  return (float)ldexp(r / 256.0, e);  // exact in float (8-bit mantissa)
}

template <typename T>
__device__ __forceinline__ float round_logit(double d);
template <>
__device__ __forceinline__ float round_logit<float>(double d) { return __double2float_rn(d); }
template <>
__device__ __forceinline__ float round_logit<__nv_bfloat16>(double d) { return round_f64_to_bf16(d); }

template <typename T, bool kVec>
__global__ void __launch_bounds__(kWarps * 32)
router_logits_kernel(const T* __restrict__ x, const T* __restrict__ w, int64_t tokens, int hidden,
                     int experts, float* __restrict__ logits_f32, T* __restrict__ logits_out) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t t0 = (int64_t)blockIdx.x * kTokTile;
  const int ntok = (int)((tokens - t0) < kTokTile ? (tokens - t0) : kTokTile);
  constexpr int kV = 16 / sizeof(T);  // elements per 16-byte vector

  for (int ej = warp; ej < kExpTile; ej += kWarps) {
    const int e = blockIdx.y * kExpTile + ej;
    if (e >= experts) break;
    double acc[kTokTile];
#pragma unroll
    for (int i = 0; i < kTokTile; ++i) acc[i] = 0.0;
    const T* wrow = w + (int64_t)e * hidden;
    if (kVec) {
      for (int h = lane * kV; h < hidden; h += 32 * kV) {
        T wv[kV];
        *reinterpret_cast<uint4*>(wv) = *reinterpret_cast<const uint4*>(wrow + h);
#pragma unroll
        for (int i = 0; i < kTokTile; ++i) {
          if (i < ntok) {
            T xv[kV];
            *reinterpret_cast<uint4*>(xv) =
                *reinterpret_cast<const uint4*>(x + (t0 + i) * hidden + h);
#pragma unroll
            for (int v = 0; v < kV; ++v)
              acc[i] = fma((double)to_f32(xv[v]), (double)to_f32(wv[v]), acc[i]);
          }
        }
      }
    } else {
      for (int h = lane; h < hidden; h += 32) {
        const double wv = (double)to_f32(wrow[h]);
#pragma unroll
        for (int i = 0; i < kTokTile; ++i)
          if (i < ntok) acc[i] = fma((double)to_f32(x[(t0 + i) * hidden + h]), wv, acc[i]);
      }
    }
#pragma unroll
    for (int i = 0; i < kTokTile; ++i) {
      double s = acc[i];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
      if (lane == 0 && i < ntok) {
        const float r = round_logit<T>(s);
        logits_f32[(t0 + i) * experts + e] = r;
        if (logits_out) logits_out[(t0 + i) * experts + e] = from_f32<T>(r);
      }
    }
  }
}

// Warp per token.  Lane l owns experts l, l+32, ... (up to 32 per lane).
__global__ void __launch_bounds__(kWarps * 32)
router_topk_kernel(const float* __restrict__ logits, int64_t tokens, int experts, int top_k,
                   int norm, float* __restrict__ probs, float* __restrict__ topk_w,
                   int64_t* __restrict__ topk_idx) {
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (t >= tokens) return;
  const float* row = logits + t * experts;
  const int per_lane = (experts + 31) / 32;

  float m = -INFINITY;
  for (int j = 0; j < per_lane; ++j) {
    const int e = lane + 32 * j;
    if (e < experts) m = fmaxf(m, row[e]);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  float s = 0.f;
  for (int j = 0; j < per_lane; ++j) {
    const int e = lane + 32 * j;
    if (e < experts) s += expf(row[e] - m);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  for (int j = 0; j < per_lane; ++j) {
    const int e = lane + 32 * j;
    if (e < experts) probs[t * experts + e] = expf(row[e] - m) / s;
  }

  // Top-k by (logit desc, id asc).  taken: bit j <-> expert lane + 32 j.
  uint32_t taken = 0;
  float sel_p = 0.f;  // lane k < top_k keeps the k-th selected prob
  int sel_e = 0;
  for (int k = 0; k < top_k; ++k) {
    // Lane-local best; e grows with j, so a strict '>' keeps the lower id on ties.
    float bv = -INFINITY;
    int be = kNone;
    for (int j = 0; j < per_lane; ++j) {
      const int e = lane + 32 * j;
      if (e < experts && !((taken >> j) & 1u)) {
        const float v = row[e];
        if (be == kNone || v > bv) {
          bv = v;
          be = e;
        }
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const int oe = __shfl_xor_sync(0xffffffffu, be, off);
      if (oe != kNone && (be == kNone || ov > bv || (ov == bv && oe < be))) {
        bv = ov;
        be = oe;
      }
    }
    if (be != kNone && (be & 31) == lane) taken |= 1u << (be >> 5);
    if (lane == k) {
      sel_e = be;
      sel_p = expf(bv - m) / s;
    }
  }
  if (norm) {
    // Sequential fp32 sum in k order, as the oracle does.
    float denom = 0.f;
    for (int k = 0; k < top_k; ++k) denom += __shfl_sync(0xffffffffu, sel_p, k);
    sel_p = sel_p / denom;
  }
  if (lane < top_k) {
    topk_w[t * top_k + lane] = sel_p;
    topk_idx[t * top_k + lane] = (int64_t)sel_e;
  }
}

template <typename T>
int launch_router(const void* hidden, const void* weight, int64_t tokens, int H, int E, int K,
                  int norm, float* probs, float* topk_w, int64_t* topk_idx, void* logits_out,
                  float* logits_ws, cudaStream_t stream) {
  const T* x = static_cast<const T*>(hidden);
  const T* w = static_cast<const T*>(weight);
  dim3 grid((unsigned)((tokens + kTokTile - 1) / kTokTile), (unsigned)((E + kExpTile - 1) / kExpTile));
  const bool vec = (H % (16 / (int)sizeof(T)) == 0) && aligned16(x) && aligned16(w);
  if (vec)
    router_logits_kernel<T, true><<<grid, kWarps * 32, 0, stream>>>(x, w, tokens, H, E, logits_ws,
                                                                    static_cast<T*>(logits_out));
  else
    router_logits_kernel<T, false><<<grid, kWarps * 32, 0, stream>>>(x, w, tokens, H, E, logits_ws,
                                                                     static_cast<T*>(logits_out));
  SF_CHECK_LAUNCH();
  router_topk_kernel<<<(unsigned)((tokens + kWarps - 1) / kWarps), kWarps * 32, 0, stream>>>(
      logits_ws, tokens, E, K, norm, probs, topk_w, topk_idx);
  SF_CHECK_LAUNCH();
  return SF_OK;
}

}  // namespace
}  // namespace sf

extern "C" size_t sf_router_topk_workspace_bytes(int64_t tokens, int num_experts) {
  if (tokens < 0 || num_experts < 0) return 0;
  return (size_t)tokens * (size_t)num_experts * sizeof(float);
}

extern "C" int sf_router_topk(const void* hidden, const void* router_weight, int dtype,
                              int64_t tokens, int hidden_size, int num_experts, int top_k,
                              int norm_topk_prob, float* probs, float* topk_weights,
                              int64_t* topk_index, void* logits_out, void* workspace,
                              size_t workspace_bytes, void* stream) {
  using namespace sf;
  SF_CHECK_ARG(tokens >= 0, "tokens must be non-negative");
  SF_CHECK_ARG(hidden_size > 0, "hidden_size must be positive");
  SF_CHECK_ARG(num_experts > 0 && num_experts <= 1024, "num_experts must be in [1, 1024]");
  SF_CHECK_ARG(top_k > 0 && top_k <= 32 && top_k <= num_experts, "top_k must be in [1, min(32, E)]");
  if (tokens == 0) return SF_OK;
  SF_CHECK_ARG(hidden && router_weight && probs && topk_weights && topk_index,
               "null pointer argument");
  if (workspace_bytes < sf_router_topk_workspace_bytes(tokens, num_experts) || !workspace)
    return set_error(SF_ERR_WORKSPACE, "router workspace needs %zu bytes",
                     sf_router_topk_workspace_bytes(tokens, num_experts));
  float* ws = static_cast<float*>(workspace);
  if (dtype == SF_DTYPE_BF16)
    return launch_router<__nv_bfloat16>(hidden, router_weight, tokens, hidden_size, num_experts,
                                        top_k, norm_topk_prob, probs, topk_weights, topk_index,
                                        logits_out, ws, as_stream(stream));
  if (dtype == SF_DTYPE_F32)
    return launch_router<float>(hidden, router_weight, tokens, hidden_size, num_experts, top_k,
                                norm_topk_prob, probs, topk_weights, topk_index, logits_out, ws,
                                as_stream(stream));
  return set_error(SF_ERR_UNSUPPORTED, "router dtype %d is not supported", dtype);
}

// ---------------------------------------------------------------------------
// Allocation-free router.
//
// Some callers cannot hand this library a workspace because they cannot
// allocate device memory at the point of the call: code that runs while a
// stream is being captured into a CUDA graph (cudaMalloc is not allowed
// there), plugins hosted by a serving runtime that reserves the GPU's memory
// for its own pools and gives extensions none, and latency-critical paths
// where cudaMalloc's implicit device-wide synchronisation is unacceptable.
// sf_router_topk_noalloc serves them: its scratch (the fp32 logits between
// the two router passes) is this file-scope device array, which every GPU
// that loads the library holds until the process exits.

namespace sf {
namespace {

// Maximum tokens * experts of one allocation-free call: 2^19 floats = 2 MiB
// (e.g. 4096 tokens at 128 experts).
constexpr int64_t kNoAllocScratchFloats = int64_t(1) << 19;
static __device__ __align__(256) float g_router_scratch[kNoAllocScratchFloats];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
float* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_router_scratch on the current device, looked up once
// per device.  The host-side symbol is only a stand-in and must never be
// passed to a kernel.
int router_scratch(float** out) {
  int dev = 0;
  SF_CHECK_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return set_error(SF_ERR_UNSUPPORTED, "device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    SF_CHECK_CUDA(cudaGetSymbolAddress(&p, g_router_scratch));
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return SF_OK;
}

}  // namespace
}  // namespace sf

extern "C" int64_t sf_router_topk_noalloc_max_elems(void) { return sf::kNoAllocScratchFloats; }

extern "C" int sf_router_topk_noalloc(const void* hidden, const void* router_weight, int dtype,
                                      int64_t tokens, int hidden_size, int num_experts, int top_k,
                                      int norm_topk_prob, float* probs, float* topk_weights,
                                      int64_t* topk_index, void* logits_out, void* stream) {
  using namespace sf;
  SF_CHECK_ARG(tokens >= 0, "tokens must be non-negative");
  SF_CHECK_ARG(hidden_size > 0, "hidden_size must be positive");
  SF_CHECK_ARG(num_experts > 0 && num_experts <= 1024, "num_experts must be in [1, 1024]");
  SF_CHECK_ARG(top_k > 0 && top_k <= 32 && top_k <= num_experts, "top_k must be in [1, min(32, E)]");
  if (tokens * (int64_t)num_experts > kNoAllocScratchFloats)
    return set_error(SF_ERR_WORKSPACE,
                     "tokens * num_experts = %lld exceeds the allocation-free router's built-in "
                     "scratch of %lld elements; use sf_router_topk with a workspace",
                     (long long)(tokens * (int64_t)num_experts), (long long)kNoAllocScratchFloats);
  if (tokens == 0) return SF_OK;
  SF_CHECK_ARG(hidden && router_weight && probs && topk_weights && topk_index,
               "null pointer argument");
  float* ws = nullptr;
  if (int rc = router_scratch(&ws)) return rc;
  if (dtype == SF_DTYPE_BF16)
    return launch_router<__nv_bfloat16>(hidden, router_weight, tokens, hidden_size, num_experts,
                                        top_k, norm_topk_prob, probs, topk_weights, topk_index,
                                        logits_out, ws, as_stream(stream));
  if (dtype == SF_DTYPE_F32)
    return launch_router<float>(hidden, router_weight, tokens, hidden_size, num_experts, top_k,
                                norm_topk_prob, probs, topk_weights, topk_index, logits_out, ws,
                                as_stream(stream));
  return set_error(SF_ERR_UNSUPPORTED, "router dtype %d is not supported", dtype);
}
