// K2: dispatch (stable grouping of routes by expert) and the row gather.
//
// Restates the grouping of Qwen3OffloadedExperts
// (src/specfit/runtime/qwen3_offloaded_experts.py:173-178):
//   sorted_ids, positions = torch.sort(top_k_index.reshape(-1), stable=True)
//   unique, counts        = torch.unique_consecutive(sorted_ids, return_counts=True)
//   route_tokens          = positions // K
// without the host synchronisation of :175: the expert list stays on the
// device.  Within each expert the route positions ascend, which is also the
// token order of torch.where(top_k_index == e) (:120-122).
//
// One CTA of 1024 threads (32 warps).  The T*K positions are cut into 32
// contiguous segments, one per warp.  Pass 1 counts each segment's routes
// per expert; a per-expert prefix over the segments plus the per-expert
// offsets gives every warp its write cursor; pass 2 walks each segment in
// 32-route chunks in order, ranking equal ids within a chunk with
// __match_any_sync, so the scatter is stable and deterministic.
#include "common.cuh"

namespace sf {
namespace {

constexpr int kThreads = 1024;
constexpr int kSegs = kThreads / 32;

__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_sums, int* total) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int o = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += o;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int w = warp_sums[lane];
    int wi = w;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int o = __shfl_up_sync(0xffffffffu, wi, off);
      if (lane >= off) wi += o;
    }
    warp_sums[lane] = wi - w;  // exclusive
    if (lane == 31) *total = wi;
  }
  __syncthreads();
  const int r = warp_sums[warp] + incl - v;
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(kThreads)
dispatch_kernel(const int64_t* __restrict__ idx, int n, int E, int32_t* __restrict__ counts,
                int32_t* __restrict__ offsets, int32_t* __restrict__ sorted_pos,
                int32_t* __restrict__ inv_pos, int32_t* __restrict__ active,
                int32_t* __restrict__ num_active, int32_t* __restrict__ error_flag) {
  extern __shared__ int smem[];
  int* seg_cnt = smem;                  // [kSegs][E]
  int* off = seg_cnt + kSegs * E;       // [E]
  __shared__ int warp_sums[32];
  __shared__ int total_routes, total_active;

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int seg_len = (n + kSegs - 1) / kSegs;
  const int seg_lo = min(n, warp * seg_len);
  const int seg_hi = min(n, seg_lo + seg_len);

  for (int i = threadIdx.x; i < kSegs * E; i += kThreads) seg_cnt[i] = 0;
  __syncthreads();

  // Pass 1: per-segment counts.
  for (int p = seg_lo + lane; p < seg_hi; p += 32) {
    const int64_t e = idx[p];
    if (e >= 0 && e < E)
      atomicAdd(&seg_cnt[warp * E + (int)e], 1);
    else
      *error_flag = 1;
  }
  __syncthreads();

  // Per expert: prefix over segments (in place) and the total count.
  // E <= 1024 = kThreads, so one pass of threads covers every expert.
  int cnt = 0;
  const int e = threadIdx.x;
  if (e < E) {
    for (int s = 0; s < kSegs; ++s) {
      const int c = seg_cnt[s * E + e];
      seg_cnt[s * E + e] = cnt;
      cnt += c;
    }
    counts[e] = cnt;
  }
  const int base = block_exclusive_scan(e < E ? cnt : 0, warp_sums, &total_routes);
  const int act_rank = block_exclusive_scan((e < E && cnt > 0) ? 1 : 0, warp_sums, &total_active);
  if (e < E) {
    off[e] = base;
    offsets[e] = base;
    if (cnt > 0) active[act_rank] = e;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    offsets[E] = total_routes;
    *num_active = total_active;
  }
  for (int i = total_active + threadIdx.x; i < E; i += kThreads) active[i] = -1;
  for (int i = total_routes + threadIdx.x; i < n; i += kThreads) sorted_pos[i] = -1;

  // Pass 2: stable scatter, one segment per warp, 32 routes at a time.
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int c0 = seg_lo; c0 < seg_hi; c0 += 32) {
    const int p = c0 + lane;
    int key = E + lane;  // unique non-matching key for idle / invalid lanes
    bool valid = false;
    if (p < seg_hi) {
      const int64_t ev = idx[p];
      if (ev >= 0 && ev < E) {
        key = (int)ev;
        valid = true;
      } else {
        inv_pos[p] = -1;
      }
    }
    const unsigned peers = __match_any_sync(0xffffffffu, key);
    int dst = 0;
    if (valid) dst = off[key] + seg_cnt[warp * E + key] + __popc(peers & lt_mask);
    __syncwarp();
    if (valid) {
      sorted_pos[dst] = p;
      inv_pos[p] = dst;
      if ((peers & lt_mask) == 0) seg_cnt[warp * E + key] += __popc(peers);
    }
    __syncwarp();
  }
}

template <typename T, typename W>
__global__ void gather_kernel(const T* __restrict__ hidden, int H, const W* __restrict__ topk_w,
                              int K, const int32_t* __restrict__ sorted_pos, int64_t rows,
                              T* __restrict__ hidden_sorted, float* __restrict__ w_sorted,
                              bool vec) {
  const int64_t r = blockIdx.x;
  if (r >= rows) return;
  const int32_t p = sorted_pos[r];
  T* dst = hidden_sorted + r * H;
  if (p < 0) {
    for (int h = threadIdx.x; h < H; h += blockDim.x) dst[h] = from_f32<T>(0.f);
    if (threadIdx.x == 0) w_sorted[r] = 0.f;
    return;
  }
  const T* src = hidden + (int64_t)(p / K) * H;
  if (vec) {
    constexpr int kV = 16 / sizeof(T);
    for (int h = threadIdx.x * kV; h < H; h += blockDim.x * kV)
      *reinterpret_cast<uint4*>(dst + h) = *reinterpret_cast<const uint4*>(src + h);
  } else {
    for (int h = threadIdx.x; h < H; h += blockDim.x) dst[h] = src[h];
  }
  if (threadIdx.x == 0) w_sorted[r] = to_f32(topk_w[p]);
}

template <typename T>
int launch_gather_w(const void* hidden, int64_t tokens, int H, const void* topk_w, int wdt, int K,
                    const int32_t* sorted_pos, void* hidden_sorted, float* w_sorted,
                    cudaStream_t stream) {
  const int64_t rows = tokens * K;
  const bool vec = (H % (16 / (int)sizeof(T)) == 0) && aligned16(hidden) && aligned16(hidden_sorted);
  const int threads = 128;
  if (wdt == SF_DTYPE_F32)
    gather_kernel<T, float><<<(unsigned)rows, threads, 0, stream>>>(
        static_cast<const T*>(hidden), H, static_cast<const float*>(topk_w), K, sorted_pos, rows,
        static_cast<T*>(hidden_sorted), w_sorted, vec);
  else
    gather_kernel<T, __nv_bfloat16><<<(unsigned)rows, threads, 0, stream>>>(
        static_cast<const T*>(hidden), H, static_cast<const __nv_bfloat16*>(topk_w), K, sorted_pos,
        rows, static_cast<T*>(hidden_sorted), w_sorted, vec);
  SF_CHECK_LAUNCH();
  return SF_OK;
}

}  // namespace
}  // namespace sf

extern "C" int sf_moe_dispatch(const int64_t* topk_index, int64_t tokens, int top_k,
                               int num_experts, int32_t* counts, int32_t* offsets,
                               int32_t* sorted_pos, int32_t* inv_pos, int32_t* active,
                               int32_t* num_active, int32_t* error_flag, void* stream) {
  using namespace sf;
  SF_CHECK_ARG(tokens >= 0 && top_k > 0, "tokens must be >= 0 and top_k > 0");
  SF_CHECK_ARG(num_experts > 0 && num_experts <= kThreads, "num_experts must be in [1, 1024]");
  SF_CHECK_ARG(tokens * top_k < (int64_t)1 << 30, "too many routes");
  SF_CHECK_ARG(counts && offsets && active && num_active && error_flag, "null pointer argument");
  const int n = (int)(tokens * top_k);
  SF_CHECK_ARG(n == 0 || (topk_index && sorted_pos && inv_pos), "null pointer argument");
  const size_t smem = (size_t)(kSegs + 1) * num_experts * sizeof(int);
  if (smem > 48 * 1024)
    SF_CHECK_CUDA(cudaFuncSetAttribute(dispatch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem));
  dispatch_kernel<<<1, kThreads, smem, as_stream(stream)>>>(topk_index, n, num_experts, counts,
                                                            offsets, sorted_pos, inv_pos, active,
                                                            num_active, error_flag);
  SF_CHECK_LAUNCH();
  return SF_OK;
}

extern "C" int sf_moe_gather(const void* hidden, int dtype, int64_t tokens, int hidden_size,
                             const void* topk_weights, int weight_dtype, int top_k,
                             const int32_t* sorted_pos, void* hidden_sorted, float* weights_sorted,
                             void* stream) {
  using namespace sf;
  SF_CHECK_ARG(tokens >= 0 && top_k > 0 && hidden_size > 0, "invalid sizes");
  if (tokens == 0) return SF_OK;
  SF_CHECK_ARG(hidden && topk_weights && sorted_pos && hidden_sorted && weights_sorted,
               "null pointer argument");
  SF_CHECK_ARG(weight_dtype == SF_DTYPE_F32 || weight_dtype == SF_DTYPE_BF16,
               "unsupported weight dtype %d", weight_dtype);
  if (dtype == SF_DTYPE_BF16)
    return launch_gather_w<__nv_bfloat16>(hidden, tokens, hidden_size, topk_weights, weight_dtype,
                                          top_k, sorted_pos, hidden_sorted, weights_sorted,
                                          as_stream(stream));
  if (dtype == SF_DTYPE_F32)
    return launch_gather_w<float>(hidden, tokens, hidden_size, topk_weights, weight_dtype, top_k,
                                  sorted_pos, hidden_sorted, weights_sorted, as_stream(stream));
  return set_error(SF_ERR_UNSUPPORTED, "gather dtype %d is not supported", dtype);
}
