// K2: dispatch (stable grouping of routes by expert) and the row gather.
//
// Restates the grouping of Qwen3OffloadedExperts
// (src/specfit/runtime/qwen3_offloaded_experts.py:173-178):
//   sorted_ids, positions = torch.sort(top_k_index.reshape(-1), stable=True)
//   unique, counts        = torch.unique_consecutive(sorted_ids, return_counts=True)
//   route_tokens          = positions // K
// without the host synchronisation of :175: the expert list stays on the
// device.  Within each expert the route positions ascend, which is also the
// token order of torch.where(top_k_index == e) (:120-122).  The grouping
// kernel itself (one CTA, stable per-warp scatter) is in dispatch.cuh.
#include "dispatch.cuh"

namespace sf {
namespace {

// Expert ids of the routes as given by the router (int64).  Anything
// outside [0, 2^31) maps to -2, which the grouping reports as invalid.
struct RouteIds {
  static constexpr bool kResetError = true;  // sf_moe_dispatch sets *error_flag to 0 or 1
  const int64_t* idx;
  unsigned long long* active_total;  // optional: += the number of active experts
  __device__ __forceinline__ void on_done(int num_active) const {
    if (active_total) atomicAdd(active_total, (unsigned long long)num_active);
  }
  __device__ __forceinline__ int size() const { return 0; }  // the count is passed explicitly
  __device__ __forceinline__ int operator()(int p) const {
    const int64_t e = idx[p];
    return (e >= 0 && e < 0x7fffffff) ? (int)e : -2;
  }
};

template <typename T, typename W>
__global__ void gather_kernel(const T* __restrict__ hidden, int H, const W* __restrict__ topk_w,
                              int K, const int32_t* __restrict__ sorted_pos, int64_t rows,
                              T* __restrict__ hidden_sorted, float* __restrict__ w_sorted,
                              bool vec) {
  pdl_wait();
  pdl_trigger();
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
    SF_CHECK_CUDA(launch_pdl(gather_kernel<T, float>, dim3((unsigned)rows), dim3(threads), 0,
                             stream, static_cast<const T*>(hidden), H,
                             static_cast<const float*>(topk_w), K, sorted_pos, rows,
                             static_cast<T*>(hidden_sorted), w_sorted, vec));
  else
    SF_CHECK_CUDA(launch_pdl(gather_kernel<T, __nv_bfloat16>, dim3((unsigned)rows), dim3(threads),
                             0, stream, static_cast<const T*>(hidden), H,
                             static_cast<const __nv_bfloat16*>(topk_w), K, sorted_pos, rows,
                             static_cast<T*>(hidden_sorted), w_sorted, vec));
  SF_CHECK_LAUNCH();
  return SF_OK;
}

}  // namespace
}  // namespace sf

extern "C" int sf_moe_dispatch(const int64_t* topk_index, int64_t tokens, int top_k,
                               int num_experts, int32_t* counts, int32_t* offsets,
                               int32_t* sorted_pos, int32_t* inv_pos, int32_t* active,
                               int32_t* num_active, int32_t* error_flag, void* stream) {
  return sf_moe_dispatch_ex(topk_index, tokens, top_k, num_experts, counts, offsets, sorted_pos,
                            inv_pos, active, num_active, error_flag, nullptr, stream);
}

extern "C" int sf_moe_dispatch_ex(const int64_t* topk_index, int64_t tokens, int top_k,
                                  int num_experts, int32_t* counts, int32_t* offsets,
                                  int32_t* sorted_pos, int32_t* inv_pos, int32_t* active,
                                  int32_t* num_active, int32_t* error_flag,
                                  int64_t* active_total, void* stream) {
  using namespace sf;
  SF_CHECK_ARG(tokens >= 0 && top_k > 0, "tokens must be >= 0 and top_k > 0");
  SF_CHECK_ARG(num_experts > 0 && num_experts <= grouping::kThreads,
               "num_experts must be in [1, 1024]");
  SF_CHECK_ARG(tokens * top_k < (int64_t)1 << 30, "too many routes");
  SF_CHECK_ARG(counts && offsets && active && num_active && error_flag, "null pointer argument");
  const int n = (int)(tokens * top_k);
  SF_CHECK_ARG(n == 0 || (topk_index && sorted_pos && inv_pos), "null pointer argument");
  const size_t smem = grouping::smem_bytes(num_experts);
  auto kernel = grouping::group_kernel<RouteIds>;
  if (smem > 48 * 1024)
    SF_CHECK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem));
  SF_CHECK_CUDA(launch_pdl(kernel, dim3(1), dim3(grouping::kThreads), smem, as_stream(stream),
                           RouteIds{topk_index, reinterpret_cast<unsigned long long*>(active_total)},
                           n, num_experts, false, counts, offsets, sorted_pos, inv_pos, active,
                           num_active, error_flag, nullptr));
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
