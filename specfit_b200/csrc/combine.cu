// K4: combine — per-token reduction of the weighted expert rows.
//
// Restates the index_add_ reduction of Qwen3OffloadedExperts
// (src/specfit/runtime/qwen3_offloaded_experts.py:144-163 and :200-202):
// the output starts at zero and each expert's weighted rows are added in
// ascending expert id (CANONICAL) or in execution order (ARRIVAL_ORDER), each
// add rounding back to the model dtype.  Here every token gathers its own K
// contributions (route positions t*K+k -> sorted rows via inv_pos), orders
// them by (rank[expert], k) and adds them in that order, so no atomics and no
// per-expert launches are needed and the result is deterministic.
#include "common.cuh"

namespace sf {
namespace {

constexpr int kMaxK = 32;

template <typename T, int kV>
__global__ void combine_kernel(const T* __restrict__ ys, const int32_t* __restrict__ inv_pos,
                               const int64_t* __restrict__ idx, const int32_t* __restrict__ rank,
                               int E, int K, int H, int reduce, T* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  __shared__ int order_rows[kMaxK];
  __shared__ int n_valid;
  const int64_t t = blockIdx.x;
  if (threadIdx.x == 0) {
    int keys[kMaxK], rows[kMaxK];
    int n = 0;
    for (int k = 0; k < K; ++k) {
      const int r = inv_pos[t * K + k];
      const int64_t e = idx[t * K + k];
      if (r < 0 || e < 0 || e >= E) continue;
      const int key = rank ? rank[e] : (int)e;
      // Insertion by (key, k): k grows, so equal keys keep k order.
      int j = n++;
      while (j > 0 && keys[j - 1] > key) {
        keys[j] = keys[j - 1];
        rows[j] = rows[j - 1];
        --j;
      }
      keys[j] = key;
      rows[j] = r;
    }
    for (int j = 0; j < n; ++j) order_rows[j] = rows[j];
    n_valid = n;
  }
  __syncthreads();
  const int n = n_valid;
  const int h0 = (blockIdx.y * blockDim.x + threadIdx.x) * kV;
  if (h0 >= H) return;
  float acc[kV];
#pragma unroll
  for (int v = 0; v < kV; ++v) acc[v] = 0.f;
  for (int j = 0; j < n; ++j) {
    const T* src = ys + (int64_t)order_rows[j] * H + h0;
    T vals[kV];
    if (kV * sizeof(T) == 16) {
      *reinterpret_cast<uint4*>(vals) = *reinterpret_cast<const uint4*>(src);
    } else {
#pragma unroll
      for (int v = 0; v < kV; ++v) vals[v] = src[v];
    }
#pragma unroll
    for (int v = 0; v < kV; ++v) {
      const float s = acc[v] + to_f32(vals[v]);
      acc[v] = (reduce == SF_REDUCE_MODEL_DTYPE) ? round_to<T>(s) : s;
    }
  }
  T* dst = out + t * H + h0;
  T res[kV];
#pragma unroll
  for (int v = 0; v < kV; ++v) res[v] = from_f32<T>(acc[v]);
  if (kV * sizeof(T) == 16) {
    *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(res);
  } else {
#pragma unroll
    for (int v = 0; v < kV; ++v) dst[v] = res[v];
  }
}

template <typename T>
int launch_combine(const void* ys, const int32_t* inv_pos, const int64_t* idx, const int32_t* rank,
                   int E, int64_t tokens, int K, int H, int reduce, void* out,
                   cudaStream_t stream) {
  constexpr int kV = 16 / sizeof(T);
  const bool vec = (H % kV == 0) && aligned16(ys) && aligned16(out);
  const int threads = 256;
  if (vec) {
    dim3 grid((unsigned)tokens, (unsigned)((H / kV + threads - 1) / threads));
    SF_CHECK_CUDA(launch_pdl(combine_kernel<T, kV>, dim3(grid), dim3(threads), 0, stream,
                             static_cast<const T*>(ys), inv_pos, idx, rank, E, K, H, reduce,
                             static_cast<T*>(out)));
  } else {
    dim3 grid((unsigned)tokens, (unsigned)((H + threads - 1) / threads));
    SF_CHECK_CUDA(launch_pdl(combine_kernel<T, 1>, dim3(grid), dim3(threads), 0, stream,
                             static_cast<const T*>(ys), inv_pos, idx, rank, E, K, H, reduce,
                             static_cast<T*>(out)));
  }
  SF_CHECK_LAUNCH();
  return SF_OK;
}

// Combine fused with the layer's residual add and the next RMSNorm, for a
// CTA per token (H <= 8192, 8 columns per thread per chunk): the token's
// combined row is formed exactly as combine_kernel forms it (same order, same
// roundings, bf16), then exactly as add_rmsnorm_kernel: h = bf16(res + moe),
// written to res_out, and out = bf16(w * bf16(h * rsqrt(mean(h^2) + eps))).
constexpr int kCnThreads = 256;

__global__ void __launch_bounds__(kCnThreads)
combine_add_rmsnorm_kernel(const __nv_bfloat16* __restrict__ ys, const int32_t* __restrict__ inv_pos,
                           const int64_t* __restrict__ idx, const int32_t* __restrict__ rank, int E,
                           int K, int H, int reduce, const __nv_bfloat16* __restrict__ res_in,
                           __nv_bfloat16* __restrict__ res_out, const __nv_bfloat16* __restrict__ w,
                           float eps, __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  __shared__ int order_rows[kMaxK];
  __shared__ int n_valid;
  __shared__ float part[kCnThreads / 32];
  const int64_t t = blockIdx.x;
  if (threadIdx.x == 0) {
    int keys[kMaxK], rows[kMaxK];
    int n = 0;
    for (int k = 0; k < K; ++k) {
      const int r = inv_pos[t * K + k];
      const int64_t e = idx[t * K + k];
      if (r < 0 || e < 0 || e >= E) continue;
      const int key = rank ? rank[e] : (int)e;
      int j = n++;
      while (j > 0 && keys[j - 1] > key) {
        keys[j] = keys[j - 1];
        rows[j] = rows[j - 1];
        --j;
      }
      keys[j] = key;
      rows[j] = r;
    }
    for (int j = 0; j < n; ++j) order_rows[j] = rows[j];
    n_valid = n;
  }
  __syncthreads();
  const int n = n_valid;
  float h[4 * 8];  // up to 4 chunks of 8 columns per thread
  float ss = 0.f;
  int nch = 0;
  for (int c0 = threadIdx.x * 8; c0 < H; c0 += kCnThreads * 8, ++nch) {
    float acc[8];
#pragma unroll
    for (int v = 0; v < 8; ++v) acc[v] = 0.f;
    for (int j = 0; j < n; ++j) {
      __nv_bfloat16 vals[8];
      *reinterpret_cast<uint4*>(vals) = *reinterpret_cast<const uint4*>(ys + (int64_t)order_rows[j] * H + c0);
#pragma unroll
      for (int v = 0; v < 8; ++v) {
        const float sum = acc[v] + __bfloat162float(vals[v]);
        acc[v] = (reduce == SF_REDUCE_MODEL_DTYPE) ? round_to<__nv_bfloat16>(sum) : sum;
      }
    }
    __nv_bfloat16 rv[8], hv[8];
    *reinterpret_cast<uint4*>(rv) = *reinterpret_cast<const uint4*>(res_in + t * H + c0);
#pragma unroll
    for (int v = 0; v < 8; ++v) {
      const float moe = __bfloat162float(__float2bfloat16_rn(acc[v]));  // the combined bf16 row
      hv[v] = __float2bfloat16_rn(__bfloat162float(rv[v]) + moe);
      const float f = __bfloat162float(hv[v]);
      h[nch * 8 + v] = f;
      ss += f * f;
    }
    *reinterpret_cast<uint4*>(res_out + t * H + c0) = *reinterpret_cast<uint4*>(hv);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kCnThreads / 32; ++i) tot += part[i];
  const float r = rsqrtf(tot / (float)H + eps);
  int ch = 0;
  for (int c0 = threadIdx.x * 8; c0 < H; c0 += kCnThreads * 8, ++ch) {
    __nv_bfloat16 wv[8], ov[8];
    *reinterpret_cast<uint4*>(wv) = *reinterpret_cast<const uint4*>(w + c0);
#pragma unroll
    for (int v = 0; v < 8; ++v)
      ov[v] = __float2bfloat16_rn(__bfloat162float(wv[v]) *
                                  __bfloat162float(__float2bfloat16_rn(h[ch * 8 + v] * r)));
    *reinterpret_cast<uint4*>(out + t * H + c0) = *reinterpret_cast<uint4*>(ov);
  }
}

}  // namespace
}  // namespace sf

extern "C" int sf_moe_combine(const void* out_sorted, int dtype, const int32_t* inv_pos,
                              const int64_t* topk_index, const int32_t* expert_rank,
                              int num_experts, int64_t tokens, int top_k, int hidden_size,
                              int reduce, void* out, void* stream) {
  using namespace sf;
  SF_CHECK_ARG(tokens >= 0 && hidden_size > 0 && num_experts > 0, "invalid sizes");
  SF_CHECK_ARG(top_k > 0 && top_k <= kMaxK, "top_k must be in [1, 32]");
  SF_CHECK_ARG(reduce == SF_REDUCE_MODEL_DTYPE || reduce == SF_REDUCE_F32, "invalid reduce mode");
  if (tokens == 0) return SF_OK;
  SF_CHECK_ARG(out_sorted && inv_pos && topk_index && out, "null pointer argument");
  SF_CHECK_ARG(out != out_sorted, "out may not alias out_sorted");
  if (dtype == SF_DTYPE_BF16)
    return launch_combine<__nv_bfloat16>(out_sorted, inv_pos, topk_index, expert_rank, num_experts,
                                         tokens, top_k, hidden_size, reduce, out,
                                         as_stream(stream));
  if (dtype == SF_DTYPE_F32)
    return launch_combine<float>(out_sorted, inv_pos, topk_index, expert_rank, num_experts, tokens,
                                 top_k, hidden_size, reduce, out, as_stream(stream));
  return set_error(SF_ERR_UNSUPPORTED, "combine dtype %d is not supported", dtype);
}

extern "C" int sf_moe_combine_add_rmsnorm(const void* out_sorted, const int32_t* inv_pos,
                                          const int64_t* topk_index, const int32_t* expert_rank,
                                          int num_experts, int64_t tokens, int top_k,
                                          int hidden_size, int reduce, const void* residual_in,
                                          void* residual_out, const void* norm_weight, float eps,
                                          void* out, void* stream) {
  using namespace sf;
  SF_CHECK_ARG(tokens >= 0 && num_experts > 0, "invalid sizes");
  SF_CHECK_ARG(hidden_size > 0 && hidden_size % 8 == 0 && hidden_size <= 8192,
               "hidden_size must be a multiple of 8 and at most 8192");
  SF_CHECK_ARG(top_k > 0 && top_k <= kMaxK, "top_k must be in [1, 32]");
  SF_CHECK_ARG(reduce == SF_REDUCE_MODEL_DTYPE || reduce == SF_REDUCE_F32, "invalid reduce mode");
  if (tokens == 0) return SF_OK;
  SF_CHECK_ARG(out_sorted && inv_pos && topk_index && residual_in && residual_out && norm_weight && out,
               "null pointer argument");
  SF_CHECK_ARG(aligned16(out_sorted) && aligned16(residual_in) && aligned16(residual_out) &&
                   aligned16(norm_weight) && aligned16(out),
               "rows must be 16-byte aligned");
  SF_CHECK_CUDA(launch_pdl(combine_add_rmsnorm_kernel, dim3((unsigned)tokens), dim3(kCnThreads), 0,
                           as_stream(stream), static_cast<const __nv_bfloat16*>(out_sorted),
                           inv_pos, topk_index, expert_rank, num_experts, top_k, hidden_size,
                           reduce, static_cast<const __nv_bfloat16*>(residual_in),
                           static_cast<__nv_bfloat16*>(residual_out),
                           static_cast<const __nv_bfloat16*>(norm_weight), eps,
                           static_cast<__nv_bfloat16*>(out)));
  return SF_OK;
}
