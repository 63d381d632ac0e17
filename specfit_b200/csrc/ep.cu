// K7: expert-parallel dispatch and return of the MoE block (new; the
// reference runs on one GPU).
//
// Rank r of `world` owns experts [r*E/world, (r+1)*E/world).  Each token is
// sent at most once to each rank it has routes on (one "pair" = token x
// destination), as one row:
//   [ hidden (H elements of the model dtype) | int32 ids[K] | float w[K] | pad ]
// ids are the pair's routes' LOCAL expert ids on the destination in
// ascending order, -1 padded; w their routing weights (fp32), 0 padded.
// Rows are grouped by destination rank and, within one, by token.
//
// The destination groups the received routes by local expert with the same
// stable grouping as the single-GPU dispatch (sources in rank order, tokens
// in order), runs the grouped SwiGLU and returns one weighted output row per
// route, in received (pair, slot) order.  The source then knows where each
// of its routes' outputs lands (route_row) and reduces them with the single-
// GPU combine, so the layer's result is the one-GPU result bit for bit.
#include "dispatch.cuh"
#include "ep.cuh"

namespace sf {
namespace {

// dst row i <- src row index(i) (H bytes each, 16-byte vectors; one warp per
// row).  Rows whose index is negative are zero-filled.  When `total` is
// non-null the row count is the sum of its even entries (pairs per rank).
__global__ void copy_rows_kernel(const uint8_t* __restrict__ src, int64_t src_pitch,
                                 const int32_t* __restrict__ index, uint8_t* __restrict__ dst,
                                 int64_t dst_pitch, int64_t bytes, int64_t rows,
                                 const int64_t* __restrict__ total, int world) {
  int64_t n = rows;
  if (total) {
    n = 0;
    for (int d = 0; d < world; ++d) n += total[2 * d];
  }
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t vecs = bytes >> 4;
  for (int64_t i = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < n; i += warps) {
    const int32_t s = index[i];
    uint4* d = reinterpret_cast<uint4*>(dst + i * dst_pitch);
    if (s < 0) {
      for (int64_t v = lane; v < vecs; v += 32) d[v] = make_uint4(0, 0, 0, 0);
      continue;
    }
    const uint4* a = reinterpret_cast<const uint4*>(src + (int64_t)s * src_pitch);
    for (int64_t v = lane; v < vecs; v += 32) d[v] = a[v];
  }
}

// Expert id of received route position p = pair * K + slot.
struct RecvIds {
  static constexpr bool kResetError = false;  // the caller zeroes *error_flag
  __device__ __forceinline__ void on_done(int) const {}
  const uint8_t* rows;
  int64_t row_bytes, meta_off;
  int K;
  __device__ __forceinline__ int size() const { return 0; }  // sizes are passed explicitly
  __device__ __forceinline__ int operator()(int p) const {
    const int pair = p / K;
    return reinterpret_cast<const int32_t*>(rows + (int64_t)pair * row_bytes + meta_off)[p - pair * K];
  }
};

// Sorted row i of the destination: the hidden row of pair sorted_pos[i] / K
// and the weight of slot sorted_pos[i] % K.  One warp per row.
__global__ void recv_gather_kernel(const uint8_t* __restrict__ rows, int64_t row_bytes,
                                   int64_t meta_off, int K, const int32_t* __restrict__ sorted_pos,
                                   int64_t n, uint8_t* __restrict__ hidden_sorted, int64_t bytes,
                                   float* __restrict__ w_sorted) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t vecs = bytes >> 4;
  for (int64_t i = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < n; i += warps) {
    const int32_t p = sorted_pos[i];
    uint4* d = reinterpret_cast<uint4*>(hidden_sorted + i * bytes);
    if (p < 0) {
      for (int64_t v = lane; v < vecs; v += 32) d[v] = make_uint4(0, 0, 0, 0);
      if (lane == 0) w_sorted[i] = 0.f;
      continue;
    }
    const int pair = p / K;
    const uint8_t* row = rows + (int64_t)pair * row_bytes;
    const uint4* a = reinterpret_cast<const uint4*>(row);
    for (int64_t v = lane; v < vecs; v += 32) d[v] = a[v];
    if (lane == 0) w_sorted[i] = reinterpret_cast<const float*>(row + meta_off + 4 * K)[p - pair * K];
  }
}

}  // namespace
}  // namespace sf

extern "C" int64_t sf_ep_row_bytes(int dtype, int hidden_size, int top_k) {
  const int es = sf::elem_size(dtype);
  if (es == 0 || hidden_size <= 0 || top_k <= 0) return -1;
  return sf::row_bytes_of(es, hidden_size, top_k);
}

extern "C" int sf_ep_send_pack(const void* hidden, int dtype, int64_t tokens, int hidden_size,
                               const int64_t* topk_index, const void* topk_weights,
                               int weight_dtype, int top_k, int num_experts, int world,
                               void* send_rows, int64_t row_bytes, int64_t* send_counts,
                               int32_t* route_row, int32_t* pair_token, int32_t* error_flag,
                               void* stream) {
  using namespace sf;
  const int es = elem_size(dtype);
  SF_CHECK_ARG(es != 0, "unsupported dtype %d", dtype);
  SF_CHECK_ARG(weight_dtype == SF_DTYPE_F32 || weight_dtype == SF_DTYPE_BF16,
               "unsupported weight dtype %d", weight_dtype);
  SF_CHECK_ARG(tokens >= 0 && tokens <= (1 << 24), "tokens must be in [0, 2^24]");
  SF_CHECK_ARG(top_k > 0 && top_k <= kMaxK, "top_k must be in [1, %d]", kMaxK);
  SF_CHECK_ARG(world >= 1 && world <= kMaxWorld, "world must be in [1, %d]", kMaxWorld);
  SF_CHECK_ARG(num_experts > 0 && num_experts % world == 0,
               "num_experts must be a positive multiple of world");
  SF_CHECK_ARG(((int64_t)hidden_size * es) % 16 == 0, "hidden row must be a multiple of 16 bytes");
  SF_CHECK_ARG(row_bytes == row_bytes_of(es, hidden_size, top_k),
               "row_bytes must equal sf_ep_row_bytes()");
  SF_CHECK_ARG(send_counts && error_flag, "null pointer argument");
  SF_CHECK_ARG(tokens == 0 || (hidden && topk_index && topk_weights && send_rows && route_row &&
                               pair_token), "null pointer argument");
  SF_CHECK_ARG(tokens == 0 || (aligned16(hidden) && aligned16(send_rows)),
               "hidden and send_rows must be 16-byte aligned");
  cudaStream_t s = as_stream(stream);
  const int64_t meta_off = (int64_t)hidden_size * es;
  uint8_t* rows = static_cast<uint8_t*>(send_rows);
  if (weight_dtype == SF_DTYPE_F32)
    launch_plan(top_k, topk_index, static_cast<const float*>(topk_weights), (int)tokens, num_experts,
                world, 0, rows, row_bytes, meta_off, send_counts, route_row, pair_token, error_flag, s);
  else
    launch_plan(top_k, topk_index, static_cast<const __nv_bfloat16*>(topk_weights), (int)tokens,
                num_experts, world, 0, rows, row_bytes, meta_off, send_counts, route_row,
                pair_token, error_flag, s);
  SF_CHECK_LAUNCH();
  if (tokens == 0) return SF_OK;
  // Hidden rows of the pairs; the pair count is read on the device.
  copy_rows_kernel<<<copy_grid(tokens * world), 256, 0, s>>>(
      static_cast<const uint8_t*>(hidden), meta_off, pair_token, static_cast<uint8_t*>(send_rows),
      row_bytes, meta_off, tokens * world, send_counts, world);
  SF_CHECK_LAUNCH();
  return SF_OK;
}

extern "C" int sf_ep_recv_group(const void* recv_rows, int64_t row_bytes, int dtype, int64_t pairs,
                                int hidden_size, int top_k, int local_experts, int32_t* counts,
                                int32_t* offsets, int32_t* sorted_pos, int32_t* inv_pos,
                                int32_t* active, int32_t* num_active, int32_t* return_src,
                                int32_t* error_flag, void* stream) {
  using namespace sf;
  const int es = elem_size(dtype);
  SF_CHECK_ARG(es != 0, "unsupported dtype %d", dtype);
  SF_CHECK_ARG(top_k > 0 && top_k <= kMaxK, "top_k must be in [1, %d]", kMaxK);
  SF_CHECK_ARG(local_experts > 0 && local_experts <= grouping::kThreads,
               "local_experts must be in [1, 1024]");
  SF_CHECK_ARG(pairs >= 0 && pairs * top_k < (int64_t)1 << 30, "too many received routes");
  SF_CHECK_ARG(row_bytes == row_bytes_of(es, hidden_size, top_k),
               "row_bytes must equal sf_ep_row_bytes()");
  SF_CHECK_ARG(counts && offsets && active && num_active && error_flag, "null pointer argument");
  SF_CHECK_ARG(pairs == 0 || (recv_rows && sorted_pos && inv_pos && return_src),
               "null pointer argument");
  const size_t smem = grouping::smem_bytes(local_experts);
  auto kernel = grouping::group_kernel<RecvIds>;
  if (smem > 48 * 1024)
    SF_CHECK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem));
  const int64_t meta_off = (int64_t)hidden_size * es;
  kernel<<<1, grouping::kThreads, smem, as_stream(stream)>>>(
      RecvIds{static_cast<const uint8_t*>(recv_rows), row_bytes, meta_off, top_k},
      (int)(pairs * top_k), local_experts, true, counts, offsets, sorted_pos, inv_pos, active,
      num_active, error_flag, return_src);
  SF_CHECK_LAUNCH();
  return SF_OK;
}

extern "C" int sf_ep_recv_gather(const void* recv_rows, int64_t row_bytes, int dtype,
                                 int hidden_size, int top_k, const int32_t* sorted_pos,
                                 int64_t routes, void* hidden_sorted, float* weights_sorted,
                                 void* stream) {
  using namespace sf;
  const int es = elem_size(dtype);
  SF_CHECK_ARG(es != 0, "unsupported dtype %d", dtype);
  SF_CHECK_ARG(top_k > 0 && top_k <= kMaxK, "top_k must be in [1, %d]", kMaxK);
  SF_CHECK_ARG(row_bytes == row_bytes_of(es, hidden_size, top_k),
               "row_bytes must equal sf_ep_row_bytes()");
  SF_CHECK_ARG(routes >= 0, "routes must be >= 0");
  if (routes == 0) return SF_OK;
  SF_CHECK_ARG(recv_rows && sorted_pos && hidden_sorted && weights_sorted, "null pointer argument");
  SF_CHECK_ARG(aligned16(recv_rows) && aligned16(hidden_sorted),
               "recv_rows and hidden_sorted must be 16-byte aligned");
  const int64_t bytes = (int64_t)hidden_size * es;
  recv_gather_kernel<<<copy_grid(routes), 256, 0, as_stream(stream)>>>(
      static_cast<const uint8_t*>(recv_rows), row_bytes, bytes, top_k, sorted_pos, routes,
      static_cast<uint8_t*>(hidden_sorted), bytes, weights_sorted);
  SF_CHECK_LAUNCH();
  return SF_OK;
}

extern "C" int sf_ep_return_pack(const void* out_sorted, int dtype, int hidden_size,
                                 const int32_t* return_src, int64_t routes, void* return_rows,
                                 void* stream) {
  using namespace sf;
  const int es = elem_size(dtype);
  SF_CHECK_ARG(es != 0, "unsupported dtype %d", dtype);
  SF_CHECK_ARG(routes >= 0 && hidden_size > 0, "invalid sizes");
  const int64_t bytes = (int64_t)hidden_size * es;
  SF_CHECK_ARG(bytes % 16 == 0, "hidden row must be a multiple of 16 bytes");
  if (routes == 0) return SF_OK;
  SF_CHECK_ARG(out_sorted && return_src && return_rows, "null pointer argument");
  SF_CHECK_ARG(aligned16(out_sorted) && aligned16(return_rows),
               "out_sorted and return_rows must be 16-byte aligned");
  copy_rows_kernel<<<copy_grid(routes), 256, 0, as_stream(stream)>>>(
      static_cast<const uint8_t*>(out_sorted), bytes, return_src,
      static_cast<uint8_t*>(return_rows), bytes, bytes, routes, nullptr, 0);
  SF_CHECK_LAUNCH();
  return SF_OK;
}
