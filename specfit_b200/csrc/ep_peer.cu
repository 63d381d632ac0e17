// K7 over peer memory: the expert-parallel exchange without NCCL and without
// any host synchronisation, so a whole verify pass can be one CUDA graph.
//
// Every rank owns one region (cudaMalloc, shared with the other ranks by
// CUDA IPC handles; each rank maps every peer region into its own device
// context) laid out identically:
//   recv_rows  [world][cap_pairs][row_bytes]    rows pushed here by source s at [s]
//   ret_rows   [world][cap_routes][out_bytes]   outputs returned here by destination d at [d]
//   recv_counts [world][2] int32                (pairs, routes) from source s
//   recv_arrive [world] u64                     push CTAs of source s that finished
//   ret_arrive  [world] u64                     return CTAs of destination d that finished
// One layer:
//   sf_ep_peer_send    plan (route rows laid out [d][cap_routes]) + push: rows,
//                      metadata and counts stored into each destination's region,
//                      then every CTA fences (system scope) and adds 1 to
//                      recv_arrive[me] on every rank.
//   sf_ep_peer_recv    wait until recv_arrive[s] reaches epoch * grid for all s,
//                      group the received slots by local expert, gather the rows.
//   (grouped SwiGLU)
//   sf_ep_peer_return  each output row stored into its source's ret_rows[me],
//                      fence, ret_arrive[me] += 1 on every rank.
//   sf_ep_peer_finish  wait for ret_arrive, combine (ascending expert id).
// A region is rewritten only after its reader has provably finished with the
// previous layer: a source pushes layer l+1 after its layer-l combine, which
// waited for every destination's layer-l return, issued after that
// destination had gathered its layer-l rows.
//
// Waits give up after a wall-clock limit (globaltimer), record the site and
// the ranks that did not arrive in `status`, and return, so a missing rank
// turns into an error the host reads instead of a hung GPU.  Counts read from
// peers are clamped to the capacities, so every access stays in bounds.
#include <cuda.h>

#include "dispatch.cuh"
#include "ep.cuh"
#include "swiglu.h"

namespace sf {
namespace {

constexpr int kPeerThreads = 256;

struct PeerLayout {
  int64_t recv_rows, ret_rows, recv_counts, recv_arrive, ret_arrive, total;
};

PeerLayout peer_layout(const sf_ep_peer& d) {
  auto al = [](int64_t x) { return (x + 255) / 256 * 256; };
  PeerLayout L;
  int64_t o = 0;
  L.recv_rows = o;
  o = al(o + (int64_t)d.world * d.cap_pairs * d.row_bytes);
  L.ret_rows = o;
  o = al(o + (int64_t)d.world * d.cap_routes * d.out_row_bytes);
  L.recv_counts = o;
  o = al(o + (int64_t)d.world * 2 * 4);
  L.recv_arrive = o;
  o = al(o + (int64_t)d.world * 8);
  L.ret_arrive = o;
  o = al(o + (int64_t)d.world * 8);
  L.total = o;
  return L;
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void copy16(uint8_t* dst, const uint8_t* src, int64_t bytes, int lane) {
  const int64_t v = bytes >> 4;
  for (int64_t i = lane; i < v; i += 32)
    reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
}

// Every CTA: after its stores, one system-scope fence and +1 on counter[me]
// of every rank's region.
__device__ __forceinline__ void arrive_all(const uint64_t* __restrict__ peers, int world, int me,
                                           int64_t counter_off) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int r = 0; r < world; ++r)
      atomicAdd_system(reinterpret_cast<unsigned long long*>(peers[r] + counter_off) + me, 1ull);
  }
}

__global__ void __launch_bounds__(kPeerThreads)
peer_push_kernel(const uint8_t* __restrict__ hidden, int64_t hbytes,
                 const uint8_t* __restrict__ staging, int64_t row_bytes,
                 const int32_t* __restrict__ pair_token, const int64_t* __restrict__ send_counts,
                 const uint64_t* __restrict__ peers, int world, int me, int64_t cap_pairs,
                 PeerLayout L) {
  __shared__ int poff[kMaxWorld + 1];
  if (threadIdx.x == 0) {
    int o = 0;
    for (int d = 0; d < world; ++d) {
      poff[d] = o;
      o += (int)send_counts[2 * d];
    }
    poff[world] = o;
  }
  if (blockIdx.x == 0 && threadIdx.x < world) {
    const int d = threadIdx.x;
    int32_t* c = reinterpret_cast<int32_t*>(peers[d] + L.recv_counts) + 2 * me;
    c[0] = (int32_t)send_counts[2 * d];
    c[1] = (int32_t)send_counts[2 * d + 1];
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (kPeerThreads / 32);
  const int P = poff[world];
  for (int64_t i = (int64_t)blockIdx.x * (kPeerThreads / 32) + (threadIdx.x >> 5); i < P;
       i += warps) {
    int d = 0;
    while (d + 1 < world && i >= poff[d + 1]) ++d;
    const int64_t j = i - poff[d];
    if (j >= cap_pairs) continue;
    uint8_t* dst = reinterpret_cast<uint8_t*>(peers[d]) + L.recv_rows +
                   ((int64_t)me * cap_pairs + j) * row_bytes;
    copy16(dst, hidden + (int64_t)pair_token[i] * hbytes, hbytes, lane);
    copy16(dst + hbytes, staging + i * row_bytes + hbytes, row_bytes - hbytes, lane);
  }
  arrive_all(peers, world, me, L.recv_arrive);
}

// One warp: lane r waits until counter[r] >= (epoch + 1) * per_epoch.
__global__ void peer_wait_kernel(const unsigned long long* __restrict__ counter, int world,
                                 unsigned long long* __restrict__ epoch,
                                 unsigned long long per_epoch, int32_t* __restrict__ status,
                                 int site, uint64_t limit_ns) {
  const int lane = threadIdx.x;
  const unsigned long long target = (*epoch + 1) * per_epoch;
  bool ok = true;
  if (lane < world) {
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_sys(counter + lane) < target) {
      if (globaltimer_ns() - t0 > limit_ns) {
        ok = false;
        break;
      }
      __nanosleep(64);
    }
  }
  const unsigned missing = __ballot_sync(0xffffffffu, !ok);
  __syncwarp();
  if (lane == 0) {
    if (missing) {
      atomicCAS(status, 0, site);
      atomicOr(status + 1, (int)missing);
    }
    *epoch += 1;
  }
}

// Received slot p = pair * K + slot over the sources' blocks in rank order.
struct PeerRecvIds {
  static constexpr bool kResetError = false;  // the caller zeroes *error_flag
  __device__ __forceinline__ void on_done(int) const {}
  const uint8_t* rows;
  const int32_t* counts;
  int64_t cap, row_bytes, meta_off;
  int world, K;
  __device__ __forceinline__ int pairs_of(int s) const {
    const int c = counts[2 * s];
    return c < 0 ? 0 : (c > cap ? (int)cap : c);
  }
  __device__ __forceinline__ int size() const {
    int n = 0;
    for (int s = 0; s < world; ++s) n += pairs_of(s);
    return n * K;
  }
  __device__ __forceinline__ const uint8_t* row(int pair) const {
    int s = 0;
    for (; s + 1 < world; ++s) {
      const int c = pairs_of(s);
      if (pair < c) break;
      pair -= c;
    }
    return rows + ((int64_t)s * cap + pair) * row_bytes;
  }
  __device__ __forceinline__ int operator()(int p) const {
    const int pair = p / K;
    return reinterpret_cast<const int32_t*>(row(pair) + meta_off)[p - pair * K];
  }
};

__global__ void __launch_bounds__(kPeerThreads)
peer_gather_kernel(PeerRecvIds src, const int32_t* __restrict__ sorted_pos,
                   const int32_t* __restrict__ n_rows, int64_t cap_rows,
                   uint8_t* __restrict__ hidden_sorted, int64_t hbytes,
                   float* __restrict__ w_sorted) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (kPeerThreads / 32);
  int64_t n = *n_rows;
  if (n > cap_rows) n = cap_rows;
  for (int64_t i = (int64_t)blockIdx.x * (kPeerThreads / 32) + (threadIdx.x >> 5); i < n;
       i += warps) {
    const int p = sorted_pos[i];
    if (p < 0) continue;
    const int pair = p / src.K;
    const uint8_t* row = src.row(pair);
    copy16(hidden_sorted + i * hbytes, row, hbytes, lane);
    if (lane == 0) w_sorted[i] = reinterpret_cast<const float*>(row + src.meta_off + 4 * src.K)[p - pair * src.K];
  }
}

__global__ void __launch_bounds__(kPeerThreads)
peer_return_kernel(const uint8_t* __restrict__ out_sorted, int64_t out_bytes,
                   const int32_t* __restrict__ return_src, const int32_t* __restrict__ n_routes,
                   const int32_t* __restrict__ counts, const uint64_t* __restrict__ peers,
                   int world, int me, int64_t cap_pairs, int64_t cap_routes, int K, PeerLayout L) {
  __shared__ int roff[kMaxWorld + 1];
  if (threadIdx.x == 0) {
    int o = 0;
    for (int s = 0; s < world; ++s) {
      roff[s] = o;
      int p = counts[2 * s], r = counts[2 * s + 1];
      p = p < 0 ? 0 : (p > cap_pairs ? (int)cap_pairs : p);
      const int64_t rmax = (int64_t)p * K < cap_routes ? (int64_t)p * K : cap_routes;
      r = r < 0 ? 0 : (r > rmax ? (int)rmax : r);
      o += r;
    }
    roff[world] = o;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (kPeerThreads / 32);
  const int R = min(*n_routes, roff[world]);
  for (int64_t q = (int64_t)blockIdx.x * (kPeerThreads / 32) + (threadIdx.x >> 5); q < R;
       q += warps) {
    int s = 0;
    while (s + 1 < world && q >= roff[s + 1]) ++s;
    const int64_t j = q - roff[s];
    uint8_t* dst = reinterpret_cast<uint8_t*>(peers[s]) + L.ret_rows +
                   ((int64_t)me * cap_routes + j) * out_bytes;
    copy16(dst, out_sorted + (int64_t)return_src[q] * out_bytes, out_bytes, lane);
  }
  arrive_all(peers, world, me, L.ret_arrive);
}

// The return destination of every sorted row (the fused return): row
// return_src[q] of route q from source s, j-th of that source, goes to
// peers[s] + ret_rows + (me * cap_routes + j) * out_bytes; other rows get 0.
// One CTA: the table is cleared, then filled.
__global__ void __launch_bounds__(1024)
peer_return_plan_kernel(const int32_t* __restrict__ return_src, const int32_t* __restrict__ n_routes,
                        const int32_t* __restrict__ counts, const uint64_t* __restrict__ peers, int world,
                        int me, int64_t cap_pairs, int64_t cap_routes, int K, int64_t out_bytes,
                        int64_t cap_rows, PeerLayout L, uint64_t* __restrict__ dst_row) {
  pdl_wait();
  pdl_trigger();
  __shared__ int roff[kMaxWorld + 1];
  if (threadIdx.x == 0) {
    int o = 0;
    for (int s = 0; s < world; ++s) {
      roff[s] = o;
      int p = counts[2 * s], r = counts[2 * s + 1];
      p = p < 0 ? 0 : (p > cap_pairs ? (int)cap_pairs : p);
      const int64_t rmax = (int64_t)p * K < cap_routes ? (int64_t)p * K : cap_routes;
      r = r < 0 ? 0 : (r > rmax ? (int)rmax : r);
      o += r;
    }
    roff[world] = o;
  }
  for (int64_t i = threadIdx.x; i < cap_rows; i += blockDim.x) dst_row[i] = 0ull;
  __syncthreads();
  const int R = min(*n_routes, roff[world]);
  for (int q = threadIdx.x; q < R; q += blockDim.x) {
    int s = 0;
    while (s + 1 < world && q >= roff[s + 1]) ++s;
    const int64_t j = q - roff[s];
    const int r = return_src[q];
    if (r >= 0 && r < cap_rows)
      dst_row[r] = peers[s] + (uint64_t)L.ret_rows + (uint64_t)((me * cap_routes + j) * out_bytes);
  }
}

int check_peer(const sf_ep_peer* d) {
  SF_CHECK_ARG(d != nullptr, "null peer descriptor");
  const int es = elem_size(d->dtype);
  SF_CHECK_ARG(es != 0, "unsupported dtype %d", d->dtype);
  SF_CHECK_ARG(d->world >= 1 && d->world <= kMaxWorld, "world must be in [1, %d]", kMaxWorld);
  SF_CHECK_ARG(d->rank >= 0 && d->rank < d->world, "rank out of range");
  SF_CHECK_ARG(d->top_k > 0 && d->top_k <= kMaxK, "top_k must be in [1, %d]", kMaxK);
  SF_CHECK_ARG(d->local_experts > 0 && d->local_experts <= grouping::kThreads,
               "local_experts must be in [1, 1024]");
  SF_CHECK_ARG(d->cap_pairs > 0 && d->cap_routes >= d->cap_pairs &&
               (int64_t)d->world * d->cap_routes < (1LL << 30),
               "invalid capacities");
  SF_CHECK_ARG(d->row_bytes == row_bytes_of(es, d->hidden_size, d->top_k),
               "row_bytes must equal sf_ep_row_bytes()");
  SF_CHECK_ARG(d->out_row_bytes == (int64_t)d->hidden_size * es && d->out_row_bytes % 16 == 0,
               "out_row_bytes must be hidden_size * element size, a multiple of 16");
  SF_CHECK_ARG(d->grid > 0 && d->grid <= 4096, "grid must be in [1, 4096]");
  SF_CHECK_ARG(d->peers && d->local && d->epochs && d->status, "null pointer in peer descriptor");
  SF_CHECK_ARG(aligned16(d->local), "peer region must be 16-byte aligned");
  return SF_OK;
}

}  // namespace
}  // namespace sf

extern "C" int64_t sf_ep_peer_layout(sf_ep_peer* d) {
  using namespace sf;
  if (!d) return -1;
  const PeerLayout L = peer_layout(*d);
  d->off_recv_rows = L.recv_rows;
  d->off_ret_rows = L.ret_rows;
  d->off_recv_counts = L.recv_counts;
  d->off_recv_arrive = L.recv_arrive;
  d->off_ret_arrive = L.ret_arrive;
  return L.total;
}

extern "C" int sf_ipc_alloc(size_t bytes, void** ptr, void* handle) {
  using namespace sf;
  SF_CHECK_ARG(bytes > 0 && ptr && handle, "invalid arguments");
  void* p = nullptr;
  SF_CHECK_CUDA(cudaMalloc(&p, bytes));
  cudaError_t e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t*>(handle), p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return set_error(SF_ERR_CUDA, "peer region setup failed: %s", cudaGetErrorString(e));
  }
  *ptr = p;
  return SF_OK;
}

extern "C" int sf_ipc_free(void* ptr) {
  using namespace sf;
  if (ptr) SF_CHECK_CUDA(cudaFree(ptr));
  return SF_OK;
}

extern "C" int sf_ipc_open(const void* handle, void** ptr) {
  using namespace sf;
  SF_CHECK_ARG(handle && ptr, "invalid arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  SF_CHECK_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return SF_OK;
}

extern "C" int sf_ipc_close(void* ptr) {
  using namespace sf;
  if (ptr) SF_CHECK_CUDA(cudaIpcCloseMemHandle(ptr));
  return SF_OK;
}

extern "C" int sf_ep_peer_send(const sf_ep_peer* d, const void* hidden, int64_t tokens,
                               const int64_t* topk_index, const void* topk_weights,
                               int weight_dtype, int num_experts, void* staging_rows,
                               int64_t* send_counts, int32_t* route_row, int32_t* pair_token,
                               int32_t* error_flag, void* stream) {
  using namespace sf;
  if (int rc = check_peer(d)) return rc;
  SF_CHECK_ARG(weight_dtype == SF_DTYPE_F32 || weight_dtype == SF_DTYPE_BF16,
               "unsupported weight dtype %d", weight_dtype);
  SF_CHECK_ARG(tokens >= 0 && tokens <= d->cap_pairs, "tokens must be in [0, cap_pairs]");
  SF_CHECK_ARG(tokens * d->top_k <= d->cap_routes, "tokens * top_k must be <= cap_routes");
  SF_CHECK_ARG(num_experts == d->local_experts * d->world, "num_experts must be local_experts * world");
  SF_CHECK_ARG(send_counts && error_flag, "null pointer argument");
  SF_CHECK_ARG(tokens == 0 || (hidden && topk_index && topk_weights && staging_rows && route_row &&
                               pair_token), "null pointer argument");
  SF_CHECK_ARG(tokens == 0 || (aligned16(hidden) && aligned16(staging_rows)),
               "hidden and staging_rows must be 16-byte aligned");
  cudaStream_t s = as_stream(stream);
  const int64_t hbytes = d->out_row_bytes;
  uint8_t* staging = static_cast<uint8_t*>(staging_rows);
  if (weight_dtype == SF_DTYPE_F32)
    launch_plan(d->top_k, topk_index, static_cast<const float*>(topk_weights), (int)tokens,
                num_experts, d->world, (int)d->cap_routes, staging, d->row_bytes, hbytes,
                send_counts, route_row, pair_token, error_flag, s);
  else
    launch_plan(d->top_k, topk_index, static_cast<const __nv_bfloat16*>(topk_weights), (int)tokens,
                num_experts, d->world, (int)d->cap_routes, staging, d->row_bytes, hbytes,
                send_counts, route_row, pair_token, error_flag, s);
  SF_CHECK_LAUNCH();
  const PeerLayout L = peer_layout(*d);
  peer_push_kernel<<<d->grid, kPeerThreads, 0, s>>>(
      static_cast<const uint8_t*>(hidden), hbytes, staging, d->row_bytes, pair_token, send_counts,
      d->peers, d->world, d->rank, d->cap_pairs, L);
  SF_CHECK_LAUNCH();
  return SF_OK;
}

extern "C" int sf_ep_peer_recv(const sf_ep_peer* d, int32_t* counts, int32_t* offsets,
                               int32_t* sorted_pos, int32_t* inv_pos, int32_t* active,
                               int32_t* num_active, int32_t* return_src, int32_t* error_flag,
                               void* hidden_sorted, float* weights_sorted, void* stream) {
  using namespace sf;
  if (int rc = check_peer(d)) return rc;
  SF_CHECK_ARG(counts && offsets && sorted_pos && inv_pos && active && num_active && return_src &&
               error_flag && hidden_sorted && weights_sorted, "null pointer argument");
  SF_CHECK_ARG(aligned16(hidden_sorted), "hidden_sorted must be 16-byte aligned");
  cudaStream_t s = as_stream(stream);
  const PeerLayout L = peer_layout(*d);
  const uint8_t* base = static_cast<const uint8_t*>(d->local);
  peer_wait_kernel<<<1, 32, 0, s>>>(
      reinterpret_cast<const unsigned long long*>(base + L.recv_arrive), d->world,
      reinterpret_cast<unsigned long long*>(d->epochs), (unsigned long long)d->grid, d->status, 1,
      (uint64_t)d->wait_limit_ms * 1000000ull);
  SF_CHECK_LAUNCH();
  PeerRecvIds src{base + L.recv_rows, reinterpret_cast<const int32_t*>(base + L.recv_counts),
                  d->cap_pairs, d->row_bytes, d->out_row_bytes, d->world, d->top_k};
  const size_t smem = grouping::smem_bytes(d->local_experts);
  auto kernel = grouping::group_kernel<PeerRecvIds>;
  if (smem > 48 * 1024)
    SF_CHECK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem));
  kernel<<<1, grouping::kThreads, smem, s>>>(src, -1, d->local_experts, true, counts, offsets,
                                             sorted_pos, inv_pos, active, num_active, error_flag,
                                             return_src);
  SF_CHECK_LAUNCH();
  const int64_t cap_rows = (int64_t)d->world * d->cap_routes;
  peer_gather_kernel<<<d->grid, kPeerThreads, 0, s>>>(
      src, sorted_pos, offsets + d->local_experts, cap_rows, static_cast<uint8_t*>(hidden_sorted),
      d->out_row_bytes, weights_sorted);
  SF_CHECK_LAUNCH();
  return SF_OK;
}

extern "C" int sf_ep_peer_return(const sf_ep_peer* d, const void* out_sorted,
                                 const int32_t* return_src, const int32_t* offsets, void* stream) {
  using namespace sf;
  if (int rc = check_peer(d)) return rc;
  SF_CHECK_ARG(out_sorted && return_src && offsets, "null pointer argument");
  SF_CHECK_ARG(aligned16(out_sorted), "out_sorted must be 16-byte aligned");
  const PeerLayout L = peer_layout(*d);
  const uint8_t* base = static_cast<const uint8_t*>(d->local);
  peer_return_kernel<<<d->grid, kPeerThreads, 0, as_stream(stream)>>>(
      static_cast<const uint8_t*>(out_sorted), d->out_row_bytes, return_src,
      offsets + d->local_experts, reinterpret_cast<const int32_t*>(base + L.recv_counts), d->peers,
      d->world, d->rank, d->cap_pairs, d->cap_routes, d->top_k, L);
  SF_CHECK_LAUNCH();
  return SF_OK;
}

extern "C" int sf_ep_peer_return_plan(const sf_ep_peer* d, const int32_t* return_src, const int32_t* offsets,
                                      uint64_t* dst_row, void* stream) {
  using namespace sf;
  if (int rc = check_peer(d)) return rc;
  SF_CHECK_ARG(return_src && offsets && dst_row, "null pointer argument");
  const PeerLayout L = peer_layout(*d);
  const uint8_t* base = static_cast<const uint8_t*>(d->local);
  SF_CHECK_CUDA(launch_pdl(peer_return_plan_kernel, dim3(1), dim3(1024), 0, as_stream(stream), return_src,
                           offsets + d->local_experts, reinterpret_cast<const int32_t*>(base + L.recv_counts),
                           d->peers, d->world, d->rank, d->cap_pairs, d->cap_routes, d->top_k,
                           d->out_row_bytes, (int64_t)d->world * d->cap_routes, L, dst_row));
  SF_CHECK_LAUNCH();
  return SF_OK;
}

extern "C" int sf_grouped_swiglu_peer(const sf_ep_peer* d, const void* hidden_sorted, const float* weights_sorted,
                                      const int32_t* offsets, const int32_t* active, const int32_t* num_active,
                                      const int32_t* expert_slot, const void* slot_storage, int64_t slot_count,
                                      int64_t slot_stride_elems, int intermediate_size, void* act_workspace,
                                      const uint64_t* dst_row, uint32_t* ticket, void* stream) {
  using namespace sf;
  if (int rc = check_peer(d)) return rc;
  SF_CHECK_ARG(d->dtype == SF_DTYPE_BF16, "the fused return needs bf16 rows");
  SF_CHECK_ARG(hidden_sorted && weights_sorted && offsets && active && num_active && expert_slot &&
                   slot_storage && act_workspace && dst_row && ticket,
               "null pointer argument");
  SF_CHECK_ARG(intermediate_size > 0 && slot_count > 0 &&
                   slot_stride_elems >= 3LL * d->hidden_size * intermediate_size,
               "slot_stride_elems must cover one packed expert");
  const PeerLayout L = peer_layout(*d);
  SwigluArgs a{hidden_sorted, weights_sorted, SF_DTYPE_BF16, offsets, active, num_active, expert_slot,
               slot_storage, slot_count, slot_stride_elems, d->local_experts, d->hidden_size,
               intermediate_size, (int64_t)d->world * d->cap_routes, act_workspace, act_workspace};
  SwigluPeerOut peer{dst_row, ticket, d->peers, L.ret_arrive, d->world, d->rank, (unsigned long long)d->grid};
  return swiglu_tcgen05_peer(a, peer, as_stream(stream));
}

extern "C" int sf_ep_peer_finish(const sf_ep_peer* d, const int64_t* topk_index,
                                 const int32_t* route_row, int64_t tokens, int num_experts,
                                 int reduce, void* out, void* stream) {
  using namespace sf;
  if (int rc = check_peer(d)) return rc;
  SF_CHECK_ARG(tokens >= 0 && tokens <= d->cap_pairs, "tokens must be in [0, cap_pairs]");
  const PeerLayout L = peer_layout(*d);
  const uint8_t* base = static_cast<const uint8_t*>(d->local);
  cudaStream_t s = as_stream(stream);
  peer_wait_kernel<<<1, 32, 0, s>>>(
      reinterpret_cast<const unsigned long long*>(base + L.ret_arrive), d->world,
      reinterpret_cast<unsigned long long*>(d->epochs) + 1, (unsigned long long)d->grid,
      d->status, 2, (uint64_t)d->wait_limit_ms * 1000000ull);
  SF_CHECK_LAUNCH();
  if (tokens == 0) return SF_OK;
  return sf_moe_combine(base + L.ret_rows, d->dtype, route_row, topk_index, nullptr, num_experts,
                        tokens, d->top_k, d->hidden_size, reduce, out, stream);
}
