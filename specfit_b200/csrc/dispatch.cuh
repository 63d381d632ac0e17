// Stable grouping of routes by expert, shared by the single-GPU dispatch
// (dispatch.cu) and the receiving side of expert parallelism (ep.cu).
//
// One CTA of 1024 threads (32 warps).  The n route positions are cut into 32
// contiguous segments, one per warp.  Pass 1 counts each segment's routes
// per expert; a per-expert prefix over the segments plus the per-expert
// offsets gives every warp its write cursor; pass 2 walks each segment in
// 32-route chunks in order, ranking equal ids within a chunk with
// __match_any_sync, so the scatter is stable and deterministic.
//
// The expert id of position p comes from `src(p)`; when n < 0 the number of
// positions is `src.size()`, read on the device.  An id of -1 is a padding
// slot when `pad_ok` (skipped silently); any other id outside [0, E) sets
// *error_flag and is skipped (with Src::kResetError the kernel first zeroes
// the flag).  When `compact` is non-null it receives, for
// the q-th valid position in increasing position order, that route's sorted
// row: compact[q] = inv_pos[p].
#pragma once

#include "common.cuh"

namespace sf {
namespace grouping {

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

inline size_t smem_bytes(int E) { return (size_t)(kSegs + 1) * E * sizeof(int); }

template <typename Src>
__global__ void __launch_bounds__(kThreads)
group_kernel(Src src, int n, int E, bool pad_ok, int32_t* __restrict__ counts,
             int32_t* __restrict__ offsets, int32_t* __restrict__ sorted_pos,
             int32_t* __restrict__ inv_pos, int32_t* __restrict__ active,
             int32_t* __restrict__ num_active, int32_t* __restrict__ error_flag,
             int32_t* __restrict__ compact) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ int smem[];
  int* seg_cnt = smem;                  // [kSegs][E]
  int* off = seg_cnt + kSegs * E;       // [E]
  __shared__ int warp_sums[32];
  __shared__ int seg_valid[kSegs];
  __shared__ int total_routes, total_active;

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  if (n < 0) n = src.size();
  const int seg_len = (n + kSegs - 1) / kSegs;
  const int seg_lo = min(n, warp * seg_len);
  const int seg_hi = min(n, seg_lo + seg_len);

  for (int i = threadIdx.x; i < kSegs * E; i += kThreads) seg_cnt[i] = 0;
  if (Src::kResetError && threadIdx.x == 0) *error_flag = 0;  // before any thread can set it
  __syncthreads();

  // Pass 1: per-segment counts.
  int my_valid = 0;
  for (int p = seg_lo + lane; p < seg_hi; p += 32) {
    const int e = src(p);
    if (e >= 0 && e < E) {
      atomicAdd(&seg_cnt[warp * E + e], 1);
      ++my_valid;
    } else if (!(pad_ok && e == -1)) {
      *error_flag = 1;
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) my_valid += __shfl_xor_sync(0xffffffffu, my_valid, o);
  if (lane == 0) seg_valid[warp] = my_valid;
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
  // Exclusive prefix of the valid routes over the segments (warp 0).
  if (warp == 0) {
    const int v = seg_valid[lane];
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int x = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += x;
    }
    seg_valid[lane] = incl - v;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    offsets[E] = total_routes;
    *num_active = total_active;
    src.on_done(total_active);
  }
  for (int i = total_active + threadIdx.x; i < E; i += kThreads) active[i] = -1;
  for (int i = total_routes + threadIdx.x; i < n; i += kThreads) sorted_pos[i] = -1;

  // Pass 2: stable scatter, one segment per warp, 32 routes at a time.
  const unsigned lt_mask = (1u << lane) - 1u;
  int compact_cursor = seg_valid[warp];
  for (int c0 = seg_lo; c0 < seg_hi; c0 += 32) {
    const int p = c0 + lane;
    int key = E + lane;  // unique non-matching key for idle / invalid lanes
    bool valid = false;
    if (p < seg_hi) {
      const int ev = src(p);
      if (ev >= 0 && ev < E) {
        key = ev;
        valid = true;
      } else {
        inv_pos[p] = -1;
      }
    }
    const unsigned peers = __match_any_sync(0xffffffffu, key);
    const unsigned valid_mask = __ballot_sync(0xffffffffu, valid);
    int dst = 0;
    if (valid) dst = off[key] + seg_cnt[warp * E + key] + __popc(peers & lt_mask);
    __syncwarp();
    if (valid) {
      sorted_pos[dst] = p;
      inv_pos[p] = dst;
      if (compact) compact[compact_cursor + __popc(valid_mask & lt_mask)] = dst;
      if ((peers & lt_mask) == 0) seg_cnt[warp * E + key] += __popc(peers);
    }
    compact_cursor += __popc(valid_mask);
    __syncwarp();
  }
}

}  // namespace grouping
}  // namespace sf
