// Device code shared by the two expert-parallel exchanges: the NCCL path
// (ep.cu: rows staged locally, all-to-all by NCCL) and the peer-memory path
// (ep_peer.cu: rows pushed straight into every destination's receive region
// over NVLink).  Included by one translation unit each; everything here has
// internal linkage.
#pragma once

#include "common.cuh"

namespace sf {
namespace {

constexpr int kMaxWorld = 8;
constexpr int kMaxK = 16;
constexpr int kPlanThreads = 1024;

int64_t row_bytes_of(int es, int H, int K) {
  const int64_t raw = (int64_t)H * es + 8LL * K;
  return (raw + 15) / 16 * 16;
}

// One thread per token (chunks of 1024 tokens).  A token's routes are sorted
// by expert id in registers (odd-even transposition network over N >= K
// slots, padded with INT_MAX); since the owner rank (id / per) grows with the
// id, the routes on rank r form one contiguous run [beg[r], beg[r+1]) of the
// sorted list.  Per chunk, every rank's (pairs, routes) prefix over the
// tokens comes from one warp scan of packed counts per rank plus a scan of
// the 32 warp totals by warp r: two block barriers per chunk for any world.
template <int N>
struct TokenRoutes {
  int id[N];
  float w[N];
  int k[N];
};

template <int N, typename W>
__device__ __forceinline__ void load_sorted(const int64_t* __restrict__ idx,
                                            const W* __restrict__ topk_w, int64_t t, int K, int E,
                                            bool with_weights, TokenRoutes<N>& r, bool& bad) {
#pragma unroll
  for (int k = 0; k < N; ++k) {
    int e = 0x7fffffff;
    float w = 0.f;
    if (k < K) {
      const int64_t v = idx[t * K + k];
      if (v >= 0 && v < E) {
        e = (int)v;
        if (with_weights) w = to_f32(topk_w[t * K + k]);
      } else {
        bad = true;
      }
    }
    r.id[k] = e;
    r.k[k] = k;
    r.w[k] = w;
  }
#pragma unroll
  for (int pass = 0; pass < N; ++pass) {
#pragma unroll
    for (int j = pass & 1; j + 1 < N; j += 2) {
      if (r.id[j] > r.id[j + 1]) {
        const int ti = r.id[j], tk = r.k[j];
        const float tw = r.w[j];
        r.id[j] = r.id[j + 1];
        r.k[j] = r.k[j + 1];
        r.w[j] = r.w[j + 1];
        r.id[j + 1] = ti;
        r.k[j + 1] = tk;
        r.w[j + 1] = tw;
      }
    }
  }
}

// beg[d] = number of sorted routes on ranks < d (valid ids only).
template <int N>
__device__ __forceinline__ void rank_starts(const TokenRoutes<N>& r, int per, int world,
                                            int (&beg)[kMaxWorld + 1]) {
#pragma unroll
  for (int d = 0; d <= kMaxWorld; ++d) {
    const int lim = d < world ? d * per : world * per;
    int c = 0;
#pragma unroll
    for (int j = 0; j < N; ++j) c += r.id[j] < lim;
    beg[d] = c;
  }
}

template <typename W, int N>
__global__ void __launch_bounds__(kPlanThreads)
ep_plan_kernel(const int64_t* __restrict__ idx, const W* __restrict__ topk_w, int T, int K, int E,
               int world, int route_stride, uint8_t* __restrict__ send, int64_t row_bytes,
               int64_t meta_off, int64_t* __restrict__ send_counts,
               int32_t* __restrict__ route_row, int32_t* __restrict__ pair_token,
               int32_t* __restrict__ error_flag) {
  __shared__ int tot_pairs[kMaxWorld], tot_routes[kMaxWorld];
  __shared__ int pair_base[kMaxWorld], route_base[kMaxWorld];
  __shared__ int wsum[32][kMaxWorld];  // per-warp packed totals of one chunk
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int per = E / world;
  if (threadIdx.x < kMaxWorld) {
    tot_pairs[threadIdx.x] = 0;
    tot_routes[threadIdx.x] = 0;
  }
  __syncthreads();

  // Pass A: totals per destination rank.
  bool bad = false;
  for (int t0 = 0; t0 < T; t0 += kPlanThreads) {
    const int t = t0 + threadIdx.x;
    TokenRoutes<N> r;
    if (t < T) {
      load_sorted<N>(idx, topk_w, t, K, E, false, r, bad);
    } else {
#pragma unroll
      for (int j = 0; j < N; ++j) r.id[j] = 0x7fffffff;
    }
    int beg[kMaxWorld + 1];
    rank_starts<N>(r, per, world, beg);
#pragma unroll
    for (int d = 0; d < kMaxWorld; ++d) {
      if (d >= world) break;
      const int c = beg[d + 1] - beg[d];
      int pc = c > 0, rc = c;
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        pc += __shfl_xor_sync(0xffffffffu, pc, o);
        rc += __shfl_xor_sync(0xffffffffu, rc, o);
      }
      if (lane == 0 && (pc | rc)) {
        atomicAdd(&tot_pairs[d], pc);
        atomicAdd(&tot_routes[d], rc);
      }
    }
  }
  if (bad) *error_flag = 1;
  __syncthreads();
  if (threadIdx.x == 0) {
    int p = 0, q = 0;
    for (int d = 0; d < world; ++d) {
      pair_base[d] = p;
      route_base[d] = route_stride > 0 ? d * route_stride : q;
      send_counts[2 * d] = tot_pairs[d];
      send_counts[2 * d + 1] = tot_routes[d];
      p += tot_pairs[d];
      q += tot_routes[d];
    }
  }
  __syncthreads();

  // Pass B: pair rows, metadata and route rows.
  for (int t0 = 0; t0 < T; t0 += kPlanThreads) {
    const int t = t0 + threadIdx.x;
    TokenRoutes<N> r;
    bool bad2 = false;
    if (t < T) {
      load_sorted<N>(idx, topk_w, t, K, E, true, r, bad2);
#pragma unroll
      for (int j = 0; j < N; ++j)  // invalid routes return nothing
        if (j < K && r.id[j] == 0x7fffffff) route_row[(int64_t)t * K + r.k[j]] = -1;
    } else {
#pragma unroll
      for (int j = 0; j < N; ++j) r.id[j] = 0x7fffffff;
    }
    int beg[kMaxWorld + 1];
    rank_starts<N>(r, per, world, beg);
    int incl[kMaxWorld], own[kMaxWorld];
#pragma unroll
    for (int d = 0; d < kMaxWorld; ++d) {
      if (d >= world) break;
      const int c = beg[d + 1] - beg[d];
      own[d] = (c > 0 ? 1 << 16 : 0) | c;
      int v = own[d];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int x = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += x;
      }
      incl[d] = v;
      if (lane == 31) wsum[warp][d] = v;
    }
    __syncthreads();
    if (warp < world) {  // warp d scans the 32 warp totals of rank d
      const int d = warp;
      const int v = wsum[lane][d];
      int x = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      wsum[lane][d] = x - v;  // exclusive over warps
      if (lane == 31) {       // this chunk's totals
        tot_pairs[d] = x >> 16;
        tot_routes[d] = x & 0xffff;
      }
    }
    __syncthreads();
    if (t < T) {
#pragma unroll
      for (int d = 0; d < kMaxWorld; ++d) {
        if (d >= world) break;
        const int c = own[d] & 0xffff;
        if (c == 0) continue;
        const int ex = wsum[warp][d] + incl[d] - own[d];
        const int pair = pair_base[d] + (ex >> 16);
        const int rb = route_base[d] + (ex & 0xffff);
        pair_token[pair] = t;
        uint8_t* meta = send + (int64_t)pair * row_bytes + meta_off;
        int32_t* mid = reinterpret_cast<int32_t*>(meta);
        float* mw = reinterpret_cast<float*>(meta + 4 * K);
        const int b = beg[d];
#pragma unroll
        for (int j = 0; j < N; ++j) {
          if (j >= K) break;
          const bool v = j < c;
          // sorted slot b + j holds the j-th route of this rank (b + j < N when v)
          int sid = 0, sk = 0;
          float sw = 0.f;
#pragma unroll
          for (int i = 0; i < N; ++i)
            if (i == b + j) {
              sid = r.id[i];
              sk = r.k[i];
              sw = r.w[i];
            }
          mid[j] = v ? sid - d * per : -1;
          mw[j] = v ? sw : 0.f;
          if (v) route_row[(int64_t)t * K + sk] = rb + j;
        }
      }
    }
    __syncthreads();
    if (threadIdx.x < world) {
      pair_base[threadIdx.x] += tot_pairs[threadIdx.x];
      route_base[threadIdx.x] += tot_routes[threadIdx.x];
    }
    __syncthreads();
  }
}

template <typename W>
void launch_plan(int K, const int64_t* idx, const W* w, int T, int E, int world, int route_stride,
                 uint8_t* send, int64_t row_bytes, int64_t meta_off, int64_t* send_counts,
                 int32_t* route_row, int32_t* pair_token, int32_t* error_flag, cudaStream_t s) {
  if (K <= 8)
    ep_plan_kernel<W, 8><<<1, kPlanThreads, 0, s>>>(idx, w, T, K, E, world, route_stride, send,
                                                    row_bytes, meta_off, send_counts, route_row,
                                                    pair_token, error_flag);
  else
    ep_plan_kernel<W, 16><<<1, kPlanThreads, 0, s>>>(idx, w, T, K, E, world, route_stride, send,
                                                     row_bytes, meta_off, send_counts, route_row,
                                                     pair_token, error_flag);
}

int elem_size(int dtype) {
  return dtype == SF_DTYPE_BF16 ? 2 : dtype == SF_DTYPE_F32 ? 4 : 0;
}

int copy_grid(int64_t rows) {
  const int64_t need = (rows + 7) / 8;  // 8 warps per CTA
  const int64_t cap = 4LL * num_sms();
  return (int)(need < 1 ? 1 : need < cap ? need : cap);
}


}  // namespace
}  // namespace sf
