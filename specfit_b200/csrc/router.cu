// K1: MoE router — logits, fp32 softmax, top-k, renormalisation.
//
// Restates Qwen3MoeTopKRouter.forward (transformers/models/qwen3_moe/
// modeling_qwen3_moe.py:263-272):
//   logits = F.linear(h, W)            -> model dtype
//   probs  = softmax(logits, fp32)
//   top    = topk(probs, k)            -> (values, indices)
//   top   /= top.sum() if norm_topk_prob
//
// Numerics: bf16 logits sum exact bf16*bf16 products in fp32 in one fixed
// order (below) and round once to bf16, like cuBLAS's fp32-accumulate GEMM
// but with an order the oracle replays bit for bit; fp32 logits sum exact
// products in fp64 and round once (the correctly rounded logit).  Top-k runs
// on the logits ordered by (value desc, expert id asc); softmax is monotone,
// so this equals topk(probs) with the tie rule "lower id wins".
//
// Two launches: a logits kernel spread over the GPU (a CTA per 8 tokens x 16
// experts) and a warp-per-token softmax / top-k kernel; for bf16 passes of
// at most 8 tokens and 128 experts, one launch of a CTA cluster that does
// both (router_fused_kernel, same bits).
#include <cooperative_groups.h>
#include <math.h>

#include <mutex>
#include <type_traits>

#include "common.cuh"

namespace sf {
namespace {

constexpr int kTokTile = 8;    // tokens per logits CTA
constexpr int kExpTile = 16;   // experts per logits CTA (2 per warp)
constexpr int kWarps = 8;
constexpr int kNone = 0x7fffffff;  // "no expert" marker in the top-k reduction

// Rounding of the accumulated dot product to the model dtype.
__device__ __forceinline__ float round_logit(double d, float*) { return __double2float_rn(d); }
__device__ __forceinline__ float round_logit(float f, __nv_bfloat16*) {
  return __bfloat162float(__float2bfloat16_rn(f));
}

// Logits.  Lane l of a warp owns hidden positions h = 256 j + 8 l + v
// (j = 0, 1, ...; v = 0..7) and adds its products in that (j, v) order; the
// 32 lane sums are then combined by an xor butterfly (offsets 16, 8, 4, 2, 1).
// The order is the same whatever the alignment or H, so the CPU oracle can
// replay it exactly.  Acc is float for bf16 inputs (bf16*bf16 products are
// exact in fp32) and double for fp32 inputs (exact products, and a sum whose
// single rounding to fp32 is the correctly rounded logit).
template <typename T, typename Acc, bool kVec>
__global__ void __launch_bounds__(kWarps * 32)
router_logits_kernel(const T* __restrict__ x, const T* __restrict__ w, int64_t tokens, int hidden,
                     int experts, float* __restrict__ logits_f32, T* __restrict__ logits_out) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t t0 = (int64_t)blockIdx.x * kTokTile;
  const int ntok = (int)((tokens - t0) < kTokTile ? (tokens - t0) : kTokTile);

  for (int ej = warp; ej < kExpTile; ej += kWarps) {
    const int e = blockIdx.y * kExpTile + ej;
    if (e >= experts) break;
    Acc acc[kTokTile];
#pragma unroll
    for (int i = 0; i < kTokTile; ++i) acc[i] = Acc(0);
    const T* wrow = w + (int64_t)e * hidden;
    for (int h0 = 8 * lane; h0 < hidden; h0 += 256) {
      T wv[8];
      if (kVec) {
#pragma unroll
        for (int q = 0; q < (int)(8 * sizeof(T) / 16); ++q)
          reinterpret_cast<uint4*>(wv)[q] = reinterpret_cast<const uint4*>(wrow + h0)[q];
      } else {
#pragma unroll
        for (int v = 0; v < 8; ++v) wv[v] = (h0 + v < hidden) ? wrow[h0 + v] : from_f32<T>(0.f);
      }
#pragma unroll
      for (int i = 0; i < kTokTile; ++i) {
        if (i < ntok) {
          const T* xrow = x + (t0 + i) * hidden;
          T xv[8];
          if (kVec) {
#pragma unroll
            for (int q = 0; q < (int)(8 * sizeof(T) / 16); ++q)
              reinterpret_cast<uint4*>(xv)[q] = reinterpret_cast<const uint4*>(xrow + h0)[q];
          } else {
#pragma unroll
            for (int v = 0; v < 8; ++v) xv[v] = (h0 + v < hidden) ? xrow[h0 + v] : from_f32<T>(0.f);
          }
#pragma unroll
          for (int v = 0; v < 8; ++v)
            acc[i] = fma((Acc)to_f32(xv[v]), (Acc)to_f32(wv[v]), acc[i]);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < kTokTile; ++i) {
      Acc s = acc[i];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
      if (lane == 0 && i < ntok) {
        const float r = round_logit(s, (T*)nullptr);
        logits_f32[(t0 + i) * experts + e] = r;
        if (logits_out) logits_out[(t0 + i) * experts + e] = from_f32<T>(r);
      }
    }
  }
}

// Staged variant for 16-byte aligned rows: the CTA's token rows and expert
// rows are first copied into shared memory with one burst of asynchronous
// 16-byte copies (cp.async), so the dot products run from shared memory
// instead of waiting on one round of L2 loads per 256 columns.  Same lane
// assignment and summation order as router_logits_kernel.  kET experts per
// CTA: 16 normally, 4 when few token tiles would leave most SMs idle (a
// verify pass of a handful of rows); every (token, expert) sum is still one
// warp's, in the same order, so the logits are the same bits either way.
template <typename T, typename Acc, int kET>
__global__ void __launch_bounds__(kWarps * 32)
router_logits_staged(const T* __restrict__ x, const T* __restrict__ w, int64_t tokens, int hidden,
                     int experts, float* __restrict__ logits_f32, T* __restrict__ logits_out) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) uint8_t smem_raw[];
  T* xs = reinterpret_cast<T*>(smem_raw);        // [kTokTile][hidden]
  T* ws = xs + (size_t)kTokTile * hidden;         // [kET][hidden]
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t t0 = (int64_t)blockIdx.x * kTokTile;
  const int ntok = (int)((tokens - t0) < kTokTile ? (tokens - t0) : kTokTile);
  const int e0 = blockIdx.y * kET;
  const int nexp = (experts - e0) < kET ? (experts - e0) : kET;
  const int vec_per_row = hidden * (int)sizeof(T) / 16;
  const int total = (ntok + nexp) * vec_per_row;
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int r = i / vec_per_row, c = i % vec_per_row;
    const T* src = (r < ntok) ? x + (t0 + r) * hidden : w + (int64_t)(e0 + r - ntok) * hidden;
    T* dst = (r < ntok) ? xs + (size_t)r * hidden : ws + (size_t)(r - ntok) * hidden;
    const uint32_t saddr = static_cast<uint32_t>(__cvta_generic_to_shared(dst + c * (16 / sizeof(T))));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr),
                 "l"(src + c * (16 / sizeof(T)))
                 : "memory");
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();

  // Warp w computes experts w, w + kWarps, ... of the CTA together (kEW of
  // them), so each token value is converted once per h-step for all of
  // them; every (token, expert) sum keeps its own order.
  constexpr int kEW = (kET + kWarps - 1) / kWarps;
  Acc acc[kEW][kTokTile];
#pragma unroll
  for (int x = 0; x < kEW; ++x)
#pragma unroll
    for (int i = 0; i < kTokTile; ++i) acc[x][i] = Acc(0);
  for (int h0 = 8 * lane; h0 < hidden; h0 += 256) {
    Acc wf[kEW][8];
#pragma unroll
    for (int x = 0; x < kEW; ++x) {
      const int ej = warp + x * kWarps;
      T wv[8];
      if (ej < nexp) {
#pragma unroll
        for (int q = 0; q < (int)(8 * sizeof(T) / 16); ++q)
          reinterpret_cast<uint4*>(wv)[q] = reinterpret_cast<const uint4*>(ws + (size_t)ej * hidden + h0)[q];
      } else {
#pragma unroll
        for (int v = 0; v < 8; ++v) wv[v] = from_f32<T>(0.f);
      }
#pragma unroll
      for (int v = 0; v < 8; ++v) wf[x][v] = (Acc)to_f32(wv[v]);
    }
#pragma unroll
    for (int i = 0; i < kTokTile; ++i) {
      if (i < ntok) {
        T xv[8];
#pragma unroll
        for (int q = 0; q < (int)(8 * sizeof(T) / 16); ++q)
          reinterpret_cast<uint4*>(xv)[q] = reinterpret_cast<const uint4*>(xs + (size_t)i * hidden + h0)[q];
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          const Acc xf = (Acc)to_f32(xv[v]);
#pragma unroll
          for (int x = 0; x < kEW; ++x) acc[x][i] = fma(xf, wf[x][v], acc[x][i]);
        }
      }
    }
  }
#pragma unroll
  for (int x = 0; x < kEW; ++x) {
    const int ej = warp + x * kWarps;
    const int e = e0 + ej;
#pragma unroll
    for (int i = 0; i < kTokTile; ++i) {
      Acc s = acc[x][i];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
      if (lane == 0 && i < ntok && ej < nexp) {
        const float r = round_logit(s, (T*)nullptr);
        logits_f32[(t0 + i) * experts + e] = r;
        if (logits_out) logits_out[(t0 + i) * experts + e] = from_f32<T>(r);
      }
    }
  }
}

// Softmax + top-k of token t's logits, one warp: lane l holds the logits of
// experts l + 32 j, j < kEpl, in val (-inf past the last expert).
template <int kEpl>
__device__ __forceinline__ void softmax_topk_warp(const float (&val)[kEpl], int lane, int64_t t,
                                                  int experts, int top_k, int norm,
                                                  float* __restrict__ probs,
                                                  float* __restrict__ topk_w,
                                                  int64_t* __restrict__ topk_idx) {
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < kEpl; ++j) m = fmaxf(m, val[j]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  float ex[kEpl];
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < kEpl; ++j) {
    ex[j] = (lane + 32 * j < experts) ? expf(val[j] - m) : 0.f;
    s += ex[j];
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
#pragma unroll
  for (int j = 0; j < kEpl; ++j) {
    const int e = lane + 32 * j;
    if (e < experts) probs[t * experts + e] = ex[j] / s;
  }

  // Top-k by (logit desc, id asc).  taken: bit j <-> expert lane + 32 j.
  uint32_t taken = 0;
  float sel_p = 0.f;  // lane k < top_k keeps the k-th selected prob
  int sel_e = 0;
  for (int k = 0; k < top_k; ++k) {
    // Lane-local best; e grows with j, so a strict '>' keeps the lower id on ties.
    float bv = -INFINITY, bp = 0.f;
    int be = kNone;
#pragma unroll
    for (int j = 0; j < kEpl; ++j) {
      const int e = lane + 32 * j;
      if (e < experts && !((taken >> j) & 1u) && (be == kNone || val[j] > bv)) {
        bv = val[j];
        bp = ex[j];
        be = e;
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
      const float op = __shfl_xor_sync(0xffffffffu, bp, off);
      const int oe = __shfl_xor_sync(0xffffffffu, be, off);
      if (oe != kNone && (be == kNone || ov > bv || (ov == bv && oe < be))) {
        bv = ov;
        bp = op;
        be = oe;
      }
    }
    if (be != kNone && (be & 31) == lane) taken |= 1u << (be >> 5);
    if (lane == k) {
      sel_e = be;
      sel_p = bp / s;
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

// Softmax + top-k, warp per token, over logits in global memory.
template <int kEpl>
__global__ void __launch_bounds__(kWarps * 32)
router_topk_kernel(const float* __restrict__ logits, int64_t tokens, int experts, int top_k,
                   int norm, float* __restrict__ probs, float* __restrict__ topk_w,
                   int64_t* __restrict__ topk_idx) {
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (t >= tokens) return;
  const float* row = logits + t * experts;
  float val[kEpl];
#pragma unroll
  for (int j = 0; j < kEpl; ++j) {
    const int e = lane + 32 * j;
    val[j] = e < experts ? row[e] : -INFINITY;
  }
  softmax_topk_warp<kEpl>(val, lane, t, experts, top_k, norm, probs, topk_w, topk_idx);
}

// One launch: a cluster of ceil(E / 8) CTAs (at most 16) of 16 warps per
// tile of kTokTile tokens (grid.x = token tiles).  Each CTA stages its tile's
// tokens and 8 router rows in shared memory; warp w computes the logits of
// router row w % 8 for tokens 4 (w / 8) .. 4 (w / 8) + 3, each (token,
// expert) sum in exactly the lane assignment and order of
// router_logits_staged, so the logits are the same bits.  CTA 0 of the
// cluster then reads every logit of the tile's tokens through distributed
// shared memory and runs the softmax / top-k of router_topk_kernel.
constexpr int kFusedET = 8;
constexpr int kFusedGroups = 2;                       // token groups per router row
constexpr int kFusedTok = kTokTile / kFusedGroups;    // tokens per warp
constexpr int kFusedWarps = kFusedET * kFusedGroups;
constexpr int kFusedMaxCluster = 16;

template <typename T, typename Acc, int kEpl>
__global__ void __launch_bounds__(kFusedWarps * 32)
router_fused_kernel(const T* __restrict__ x, const T* __restrict__ w, int tokens, int hidden,
                    int experts, int top_k, int norm, float* __restrict__ probs,
                    float* __restrict__ topk_w, int64_t* __restrict__ topk_idx,
                    T* __restrict__ logits_out) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __shared__ float lg[kTokTile][kFusedET];
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const int crank = (int)cluster.block_rank();
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int tb = blockIdx.x * kTokTile;  // first token of this cluster's tile
  const int ntok = min(kTokTile, tokens - tb);
  x += (int64_t)tb * hidden;
  T* xs = reinterpret_cast<T*>(smem_raw);        // [ntok][hidden]
  T* ws = xs + (size_t)ntok * hidden;             // [kFusedET][hidden]
  const int e0 = crank * kFusedET;
  const int nexp = max(0, min(kFusedET, experts - e0));
  const int vec_per_row = hidden * (int)sizeof(T) / 16;
  const int total = (ntok + nexp) * vec_per_row;
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int r = i / vec_per_row, c = i % vec_per_row;
    const T* src = (r < ntok) ? x + (int64_t)r * hidden : w + (int64_t)(e0 + r - ntok) * hidden;
    T* dst = (r < ntok) ? xs + (size_t)r * hidden : ws + (size_t)(r - ntok) * hidden;
    const uint32_t saddr = static_cast<uint32_t>(__cvta_generic_to_shared(dst + c * (16 / sizeof(T))));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr),
                 "l"(src + c * (16 / sizeof(T)))
                 : "memory");
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();

  const int ej = warp % kFusedET;
  const int t0 = (warp / kFusedET) * kFusedTok;
  if (ej < nexp && t0 < ntok) {
    Acc acc[kFusedTok];
#pragma unroll
    for (int i = 0; i < kFusedTok; ++i) acc[i] = Acc(0);
    const T* wrow = ws + (size_t)ej * hidden;
    for (int h0 = 8 * lane; h0 < hidden; h0 += 256) {
      T wv[8];
#pragma unroll
      for (int q = 0; q < (int)(8 * sizeof(T) / 16); ++q)
        reinterpret_cast<uint4*>(wv)[q] = reinterpret_cast<const uint4*>(wrow + h0)[q];
#pragma unroll
      for (int i = 0; i < kFusedTok; ++i) {
        if (t0 + i < ntok) {
          T xv[8];
#pragma unroll
          for (int q = 0; q < (int)(8 * sizeof(T) / 16); ++q)
            reinterpret_cast<uint4*>(xv)[q] =
                reinterpret_cast<const uint4*>(xs + (size_t)(t0 + i) * hidden + h0)[q];
#pragma unroll
          for (int v = 0; v < 8; ++v)
            acc[i] = fma((Acc)to_f32(xv[v]), (Acc)to_f32(wv[v]), acc[i]);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < kFusedTok; ++i) {
      Acc sum = acc[i];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      if (lane == 0 && t0 + i < ntok) {
        const float r = round_logit(sum, (T*)nullptr);
        lg[t0 + i][ej] = r;
        if (logits_out) logits_out[(int64_t)(tb + t0 + i) * experts + e0 + ej] = from_f32<T>(r);
      }
    }
  }
  cluster.sync();  // every CTA's logits are in its shared memory
  if (crank == 0 && warp < ntok) {
    float val[kEpl];
#pragma unroll
    for (int j = 0; j < kEpl; ++j) {
      const int e = lane + 32 * j;
      val[j] = e < experts ? *cluster.map_shared_rank(&lg[warp][e % kFusedET], e / kFusedET)
                           : -INFINITY;
    }
    softmax_topk_warp<kEpl>(val, lane, (int64_t)tb + warp, experts, top_k, norm, probs, topk_w, topk_idx);
  }
  cluster.sync();  // peers keep their shared memory until CTA 0 has read it
}

template <int kEpl>
void launch_topk(const float* logits, int64_t tokens, int E, int K, int norm, float* probs,
                 float* topk_w, int64_t* topk_idx, cudaStream_t stream) {
  // Launch errors surface through the caller's cudaGetLastError check.
  (void)launch_pdl(router_topk_kernel<kEpl>, dim3((unsigned)((tokens + kWarps - 1) / kWarps)),
                   dim3(kWarps * 32), 0, stream, logits, tokens, E, K, norm, probs, topk_w,
                   topk_idx);
}

template <typename T, typename Acc, int kEpl>
int launch_fused_epl(const T* x, const T* w, int tokens, int H, int E, int K, int norm,
                     float* probs, float* topk_w, int64_t* topk_idx, T* logits_out, size_t smem,
                     cudaStream_t stream) {
  static std::atomic<unsigned long long> configured{0};
  if (int rc = once_per_device(configured, [] {
        SF_CHECK_CUDA(cudaFuncSetAttribute(router_fused_kernel<T, Acc, kEpl>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        SF_CHECK_CUDA(cudaFuncSetAttribute(router_fused_kernel<T, Acc, kEpl>,
                                           cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
        return SF_OK;
      }))
    return rc;
  const unsigned cluster = (unsigned)((E + kFusedET - 1) / kFusedET);  // <= kFusedMaxCluster
  const unsigned tiles = (unsigned)((tokens + kTokTile - 1) / kTokTile);
  SF_CHECK_CUDA(launch_pdl_cluster(router_fused_kernel<T, Acc, kEpl>, dim3(tiles, cluster, 1),
                                   dim3(kFusedWarps * 32), smem, stream, 1u, cluster, x, w, tokens,
                                   H, E, K, norm, probs, topk_w, topk_idx, logits_out));
  return SF_OK;
}

// Whether this device co-schedules clusters of `size` CTAs of the fused
// kernel (16 exceeds the portable limit of 8), checked once per device and
// size; the two-launch path serves devices that do not.
template <typename T, typename Acc>
bool fused_clusters_ok(int size, size_t smem) {
  static std::mutex mu;
  static int known[64][kFusedMaxCluster + 1] = {};  // 0 unknown, 1 yes, 2 no
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
  std::lock_guard<std::mutex> lock(mu);
  int& k = known[dev][size];
  if (k == 0) {
    bool ok = cudaFuncSetAttribute(router_fused_kernel<T, Acc, 4>,
                                   cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess &&
              cudaFuncSetAttribute(router_fused_kernel<T, Acc, 4>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) == cudaSuccess;
    if (ok) {
      cudaLaunchConfig_t probe = {};
      probe.gridDim = dim3(1, (unsigned)size, 1);
      probe.blockDim = dim3(kFusedWarps * 32, 1, 1);
      probe.dynamicSmemBytes = smem;
      cudaLaunchAttribute a[1];
      a[0].id = cudaLaunchAttributeClusterDimension;
      a[0].val.clusterDim.x = 1;
      a[0].val.clusterDim.y = (unsigned)size;
      a[0].val.clusterDim.z = 1;
      probe.attrs = a;
      probe.numAttrs = 1;
      int clusters = 0;
      ok = cudaOccupancyMaxActiveClusters(&clusters, router_fused_kernel<T, Acc, 4>, &probe) ==
               cudaSuccess && clusters > 0;
    }
    (void)cudaGetLastError();
    k = ok ? 1 : 2;
  }
  return k == 1;
}

template <typename T, typename Acc>
int launch_fused(const T* x, const T* w, int tokens, int H, int E, int K, int norm, float* probs,
                 float* topk_w, int64_t* topk_idx, T* logits_out, size_t smem, cudaStream_t stream) {
  const int epl = (E + 31) / 32;
  if (epl <= 1)
    return launch_fused_epl<T, Acc, 1>(x, w, tokens, H, E, K, norm, probs, topk_w, topk_idx,
                                       logits_out, smem, stream);
  if (epl <= 2)
    return launch_fused_epl<T, Acc, 2>(x, w, tokens, H, E, K, norm, probs, topk_w, topk_idx,
                                       logits_out, smem, stream);
  return launch_fused_epl<T, Acc, 4>(x, w, tokens, H, E, K, norm, probs, topk_w, topk_idx,
                                     logits_out, smem, stream);
}

template <typename T>
int launch_router(const void* hidden, const void* weight, int64_t tokens, int H, int E, int K,
                  int norm, float* probs, float* topk_w, int64_t* topk_idx, void* logits_out,
                  float* logits_ws, cudaStream_t stream) {
  using Acc = typename std::conditional<std::is_same<T, float>::value, double, float>::type;
  const T* x = static_cast<const T*>(hidden);
  const T* w = static_cast<const T*>(weight);
  dim3 grid((unsigned)((tokens + kTokTile - 1) / kTokTile), (unsigned)((E + kExpTile - 1) / kExpTile));
  const bool vec = (H % 8 == 0) && aligned16(x) && aligned16(w);
  const size_t fused_smem = (size_t)((tokens < kTokTile ? tokens : kTokTile) + kFusedET) * H * sizeof(T);
  // The cluster launch pays off only for a handful of tokens: at 65 and 512
  // rows it measured slower on a B200 than the two launches below (15.4 vs
  // 14.0 us and 56.7 vs 46.3 us inside a graph).
  if (std::is_same<T, __nv_bfloat16>::value && vec && tokens <= kTokTile &&
      E <= kFusedET * kFusedMaxCluster && fused_smem <= 200 * 1024 &&
      fused_clusters_ok<T, Acc>((E + kFusedET - 1) / kFusedET, fused_smem))
    return launch_fused<T, Acc>(x, w, (int)tokens, H, E, K, norm, probs, topk_w, topk_idx,
                                static_cast<T*>(logits_out), fused_smem, stream);
  const bool few = (int64_t)grid.x * grid.y < num_sms();
  constexpr int kSmallTile = 4;
  const size_t staged_smem = (size_t)(kTokTile + (few ? kSmallTile : kExpTile)) * H * sizeof(T);
  if (vec && staged_smem <= 200 * 1024) {
    static std::atomic<unsigned long long> configured{0};
    if (int rc = once_per_device(configured, [] {
          SF_CHECK_CUDA(cudaFuncSetAttribute(router_logits_staged<T, Acc, kExpTile>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
          SF_CHECK_CUDA(cudaFuncSetAttribute(router_logits_staged<T, Acc, kSmallTile>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
          return SF_OK;
        }))
      return rc;
    if (few) {
      grid.y = (unsigned)((E + kSmallTile - 1) / kSmallTile);
      SF_CHECK_CUDA(launch_pdl(router_logits_staged<T, Acc, kSmallTile>, dim3(grid),
                               dim3(kWarps * 32), staged_smem, stream, x, w, tokens, H, E,
                               logits_ws, static_cast<T*>(logits_out)));
    } else {
      SF_CHECK_CUDA(launch_pdl(router_logits_staged<T, Acc, kExpTile>, dim3(grid),
                               dim3(kWarps * 32), staged_smem, stream, x, w, tokens, H, E,
                               logits_ws, static_cast<T*>(logits_out)));
    }
  } else if (vec)
    SF_CHECK_CUDA(launch_pdl(router_logits_kernel<T, Acc, true>, dim3(grid), dim3(kWarps * 32), 0,
                             stream, x, w, tokens, H, E, logits_ws, static_cast<T*>(logits_out)));
  else
    SF_CHECK_CUDA(launch_pdl(router_logits_kernel<T, Acc, false>, dim3(grid), dim3(kWarps * 32), 0,
                             stream, x, w, tokens, H, E, logits_ws, static_cast<T*>(logits_out)));
  SF_CHECK_LAUNCH();
  const int epl = (E + 31) / 32;
  if (epl <= 1) launch_topk<1>(logits_ws, tokens, E, K, norm, probs, topk_w, topk_idx, stream);
  else if (epl <= 2) launch_topk<2>(logits_ws, tokens, E, K, norm, probs, topk_w, topk_idx, stream);
  else if (epl <= 4) launch_topk<4>(logits_ws, tokens, E, K, norm, probs, topk_w, topk_idx, stream);
  else if (epl <= 8) launch_topk<8>(logits_ws, tokens, E, K, norm, probs, topk_w, topk_idx, stream);
  else if (epl <= 16) launch_topk<16>(logits_ws, tokens, E, K, norm, probs, topk_w, topk_idx, stream);
  else launch_topk<32>(logits_ws, tokens, E, K, norm, probs, topk_w, topk_idx, stream);
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
// Some callers cannot hand this library a workspace because they cannot get
// device memory at the point of the call: plugins loaded into a serving
// engine that reserves the GPU's memory for its own pools at start-up (a
// cudaMalloc there fails or fragments the engine's pool), hosts that bind the
// library through a plain C FFI with no device allocator to carve a
// workspace from, and latency-critical paths where cudaMalloc's implicit
// device-wide synchronisation would stall every other stream.
// sf_router_topk_noalloc serves them: its scratch (the fp32 logits between
// the two router passes) is this file-scope device array, which every GPU
// that loads the library holds until the process exits.  Calls on one device
// share it, so calls that overlap on the GPU race.

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
// per device (the first call on a device, which must come before any stream
// capture) and kept.  The host-side symbol is only a stand-in and must never
// be passed to a kernel.  The kept address belongs to the device's primary
// context and is stale after cudaDeviceReset.
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
