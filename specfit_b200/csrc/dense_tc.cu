// Skinny bf16 projection GEMM on tcgen05 for verify-sized row counts.
//
//   Y[T, N] = X[T, K] . W[N, K]^T      (F.linear without bias), T <= 128
//   argmax_n bf16(Y[t, n])              (optional, fused: lm_head + greedy pick)
//
// The projections of a verify pass (q|k|v, o, the drafter's layers and
// lm_head) see a handful of token rows against weight matrices of tens to
// hundreds of MB, so they are weight-streaming problems: the bound is reading
// W once from HBM.  Layout "swap AB" as in the grouped SwiGLU: 128 weight
// rows fill the MMA's M dimension and the T token rows form N (16, 32, 64
// or 128), both operands K-major and loaded by TMA with 128-byte swizzling.
//
// Parallelism comes from splitting K: the CTAs of a thread-block cluster
// (up to 8) share one 128-row tile, each accumulating its K range in TMEM.
// CTA r owns rows [r*128/S, (r+1)*128/S) of the output: every CTA stores its
// fp32 partial of those rows into the owner's shared memory (distributed
// shared memory), and after one cluster barrier the owner adds the S
// partials in rank order (a fixed order: the result does not depend on
// timing) and rounds once to bf16.
//
// With an argmax workspace the same owner pass also reduces its rows of
// every token: bf16-rounded values, the largest one and, among equal ones,
// the lowest row (what torch.argmax returns on the bf16 logits; a NaN counts
// as the largest value and -0 equals +0, as there); one (key, row) pair per
// (tile, cluster rank, token) goes to the workspace and a second launch
// picks each token's winner over them.  The order is total, so the winner
// does not depend on the order of the reduction.
//
// Wide outputs (the 151,936-row lm_head: more 128-row tiles than SMs) take a
// second kernel, dense_stream_kernel: one persistent CTA per SM walks its
// tiles with the whole K range each, the TMA ring running on across tiles
// and two TMEM accumulators letting the epilogue of one tile (rounding, the
// store, the argmax) overlap the MMAs of the next.  Its epilogue warps keep a
// running best per token across their tiles, so one (key, row) pair per
// (CTA, epilogue warp, token) reaches the workspace.
//
// Roles per CTA (192 threads): warp 0 lane 0 issues TMA (weights for the
// first stages before waiting on the preceding kernel, since they do not
// depend on it), warp 1 lane 0 allocates TMEM and issues the MMAs, warps
// 2..5 read the accumulator back.  Every TMA load is issued by a CTA for its
// own shared memory.  Waits give up after a bounded time, record a site code
// in the status word read by sf_device_status and let the kernel finish.
#include <cooperative_groups.h>
#include <cuda.h>

#include "common.cuh"
#include "sm100_ptx.cuh"
#include "swiglu.h"

namespace sf {
namespace {

namespace cg = cooperative_groups;

__device__ int g_dense_status;

constexpr int kBM = 128;       // weight rows per tile (MMA M)
constexpr int kBK = 64;        // K per stage: one 128-byte swizzle atom of bf16
constexpr int kStages = 4;
constexpr int kThreads = 192;
constexpr int kABytes = kBM * kBK * 2;
constexpr int kMaxSplit = 8;   // portable cluster size

template <int kBN>
constexpr uint32_t tmem_cols() {  // a power of two >= 32 holding kBN fp32 columns
  return kBN < 32 ? 32u : (uint32_t)kBN;
}

struct ArgmaxPart {
  uint32_t key;  // order_key of the bf16-rounded value
  int32_t row;   // -1: no candidate
};

// An unsigned key with the order torch.argmax uses on floats: NaN above every
// number, -0 equal to +0, otherwise the numeric order.  Every non-NaN key is
// at least order_key(-inf) = 0x007fffff, so 0 is free for "no value".
__device__ __forceinline__ uint32_t order_key(float v) {
  if (v != v) return 0xffffffffu;
  if (v == 0.f) v = 0.f;
  const uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// The better of two candidates: larger key, then lower row.
__device__ __forceinline__ ArgmaxPart better(ArgmaxPart a, ArgmaxPart b) {
  if (b.row < 0) return a;
  if (a.row < 0) return b;
  if (b.key > a.key || (b.key == a.key && b.row < a.row)) return b;
  return a;
}

template <int kBN>
struct __align__(1024) DenseSmem {
  uint8_t a[kStages][kABytes];
  uint8_t b[kStages][kBN * kBK * 2];
  // This CTA's rows of every split's partial tile: slot s * rows_per + r
  // holds split s's accumulator of row r0 + r (rows_per = ceil(128 / S)).
  float part[kBM + kMaxSplit][kBN + 1];
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t acc_full;
  uint32_t tmem_base;
  int abort_flag;
};

template <int kBN>
constexpr size_t dense_smem_bytes() {
  return sizeof(DenseSmem<kBN>) + 1024;  // + alignment slack
}

template <int kBN>
__global__ void __launch_bounds__(kThreads)
dense_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                int T, int N, int K, __nv_bfloat16* __restrict__ y, ArgmaxPart* __restrict__ argmax_part) {
  constexpr uint32_t kBBytes = kBN * kBK * 2;
  constexpr uint32_t kTmemCols = tmem_cols<kBN>();
  extern __shared__ uint8_t smem_raw[];
  auto* sm = reinterpret_cast<DenseSmem<kBN>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  cg::cluster_group cluster = cg::this_cluster();
  const int split = (int)cluster.num_blocks();
  const int crank = (int)cluster.block_rank();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * kBM;
  const int kb_total = K / kBK;
  const int per = (kb_total + split - 1) / split;
  const int kb0 = min(kb_total, crank * per);
  const int nkb = min(kb_total, kb0 + per) - kb0;
  const int rows_per = (kBM + split - 1) / split;
  volatile int* abort_flag = &sm->abort_flag;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      ptx::mbar_init(&sm->full[s], 1);
      ptx::mbar_init(&sm->empty[s], 1);
    }
    ptx::mbar_init(&sm->acc_full, 1);
    sm->abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tensormap(&tm_w);
    ptx::prefetch_tensormap(&tm_x);
  }
  if (warp == 1) {
    ptx::tmem_alloc(&sm->tmem_base, kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = sm->tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      const int pre = min(nkb, kStages);
      // Weight tiles of the first stages: independent of the preceding kernel.
      for (int i = 0; i < pre; ++i) {
        ptx::mbar_arrive_expect_tx(&sm->full[i], kABytes + kBBytes);
        ptx::tma_load_2d(sm->a[i], &tm_w, &sm->full[i], (kb0 + i) * kBK, m0);
      }
      pdl_wait();
      pdl_trigger();
      for (int i = 0; i < pre; ++i)
        ptx::tma_load_2d(sm->b[i], &tm_x, &sm->full[i], (kb0 + i) * kBK, 0);
      int issued = pre;
      for (int i = pre; i < nkb; ++i) {
        const int s = i % kStages;
        const uint32_t ph = (i / kStages) & 1;
        if (!ptx::mbar_wait(&sm->empty[s], ph ^ 1, abort_flag, &g_dense_status, 11)) break;
        ptx::mbar_arrive_expect_tx(&sm->full[s], kABytes + kBBytes);
        ptx::tma_load_2d(sm->a[s], &tm_w, &sm->full[s], (kb0 + i) * kBK, m0);
        ptx::tma_load_2d(sm->b[s], &tm_x, &sm->full[s], (kb0 + i) * kBK, 0);
        issued = i + 1;
      }
      // Let every load issued above land before the CTA can exit.
      volatile int never = 0;
      for (int i = (issued > kStages ? issued - kStages : 0); i < issued; ++i)
        ptx::mbar_wait(&sm->full[i % kStages], (i / kStages) & 1, &never, &g_dense_status, 12);
    } else {
      pdl_wait();
    }
  } else if (warp == 1) {
    pdl_wait();
    if (lane == 0) {
      const uint32_t idesc = ptx::idesc_bf16_f32(kBM, kBN);
      for (int i = 0; i < nkb; ++i) {
        const int s = i % kStages;
        const uint32_t ph = (i / kStages) & 1;
        if (!ptx::mbar_wait(&sm->full[s], ph, abort_flag, &g_dense_status, 13)) break;
        ptx::tc_fence_after();
        const uint64_t adesc = ptx::smem_desc_k_sw128(ptx::smem_u32(sm->a[s]));
        const uint64_t bdesc = ptx::smem_desc_k_sw128(ptx::smem_u32(sm->b[s]));
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k)
          ptx::umma_f16(tmem, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), idesc,
                        (i | k) != 0);
        ptx::umma_commit(&sm->empty[s]);
      }
      ptx::umma_commit(&sm->acc_full);
    }
  } else {
    pdl_wait();
    // Epilogue: TMEM lane quadrant (warp % 4) -> accumulator row; the row's
    // partial goes straight into the shared memory of the CTA that reduces
    // it (asynchronous stores through distributed shared memory).
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const int owner = row / rows_per;
    float* dst = cluster.map_shared_rank(&sm->part[0][0], owner) +
                 (crank * rows_per + (row - owner * rows_per)) * (kBN + 1);
    bool have = nkb > 0;
    if (have) have = ptx::mbar_wait(&sm->acc_full, 0, abort_flag, &g_dense_status, 14);
    if (have) {
      ptx::tc_fence_after();
#pragma unroll
      for (int c = 0; c < kBN / 16; ++c) {
        float v[16];
        ptx::tmem_ld_16(tmem + ((uint32_t)(quad * 32) << 16) + c * 16, v);
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if (c * 16 + i < T) dst[c * 16 + i] = v[i];
      }
    } else {
      for (int i = 0; i < T; ++i) dst[i] = 0.f;
    }
  }
  ptx::tc_fence_before();
  __syncthreads();  // TMEM reads done
  if (warp == 1) {
    __syncwarp();
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, kTmemCols);
  }
  cluster.sync();  // every split's partial rows have landed with their owner
  const int r0 = min(kBM, crank * rows_per);
  const int nr = min(kBM, r0 + rows_per) - r0;
  if (y != nullptr) {
    for (int idx = threadIdx.x; idx < nr * T; idx += kThreads) {
      const int t = idx / nr, r = idx % nr;
      if (m0 + r0 + r >= N) continue;
      float acc = 0.f;
      for (int s = 0; s < split; ++s) acc += sm->part[s * rows_per + r][t];  // rank order
      y[(int64_t)t * N + m0 + r0 + r] = __float2bfloat16_rn(acc);
    }
  }
  if (argmax_part != nullptr) {
    // One warp per token: lanes stride over this CTA's rows, then a
    // butterfly keeps the larger value / lower row.
    for (int t = warp; t < T; t += kThreads / 32) {
      ArgmaxPart best{0u, -1};
      for (int r = lane; r < nr; r += 32) {
        const int row = m0 + r0 + r;
        if (row >= N) break;
        float acc = 0.f;
        for (int s = 0; s < split; ++s) acc += sm->part[s * rows_per + r][t];  // the same sum as y
        best = better(best, ArgmaxPart{order_key(__bfloat162float(__float2bfloat16_rn(acc))), row});
      }
#pragma unroll
      for (int off = 16; off; off >>= 1) {
        ArgmaxPart o{__shfl_xor_sync(0xffffffffu, best.key, off),
                     __shfl_xor_sync(0xffffffffu, best.row, off)};
        best = better(best, o);
      }
      if (lane == 0) argmax_part[((int64_t)blockIdx.y * split + crank) * T + t] = best;
    }
  }
}

// Each token's winner over the candidates (part p of token t at p * T + t).
__global__ void __launch_bounds__(256)
argmax_reduce_kernel(const ArgmaxPart* __restrict__ part, int nparts, int T, int64_t* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  ArgmaxPart best{0u, -1};
  for (int p = lane; p < nparts; p += 32) best = better(best, part[(int64_t)p * T + t]);
#pragma unroll
  for (int off = 16; off; off >>= 1) {
    ArgmaxPart o{__shfl_xor_sync(0xffffffffu, best.key, off), __shfl_xor_sync(0xffffffffu, best.row, off)};
    best = better(best, o);
  }
  if (lane == 0) out[t] = best.row;
}

// ---------------------------------------------------------------------------
// Persistent variant for wide outputs (m_tiles >= SMs).

template <int kBN>
struct StreamCfg {
  static constexpr uint32_t kBBytes = kBN * kBK * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = (200u * 1024u) / kStageBytes < 12u ? (int)((200u * 1024u) / kStageBytes) : 12;
  // Two accumulators of kBN fp32 columns, rounded up to a power of two >= 32.
  static constexpr uint32_t kTmemCols = 2 * kBN <= 32 ? 32u : 2 * kBN <= 64 ? 64u : 2 * kBN <= 128 ? 128u : 256u;
  static constexpr int kSlots = (kBN + 31) / 32;  // running-best registers per lane
  static constexpr uint32_t kAccStride = kTmemCols / 2;  // column of accumulator 1 (a power of two)
};

template <int kBN>
struct __align__(1024) StreamSmem {
  uint8_t a[StreamCfg<kBN>::kStages][kABytes];
  uint8_t b[StreamCfg<kBN>::kStages][StreamCfg<kBN>::kBBytes];
  uint64_t full[StreamCfg<kBN>::kStages];
  uint64_t empty[StreamCfg<kBN>::kStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort_flag;
  int epi_go;
};

template <int kBN>
constexpr size_t stream_smem_bytes() {
  return sizeof(StreamSmem<kBN>) + 1024;  // + alignment slack
}

// CTA b takes tiles b, b + G, ...; every role walks the same list.
template <int kBN>
__global__ void __launch_bounds__(kThreads, 1)
dense_stream_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                    int T, int N, int K, __nv_bfloat16* __restrict__ y, ArgmaxPart* __restrict__ argmax_part) {
  using Cfg = StreamCfg<kBN>;
  constexpr int kSt = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  auto* sm = reinterpret_cast<StreamSmem<kBN>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = (N + kBM - 1) / kBM;
  const int kb_total = K / kBK;
  volatile int* abort_flag = &sm->abort_flag;
  if ((int)blockIdx.x >= m_tiles) return;  // the grid never exceeds the tiles

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSt; ++s) {
      ptx::mbar_init(&sm->full[s], 1);
      ptx::mbar_init(&sm->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(&sm->acc_full[b], 1);
      ptx::mbar_init(&sm->acc_empty[b], 128);
    }
    ptx::mbar_init(&sm->mma_done, 1);
    sm->abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tensormap(&tm_w);
    ptx::prefetch_tensormap(&tm_x);
  }
  if (warp == 1) {
    ptx::tmem_alloc(&sm->tmem_base, Cfg::kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = sm->tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      // The first stages' weight tiles do not depend on the preceding kernel:
      // issue them before waiting for it.
      const int first = min(kb_total, kSt);
      const int m0 = blockIdx.x * kBM;
      for (int i = 0; i < first; ++i) {
        ptx::mbar_arrive_expect_tx(&sm->full[i], Cfg::kStageBytes);
        ptx::tma_load_2d(sm->a[i], &tm_w, &sm->full[i], i * kBK, m0);
      }
      pdl_wait();
      pdl_trigger();
      for (int i = 0; i < first; ++i) ptx::tma_load_2d(sm->b[i], &tm_x, &sm->full[i], i * kBK, 0);
      uint32_t it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < m_tiles && ok; tile += gridDim.x) {
        const int m0t = tile * kBM;
        for (int kb = 0; kb < kb_total; ++kb, ++it) {
          if (it < (uint32_t)first) continue;  // issued above
          const int s = it % kSt;
          const uint32_t ph = (it / kSt) & 1;
          if (!ptx::mbar_wait(&sm->empty[s], ph ^ 1, abort_flag, &g_dense_status, 21)) {
            ok = false;
            break;
          }
          ptx::mbar_arrive_expect_tx(&sm->full[s], Cfg::kStageBytes);
          ptx::tma_load_2d(sm->a[s], &tm_w, &sm->full[s], kb * kBK, m0t);
          ptx::tma_load_2d(sm->b[s], &tm_x, &sm->full[s], kb * kBK, 0);
        }
      }
      // Let every load issued above land before the CTA can exit.
      volatile int never = 0;
      for (uint32_t i = (it > (uint32_t)kSt ? it - kSt : 0u); i < it; ++i)
        ptx::mbar_wait(&sm->full[i % kSt], (i / kSt) & 1, &never, &g_dense_status, 22);
    } else {
      pdl_wait();
    }
  } else if (warp == 1) {
    pdl_wait();
    if (lane == 0) {
      const uint32_t idesc = ptx::idesc_bf16_f32(kBM, kBN);
      uint32_t it = 0, unit = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < m_tiles && ok; tile += gridDim.x, ++unit) {
        const int buf = unit & 1;
        if (!ptx::mbar_wait(&sm->acc_empty[buf], ((unit >> 1) & 1) ^ 1, abort_flag, &g_dense_status, 23)) break;
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem + buf * Cfg::kAccStride;
        for (int kb = 0; kb < kb_total; ++kb, ++it) {
          const int s = it % kSt;
          if (!ptx::mbar_wait(&sm->full[s], (it / kSt) & 1, abort_flag, &g_dense_status, 24)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint64_t adesc = ptx::smem_desc_k_sw128(ptx::smem_u32(sm->a[s]));
          const uint64_t bdesc = ptx::smem_desc_k_sw128(ptx::smem_u32(sm->b[s]));
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            ptx::umma_f16(d_tmem, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), idesc, (kb | k) != 0);
          ptx::umma_commit(&sm->empty[s]);
        }
        if (ok) ptx::umma_commit(&sm->acc_full[buf]);
      }
      // Drain: fires once every MMA issued above has completed.
      ptx::umma_commit(&sm->mma_done);
      volatile int never = 0;
      ptx::mbar_wait(&sm->mma_done, 0, &never, &g_dense_status, 25);
    }
  } else {
    pdl_wait();
    // Epilogue: TMEM lane quadrant (warp % 4) -> weight row of the tile.
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    uint32_t best_key[Cfg::kSlots];
    int32_t best_row[Cfg::kSlots];
#pragma unroll
    for (int j = 0; j < Cfg::kSlots; ++j) {
      best_key[j] = 0u;
      best_row[j] = -1;
    }
    uint32_t unit = 0;
    for (int tile = blockIdx.x; tile < m_tiles; tile += gridDim.x, ++unit) {
      const int buf = unit & 1;
      ptx::mbar_wait(&sm->acc_full[buf], (unit >> 1) & 1, abort_flag, &g_dense_status, 26);
      // One consistent go/stop decision for the four epilogue warps.
      ptx::named_bar_sync(2, 128);
      if (threadIdx.x == 64) sm->epi_go = !*abort_flag;
      ptx::named_bar_sync(2, 128);
      if (!sm->epi_go) break;
      ptx::tc_fence_after();
      const int n = tile * kBM + row;
      const bool valid = n < N;
      const uint32_t tbase = tmem + ((uint32_t)(quad * 32) << 16) + buf * Cfg::kAccStride;
#pragma unroll
      for (int c = 0; c < kBN / 16; ++c) {
        if (c * 16 < T) {
          float v[16];
          ptx::tmem_ld_16(tbase + c * 16, v);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int t = c * 16 + i;
            if (t < T) {
              const __nv_bfloat16 h = __float2bfloat16_rn(v[i]);
              if (y != nullptr && valid) y[(int64_t)t * N + n] = h;
              if (argmax_part != nullptr) {
                const uint32_t key = valid ? order_key(__bfloat162float(h)) : 0u;
                const uint32_t kmax = __reduce_max_sync(0xffffffffu, key);
                const int rmin = __reduce_min_sync(0xffffffffu, (valid && key == kmax) ? n : 0x7fffffff);
                const int j = (c * 16 + i) >> 5;  // this token's running-best slot (unrolled: static)
                if (lane == (t & 31) && rmin != 0x7fffffff &&
                    (best_row[j] < 0 || kmax > best_key[j] || (kmax == best_key[j] && rmin < best_row[j]))) {
                  best_key[j] = kmax;
                  best_row[j] = rmin;
                }
              }
            }
          }
        }
      }
      ptx::tc_fence_before();
      ptx::mbar_arrive(&sm->acc_empty[buf]);
    }
    if (argmax_part != nullptr) {
#pragma unroll
      for (int j = 0; j < Cfg::kSlots; ++j) {
        const int t = j * 32 + lane;
        if (t < T)
          argmax_part[((int64_t)blockIdx.x * 4 + quad) * T + t] = ArgmaxPart{best_key[j], best_row[j]};
      }
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

// Split of K over a cluster: while the tiles alone are fewer than the SMs,
// keeping the whole grid in one wave (clusters are placed one CTA per SM).
int dense_split(int N, int K) {
  const int m_tiles = (N + kBM - 1) / kBM;
  int split = num_sms() / m_tiles;
  return std::max(1, std::min(std::min(split, kMaxSplit), K / kBK));
}

// Wide outputs (at least one 128-row tile per SM) take the persistent kernel.
bool dense_streams(int N) { return (N + kBM - 1) / kBM >= num_sms(); }

// Argmax candidates per token that a launch writes.
int dense_argmax_parts(int N, int K) {
  const int m_tiles = (N + kBM - 1) / kBM;
  if (dense_streams(N)) return std::min(num_sms(), m_tiles) * 4;
  return m_tiles * dense_split(N, K);
}

template <int kBN>
int encode_dense_maps(const void* x, const void* w, int T, int N, int K, CUtensorMap* tm_w, CUtensorMap* tm_x) {
  {
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)N};
    cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    cuuint32_t box[2] = {kBK, kBM};  // rows past N read as zeros
    if (int rc = tma_encode_bf16(tm_w, w, 2, dims, strides, box)) return rc;
  }
  {
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)T};
    cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    cuuint32_t box[2] = {kBK, (cuuint32_t)kBN};  // rows past T read as zeros
    if (int rc = tma_encode_bf16(tm_x, x, 2, dims, strides, box)) return rc;
  }
  return SF_OK;
}

template <int kBN>
int launch_dense(const void* x, const void* w, void* y, int T, int N, int K, cudaStream_t stream,
                 ArgmaxPart* argmax_part = nullptr) {
  CUtensorMap tm_w, tm_x;
  if (int rc = encode_dense_maps<kBN>(x, w, T, N, K, &tm_w, &tm_x)) return rc;
  const int m_tiles = (N + kBM - 1) / kBM;
  auto* out = static_cast<__nv_bfloat16*>(y);
  if (dense_streams(N)) {
    static std::atomic<unsigned long long> configured{0};
    if (int rc = once_per_device(configured, [] {
          SF_CHECK_CUDA(cudaFuncSetAttribute(dense_stream_kernel<kBN>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)stream_smem_bytes<kBN>()));
          return SF_OK;
        }))
      return rc;
    const int grid = std::min(num_sms(), m_tiles);
    SF_CHECK_CUDA(launch_pdl(dense_stream_kernel<kBN>, dim3((unsigned)grid), dim3(kThreads),
                             stream_smem_bytes<kBN>(), stream, tm_w, tm_x, T, N, K, out, argmax_part));
    SF_CHECK_LAUNCH();
    return SF_OK;
  }
  if constexpr (kBN == 80 || kBN == 96) {
    return set_error(SF_ERR_UNSUPPORTED, "internal: %d-row token tiles are for wide outputs only", kBN);
  } else {
  static std::atomic<unsigned long long> configured{0};
  if (int rc = once_per_device(configured, [] {
        SF_CHECK_CUDA(cudaFuncSetAttribute(dense_tc_kernel<kBN>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)dense_smem_bytes<kBN>()));
        return SF_OK;
      }))
    return rc;
  const int split = dense_split(N, K);
  SF_CHECK_CUDA(launch_pdl_cluster(dense_tc_kernel<kBN>, dim3((unsigned)split, (unsigned)m_tiles, 1),
                                   dim3(kThreads), dense_smem_bytes<kBN>(), stream, (unsigned)split,
                                   1u, tm_w, tm_x, T, N, K, out, argmax_part));
  return SF_OK;
  }
}

int launch_dense_any(const void* x, const void* w, void* y, int T, int N, int K, cudaStream_t stream,
                     ArgmaxPart* argmax_part) {
  // The persistent kernel also takes token tiles of 80 and 96 rows: a
  // narrower token tile leaves room for one more stage of the weight ring.
  if (dense_streams(N) && T > 64 && T <= 80) return launch_dense<80>(x, w, y, T, N, K, stream, argmax_part);
  if (dense_streams(N) && T > 80 && T <= 96) return launch_dense<96>(x, w, y, T, N, K, stream, argmax_part);
  if (T <= 16) return launch_dense<16>(x, w, y, T, N, K, stream, argmax_part);
  if (T <= 32) return launch_dense<32>(x, w, y, T, N, K, stream, argmax_part);
  if (T <= 64) return launch_dense<64>(x, w, y, T, N, K, stream, argmax_part);
  return launch_dense<128>(x, w, y, T, N, K, stream, argmax_part);
}

}  // namespace

int dense_status(int* status, int reset) {
  SF_CHECK_CUDA(cudaMemcpyFromSymbol(status, g_dense_status, sizeof(int)));
  if (reset) {
    const int zero = 0;
    SF_CHECK_CUDA(cudaMemcpyToSymbol(g_dense_status, &zero, sizeof(int)));
  }
  return SF_OK;
}

}  // namespace sf

extern "C" int sf_linear_bf16(const void* x, int64_t rows, int64_t in_features, const void* weight,
                              int64_t out_features, void* out, void* stream) {
  using namespace sf;
  SF_CHECK_ARG(rows >= 0 && in_features > 0 && out_features > 0, "invalid sizes");
  if (rows == 0) return SF_OK;
  SF_CHECK_ARG(x && weight && out, "null pointer argument");
  if (rows > 128 || in_features % kBK != 0 || in_features >= (1LL << 31) ||
      out_features >= (1LL << 31) || !aligned16(x) || !aligned16(weight))
    return SF_ERR_UNSUPPORTED;  // no message: callers fall back to a library GEMM
  const int T = (int)rows, N = (int)out_features, K = (int)in_features;
  return launch_dense_any(x, weight, out, T, N, K, as_stream(stream), nullptr);
}

extern "C" size_t sf_linear_argmax_workspace_bytes(int64_t rows, int64_t in_features, int64_t out_features) {
  using namespace sf;
  if (rows <= 0 || out_features <= 0 || in_features <= 0) return 0;
  const int64_t m_tiles = (out_features + kBM - 1) / kBM;
  return (size_t)(m_tiles * kMaxSplit * rows) * sizeof(ArgmaxPart);
}

extern "C" int sf_linear_bf16_argmax(const void* x, int64_t rows, int64_t in_features, const void* weight,
                                     int64_t out_features, void* out, int64_t* argmax, void* workspace,
                                     size_t workspace_bytes, void* stream) {
  using namespace sf;
  SF_CHECK_ARG(rows >= 0 && in_features > 0 && out_features > 0, "invalid sizes");
  if (rows == 0) return SF_OK;
  SF_CHECK_ARG(x && weight && argmax && workspace, "null pointer argument");
  SF_CHECK_ARG(rows <= 128, "at most 128 rows");
  SF_CHECK_ARG(in_features % kBK == 0 && in_features < (1LL << 31) && out_features < (1LL << 31),
               "in_features must be a multiple of 64");
  SF_CHECK_ARG(aligned16(x) && aligned16(weight), "x and weight must be 16-byte aligned");
  if (workspace_bytes < sf_linear_argmax_workspace_bytes(rows, in_features, out_features))
    return set_error(SF_ERR_WORKSPACE, "argmax workspace needs %zu bytes",
                     sf_linear_argmax_workspace_bytes(rows, in_features, out_features));
  const int T = (int)rows, N = (int)out_features, K = (int)in_features;
  auto* part = static_cast<ArgmaxPart*>(workspace);
  cudaStream_t s = as_stream(stream);
  if (int rc = launch_dense_any(x, weight, out, T, N, K, s, part)) return rc;
  const int nparts = dense_argmax_parts(N, K);
  SF_CHECK_CUDA(launch_pdl(argmax_reduce_kernel, dim3((unsigned)((T + 7) / 8)), dim3(256), 0, s,
                           static_cast<const ArgmaxPart*>(part), nparts, T, argmax));
  SF_CHECK_LAUNCH();
  return SF_OK;
}
