// K3 (tensor cores): grouped SwiGLU on tcgen05/TMEM, operands staged by TMA.
//
// Same contract as the CUDA-core path (see swiglu_simt.cu), which restates
// _expert_forward (src/specfit/runtime/qwen3_offloaded_experts.py:38-62) and
// the weighting mul_ (:132-138, :198), for bf16 models with H % 128 == 0 and
// I % 64 == 0 (Qwen3-30B-A3B: H = 2048, I = 768).
//
// Layout ("swap AB"): at verification sizes an expert sees a handful of rows
// (m_e ~ T*K/E), far below a 128-row MMA tile, so the WEIGHT rows fill the
// MMA's M dimension and the expert's token rows form N (16..128 per pass):
//   phase 1: D[128 weight rows, N tokens] = W_gate|up[rows, H] . X_e[N, H]^T
//   phase 2: D[128 hidden rows, N tokens] = W_down[rows, I]   . Act_e[N, I]^T
// Both operands are K-major, loaded by TMA with 128-byte swizzling.  A phase-1
// tile holds 64 gate rows and the 64 matching up rows, so SiLU(gate)*up is
// fused into its epilogue.  The routing weight is fused into phase 2's.
//
// Each launch is persistent (one CTA per SM, 192 threads):
//   warp 0      TMA producer (one lane), 6-stage shared-memory ring
//   warp 1      TMEM allocator and MMA issuer (one lane)
//   warps 2..5  epilogue: TMEM -> registers -> rounding -> global stores
// Two TMEM accumulators (128 columns each) let the epilogue of one tile
// overlap the MMAs of the next.  At these sizes the kernel streams expert
// weights: a weight tile is read once per pass of up to 128 token rows, and
// an expert with more rows (a hot expert under skewed routes) has its passes
// on neighbouring CTAs at about the same time, so the repeats hit L2.
//
// Every TMA load here is issued by one CTA for its own shared memory.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "sm100_ptx.cuh"
#include "swiglu.h"

namespace sf {

namespace {

// Sticky device-side status of this file's kernels: 0, or the site code of
// the first barrier wait that gave up (1..6).
__device__ int g_swiglu_status;

constexpr int kBM = 128;       // MMA M: weight rows per tile
constexpr int kBK = 64;        // K elements per stage (one 128-byte swizzle atom)
constexpr int kBN = 128;       // max token rows per pass (MMA N)
constexpr int kStages = 6;
constexpr int kABytes = kBM * kBK * 2;
constexpr int kBBytes = kBN * kBK * 2;
constexpr int kBBox = 16;      // token rows per B TMA box
constexpr int kBWide = 64;     // token rows per wide B box (passes of more than kWideMin rows)
constexpr int kWideMin = 48;
constexpr int kThreads = 192;
constexpr int kTmemCols = 2 * kBN;
constexpr int kUpPitch = 17;   // padded row pitch of the gate/up exchange buffer
constexpr int kMaxExperts = 1024;  // experts per launch (the unit table lives in shared memory)

struct __align__(8) SmemTail {
  float upbuf[64 * kUpPitch];
  int rowtok[kBN];  // gathered variant: token row of each row of the current pass
  float w_sm[kBN];        // phase 2: routing weight of each row of the unit's pass
  uint64_t dst_sm[kBN];   // phase 2, fused return: destination of each row of the pass
  int unit_first[kMaxExperts + 1];  // number of the first unit of active[a]; [n_active] = all units
  int unit_expert[kMaxExperts];     // active[a]
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort_flag;
  int epi_go;
};

constexpr size_t kSmemBytes = 1024 /*alignment slack*/ + (size_t)kStages * (kABytes + kBBytes) +
                              sizeof(SmemTail);

// Work unit = (tile, pass).  A tile is one expert x one block of 128 weight
// rows; a pass is up to kBN of that expert's token rows.
struct Unit {
  int e, slot, m_tile, n0, npass;
};

template <int kPhase>
struct TileSpace {
  int m_tiles;  // weight-row tiles per expert
  int k_blocks;
  __device__ TileSpace(int H, int I) {
    m_tiles = (kPhase == 1) ? I / 64 : H / kBM;
    k_blocks = (kPhase == 1) ? H / kBK : I / kBK;
  }
};

__device__ __forceinline__ float bf16r(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// Numbers the units in shared memory, once per CTA: expert by expert
// (active-list order), inside an expert weight tile by weight tile with the
// passes of a tile adjacent.  Returns the number of units.
__device__ __forceinline__ int number_units(SmemTail* tail, int m_tiles, const int32_t* offsets,
                                            const int32_t* active, int n_active) {
  for (int a = threadIdx.x; a < n_active; a += blockDim.x) {
    const int e = active[a];
    tail->unit_expert[a] = e;
    tail->unit_first[a + 1] = (offsets[e + 1] - offsets[e] + kBN - 1) / kBN * m_tiles;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    // Exclusive scan: lane l sums a contiguous chunk, the chunk totals are
    // scanned with shuffles, then each lane writes its chunk's prefix.
    const int lane = threadIdx.x;
    const int per = (n_active + 31) / 32;
    const int lo = min(n_active, lane * per), hi = min(n_active, lo + per);
    int sum = 0;
    for (int a = lo; a < hi; ++a) sum += tail->unit_first[a + 1];
    int incl = sum;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += v;
    }
    int run = incl - sum;
    for (int a = lo; a < hi; ++a) {
      run += tail->unit_first[a + 1];
      tail->unit_first[a + 1] = run;
    }
    if (lane == 0) tail->unit_first[0] = 0;
  }
  __syncthreads();
  return tail->unit_first[n_active];
}

// Iterates this CTA's units in a fixed order; every role walks the same list.
// CTA b takes units b, b + G, b + 2G, ... (G working CTAs).  Dealing out units rather than
// whole tiles keeps the CTAs within one unit of each other when a few hot
// experts need several passes (skewed routes), and the passes of one tile
// run on neighbouring CTAs at about the same time, so the tile's repeated
// weight reads are served by L2.
// `ctas`: the CTAs that take units (see balanced_ctas).
template <typename F>
__device__ __forceinline__ void for_each_unit(const SmemTail* tail, int m_tiles, int n_active, int units,
                                              int ctas, const int32_t* offsets, const int32_t* expert_slot,
                                              F&& f) {
  int a = 0;
  for (int u = blockIdx.x; u < units; u += ctas) {
    while (tail->unit_first[a + 1] <= u) ++a;
    const int e = tail->unit_expert[a];
    const int base = tail->unit_first[a];
    const int passes = (tail->unit_first[a + 1] - base) / m_tiles;
    const int local = u - base;
    const int r0 = offsets[e], r1 = offsets[e + 1];
    const int n0 = r0 + (local % passes) * kBN;
    Unit unit{e, expert_slot[e], local / passes, n0, min(kBN, r1 - n0)};
    if (!f(unit)) return;
  }
}

// kGather (the gathered variant): phase 1 reads each pass's token rows
// straight from the unsorted hidden states [T, H] with TMA gather4 (row of
// sorted row r = sorted_pos[r] / top_k) instead of from a gathered copy, and
// phase 2 reads the routing weight of row r as topk_w[sorted_pos[r]].  The
// staged tiles, and so every result, are the same as with the copy.
// The CTAs that take units: as few as still finish in the same number of
// rounds (ceil(units / grid)), so every working CTA takes that many units or
// one fewer instead of a few CTAs taking one more than the rest; the SMs
// left idle give their share of HBM bandwidth to the others (a weight
// stream is bound by the device's bandwidth, not by one SM's).
__device__ __forceinline__ int balanced_ctas(int units) {
  const int g = (int)gridDim.x;
  const int rounds = (units + g - 1) / g;
  return rounds > 0 ? (units + rounds - 1) / rounds : g;
}

// The last CTA of a fused-return launch signals every rank (SwigluPeerOut).
__device__ __forceinline__ void peer_out_arrive(const SwigluPeerOut& p) {
  __threadfence_system();  // this CTA's row stores, before its ticket
  const unsigned int t = atomicAdd(p.ticket, 1u);
  if (t == gridDim.x - 1) {
    *p.ticket = 0u;
    __threadfence_system();  // every CTA's ticket (and so its stores), before the arrivals
    for (int r = 0; r < p.world; ++r)
      atomicAdd_system(reinterpret_cast<unsigned long long*>(p.peers[r] + p.arrive_off) + p.me, p.per_epoch);
  }
}

template <int kPhase, bool kGather = false, bool kPeerOut = false>
__global__ void __launch_bounds__(kThreads, 1)
swiglu_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
                 const __grid_constant__ CUtensorMap tm_xw, const int32_t* __restrict__ offsets, const int32_t* __restrict__ active,
                 const int32_t* __restrict__ num_active, const int32_t* __restrict__ expert_slot,
                 const float* __restrict__ w_sorted, int H, int I,
                 __nv_bfloat16* __restrict__ out, const int32_t* __restrict__ sorted_pos = nullptr,
                 int top_k = 1, const float* __restrict__ topk_w = nullptr, SwigluPeerOut peer = {}) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* a_stage = smem;
  uint8_t* b_stage = smem + (size_t)kStages * kABytes;
  SmemTail* tail = reinterpret_cast<SmemTail*>(b_stage + (size_t)kStages * kBBytes);
  volatile int* abort_flag = &tail->abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const TileSpace<kPhase> space(H, I);
  const int n_active = min(*num_active, kMaxExperts);
  // A CTA with no unit (an empty wave of a device-managed cache, or a grid
  // larger than the work) leaves before touching barriers or TMEM.
  if (n_active <= 0) {
    if constexpr (kPeerOut) {
      if (threadIdx.x == 0) peer_out_arrive(peer);
    }
    return;
  }
  const int units = number_units(tail, space.m_tiles, offsets, active, n_active);
  const int ctas = balanced_ctas(units);
  if ((int)blockIdx.x >= ctas) {
    if constexpr (kPeerOut) {
      if (threadIdx.x == 0) peer_out_arrive(peer);
    }
    return;
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      ptx::mbar_init(&tail->full[s], 1);
      ptx::mbar_init(&tail->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(&tail->acc_full[b], 1);
      ptx::mbar_init(&tail->acc_empty[b], 128);
    }
    ptx::mbar_init(&tail->mma_done, 1);
    tail->abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tensormap(&tm_w);
    ptx::prefetch_tensormap(&tm_x);
  }
  if (warp == 1) {
    ptx::tmem_alloc(&tail->tmem_base, kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = tail->tmem_base;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      uint32_t it = 0;
      for_each_unit(tail, space.m_tiles, n_active, units, ctas, offsets, expert_slot, [&](const Unit& u) {
        const int nb = (u.npass + kBBox - 1) / kBBox;
        // A pass of many rows takes its token rows in one or two wide boxes
        // (fewer TMA requests per stage); rows past the pass are loaded but
        // never stored.
        const bool wide = !kGather && u.npass > kWideMin;
        const int nw = (u.npass + kBWide - 1) / kBWide;
        const uint32_t bytes = kABytes + (wide ? nw * kBWide : nb * kBBox) * kBK * 2;
        if constexpr (kGather && kPhase == 1) {
          // Token rows of this pass; rows past it read token 0 (their
          // products are never stored).
#pragma unroll 8
          for (int i = 0; i < nb * kBBox; ++i)
            tail->rowtok[i] = i < u.npass ? sorted_pos[u.n0 + i] / top_k : 0;
        }
        for (int kb = 0; kb < space.k_blocks; ++kb, ++it) {
          const int s = it % kStages;
          const uint32_t ph = (it / kStages) & 1;
          if (!ptx::mbar_wait(&tail->empty[s], ph ^ 1, abort_flag, &g_swiglu_status, 1)) return false;
          ptx::mbar_arrive_expect_tx(&tail->full[s], bytes);
          uint8_t* a = a_stage + (size_t)s * kABytes;
          if (kPhase == 1) {
            const int g0 = u.m_tile * 64;
            ptx::tma_load_3d(a, &tm_w, &tail->full[s], kb * kBK, g0, u.slot);
            ptx::tma_load_3d(a + kABytes / 2, &tm_w, &tail->full[s], kb * kBK, I + g0, u.slot);
          } else {
            ptx::tma_load_3d(a, &tm_w, &tail->full[s], kb * kBK, u.m_tile * kBM, u.slot);
          }
          uint8_t* b = b_stage + (size_t)s * kBBytes;
          if constexpr (kGather && kPhase == 1) {
            for (int g = 0; g < nb * (kBBox / 4); ++g) {
              const int* t = &tail->rowtok[g * 4];
              ptx::tma_gather4(b + g * 4 * kBK * 2, &tm_x, &tail->full[s], kb * kBK, t[0], t[1], t[2], t[3]);
            }
          } else if (wide) {
            for (int q = 0; q < nw; ++q)
              ptx::tma_load_2d(b + q * kBWide * kBK * 2, &tm_xw, &tail->full[s], kb * kBK,
                               u.n0 + q * kBWide);
          } else {
            for (int q = 0; q < nb; ++q)
              ptx::tma_load_2d(b + q * kBBox * kBK * 2, &tm_x, &tail->full[s], kb * kBK,
                               u.n0 + q * kBBox);
          }
        }
        return true;
      });
      // Let every load this thread issued land before the CTA can exit.
      volatile int never = 0;
      for (uint32_t i = (it > (uint32_t)kStages ? it - kStages : 0u); i < it; ++i)
        ptx::mbar_wait(&tail->full[i % kStages], (i / kStages) & 1, &never, &g_swiglu_status, 2);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      uint32_t it = 0, unit = 0;
      for_each_unit(tail, space.m_tiles, n_active, units, ctas, offsets, expert_slot, [&](const Unit& u) {
        const int buf = unit & 1;
        const uint32_t aph = (unit >> 1) & 1;
        if (!ptx::mbar_wait(&tail->acc_empty[buf], aph ^ 1, abort_flag, &g_swiglu_status, 3)) return false;
        ptx::tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * kBN;
        const uint32_t npad = (u.npass + 15) & ~15;
        const uint32_t idesc = ptx::idesc_bf16_f32(kBM, npad);
        for (int kb = 0; kb < space.k_blocks; ++kb, ++it) {
          const int s = it % kStages;
          const uint32_t ph = (it / kStages) & 1;
          if (!ptx::mbar_wait(&tail->full[s], ph, abort_flag, &g_swiglu_status, 4)) return false;
          ptx::tc_fence_after();
          const uint64_t adesc = ptx::smem_desc_k_sw128(ptx::smem_u32(a_stage + (size_t)s * kABytes));
          const uint64_t bdesc = ptx::smem_desc_k_sw128(ptx::smem_u32(b_stage + (size_t)s * kBBytes));
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k) {
            // +32 bytes per K=16 step inside the 128-byte swizzle atom.
            ptx::umma_f16(d_tmem, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), idesc,
                          (kb | k) != 0);
          }
          ptx::umma_commit(&tail->empty[s]);
        }
        ptx::umma_commit(&tail->acc_full[buf]);
        ++unit;
        return true;
      });
      // Drain: the barrier fires once every MMA issued above has completed.
      ptx::umma_commit(&tail->mma_done);
      volatile int never = 0;
      ptx::mbar_wait(&tail->mma_done, 0, &never, &g_swiglu_status, 5);
    }
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int quad = warp & 3;             // TMEM lane quadrant this warp may read
    const int row = quad * 32 + lane;      // accumulator row = TMEM lane
    uint32_t unit = 0;
    for_each_unit(tail, space.m_tiles, n_active, units, ctas, offsets, expert_slot, [&](const Unit& u) {
      const int buf = unit & 1;
      const uint32_t aph = (unit >> 1) & 1;
      ptx::mbar_wait(&tail->acc_full[buf], aph, abort_flag, &g_swiglu_status, 6);
      // The four epilogue warps take one consistent go/stop decision before
      // any of them enters the per-chunk named barriers below.
      ptx::named_bar_sync(2, 128);
      if (threadIdx.x == 64) tail->epi_go = !*abort_flag;
      ptx::named_bar_sync(2, 128);
      if (!tail->epi_go) return false;
      ptx::tc_fence_after();
      const int chunks = (u.npass + 15) / 16;
      const uint32_t tbase = tmem_base + ((uint32_t)(quad * 32) << 16) + buf * kBN;
      if constexpr (kPhase == 2) {
        // The pass's routing weights (and return destinations) once per
        // unit, instead of one global load per row by every thread.
        if (row < u.npass) {
          const int r = u.n0 + row;
          tail->w_sm[row] = kGather ? topk_w[sorted_pos[r]] : w_sorted[r];
          if constexpr (kPeerOut) tail->dst_sm[row] = peer.dst_row[r];
        }
        ptx::named_bar_sync(1, 128);
      }
      for (int c = 0; c < chunks; ++c) {
        float v[16];
        ptx::tmem_ld_16(tbase + c * 16, v);
        if (kPhase == 1) {
          // Rows 0..63 hold gate rows g0.., rows 64..127 the matching up rows.
          if (row >= 64) {
#pragma unroll
            for (int i = 0; i < 16; ++i) tail->upbuf[(row - 64) * kUpPitch + i] = v[i];
          }
          ptx::named_bar_sync(1, 128);
          if (row < 64) {
            const int col = u.m_tile * 64 + row;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int j = c * 16 + i;
              if (j < u.npass) {
                const float g = bf16r(v[i]);
                const float up = bf16r(tail->upbuf[row * kUpPitch + i]);
                const float act = bf16r(bf16r(silu_f32(g)) * up);
                out[(int64_t)(u.n0 + j) * I + col] = __float2bfloat16_rn(act);
              }
            }
          }
          ptx::named_bar_sync(1, 128);
        } else if constexpr (kPeerOut) {
          // Straight into the source ranks' return rows (over NVLink for a
          // peer), 16 bytes at a time: the warp's 32 columns x 16 rows go
          // through shared memory (the gate/up buffer, idle in phase 2) so
          // each lane stores whole 8-column pieces of a row.
          __nv_bfloat16* stage = reinterpret_cast<__nv_bfloat16*>(tail->upbuf) + quad * (16 * 32);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int j = c * 16 + i;
            const float w = j < u.npass ? tail->w_sm[j] : 0.f;
            stage[i * 32 + lane] = __float2bfloat16_rn(bf16r(v[i]) * w);
          }
          __syncwarp();
          const int col0 = u.m_tile * kBM + quad * 32;
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            const int piece = k * 32 + lane;  // 16 rows x 4 pieces of 8 columns
            const int i = piece >> 2, q = piece & 3;
            const int j = c * 16 + i;
            const uint64_t dst = j < u.npass ? tail->dst_sm[j] : 0ull;
            if (dst)
              *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(dst) + col0 + q * 8) =
                  *reinterpret_cast<const uint4*>(stage + i * 32 + q * 8);
          }
          __syncwarp();
        } else {
          const int col = u.m_tile * kBM + row;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int j = c * 16 + i;
            if (j < u.npass) {
              const int r = u.n0 + j;
              const float y = bf16r(v[i]);
              const float w = tail->w_sm[j];
              out[(int64_t)r * H + col] = __float2bfloat16_rn(y * w);
            }
          }
        }
      }
      ptx::tc_fence_before();
      ptx::mbar_arrive(&tail->acc_empty[buf]);
      ++unit;
      return true;
    });
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, kTmemCols);
  }
  if constexpr (kPeerOut) {
    __syncthreads();  // every epilogue store of this CTA is issued
    if (threadIdx.x == 0) peer_out_arrive(peer);
  }
}

bool device_is_sm100() {
  static std::atomic<int> cache[64];  // 0 unknown, 1 yes, 2 no
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  int v = cache[dev & 63].load(std::memory_order_relaxed);
  if (v == 0) {
    int major = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return false;
    v = (major == 10) ? 1 : 2;
    cache[dev & 63].store(v, std::memory_order_relaxed);
  }
  return v == 1;
}

}  // namespace

// ---------------------------------------------------------------------------
// Host side: tensor maps.

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int tma_encode_bf16(CUtensorMap* map, const void* base, int rank, const cuuint64_t* dims,
                const cuuint64_t* strides_bytes, const cuuint32_t* box) {
  auto fn = encode_fn();
  if (!fn) return set_error(SF_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if (rank < 1 || rank > 5) return set_error(SF_ERR_INVALID_ARGUMENT, "tensor map rank %d", rank);
  cuuint32_t elem_strides[5] = {1, 1, 1, 1, 1};  // rank <= 5
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), dims,
                  strides_bytes, box, elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(SF_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return SF_OK;
}

bool swiglu_tcgen05_supports(const SwigluArgs& a) {
  return a.dtype == SF_DTYPE_BF16 && a.hidden % kBM == 0 && a.inter % 64 == 0 && a.hidden > 0 &&
         a.num_experts > 0 && a.num_experts <= kMaxExperts &&
         a.inter > 0 && a.slot_stride % 8 == 0 && a.slot_stride >= 3LL * a.hidden * a.inter &&
         a.slot_count > 0 && aligned16(a.slot_storage) && aligned16(a.hidden_sorted) &&
         aligned16(a.act_workspace) && a.rows < (1LL << 31) && a.slot_count < (1LL << 31);
}

namespace {

// Encodes the four tensor maps and launches both phases.  With `gather`
// (the gathered variant) a.hidden_sorted is the unsorted hidden [tokens, H]
// and phase 1 loads its rows one box row at a time with gather4.
int swiglu_tcgen05_launch(const SwigluArgs& a, const SwigluGather* gather, const SwigluPeerOut* peer,
                          cudaStream_t stream) {
  static std::atomic<unsigned long long> configured{0};
  if (int rc = once_per_device(configured, [] {
        int dev = 0, major = 0;
        SF_CHECK_CUDA(cudaGetDevice(&dev));
        SF_CHECK_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
        if (major != 10) return set_error(SF_ERR_UNSUPPORTED, "tcgen05 SwiGLU needs an sm_100 device");
        SF_CHECK_CUDA(cudaFuncSetAttribute(swiglu_tc_kernel<1>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes));
        SF_CHECK_CUDA(cudaFuncSetAttribute(swiglu_tc_kernel<2>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes));
        SF_CHECK_CUDA(cudaFuncSetAttribute(swiglu_tc_kernel<1, true>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes));
        SF_CHECK_CUDA(cudaFuncSetAttribute(swiglu_tc_kernel<2, true>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes));
        SF_CHECK_CUDA(cudaFuncSetAttribute(swiglu_tc_kernel<2, false, true>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes));
        return SF_OK;
      }))
    return rc;

  const int H = a.hidden, I = a.inter;
  const uint64_t slot_bytes = (uint64_t)a.slot_stride * 2;
  const __nv_bfloat16* storage = static_cast<const __nv_bfloat16*>(a.slot_storage);
  CUtensorMap tm_w1, tm_x1, tm_w2, tm_x2, tm_x1w, tm_x2w;
  {
    cuuint64_t dims[3] = {(cuuint64_t)H, (cuuint64_t)(2 * I), (cuuint64_t)a.slot_count};
    cuuint64_t strides[2] = {(cuuint64_t)H * 2, slot_bytes};
    cuuint32_t box[3] = {kBK, 64, 1};
    if (int rc = tma_encode_bf16(&tm_w1, storage, 3, dims, strides, box)) return rc;
  }
  {
    const int64_t x_rows = gather ? gather->tokens : a.rows;
    cuuint64_t dims[2] = {(cuuint64_t)H, (cuuint64_t)x_rows};
    cuuint64_t strides[1] = {(cuuint64_t)H * 2};
    cuuint32_t box[2] = {kBK, gather ? 1u : (cuuint32_t)kBBox};  // gather4 boxes are one row high
    if (int rc = tma_encode_bf16(&tm_x1, a.hidden_sorted, 2, dims, strides, box)) return rc;
    box[1] = gather ? 1u : (cuuint32_t)kBWide;
    if (int rc = tma_encode_bf16(&tm_x1w, a.hidden_sorted, 2, dims, strides, box)) return rc;
  }
  {
    cuuint64_t dims[3] = {(cuuint64_t)I, (cuuint64_t)H, (cuuint64_t)a.slot_count};
    cuuint64_t strides[2] = {(cuuint64_t)I * 2, slot_bytes};
    cuuint32_t box[3] = {kBK, kBM, 1};
    if (int rc = tma_encode_bf16(&tm_w2, storage + 2LL * I * H, 3, dims, strides, box)) return rc;
  }
  {
    cuuint64_t dims[2] = {(cuuint64_t)I, (cuuint64_t)a.rows};
    cuuint64_t strides[1] = {(cuuint64_t)I * 2};
    cuuint32_t box[2] = {kBK, kBBox};
    if (int rc = tma_encode_bf16(&tm_x2, a.act_workspace, 2, dims, strides, box)) return rc;
    box[1] = kBWide;
    if (int rc = tma_encode_bf16(&tm_x2w, a.act_workspace, 2, dims, strides, box)) return rc;
  }
  const int grid = num_sms();
  auto* act = static_cast<__nv_bfloat16*>(a.act_workspace);
  auto* out = static_cast<__nv_bfloat16*>(a.out_sorted);
  if (gather) {
    SF_CHECK_CUDA(launch_pdl(swiglu_tc_kernel<1, true>, dim3(grid), dim3(kThreads), kSmemBytes, stream,
                             tm_w1, tm_x1, tm_x1w, a.offsets, a.active, a.num_active, a.expert_slot,
                             a.weights_sorted, H, I, act, gather->sorted_pos, gather->top_k,
                             gather->topk_weights, SwigluPeerOut{}));
    SF_CHECK_LAUNCH();
    SF_CHECK_CUDA(launch_pdl(swiglu_tc_kernel<2, true>, dim3(grid), dim3(kThreads), kSmemBytes, stream,
                             tm_w2, tm_x2, tm_x2w, a.offsets, a.active, a.num_active, a.expert_slot,
                             a.weights_sorted, H, I, out, gather->sorted_pos, gather->top_k,
                             gather->topk_weights, SwigluPeerOut{}));
    SF_CHECK_LAUNCH();
    return SF_OK;
  }
  const int32_t* no_pos = nullptr;
  const float* no_w = nullptr;
  SF_CHECK_CUDA(launch_pdl(swiglu_tc_kernel<1>, dim3(grid), dim3(kThreads), kSmemBytes, stream,
                           tm_w1, tm_x1, tm_x1w, a.offsets, a.active, a.num_active, a.expert_slot,
                           a.weights_sorted, H, I, act, no_pos, 1, no_w, SwigluPeerOut{}));
  SF_CHECK_LAUNCH();
  if (peer) {
    SF_CHECK_CUDA(launch_pdl(swiglu_tc_kernel<2, false, true>, dim3(grid), dim3(kThreads), kSmemBytes, stream,
                             tm_w2, tm_x2, tm_x2w, a.offsets, a.active, a.num_active, a.expert_slot,
                             a.weights_sorted, H, I, out, no_pos, 1, no_w, *peer));
    SF_CHECK_LAUNCH();
    return SF_OK;
  }
  SF_CHECK_CUDA(launch_pdl(swiglu_tc_kernel<2>, dim3(grid), dim3(kThreads), kSmemBytes, stream,
                           tm_w2, tm_x2, tm_x2w, a.offsets, a.active, a.num_active, a.expert_slot,
                           a.weights_sorted, H, I, out, no_pos, 1, no_w, SwigluPeerOut{}));
  SF_CHECK_LAUNCH();
  return SF_OK;
}

}  // namespace

int swiglu_tcgen05(const SwigluArgs& a, cudaStream_t stream) {
  if (!swiglu_tcgen05_supports(a))
    return set_error(SF_ERR_UNSUPPORTED,
                     "tcgen05 SwiGLU needs bf16, H%%128==0, I%%64==0 and 16-byte aligned buffers");
  if (a.rows == 0) return SF_OK;
  return swiglu_tcgen05_launch(a, nullptr, nullptr, stream);
}

int swiglu_tcgen05_gathered(const SwigluArgs& a, const SwigluGather& g, cudaStream_t stream) {
  if (!swiglu_tcgen05_supports(a) || g.tokens <= 0 || g.tokens >= (1LL << 31) || g.top_k <= 0 ||
      !g.sorted_pos || !g.topk_weights || a.rows != g.tokens * g.top_k)
    return set_error(SF_ERR_UNSUPPORTED,
                     "gathered tcgen05 SwiGLU needs bf16, H%%128==0, I%%64==0, 16-byte aligned buffers "
                     "and rows == tokens * top_k");
  return swiglu_tcgen05_launch(a, &g, nullptr, stream);
}

int swiglu_tcgen05_peer(const SwigluArgs& a, const SwigluPeerOut& peer, cudaStream_t stream) {
  if (!swiglu_tcgen05_supports(a) || !device_is_sm100())
    return set_error(SF_ERR_UNSUPPORTED,
                     "the fused-return SwiGLU needs the tcgen05 kernel (bf16, H%%128==0, I%%64==0, aligned buffers)");
  return swiglu_tcgen05_launch(a, nullptr, &peer, stream);
}

int swiglu_status(int* status, int reset) {
  SF_CHECK_CUDA(cudaMemcpyFromSymbol(status, g_swiglu_status, sizeof(int)));
  if (reset) {
    const int zero = 0;
    SF_CHECK_CUDA(cudaMemcpyToSymbol(g_swiglu_status, &zero, sizeof(int)));
  }
  return SF_OK;
}

}  // namespace sf

extern "C" int sf_grouped_swiglu_ex(const void* hidden_sorted, const float* weights_sorted,
                                    int dtype, const int32_t* offsets, const int32_t* active,
                                    const int32_t* num_active, const int32_t* expert_slot,
                                    const void* slot_storage, int64_t slot_count,
                                    int64_t slot_stride_elems, int num_experts, int hidden_size,
                                    int intermediate_size, int64_t rows, void* act_workspace,
                                    void* out_sorted, int impl, void* stream) {
  using namespace sf;
  SF_CHECK_ARG(hidden_size > 0 && intermediate_size > 0 && num_experts > 0 && rows >= 0,
               "invalid sizes");
  SF_CHECK_ARG(slot_count > 0 && slot_stride_elems >= 3LL * hidden_size * intermediate_size,
               "slot_stride_elems must cover one packed expert");
  if (rows == 0) return SF_OK;
  SF_CHECK_ARG(hidden_sorted && weights_sorted && offsets && active && num_active &&
                   expert_slot && slot_storage && act_workspace && out_sorted,
               "null pointer argument");
  SwigluArgs a{hidden_sorted, weights_sorted, dtype,       offsets,         active,
               num_active,    expert_slot,    slot_storage, slot_count,     slot_stride_elems,
               num_experts,   hidden_size,    intermediate_size, rows,      act_workspace,
               out_sorted};
  cudaStream_t s = as_stream(stream);
  if (impl == SF_SWIGLU_SIMT) return swiglu_simt(a, s);
  if (impl == SF_SWIGLU_TCGEN05) return swiglu_tcgen05(a, s);
  SF_CHECK_ARG(impl == SF_SWIGLU_AUTO, "unknown implementation %d", impl);
  if (swiglu_tcgen05_supports(a) && device_is_sm100()) return swiglu_tcgen05(a, s);
  return swiglu_simt(a, s);
}

extern "C" int sf_grouped_swiglu_gathered(const void* hidden, int64_t tokens, const float* topk_weights,
                                          int top_k, const int32_t* sorted_pos, const int32_t* offsets,
                                          const int32_t* active, const int32_t* num_active,
                                          const int32_t* expert_slot, const void* slot_storage,
                                          int64_t slot_count, int64_t slot_stride_elems, int num_experts,
                                          int hidden_size, int intermediate_size, void* act_workspace,
                                          void* out_sorted, void* stream) {
  using namespace sf;
  SF_CHECK_ARG(hidden_size > 0 && intermediate_size > 0 && num_experts > 0 && tokens >= 0 && top_k > 0,
               "invalid sizes");
  SF_CHECK_ARG(slot_count > 0 && slot_stride_elems >= 3LL * hidden_size * intermediate_size,
               "slot_stride_elems must cover one packed expert");
  if (tokens == 0) return SF_OK;
  SF_CHECK_ARG(hidden && topk_weights && sorted_pos && offsets && active && num_active && expert_slot &&
                   slot_storage && act_workspace && out_sorted,
               "null pointer argument");
  SwigluArgs a{hidden,        nullptr,        SF_DTYPE_BF16,  offsets,           active,
               num_active,    expert_slot,    slot_storage,   slot_count,        slot_stride_elems,
               num_experts,   hidden_size,    intermediate_size, tokens * top_k, act_workspace,
               out_sorted};
  SwigluGather g{tokens, top_k, sorted_pos, topk_weights};
  if (!swiglu_tcgen05_supports(a) || !device_is_sm100())
    return SF_ERR_UNSUPPORTED;  // the caller gathers and calls sf_grouped_swiglu
  return swiglu_tcgen05_gathered(a, g, as_stream(stream));
}

extern "C" int sf_grouped_swiglu(const void* hidden_sorted, const float* weights_sorted, int dtype,
                                 const int32_t* offsets, const int32_t* active,
                                 const int32_t* num_active, const int32_t* expert_slot,
                                 const void* slot_storage, int64_t slot_count,
                                 int64_t slot_stride_elems, int num_experts, int hidden_size,
                                 int intermediate_size, int64_t rows, void* act_workspace,
                                 void* out_sorted, void* stream) {
  return sf_grouped_swiglu_ex(hidden_sorted, weights_sorted, dtype, offsets, active, num_active,
                              expert_slot, slot_storage, slot_count, slot_stride_elems,
                              num_experts, hidden_size, intermediate_size, rows, act_workspace,
                              out_sorted, SF_SWIGLU_AUTO, stream);
}
