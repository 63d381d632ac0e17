// Device-resident expert directory: the slot bookkeeping of one layer's
// expert cache kept in HBM, so a verify pass with cache misses runs with no
// host round trip (and can be captured in one CUDA graph).
//
// The host path (GpuExpertCache + Qwen3OffloadedExperts._forward_waves, after
// src/specfit/runtime/qwen3_offloaded_experts.py:98-164 and
// gpu_expert_cache.py:224-718) learns the layer's experts by a device-to-host
// copy, leases them in execution order a wave at a time (a wave ends when
// every slot is leased), submits each miss to the copy engine, runs the
// wave's grouped SwiGLU and releases the leases.  Here the same decisions are
// taken on the device, in the same order, so slots, generations, LRU clock and
// counters end up exactly as the host path would leave them:
//
//   sf_dir_plan   one CTA: orders the dispatch's active experts (ascending,
//                 or resident ones first), then per wave ranks the slots by
//                 the LRU key (occupied, last use, slot id) in parallel and
//                 walks the experts — a resident expert's slot is leased and
//                 touched, a missing one takes the next unleased slot of the
//                 ranking (evicting its expert), gets a new generation and a
//                 fill record, and is touched; the wave's leases are then
//                 released (touched) in wave order.  Output per wave: the
//                 expert->slot table and active list the grouped SwiGLU
//                 reads, and the wave's fill list.
//   sf_dir_fill   copies one wave's missing experts from page-locked host
//                 memory into their slots with SM loads over PCIe (the host
//                 pages are device-mapped), 64 bytes in flight per thread.
//
// Between waves the stream order keeps a fill behind the SwiGLU that read
// the slot before.  The directory is only valid while the owning cache is in
// device-managed mode; the host manager adopts its state when that ends.
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace sf {
namespace {

struct PlanArgs {
  int32_t* slot_expert;  // [S]
  int32_t* slot_gen;     // [S]
  int64_t* slot_stamp;   // [S]
  int32_t* expert_slot;  // [E]
  int64_t* clock;        // [1] LRU clock (last sequence number handed out)
  int64_t* counters;     // [4] h2d submissions, resident hits, in-flight joins, evictions
  const int32_t* active;      // [E] dispatch order (ascending ids)
  const int32_t* num_active;  // [1]
  int32_t* wave_table;   // [W][E] expert -> slot of the wave, -1 elsewhere
  int32_t* wave_active;  // [W][E]
  int32_t* wave_count;   // [W]
  int32_t* fill_expert;  // [W][S]
  int32_t* fill_slot;    // [W][S]
  int32_t* fill_count;   // [W]
  int32_t* status;       // [1] set to 1 if the experts did not fit W waves
  int E, S, W, resident_first;
  // Conditional handle of a captured graph (0: none): set to whether any
  // wave after the first has experts, so the graph runs those waves only then.
  unsigned long long later_waves;
};

__global__ void __launch_bounds__(1024) dir_plan_kernel(PlanArgs a) {
  pdl_wait();
  pdl_trigger();
  // Everything the sequential walk reads or writes lives in shared memory
  // (the wave's outputs are staged there and copied out by all threads), so
  // the one walking thread never waits on global memory.
  extern __shared__ __align__(16) uint8_t smem[];
  const int E = a.E, S = a.S;
  int64_t* stamp = reinterpret_cast<int64_t*>(smem);
  int32_t* sexp = reinterpret_cast<int32_t*>(stamp + S);
  int32_t* sgen = sexp + S;
  int32_t* perm = sgen + S;
  int32_t* fe_sm = perm + S;
  int32_t* fs_sm = fe_sm + S;
  int32_t* eslot = fs_sm + S;
  int32_t* order = eslot + E;
  int32_t* act_in = order + E;
  int32_t* table_sm = act_in + E;
  uint8_t* leased = reinterpret_cast<uint8_t*>(table_sm + E);
  __shared__ int n_sh, pos_sh, w_sh, bad_sh, cnt_sh, nf_sh, start_sh, cnt0_sh;
  const int tid = threadIdx.x, nt = blockDim.x;

  if (tid == 0) {
    const int n = *a.num_active;
    n_sh = n < 0 ? 0 : (n > E ? E : n);
    pos_sh = 0;
    w_sh = 0;
    bad_sh = 0;
  }
  for (int i = tid; i < S; i += nt) {
    stamp[i] = a.slot_stamp[i];
    sexp[i] = a.slot_expert[i];
    sgen[i] = a.slot_gen[i];
  }
  for (int i = tid; i < E; i += nt) {
    eslot[i] = a.expert_slot[i];
    act_in[i] = a.active[i];
  }
  for (int i = tid; i < a.W; i += nt) {
    a.wave_count[i] = 0;
    a.fill_count[i] = 0;
  }
  __syncthreads();
  if (tid == 0) {
    const int n = n_sh;
    int k = 0;
    for (int i = 0; i < n; ++i) {  // ids outside [0, E) are dropped and flagged
      const int e = act_in[i];
      if (e < 0 || e >= E) {
        bad_sh = 1;
        continue;
      }
      if (!a.resident_first || eslot[e] >= 0) order[k++] = e;
    }
    if (a.resident_first)
      for (int i = 0; i < n; ++i) {
        const int e = act_in[i];
        if (e >= 0 && e < E && eslot[e] < 0) order[k++] = e;
      }
    n_sh = k;
  }
  int64_t clock = 0, h2d = 0, hits = 0, evictions = 0;
  if (tid == 0) clock = *a.clock;
  __syncthreads();  // n_sh is final
  for (int w = 0; w < a.W; ++w) {
    if (pos_sh >= n_sh && w > 0) {
      // Every expert has its wave: the rest stay empty (counts are 0 from the
      // start); their tables are still written (-1) so a stale wave can never
      // be read.
      int32_t* table = a.wave_table + (size_t)w * E;
      for (int i = tid; i < E; i += nt) table[i] = -1;
      continue;
    }
    // Rank every slot by its LRU key; nothing is leased at a wave's start.
    for (int s = tid; s < S; s += nt) {
      const int occ = sexp[s] >= 0;
      const int64_t st = stamp[s];
      int r = 0;
      for (int t = 0; t < S; ++t) {
        const int ot = sexp[t] >= 0;
        r += ot < occ || (ot == occ && (stamp[t] < st || (stamp[t] == st && t < s)));
      }
      perm[r] = s;
      leased[s] = 0;
    }
    for (int i = tid; i < E; i += nt) table_sm[i] = -1;
    __syncthreads();
    if (tid == 0) {
      int q = 0, cnt = 0, nf = 0, pos = pos_sh;
      const int start = pos;
      for (; pos < n_sh; ++pos) {
        const int e = order[pos];
        int s = eslot[e];
        if (s >= 0) {
          ++hits;
        } else {
          while (q < S && leased[perm[q]]) ++q;
          if (q == S) break;  // every slot is leased: the wave is full
          s = perm[q++];
          const int old = sexp[s];
          if (old >= 0) {
            eslot[old] = -1;
            ++evictions;
          }
          sgen[s] += 1;
          sexp[s] = e;
          eslot[e] = s;
          ++h2d;
          fe_sm[nf] = e;
          fs_sm[nf] = s;
          ++nf;
        }
        leased[s] = 1;
        stamp[s] = ++clock;  // acquire touches the slot
        table_sm[e] = s;
        ++cnt;
      }
      for (int j = start; j < start + cnt; ++j) stamp[eslot[order[j]]] = ++clock;  // release, in wave order
      start_sh = start;
      cnt_sh = cnt;
      nf_sh = nf;
      pos_sh = pos;
      if (w == 0) cnt0_sh = cnt;
    }
    __syncthreads();
    // The wave's outputs, written by every thread.
    const int start = start_sh, cnt = cnt_sh, nf = nf_sh;
    int32_t* table = a.wave_table + (size_t)w * E;
    for (int i = tid; i < E; i += nt) table[i] = table_sm[i];
    for (int i = tid; i < cnt; i += nt) a.wave_active[(size_t)w * E + i] = order[start + i];
    for (int i = tid; i < nf; i += nt) {
      a.fill_expert[(size_t)w * S + i] = fe_sm[i];
      a.fill_slot[(size_t)w * S + i] = fs_sm[i];
    }
    if (tid == 0) {
      a.wave_count[w] = cnt;
      a.fill_count[w] = nf;
    }
  }
  __syncthreads();
  for (int i = tid; i < S; i += nt) {
    a.slot_stamp[i] = stamp[i];
    a.slot_expert[i] = sexp[i];
    a.slot_gen[i] = sgen[i];
  }
  for (int i = tid; i < E; i += nt) a.expert_slot[i] = eslot[i];
  if (tid == 0) {
    *a.clock = clock;
    a.counters[0] += h2d;
    a.counters[1] += hits;
    a.counters[3] += evictions;
    if (bad_sh) *a.status = 2;
    else if (pos_sh < n_sh) *a.status = 1;
    // Wave 0 holds at most S experts; the later waves have work iff it could
    // not take them all.
    if (a.later_waves != 0ull) cudaGraphSetConditional(a.later_waves, n_sh > cnt0_sh ? 1u : 0u);
  }
}

__global__ void __launch_bounds__(256) dir_fill_kernel(const uint64_t* __restrict__ src, uint8_t* storage,
                                                       int64_t slot_stride, int32_t units,
                                                       const int32_t* __restrict__ fill_expert,
                                                       const int32_t* __restrict__ fill_slot,
                                                       const int32_t* __restrict__ fill_count, int S) {
  pdl_wait();
  pdl_trigger();
  int n = *fill_count;
  n = n > S ? S : n;
  if (n <= 0) return;
  const int32_t total = n * units;
  const int32_t stride = (int32_t)(gridDim.x * blockDim.x);
  for (int32_t u0 = (int32_t)(blockIdx.x * blockDim.x + threadIdx.x); u0 < total; u0 += 4 * stride) {
    uint4 v[4];
    uint4* dst[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int32_t u = u0 + k * stride;
      dst[k] = nullptr;
      if (u < total) {
        const int32_t j = u / units, off = u - j * units;
        v[k] = reinterpret_cast<const uint4*>(src[fill_expert[j]])[off];
        dst[k] = reinterpret_cast<uint4*>(storage + (int64_t)fill_slot[j] * slot_stride) + off;
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k)
      if (dst[k]) *dst[k] = v[k];
  }
}

}  // namespace
}  // namespace sf

extern "C" int sf_dir_plan_ex(void* slot_expert, void* slot_gen, void* slot_stamp, void* expert_slot,
                              void* clock, void* counters, const void* active, const void* num_active,
                              int num_experts, int num_slots, int waves, int resident_first,
                              void* wave_table, void* wave_active, void* wave_count, void* fill_expert,
                              void* fill_slot, void* fill_count, void* status, uint64_t later_waves,
                              void* stream) {
  using namespace sf;
  SF_CHECK_ARG(num_experts > 0 && num_experts <= 4096, "num_experts must be in [1, 4096]");
  SF_CHECK_ARG(num_slots > 0 && num_slots <= 4096, "num_slots must be in [1, 4096]");
  SF_CHECK_ARG(waves >= (num_experts + num_slots - 1) / num_slots,
               "waves must cover every expert (at least ceil(E / S))");
  SF_CHECK_ARG(slot_expert && slot_gen && slot_stamp && expert_slot && clock && counters && active &&
                   num_active && wave_table && wave_active && wave_count && fill_expert && fill_slot &&
                   fill_count && status,
               "null pointer argument");
  PlanArgs a;
  a.slot_expert = static_cast<int32_t*>(slot_expert);
  a.slot_gen = static_cast<int32_t*>(slot_gen);
  a.slot_stamp = static_cast<int64_t*>(slot_stamp);
  a.expert_slot = static_cast<int32_t*>(expert_slot);
  a.clock = static_cast<int64_t*>(clock);
  a.counters = static_cast<int64_t*>(counters);
  a.active = static_cast<const int32_t*>(active);
  a.num_active = static_cast<const int32_t*>(num_active);
  a.wave_table = static_cast<int32_t*>(wave_table);
  a.wave_active = static_cast<int32_t*>(wave_active);
  a.wave_count = static_cast<int32_t*>(wave_count);
  a.fill_expert = static_cast<int32_t*>(fill_expert);
  a.fill_slot = static_cast<int32_t*>(fill_slot);
  a.fill_count = static_cast<int32_t*>(fill_count);
  a.status = static_cast<int32_t*>(status);
  a.E = num_experts;
  a.S = num_slots;
  a.W = waves;
  a.resident_first = resident_first;
  a.later_waves = later_waves;
  const size_t smem = (size_t)num_slots * (8 + 4 * 5 + 1) + (size_t)num_experts * 16;
  SF_CHECK_ARG(smem <= 160 * 1024, "directory too large for one CTA");
  if (smem > 48 * 1024)
    SF_CHECK_CUDA(cudaFuncSetAttribute(dir_plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int threads = ((num_slots + 31) / 32) * 32;  // one thread per slot for the ranking
  threads = threads < 128 ? 128 : (threads > 1024 ? 1024 : threads);
  SF_CHECK_CUDA(launch_pdl(dir_plan_kernel, dim3(1), dim3(threads), smem, as_stream(stream), a));
  SF_CHECK_LAUNCH();
  return SF_OK;
}

extern "C" int sf_dir_plan(void* slot_expert, void* slot_gen, void* slot_stamp, void* expert_slot,
                           void* clock, void* counters, const void* active, const void* num_active,
                           int num_experts, int num_slots, int waves, int resident_first,
                           void* wave_table, void* wave_active, void* wave_count, void* fill_expert,
                           void* fill_slot, void* fill_count, void* status, void* stream) {
  return sf_dir_plan_ex(slot_expert, slot_gen, slot_stamp, expert_slot, clock, counters, active, num_active,
                        num_experts, num_slots, waves, resident_first, wave_table, wave_active, wave_count,
                        fill_expert, fill_slot, fill_count, status, 0, stream);
}

extern "C" int sf_dir_fill(const void* expert_src, void* storage, int64_t slot_stride_bytes, int64_t expert_bytes,
                           const void* fill_expert, const void* fill_slot, const void* fill_count, int num_slots,
                           int grid, void* stream) {
  using namespace sf;
  SF_CHECK_ARG(expert_src && storage && fill_expert && fill_slot && fill_count, "null pointer argument");
  SF_CHECK_ARG(expert_bytes > 0 && expert_bytes % 16 == 0 && slot_stride_bytes % 16 == 0 &&
                   expert_bytes <= slot_stride_bytes,
               "expert bytes and slot stride must be positive multiples of 16");
  SF_CHECK_ARG(aligned16(storage), "slot storage must be 16-byte aligned");
  SF_CHECK_ARG(grid > 0 && grid <= 65535, "grid must be in [1, 65535]");
  SF_CHECK_ARG(num_slots > 0 &&
                   (int64_t)num_slots * (expert_bytes / 16) + 4LL * grid * 256 < (int64_t(1) << 31),
               "fill too large for 32-bit unit indexing");
  SF_CHECK_CUDA(launch_pdl(dir_fill_kernel, dim3(grid), dim3(256), 0, as_stream(stream),
                           static_cast<const uint64_t*>(expert_src), static_cast<uint8_t*>(storage),
                           slot_stride_bytes, (int32_t)(expert_bytes / 16),
                           static_cast<const int32_t*>(fill_expert), static_cast<const int32_t*>(fill_slot),
                           static_cast<const int32_t*>(fill_count), num_slots));
  SF_CHECK_LAUNCH();
  return SF_OK;
}

// Device address of page-locked host memory (0 when it is not device-mapped):
// the fill kernel reads expert sources through these addresses.
extern "C" int sf_host_device_address(const void* host, uint64_t* device_address) {
  using namespace sf;
  SF_CHECK_ARG(host && device_address, "null pointer argument");
  *device_address = 0;
  cudaPointerAttributes attr;
  cudaError_t e = cudaPointerGetAttributes(&attr, host);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return set_error(SF_ERR_UNSUPPORTED, "host memory %p is not known to CUDA", host);
  }
  if (attr.type != cudaMemoryTypeHost || attr.devicePointer == nullptr)
    return set_error(SF_ERR_UNSUPPORTED, "host memory %p is not page-locked and device-mapped", host);
  *device_address = reinterpret_cast<uint64_t>(attr.devicePointer);
  return SF_OK;
}
