// K3 (any shape): grouped SwiGLU expert product on CUDA cores.
//
// Restates _expert_forward (src/specfit/runtime/qwen3_offloaded_experts.py:38-62)
// and the weighting mul_ (:132-138, :198) for every active expert of a layer
// in two launches.  This kernel serves the shapes and dtypes the tensor-core
// path does not take (fp32 models, hidden/intermediate sizes that are not
// multiples of 64, the reference's tiny unit-test shapes).
//
// Phase 1: act[r, i] = round(round(silu(round(x_r.gate_i))) * round(x_r.up_i))
// Phase 2: out[r, h] = round(round(act_r . down_h) * w_r)
// where round() is the model dtype's rounding (identity for fp32), matching
// the bf16 tensors the reference materialises between torch ops.
#include "common.cuh"
#include "swiglu.h"

namespace sf {
namespace {

constexpr int kWarps = 8;
constexpr int kRows = 4;  // rows accumulated together per pass

template <typename T>
__global__ void __launch_bounds__(kWarps * 32)
swiglu_up_simt(const T* __restrict__ xs, const int32_t* __restrict__ offsets,
               const int32_t* __restrict__ active, const int32_t* __restrict__ num_active,
               const int32_t* __restrict__ slot_of, const T* __restrict__ storage,
               int64_t slot_count, int64_t slot_stride, int H, int I, T* __restrict__ act) {
  pdl_wait();
  pdl_trigger();
  const int j = blockIdx.x;
  if (j >= *num_active) return;
  const int e = active[j];
  if (slot_of[e] < 0 || slot_of[e] >= slot_count) return;  // no such slot: skip
  const int i = blockIdx.y * kWarps + (threadIdx.x >> 5);
  if (i >= I) return;
  const int lane = threadIdx.x & 31;
  const int r0 = offsets[e], r1 = offsets[e + 1];
  const T* base = storage + (int64_t)slot_of[e] * slot_stride;
  const T* gate = base + (int64_t)i * H;
  const T* up = base + (int64_t)(I + i) * H;
  for (int rb = r0; rb < r1; rb += kRows) {
    float ag[kRows], au[kRows];
#pragma unroll
    for (int q = 0; q < kRows; ++q) ag[q] = au[q] = 0.f;
    for (int h = lane; h < H; h += 32) {
      const float g = to_f32(gate[h]);
      const float u = to_f32(up[h]);
#pragma unroll
      for (int q = 0; q < kRows; ++q) {
        if (rb + q < r1) {
          const float xv = to_f32(xs[(int64_t)(rb + q) * H + h]);
          ag[q] = fmaf(xv, g, ag[q]);
          au[q] = fmaf(xv, u, au[q]);
        }
      }
    }
#pragma unroll
    for (int q = 0; q < kRows; ++q) {
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        ag[q] += __shfl_xor_sync(0xffffffffu, ag[q], off);
        au[q] += __shfl_xor_sync(0xffffffffu, au[q], off);
      }
      if (lane == 0 && rb + q < r1) {
        const float g = round_to<T>(ag[q]);
        const float u = round_to<T>(au[q]);
        act[(int64_t)(rb + q) * I + i] = from_f32<T>(round_to<T>(silu_f32(g)) * u);
      }
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kWarps * 32)
swiglu_down_simt(const T* __restrict__ act, const float* __restrict__ ws,
                 const int32_t* __restrict__ offsets, const int32_t* __restrict__ active,
                 const int32_t* __restrict__ num_active, const int32_t* __restrict__ slot_of,
                 const T* __restrict__ storage, int64_t slot_count, int64_t slot_stride, int H,
                 int I, T* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int j = blockIdx.x;
  if (j >= *num_active) return;
  const int e = active[j];
  if (slot_of[e] < 0 || slot_of[e] >= slot_count) return;
  const int h = blockIdx.y * kWarps + (threadIdx.x >> 5);
  if (h >= H) return;
  const int lane = threadIdx.x & 31;
  const int r0 = offsets[e], r1 = offsets[e + 1];
  const T* down = storage + (int64_t)slot_of[e] * slot_stride + 2 * (int64_t)I * H + (int64_t)h * I;
  for (int rb = r0; rb < r1; rb += kRows) {
    float acc[kRows];
#pragma unroll
    for (int q = 0; q < kRows; ++q) acc[q] = 0.f;
    for (int i = lane; i < I; i += 32) {
      const float d = to_f32(down[i]);
#pragma unroll
      for (int q = 0; q < kRows; ++q)
        if (rb + q < r1) acc[q] = fmaf(to_f32(act[(int64_t)(rb + q) * I + i]), d, acc[q]);
    }
#pragma unroll
    for (int q = 0; q < kRows; ++q) {
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) acc[q] += __shfl_xor_sync(0xffffffffu, acc[q], off);
      if (lane == 0 && rb + q < r1) {
        const float y = round_to<T>(acc[q]);
        out[(int64_t)(rb + q) * H + h] = from_f32<T>(y * ws[rb + q]);
      }
    }
  }
}

template <typename T>
int launch_simt(const SwigluArgs& a, cudaStream_t stream) {
  const T* xs = static_cast<const T*>(a.hidden_sorted);
  const T* storage = static_cast<const T*>(a.slot_storage);
  T* act = static_cast<T*>(a.act_workspace);
  T* out = static_cast<T*>(a.out_sorted);
  dim3 g1((unsigned)a.num_experts, (unsigned)((a.inter + kWarps - 1) / kWarps));
  SF_CHECK_CUDA(launch_pdl(swiglu_up_simt<T>, dim3(g1), dim3(kWarps * 32), 0, stream, xs, a.offsets,
                           a.active, a.num_active, a.expert_slot, storage, a.slot_count,
                           a.slot_stride, a.hidden, a.inter, act));
  SF_CHECK_LAUNCH();
  dim3 g2((unsigned)a.num_experts, (unsigned)((a.hidden + kWarps - 1) / kWarps));
  SF_CHECK_CUDA(launch_pdl(swiglu_down_simt<T>, dim3(g2), dim3(kWarps * 32), 0, stream, act,
                           a.weights_sorted, a.offsets, a.active, a.num_active, a.expert_slot,
                           storage, a.slot_count, a.slot_stride, a.hidden, a.inter, out));
  SF_CHECK_LAUNCH();
  return SF_OK;
}

}  // namespace

int swiglu_simt(const SwigluArgs& a, cudaStream_t stream) {
  if (a.dtype == SF_DTYPE_BF16) return launch_simt<__nv_bfloat16>(a, stream);
  if (a.dtype == SF_DTYPE_F32) return launch_simt<float>(a, stream);
  return set_error(SF_ERR_UNSUPPORTED, "swiglu dtype %d is not supported", a.dtype);
}

}  // namespace sf
