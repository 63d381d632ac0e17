// Internal interface between the sf_grouped_swiglu entry point and its two
// implementations (CUDA-core and tcgen05).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace sf {

struct SwigluArgs {
  const void* hidden_sorted;
  const float* weights_sorted;
  int dtype;
  const int32_t* offsets;
  const int32_t* active;
  const int32_t* num_active;
  const int32_t* expert_slot;
  const void* slot_storage;
  int64_t slot_count;
  int64_t slot_stride;  // elements between consecutive slots
  int num_experts;
  int hidden;
  int inter;
  int64_t rows;
  void* act_workspace;
  void* out_sorted;
};

// The gathered variant's extra inputs: SwigluArgs::hidden_sorted is then the
// unsorted hidden [tokens, H]; sorted row r reads hidden row
// sorted_pos[r] / top_k and weight topk_weights[sorted_pos[r]] (fp32).
struct SwigluGather {
  int64_t tokens;
  int top_k;
  const int32_t* sorted_pos;
  const float* topk_weights;
};

// Phase 2 of the expert-parallel pass with the return all-to-all fused into
// its epilogue: sorted row r is stored at the address dst_row[r] (a row of a
// source rank's return buffer, 0: not stored) instead of out_sorted; after
// its stores every CTA counts itself on `ticket` (zero before the launch,
// zero again after it), and the last one adds `per_epoch` to the arrival
// counter of this rank in every rank's region
// (peers[r] + arrive_off + 8 * me).
struct SwigluPeerOut {
  const uint64_t* dst_row;
  unsigned int* ticket;
  const uint64_t* peers;  // device [world]
  int64_t arrive_off;
  int world, me;
  unsigned long long per_epoch;
};

int swiglu_simt(const SwigluArgs& a, cudaStream_t stream);
// Returns SF_ERR_UNSUPPORTED (without a message) when the shape does not fit.
int swiglu_tcgen05(const SwigluArgs& a, cudaStream_t stream);
bool swiglu_tcgen05_supports(const SwigluArgs& a);
int swiglu_tcgen05_gathered(const SwigluArgs& a, const SwigluGather& g, cudaStream_t stream);
int swiglu_tcgen05_peer(const SwigluArgs& a, const SwigluPeerOut& peer, cudaStream_t stream);
// Reads (and with reset clears) the device status word of the tcgen05 kernels.
int swiglu_status(int* status, int reset);
int dense_status(int* status, int reset);

// A bf16 tiled tensor map with 128-byte swizzling (rank 1 to 5; dims and
// box innermost first, strides in bytes for dims 1..rank-1).
int tma_encode_bf16(CUtensorMap* map, const void* base, int rank, const cuuint64_t* dims,
                    const cuuint64_t* strides_bytes, const cuuint32_t* box);

}  // namespace sf
