// Parameters shared by the tree-attention split kernels and the merge kernel
// that combines their partials.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace sf {

struct AttnParams {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  const uint32_t* bits;
  int bit_words;
  int q_len, kv_len, prefix_len;
  int num_heads, num_kv_heads, group;
  int64_t q_hs, q_rs, kv_hs, kv_rs;
  float scale;
  int splits, keys_per_split;
  float* part_o;   // [splits, Hq, Tq, D] unnormalised outputs
  float* part_ml;  // [splits, Hq, Tq, 2] (row max of scaled scores, row sum)
};

bool tree_attention_mma_supports(const AttnParams& p, int head_dim);
// Launches the mma.sync split kernel: chooses p.splits / p.keys_per_split,
// sets p.part_ml, writes the split partials.  When the splits of a row block
// fit one thread-block cluster (at most 16) and the device can place it, the
// splits are merged inside the kernel through distributed shared memory and
// `out` ([Tq, Hq, D] bf16) is written directly: *merged is set to true.
int tree_attention_mma(AttnParams& p, void* out, bool* merged, cudaStream_t stream);

}  // namespace sf
