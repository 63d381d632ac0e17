// Internal interface between sf_tree_attention and its two implementations
// (CUDA-core split kernel and the tcgen05 kernel); both write split partials
// that tree_attn_merge_kernel combines.
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

bool tree_attention_tc_supports(const AttnParams& p, int head_dim);
// Launches the tcgen05 split kernel; sets *splits (partials written).
int tree_attention_tc(const AttnParams& p, cudaStream_t stream, int* splits);

}  // namespace sf
