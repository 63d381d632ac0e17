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
  int head_dim;  // <= 128; the split kernels zero-fill dims past it
  int64_t q_hs, q_rs, kv_hs, kv_rs;
  float scale;
  int splits, keys_per_split;
  float* part_o;   // [batch, splits, Hq, Tq, D] unnormalised outputs
  float* part_ml;  // [batch, splits, Hq, Tq, 2] (row max of scaled scores, row sum)
  // Requests in one launch (the tcgen05 kernel and the merge; 1 elsewhere):
  // request b's q, k/v, tree bits and output start b * (q_bs, kv_bs,
  // bits_bs, out_bs) elements (words for the bits) after request 0's.
  int batch = 1;
  int64_t q_bs = 0, kv_bs = 0, bits_bs = 0, out_bs = 0;
};

// Visibility of keys prefix_len + j0 + i, i in [0, 64), as bit i, from a
// query row's tree bits (little-endian uint32 words over the tree columns):
// keys before the tree block (j0 + i < 0) are visible; bits past the row's
// words are 0.
__device__ __forceinline__ uint64_t tree_mask_window(const uint32_t* __restrict__ bits, int words,
                                                     int j0) {
  if (j0 + 64 <= 0) return ~0ull;
  if (j0 >= 0) {
    const int w = j0 >> 5, sh = j0 & 31;
    const uint64_t lo = w < words ? bits[w] : 0u;
    const uint64_t mid = w + 1 < words ? bits[w + 1] : 0u;
    uint64_t x = lo | (mid << 32);
    if (sh) {
      const uint64_t hi = w + 2 < words ? bits[w + 2] : 0u;
      x = (x >> sh) | (hi << (64 - sh));
    }
    return x;
  }
  const int d = -j0;  // 1..63 keys of the block precede the tree
  const uint64_t x = (uint64_t)(words > 0 ? bits[0] : 0u) |
                     ((uint64_t)(words > 1 ? bits[1] : 0u) << 32);
  return (x << d) | ((1ull << d) - 1);
}

bool tree_attention_mma_supports(const AttnParams& p, int head_dim);
// Launches the mma.sync split kernel: chooses p.splits / p.keys_per_split,
// sets p.part_ml, writes the split partials.  When the splits of a row block
// fit one thread-block cluster (at most 16) and the device can place it, the
// splits are merged inside the kernel through distributed shared memory and
// `out` ([Tq, Hq, D] bf16) is written directly: *merged is set to true.
int tree_attention_mma(AttnParams& p, void* out, bool* merged, cudaStream_t stream);

// The tcgen05 kernel (tree_attn_tc.cu): 128 packed query rows per CTA in
// TMEM, K/V blocks of 128 keys staged by TMA.  Same split / merge contract as
// tree_attention_mma; with one split it writes `out` itself (*merged true).
bool tree_attention_tc_supports(const AttnParams& p, int head_dim);
int tree_attention_tc(AttnParams& p, void* out, bool* merged, cudaStream_t stream);
// Reads (and with reset clears) the device status word of the tcgen05 kernel.
int tree_attention_tc_status(int* status, int reset);

}  // namespace sf
