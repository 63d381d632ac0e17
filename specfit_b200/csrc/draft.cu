// Device steps of drafting a candidate pool (the EAGLE-3 tree builder's
// level loop, src/specfit/runtime/eagle3_tree.py:611-803), so one drafting
// pass replays from a CUDA graph as a short chain of kernels:
//
//   sf_draft_level  one level's selection: among the frontier's rows x k
//                   children (each row's k most likely next tokens), the
//                   `width` best by (cumulative log-probability desc, parent
//                   asc, token asc) -- the order the eager builder sorts its
//                   options in -- written as pool rows, plus the next
//                   frontier's tokens, scores, ancestor sets, positions and
//                   parent hidden states;
//   sf_rope_rows    cos / sin rows of the rotary embedding at device-side
//                   positions (fp32 angle pos * inv_freq, rounded to bf16).
#include "common.cuh"

namespace sf {
namespace {

constexpr int kLevelThreads = 256;
constexpr int kMaxCandidates = 32;  // frontier rows x k, one per lane of warp 0

__global__ void __launch_bounds__(kLevelThreads)
draft_level_kernel(const float* __restrict__ v, const int64_t* __restrict__ t, int rows, int k,
                   const double* __restrict__ cum, const int64_t* __restrict__ vis,
                   const __nv_bfloat16* __restrict__ hidden, int H, int width, int64_t first,
                   int depth, int row_base, const int64_t* __restrict__ seed_pos,
                   int64_t* __restrict__ next_tok, double* __restrict__ next_cum,
                   int64_t* __restrict__ next_vis, int64_t* __restrict__ next_pos,
                   __nv_bfloat16* __restrict__ next_hidden, double* __restrict__ out_rows) {
  pdl_wait();
  pdl_trigger();
  __shared__ int sel_parent[kMaxCandidates];
  const int n = rows * k;
  if (threadIdx.x < 32) {
    const int i = threadIdx.x;
    const bool ok = i < n;
    const int par = ok ? i / k : 0x7fffffff;
    const float cv = ok ? v[i] : 0.f;
    const double sc = ok ? cum[par] + (double)cv : -INFINITY;
    const long long tok = ok ? (long long)t[i] : 0x7fffffffffffffffLL;
    // Rank of candidate i in (score desc, parent asc, token asc); a row's k
    // tokens are distinct, so no two candidates compare equal.
    int rank = 0;
    for (int m = 0; m < 32; ++m) {
      const double sm = __shfl_sync(0xffffffffu, sc, m);
      const int pm = __shfl_sync(0xffffffffu, par, m);
      const long long tm = __shfl_sync(0xffffffffu, tok, m);
      if (ok && m < n && m != i)
        rank += (sm > sc || (sm == sc && (pm < par || (pm == par && tm < tok)))) ? 1 : 0;
    }
    if (ok && rank < width) {
      next_tok[rank] = tok;
      next_cum[rank] = sc;
      next_vis[rank] = vis[par] | (int64_t)(1ull << (row_base + rank));
      next_pos[rank] = *seed_pos + depth + 1;
      double* o = out_rows + (int64_t)rank * 5;
      o[0] = (double)tok;
      o[1] = (double)(first + par);
      o[2] = (double)cv;
      o[3] = sc;
      o[4] = (double)(depth + 1);
      sel_parent[rank] = par;
    }
  }
  __syncthreads();
  const int vec = H / 8;
  for (int idx = threadIdx.x; idx < width * vec; idx += kLevelThreads) {
    const int s = idx / vec, c = idx - s * vec;
    reinterpret_cast<uint4*>(next_hidden + (int64_t)s * H)[c] =
        reinterpret_cast<const uint4*>(hidden + (int64_t)sel_parent[s] * H)[c];
  }
}

__global__ void rope_rows_kernel(const int64_t* __restrict__ pos, int n, const float* __restrict__ inv_freq,
                                 int half, __nv_bfloat16* __restrict__ cos_out,
                                 __nv_bfloat16* __restrict__ sin_out) {
  pdl_wait();
  pdl_trigger();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n * half) return;
  const int r = i / half, d = i - r * half;
  const float a = (float)pos[r] * inv_freq[d];  // the fp32 product torch forms
  const __nv_bfloat16 c = __float2bfloat16_rn(cosf(a)), s = __float2bfloat16_rn(sinf(a));
  const int64_t base = (int64_t)r * 2 * half;
  cos_out[base + d] = c;
  cos_out[base + half + d] = c;
  sin_out[base + d] = s;
  sin_out[base + half + d] = s;
}

}  // namespace
}  // namespace sf

extern "C" int sf_draft_level(const float* top_values, const int64_t* top_indices, int rows, int k,
                              const double* cum, const int64_t* ancestor_sets, const void* hidden,
                              int hidden_size, int width, int64_t first, int depth, int row_base,
                              const int64_t* seed_pos, int64_t* next_tokens, double* next_cum,
                              int64_t* next_ancestor_sets, int64_t* next_positions,
                              void* next_hidden, double* out_rows, void* stream) {
  using namespace sf;
  SF_CHECK_ARG(rows >= 1 && k >= 1 && rows * k <= kMaxCandidates, "rows * k must be in [1, %d]",
               kMaxCandidates);
  SF_CHECK_ARG(width >= 1 && width <= rows * k, "width must be in [1, rows * k]");
  SF_CHECK_ARG(row_base >= 0 && row_base + width <= 64, "the next level must fit the 64-row block");
  SF_CHECK_ARG(hidden_size > 0 && hidden_size % 8 == 0, "hidden_size must be a positive multiple of 8");
  SF_CHECK_ARG(top_values && top_indices && cum && ancestor_sets && hidden && seed_pos &&
                   next_tokens && next_cum && next_ancestor_sets && next_positions && next_hidden &&
                   out_rows,
               "null pointer argument");
  SF_CHECK_ARG(aligned16(hidden) && aligned16(next_hidden), "hidden rows must be 16-byte aligned");
  SF_CHECK_CUDA(launch_pdl(draft_level_kernel, dim3(1), dim3(kLevelThreads), 0, as_stream(stream),
                           top_values, top_indices, rows, k, cum, ancestor_sets,
                           static_cast<const __nv_bfloat16*>(hidden), hidden_size, width, first,
                           depth, row_base, seed_pos, next_tokens, next_cum, next_ancestor_sets,
                           next_positions, static_cast<__nv_bfloat16*>(next_hidden), out_rows));
  return SF_OK;
}

extern "C" int sf_rope_rows(const int64_t* positions, int rows, const float* inv_freq, int head_dim,
                            void* cos_out, void* sin_out, void* stream) {
  using namespace sf;
  SF_CHECK_ARG(rows >= 0 && head_dim > 0 && head_dim % 2 == 0, "invalid sizes");
  if (rows == 0) return SF_OK;
  SF_CHECK_ARG(positions && inv_freq && cos_out && sin_out, "null pointer argument");
  const int half = head_dim / 2;
  const int total = rows * half;
  SF_CHECK_CUDA(launch_pdl(rope_rows_kernel, dim3((unsigned)((total + 255) / 256)), dim3(256), 0,
                           as_stream(stream), positions, rows, inv_freq, half,
                           static_cast<__nv_bfloat16*>(cos_out), static_cast<__nv_bfloat16*>(sin_out)));
  return SF_OK;
}
