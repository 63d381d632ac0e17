// SpecFit exact subtree selection (host code).
//
// Restates the exact search of src/specfit/specfit_exact.py:58-94 with the
// topology enumeration of src/specfit/cache_selection_diagnostic.py:20-39:
// every ancestor-closed subset S of the draft pool with |S| <= max_nodes
// (always containing the verification seed, raw id 0) is scored as
//   reward(S)  = 1 + sum_{i in S} exp(cum_logp_i)      (compensated sum)
//   elapsed(S) = b[|S|] + expert_ns * |F(S)| (+ missing_ns * |F(S) \ R|)
//   score(S)   = reward / elapsed
// where F(S) is the union of the (layer, expert) routes of the seed and of S
// and R the resident set; the winner maximises score, ties broken by the
// smallest (-reward, |F|, |S|, ids) with ids in increasing raw order.
//
// Footprints are bitsets of `words` 64-bit words (48 layers x 128 experts =
// 96 words in the reference), OR-ed incrementally along a depth-first walk,
// so each subset costs one OR and one or two population counts.  A subtree
// of the walk is skipped only when an upper bound on its best score is
// strictly below the best found (reward: the r largest remaining
// probabilities; elapsed: the smallest intercept of a larger size and the
// current footprint, which only grows), so the winner and its tie order are
// those of the full enumeration.
//
// The reward sum reproduces Python's builtin sum over floats (compensated,
// Neumaier's variant of Kahan summation, in the order of the ids) because
// the reference relies on it for ties (tests/unit/test_selection_refinement.py:65).
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <vector>

#include "specfit_b200.h"

namespace sf {
int set_error(int status, const char* fmt, ...);
}

namespace {

// Neumaier's compensated summation, left to right.
double compensated_sum(const double* xs, int n) {
  double s = 0.0, c = 0.0;
  for (int i = 0; i < n; ++i) {
    const double x = xs[i];
    const double t = s + x;
    if (fabs(s) >= fabs(x))
      c += (s - t) + x;
    else
      c += (x - t) + s;
    s = t;
  }
  return s + c;
}

struct Search {
  int n, words, max_nodes;
  const int32_t* parents;
  const uint64_t* footprints;  // [(n + 1) * words]
  const uint64_t* resident;    // [words] or null
  const double* intercept;     // [max_nodes + 1]
  double expert_ns, missing_ns;
  std::vector<double> prob;    // prob[raw], raw 1..n
  std::vector<uint64_t> stack; // footprint per depth: [(max_nodes + 1) * words]
  int ids[64];
  double probs_in_order[64];
  // best so far
  bool have = false;
  double best_score = -1.0, best_reward = 0.0;
  int best_experts = 0, best_count = 0;
  int best_ids[64];

  static int popcount_words(const uint64_t* a, int w) {
    int c = 0;
    for (int i = 0; i < w; ++i) c += __builtin_popcountll(a[i]);
    return c;
  }

  int missing_count(const uint64_t* f) const {
    int c = 0;
    for (int i = 0; i < words; ++i) c += __builtin_popcountll(f[i] & ~resident[i]);
    return c;
  }

  // True when (reward, experts, count, ids) ranks before the current best's tie key.
  bool tie_better(double reward, int experts, int count) const {
    if (-reward != -best_reward) return -reward < -best_reward;
    if (experts != best_experts) return experts < best_experts;
    if (count != best_count) return count < best_count;
    const int m = count < best_count ? count : best_count;
    for (int i = 0; i < m; ++i)
      if (ids[i] != best_ids[i]) return ids[i] < best_ids[i];
    return count < best_count;
  }

  // Scores the subset in ids[0..count) with footprint f; returns |F|.
  int score(const uint64_t* f, int count) {
    const int experts = popcount_words(f, words);
    double elapsed = intercept[count] + expert_ns * (double)experts;
    if (missing_ns != 0.0 && resident) elapsed += missing_ns * (double)missing_count(f);
    else if (missing_ns != 0.0) elapsed += missing_ns * (double)experts;
    double reward;
    if (count > 1) {
      for (int i = 0; i < count; ++i) probs_in_order[i] = prob[ids[i]];
      reward = 1.0 + compensated_sum(probs_in_order, count);
    } else if (count == 1) {
      reward = 1.0 + prob[ids[0]];
    } else {
      reward = 1.0;
    }
    const double s = reward / elapsed;
    if (s >= best_score) {
      if (s > best_score || !have || tie_better(reward, experts, count)) {
        have = true;
        best_score = s;
        best_reward = reward;
        best_experts = experts;
        best_count = count;
        for (int i = 0; i < count; ++i) best_ids[i] = ids[i];
      }
    }
    return experts;
  }

  // suffix_top[start * (max_nodes + 1) + r]: the sum of the r largest
  // probabilities among raw ids >= start (an upper bound on what r more
  // nodes can add to the reward).  min_intercept[c]: the smallest intercept
  // over sizes c..max_nodes.
  std::vector<double> suffix_top, min_intercept;

  void prepare_bounds() {
    const int m = max_nodes;
    suffix_top.assign((size_t)(n + 2) * (m + 1), 0.0);
    std::vector<double> top;  // the m largest probabilities of the suffix, descending
    for (int start = n; start >= 1; --start) {
      const double p = prob[start];
      auto it = top.begin();
      while (it != top.end() && *it >= p) ++it;
      top.insert(it, p);
      if ((int)top.size() > m) top.pop_back();
      double acc = 0.0;
      for (int r = 1; r <= m; ++r) {
        if (r <= (int)top.size()) acc += top[r - 1];
        suffix_top[(size_t)start * (m + 1) + r] = acc;
      }
    }
    min_intercept.assign((size_t)m + 2, INFINITY);
    for (int c = m; c >= 0; --c) min_intercept[c] = fmin(intercept[c], min_intercept[c + 1]);
  }

  // Depth-first over ancestor-closed subsets in increasing raw order; the
  // subset in ids[0..count) with footprint at stack[count], `experts` bits
  // and probability sum `psum`.  Extensions are skipped when even the best
  // r remaining probabilities over the cheapest larger size and the current
  // footprint score strictly below the best so far (a margin of 1e-9 keeps
  // every possible tie), so the result is the full enumeration's.
  void visit(int start, uint64_t included, int count, int experts, double psum) {
    if (count == max_nodes || start > n) return;
    const uint64_t* f = &stack[(size_t)count * words];
    const double reward_ub = 1.0 + psum + suffix_top[(size_t)start * (max_nodes + 1) + (max_nodes - count)];
    double elapsed_lb = min_intercept[count + 1] + expert_ns * (double)experts;
    if (missing_ns > 0.0 && resident) elapsed_lb += missing_ns * (double)missing_count(f);
    else if (missing_ns > 0.0) elapsed_lb += missing_ns * (double)experts;
    if (have && elapsed_lb > 0.0 && reward_ub / elapsed_lb * (1.0 + 1e-9) < best_score) return;
    uint64_t* child = &stack[(size_t)(count + 1) * words];
    for (int raw = start; raw <= n; ++raw) {
      if (!((included >> parents[raw - 1]) & 1ull)) continue;
      const uint64_t* g = footprints + (size_t)raw * words;
      for (int i = 0; i < words; ++i) child[i] = f[i] | g[i];
      ids[count] = raw;
      const int child_experts = score(child, count + 1);
      visit(raw + 1, included | (1ull << raw), count + 1, child_experts, psum + prob[raw]);
    }
  }
};

}  // namespace

extern "C" int sf_specfit_select(int num_nodes, const int32_t* parents, const double* cum_logp,
                                 const uint64_t* footprints, int words, const uint64_t* resident,
                                 const double* size_intercept_ns, int max_nodes, double expert_ns,
                                 double missing_ns, int32_t* selected, int32_t* num_selected,
                                 double* best_score) {
  using sf::set_error;
  if (num_nodes < 0 || num_nodes > 63)
    return set_error(SF_ERR_INVALID_ARGUMENT, "num_nodes must be in [0, 63]");
  if (max_nodes < 0 || max_nodes > 63)
    return set_error(SF_ERR_INVALID_ARGUMENT, "max_nodes must be in [0, 63]");
  if (words <= 0) return set_error(SF_ERR_INVALID_ARGUMENT, "words must be positive");
  if (!footprints || !size_intercept_ns || !selected || !num_selected)
    return set_error(SF_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (num_nodes > 0 && (!parents || !cum_logp))
    return set_error(SF_ERR_INVALID_ARGUMENT, "null pointer argument");
  for (int raw = 1; raw <= num_nodes; ++raw)
    if (parents[raw - 1] < 0 || parents[raw - 1] >= raw)
      return set_error(SF_ERR_INVALID_ARGUMENT, "parent of node %d must precede it", raw);
  Search s;
  s.n = num_nodes;
  s.words = words;
  s.max_nodes = max_nodes;
  s.parents = parents;
  s.footprints = footprints;
  s.resident = resident;
  s.intercept = size_intercept_ns;
  s.expert_ns = expert_ns;
  s.missing_ns = missing_ns;
  s.prob.assign((size_t)num_nodes + 1, 0.0);
  for (int raw = 1; raw <= num_nodes; ++raw) s.prob[raw] = exp(cum_logp[raw - 1]);
  s.stack.assign((size_t)(max_nodes + 1) * words, 0);
  memcpy(s.stack.data(), footprints, sizeof(uint64_t) * words);  // the seed's routes
  s.prepare_bounds();
  const int seed_experts = s.score(s.stack.data(), 0);
  s.visit(1, 1ull, 0, seed_experts, 0.0);
  *num_selected = s.best_count;
  for (int i = 0; i < s.best_count; ++i) selected[i] = s.best_ids[i];
  if (best_score) *best_score = s.best_score;
  return SF_OK;
}

extern "C" double sf_compensated_sum(const double* values, int n) {
  return (values && n > 0) ? compensated_sum(values, n) : 0.0;
}

extern "C" int sf_specfit_pack_routes(const int32_t* routes, int tokens, int layers, int top_k,
                                      int experts, uint64_t* footprints, int words) {
  using sf::set_error;
  if (tokens < 0 || layers <= 0 || top_k <= 0 || experts <= 0 || words <= 0)
    return set_error(SF_ERR_INVALID_ARGUMENT, "invalid sizes");
  if ((int64_t)layers * experts > (int64_t)words * 64)
    return set_error(SF_ERR_INVALID_ARGUMENT, "footprint words too small for layers x experts");
  if (tokens > 0 && (!routes || !footprints)) return set_error(SF_ERR_INVALID_ARGUMENT, "null pointer argument");
  memset(footprints, 0, sizeof(uint64_t) * (size_t)tokens * words);
  for (int t = 0; t < tokens; ++t) {
    uint64_t* f = footprints + (size_t)t * words;
    for (int l = 0; l < layers; ++l) {
      const int32_t* r = routes + ((size_t)t * layers + l) * top_k;
      for (int k = 0; k < top_k; ++k) {
        if (r[k] < 0 || r[k] >= experts) return set_error(SF_ERR_INVALID_ARGUMENT, "invalid expert ID");
        const int64_t bit = (int64_t)l * experts + r[k];
        const uint64_t m = 1ull << (bit & 63);
        if (f[bit >> 6] & m) return set_error(SF_ERR_INVALID_ARGUMENT, "duplicate expert ID");
        f[bit >> 6] |= m;
      }
    }
  }
  return SF_OK;
}
