// Diverse beam search selection (DiverseBeamSearchStrategy.select_candidates,
// src/beam_engine/beam_strategy.py:173-317), native host code.
//
// Per prompt: every (parent, child) choice is ordered once by the child's raw
// log-probability (stable, descending).  Groups then pick in turn: each group
// re-scores the choices not yet taken with
//     (log_prob - diversity_penalty) / length ** length_penalty
// (length = parent sequence + 1; no division when length_penalty == 0), sorts
// them stably by that score and takes beams_per_group = max(1, beam_size /
// num_groups) of them.  The diversity penalty of a choice is
//   * hamming: diversity_penalty if its token was taken by any earlier pick of
//     this step, else 0 (beam_strategy.py:105-125);
//   * cumulative: the mean over all earlier picks of (positions where the two
//     sequences -- parent + token each -- agree) * diversity_penalty, the sum
//     taken in pick order (beam_strategy.py:127-155).
// Picks are regrouped per parent in pick order with accumulated score
// parent_score + log_prob; if more than beam_size were picked (num_groups >
// beam_size), children are dropped from the end, last parent first
// (beam_strategy.py:303-315).
//
// Cumulative overlap without re-walking the prompt: for parents i, j of
// lengths la, lb the overlap of (seq_i + t) and (seq_j + u) over their common
// length is ov(i, j) -- agreements of seq_i and seq_j over min(la, lb)
// positions, cached per pair -- plus one comparison at position min(la, lb):
// t vs u when la == lb, t vs seq_j[la] when la < lb, seq_i[lb] vs u otherwise.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <unordered_set>
#include <vector>

#include "beam_b200.h"

namespace be {
void set_error(const char* fmt, ...);
}
using be::set_error;

namespace {

struct Choice {
  int32_t parent;   // local parent index
  int32_t token;
  double logp;
};

int select_one(int n, int k, const double* parent_scores, const int32_t* tokens,
               const double* logps, const int32_t* seq_ptr, const int32_t* seq_tokens,
               int beam_size, int num_groups, double dpen, int dtype, double lpen,
               std::vector<std::vector<std::pair<int32_t, double>>>& kids) {
  const int64_t total = (int64_t)n * k;
  std::vector<Choice> all((size_t)total);
  for (int64_t e = 0; e < total; ++e) all[e] = Choice{(int32_t)(e / k), tokens[e], logps[e]};
  std::vector<int64_t> order((size_t)total);
  for (int64_t e = 0; e < total; ++e) order[e] = e;
  std::stable_sort(order.begin(), order.end(),
                   [&](int64_t a, int64_t b) { return all[a].logp > all[b].logp; });

  const int bpg = std::max(1, beam_size / std::max(1, num_groups));
  std::vector<int64_t> picked;                           // choice ids in pick order
  std::unordered_set<int64_t> taken;                     // (parent, token) keys
  std::unordered_set<int32_t> step_tokens;               // hamming
  auto key = [](int32_t p, int32_t t) { return ((int64_t)p << 32) | (uint32_t)t; };
  auto len = [&](int i) { return (int64_t)seq_ptr[i + 1] - seq_ptr[i]; };
  // cumulative: pair overlaps of parent sequences, computed on demand
  std::vector<int32_t> pov;
  if (dtype != 0) pov.assign((size_t)n * n, -1);
  auto pair_ov = [&](int i, int j) -> int32_t {
    int32_t& v = pov[(size_t)i * n + j];
    if (v < 0) {
      const int64_t m = std::min(len(i), len(j));
      const int32_t* a = seq_tokens + seq_ptr[i];
      const int32_t* b = seq_tokens + seq_ptr[j];
      int32_t c = 0;
      for (int64_t p = 0; p < m; ++p) c += a[p] == b[p];
      v = c;
      pov[(size_t)j * n + i] = c;
    }
    return v;
  };

  std::vector<std::pair<int64_t, double>> adj;
  adj.reserve((size_t)total);
  for (int g = 0; g < num_groups; ++g) {
    adj.clear();
    for (int64_t e : order) {
      const Choice& c = all[e];
      if (taken.count(key(c.parent, c.token))) continue;
      const int64_t la = len(c.parent);
      double pen = 0.0;
      if (dtype == 0) {
        if (step_tokens.count(c.token)) pen = dpen;
      } else if (!picked.empty()) {
        double sum = 0.0;
        for (int64_t q : picked) {
          const Choice& s = all[q];
          const int64_t lb = len(s.parent);
          int64_t ov = pair_ov(c.parent, s.parent);
          if (la == lb)
            ov += c.token == s.token;
          else if (la < lb)
            ov += c.token == seq_tokens[seq_ptr[s.parent] + la];
          else
            ov += seq_tokens[seq_ptr[c.parent] + lb] == s.token;
          sum += (double)ov * dpen;
        }
        pen = sum / (double)picked.size();
      }
      double score = c.logp - pen;
      if (lpen != 0.0) score = score / std::pow((double)(la + 1), lpen);
      adj.emplace_back(e, score);
    }
    std::stable_sort(adj.begin(), adj.end(),
                     [](const std::pair<int64_t, double>& a, const std::pair<int64_t, double>& b) {
                       return a.second > b.second;
                     });
    const int take = std::min<int64_t>(bpg, (int64_t)adj.size());
    for (int r = 0; r < take; ++r) {
      const Choice& c = all[adj[r].first];
      picked.push_back(adj[r].first);
      taken.insert(key(c.parent, c.token));
      step_tokens.insert(c.token);
    }
  }
  kids.assign(n, {});
  for (int64_t q : picked) {
    const Choice& c = all[q];
    kids[c.parent].emplace_back(c.token, parent_scores[c.parent] + c.logp);
  }
  int64_t count = (int64_t)picked.size();
  for (int i = n - 1; i >= 0 && count > beam_size; --i)
    while (count > beam_size && !kids[i].empty()) {
      kids[i].pop_back();
      --count;
    }
  return BE_OK;
}

}  // namespace

extern "C" int be_diverse_select(int nseg, const int32_t* seg_ptr, int k, const double* parent_scores,
                                 const int32_t* tokens, const double* logps, const int32_t* seq_ptr,
                                 const int32_t* seq_tokens, int beam_size, int num_groups,
                                 double diversity_penalty, int diversity_type,
                                 double length_penalty, int32_t* child_ptr,
                                 int32_t* child_tokens, double* child_scores,
                                 int32_t* new_seg_ptr) {
  if (nseg < 0 || k < 0 || beam_size < 1 || num_groups < 1 || !seg_ptr || !child_ptr ||
      !new_seg_ptr || (diversity_type != 0 && diversity_type != 1) ||
      (seg_ptr[nseg] > 0 && (!seq_ptr || !parent_scores)) ||
      (diversity_type == 1 && seg_ptr[nseg] > 0 && !seq_tokens)) {
    set_error("be_diverse_select: invalid arguments");
    return BE_EINVAL;
  }
  std::vector<std::vector<std::pair<int32_t, double>>> kids;
  std::vector<int32_t> local_ptr;
  int32_t out = 0;
  child_ptr[0] = 0;
  new_seg_ptr[0] = 0;
  for (int s = 0; s < nseg; ++s) {
    const int a = seg_ptr[s], b = seg_ptr[s + 1];
    if (b < a) {
      set_error("be_diverse_select: seg_ptr not ascending at %d", s);
      return BE_EINVAL;
    }
    const int n = b - a;
    // the segment's sequences, re-based so parent i's tokens start at local_ptr[i]
    local_ptr.resize(n + 1);
    for (int i = 0; i <= n; ++i) local_ptr[i] = seq_ptr[a + i] - seq_ptr[a];
    const int32_t* seg_tokens = seq_tokens ? seq_tokens + seq_ptr[a] : nullptr;
    int rc = select_one(n, k, parent_scores + a, tokens + (int64_t)a * k, logps + (int64_t)a * k,
                        local_ptr.data(), seg_tokens, beam_size, num_groups, diversity_penalty,
                        diversity_type, length_penalty, kids);
    if (rc) return rc;
    for (int i = 0; i < n; ++i) {
      for (const auto& c : kids[i]) {
        child_tokens[out] = c.first;
        child_scores[out] = c.second;
        ++out;
      }
      child_ptr[a + i + 1] = out;
    }
    new_seg_ptr[s + 1] = out;
  }
  return BE_OK;
}
