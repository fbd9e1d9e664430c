// Host-side attention planners: cascade levels / FastTree vnodes -> work items.
//
// The planner turns the reference's per-level cascade indices (or FastTree's
// vnode metadata) into one flat int32 buffer that a single kernel launch
// consumes: work items ordered heaviest-first (wide tiles, then narrow), the
// query list, the KV list and the per-query merge lists.
#include <algorithm>
#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <numeric>
#include <vector>

#include "beam_b200.h"

static_assert(sizeof(be_attn_plan_info) <= BE_PLAN_HEADER_INTS * sizeof(int32_t), "header");

namespace be {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

namespace {

struct W {
  be_attn_work w;
  int64_t cost;
  bool wide;
};

// Tokens per decode-time wide (tensor-core) chunk when > 0 (BE_PLAN_WIDE_CHUNK,
// rounded to pages and capped at the resident tile); 0 = balance the split.
inline int wide_chunk_override() {
  static const int v = [] {
    const char* e = getenv("BE_PLAN_WIDE_CHUNK");
    return e ? std::max(0, atoi(e)) : 0;
  }();
  return v;
}

// Tokens per causal (prefill) wide chunk when > 0 (BE_PLAN_CAUSAL_WIDE_CHUNK,
// e.g. 128: the chunks then fit the resident tcgen05 tile, which masks causally);
// 0 = balance the split like any other group.
inline int causal_wide_chunk() {
  static const int v = [] {
    const char* e = getenv("BE_PLAN_CAUSAL_WIDE_CHUNK");
    return e ? std::max(0, atoi(e)) : 0;
  }();
  return v;
}

// BE_ATTN_WIDE_RUNS=1: wide items keep their creation order (each group's chunks
// adjacent, so the persistent kernel's contiguous task ranges form long runs)
// instead of being sorted by cost.
inline bool wide_runs_order() {
  static const bool v = [] {
    const char* e = getenv("BE_ATTN_WIDE_RUNS");
    return e && e[0] == '1';
  }();
  return v;
}

// Wide tiles hold up to 64 rows, narrow tiles 16 (rows = queries x group size).
inline int tile_queries(int qlen, int g) {
  if (qlen * g <= 16) return qlen;
  return std::max(1, 64 / g);
}

int emit_plan(std::vector<W>& items, const std::vector<int32_t>& qlist,
              const std::vector<int32_t>& kvlist, int num_queries, bool allow_direct,
              int page_size, int g, int32_t* plan, int64_t cap, be_attn_plan_info* info) {
  // per-thread scratch (one lookup per call; the planner runs every decode step)
  struct Scratch {
    std::vector<int32_t> cover, pcount, pfill, pflat, mq, mptr, mparts, order;
    std::vector<char> direct_q;
  };
  static thread_local Scratch tls;
  Scratch& S = tls;
  // Which queries are covered exactly once (direct write) and which need merging.
  auto& cover = S.cover;
  cover.assign(num_queries, 0);
  for (auto& it : items)
    for (int i = 0; i < it.w.q_len; ++i) cover[qlist[it.w.q_off + i]]++;
  int n_parts = 0;
  for (auto& it : items) {
    bool direct = allow_direct;
    for (int i = 0; i < it.w.q_len && direct; ++i) direct = cover[qlist[it.w.q_off + i]] == 1;
    if (direct) {
      it.w.part_base = -1;
    } else {
      it.w.part_base = n_parts;
      n_parts += it.w.q_len;
    }
  }
  // partial rows per query as CSR (items in plan order, as a per-query list would hold them)
  auto& direct_q = S.direct_q;
  auto& pcount = S.pcount;
  direct_q.assign(num_queries, 0);
  pcount.assign(num_queries + 1, 0);
  for (auto& it : items)
    for (int i = 0; i < it.w.q_len; ++i) {
      const int q = qlist[it.w.q_off + i];
      if (it.w.part_base < 0) direct_q[q] = 1;
      else pcount[q + 1]++;
    }
  for (int q = 0; q < num_queries; ++q) pcount[q + 1] += pcount[q];
  auto& pfill = S.pfill;
  auto& pflat = S.pflat;
  pfill.assign(pcount.begin(), pcount.end() - 1);
  pflat.resize(pcount[num_queries]);
  for (auto& it : items)
    for (int i = 0; i < it.w.q_len; ++i)
      if (it.w.part_base >= 0) pflat[pfill[qlist[it.w.q_off + i]]++] = it.w.part_base + i;
  // wide items first, each class by cost descending, ties in creation order (the
  // order of a stable sort), as an index sort: no temporary buffer
  auto& order = S.order;
  order.resize(items.size());
  int64_t maxc = 0;
  bool small = true;
  for (const auto& it : items) {
    maxc = std::max(maxc, it.cost);
    small = small && it.cost >= 0;
  }
  if (small && maxc <= (1 << 16)) {
    // counting sort on (wide first, cost descending), items in creation order
    // within a key: the stable order in two linear passes
    auto& cnt = S.pfill;   // reused scratch
    const int64_t nk = 2 * (maxc + 1);
    cnt.assign((size_t)nk + 1, 0);
    const bool keep_wide = wide_runs_order();
    auto key = [&](const W& it) {
      return it.wide ? (keep_wide ? 0 : maxc - it.cost) : maxc + 1 + (maxc - it.cost);
    };
    for (const auto& it : items) cnt[key(it) + 1]++;
    for (int64_t k = 0; k < nk; ++k) cnt[k + 1] += cnt[k];
    for (size_t i = 0; i < items.size(); ++i) order[cnt[key(items[i])]++] = (int32_t)i;
  } else {
    for (size_t i = 0; i < items.size(); ++i) order[i] = (int32_t)i;
    const bool keep_wide = wide_runs_order();
    std::sort(order.begin(), order.end(), [&](int32_t a, int32_t b) {
      const W& x = items[a];
      const W& y = items[b];
      if (x.wide != y.wide) return x.wide;
      if (!(x.wide && keep_wide) && x.cost != y.cost) return x.cost > y.cost;
      return a < b;
    });
  }
  auto& mq = S.mq;
  auto& mptr = S.mptr;
  auto& mparts = S.mparts;
  mq.clear();
  mparts.clear();
  mptr.assign(1, 0);
  for (int q = 0; q < num_queries; ++q) {
    if (direct_q[q]) continue;
    mq.push_back(q);
    mparts.insert(mparts.end(), pflat.begin() + pcount[q], pflat.begin() + pcount[q + 1]);
    mptr.push_back((int32_t)mparts.size());
  }
  be_attn_plan_info in{};
  in.n_work = (int32_t)items.size();
  in.n_work_wide = (int32_t)std::count_if(items.begin(), items.end(), [](const W& x) { return x.wide; });
  in.n_queries = num_queries;
  in.n_parts = n_parts;
  in.n_merge = (int32_t)mq.size();
  int64_t off = BE_PLAN_HEADER_INTS;   // the header (this struct) leads the buffer
  in.off_work = (int32_t)off;
  off += (int64_t)items.size() * 8;
  in.off_qlist = (int32_t)off;
  off += qlist.size();
  in.off_kvlist = (int32_t)off;
  off += kvlist.size();
  in.off_merge_q = (int32_t)off;
  off += mq.size();
  in.off_merge_ptr = (int32_t)off;
  off += mptr.size();
  in.off_merge_parts = (int32_t)off;
  off += mparts.size();
  if (off > INT32_MAX) {
    set_error("plan too large (%lld ints)", (long long)off);
    return BE_EINVAL;
  }
  in.total_ints = (int32_t)off;
  in.page_size = page_size;
  in.group_size = g;
  for (auto& it : items) {
    const int len = it.w.kv_end - it.w.kv_begin;
    in.max_item_tokens = std::max(in.max_item_tokens, len);
    in.total_tokens += len;
    if (it.wide) in.max_wide_tokens = std::max(in.max_wide_tokens, len);
    if (it.w.flags & BE_WORK_SLOTS) in.any_slots = 1;
  }
  *info = in;
  if (off > cap || !plan) {
    set_error("plan buffer too small: need %lld ints, have %lld", (long long)off, (long long)cap);
    return BE_ECAPACITY;
  }
  std::memset(plan, 0, BE_PLAN_HEADER_INTS * sizeof(int32_t));
  std::memcpy(plan, &in, sizeof(in));
  int32_t* p = plan + BE_PLAN_HEADER_INTS;
  for (int32_t i : order) {
    std::memcpy(p, &items[i].w, sizeof(be_attn_work));
    p += 8;
  }
  auto put = [&](const std::vector<int32_t>& v) {
    if (!v.empty()) std::memcpy(p, v.data(), v.size() * sizeof(int32_t));
    p += v.size();
  };
  put(qlist);
  put(kvlist);
  put(mq);
  put(mptr);
  put(mparts);
  return BE_OK;
}

// Queries gq[q_at .. q_at + qlen) attending one contiguous KV range (page list
// from kv_off); causal groups hold consecutive queries in order.
struct Grp {
  bool causal;
  int q_at, qlen, kv_off, kv_len;
};

// Groups -> work items: tiles of <= 64 (wide) or <= 16 (narrow) rows, the KV
// split for ~4 CTAs per SM (decode wide chunks capped at the resident tensor-
// core tile), then emit_plan.
int plan_groups(const std::vector<Grp>& groups, const std::vector<int32_t>& gq,
                const std::vector<int32_t>& kvlist, int num_queries, int page_size, int g, int num_kv_heads, int split_tokens,
                int num_sms, int32_t* plan, int64_t plan_capacity, be_attn_plan_info* info) {
  int64_t total_cost = 0;
  for (const auto& gr : groups)
    total_cost += (int64_t)gr.kv_len *
                  ((gr.qlen + tile_queries(gr.qlen, g) - 1) / std::max(1, tile_queries(gr.qlen, g)));
  // KV split: aim for ~4 CTAs per SM in total (CTAs = items x kv heads), but keep
  // chunks long enough that the fp32 partial rows stay small next to the KV bytes
  // they summarise (>= 8 tokens per row of the tile).
  const int sms = num_sms > 0 ? num_sms : 148;
  const int64_t target_items = std::max<int64_t>(1, (int64_t)sms * 4 / num_kv_heads);
  auto round_pages = [&](int64_t t) {
    return (int)std::max<int64_t>(page_size, (t + page_size - 1) / page_size * page_size);
  };
  const int balanced = round_pages((total_cost + target_items - 1) / target_items);
  static thread_local std::vector<W> items_tls;
  static thread_local std::vector<int32_t> qlist_tls;
  std::vector<W>& items = items_tls;
  std::vector<int32_t>& qlist = qlist_tls;
  items.clear();
  qlist.clear();
  for (const auto& gr : groups) {
    if (gr.kv_len <= 0 || gr.qlen <= 0) continue;  // empty KV: lse = -inf, contributes nothing
    const bool causal = gr.causal;
    const int tq = tile_queries(gr.qlen, g);
    const bool wide = tq * g > 16;
    int chunk;
    if (split_tokens > 0) {
      chunk = round_pages(split_tokens);
    } else {
      const int min_chunk = round_pages((int64_t)std::min(gr.qlen, tq) * g * 8);
      chunk = std::max(min_chunk, balanced);
      // decode-time wide tiles run as one resident tensor-core tile
      if (wide && !causal) {
        chunk = std::min(chunk, BE_UMMA_MAX_TOKENS);
        if (wide_chunk_override() > 0)
          chunk = std::min(round_pages(wide_chunk_override()), BE_UMMA_MAX_TOKENS);
      }
      if (wide && causal && causal_wide_chunk() > 0)
        chunk = std::min(chunk, std::max(page_size, causal_wide_chunk() / page_size * page_size));
      const int nsplit = (gr.kv_len + chunk - 1) / chunk;
      chunk = round_pages((gr.kv_len + nsplit - 1) / nsplit);
    }
    for (int qs = 0; qs < gr.qlen; qs += tq) {
      const int ql = std::min(tq, gr.qlen - qs);
      const int q_off = (int)qlist.size();
      for (int i = 0; i < ql; ++i) qlist.push_back(gq[gr.q_at + qs + i]);
      // causal limit of query i of this tile: kv_len - qlen + (qs + i) + 1
      const int kv_total_eff = gr.kv_len - gr.qlen + qs + ql;
      for (int t = 0; t < gr.kv_len; t += chunk) {
        const int t1 = std::min(gr.kv_len, t + chunk);
        if (causal && t >= kv_total_eff) break;  // no query of the tile sees this chunk
        W it;
        it.w.q_off = q_off;
        it.w.q_len = ql;
        it.w.kv_off = gr.kv_off;
        it.w.kv_begin = t;
        it.w.kv_end = t1;
        it.w.kv_total = kv_total_eff;
        it.w.part_base = 0;
        it.w.flags = causal ? BE_WORK_CAUSAL : 0;
        it.cost = (int64_t)(t1 - t);
        it.wide = wide;
        items.push_back(it);
      }
    }
  }
  return emit_plan(items, qlist, kvlist, num_queries, true, page_size, g, plan, plan_capacity, info);
}

}  // namespace
}  // namespace be

using namespace be;

extern "C" const char* be_last_error(void) { return g_err; }
extern "C" int be_version(void) { return 1; }

extern "C" int be_cascade_plan(int num_levels, const int32_t* const* qo_indptr,
                               const int32_t* const* kv_indptr, const int32_t* const* kv_indices,
                               const int32_t* const* last_page_len, const int32_t* num_groups,
                               int num_queries, int page_size, int num_qo_heads, int num_kv_heads,
                               int causal_last, int split_tokens, int num_sms, int32_t* plan,
                               int64_t plan_capacity, be_attn_plan_info* info) {
  if (num_levels < 0 || num_queries < 0 || page_size < 1 || num_kv_heads < 1 ||
      num_qo_heads % num_kv_heads || !info) {
    set_error("be_cascade_plan: invalid arguments");
    return BE_EINVAL;
  }
  const int g = num_qo_heads / num_kv_heads;
  if (g > 64) {
    set_error("be_cascade_plan: group size %d > 64 unsupported", g);
    return BE_EINVAL;
  }
  static thread_local std::vector<Grp> groups_tls;
  static thread_local std::vector<int32_t> kvlist_tls, gq_tls;
  std::vector<Grp>& groups = groups_tls;
  std::vector<int32_t>& kvlist = kvlist_tls;
  std::vector<int32_t>& gq = gq_tls;
  groups.clear();
  kvlist.clear();
  gq.clear();
  for (int l = 0; l < num_levels; ++l) {
    const int G = num_groups[l];
    const int base = (int)kvlist.size();
    const int npages_total = G > 0 ? kv_indptr[l][G] : 0;
    if (G > 0 && (qo_indptr[l][0] != 0 || kv_indptr[l][0] != 0 || qo_indptr[l][G] > num_queries)) {
      set_error("be_cascade_plan: level %d indptr does not start at 0 or exceeds %d queries", l,
                num_queries);
      return BE_EINVAL;
    }
    kvlist.insert(kvlist.end(), kv_indices[l], kv_indices[l] + npages_total);
    for (int gi = 0; gi < G; ++gi) {
      const int qlen = qo_indptr[l][gi + 1] - qo_indptr[l][gi];
      const int np = kv_indptr[l][gi + 1] - kv_indptr[l][gi];
      if (qlen < 0 || np < 0) {
        set_error("be_cascade_plan: level %d group %d has negative extent", l, gi);
        return BE_EINVAL;
      }
      const int last = last_page_len[l][gi];
      if (np > 0 && (last < 0 || last > page_size)) {
        set_error("be_cascade_plan: level %d group %d last_page_len %d outside [0, %d]", l, gi, last,
                  page_size);
        return BE_EINVAL;
      }
      const int kv_len = np > 0 ? (np - 1) * page_size + last : 0;
      groups.push_back({causal_last != 0 && l == num_levels - 1, (int)gq.size(), qlen,
                        base + kv_indptr[l][gi], kv_len});
      for (int i = 0; i < qlen; ++i) gq.push_back(qo_indptr[l][gi] + i);
    }
  }
  return plan_groups(groups, gq, kvlist, num_queries, page_size, g, num_kv_heads, split_tokens,
                     num_sms, plan, plan_capacity, info);
}

extern "C" int be_tree_plan(int num_vnodes, const int32_t* q_entries, int num_q_entries,
                            const int32_t* q_offs, const int32_t* q_lens, const int32_t* kv_offs,
                            const int32_t* kv_lens, const int32_t* r2v_entries,
                            const int32_t* r2v_offs, const int32_t* r2v_lens, int batch_size,
                            int page_size, int num_qo_heads, int num_kv_heads, int32_t* plan,
                            int64_t plan_capacity, be_attn_plan_info* info) {
  if (num_vnodes < 0 || batch_size < 0 || page_size < 1 || num_kv_heads < 1 ||
      num_qo_heads % num_kv_heads || !info) {
    set_error("be_tree_plan: invalid arguments");
    return BE_EINVAL;
  }
  const int g = num_qo_heads / num_kv_heads;
  std::vector<W> items;
  for (int v = 0; v < num_vnodes; ++v) {
    if (q_lens[v] <= 0) continue;
    if (q_lens[v] * g > 64) {
      set_error("be_tree_plan: vnode %d has %d queries x group %d > 64 rows", v, q_lens[v], g);
      return BE_EINVAL;
    }
    if (q_offs[v] < 0 || q_offs[v] + q_lens[v] > num_q_entries) {
      set_error("be_tree_plan: vnode %d query range outside the entry list", v);
      return BE_EINVAL;
    }
    W it;
    it.w.q_off = q_offs[v];
    it.w.q_len = q_lens[v];
    it.w.kv_off = kv_offs[v];
    it.w.kv_begin = 0;
    it.w.kv_end = kv_lens[v];
    it.w.kv_total = kv_lens[v];
    it.w.part_base = 0;
    it.w.flags = BE_WORK_SLOTS;
    it.cost = kv_lens[v];
    it.wide = q_lens[v] * g > 16;
    items.push_back(it);
  }
  std::vector<int32_t> qlist(q_entries, q_entries + num_q_entries);
  // Partial rows follow FastTree's layout: entry e of the query list owns row e.
  std::stable_sort(items.begin(), items.end(), [](const W& a, const W& b) {
    if (a.wide != b.wide) return a.wide;
    return a.cost > b.cost;
  });
  std::vector<int32_t> mq, mptr{0}, mparts;
  for (int b = 0; b < batch_size; ++b) {
    mq.push_back(b);
    for (int k = 0; k < r2v_lens[b]; ++k) mparts.push_back(r2v_entries[r2v_offs[b] + k]);
    mptr.push_back((int32_t)mparts.size());
  }
  be_attn_plan_info in{};
  in.n_work = (int32_t)items.size();
  in.n_work_wide = (int32_t)std::count_if(items.begin(), items.end(), [](const W& x) { return x.wide; });
  in.n_queries = batch_size;
  in.n_parts = num_q_entries;
  in.n_merge = batch_size;
  int64_t off = BE_PLAN_HEADER_INTS + (int64_t)items.size() * 8;
  in.off_work = BE_PLAN_HEADER_INTS;
  in.off_qlist = (int32_t)off;
  off += qlist.size();
  in.off_kvlist = (int32_t)off;
  in.off_merge_q = (int32_t)off;
  off += mq.size();
  in.off_merge_ptr = (int32_t)off;
  off += mptr.size();
  in.off_merge_parts = (int32_t)off;
  off += mparts.size();
  in.total_ints = (int32_t)off;
  in.page_size = page_size;
  in.group_size = g;
  in.any_slots = 1;
  for (auto& it : items) {
    const int len = it.w.kv_end - it.w.kv_begin;
    in.max_item_tokens = std::max(in.max_item_tokens, len);
    in.total_tokens += len;
    if (it.wide) in.max_wide_tokens = std::max(in.max_wide_tokens, len);
  }
  *info = in;
  if (off > plan_capacity || !plan) {
    set_error("plan buffer too small: need %lld ints, have %lld", (long long)off,
              (long long)plan_capacity);
    return BE_ECAPACITY;
  }
  std::memset(plan, 0, BE_PLAN_HEADER_INTS * sizeof(int32_t));
  std::memcpy(plan, &in, sizeof(in));
  int32_t* p = plan + BE_PLAN_HEADER_INTS;
  for (auto& it : items) {
    it.w.part_base = it.w.q_off;
    std::memcpy(p, &it.w, sizeof(be_attn_work));
    p += 8;
  }
  auto put = [&](const std::vector<int32_t>& v) {
    if (!v.empty()) std::memcpy(p, v.data(), v.size() * sizeof(int32_t));
    p += v.size();
  };
  put(qlist);
  put(mq);
  put(mptr);
  put(mparts);
  return BE_OK;
}

// FastTree vnodes as page-list groups (for the tensor-core decode kernels).
// In the beam trie every node starts at slot 0 of its page and every non-leaf
// node is full, so a vnode's token range [kv_off, kv_off + kv_len) of the slot
// table maps to whole pages: token t of the range lives in page
// slots[kv_off + t - t % ps] / ps at slot t % ps (checked at both ends of every
// page).  A vnode's requests may be any set (FastTree folds a small parent into
// some children's vnodes).  Returns BE_EINVAL (nothing written) when a range is
// not page aligned; the caller then plans with slot lists.
extern "C" int be_tree_plan_pages(int num_vnodes, const int32_t* q_entries, int num_q_entries,
                                  const int32_t* q_offs, const int32_t* q_lens,
                                  const int32_t* kv_offs, const int32_t* kv_lens,
                                  const int32_t* slots, int64_t num_slots, int batch_size,
                                  int page_size, int num_qo_heads, int num_kv_heads, int num_sms,
                                  int32_t* plan, int64_t plan_capacity, be_attn_plan_info* info) {
  if (num_vnodes < 0 || batch_size < 0 || page_size < 1 || num_kv_heads < 1 ||
      num_qo_heads % num_kv_heads || !info || !slots) {
    set_error("be_tree_plan_pages: invalid arguments");
    return BE_EINVAL;
  }
  const int g = num_qo_heads / num_kv_heads;
  if (g > 64) {
    set_error("be_tree_plan_pages: group size %d > 64 unsupported", g);
    return BE_EINVAL;
  }
  std::vector<Grp> groups;
  std::vector<int32_t> kvlist, gq;
  for (int v = 0; v < num_vnodes; ++v) {
    const int ql = q_lens[v], len = kv_lens[v];
    if (ql <= 0 || len <= 0) continue;
    if (q_offs[v] < 0 || q_offs[v] + ql > num_q_entries) {
      set_error("be_tree_plan_pages: vnode %d query range outside the entry list", v);
      return BE_EINVAL;
    }
    const int q_at = (int)gq.size();
    for (int e = 0; e < ql; ++e) {
      const int r = q_entries[q_offs[v] + e];
      if (r < 0 || r >= batch_size) {
        set_error("be_tree_plan_pages: vnode %d request %d outside the batch", v, r);
        return BE_EINVAL;
      }
      gq.push_back(r);
    }
    const int64_t off = kv_offs[v];
    if (off < 0 || off + len > num_slots) {
      set_error("be_tree_plan_pages: vnode %d token range outside the slot table", v);
      return BE_EINVAL;
    }
    const int kv_off = (int)kvlist.size();
    for (int t = 0; t < len; t += page_size) {
      const int m = std::min(page_size, len - t);   // tokens of this page in the range
      const int32_t s0 = slots[off + t], s1 = slots[off + t + m - 1];
      if (s0 < 0 || s0 % page_size != 0 || s1 != s0 + m - 1) {
        set_error("be_tree_plan_pages: vnode %d token %d is not page aligned", v, t);
        return BE_EINVAL;
      }
      kvlist.push_back(s0 / page_size);
    }
    groups.push_back({false, q_at, ql, kv_off, len});
  }
  return plan_groups(groups, gq, kvlist, batch_size, page_size, g, num_kv_heads, 0, num_sms, plan,
                     plan_capacity, info);
}

// True (1) when some query attends one page at two levels of a cascade plan:
// the reference's uneven-tree quirk (a candidate whose branch ends above the
// deepest level re-uses its deepest nodes at every later level,
// beam_state.py:299-302).  Pages are marked per query with a stamp.
extern "C" int be_cascade_pages_twice(int num_levels, const int32_t* const* qo_indptr,
                                      const int32_t* const* kv_indptr,
                                      const int32_t* const* kv_indices, const int32_t* num_groups,
                                      int num_queries) {
  if (num_levels < 0 || num_queries < 0) {
    set_error("be_cascade_pages_twice: invalid arguments");
    return -BE_EINVAL;
  }
  int32_t max_page = -1;
  for (int l = 0; l < num_levels; ++l) {
    const int G = num_groups[l];
    const int np = G > 0 ? kv_indptr[l][G] : 0;
    for (int i = 0; i < np; ++i) max_page = std::max(max_page, kv_indices[l][i]);
  }
  std::vector<int32_t> mark((size_t)max_page + 2, -1);
  std::vector<int> gi(num_levels, 0);   // current group of each level (queries ascend)
  for (int q = 0; q < num_queries; ++q) {
    for (int l = 0; l < num_levels; ++l) {
      const int G = num_groups[l];
      int& g = gi[l];
      while (g < G && qo_indptr[l][g + 1] <= q) ++g;
      if (g >= G || qo_indptr[l][g] > q) continue;   // q in no group of this level
      for (int i = kv_indptr[l][g]; i < kv_indptr[l][g + 1]; ++i) {
        const int32_t pg = kv_indices[l][i];
        if (pg < 0) continue;
        if (mark[pg] == q) return 1;
        mark[pg] = q;
      }
    }
  }
  return 0;
}

// ---------------------------------------------------------------------------
// Beam-tile plans (decode): tiles of consecutive queries, per-tile page entries
// with query ranges, pieces balanced by pages.
// ---------------------------------------------------------------------------
static_assert(sizeof(be_tile_plan_info) <= BE_PLAN_HEADER_INTS * sizeof(int32_t), "tile header");
static_assert(sizeof(be_attn_tile) == 8 * sizeof(int32_t), "tile layout");
static_assert(sizeof(be_attn_piece) == 24 * sizeof(int32_t), "piece layout");
static_assert(sizeof(be_attn_entry) == 4 * sizeof(int32_t), "entry layout");

extern "C" int be_tile_plan(int num_levels, const int32_t* const* qo_indptr,
                            const int32_t* const* kv_indptr, const int32_t* const* kv_indices,
                            const int32_t* const* last_page_len, const int32_t* num_groups,
                            int num_queries, int page_size, int num_qo_heads, int num_kv_heads,
                            int causal_last, int tile_rows, int target_pieces, int cluster,
                            int32_t* plan, int64_t plan_capacity, be_tile_plan_info* info) {
  if (num_levels < 0 || num_queries < 0 || page_size < 1 || num_kv_heads < 1 ||
      num_qo_heads % num_kv_heads || !info || (tile_rows != 64 && tile_rows != 128) ||
      cluster < -1 || cluster > 16) {
    set_error("be_tile_plan: invalid arguments");
    return BE_EINVAL;
  }
  const int g = num_qo_heads / num_kv_heads;
  const int R = tile_rows / g;   // queries per tile
  if (R < 1) {
    set_error("be_tile_plan: group size %d exceeds %d tile rows", g, tile_rows);
    return BE_ENOTSUP;
  }
  const int nq = num_queries;
  // level checks; a causal last level must be decode-shaped (<= 1 query per group)
  for (int l = 0; l < num_levels; ++l) {
    const int G = num_groups[l];
    if (G < 0) {
      set_error("be_tile_plan: level %d has a negative group count", l);
      return BE_EINVAL;
    }
    if (G > 0 && (qo_indptr[l][0] != 0 || kv_indptr[l][0] != 0 || qo_indptr[l][G] > nq)) {
      set_error("be_tile_plan: level %d indptr does not start at 0 or exceeds %d queries", l, nq);
      return BE_EINVAL;
    }
    for (int gi = 0; gi < G; ++gi) {
      const int qlen = qo_indptr[l][gi + 1] - qo_indptr[l][gi];
      const int np = kv_indptr[l][gi + 1] - kv_indptr[l][gi];
      if (qlen < 0 || np < 0) {
        set_error("be_tile_plan: level %d group %d has negative extent", l, gi);
        return BE_EINVAL;
      }
      const int last = last_page_len[l][gi];
      if (np > 0 && (last < 0 || last > page_size)) {
        set_error("be_tile_plan: level %d group %d last_page_len %d outside [0, %d]", l, gi, last,
                  page_size);
        return BE_EINVAL;
      }
      if (causal_last && l == num_levels - 1 && qlen > 1 && np > 0) {
        set_error("be_tile_plan: causal group with %d queries (prefill) is not a decode plan",
                  qlen);
        return BE_ENOTSUP;
      }
    }
  }
  // tiles: cut at level-0 group boundaries and every R queries
  struct TL {
    std::vector<int32_t> cut, q0, q1, tile_of, ecount, estart, efill, ents;
  };
  static thread_local TL S;
  S.cut.assign(nq + 1, 0);
  if (num_levels > 0)
    for (int gi = 0; gi <= num_groups[0]; ++gi) {
      const int q = qo_indptr[0][gi];
      if (q >= 0 && q <= nq) S.cut[q] = 1;
    }
  S.q0.clear();
  S.q1.clear();
  S.tile_of.assign(nq, 0);
  for (int q = 0; q < nq;) {
    const int a = q++;
    while (q < nq && !S.cut[q] && q - a < R) ++q;
    for (int i = a; i < q; ++i) S.tile_of[i] = (int32_t)S.q0.size();
    S.q0.push_back(a);
    S.q1.push_back(q);
  }
  const int nt = (int)S.q0.size();
  // entries: count per tile, then fill (tile-major, levels in order within a tile)
  S.ecount.assign(nt + 1, 0);
  for (int pass = 0; pass < 2; ++pass) {
    if (pass == 1) {
      S.estart.assign(nt + 1, 0);
      for (int t = 0; t < nt; ++t) S.estart[t + 1] = S.estart[t] + S.ecount[t];
      S.efill.assign(S.estart.begin(), S.estart.end() - 1);
      S.ents.resize((size_t)S.estart[nt] * 4);
    }
    for (int l = 0; l < num_levels; ++l) {
      for (int gi = 0; gi < num_groups[l]; ++gi) {
        const int a = qo_indptr[l][gi], b = std::min(nq, qo_indptr[l][gi + 1]);
        const int p0 = kv_indptr[l][gi], np = kv_indptr[l][gi + 1] - p0;
        if (a >= b || np <= 0) continue;
        for (int j = 0; j < np; ++j) {
          const int ntok = j == np - 1 ? last_page_len[l][gi] : page_size;
          if (ntok <= 0) continue;
          for (int t = S.tile_of[a]; t < nt && S.q0[t] < b; ++t) {
            if (pass == 0) {
              S.ecount[t]++;
            } else {
              int32_t* e = &S.ents[(size_t)S.efill[t]++ * 4];
              e[0] = kv_indices[l][p0 + j];
              e[1] = ntok;
              e[2] = std::max(a, S.q0[t]) - S.q0[t];
              e[3] = std::min(b, S.q1[t]) - S.q0[t];
            }
          }
        }
      }
    }
  }
  const int64_t n_ent = nt ? S.estart[nt] : 0;
  if (cluster < 0) {
    // auto: about target_pieces pieces over the tiles, as a cluster per (tile, KV
    // head) of a power-of-two size: clusters of up to 8 CTAs pack two CTAs per
    // SM into one wave (a cluster of 9 left CTAs waiting for a second wave), and
    // 16 only when half the target still fills the grid (16-CTA clusters of two
    // CTAs per SM did not all fit in one wave at 256 CTAs).  One piece per tile
    // needs no merge.
    const int per_tile = nt ? std::max(1, target_pieces) / nt : 1;
    cluster = 1;
    while (cluster * 2 <= std::min(per_tile, 8)) cluster *= 2;
    if (per_tile >= 32) cluster = 16;
    // few, long tiles (one prompt, a long prefix): the largest cluster caps a
    // tile at 16 pieces; when the tiles' entries would make at least half as
    // many pieces again (>= 8 entries each), the merge kernel's form keeps them
    // all (cfg4 state, one 128-row tile of 298 entries: 25 merged pieces 29.4 us
    // against 16 clustered 34.9 us)
    if (cluster == 16 && nt > 0) {
      const int64_t per_m = std::max<int64_t>(8, (n_ent + std::max(1, target_pieces) - 1) /
                                                     std::max(1, target_pieces));
      const int64_t np_m = (n_ent / nt + per_m / 2) / per_m;
      if (2 * np_m >= 3 * (int64_t)cluster) cluster = 0;
    }
    if (cluster == 1) cluster = 0;
  }
  // pieces: about target_pieces in all, >= 8 entries (two 4-page chunks) each,
  // sizes rounded to whole chunks
  const int64_t per = std::max<int64_t>(8, (n_ent + std::max(1, target_pieces) - 1) /
                                               std::max(1, target_pieces));
  static thread_local std::vector<int32_t> tiles, pieces;
  tiles.assign((size_t)nt * 8, 0);
  pieces.clear();
  int n_part = 0, max_pe = 0;
  int64_t tokens = 0;
  for (int t = 0; t < nt; ++t) {
    const int e0 = S.estart[t], e = S.estart[t + 1] - e0;
    int np, base;
    if (cluster > 1) {          // exactly `cluster` pieces, trailing ones may be empty
      np = cluster;
      base = std::max(4, ((e + np - 1) / np + 3) / 4 * 4);
    } else {
      np = (int)std::max<int64_t>(1, (e + per / 2) / per);
      base = (e + np - 1) / np;
      base = std::max(4, (base + 3) / 4 * 4);
      np = std::max(1, (e + base - 1) / base);
    }
    int32_t* T = &tiles[(size_t)t * 8];
    T[0] = S.q0[t];
    T[1] = S.q1[t] - S.q0[t];
    T[2] = (int32_t)(pieces.size() / 24);
    T[3] = np;
    T[4] = (np > 1 && cluster <= 1) ? n_part : -1;   // clusters merge on chip
    if (np > 1 && cluster <= 1) n_part += np;
    for (int k = 0; k < np; ++k) {
      const int b0 = e0 + std::min(e, k * base), b1 = e0 + std::min(e, (k + 1) * base);
      pieces.insert(pieces.end(), {t, b0, b1, k, T[0], T[1], T[3], T[4]});
      for (int j = 0; j < 4; ++j)       // the first chunk's entries, read with the piece
        for (int f = 0; f < 4; ++f)
          pieces.push_back(b0 + j < b1 ? S.ents[(size_t)(b0 + j) * 4 + f] : 0);
      max_pe = std::max(max_pe, b1 - b0);
    }
    for (int i = e0; i < e0 + e; ++i) tokens += S.ents[(size_t)i * 4 + 1];
  }
  be_tile_plan_info in{};
  in.n_tiles = nt;
  in.n_pieces = (int32_t)(pieces.size() / 24);
  in.n_entries = (int32_t)n_ent;
  in.n_queries = nq;
  int64_t off = BE_PLAN_HEADER_INTS;   // pieces first: a CTA finds its piece without the header
  in.off_pieces = (int32_t)off;
  off += pieces.size();
  in.off_tiles = (int32_t)off;
  off += tiles.size();
  in.off_entries = (int32_t)off;
  off += n_ent * 4;
  if (off > INT32_MAX || tokens > INT32_MAX) {
    set_error("be_tile_plan: plan too large (%lld ints)", (long long)off);
    return BE_EINVAL;
  }
  in.total_ints = (int32_t)off;
  in.page_size = page_size;
  in.group_size = g;
  in.tile_rows = tile_rows;
  in.n_part_pieces = n_part;
  in.total_tokens = (int32_t)tokens;
  in.max_piece_entries = max_pe;
  in.cluster = cluster > 1 ? cluster : 0;
  *info = in;
  if (off > plan_capacity || !plan) {
    set_error("plan buffer too small: need %lld ints, have %lld", (long long)off,
              (long long)plan_capacity);
    return BE_ECAPACITY;
  }
  std::memset(plan, 0, BE_PLAN_HEADER_INTS * sizeof(int32_t));
  std::memcpy(plan, &in, sizeof(in));
  if (!tiles.empty()) std::memcpy(plan + in.off_tiles, tiles.data(), tiles.size() * 4);
  if (!pieces.empty()) std::memcpy(plan + in.off_pieces, pieces.data(), pieces.size() * 4);
  if (n_ent) std::memcpy(plan + in.off_entries, S.ents.data(), (size_t)n_ent * 16);
  return BE_OK;
}
