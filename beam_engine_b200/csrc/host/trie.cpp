// Host page manager: FIFO page allocator + beam trie with copy-on-write forks,
// cascade / FastTree metadata builders and the vanilla beam selection.
//
// Semantics follow the reference (brian030128/beam_engine):
//   allocator            src/beam_engine/page_table.py:59-60, 77-124
//   trie + fork/free      src/beam_engine/beam_state.py:12-30, 76-209
//   cascade levels        src/beam_engine/beam_state.py:211-412
//   FastTree inputs       src/beam_engine/beam_state.py:414-633
//   FastTree planner      src/beam_engine/attention/fasttree/preparation.py:11-225
//   vanilla selection     src/beam_engine/beam_strategy.py:433-488
//   final ranking         src/beam_engine/beam_state.py:646-682
// Node ids are stable handles; pages are plain ints shared with the device pools.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <deque>
#include <numeric>
#include <unordered_map>
#include <vector>

#include "beam_b200.h"

namespace be {
void set_error(const char* fmt, ...);
}
using be::set_error;

struct be_trie {
  struct Node {
    int32_t parent = -1;
    int32_t page = -1;
    int64_t prefix = 0;   // tokens of the strict ancestors (kept by add_node / append_tok)
    std::vector<int32_t> tokens;
    std::vector<int32_t> children;
  };
  int page_size = 0;
  int max_pages = 0;
  std::deque<int32_t> free_pages;
  std::vector<char> allocated;
  std::vector<Node> nodes;
  std::vector<int32_t> level_memo;  // per call scratch
  std::vector<int32_t> head_memo;   // first node of the node's level segment (same gen)
  std::vector<int32_t> memo_gen;
  int32_t gen = 0;
  std::vector<int32_t> level_stack;  // scratch of level()
  std::vector<int32_t> node_mark, node_val, page_mark;   // stamped scratch of the builders
  int32_t stamp = 0;
  int64_t warnings = 0;

  int alloc(int32_t* out) {
    if (free_pages.empty()) {
      set_error("No free pages available");
      return BE_ENOMEM;
    }
    *out = free_pages.front();
    free_pages.pop_front();
    allocated[*out] = 1;
    return BE_OK;
  }
  int release(int32_t p) {
    if (p < 0 || p >= max_pages || !allocated[p]) {
      ++warnings;
      set_error("Page %d is not allocated", p);
      return BE_ENOT_ALLOCATED;
    }
    allocated[p] = 0;
    free_pages.push_back(p);
    return BE_OK;
  }
  int32_t add_node(int32_t parent, int32_t page, const int32_t* tok, int n) {
    Node nd;
    nd.parent = parent;
    nd.page = page;
    nd.tokens.assign(tok, tok + n);
    if (parent >= 0) nd.prefix = nodes[parent].prefix + (int64_t)nodes[parent].tokens.size();
    nodes.push_back(std::move(nd));
    const int32_t id = (int32_t)nodes.size() - 1;
    if (parent >= 0) nodes[parent].children.push_back(id);
    return id;
  }
  bool valid(int32_t n) const { return n >= 0 && n < (int32_t)nodes.size(); }
  void path(int32_t leaf, std::vector<int32_t>& out) const {
    out.clear();
    for (int32_t n = leaf; n >= 0; n = nodes[n].parent) out.push_back(n);
    std::reverse(out.begin(), out.end());
  }
  int64_t seq_len(int32_t leaf) const {
    return nodes[leaf].prefix + (int64_t)nodes[leaf].tokens.size();
  }
  // append one token; descendants (only a node built through the object API can
  // have any) get their ancestor lengths refreshed
  void append_tok(int32_t n, int32_t tok) {
    nodes[n].tokens.push_back(tok);
    if (nodes[n].children.empty()) return;
    std::vector<int32_t> st(nodes[n].children.begin(), nodes[n].children.end());
    while (!st.empty()) {
      const int32_t c = st.back();
      st.pop_back();
      const Node& par = nodes[nodes[c].parent];
      nodes[c].prefix = par.prefix + (int64_t)par.tokens.size();
      st.insert(st.end(), nodes[c].children.begin(), nodes[c].children.end());
    }
  }
  int32_t level(int32_t n) {
    // level(root) = 0; level(n) = level(parent) + (parent has > 1 children)
    auto& stack = level_stack;
    stack.clear();
    int32_t cur = n;
    while (cur >= 0 && memo_gen[cur] != gen) {
      stack.push_back(cur);
      cur = nodes[cur].parent;
    }
    int32_t lv = cur >= 0 ? level_memo[cur] : 0;
    for (auto it = stack.rbegin(); it != stack.rend(); ++it) {
      const int32_t p = nodes[*it].parent;
      const bool split = p >= 0 && nodes[p].children.size() > 1;
      lv = p < 0 ? 0 : lv + (split ? 1 : 0);
      level_memo[*it] = lv;
      head_memo[*it] = (p >= 0 && !split) ? head_memo[p] : *it;
      memo_gen[*it] = gen;
    }
    return level_memo[n];
  }
  void new_generation() {
    ++gen;
    if (level_memo.size() < nodes.size()) {
      level_memo.resize(nodes.size(), 0);
      head_memo.resize(nodes.size(), 0);
      memo_gen.resize(nodes.size(), 0);
    }
  }
  // fresh stamp for node_mark / page_mark (a mark equals `stamp` = set in this pass)
  int32_t next_stamp() {
    if (node_mark.size() < nodes.size()) {
      node_mark.resize(nodes.size(), 0);
      node_val.resize(nodes.size(), 0);
    }
    if ((int)page_mark.size() < max_pages) page_mark.resize(max_pages, 0);
    return ++stamp;
  }
};

extern "C" {

be_trie* be_trie_create(int page_size, int max_num_pages) {
  if (page_size < 1 || max_num_pages < 0) {
    set_error("be_trie_create: invalid page_size/max_num_pages");
    return nullptr;
  }
  auto* t = new be_trie();
  t->page_size = page_size;
  t->max_pages = max_num_pages;
  for (int i = 0; i < max_num_pages; ++i) t->free_pages.push_back(i);
  t->allocated.assign(max_num_pages, 0);
  return t;
}

void be_trie_destroy(be_trie* t) { delete t; }

int be_alloc_page(be_trie* t, int32_t* page) { return t->alloc(page); }
int be_free_page(be_trie* t, int32_t page) { return t->release(page); }
int be_num_free_pages(be_trie* t) { return (int)t->free_pages.size(); }
int be_is_allocated(be_trie* t, int32_t page) {
  return page >= 0 && page < t->max_pages && t->allocated[page];
}
int be_free_list(be_trie* t, int32_t* out, int cap) {
  const int n = (int)t->free_pages.size();
  for (int i = 0; i < n && i < cap; ++i) out[i] = t->free_pages[i];
  return n;
}
int64_t be_trie_warnings(be_trie* t) { return t->warnings; }
int be_trie_num_nodes(be_trie* t) { return (int)t->nodes.size(); }

int be_node_new(be_trie* t, int32_t parent, int32_t page, const int32_t* tokens, int n,
                int32_t* node_out) {
  if (parent >= 0 && !t->valid(parent)) {
    set_error("be_node_new: bad parent %d", parent);
    return BE_EINVAL;
  }
  *node_out = t->add_node(parent, page, tokens, n);
  return BE_OK;
}

int be_node_info(be_trie* t, int32_t node, int32_t* parent, int32_t* page, int32_t* ntokens,
                 int32_t* nchildren) {
  if (!t->valid(node)) {
    set_error("be_node_info: bad node %d", node);
    return BE_EINVAL;
  }
  const auto& nd = t->nodes[node];
  if (parent) *parent = nd.parent;
  if (page) *page = nd.page;
  if (ntokens) *ntokens = (int32_t)nd.tokens.size();
  if (nchildren) *nchildren = (int32_t)nd.children.size();
  return BE_OK;
}

int be_node_tokens(be_trie* t, int32_t node, int32_t* out, int cap) {
  if (!t->valid(node)) return -1;
  const auto& v = t->nodes[node].tokens;
  for (int i = 0; i < (int)v.size() && i < cap; ++i) out[i] = v[i];
  return (int)v.size();
}

int be_node_children(be_trie* t, int32_t node, int32_t* out, int cap) {
  if (!t->valid(node)) return -1;
  const auto& v = t->nodes[node].children;
  for (int i = 0; i < (int)v.size() && i < cap; ++i) out[i] = v[i];
  return (int)v.size();
}

int be_node_append_token(be_trie* t, int32_t node, int32_t token) {
  if (!t->valid(node)) {
    set_error("be_node_append_token: bad node %d", node);
    return BE_EINVAL;
  }
  t->append_tok(node, token);
  return BE_OK;
}

// Token sequence root -> leaf; returns its length (writes up to cap tokens).
int64_t be_node_sequence(be_trie* t, int32_t leaf, int32_t* out, int64_t cap) {
  if (!t->valid(leaf)) return -1;
  std::vector<int32_t> p;
  t->path(leaf, p);
  int64_t k = 0;
  for (int32_t n : p)
    for (int32_t tok : t->nodes[n].tokens) {
      if (k < cap) out[k] = tok;
      ++k;
    }
  return k;
}

// Token sequences of many leaves as CSR (DiverseBeamSearchStrategy.
// _get_sequence_from_node, beam_strategy.py:96-103): tokens of the leaf's
// ancestors front to back, stopping at the first node (walking up) that holds
// no tokens.  seq_ptr [n + 1]; seq_tokens is written while it has room (cap);
// returns the total, -1 for an unknown leaf.
int64_t be_leaf_sequences(be_trie* t, int n, const int32_t* leaves, int32_t* seq_ptr,
                          int32_t* seq_tokens, int64_t cap) {
  int64_t k = 0;
  seq_ptr[0] = 0;
  std::vector<int32_t> chain;
  for (int i = 0; i < n; ++i) {
    if (!t->valid(leaves[i])) {
      set_error("be_leaf_sequences: unknown node %d", leaves[i]);
      return -1;
    }
    chain.clear();
    for (int32_t c = leaves[i]; c >= 0 && !t->nodes[c].tokens.empty(); c = t->nodes[c].parent)
      chain.push_back(c);
    for (auto it = chain.rbegin(); it != chain.rend(); ++it)
      for (int32_t tok : t->nodes[*it].tokens) {
        if (seq_tokens && k < cap) seq_tokens[k] = tok;
        ++k;
      }
    seq_ptr[i + 1] = (int32_t)k;
  }
  return k;
}

// BeamState.add_root_sequence (beam_state.py:76-98).
int be_beam_add_root(be_trie* t, const int32_t* tokens, int n, int32_t* leaf_out,
                     int32_t* pages_out) {
  int32_t cur = -1;
  int k = 0;
  for (int s = 0; s < n; s += t->page_size) {
    int32_t page;
    int rc = t->alloc(&page);
    if (rc) return rc;
    const int e = std::min(n, s + t->page_size);
    cur = t->add_node(cur, page, tokens + s, e - s);
    if (pages_out) pages_out[k] = page;
    ++k;
  }
  *leaf_out = cur;
  return BE_OK;
}

// BeamState.add_filtered_results (beam_state.py:101-209).
// Candidate i's children are child_tokens[child_ptr[i] .. child_ptr[i+1]).
// Outputs, in the reference's new-candidate order: new_leaf[k] and new_child[k]
// (index into child_tokens, to carry the score), count in *n_new; the
// copy-on-write copies (src page, dst page, tokens) in issue order, count in
// *n_copies.  Output arrays need room for child_ptr[ncand] entries.
int be_beam_update(be_trie* t, int ncand, const int32_t* cand_leaf, const int32_t* child_ptr,
                   const int32_t* child_tokens, int32_t* new_leaf, int32_t* new_child,
                   int32_t* n_new, int32_t* copy_src, int32_t* copy_dst, int32_t* copy_len,
                   int32_t* n_copies) {
  for (int i = 0; i < ncand; ++i)
    if (!t->valid(cand_leaf[i])) {
      set_error("be_beam_update: bad leaf %d", cand_leaf[i]);
      return BE_EINVAL;
    }
  // 1. free dead branches upward
  for (int i = 0; i < ncand; ++i) {
    if (child_ptr[i + 1] > child_ptr[i]) continue;
    int32_t n = cand_leaf[i];
    while (n >= 0 && t->nodes[n].children.empty()) {
      t->release(t->nodes[n].page);
      const int32_t par = t->nodes[n].parent;
      if (par >= 0) {
        auto& ch = t->nodes[par].children;
        auto it = std::find(ch.begin(), ch.end(), n);
        if (it != ch.end()) ch.erase(it);
      }
      n = par;
    }
  }
  // 2. expand survivors
  int k = 0, c = 0;
  const int ps = t->page_size;
  for (int i = 0; i < ncand; ++i) {
    const int c0 = child_ptr[i], c1 = child_ptr[i + 1];
    if (c1 <= c0) continue;
    const int32_t nid = cand_leaf[i];
    if (c1 - c0 == 1) {
      if ((int)t->nodes[nid].tokens.size() < ps) {
        t->append_tok(nid, child_tokens[c0]);
        new_leaf[k] = nid;
      } else {
        int32_t page;
        int rc = t->alloc(&page);
        if (rc) return rc;
        new_leaf[k] = t->add_node(nid, page, &child_tokens[c0], 1);
      }
      new_child[k++] = c0;
      continue;
    }
    if ((int)t->nodes[nid].tokens.size() == ps) {
      for (int j = c0; j < c1; ++j) {
        int32_t page;
        int rc = t->alloc(&page);
        if (rc) return rc;
        new_leaf[k] = t->add_node(nid, page, &child_tokens[j], 1);
        new_child[k++] = j;
      }
    } else {
      const std::vector<int32_t> base = t->nodes[nid].tokens;
      const int32_t src_page = t->nodes[nid].page;
      for (int j = c0 + 1; j < c1; ++j) {
        int32_t page;
        int rc = t->alloc(&page);
        if (rc) return rc;
        copy_src[c] = src_page;
        copy_dst[c] = page;
        copy_len[c] = (int32_t)base.size();
        ++c;
        std::vector<int32_t> tk = base;
        tk.push_back(child_tokens[j]);
        new_leaf[k] = t->add_node(t->nodes[nid].parent, page, tk.data(), (int)tk.size());
        new_child[k++] = j;
      }
      t->append_tok(nid, child_tokens[c0]);
      new_leaf[k] = nid;
      new_child[k++] = c0;
    }
  }
  *n_new = k;
  *n_copies = c;
  return BE_OK;
}

// Per-candidate decode inputs (beam.py:168-221): query token (last token of the
// leaf, 0 if empty), append target (leaf page, len(leaf tokens) - 1) and the
// RoPE position (sequence length - 1).
int be_beam_step_inputs(be_trie* t, int ncand, const int32_t* cand_leaf, int32_t* query_tok,
                        int32_t* write_page, int32_t* write_pos, int32_t* position) {
  for (int i = 0; i < ncand; ++i) {
    const int32_t n = cand_leaf[i];
    if (!t->valid(n)) {
      set_error("be_beam_step_inputs: bad leaf %d", n);
      return BE_EINVAL;
    }
    const auto& nd = t->nodes[n];
    if (query_tok) query_tok[i] = nd.tokens.empty() ? 0 : nd.tokens.back();
    if (write_page) write_page[i] = nd.page;
    if (write_pos) write_pos[i] = (int32_t)nd.tokens.size() - 1;
    if (position) position[i] = (int32_t)(t->seq_len(n) - 1);
  }
  return BE_OK;
}

// BeamState.get_cascade_input (beam_state.py:211-412).  Writes, per level l,
// groups qo/kv indptr, page list and last-page lengths into flat arrays:
// level l's groups are level_group_ptr[l]..[l+1] (qo_indptr/kv_indptr/last use
// one entry per group plus a leading 0 per level for the indptrs), its pages
// level_page_ptr[l]..[l+1].  Returns the number of levels (>= 0) or -status.
// Capacities: levels <= cap_levels, groups <= cap_groups, pages <= cap_pages.
int be_cascade_build(be_trie* t, int ncand, const int32_t* cand_leaf, int cap_levels,
                     int cap_groups, int cap_pages, int32_t* level_group_ptr,
                     int32_t* level_page_ptr, int32_t* qo_indptr, int32_t* kv_indptr,
                     int32_t* kv_indices, int32_t* last_page_len) {
  t->new_generation();
  // A candidate's root path splits into one segment per level 0..level(leaf):
  // segment lv runs from head (first node of the level) to the node before the
  // next level's head.  level() memoises each node's level and head for this
  // generation, so walking a path hops once per level instead of once per node.
  struct Seg {
    int32_t first, last;  // node ids, first is an ancestor of (or equal to) last
  };
  struct G {
    int cand0, count;
    Seg seg;
  };
  struct Scratch {
    std::vector<std::vector<Seg>> segs;  // by candidate, by level
    std::vector<int32_t> chain;
    std::vector<G> groups;
  };
  static thread_local Scratch tls;   // looked up once (TLS access is a call in a shared library)
  Scratch& S = tls;
  auto& segs = S.segs;
  auto& chain = S.chain;
  auto& groups = S.groups;
  if ((int)segs.size() < ncand) segs.resize(ncand);
  int top = 0;
  for (int c = 0; c < ncand; ++c) {
    if (!t->valid(cand_leaf[c])) {
      set_error("be_cascade_build: bad leaf %d", cand_leaf[c]);
      return -BE_EINVAL;
    }
    auto& sg = segs[c];
    const int32_t leaf = cand_leaf[c];
    const int lv_leaf = t->level(leaf);
    sg.resize(lv_leaf + 1);
    int32_t x = leaf;
    for (int lv = lv_leaf; lv >= 0; --lv) {
      const int32_t h = t->head_memo[x];
      sg[lv] = {h, x};
      x = t->nodes[h].parent;
    }
    top = std::max(top, lv_leaf);
  }
  const int nlev = ncand > 0 ? top + 1 : 0;
  if (nlev > cap_levels) {
    set_error("be_cascade_build: %d levels exceed capacity %d", nlev, cap_levels);
    return -BE_ECAPACITY;
  }
  int gbase = 0, pbase = 0;
  for (int lv = 0; lv < nlev; ++lv) {
    level_group_ptr[lv] = gbase;
    level_page_ptr[lv] = pbase;
    // group of a key node this level: node_val[key] when node_mark[key] == stamp
    const int32_t kst = t->next_stamp();
    groups.clear();
    for (int c = 0; c < ncand; ++c) {
      const auto& sg = segs[c];
      // a candidate with no segment this deep reuses its deepest one
      const Seg s = lv < (int)sg.size() ? sg[lv] : sg.back();
      const int32_t key = s.last;
      if (t->node_mark[key] != kst) {
        t->node_mark[key] = kst;
        t->node_val[key] = (int32_t)groups.size();
        groups.push_back({c, 1, s});
      } else {
        groups[t->node_val[key]].count++;
      }
    }
    if (gbase + (int)groups.size() > cap_groups) {
      set_error("be_cascade_build: group capacity %d exceeded", cap_groups);
      return -BE_ECAPACITY;
    }
    // indptr arrays carry one leading zero per level: level lv occupies
    // [gbase + lv, gbase + lv + ngroups]
    int32_t* qo = qo_indptr + gbase + lv;
    int32_t* kvp = kv_indptr + gbase + lv;
    qo[0] = 0;
    kvp[0] = 0;
    int npages = 0;
    for (size_t gi = 0; gi < groups.size(); ++gi) {
      const auto& g = groups[gi];
      chain.clear();   // the segment's nodes, last to first
      for (int32_t x = g.seg.last;; x = t->nodes[x].parent) {
        chain.push_back(x);
        if (x == g.seg.first) break;
      }
      const int32_t pst = t->next_stamp();   // pages already listed for this group
      for (auto it = chain.rbegin(); it != chain.rend(); ++it) {
        const int32_t pg = t->nodes[*it].page;
        if (pg >= 0 && pg < t->max_pages) {
          if (t->page_mark[pg] == pst) continue;
          t->page_mark[pg] = pst;
        }
        if (pbase + npages >= cap_pages) {
          set_error("be_cascade_build: page capacity %d exceeded", cap_pages);
          return -BE_ECAPACITY;
        }
        kv_indices[pbase + npages++] = pg;
      }
      const int32_t tail = g.seg.last;
      const int ln = (int)t->nodes[tail].tokens.size();
      last_page_len[gbase + gi] = (tail == cand_leaf[g.cand0]) ? std::max(0, ln - 1) : ln;
      kvp[gi + 1] = npages;
      qo[gi + 1] = qo[gi] + g.count;
    }
    gbase += (int)groups.size();
    pbase += npages;
  }
  level_group_ptr[nlev] = gbase;
  level_page_ptr[nlev] = pbase;
  return nlev;
}

// BeamState._build_kv_tree_structure + _build_req_to_token (beam_state.py:414-564).
// Nodes in BFS order from the roots: node_parent / node_seqlen / node_children
// and their request lists (CSR req_ptr / req_list); per_node != 0 gives each
// node's own token count as seqlen (the reference stores the cumulative length,
// which its planner then misreads as a per-node length).  page_size > 0
// overrides the trie's page size for the slot ids.  req_to_token is
// [ncand][*max_len] slot ids (page * page_size + i), zero padded; pass
// req_to_token = NULL to query *max_len and *num_nodes first.
int be_tree_build(be_trie* t, int ncand, const int32_t* cand_leaf, int per_node, int page_size,
                  int cap_nodes,
                  int32_t* num_nodes, int32_t* node_parent, int32_t* node_seqlen,
                  int32_t* node_children, int32_t* req_ptr, int32_t* req_list,
                  int64_t cap_req_list, int32_t* max_len, int32_t* req_to_token,
                  int64_t cap_req_to_token) {
  // per_node bit 1: one tree node per chain of trie nodes with a single live
  // child (a 1024-token prefix is one node, not 64); needs per-node lengths
  const bool compress = (per_node & 2) != 0;
  const bool own_len = (per_node & 1) != 0 || compress;
  // per-thread scratch, node-indexed arrays validated by stamps (no clearing,
  // no hash maps): live children lists (compress) and trie node -> tree node
  struct Scratch {
    std::vector<std::vector<int32_t>> paths, lk_lists;
    std::vector<int32_t> lk_stamp, lk_slot, tid_stamp, tid_val, vis_stamp, vis_cand, vis_pos, up;
    std::vector<int32_t> fresh, src_cand;   // per candidate: first new path index, copied-from
    int32_t stamp = 0;
  };
  static thread_local Scratch tls;
  Scratch& S = tls;
  if (S.lk_stamp.size() < t->nodes.size()) {
    S.lk_stamp.resize(t->nodes.size(), 0);
    S.lk_slot.resize(t->nodes.size(), 0);
    S.tid_stamp.resize(t->nodes.size(), 0);
    S.tid_val.resize(t->nodes.size(), 0);
    S.vis_stamp.resize(t->nodes.size(), 0);
    S.vis_cand.resize(t->nodes.size(), 0);
    S.vis_pos.resize(t->nodes.size(), 0);
  }
  const int32_t st = ++S.stamp;
  std::vector<int32_t> roots;
  auto& paths = S.paths;
  if ((int)paths.size() < ncand) paths.resize(ncand);
  S.fresh.assign(ncand, 0);
  S.src_cand.assign(ncand, -1);
  int64_t ml = 0;
  for (int c = 0; c < ncand; ++c) {
    if (!t->valid(cand_leaf[c])) {
      set_error("be_tree_build: bad leaf %d", cand_leaf[c]);
      return BE_EINVAL;
    }
    // root path: walk up to the first node an earlier candidate's path holds
    // and copy that path's prefix (candidates share long prefixes)
    auto& up = S.up;
    up.clear();
    int32_t a = cand_leaf[c];
    while (a >= 0 && S.vis_stamp[a] != st) {
      up.push_back(a);
      a = t->nodes[a].parent;
    }
    auto& pc = paths[c];
    pc.clear();
    if (a >= 0) {
      const auto& src = paths[S.vis_cand[a]];
      pc.insert(pc.end(), src.begin(), src.begin() + S.vis_pos[a] + 1);
      S.src_cand[c] = S.vis_cand[a];
    }
    S.fresh[c] = (int32_t)pc.size();
    for (auto it = up.rbegin(); it != up.rend(); ++it) {
      S.vis_stamp[*it] = st;
      S.vis_cand[*it] = c;
      S.vis_pos[*it] = (int32_t)pc.size();
      pc.push_back(*it);
    }
    if (std::find(roots.begin(), roots.end(), pc[0]) == roots.end()) roots.push_back(pc[0]);
    ml = std::max(ml, t->seq_len(cand_leaf[c]));
  }
  // live children (on some candidate's path) of every live trie node, in order
  // of first appearance
  int n_lists = 0;
  auto live_list = [&](int32_t n) -> std::vector<int32_t>* {
    return S.lk_stamp[n] == st ? &S.lk_lists[S.lk_slot[n]] : nullptr;
  };
  if (compress) {
    for (int c = 0; c < ncand; ++c)   // pairs inside a copied prefix were seen already
      for (size_t i = (size_t)std::max(0, S.fresh[c] - 1); i + 1 < paths[c].size(); ++i) {
        const int32_t a = paths[c][i], b = paths[c][i + 1];
        if (S.lk_stamp[a] != st) {
          S.lk_stamp[a] = st;
          S.lk_slot[a] = n_lists;
          if ((int)S.lk_lists.size() <= n_lists) S.lk_lists.emplace_back();
          S.lk_lists[n_lists++].clear();
        }
        auto& v = S.lk_lists[S.lk_slot[a]];
        if (std::find(v.begin(), v.end(), b) == v.end()) v.push_back(b);
      }
  }
  auto chain_end = [&](int32_t n) {   // last trie node of the chain starting at n
    if (!compress) return n;
    for (;;) {
      const auto* v = live_list(n);
      if (!v || v->size() != 1) return n;
      n = (*v)[0];
    }
  };
  static const std::vector<int32_t> kNone;
  auto kids_of = [&](int32_t last) -> const std::vector<int32_t>& {
    if (!compress) return t->nodes[last].children;
    const auto* v = live_list(last);
    return v ? *v : kNone;
  };
  auto has_tid = [&](int32_t n) { return S.tid_stamp[n] == st; };
  // tree nodes in BFS order; a node is a chain head (one trie node unless compressed)
  std::vector<int32_t> order, order_last;
  std::deque<int32_t> q(roots.begin(), roots.end());
  while (!q.empty()) {
    const int32_t n = q.front();
    q.pop_front();
    if (has_tid(n)) continue;
    const int32_t id = (int32_t)order.size();
    const int32_t last = chain_end(n);
    for (int32_t m = last;; m = t->nodes[m].parent) {
      S.tid_stamp[m] = st;
      S.tid_val[m] = id;
      if (m == n) break;
    }
    order.push_back(n);
    order_last.push_back(last);
    for (int32_t ch : kids_of(last))
      if (!has_tid(ch)) q.push_back(ch);
  }
  *num_nodes = (int32_t)order.size();
  *max_len = (int32_t)ml;
  if (!req_to_token) return BE_OK;
  if ((int)order.size() > cap_nodes || (int64_t)ncand * ml > cap_req_to_token) {
    set_error("be_tree_build: capacity exceeded");
    return BE_ECAPACITY;
  }
  for (size_t i = 0; i < order.size(); ++i) {
    const auto& head = t->nodes[order[i]];
    const int32_t last = order_last[i];
    node_parent[i] = head.parent < 0 ? -1 : (has_tid(head.parent) ? S.tid_val[head.parent] : -1);
    int64_t len = 0;
    for (int32_t m = last;; m = t->nodes[m].parent) {
      len += (int64_t)t->nodes[m].tokens.size();
      if (m == order[i]) break;
    }
    node_seqlen[i] = own_len ? (int32_t)len : (int32_t)t->seq_len(last);
    node_children[i] = (int32_t)kids_of(last).size();
  }
  // requests per node (candidate order): a candidate's path passes whole tree
  // nodes, so its tree nodes are its leaf's node and that node's ancestors
  std::vector<std::vector<int32_t>> reqs(order.size());
  for (int c = 0; c < ncand; ++c)
    for (int32_t tn = S.tid_val[cand_leaf[c]]; tn >= 0; tn = node_parent[tn]) reqs[tn].push_back(c);
  int64_t rp = 0;
  for (size_t i = 0; i < order.size(); ++i) {
    req_ptr[i] = (int32_t)rp;
    for (int32_t r : reqs[i]) {
      if (rp >= cap_req_list) {
        set_error("be_tree_build: request list capacity exceeded");
        return BE_ECAPACITY;
      }
      req_list[rp++] = r;
    }
  }
  req_ptr[order.size()] = (int32_t)rp;
  const int ps = page_size > 0 ? page_size : t->page_size;
  for (int c = 0; c < ncand; ++c) {
    int32_t* row = req_to_token + (int64_t)c * ml;
    int64_t k = 0;
    size_t i0 = 0;
    const auto& pc = paths[c];
    if (S.src_cand[c] >= 0 && S.fresh[c] < (int32_t)pc.size()) {
      // the prefix shared with an earlier candidate: copy its slots
      k = t->nodes[pc[S.fresh[c]]].prefix;
      std::memcpy(row, req_to_token + (int64_t)S.src_cand[c] * ml, (size_t)k * sizeof(int32_t));
      i0 = (size_t)S.fresh[c];
    }
    for (size_t j = i0; j < pc.size(); ++j) {
      const auto& nd = t->nodes[pc[j]];
      const int32_t base = nd.page * ps;
      for (size_t i = 0; i < nd.tokens.size(); ++i) row[k++] = base + (int32_t)i;
    }
    for (; k < ml; ++k) row[k] = 0;
  }
  return BE_OK;
}

// prepare_fasttree_metadata_for_paged_cache (preparation.py:11-225, parameters
// metadata.py:12-38): SplitK/SplitQ cost model per edge, merged request sets,
// vnode emission with KV splits, req->vnode lists and the two-phase reorder.
// Tree arrays as written by be_tree_build.  Output capacities: cap_vnodes for
// the per-vnode arrays, cap_entries for q_entries / r2v_entries.  counts[0] =
// vnodes, counts[1] = entries, counts[2..3] = phase node counts.
int be_fasttree_prepare(int num_nodes, const int32_t* node_parent, const int32_t* node_seqlen,
                        const int32_t* node_children, const int32_t* req_ptr,
                        const int32_t* req_list, int64_t req_to_token_stride, int batch_size,
                        int num_qo_heads, int num_kv_heads, int cap_vnodes, int cap_entries,
                        int32_t* q_entries, int32_t* q_offs, int32_t* q_lens, int32_t* kv_offs,
                        int32_t* kv_lens, int32_t* r2v_entries, int32_t* r2v_offs,
                        int32_t* r2v_lens, int32_t* counts) {
  if (num_kv_heads < 1 || num_qo_heads % num_kv_heads) {
    set_error("be_fasttree_prepare: bad head counts");
    return BE_EINVAL;
  }
  const int g = num_qo_heads / num_kv_heads;
  const int tsq[2] = {std::max(1, 64 / g), std::max(1, 16 / g)};
  const int tsk[2] = {32, 32};
  const int split[2] = {1024, 1024};  // preparation.py:39 uses kv_split_sizes[0] for both phases
  const double alpha = 0.6, beta = 0.3, gamma = 0.1;
  // Python's floor modulo: ((n - 1) % ts) is ts - 1 for n = 0
  auto padq = [](int ts, int n) { return ts - ((((n - 1) % ts) + ts) % ts + 1); };
  auto padk = [](int ts, int n) { return std::max(0, ts - n); };
  auto cmm = [&](int nq, int nk) {
    const int ph = nq > tsq[1] ? 0 : 1;
    return alpha * padq(tsq[ph], nq) * g * nk + beta * padk(tsk[ph], nk) * nq * g;
  };
  const int n = num_nodes;
  auto nreq = [&](int i) { return req_ptr[i + 1] - req_ptr[i]; };
  std::vector<std::vector<int>> kids(n);
  for (int i = 0; i < n; ++i)
    if (node_parent[i] != -1) kids[node_parent[i]].push_back(i);
  std::vector<int64_t> L(node_seqlen, node_seqlen + n);
  std::vector<int> merged(n, 0);
  if (n > 0) {
    // BFS from every root: the reference decodes one prompt (one root, node 0);
    // several prompts decoded together make a forest
    std::deque<int> fifo;
    for (int i = 0; i < n; ++i)
      if (node_parent[i] == -1) fifo.push_back(i);
    while (!fifo.empty()) {
      const int v = fifo.front();
      fifo.pop_front();
      int nq_cur = nreq(v);
      const int64_t lenv = L[v];
      for (int c : kids[v]) {
        const int nql = nreq(c);
        const int64_t lenl = L[c];
        const double sk = cmm(nq_cur, (int)lenv) + cmm(nql, (int)lenl) + gamma * nql;
        const double sq = cmm(nq_cur - nql, (int)lenv) + cmm(nql, (int)(lenl + lenv));
        if (sk > sq) {
          merged[c] = 1;
          nq_cur -= nql;
          L[c] = lenl + lenv;
        }
        fifo.push_back(c);
      }
    }
  }
  std::vector<std::vector<int32_t>> node_reqs(n);
  std::deque<int> fifo;
  for (int i = 0; i < n; ++i)
    if (node_children[i] == 0) {
      fifo.push_back(i);
      node_reqs[i].assign(req_list + req_ptr[i], req_list + req_ptr[i + 1]);
    }
  std::vector<int> vkids(node_children, node_children + n);
  while (!fifo.empty()) {
    const int v = fifo.front();
    fifo.pop_front();
    const int par = node_parent[v];
    if (par < 0) continue;   // a root: its requests stay with it (node 0 in the reference)
    if (merged[v] == 0)
      node_reqs[par].insert(node_reqs[par].end(), req_list + req_ptr[v], req_list + req_ptr[v + 1]);
    vkids[par] -= 1;
    if (vkids[par] == 0) fifo.push_back(par);
  }
  std::vector<int64_t> tok_off(n, 0);
  // token offset of each node within its requests' rows (roots start at 0); nodes
  // are in BFS order, so a parent's offset is known before its children's
  for (int i = 0; i < n; ++i)
    tok_off[i] = node_parent[i] < 0 ? 0 : tok_off[node_parent[i]] + node_seqlen[node_parent[i]];
  std::vector<int32_t> qe, qo, ql, ko, kl;
  for (int i = 0; i < n; ++i) {
    const auto& reqs = node_reqs[i];
    if (reqs.empty()) continue;
    int64_t kv_len = node_seqlen[i];
    int v = i;
    while (merged[v] == 1) {
      v = node_parent[v];
      kv_len += node_seqlen[v];
    }
    const int nr = (int)reqs.size();
    const int ph = nr > tsq[1] ? 0 : 1;
    const int kvs = split[ph], qs = tsq[ph];
    const int64_t kv_start = req_to_token_stride * reqs[0] + tok_off[v];
    for (int64_t s = 0; s < (kv_len - 1) / kvs + 1; ++s) {
      const int q0 = (int)qe.size();
      qe.insert(qe.end(), reqs.begin(), reqs.end());
      const int64_t koff = s * kvs;
      const int64_t klen = std::min<int64_t>(koff + kvs, kv_len) - koff;
      for (int j = 0; j < (nr - 1) / qs + 1; ++j) {
        const int qoff = j * qs;
        ko.push_back((int32_t)(kv_start + koff));
        kl.push_back((int32_t)klen);
        qo.push_back(q0 + qoff);
        ql.push_back(std::min(qoff + qs, nr) - qoff);
      }
    }
  }
  const int nv = (int)ko.size(), ne = (int)qe.size();
  if (nv > cap_vnodes || ne > cap_entries) {
    set_error("be_fasttree_prepare: %d vnodes / %d entries exceed capacity", nv, ne);
    counts[0] = nv;
    counts[1] = ne;
    return BE_ECAPACITY;
  }
  std::vector<std::vector<int32_t>> r2v(batch_size);
  for (int e = 0; e < ne; ++e) r2v[qe[e]].push_back(e);
  int off = 0, k = 0;
  for (int b = 0; b < batch_size; ++b) {
    r2v_offs[b] = off;
    r2v_lens[b] = (int32_t)r2v[b].size();
    off += (int)r2v[b].size();
    for (int32_t e : r2v[b]) r2v_entries[k++] = e;
  }
  std::copy(qe.begin(), qe.end(), q_entries);
  int w = 0, above = 0;
  for (int pass = 0; pass < 2; ++pass)
    for (int i = 0; i < nv; ++i) {
      const bool is_above = ql[i] > tsq[1];
      if ((pass == 0) != is_above) continue;
      q_offs[w] = qo[i];
      q_lens[w] = ql[i];
      kv_offs[w] = ko[i];
      kv_lens[w] = kl[i];
      ++w;
      if (pass == 0) ++above;
    }
  counts[0] = nv;
  counts[1] = ne;
  counts[2] = above;
  counts[3] = nv - above;
  return BE_OK;
}

// VanillaBeamSearchStrategy.select_candidates (beam_strategy.py:433-488).
// Candidate i offers k children (tokens[i*k + j], logps[i*k + j], in top-k
// order; the reference's log-probs are fp32 values held as Python floats); totals are parent_scores[i] + logp in double; a stable descending
// sort keeps the first beam_size; results regroup per parent in sorted order.
// Outputs: child_ptr [n+1], child_tokens / child_scores [beam_size].
int be_vanilla_select(int n, int k, const double* parent_scores, const int32_t* tokens,
                      const double* logps, int beam_size, int32_t* child_ptr,
                      int32_t* child_tokens, double* child_scores) {
  // Global top-beam_size of parent + logp in the order of a stable sort by
  // score (ties: candidate order, then top-k order), then grouped by parent.
  // Only the first beam_size of that order matter, so a partial sort with the
  // index as the tie-break gives the same result as the full stable sort.
  const int64_t total = (int64_t)n * k;
  // per-thread scratch, looked up once per call (a thread_local in a shared
  // library costs a TLS call per access otherwise)
  struct Scratch {
    std::vector<int64_t> idx;
    std::vector<double> sc;
    std::vector<int32_t> cnt, head, off;
  };
  static thread_local Scratch tls;
  Scratch& S = tls;
  auto& idx = S.idx;
  auto& sc = S.sc;
  idx.resize(total);
  sc.resize(total);
  for (int i = 0; i < n; ++i) {   // nested loops: no 64-bit division per element
    const double ps = parent_scores[i];
    const int64_t b = (int64_t)i * k;
    for (int j = 0; j < k; ++j) {
      idx[b + j] = b + j;
      sc[b + j] = ps + logps[b + j];
    }
  }
  const int64_t keep = std::min<int64_t>(beam_size, total);
  auto before = [&](int64_t a, int64_t b) {   // the stable sort's order
    return sc[a] > sc[b] || (!(sc[b] > sc[a]) && a < b);
  };
  // Rows straight from a top-k are already in that order (parent + logp is
  // non-increasing along a row, ties keep the row order): merge the row heads
  // instead of sorting.  Otherwise (or with NaNs) a partial sort.
  bool rows_sorted = n <= 64;
  for (int i = 0; rows_sorted && i < n; ++i) {
    const double* r = sc.data() + (int64_t)i * k;
    for (int j = 0; j < k; ++j)
      if (std::isnan(r[j]) || (j + 1 < k && r[j + 1] > r[j])) {
        rows_sorted = false;
        break;
      }
  }
  auto& row = S.cnt;   // parent row of each kept entry
  row.resize(std::max<int64_t>(keep, n + 1));
  if (rows_sorted) {
    // equal scores: the lower row comes first (its flat index is smaller), so a
    // strict '>' scan over the rows in order picks exactly the stable order
    auto& head = S.head;
    head.assign(n, 0);
    for (int64_t r = 0; r < keep; ++r) {
      int bi = -1;
      double bs = 0.0;
      for (int i = 0; i < n; ++i) {
        if (head[i] >= k) continue;
        const double v = sc[(int64_t)i * k + head[i]];
        if (bi < 0 || v > bs) {
          bi = i;
          bs = v;
        }
      }
      idx[r] = (int64_t)bi * k + head[bi];
      row[r] = bi;
      head[bi]++;
    }
  } else {
    std::partial_sort(idx.begin(), idx.begin() + keep, idx.end(), before);
    for (int64_t r = 0; r < keep; ++r) row[r] = (int)(idx[r] / k);
  }
  // group the kept candidates by parent, each parent's in score order
  auto& off = S.off;
  off.assign(n + 1, 0);
  for (int64_t r = 0; r < keep; ++r) off[row[r] + 1]++;
  for (int i = 0; i < n; ++i) off[i + 1] += off[i];
  for (int i = 0; i <= n; ++i) child_ptr[i] = off[i];
  for (int64_t r = 0; r < keep; ++r) {
    const int64_t e = idx[r];
    const int o = off[row[r]]++;
    child_tokens[o] = tokens[e];
    child_scores[o] = sc[e];
  }
  return BE_OK;
}

}  // extern "C"

extern "C" {

// Vanilla selection for several independent prompts in one call: candidates
// seg_ptr[s]..seg_ptr[s+1] belong to prompt s and compete only with each other
// (each prompt keeps its own beam_size).  Outputs cover all candidates:
// child_ptr [ncand + 1], child_tokens / child_scores [<= nseg * beam_size],
// new_seg_ptr [nseg + 1] (new candidates per prompt, in order).
int be_vanilla_select_segments(int nseg, const int32_t* seg_ptr, int k,
                               const double* parent_scores, const int32_t* tokens,
                               const double* logps, int beam_size, int32_t* child_ptr,
                               int32_t* child_tokens, double* child_scores,
                               int32_t* new_seg_ptr) {
  int out = 0;
  child_ptr[0] = 0;
  new_seg_ptr[0] = 0;
  std::vector<int32_t> ptr;
  for (int s = 0; s < nseg; ++s) {
    const int a = seg_ptr[s], b = seg_ptr[s + 1];
    const int n = b - a;
    ptr.assign(n + 1, 0);
    int rc = be_vanilla_select(n, k, parent_scores + a, tokens + (int64_t)a * k,
                               logps + (int64_t)a * k, beam_size, ptr.data(), child_tokens + out,
                               child_scores + out);
    if (rc) return rc;
    for (int i = 0; i < n; ++i) child_ptr[a + i + 1] = out + ptr[i + 1];
    out += ptr[n];
    new_seg_ptr[s + 1] = out;
  }
  return BE_OK;
}

// One host call per decode step after the device's top-k: vanilla selection of
// every prompt (be_vanilla_select_segments) followed by the trie update
// (be_beam_update) of the selected children.  Outputs: the new candidates'
// leaves and scores (in the reference's order), the new per-prompt candidate
// ranges, the copy-on-write copies and (optional) the selection's children per
// old candidate as CSR.  new_leaf / new_score / copy_* need nseg * beam_size
// entries, child_ptr ncand + 1.
int be_beam_select_update(be_trie* t, int nseg, const int32_t* seg_ptr, int k,
                          const int32_t* cand_leaf, const double* parent_scores,
                          const int32_t* tokens, const double* logps, int beam_size,
                          int32_t* new_leaf, double* new_score, int32_t* n_new,
                          int32_t* new_seg_ptr, int32_t* copy_src, int32_t* copy_dst,
                          int32_t* copy_len, int32_t* n_copies, int32_t* child_ptr) {
  if (nseg < 0 || !seg_ptr || beam_size < 1) {
    set_error("be_beam_select_update: invalid arguments");
    return BE_EINVAL;
  }
  const int ncand = seg_ptr[nseg];
  struct Scratch {
    std::vector<int32_t> ptr, ct, child;
    std::vector<double> cs;
  };
  static thread_local Scratch tls;
  Scratch& S = tls;
  const int cap = std::max(1, nseg * beam_size);
  S.ptr.resize(ncand + 1);
  S.ct.resize(cap);
  S.cs.resize(cap);
  S.child.resize(cap);
  int rc = be_vanilla_select_segments(nseg, seg_ptr, k, parent_scores, tokens, logps, beam_size,
                                      S.ptr.data(), S.ct.data(), S.cs.data(), new_seg_ptr);
  if (rc) return rc;
  rc = be_beam_update(t, ncand, cand_leaf, S.ptr.data(), S.ct.data(), new_leaf, S.child.data(),
                      n_new, copy_src, copy_dst, copy_len, n_copies);
  if (rc) return rc;
  for (int i = 0; i < *n_new; ++i) new_score[i] = S.cs[S.child[i]];
  if (child_ptr) std::copy(S.ptr.begin(), S.ptr.begin() + ncand + 1, child_ptr);
  return BE_OK;
}

int be_beam_update_selected(be_trie* t, int nseg, const int32_t* seg_ptr, const int32_t* cand_leaf,
                            const int32_t* sel_parent, const int32_t* sel_token,
                            const double* sel_score, int beam_size, int32_t* new_leaf,
                            double* new_score, int32_t* n_new, int32_t* new_seg_ptr,
                            int32_t* copy_src, int32_t* copy_dst, int32_t* copy_len,
                            int32_t* n_copies, int32_t* child_ptr) {
  if (nseg < 0 || !seg_ptr || beam_size < 1 || !sel_parent || !sel_token || !sel_score) {
    set_error("be_beam_update_selected: invalid arguments");
    return BE_EINVAL;
  }
  const int ncand = seg_ptr[nseg];
  struct Scratch {
    std::vector<int32_t> ptr, fill, ct, child;
    std::vector<double> cs;
  };
  static thread_local Scratch tls;
  Scratch& S = tls;
  const int cap = std::max(1, nseg * beam_size);
  S.ptr.assign(ncand + 1, 0);
  S.ct.resize(cap);
  S.cs.resize(cap);
  S.child.resize(cap);
  // children per candidate, counted then placed in rank order (results_map of
  // select_candidates, beam_strategy.py:470-476)
  new_seg_ptr[0] = 0;
  for (int s = 0; s < nseg; ++s) {
    int got = 0;
    for (int r = 0; r < beam_size; ++r) {
      const int c = sel_parent[(int64_t)s * beam_size + r];
      if (c < 0) break;
      if (c < seg_ptr[s] || c >= seg_ptr[s + 1]) {
        set_error("be_beam_update_selected: prompt %d selection %d names candidate %d", s, r, c);
        return BE_EINVAL;
      }
      S.ptr[c + 1]++;
      ++got;
    }
    new_seg_ptr[s + 1] = new_seg_ptr[s] + got;
  }
  for (int c = 0; c < ncand; ++c) S.ptr[c + 1] += S.ptr[c];
  S.fill.assign(S.ptr.begin(), S.ptr.end() - 1);
  for (int s = 0; s < nseg; ++s)
    for (int r = 0; r < beam_size; ++r) {
      const int64_t o = (int64_t)s * beam_size + r;
      const int c = sel_parent[o];
      if (c < 0) break;
      const int at = S.fill[c]++;
      S.ct[at] = sel_token[o];
      S.cs[at] = sel_score[o];
    }
  int rc = be_beam_update(t, ncand, cand_leaf, S.ptr.data(), S.ct.data(), new_leaf, S.child.data(),
                          n_new, copy_src, copy_dst, copy_len, n_copies);
  if (rc) return rc;
  for (int i = 0; i < *n_new; ++i) new_score[i] = S.cs[S.child[i]];
  if (child_ptr) std::copy(S.ptr.begin(), S.ptr.begin() + ncand + 1, child_ptr);
  return BE_OK;
}

// Everything one cascade decode step needs from the host, in one call: the
// per-candidate inputs (query token, RoPE position, append page, append slot)
// at out[0 .. 4 * ncand) and the attention plan (header included) at
// out[plan_offset ..).  Semantics: be_beam_step_inputs + be_cascade_build +
// be_cascade_plan.  BE_ECAPACITY reports the plan size in info->total_ints.
namespace {
// The cascade levels of a decode step (be_cascade_build into growable scratch)
// as per-level array pointers.
struct StepLevels {
  std::vector<int32_t> lg, lp, qo, kvp, kvi, last, ng;
  std::vector<const int32_t*> a_qo, a_kvp, a_kvi, a_last;
  int nlev = 0;
};
int build_step_levels(be_trie* t, int ncand, const int32_t* cand_leaf, StepLevels& L) {
  int cap_l = 64, cap_g = 64 * (ncand + 1), cap_p = 8192;
  for (;;) {
    L.lg.resize(cap_l + 1);
    L.lp.resize(cap_l + 1);
    L.qo.resize(cap_g + cap_l);
    L.kvp.resize(cap_g + cap_l);
    L.kvi.resize(cap_p);
    L.last.resize(cap_g);
    L.nlev = be_cascade_build(t, ncand, cand_leaf, cap_l, cap_g, cap_p, L.lg.data(), L.lp.data(),
                              L.qo.data(), L.kvp.data(), L.kvi.data(), L.last.data());
    if (L.nlev == -BE_ECAPACITY) {
      cap_l *= 2;
      cap_g *= 2;
      cap_p *= 4;
      continue;
    }
    if (L.nlev < 0) return -L.nlev;
    break;
  }
  const int nlev = L.nlev;
  L.a_qo.resize(nlev);
  L.a_kvp.resize(nlev);
  L.a_kvi.resize(nlev);
  L.a_last.resize(nlev);
  L.ng.resize(nlev);
  for (int l = 0; l < nlev; ++l) {
    L.a_qo[l] = L.qo.data() + L.lg[l] + l;
    L.a_kvp[l] = L.kvp.data() + L.lg[l] + l;
    L.a_kvi[l] = L.kvi.data() + L.lp[l];
    L.a_last[l] = L.last.data() + L.lg[l];
    L.ng[l] = L.lg[l + 1] - L.lg[l];
  }
  return BE_OK;
}
}  // namespace

int be_beam_decode_inputs(be_trie* t, int ncand, const int32_t* cand_leaf, int num_qo_heads,
                          int num_kv_heads, int num_sms, int32_t* out, int64_t cap,
                          int32_t plan_offset, be_attn_plan_info* info) {
  if ((int64_t)4 * ncand > plan_offset || plan_offset > cap) {
    set_error("be_beam_decode_inputs: plan_offset %d too small for %d candidates", plan_offset,
              ncand);
    return BE_EINVAL;
  }
  int rc = be_beam_step_inputs(t, ncand, cand_leaf, out, out + 2 * ncand, out + 3 * ncand,
                               out + ncand);
  if (rc) return rc;
  static thread_local StepLevels L;
  rc = build_step_levels(t, ncand, cand_leaf, L);
  if (rc) return rc;
  return be_cascade_plan(L.nlev, L.a_qo.data(), L.a_kvp.data(), L.a_kvi.data(), L.a_last.data(),
                         L.ng.data(), ncand, t->page_size, num_qo_heads, num_kv_heads, 1, 0,
                         num_sms, out + plan_offset, cap - plan_offset, info);
}

int be_beam_decode_tiles(be_trie* t, int ncand, const int32_t* cand_leaf, int num_qo_heads,
                         int num_kv_heads, int tile_rows, int target_pieces, int cluster,
                         int32_t* out, int64_t cap, int32_t plan_offset,
                         be_tile_plan_info* info) {
  if ((int64_t)4 * ncand > plan_offset || plan_offset > cap) {
    set_error("be_beam_decode_tiles: plan_offset %d too small for %d candidates", plan_offset,
              ncand);
    return BE_EINVAL;
  }
  int rc = be_beam_step_inputs(t, ncand, cand_leaf, out, out + 2 * ncand, out + 3 * ncand,
                               out + ncand);
  if (rc) return rc;
  static thread_local StepLevels L;
  rc = build_step_levels(t, ncand, cand_leaf, L);
  if (rc) return rc;
  return be_tile_plan(L.nlev, L.a_qo.data(), L.a_kvp.data(), L.a_kvi.data(), L.a_last.data(),
                      L.ng.data(), ncand, t->page_size, num_qo_heads, num_kv_heads, 1, tile_rows,
                      target_pieces, cluster, out + plan_offset, cap - plan_offset, info);
}

}  // extern "C"
