"""Oracle: beam trie, copy-on-write forks and metadata builders (test infrastructure).

Restates ``src/beam_engine/beam_state.py`` of the reference.  Nodes live in a
flat list and are addressed by integer ids; the semantics are the reference's:

* ``add_root_sequence``: a chain of ``ceil(n / page_size)`` nodes, one page
  each, allocated front to back (beam_state.py:76-98).
* ``add_filtered_results`` (beam_state.py:101-209): first every result with no
  children frees pages upward from its leaf until a node that still has
  children (unlinking each freed node from its parent); then each surviving
  result, in order: one child -> append in place if the leaf page has room,
  else a new child page; several children on a full page -> one new page per
  child; several children on a partial page -> children 2..n each get a
  ``copy_block`` of the leaf page with ``[*tokens, tok]`` and become SIBLINGS
  of the leaf (same parent), then child 1 appends in place.
* ``cascade_input`` (beam_state.py:211-412): branch level of a node = level of
  its parent + 1 if the parent has more than one child; every candidate
  appears at every level, reusing its deepest level's nodes where it has none
  (quirk: pages may appear at several levels); groups are keyed by the last
  node of the candidate's chain at that level and ordered by their first
  candidate; ``last_page_len`` is ``len(tokens) - 1`` when that node is the
  group's first candidate's leaf, else ``len(tokens)``.
* ``tree_input`` (beam_state.py:414-633): BFS node order, cumulative
  ``seqlen`` as the reference computes it (``per_node=True`` gives the
  corrected per-node length the FastTree planner actually assumes),
  ``req_to_token`` slot table ``page * page_size + i``, write page / position.
"""
from __future__ import annotations

from collections import defaultdict, deque


class ONode:
    __slots__ = ("tokens", "parent", "children", "page", "nid")

    def __init__(self, nid, tokens, page, parent):
        self.nid = nid
        self.tokens = list(tokens)
        self.page = page
        self.parent = parent
        self.children = []


class OracleBeamState:
    def __init__(self, beam_size, table):
        self.beam_size = beam_size
        self.table = table          # needs allocate_block/free_block/copy_block/page_size
        self.nodes = []
        self.cand_leaf = []         # node id per candidate
        self.cand_score = []
        self.copies = []            # (src_page, dst_page, length) in issue order

    # -- construction -----------------------------------------------------
    def new_node(self, tokens, page, parent):
        n = ONode(len(self.nodes), tokens, page, parent)
        self.nodes.append(n)
        if parent is not None:
            self.nodes[parent].children.append(n.nid)
        return n.nid

    def add_root_sequence(self, seq):
        ps = self.table.page_size
        cur = None
        made = []
        for s in range(0, len(seq), ps):
            page = self.table.allocate_block()
            cur = self.new_node(seq[s:s + ps], page, cur)
            made.append(cur)
        self.cand_leaf.append(cur)
        self.cand_score.append(0.0)
        return made

    # -- fork / free ------------------------------------------------------
    def add_filtered_results(self, results):
        """results[i] = list of (token, score) children for candidate i."""
        assert len(results) == len(self.cand_leaf)
        ps = self.table.page_size
        for i, ch in enumerate(results):
            if ch:
                continue
            n = self.cand_leaf[i]
            while n is not None and not self.nodes[n].children:
                self.table.free_block(self.nodes[n].page)
                par = self.nodes[n].parent
                if par is not None:
                    self.nodes[par].children.remove(n)
                n = par
        leaves, scores = [], []
        for i, ch in enumerate(results):
            if not ch:
                continue
            nid = self.cand_leaf[i]
            node = self.nodes[nid]
            if len(ch) == 1:
                tok, sc = ch[0]
                if len(node.tokens) < ps:
                    node.tokens.append(tok)
                    leaves.append(nid)
                else:
                    leaves.append(self.new_node([tok], self.table.allocate_block(), nid))
                scores.append(sc)
                continue
            if len(node.tokens) == ps:
                for tok, sc in ch:
                    leaves.append(self.new_node([tok], self.table.allocate_block(), nid))
                    scores.append(sc)
            else:
                base = list(node.tokens)
                for tok, sc in ch[1:]:
                    dst = self.table.copy_block(node.page, len(base))
                    self.copies.append((node.page, dst, len(base)))
                    leaves.append(self.new_node(base + [tok], dst, node.parent))
                    scores.append(sc)
                node.tokens.append(ch[0][0])
                leaves.append(nid)
                scores.append(ch[0][1])
        self.cand_leaf, self.cand_score = leaves, scores

    # -- helpers ----------------------------------------------------------
    def path(self, nid):
        out = []
        while nid is not None:
            out.append(nid)
            nid = self.nodes[nid].parent
        return out[::-1]

    def sequence(self, cand):
        seq = []
        for n in self.path(self.cand_leaf[cand]):
            seq.extend(self.nodes[n].tokens)
        return seq

    def query_tokens(self):
        return [self.nodes[n].tokens[-1] if self.nodes[n].tokens else 0 for n in self.cand_leaf]

    def write_targets(self):
        return ([self.nodes[n].page for n in self.cand_leaf],
                [len(self.nodes[n].tokens) - 1 for n in self.cand_leaf])

    def position_ids(self):
        return [len(self.sequence(c)) - 1 for c in range(len(self.cand_leaf))]

    # -- cascade metadata (beam_state.py:211-412) --------------------------
    def level(self, nid, memo):
        if nid in memo:
            return memo[nid]
        p = self.nodes[nid].parent
        lv = 0 if p is None else self.level(p, memo) + (len(self.nodes[p].children) > 1)
        memo[nid] = lv
        return lv

    def cascade_input(self):
        memo = {}
        per_cand = []
        top = 0
        for leaf in self.cand_leaf:
            by = defaultdict(list)
            for n in self.path(leaf):
                lv = self.level(n, memo)
                by[lv].append(n)
                top = max(top, lv)
            per_cand.append(by)
        levels = []
        for lv in range(top + 1):
            groups = {}   # key: representative node -> [first cand, count, nodes]
            order = []
            for c, by in enumerate(per_cand):
                nodes = by[lv] if lv in by else by[max(by)]
                key = nodes[-1]
                if key not in groups:
                    groups[key] = [c, 0, nodes]
                    order.append(key)
                groups[key][1] += 1
            order.sort(key=lambda k: groups[k][0])
            qo, kvp, kvi, last = [0], [0], [], []
            for k in order:
                c0, cnt, nodes = groups[k]
                seen = set()
                for n in nodes:
                    pg = self.nodes[n].page
                    if pg not in seen:
                        kvi.append(pg)
                        seen.add(pg)
                tail = nodes[-1]
                ln = len(self.nodes[tail].tokens)
                last.append(max(0, ln - 1) if tail == self.cand_leaf[c0] else ln)
                kvp.append(len(kvi))
                qo.append(qo[-1] + cnt)
            levels.append(dict(qo_indptr=qo, kv_indptr=kvp, kv_indices=kvi, kv_last_page_len=last))
        return levels, self.query_tokens()

    # -- FastTree metadata (beam_state.py:414-633) -------------------------
    def tree_input(self, per_node=False):
        live = set()
        roots = []
        for leaf in self.cand_leaf:
            for n in self.path(leaf):
                live.add(n)
            r = self.path(leaf)[0]
            if r not in roots:
                roots.append(r)
        order, tid = [], {}
        q = deque(roots)
        seen = set()
        while q:
            n = q.popleft()
            if n in seen:
                continue
            seen.add(n)
            tid[n] = len(order)
            order.append(n)
            for ch in self.nodes[n].children:
                if ch not in seen:
                    q.append(ch)
        tree = []
        for n in order:
            node = self.nodes[n]
            par = -1 if node.parent is None else tid.get(node.parent, -1)
            if per_node:
                seqlen = len(node.tokens)
            else:
                seqlen = sum(len(self.nodes[m].tokens) for m in self.path(n))
            reqs = [c for c, leaf in enumerate(self.cand_leaf) if n in self.path(leaf)]
            tree.append(dict(parent=par, id=tid[n], seqlen=seqlen,
                             num_children=len(node.children), requests=reqs))
        ps = self.table.page_size
        seqs = [self.path(leaf) for leaf in self.cand_leaf]
        maxlen = max(sum(len(self.nodes[m].tokens) for m in p) for p in seqs) if seqs else 0
        r2t = [[0] * maxlen for _ in seqs]
        for c, p in enumerate(seqs):
            t = 0
            for m in p:
                for i in range(len(self.nodes[m].tokens)):
                    r2t[c][t] = self.nodes[m].page * ps + i
                    t += 1
        pages, pos = self.write_targets()
        return tree, r2t, self.query_tokens(), pages, pos

    # -- final ranking (beam_state.py:646-682) -----------------------------
    def final_sequences(self, num_return, length_penalty=1.0):
        res = []
        for c in range(len(self.cand_leaf)):
            seq = self.sequence(c)
            sc = self.cand_score[c]
            if length_penalty != 0 and len(seq) > 1:
                sc = sc / (len(seq) ** length_penalty)
            res.append((seq, sc))
        res.sort(key=lambda x: x[1], reverse=True)
        return res[:num_return]


def vanilla_select(parent_scores, child_tokens, child_logps, beam_size):
    """VanillaBeamSearchStrategy.select_candidates (beam_strategy.py:433-488).

    Flatten (parent, token, parent_score + logp) in parent-major, top-k order;
    stable sort descending; keep ``beam_size``; regroup per parent in the
    sorted order.  Returns per-parent lists of (token, total_score).
    """
    flat = []
    for i, ps in enumerate(parent_scores):
        for tok, lp in zip(child_tokens[i], child_logps[i]):
            flat.append((i, int(tok), ps + float(lp)))
    flat.sort(key=lambda x: x[2], reverse=True)
    out = [[] for _ in parent_scores]
    for i, tok, sc in flat[:beam_size]:
        out[i].append((tok, sc))
    return out


def diverse_select(parent_scores, parent_seqs, child_tokens, child_logps, beam_size, num_groups=4,
                   diversity_penalty=0.5, diversity_type="hamming", length_penalty=1.0):
    """DiverseBeamSearchStrategy.select_candidates (beam_strategy.py:173-317).

    Choices (parent, token, logp) in parent-major, top-k order, stable-sorted
    by logp descending once (:215).  Each of ``num_groups`` groups re-scores
    every choice not yet picked (same parent and token, :225-227) as
    ``(logp - penalty) / len ** length_penalty`` with len = parent sequence + 1
    (:229-247; no division when length_penalty == 0, :157-170), stable-sorts
    descending and picks ``max(1, beam_size // num_groups)`` (:250-262).
    Penalty: hamming = diversity_penalty if the token was picked before this
    group (:105-125); otherwise cumulative = mean over earlier picks of
    position-wise agreements of the two sequences (zip) * diversity_penalty,
    summed in pick order (:127-155).  Picks are regrouped per parent in pick
    order with score parent_score + logp (:264-300); if more than beam_size
    were picked, children drop from the end, last parent first (:303-315).
    Returns per-parent lists of (token, score).
    """
    bpg = max(1, beam_size // num_groups)
    choices = []
    for i in range(len(parent_scores)):
        for tok, lp in zip(child_tokens[i], child_logps[i]):
            choices.append((i, int(tok), float(lp)))
    choices.sort(key=lambda x: x[2], reverse=True)
    picked, picked_tokens, picked_seqs = [], set(), []
    for _ in range(num_groups):
        adj = []
        for i, tok, lp in choices:
            if any(pi == i and pt == tok for pi, pt, _ in picked):
                continue
            seq = list(parent_seqs[i]) + [tok]
            if diversity_type == "hamming":
                pen = diversity_penalty if tok in picked_tokens else 0.0
            elif not picked_seqs:
                pen = 0.0
            else:
                tot = 0.0
                for s in picked_seqs:
                    tot += sum(1 for a, b in zip(seq, s) if a == b) * diversity_penalty
                pen = tot / len(picked_seqs)
            sc = lp - pen
            if length_penalty != 0:
                sc = sc / (len(seq) ** length_penalty)
            adj.append((i, tok, lp, sc))
        adj.sort(key=lambda x: x[3], reverse=True)
        for i, tok, lp, _ in adj[:bpg]:
            picked.append((i, tok, lp))
            picked_tokens.add(tok)
            picked_seqs.append(list(parent_seqs[i]) + [tok])
    out = [[] for _ in parent_scores]
    for i, tok, lp in picked:
        out[i].append((tok, parent_scores[i] + lp))
    extra = sum(len(o) for o in out) - beam_size
    for o in reversed(out):
        while extra > 0 and o:
            o.pop()
            extra -= 1
        if extra <= 0:
            break
    return out
