"""BeamState: the beam trie over KV pages, same interface as the reference's
``src/beam_engine/beam_state.py`` (``TrieNode`` :12-30, dataclasses :33-60,
``BeamState`` :62-682), backed by the native host page manager.

The trie (nodes, tokens, children) and the FIFO page allocator live in C++
(``be_trie``, shared with the :class:`PageTable`); a :class:`TrieNode` is a
handle ``(trie, node id)``.  Fork/free (``add_filtered_results``), cascade
levels (``get_cascade_input``) and FastTree inputs (``get_fasttree_input``)
run natively with the reference's semantics, including its quirks (the
query's own K/V is excluded from the cascade; shallow candidates repeat their
deepest pages at later levels).  Copy-on-write tail copies are collected and
issued as ONE batched kernel (all copies, all layers) per update.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch

from . import _lib
from ._lib import check, lib
from .fasttree import KVTreeNode


class TrieNode:
    """Handle to a trie node.  ``TrieNode(tokens, page_id, parent)`` creates a node
    like the reference's constructor (a root without ``trie=`` gets its own trie)."""

    __slots__ = ("_t", "_id", "_owner")

    def __init__(self, tokens: List[int] = None, page_id: int = -1,
                 parent: Optional["TrieNode"] = None, *, trie=None, node_id: int = None,
                 _owner=None):
        if node_id is not None:
            self._t, self._id, self._owner = trie, node_id, _owner
            return
        if parent is not None:
            self._t, self._owner = parent._t, parent._owner
        elif trie is not None:
            self._t, self._owner = trie, _owner
        else:
            self._owner = _StandaloneTrie()
            self._t = self._owner.ptr
        toks = np.asarray(list(tokens or []), np.int32)
        out = C.c_int32()
        check(lib().be_node_new(self._t, parent._id if parent is not None else -1, int(page_id),
                                _lib.ptr32(toks), len(toks), C.byref(out)), "TrieNode")
        self._id = out.value

    def _info(self):
        par, page, nt, nc = C.c_int32(), C.c_int32(), C.c_int32(), C.c_int32()
        check(lib().be_node_info(self._t, self._id, C.byref(par), C.byref(page), C.byref(nt),
                                 C.byref(nc)), "node info")
        return par.value, page.value, nt.value, nc.value

    @property
    def tokens(self) -> List[int]:
        n = self._info()[2]
        buf = np.zeros(max(n, 1), np.int32)
        lib().be_node_tokens(self._t, self._id, _lib.ptr32(buf), n)
        return buf[:n].tolist()

    @property
    def page_id(self) -> int:
        return self._info()[1]

    @property
    def parent(self) -> Optional["TrieNode"]:
        p = self._info()[0]
        return None if p < 0 else TrieNode(trie=self._t, node_id=p, _owner=self._owner)

    @property
    def children(self) -> List["TrieNode"]:
        n = self._info()[3]
        buf = np.zeros(max(n, 1), np.int32)
        lib().be_node_children(self._t, self._id, _lib.ptr32(buf), n)
        return [TrieNode(trie=self._t, node_id=int(c), _owner=self._owner) for c in buf[:n]]

    def append_token(self, token: int):
        check(lib().be_node_append_token(self._t, self._id, int(token)), "append_token")

    def __eq__(self, other):
        return isinstance(other, TrieNode) and other._t == self._t and other._id == self._id

    def __hash__(self):
        return hash((self._t, self._id))

    def __repr__(self):
        par, page, nt, nc = self._info()
        return f"TrieNode(tokens={self.tokens}, page_id={page}, children={nc})"


class _StandaloneTrie:
    """Trie for hand-built nodes that belong to no PageTable (as in test trees)."""

    def __init__(self, page_size=1):
        self.ptr = lib().be_trie_create(page_size, 0)

    def __del__(self):
        if getattr(self, "ptr", None):
            lib().be_trie_destroy(self.ptr)
            self.ptr = None


@dataclass
class BeamCandidate:
    trie_node: TrieNode
    score: float
    finished: bool = False


@dataclass
class BeamTokenCandidate:
    token_id: int
    log_prob: float


@dataclass
class BeamToken:
    token_id: int
    accumulated_score: float


@dataclass
class BeamGenerateInput:
    candidate: BeamCandidate
    children: List[BeamTokenCandidate]


@dataclass
class BeamGenerateResult:
    candidate: BeamCandidate
    children: List[BeamToken]


class BeamState:
    """Current beam candidates over the page trie (beam_state.py:62-682)."""

    def __init__(self, beam_size: int, page_table):
        self.beam_size = beam_size
        self.page_table = page_table
        self._t = page_table._trie
        self._owner = page_table
        self.root = None
        self._leaves = np.zeros(0, np.int32)
        self._scores = np.zeros(0, np.float64)
        self._cand_objs = None
        self.finished_candidates: List[BeamCandidate] = []
        self._cached_write_batch_indices = None
        self._cached_write_kv_indptr = None
        self.last_copies = (np.zeros(0, np.int32),) * 3
        self.defer_copies = False   # engine mode: caller issues the batched copy itself

    # -- candidates view ----------------------------------------------------
    @property
    def candidates(self) -> List[BeamCandidate]:
        if self._cand_objs is None:
            self._cand_objs = [BeamCandidate(TrieNode(trie=self._t, node_id=int(n), _owner=self._owner),
                                             float(s)) for n, s in zip(self._leaves, self._scores)]
        return self._cand_objs

    @candidates.setter
    def candidates(self, cands: List[BeamCandidate]):
        if cands:
            self._t = cands[0].trie_node._t
            self._owner = cands[0].trie_node._owner
        self._leaves = np.asarray([c.trie_node._id for c in cands], np.int32)
        self._scores = np.asarray([c.score for c in cands], np.float64)
        self._cand_objs = None

    def set_state(self, leaves, scores):
        self._leaves = np.ascontiguousarray(leaves, np.int32)
        self._scores = np.ascontiguousarray(scores, np.float64)
        self._cand_objs = None

    @property
    def leaves(self) -> np.ndarray:
        return self._leaves

    @property
    def scores(self) -> np.ndarray:
        return self._scores

    # -- beam_state.py:76-98 ------------------------------------------------
    def add_root_sequence(self, sequence: List[int]) -> List[TrieNode]:
        toks = np.asarray(sequence, np.int32)
        leaf = C.c_int32()
        pages = np.zeros(max(1, -(-len(toks) // self.page_table.page_size)), np.int32)
        check(lib().be_beam_add_root(self._t, _lib.ptr32(toks), len(toks), C.byref(leaf),
                                     _lib.ptr32(pages)), "add_root_sequence")
        chain = []
        n = TrieNode(trie=self._t, node_id=leaf.value, _owner=self._owner)
        while n is not None:
            chain.append(n)
            n = n.parent
        chain.reverse()
        if self.root is None and chain:
            self.root = chain[0]
        self._leaves = np.append(self._leaves, np.int32(leaf.value))
        self._scores = np.append(self._scores, 0.0)
        self._cand_objs = None
        return chain

    # -- beam_state.py:101-209 ----------------------------------------------
    def add_filtered_results(self, results: List[BeamGenerateResult]):
        if len(results) != len(self._leaves):
            self.candidates = [r.candidate for r in results]
        ptr = np.zeros(len(results) + 1, np.int32)
        toks, scores = [], []
        for i, r in enumerate(results):
            ptr[i + 1] = ptr[i] + len(r.children)
            toks.extend(c.token_id for c in r.children)
            scores.extend(c.accumulated_score for c in r.children)
        leaves = np.asarray([r.candidate.trie_node._id for r in results], np.int32)
        self.update_native(leaves, ptr, np.asarray(toks, np.int32), np.asarray(scores, np.float64))

    def update_native(self, leaves, child_ptr, child_tokens, child_scores):
        """Array form of add_filtered_results: candidate i's children are
        child_tokens[child_ptr[i]:child_ptr[i+1]] with their accumulated scores."""
        nc = max(int(child_ptr[-1]), 1)
        new_leaf = np.zeros(nc, np.int32)
        new_child = np.zeros(nc, np.int32)
        cs, cd, cl = (np.zeros(nc, np.int32) for _ in range(3))
        n_new, n_cp = C.c_int32(), C.c_int32()
        leaves = np.ascontiguousarray(leaves, np.int32)
        child_ptr = np.ascontiguousarray(child_ptr, np.int32)
        child_tokens = np.ascontiguousarray(child_tokens, np.int32)
        rc = lib().be_beam_update(self._t, len(leaves), _lib.addr(leaves), _lib.addr(child_ptr),
                                  _lib.addr(child_tokens), _lib.addr(new_leaf),
                                  _lib.addr(new_child), C.byref(n_new), _lib.addr(cs),
                                  _lib.addr(cd), _lib.addr(cl), C.byref(n_cp))
        if rc == _lib.BE_ENOMEM:
            raise MemoryError("No free pages available")
        check(rc, "add_filtered_results")
        k, c = n_new.value, n_cp.value
        self.last_child_ptr = np.asarray(child_ptr, np.int32).copy()
        self._leaves = new_leaf[:k].copy()
        self._scores = np.asarray(child_scores, np.float64)[new_child[:k]]
        self._cand_objs = None
        self.last_copies = (cs[:c].copy(), cd[:c].copy(), cl[:c].copy())
        if c and not self.defer_copies and self.page_table.kv_cache.is_cuda:
            self.page_table.copy_blocks(*self.last_copies)

    def vanilla_step_selected(self, seg, sel_parent, sel_token, sel_score, beam_size):
        """The trie update of a vanilla step whose selection ran on the device
        (be_vanilla_select_device: per prompt, beam_size (parent, token, score)
        in rank order, parent -1 past the prompt's entries).  Returns the new
        per-prompt candidate ranges, like vanilla_step."""
        seg = np.ascontiguousarray(seg, np.int32)
        nseg = len(seg) - 1
        ncand = int(seg[-1])
        cap = max(1, nseg * beam_size)
        nl, cs, cd, cl = (np.zeros(cap, np.int32) for _ in range(4))
        ns = np.zeros(cap, np.float64)
        nseg_ptr = np.zeros(nseg + 1, np.int32)
        cptr = np.zeros(ncand + 1, np.int32)
        n_new, n_cp = C.c_int32(), C.c_int32()
        leaves = np.ascontiguousarray(self._leaves, np.int32)
        sp = np.ascontiguousarray(sel_parent, np.int32)
        st = np.ascontiguousarray(sel_token, np.int32)
        sc = np.ascontiguousarray(sel_score, np.float64)
        rc = lib().be_beam_update_selected(self._t, nseg, _lib.addr(seg), _lib.addr(leaves),
                                           _lib.addr(sp), _lib.addr(st), _lib.addr(sc), beam_size,
                                           _lib.addr(nl), _lib.addr(ns), C.byref(n_new),
                                           _lib.addr(nseg_ptr), _lib.addr(cs), _lib.addr(cd),
                                           _lib.addr(cl), C.byref(n_cp), _lib.addr(cptr))
        if rc == _lib.BE_ENOMEM:
            raise MemoryError("No free pages available")
        check(rc, "vanilla step (device selection)")
        self.last_child_ptr = cptr.copy()
        m, c = n_new.value, n_cp.value
        self._leaves = nl[:m].copy()
        self._scores = ns[:m].copy()
        self._cand_objs = None
        self.last_copies = (cs[:c].copy(), cd[:c].copy(), cl[:c].copy())
        if c and not self.defer_copies and self.page_table.kv_cache.is_cuda:
            self.page_table.copy_blocks(*self.last_copies)
        return nseg_ptr.copy()

    def vanilla_step(self, seg, tokens, logps, beam_size):
        """Vanilla selection of every prompt (candidates seg[s]:seg[s+1]) on the
        top-k (tokens / logps [ncand, k]) plus the trie update, one native call
        (be_beam_select_update).  Returns the new per-prompt candidate ranges."""
        seg = np.ascontiguousarray(seg, np.int32)
        tokens = np.ascontiguousarray(tokens, np.int32)
        logps = np.ascontiguousarray(logps, np.float64)
        nseg = len(seg) - 1
        k = tokens.shape[1] if tokens.ndim == 2 else 0
        cap = max(1, nseg * beam_size)
        buf = getattr(self, "_vs_buf", None)
        ncand = int(seg[-1])
        if (buf is None or buf[0] < cap or len(buf[5]) != nseg + 1
                or len(buf[9]) < ncand + 1):
            buf = self._vs_buf = (cap, np.zeros(cap, np.int32), np.zeros(cap, np.float64),
                                  np.zeros(cap, np.int32), np.zeros(cap, np.int32),
                                  np.zeros(nseg + 1, np.int32), np.zeros(cap, np.int32),
                                  C.c_int32(), C.c_int32(), np.zeros(max(ncand + 1, cap + 1), np.int32))
        _, nl, ns, cs, cd, nseg_ptr, cl, n_new, n_cp, cptr = buf
        leaves = np.ascontiguousarray(self._leaves, np.int32)
        scores = np.ascontiguousarray(self._scores, np.float64)
        rc = lib().be_beam_select_update(self._t, nseg, _lib.addr(seg), k, _lib.addr(leaves),
                                         _lib.addr(scores), _lib.addr(tokens), _lib.addr(logps),
                                         beam_size, _lib.addr(nl), _lib.addr(ns), C.byref(n_new),
                                         _lib.addr(nseg_ptr), _lib.addr(cs), _lib.addr(cd),
                                         _lib.addr(cl), C.byref(n_cp), _lib.addr(cptr))
        if rc == _lib.BE_ENOMEM:
            raise MemoryError("No free pages available")
        check(rc, "vanilla step")
        self.last_child_ptr = cptr[:ncand + 1].copy()
        m, c = n_new.value, n_cp.value
        self._leaves = nl[:m].copy()
        self._scores = ns[:m].copy()
        self._cand_objs = None
        self.last_copies = (cs[:c].copy(), cd[:c].copy(), cl[:c].copy())
        if c and not self.defer_copies and self.page_table.kv_cache.is_cuda:
            self.page_table.copy_blocks(*self.last_copies)
        return nseg_ptr.copy()

    # -- decode inputs -------------------------------------------------------
    def step_inputs(self):
        """(query tokens, write pages, write positions, RoPE positions), int32 arrays."""
        n = len(self._leaves)
        out = [np.zeros(max(n, 1), np.int32) for _ in range(4)]
        check(lib().be_beam_step_inputs(self._t, n, _lib.addr(self._leaves),
                                        *[_lib.addr(o) for o in out]), "step inputs")
        return [o[:n] for o in out]

    def cascade_levels(self):
        """Native get_cascade_input: list of per-level dicts of int32 numpy arrays."""
        n = len(self._leaves)
        if n == 0:
            return []
        cap_l, cap_g, cap_p = 64, 64 * (n + 1), 4096
        while True:
            lg = np.zeros(cap_l + 1, np.int32)
            lp = np.zeros(cap_l + 1, np.int32)
            qo = np.zeros(cap_g + cap_l, np.int32)
            kvp = np.zeros(cap_g + cap_l, np.int32)
            kvi = np.zeros(cap_p, np.int32)
            last = np.zeros(cap_g, np.int32)
            r = lib().be_cascade_build(self._t, n, _lib.ptr32(self._leaves), cap_l, cap_g, cap_p,
                                       _lib.ptr32(lg), _lib.ptr32(lp), _lib.ptr32(qo),
                                       _lib.ptr32(kvp), _lib.ptr32(kvi), _lib.ptr32(last))
            if r == -_lib.BE_ECAPACITY:
                cap_l, cap_g, cap_p = cap_l * 2, cap_g * 2, cap_p * 4
                continue
            if r < 0:
                check(-r, "get_cascade_input")
            break
        levels = []
        for lv in range(r):
            g0, g1 = lg[lv], lg[lv + 1]
            p0, p1 = lp[lv], lp[lv + 1]
            levels.append(dict(qo_indptr=qo[g0 + lv:g1 + lv + 1], kv_indptr=kvp[g0 + lv:g1 + lv + 1],
                               kv_indices=kvi[p0:p1], kv_last_page_len=last[g0:g1]))
        return levels

    def get_cascade_input(self):
        """beam_state.py:211-412 -- same 7-tuple as the reference."""
        if len(self._leaves) == 0:
            return ([], [], [], [], torch.empty(0, 0, 0))
        levels = self.cascade_levels()
        qtok = self.step_inputs()[0]
        dev = self.page_table.device
        n = len(self._leaves)
        if (self._cached_write_batch_indices is None
                or self._cached_write_batch_indices.shape[0] != n):
            self._cached_write_batch_indices = torch.arange(n, dtype=torch.int32, device=dev)
            self._cached_write_kv_indptr = torch.arange(n + 1, dtype=torch.int32, device=dev)
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.int32))  # noqa: E731
        return ([t(lv["qo_indptr"]) for lv in levels], [t(lv["kv_indptr"]) for lv in levels],
                [t(lv["kv_indices"]) for lv in levels], [t(lv["kv_last_page_len"]) for lv in levels],
                torch.tensor(qtok.astype(np.int64), device=dev), self._cached_write_batch_indices,
                self._cached_write_kv_indptr)

    # -- beam_state.py:414-633 ----------------------------------------------
    def tree_arrays(self, per_node: bool = False, compress: bool = False):
        """Tree nodes (BFS), their parents / lengths / child counts, request
        lists and req_to_token.  ``compress`` merges chains of single-child trie
        nodes into one tree node (per-node lengths), which the engine's tree
        plans use; the reference's layout is one node per trie node."""
        n = len(self._leaves)
        nn, ml = C.c_int32(), C.c_int32()
        leaves = np.ascontiguousarray(self._leaves, np.int32)
        args = [self._t, n, _lib.ptr32(leaves), (1 if per_node else 0) | (2 if compress else 0),
                self.page_table.page_size]
        # one native pass with the capacities of the last call (grown and retried when short)
        N, M = getattr(self, "_tree_caps", (64, 64))
        while True:
            par, seql, kids = (np.zeros(max(N, 1), np.int32) for _ in range(3))
            rptr = np.zeros(N + 1, np.int32)
            cap_r = max(1, N * n)
            rl = np.zeros(cap_r, np.int32)
            r2t = np.empty(max(n, 1) * max(M, 1), np.int32)
            rc = lib().be_tree_build(*args, N, C.byref(nn), _lib.ptr32(par), _lib.ptr32(seql),
                                     _lib.ptr32(kids), _lib.ptr32(rptr), _lib.ptr32(rl), cap_r,
                                     C.byref(ml), _lib.ptr32(r2t), r2t.size)
            if rc != _lib.BE_ECAPACITY:
                break
            N, M = max(N, nn.value + nn.value // 4 + 16), max(M, ml.value + 64)
        check(rc, "tree build")
        self._tree_caps = (N, M)
        Nn, Mm = nn.value, ml.value
        return (par[:Nn], seql[:Nn], kids[:Nn], rptr[:Nn + 1], rl[:rptr[Nn]],
                r2t[:max(n, 1) * Mm].reshape(max(n, 1), Mm)[:n])

    def get_fasttree_input(self, per_node: bool = True):
        """beam_state.py:566-633.  ``seqlen`` is per node by default -- the length
        the FastTree planner assumes; ``per_node=False`` gives the reference's
        cumulative value (which makes the reference's tree path attend the wrong
        tokens)."""
        par, seql, kids, rptr, rl, r2t = self.tree_arrays(per_node)
        nodes = []
        for i in range(len(par)):
            k = KVTreeNode()
            k.id, k.parent, k.seqlen, k.num_children = i, int(par[i]), int(seql[i]), int(kids[i])
            k.requests = rl[rptr[i]:rptr[i + 1]].tolist()
            nodes.append(k)
        q, wp, wpos, _ = self.step_inputs()
        dev = self.page_table.device
        return (nodes, torch.from_numpy(r2t.copy()).to(dev), torch.tensor(q.astype(np.int64), device=dev),
                torch.tensor(wp, device=dev), torch.tensor(wpos, device=dev))

    # -- beam_state.py:646-682 ----------------------------------------------
    def _seq_len(self, node: int) -> int:
        n = lib().be_node_sequence(self._t, int(node), None, 0)
        if n < 0:
            raise ValueError(f"unknown trie node {node}: "
                             f"{lib().be_last_error().decode(errors='replace')}")
        return n

    def sequence(self, leaf: int) -> List[int]:
        n = self._seq_len(leaf)
        buf = np.zeros(max(n, 1), np.int32)
        lib().be_node_sequence(self._t, int(leaf), _lib.ptr32(buf), n)
        return buf[:n].tolist()

    def leaf_sequences(self, leaves=None):
        """Token sequences of ``leaves`` (default: the candidates) as CSR
        ``(seq_ptr [n+1], seq_tokens)``, walking up to the first node without
        tokens (beam_strategy.py:96-103)."""
        leaves = np.ascontiguousarray(self._leaves if leaves is None else leaves, np.int32)
        n = len(leaves)
        ptr = np.zeros(n + 1, np.int32)
        cap = int(getattr(self, "_seq_cap", 0))
        buf = np.zeros(max(cap, 1), np.int32)
        total = lib().be_leaf_sequences(self._t, n, _lib.addr(leaves), _lib.addr(ptr),
                                        _lib.addr(buf), cap)
        if total < 0:
            check(_lib.BE_EINVAL, "leaf_sequences")
        if total > cap:
            self._seq_cap = cap = int(total * 1.25) + 64
            buf = np.zeros(cap, np.int32)
            lib().be_leaf_sequences(self._t, n, _lib.addr(leaves), _lib.addr(ptr),
                                    _lib.addr(buf), cap)
        return ptr, buf[:total]

    def get_best_finished(self, num_return: int) -> List[BeamCandidate]:
        """beam_state.py:635-644: the best finished candidates (else the best
        active ones) by score / length.  The reference reads ``candidate.length``,
        which its BeamCandidate does not have (an AttributeError whenever a
        candidate exists); the length here is the candidate's sequence length."""
        pool = self.finished_candidates or self.candidates

        def norm(c):
            return c.score / max(1, len(self.sequence(c.trie_node._id)))
        return sorted(pool, key=norm, reverse=True)[:num_return]

    def get_final_sequences(self, num_return: int, length_penalty: float = 1.0
                            ) -> List[Tuple[List[int], float]]:
        # rank by the length-penalised score first (lengths are one native call
        # each), then materialise only the sequences that are returned
        nodes = [c.trie_node._id for c in self.finished_candidates] + [int(x) for x in self._leaves]
        raw = [c.score for c in self.finished_candidates] + [float(x) for x in self._scores]
        ranked = []
        for node, sc in zip(nodes, raw):
            n = self._seq_len(node)
            if length_penalty != 0 and n > 1:
                sc = sc / (n ** length_penalty)
            ranked.append((node, sc))
        ranked.sort(key=lambda x: x[1], reverse=True)   # stable: ties keep candidate order
        return [(self.sequence(node), sc) for node, sc in ranked[:num_return]]
