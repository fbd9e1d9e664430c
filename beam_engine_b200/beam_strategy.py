"""Beam strategies with the reference's interface (src/beam_engine/beam_strategy.py).

``VanillaBeamSearchStrategy`` (beam_strategy.py:403-553): global top-``beam_size``
of ``parent.score + log_prob`` over every offered child, stable descending sort
in double precision, children regrouped per parent in sorted order; the native
``be_vanilla_select`` does the sort.  ``select_arrays`` is the array form the
engine uses (no per-token Python objects).

``DiverseBeamSearchStrategy`` (beam_strategy.py:60-400): groups pick in turn,
each penalised for tokens (hamming) or sequence overlap (cumulative) with the
picks of earlier groups; the native ``be_diverse_select`` does the selection,
``select_segments(..., state=)`` is the engine's batched form.
"""
from __future__ import annotations

import ctypes as C
from abc import ABC, abstractmethod
from typing import List, Optional, Tuple

import numpy as np

from . import _lib
from ._lib import check, lib
from .beam_state import BeamGenerateInput, BeamGenerateResult, BeamState, BeamToken


class BeamStrategy(ABC):
    @abstractmethod
    def select_candidates(self, beam_state: BeamState, new_candidates: List[BeamGenerateInput],
                          step: int) -> List[BeamGenerateResult]:
        ...

    @abstractmethod
    def should_stop(self, beam_state: BeamState, max_length: int, step: int) -> bool:
        ...

    @abstractmethod
    def get_final_sequences(self, beam_state: BeamState, num_return: Optional[int] = None
                            ) -> List[Tuple[List[int], float]]:
        ...


_DIVERSITY_TYPES = {"hamming": 0}


def diverse_select_segments(seg, parent_scores, tokens, logps, seq_ptr, seq_tokens, beam_size,
                            num_groups, diversity_penalty, diversity_type, length_penalty):
    """be_diverse_select over prompts seg[s]:seg[s+1].  Returns (child_ptr, tokens,
    scores, new_seg) like ``select_segments``."""
    seg = np.ascontiguousarray(seg, np.int32)
    n = int(seg[-1])
    tokens = np.ascontiguousarray(tokens, np.int32)
    if tokens.ndim != 2:
        tokens = tokens.reshape(n, -1)
    k = tokens.shape[1]
    logps = np.ascontiguousarray(logps, np.float64).reshape(n, k)
    ps = np.ascontiguousarray(parent_scores, np.float64)
    seq_ptr = np.ascontiguousarray(seq_ptr, np.int32)
    seq_tokens = np.ascontiguousarray(seq_tokens, np.int32)
    if len(seq_tokens) == 0:
        seq_tokens = np.zeros(1, np.int32)
    # the reference treats every type but "hamming" as cumulative
    dtype = _DIVERSITY_TYPES.get(diversity_type, 1)
    cap = max(1, (len(seg) - 1) * max(beam_size, num_groups))
    ptr = np.zeros(n + 1, np.int32)
    ct = np.zeros(cap, np.int32)
    cs = np.zeros(cap, np.float64)
    ns = np.zeros(len(seg), np.int32)
    D = C.POINTER(C.c_double)
    check(lib().be_diverse_select(len(seg) - 1, _lib.addr(seg), k, ps.ctypes.data,
                                  _lib.addr(tokens), logps.ctypes.data, _lib.addr(seq_ptr),
                                  _lib.addr(seq_tokens), int(beam_size), int(num_groups),
                                  float(diversity_penalty), dtype, float(length_penalty),
                                  _lib.addr(ptr), _lib.addr(ct), cs.ctypes.data,
                                  _lib.addr(ns)), "diverse select")
    m = int(ptr[-1])
    return ptr, ct[:m], cs[:m], ns


def diverse_select_device(seg, parent_scores, tokens, logps, seq_ptr, beam_size, num_groups,
                          diversity_penalty, length_penalty, stream=None):
    """be_diverse_select_device (hamming penalty) on device tensors: ``seg``
    int32 [nseg + 1], ``parent_scores`` float64 [ncand], ``tokens`` int32 /
    ``logps`` float64 [ncand, k], ``seq_ptr`` int32 [ncand + 1] (the parents'
    lengths).  Returns device tensors (child_ptr, child_tokens, child_scores,
    new_seg) sized like ``diverse_select_segments``'s outputs; the children are
    the first new_seg[-1] entries.  ``seg`` is also read on the host once, for
    the launch's largest prompt."""
    import torch
    nseg = seg.numel() - 1
    ncand, k = tokens.shape
    segh = seg.cpu().numpy()
    max_cands = int(np.max(np.diff(segh))) if nseg > 0 else 0
    dev = tokens.device
    cap = max(1, nseg * max(beam_size, num_groups))
    ptr = torch.zeros(ncand + 1, dtype=torch.int32, device=dev)
    ct = torch.zeros(cap, dtype=torch.int32, device=dev)
    cs = torch.zeros(cap, dtype=torch.float64, device=dev)
    ns = torch.zeros(nseg + 1, dtype=torch.int32, device=dev)
    st = stream if stream is not None else torch.cuda.current_stream(dev).cuda_stream
    check(lib().be_diverse_select_device(nseg, seg.data_ptr(), k, parent_scores.data_ptr(),
                                         tokens.data_ptr(), logps.data_ptr(), seq_ptr.data_ptr(),
                                         int(beam_size), int(num_groups), float(diversity_penalty),
                                         0, float(length_penalty), max_cands, ptr.data_ptr(),
                                         ct.data_ptr(), cs.data_ptr(), ns.data_ptr(),
                                         C.c_void_p(st)), "diverse select (device)")
    return ptr, ct, cs, ns


def vanilla_select_arrays(parent_scores, tokens, logps, beam_size):
    """parent_scores [n] f64, tokens/logps [n, k] -> (child_ptr [n+1], child_tokens,
    child_scores)."""
    parent_scores = np.ascontiguousarray(parent_scores, np.float64)
    tokens = np.ascontiguousarray(tokens, np.int32)
    logps = np.ascontiguousarray(logps, np.float64)
    n, k = tokens.shape if tokens.ndim == 2 else (len(parent_scores), 0)
    ptr = np.zeros(n + 1, np.int32)
    ct = np.zeros(max(beam_size, 1), np.int32)
    cs = np.zeros(max(beam_size, 1), np.float64)
    check(lib().be_vanilla_select(n, k, parent_scores.ctypes.data,
                                  _lib.addr(tokens), logps.ctypes.data,
                                  beam_size, _lib.addr(ptr), _lib.addr(ct),
                                  cs.ctypes.data), "vanilla select")
    m = int(ptr[-1])
    return ptr, ct[:m], cs[:m]


class VanillaBeamSearchStrategy(BeamStrategy):
    def __init__(self, length_penalty: float = 1.0, early_stopping: bool = True):
        self.length_penalty = length_penalty
        self.early_stopping = early_stopping

    def _apply_length_penalty(self, log_prob: float, length: int) -> float:
        if self.length_penalty == 0 or length <= 1:
            return log_prob
        return log_prob / (length ** self.length_penalty)

    def select_candidates(self, beam_state, new_candidates, step):
        if not new_candidates:
            return []
        k = max(len(x.children) for x in new_candidates)
        if any(len(x.children) != k for x in new_candidates):
            raise ValueError("every candidate must offer the same number of children")
        n = len(new_candidates)
        ps = np.asarray([x.candidate.score for x in new_candidates], np.float64)
        toks = np.asarray([[c.token_id for c in x.children] for x in new_candidates],
                          np.int32).reshape(n, k)
        lps = np.asarray([[c.log_prob for c in x.children] for x in new_candidates],
                         np.float64).reshape(n, k)
        ptr, ct, cs = vanilla_select_arrays(ps, toks, lps, beam_state.beam_size)
        return [BeamGenerateResult(candidate=x.candidate,
                                   children=[BeamToken(int(ct[j]), float(cs[j]))
                                             for j in range(ptr[i], ptr[i + 1])])
                for i, x in enumerate(new_candidates)]

    def select_segments(self, seg, parent_scores, tokens, logps, beam_size):
        """select_candidates for several prompts at once (candidates seg[s]:seg[s+1]
        compete within prompt s).  Returns (child_ptr, tokens, scores, new_seg)."""
        seg = np.ascontiguousarray(seg, np.int32)
        n = int(seg[-1])
        tokens = np.ascontiguousarray(tokens, np.int32)
        logps = np.ascontiguousarray(logps, np.float64)
        k = tokens.shape[1] if tokens.ndim == 2 else 0
        ps = np.ascontiguousarray(parent_scores, np.float64)
        cap = max(1, (len(seg) - 1) * beam_size)
        ptr = np.zeros(n + 1, np.int32)
        ct = np.zeros(cap, np.int32)
        cs = np.zeros(cap, np.float64)
        ns = np.zeros(len(seg), np.int32)
        D = C.POINTER(C.c_double)
        check(lib().be_vanilla_select_segments(len(seg) - 1, _lib.addr(seg), k, ps.ctypes.data,
                                               _lib.addr(tokens), logps.ctypes.data,
                                               beam_size, _lib.addr(ptr), _lib.addr(ct),
                                               cs.ctypes.data, _lib.addr(ns)),
              "select_segments")
        m = int(ptr[-1])
        return ptr, ct[:m], cs[:m], ns

    def select_arrays(self, parent_scores, tokens, logps, beam_size):
        return vanilla_select_arrays(parent_scores, tokens, logps, beam_size)

    def should_stop(self, beam_state, max_length, step):
        if step >= max_length:
            return True
        if len(beam_state.leaves) == 0:
            return True
        if self.early_stopping and len(beam_state.finished_candidates) >= beam_state.beam_size:
            return True
        return False

    def get_final_sequences(self, beam_state, num_return=None):
        if num_return is None:
            num_return = beam_state.beam_size
        return beam_state.get_final_sequences(num_return, self.length_penalty)


class DiverseBeamSearchStrategy(BeamStrategy):
    """Diverse beam search (beam_strategy.py:60-400; Vijayakumar et al., AAAI 2018)."""

    # the engine passes its BeamState to select_segments (parent sequences)
    needs_state = True

    def __init__(self, num_groups: int = 4, diversity_penalty: float = 0.5,
                 diversity_type: str = "hamming", length_penalty: float = 1.0,
                 early_stopping: bool = True):
        self.num_groups = num_groups
        self.diversity_penalty = diversity_penalty
        self.diversity_type = diversity_type
        self.length_penalty = length_penalty
        self.early_stopping = early_stopping

    # -- beam_strategy.py:105-170 (single-choice helpers, kept for callers) --
    def _compute_hamming_diversity(self, candidate_token: int, selected_tokens) -> float:
        return self.diversity_penalty if candidate_token in selected_tokens else 0.0

    def _compute_cumulative_diversity(self, candidate_sequence, selected_sequences) -> float:
        if not selected_sequences:
            return 0.0
        total = 0.0
        for sel in selected_sequences:
            total += sum(1 for a, b in zip(candidate_sequence, sel) if a == b) * self.diversity_penalty
        return total / len(selected_sequences)

    def _apply_length_penalty(self, score: float, length: int) -> float:
        if self.length_penalty == 0:
            return score
        return score / (length ** self.length_penalty)

    # -- beam_strategy.py:173-317 --------------------------------------------
    def select_candidates(self, beam_state, new_candidates, step):
        if not new_candidates:
            return []
        n = len(new_candidates)
        k = max(len(x.children) for x in new_candidates)
        if any(len(x.children) != k for x in new_candidates):
            raise ValueError("every candidate must offer the same number of children")
        ps = np.asarray([x.candidate.score for x in new_candidates], np.float64)
        toks = np.asarray([[c.token_id for c in x.children] for x in new_candidates],
                          np.int32).reshape(n, k)
        lps = np.asarray([[c.log_prob for c in x.children] for x in new_candidates],
                         np.float64).reshape(n, k)
        leaves = np.asarray([x.candidate.trie_node._id for x in new_candidates], np.int32)
        sp, st = beam_state.leaf_sequences(leaves)
        ptr, ct, cs, _ = diverse_select_segments(
            np.array([0, n]), ps, toks, lps, sp, st, beam_state.beam_size, self.num_groups,
            self.diversity_penalty, self.diversity_type, self.length_penalty)
        return [BeamGenerateResult(candidate=x.candidate,
                                   children=[BeamToken(int(ct[j]), float(cs[j]))
                                             for j in range(ptr[i], ptr[i + 1])])
                for i, x in enumerate(new_candidates)]

    def select_segments(self, seg, parent_scores, tokens, logps, beam_size, state=None):
        """select_candidates for several prompts at once; ``state`` supplies the
        parents' sequences (its candidates are seg[0]..seg[-1])."""
        if state is None:
            raise ValueError("DiverseBeamSearchStrategy.select_segments needs the BeamState")
        sp, st = state.leaf_sequences()
        return diverse_select_segments(seg, parent_scores, tokens, logps, sp, st, beam_size,
                                       self.num_groups, self.diversity_penalty,
                                       self.diversity_type, self.length_penalty)

    # -- beam_strategy.py:319-353 --------------------------------------------
    def should_stop(self, beam_state, max_length, step):
        if step >= max_length:
            return True
        if self.early_stopping:
            if len(beam_state.leaves) == 0:
                return True
            # candidates only carry a finished flag once a caller materialised them
            objs = getattr(beam_state, "_cand_objs", None)
            if objs is not None and all(c.finished for c in objs):
                return True
        if len(beam_state.finished_candidates) >= beam_state.beam_size:
            return True
        return False

    def get_final_sequences(self, beam_state, num_return=None):
        if num_return is None:
            num_return = beam_state.beam_size
        return beam_state.get_final_sequences(num_return, self.length_penalty)

    # -- beam_strategy.py:375-400 --------------------------------------------
    def get_diverse_groups(self, beam_state):
        bpg = max(1, beam_state.beam_size // self.num_groups)
        cands = list(beam_state.finished_candidates) + list(beam_state.candidates)
        cands.sort(key=lambda x: x.score, reverse=True)
        groups = []
        for i in range(self.num_groups):
            a = i * bpg
            if a < len(cands):
                groups.append(cands[a:min(a + bpg, len(cands))])
        return groups
