"""Beam strategies with the reference's interface (src/beam_engine/beam_strategy.py).

``VanillaBeamSearchStrategy`` (beam_strategy.py:403-553): global top-``beam_size``
of ``parent.score + log_prob`` over every offered child, stable descending sort
in double precision, children regrouped per parent in sorted order; the native
``be_vanilla_select`` does the sort.  ``select_arrays`` is the array form the
engine uses (no per-token Python objects).
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
    check(lib().be_vanilla_select(n, k, parent_scores.ctypes.data_as(C.POINTER(C.c_double)),
                                  _lib.ptr32(tokens), logps.ctypes.data_as(C.POINTER(C.c_double)),
                                  beam_size, _lib.ptr32(ptr), _lib.ptr32(ct),
                                  cs.ctypes.data_as(C.POINTER(C.c_double))), "vanilla select")
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
        check(lib().be_vanilla_select_segments(len(seg) - 1, _lib.ptr32(seg), k, ps.ctypes.data_as(D),
                                               _lib.ptr32(tokens), logps.ctypes.data_as(D),
                                               beam_size, _lib.ptr32(ptr), _lib.ptr32(ct),
                                               cs.ctypes.data_as(D), _lib.ptr32(ns)),
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
