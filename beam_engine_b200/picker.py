"""Tree-vs-cascade attention picker (``kernel_type="auto"``).

The reference has no picker: ``kernel_type`` is a fixed user choice
(``beam.py:20,34,168-206``), and its only cost model is FastTree's per-edge
split decision (``preparation.py:11-225``, alpha 0.6 / beta 0.3 / gamma 0.1),
which this build keeps inside the tree planner.  Here the choice is made per
decode step from the two plans the host builds anyway:

* exactness first: the reference's cascade metadata lists some pages at
  several levels when the beam tree is uneven (a candidate whose branch ends
  above the deepest level re-uses its deepest nodes at every later level,
  ``beam_state.py:299-302``), so those pages enter the softmax twice.  When a
  step's cascade levels do that, the tree plan (one vnode per trie node, each
  page once) is taken;
* otherwise, when the step runs on the beam-tile kernel (2-byte pools, head_dim
  128, page size 16), the cascade: measured on B200 at the cfg3 decode state
  (bench.py, CUDA events inside the step graph) it takes 28.3 us per layer for
  43 MB of K/V where the work-item kernels that run a tree page plan take
  55.6 us for the same tokens, so an exact cascade step is always cheaper;
* otherwise (fp32 parity mode, other shapes) the cheaper plan by a
  launch-level model of the work-item kernels:
  ``time = launches * t_launch + waves * t_cta + bytes / HBM``, where a wave
  is one CTA per SM (two for the tcgen05 prefix tiles), the bytes are every
  work item's K/V plus the partial rows written and merged.  The launch,
  per-wave and bandwidth terms are a least-squares fit
  (``fit_work_item_model``) to 32 cascade runs on the work-item kernels on
  B200 (``bench.py --op picker``: shared prefixes of 256-4096 tokens, 4-64
  beams with suffixes of up to 16 or 256 tokens, Hq 32 / Hkv 8 / D 128, bf16,
  cold L2; median error 5.5 %, largest 23 %): 6.17 us per launch, 0.60 us per
  wave of tcgen05 prefix tiles, 2.06 us per wave of suffix tiles, bytes at an
  effective 2 315 GB/s.  The slot-list (tree) tile's ~18 us is its measured
  lifetime; it only matters when page-list tree plans are off.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np


@dataclass
class PickerModel:
    num_sms: int = 148
    hbm_gbs: float = 2315.0          # effective, fitted (the copy peak is ~6 540)
    t_launch_us: float = 6.17
    t_wide_cta_us: float = 0.60      # per wave of tcgen05 prefix tiles (two CTAs per SM)
    t_narrow_cta_us: float = 2.06    # per wave of all-heads suffix tiles (one CTA per SM)
    t_slot_cta_us: float = 18.0      # slot-list tile of the tree plan (two CTAs per SM)

    def cascade_us(self, info, hkv, hq, d, elt=2):
        narrow = info.n_work - info.n_work_wide
        waves = (math.ceil(info.n_work_wide * hkv / (2 * self.num_sms)) * self.t_wide_cta_us
                 + math.ceil(narrow / self.num_sms) * self.t_narrow_cta_us)
        return 3 * self.t_launch_us + waves + self._bytes_us(info, hkv, hq, d, elt)

    def tree_us(self, info, hkv, hq, d, elt=2):
        waves = math.ceil(info.n_work * hkv / (2 * self.num_sms)) * self.t_slot_cta_us
        return 2 * self.t_launch_us + waves + self._bytes_us(info, hkv, hq, d, elt)

    def _bytes_us(self, info, hkv, hq, d, elt):
        kv = info.total_tokens * 2 * hkv * d * elt
        parts = info.n_parts * hq * (d + 1) * 4 * 2          # written, then read by the merge
        return (kv + parts) / (self.hbm_gbs * 1e3)


def work_item_waves(model: PickerModel, n_work, n_work_wide, hkv):
    """(wide waves, narrow waves) of a work-item plan, as ``cascade_us`` counts them."""
    return (math.ceil(n_work_wide * hkv / (2 * model.num_sms)),
            math.ceil((n_work - n_work_wide) / model.num_sms))


def fit_work_item_model(samples, base: PickerModel | None = None) -> PickerModel:
    """Least-squares fit of the work-item cost model to measured launches.

    ``samples``: dicts with the measured time of one cascade run on the
    work-item kernels (``us``) and its plan (``n_work``, ``n_work_wide``,
    ``n_parts``, ``total_tokens``, ``hkv``, ``hq``, ``d``, ``elt``).  Each time
    is fitted as ``3 * t_launch + wide_waves * t_wide_cta + narrow_waves *
    t_narrow_cta + bytes / hbm`` with the effective bandwidth ``hbm`` fitted
    too (as a multiple of ``base.hbm_gbs``).  A coefficient that comes out
    negative is dropped (held at zero) and the rest refitted, so the model
    never credits a CTA with negative time.  ``t_slot_cta_us`` (slot-list tree
    tiles, only used when page-list tree plans are off) is carried over from
    ``base``."""
    base = base or PickerModel()
    if len(samples) < 4:
        raise ValueError("need at least 4 samples to fit 4 coefficients")
    rows, rhs = [], []
    for s in samples:
        wide, narrow = work_item_waves(base, s["n_work"], s["n_work_wide"], s["hkv"])
        info = _PlanCounts(s["n_parts"], s["total_tokens"])
        rows.append([3.0, float(wide), float(narrow),
                     base._bytes_us(info, s["hkv"], s["hq"], s["d"], s.get("elt", 2))])
        rhs.append(s["us"])
    A, y = np.asarray(rows), np.asarray(rhs)
    keep = [0, 1, 2, 3]
    coef = np.zeros(4)
    while keep:
        sol = np.linalg.lstsq(A[:, keep], y, rcond=None)[0]
        if (sol >= 0).all():
            coef[keep] = sol
            break
        keep = [k for k, c in zip(keep, sol) if c >= 0]
    hbm = base.hbm_gbs / coef[3] if coef[3] > 0 else float("inf")
    return PickerModel(num_sms=base.num_sms, hbm_gbs=float(hbm),
                       t_launch_us=float(coef[0]), t_wide_cta_us=float(coef[1]),
                       t_narrow_cta_us=float(coef[2]), t_slot_cta_us=base.t_slot_cta_us)


@dataclass
class _PlanCounts:
    n_parts: int
    total_tokens: int


def cascade_counts_pages_twice(levels) -> bool:
    """True when some query attends one page at two levels (uneven trees);
    native (``be_cascade_pages_twice``)."""
    import ctypes as C
    from . import _lib
    from ._lib import check, lib
    L = len(levels)
    if L == 0:
        return False
    arrs = [[np.ascontiguousarray(lv[k], np.int32) for lv in levels]
            for k in ("qo_indptr", "kv_indptr", "kv_indices")]
    ptrs = [(C.c_void_p * L)(*[a.ctypes.data for a in grp]) for grp in arrs]
    ng = np.asarray([len(a) - 1 for a in arrs[0]], np.int32)
    nq = max(int(a[-1]) if len(a) else 0 for a in arrs[0])
    rc = lib().be_cascade_pages_twice(L, ptrs[0], ptrs[1], ptrs[2], _lib.addr(ng), nq)
    if rc < 0:
        check(-rc, "be_cascade_pages_twice")
    return rc == 1


def cascade_counts_pages_twice_py(levels) -> bool:
    """Pure-Python statement of the same check (kept as the test's reference)."""
    seen = {}
    for lv in levels:
        qo = np.asarray(lv["qo_indptr"])
        kvp = np.asarray(lv["kv_indptr"])
        kvi = np.asarray(lv["kv_indices"])
        for g in range(len(qo) - 1):
            pages = kvi[kvp[g]:kvp[g + 1]]
            if len(pages) == 0:
                continue
            for q in range(int(qo[g]), int(qo[g + 1])):
                s = seen.setdefault(q, set())
                for p in pages.tolist():
                    if p in s:
                        return True
                    s.add(p)
    return False


def choose(cascade_levels, cascade_info, tree_info, hkv, hq, d, model: PickerModel | None = None,
           elt=2, tree_pages=False, cascade_tiles=False) -> str:
    """'cascade' or 'fasttree' for one decode step.  ``tree_pages``: the tree
    step runs as a page-list plan on the same kernels as the cascade step, so it
    is costed by the cascade model on its own plan (``tree_info``).
    ``cascade_tiles``: the cascade step runs on the beam-tile kernel (the plan
    infos are not needed then)."""
    if cascade_counts_pages_twice(cascade_levels):
        return "fasttree"
    if cascade_tiles:
        return "cascade"
    m = model or PickerModel()
    tree = (m.cascade_us(tree_info, hkv, hq, d, elt) if tree_pages
            else m.tree_us(tree_info, hkv, hq, d, elt))
    return "cascade" if m.cascade_us(cascade_info, hkv, hq, d, elt) <= tree else "fasttree"
