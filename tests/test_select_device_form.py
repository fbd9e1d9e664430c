"""Global top-W selection in the form the device writes it
(be_vanilla_select_device: per prompt, beam_size (parent, token, score) in
rank order) and the trie update from it (be_beam_update_selected): on CPU,
a step driven by the rank-form selection -- made here by the reference's
stable sort, VanillaBeamSearchStrategy.select_candidates
(beam_strategy.py:433-488) -- leaves the trie, scores, copies and free list
exactly as be_beam_select_update does.  The device kernel itself is checked
against the same rank form in tests/test_gpu_select.py."""
import numpy as np
import pytest

from beam_engine_b200.beam_state import BeamState
from test_host_native import cpu_table


def rank_form(seg, parent_scores, tokens, logps, W):
    """Per prompt: the reference's stable descending sort of (candidate, j)
    by parent score + logp, first W, as (parent, token, score) arrays of
    nseg * W entries (parent -1 past the prompt's entries)."""
    nseg = len(seg) - 1
    sp = np.full(nseg * W, -1, np.int32)
    st = np.zeros(nseg * W, np.int32)
    ss = np.zeros(nseg * W, np.float64)
    for s in range(nseg):
        flat = []
        for c in range(seg[s], seg[s + 1]):
            for j in range(tokens.shape[1]):
                flat.append((c, int(tokens[c, j]), float(parent_scores[c]) + float(logps[c, j])))
        flat.sort(key=lambda x: x[2], reverse=True)          # stable, like the reference
        for r, (c, t, sc) in enumerate(flat[:W]):
            sp[s * W + r], st[s * W + r], ss[s * W + r] = c, t, sc
    return sp, st, ss


@pytest.mark.parametrize("seed", range(6))
def test_update_from_rank_form_matches_select_update(seed):
    rng = np.random.default_rng(seed)
    W, k, ps = 6, 12, 8
    prompts = [rng.integers(0, 500, int(rng.integers(5, 40))).tolist() for _ in range(3)]
    states = []
    for _ in range(2):
        bs = BeamState(W, cpu_table(ps, 4096))
        bs.defer_copies = True
        for p in prompts:
            bs.add_root_sequence(p)
        states.append(bs)
    seg = np.arange(len(prompts) + 1, dtype=np.int32)        # one root candidate per prompt
    for step in range(12):
        n = int(seg[-1])
        # sorted rows (as the device top-k writes them) with frequent exact ties
        lp = -np.sort(np.round(rng.uniform(0, 3, (n, k)) * 4) / 4, axis=1)
        toks = rng.integers(0, 500, (n, k)).astype(np.int32)
        a, b = states
        seg_a = a.vanilla_step(seg, toks, lp, W)
        sp, st, ss = rank_form(seg, b.scores, toks, lp, W)
        seg_b = b.vanilla_step_selected(seg, sp, st, ss, W)
        assert seg_a.tolist() == seg_b.tolist()
        assert np.asarray(a.leaves).tolist() == np.asarray(b.leaves).tolist()
        assert np.asarray(a.scores).tolist() == np.asarray(b.scores).tolist()
        assert [x.tolist() for x in a.last_copies] == [x.tolist() for x in b.last_copies]
        assert a.last_child_ptr.tolist() == b.last_child_ptr.tolist()
        assert list(a.page_table.free_pages) == list(b.page_table.free_pages)
        seg = seg_a
