"""Diverse beam search (beam_strategy.py:60-400): the CPU oracle and the native
selection (be_diverse_select) against trajectories recorded from the
unmodified reference strategy, plus randomized agreement of the two on
shapes the fixtures do not reach (parents of different lengths).  CPU only."""
import random

import numpy as np
import pytest
import torch

from conftest import load_json
from beam_engine_b200.beam_state import BeamGenerateInput, BeamState, BeamTokenCandidate
from beam_engine_b200.beam_strategy import DiverseBeamSearchStrategy, diverse_select_segments
from beam_engine_b200.page_table import PageTable
from oracle.beam_state import diverse_select

CASES = ["ham_w4_g2", "ham_w8_g4_ties_nolp", "cum_w4_g4", "cum_w6_g4_lp07_ties", "ham_w3_g5_trunc",
         "cum_w4_g1", "other_type_w4_g2"]


@pytest.fixture(scope="module")
def diverse():
    return load_json("diverse_trajectories.json")


def as_lists(per_parent):
    return [[[int(t), float(s)] for t, s in kids] for kids in per_parent]


def native_step(step, W, strat, seg=None):
    n = len(step["scores"])
    seqs = step["seqs"]
    sp = np.zeros(n + 1, np.int32)
    sp[1:] = np.cumsum([len(s) for s in seqs])
    st = np.asarray([t for s in seqs for t in s], np.int32)
    toks = np.asarray([c[0] for c in step["children"]], np.int32)
    lps = np.asarray([c[1] for c in step["children"]], np.float64)
    seg = np.array([0, n]) if seg is None else seg
    ptr, ct, cs, ns = diverse_select_segments(seg, step["scores"], toks, lps, sp, st, W,
                                              strat["num_groups"], strat["diversity_penalty"],
                                              strat["diversity_type"], strat["length_penalty"])
    return [[[int(ct[j]), float(cs[j])] for j in range(ptr[i], ptr[i + 1])] for i in range(n)], ns


@pytest.mark.parametrize("case", CASES)
def test_oracle_matches_reference(diverse, case):
    rec = diverse[case]
    st, W = rec["case"]["strat"], rec["case"]["W"]
    for step in rec["steps"]:
        got = diverse_select(step["scores"], step["seqs"], [c[0] for c in step["children"]],
                             [c[1] for c in step["children"]], W, **st)
        assert as_lists(got) == step["selected"]


@pytest.mark.parametrize("case", CASES)
def test_native_matches_reference(diverse, case):
    rec = diverse[case]
    st, W = rec["case"]["strat"], rec["case"]["W"]
    for step in rec["steps"]:
        got, _ = native_step(step, W, st)
        assert got == step["selected"]


def spec_of(bs):
    """The fixture's trie layout: nodes in BFS order from the roots."""
    roots = []
    for c in bs.candidates:
        n = c.trie_node
        while n.parent is not None:
            n = n.parent
        if n not in roots:
            roots.append(n)
    order, index, q = [], {}, list(roots)
    while q:
        n = q.pop(0)
        if n in index:
            continue
        index[n] = len(order)
        order.append(n)
        q.extend(n.children)
    nodes = [dict(tokens=n.tokens, page=n.page_id,
                  parent=(index[n.parent] if n.parent is not None else -1)) for n in order]
    return [nodes, [index[c.trie_node] for c in bs.candidates]]


@pytest.mark.parametrize("case", CASES)
def test_trajectory_through_object_api(diverse, case):
    """Reference-style objects end to end: sequences, selection, forks, free list,
    trie layout, final ranking and groups."""
    rec = diverse[case]
    cs = rec["case"]
    pt = PageTable(layer_num=1, page_size=cs["ps"], max_num_pages=cs["pages"], head_num=1,
                   head_dim=4, device="cpu", store_dtype=torch.float32)
    bs = BeamState(cs["W"], pt)
    strat = DiverseBeamSearchStrategy(**cs["strat"])
    bs.add_root_sequence(rec["prompt"])
    toks, sc = rec["root_children"]
    bs.update_native(bs.leaves, np.array([0, len(toks)]), np.array(toks), np.array(sc))
    for i, step in enumerate(rec["steps"]):
        assert [c.score for c in bs.candidates] == step["scores"]
        sp, st = bs.leaf_sequences()
        assert [st[sp[j]:sp[j + 1]].tolist() for j in range(len(sp) - 1)] == step["seqs"]
        inputs = [BeamGenerateInput(c, [BeamTokenCandidate(t, lp) for t, lp in zip(*kids)])
                  for c, kids in zip(bs.candidates, step["children"])]
        res = strat.select_candidates(bs, inputs, i)
        assert [[[x.token_id, x.accumulated_score] for x in r.children] for r in res] == step["selected"]
        bs.add_filtered_results(res)
        assert [list(map(int, c)) for c in zip(*bs.last_copies)] == step["copies"]
        assert pt.free_pages == step["free_after"]
        assert spec_of(bs) == step["spec_after"]
    assert [[s, x] for s, x in strat.get_final_sequences(bs)] == rec["final"]
    assert [[c.score for c in g] for g in strat.get_diverse_groups(bs)] == rec["groups"]


def test_segments_are_independent(diverse):
    """Two prompts in one call select exactly as two separate calls."""
    rec = diverse["ham_w4_g2"]
    st, W = rec["case"]["strat"], rec["case"]["W"]
    a, b = rec["steps"][2], rec["steps"][5]
    both = dict(scores=a["scores"] + b["scores"], seqs=a["seqs"] + b["seqs"],
                children=a["children"] + b["children"])
    na = len(a["scores"])
    got, ns = native_step(both, W, st, seg=np.array([0, na, na + len(b["scores"])]))
    assert got[:na] == a["selected"] and got[na:] == b["selected"]
    assert ns.tolist() == [0, sum(map(len, a["selected"])),
                           sum(map(len, a["selected"])) + sum(map(len, b["selected"]))]


@pytest.mark.parametrize("seed", range(40))
def test_native_matches_oracle_randomized(seed):
    """Parents of different lengths (the overlap's unequal-length branches),
    shared prefixes, ties, unknown type strings, groups > choices."""
    rng = random.Random(seed)
    n = rng.randint(1, 6)
    k = rng.randint(1, 5)
    W = rng.randint(1, 8)
    vocab = rng.randint(k, k + 4)
    base = [rng.randrange(vocab) for _ in range(rng.randint(0, 6))]
    seqs = [base[:rng.randint(0, len(base))] + [rng.randrange(vocab) for _ in range(rng.randint(0, 4))]
            for _ in range(n)]
    scores = [round(rng.uniform(-4, 0), 1) for _ in range(n)]
    toks = [rng.sample(range(vocab), k) for _ in range(n)]
    lps = [sorted((round(rng.uniform(-3, 0) * 4) / 4 for _ in range(k)), reverse=True)
           for _ in range(n)]
    strat = dict(num_groups=rng.randint(1, 6), diversity_penalty=rng.choice([0.0, 0.25, 0.5, 1.3]),
                 diversity_type=rng.choice(["hamming", "cumulative", "other"]),
                 length_penalty=rng.choice([0, 0.5, 1.0, 2]))
    want = as_lists(diverse_select(scores, seqs, toks, lps, W, **strat))
    step = dict(scores=scores, seqs=seqs, children=[[t, l] for t, l in zip(toks, lps)])
    got, _ = native_step(step, W, strat)
    assert got == want


def test_empty_and_invalid():
    strat = DiverseBeamSearchStrategy()
    assert strat.select_candidates(None, [], 0) == []
    ptr, ct, cs, ns = diverse_select_segments(np.array([0]), np.zeros(0), np.zeros((0, 2), np.int32),
                                              np.zeros((0, 2)), np.zeros(1, np.int32),
                                              np.zeros(0, np.int32), 4, 2, 0.5, "hamming", 1.0)
    assert len(ct) == 0 and ns.tolist() == [0]
    with pytest.raises(ValueError):
        diverse_select_segments(np.array([0, 1]), np.zeros(1), np.zeros((1, 2), np.int32),
                                np.zeros((1, 2)), np.array([0, 1], np.int32), np.zeros(1, np.int32),
                                0, 2, 0.5, "hamming", 1.0)


def test_single_choice_helpers():
    """The reference's per-choice helpers (beam_strategy.py:105-155) kept on the class."""
    s = DiverseBeamSearchStrategy(diversity_penalty=0.5)
    assert s._compute_hamming_diversity(3, {1, 3}) == 0.5
    assert s._compute_hamming_diversity(4, {1, 3}) == 0.0
    assert s._compute_cumulative_diversity([1, 2, 3], []) == 0.0
    # overlaps 2 and 1 -> (2 * 0.5 + 1 * 0.5) / 2
    assert s._compute_cumulative_diversity([1, 2, 3], [[1, 2, 9], [7, 2]]) == 0.75
    assert s._apply_length_penalty(-2.0, 4) == -0.5
    assert DiverseBeamSearchStrategy(length_penalty=0)._apply_length_penalty(-2.0, 4) == -2.0
