"""The CPU oracle against the reference's own outputs (fixtures made by
tests/golden/make_golden.py from the unmodified reference).  These pin the
oracle before it is trusted as the checker of the CUDA path."""
import numpy as np
import pytest

from conftest import initial_pool, load_json, load_npz
from oracle.attention import (cascade_attention, dense_attention, fasttree_attention,
                              fasttree_plan)
from oracle.beam_state import OracleBeamState, vanilla_select
from oracle.paging import OraclePageTable


def state_from_spec(spec, ps, pages=1024):
    nodes, cands = spec
    table = OraclePageTable(1, ps, pages, 1, 1, storage=False)
    st = OracleBeamState(len(cands), table)
    for n in nodes:
        st.new_node(n["tokens"], n["page"], None if n["parent"] < 0 else n["parent"])
    st.cand_leaf = list(cands)
    st.cand_score = [0.0] * len(cands)
    return st


@pytest.mark.parametrize("name", ["example", "swapped", "uneven"])
def test_cascade_known_answers(cascade_trees, name):
    t = cascade_trees[name]
    st = state_from_spec((t["nodes"], t["candidates"]), t["page_size"])
    levels, q = st.cascade_input()
    assert levels == t["expect"]["levels"]
    assert q == t["expect"]["query"]


def replay(case_rec, storage=True):
    cs = case_rec["case"]
    table = OraclePageTable(2, cs["ps"], cs["pages"], 2, 8, storage=storage)
    if storage:
        init = initial_pool(cs)
        table.kv = [init[0].copy(), init[1].copy()]
    st = OracleBeamState(cs["W"], table)
    st.add_root_sequence(case_rec["prompt"])
    toks, sc = case_rec["root_children"]
    st.add_filtered_results([list(zip(toks, sc))])
    return st, table


@pytest.mark.parametrize("case", ["ps4_w4", "ps16_w8", "ps8_w6_churn", "ps16_w16"])
def test_trajectory_replay(trajectories, case):
    rec = trajectories[case]
    cs = rec["case"]
    st, table = replay(rec)
    for step in rec["steps"]:
        levels, q = st.cascade_input()
        assert levels == step["cascade"]["levels"]
        assert q == step["cascade"]["query"]
        tree, r2t, _, wp, wpos = st.tree_input()
        assert tree == step["tree"]
        assert r2t == step["req_to_token"]
        assert (wp, wpos) == (step["write_pages"], step["write_pos"])
        B = len(st.cand_leaf)
        stride = len(r2t[0])
        for key, per_node in (("ft_cumulative", False), ("ft_per_node", True)):
            tr = tree if not per_node else st.tree_input(per_node=True)[0]
            plan = fasttree_plan(tr, stride, B, cs["hq"], cs["hkv"])
            exp = step[key]
            for k, v in exp.items():
                assert list(plan[k]) == v, (key, k)
        toks = [c[0] for c in step["children"]]
        lps = [c[1] for c in step["children"]]
        sel = vanilla_select(st.cand_score, toks, lps, cs["W"])
        assert [[[t, s] for t, s in x] for x in sel] == step["selected"]
        ncopy = len(st.copies)
        st.add_filtered_results(sel)
        assert [list(c) for c in st.copies[ncopy:]] == step["copies"]
        assert list(table.free_pages) == step["free_after"]
        assert sorted(table.allocated) == step["allocated_after"]
    final = st.final_sequences(cs["W"], 1.0)
    assert [[s, x] for s, x in final] == rec["final"]
    pools = load_npz("trajectory_pools.npz")
    np.testing.assert_array_equal(np.stack(table.kv), pools[case + "/final"])


@pytest.mark.parametrize("name", ["ps16_w8", "ps8_w6_churn"])
def test_fasttree_math_matches_reference_triton(trajectories, name):
    z = load_npz("fasttree_kernel.npz")
    step_i, hq, hkv, D = z[f"{name}/meta"].tolist()
    rec = trajectories[name]["steps"][step_i]
    pool, q, o_ref = z[f"{name}/pool"], z[f"{name}/q"], z[f"{name}/o"]
    P, _, ps = pool.shape[:3]
    B = q.shape[0]
    st = state_from_spec(rec["spec"], ps)
    tree = st.tree_input(per_node=True)[0]
    r2t = rec["req_to_token"]
    plan = fasttree_plan(tree, len(r2t[0]), B, hq, hkv)
    entries = [x for row in r2t for x in row]
    kf = pool[:, 0].reshape(P * ps, hkv, D)
    vf = pool[:, 1].reshape(P * ps, hkv, D)
    o = fasttree_attention(q, kf, vf, plan, entries, D ** -0.5)
    np.testing.assert_allclose(o, o_ref, atol=2e-5, rtol=1e-5)
    # and the tree path is plain attention over each request's full token list
    for b in range(B):
        sl = np.asarray(r2t[b][:sum(1 for _ in r2t[b])], np.int64)
        ln = len(st.sequence(b))
        dense = dense_attention(q[b], kf[sl[:ln]], vf[sl[:ln]], D ** -0.5)
        np.testing.assert_allclose(o[b], dense, atol=1e-9)


def test_cascade_equals_dense_attention_minus_own_token(trajectories):
    """Cascade semantics pinned against the reference's own slot tables: on
    trees where every candidate reaches the deepest level, the merged cascade
    output equals plain attention over the candidate's tokens except the
    newest one (quirk: the query's own K/V is appended but not attended)."""
    rec = trajectories["ps16_w8"]["steps"][12]
    rng = np.random.default_rng(0)
    ps, hq, hkv, D = 16, 8, 2, 16
    st = state_from_spec(rec["spec"], ps)
    pool = rng.standard_normal((64, 2, ps, hkv, D))
    B = len(st.cand_leaf)
    q = rng.standard_normal((B, hq, D))
    levels = rec["cascade"]["levels"]
    o = cascade_attention(q, pool, levels, ps, D ** -0.5)
    per_level = {}
    memo = {}
    depth = [st.level(leaf, memo) for leaf in st.cand_leaf]
    kf = pool[:, 0].reshape(-1, hkv, D)
    vf = pool[:, 1].reshape(-1, hkv, D)
    checked = 0
    for b in range(B):
        if depth[b] != len(levels) - 1:
            continue
        sl = np.asarray(rec["req_to_token"][b][:len(st.sequence(b)) - 1])
        dense = dense_attention(q[b], kf[sl], vf[sl], D ** -0.5)
        np.testing.assert_allclose(o[b], dense, atol=1e-10)
        checked += 1
    assert checked > 0
    del per_level


def test_e2e_cfg1_oracle_matches_reference():
    import torch
    from beam_engine_b200.weights import random_llama_weights
    from oracle.llama import OracleLlama, generate
    g = load_json("e2e_cfg1.json")
    cfg = g["config"]
    w = {k: v.numpy() for k, v in random_llama_weights(cfg, seed=0, dtype=torch.float32).items()}
    model = OracleLlama(cfg, w)
    trace = []
    final, st = generate(model, g["prompt"], g["beam_size"], g["max_length"], g["page_size"], 256,
                         trace=trace)
    assert [t["sel"] for t in trace] == g["selections"][1:]
    seqs = [s for s, _ in st.final_sequences(g["beam_size"], 1.0)]
    assert seqs == [s for s, _ in g["final"]]
    np.testing.assert_allclose([x for _, x in st.final_sequences(g["beam_size"], 1.0)],
                               [x for _, x in g["final"]], rtol=1e-5)
