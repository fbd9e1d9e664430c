"""Native host page manager (C++ via the C ABI) against the reference fixtures.
CPU only: allocation, trie forks, cascade / FastTree metadata, selection."""
import math
import re
import os

import numpy as np
import pytest
import torch

from conftest import ROOT, load_json
from beam_engine_b200 import _lib
from beam_engine_b200.beam_state import BeamCandidate, BeamState, TrieNode
from beam_engine_b200.beam_strategy import VanillaBeamSearchStrategy, vanilla_select_arrays
from beam_engine_b200.fasttree import plan_vnodes
from beam_engine_b200.page_table import PageTable


def header_functions():
    names = set()
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            src = open(os.path.join(ROOT, "include", fn)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names |= set(re.findall(r"\b(be_\w+)\s*\(", src))
    return names


def test_library_exports_every_header_symbol():
    lib = _lib.lib()
    names = header_functions()
    assert len(names) > 20
    for n in sorted(names):
        assert hasattr(lib, n), n
    assert set(_lib.exported_symbols()) <= names | set()
    assert lib.be_version() >= 1


def cpu_table(ps, pages, layers=1):
    return PageTable(layer_num=layers, page_size=ps, max_num_pages=pages, head_num=1, head_dim=8,
                     device="cpu", store_dtype=torch.float32)


def state_from_spec(spec, ps):
    nodes, cands = spec
    made = []
    for n in nodes:
        par = made[n["parent"]] if n["parent"] >= 0 else None
        made.append(TrieNode(tokens=n["tokens"], page_id=n["page"], parent=par))
    bs = BeamState(len(cands), cpu_table(ps, 4))
    bs.candidates = [BeamCandidate(trie_node=made[c], score=0.0) for c in cands]
    return bs


def levels_as_lists(levels):
    return [{k: [int(x) for x in v] for k, v in lv.items()} for lv in levels]


@pytest.mark.parametrize("name", ["example", "swapped", "uneven"])
def test_cascade_known_answers_native(cascade_trees, name):
    t = cascade_trees[name]
    bs = state_from_spec((t["nodes"], t["candidates"]), t["page_size"])
    out = bs.get_cascade_input()
    qo, kvp, kvi, last, q = out[:5]
    got = [dict(qo_indptr=a.tolist(), kv_indptr=b.tolist(), kv_indices=c.tolist(),
                kv_last_page_len=d.tolist()) for a, b, c, d in zip(qo, kvp, kvi, last)]
    assert got == t["expect"]["levels"]
    assert q.tolist() == t["expect"]["query"]


@pytest.mark.parametrize("case", ["ps4_w4", "ps16_w8", "ps8_w6_churn", "ps16_w16"])
def test_trajectory_native(trajectories, case):
    rec = trajectories[case]
    cs = rec["case"]
    pt = cpu_table(cs["ps"], cs["pages"])
    bs = BeamState(cs["W"], pt)
    bs.add_root_sequence(rec["prompt"])
    toks, sc = rec["root_children"]
    bs.update_native(bs.leaves, np.array([0, len(toks)]), np.array(toks), np.array(sc))
    for step in rec["steps"]:
        assert levels_as_lists(bs.cascade_levels()) == step["cascade"]["levels"]
        q, wp, wpos, pos = bs.step_inputs()
        assert q.tolist() == step["cascade"]["query"]
        assert (wp.tolist(), wpos.tolist()) == (step["write_pages"], step["write_pos"])
        par, seql, kids, rptr, rl, r2t = bs.tree_arrays(per_node=False)
        tree = [dict(parent=int(par[i]), id=i, seqlen=int(seql[i]), num_children=int(kids[i]),
                     requests=rl[rptr[i]:rptr[i + 1]].tolist()) for i in range(len(par))]
        assert tree == step["tree"]
        assert r2t.tolist() == step["req_to_token"]
        B = len(bs.leaves)
        for key, per_node in (("ft_cumulative", False), ("ft_per_node", True)):
            p2, s2, k2, rp2, rl2, _ = bs.tree_arrays(per_node=per_node)
            v = plan_vnodes(p2, s2, k2, rp2, np.ascontiguousarray(rl2) if len(rl2) else np.zeros(1, np.int32),
                            r2t.shape[1], B, cs["hq"], cs["hkv"])
            for k, exp in step[key].items():
                assert [int(x) for x in v[k]] == exp, (key, k)
        kid_t = np.array([c[0] for c in step["children"]], np.int32)
        kid_l = np.array([c[1] for c in step["children"]], np.float64)
        ptr, ct, csc = vanilla_select_arrays(bs.scores, kid_t, kid_l, cs["W"])
        sel = [[[int(ct[j]), float(csc[j])] for j in range(ptr[i], ptr[i + 1])] for i in range(B)]
        assert sel == step["selected"]
        bs.update_native(bs.leaves, ptr, ct, csc)
        copies = [list(map(int, c)) for c in zip(*bs.last_copies)]
        assert copies == step["copies"]
        assert pt.free_pages == step["free_after"]
    final = bs.get_final_sequences(cs["W"], 1.0)
    assert [[s, x] for s, x in final] == rec["final"]


def test_allocator_errors_and_warnings():
    pt = cpu_table(4, 3)
    pages = [pt.allocate_block() for _ in range(3)]
    assert pages == [0, 1, 2]
    with pytest.raises(MemoryError):
        pt.allocate_block()
    pt.free_block(1)
    pt.free_block(1)          # double free: warning, no change
    assert pt.free_pages == [1]
    assert _lib.lib().be_trie_warnings(pt._trie) == 1
    pt.free_block(0)
    assert pt.free_pages == [1, 0]
    assert pt.allocate_block() == 1


def test_object_api_select_and_update():
    """The reference-style object API (BeamGenerateInput/Result) end to end."""
    from beam_engine_b200.beam_state import BeamGenerateInput, BeamTokenCandidate
    from beam_engine_b200.beam_strategy import VanillaBeamSearchStrategy
    pt = cpu_table(4, 32)
    bs = BeamState(2, pt)
    bs.add_root_sequence([1, 2, 3, 4, 5, 6])
    st = VanillaBeamSearchStrategy()
    inputs = [BeamGenerateInput(bs.candidates[0], [BeamTokenCandidate(7, -0.1),
                                                   BeamTokenCandidate(8, -0.2),
                                                   BeamTokenCandidate(9, -0.3)])]
    res = st.select_candidates(bs, inputs, 0)
    assert [(c.token_id, c.accumulated_score) for c in res[0].children] == [(7, -0.1), (8, -0.2)]
    bs.add_filtered_results(res)
    # partial tail page [5, 6] forked: copy for child 2 first, child 1 appends in place
    assert [c.trie_node.tokens for c in bs.candidates] == [[5, 6, 8], [5, 6, 7]]
    assert [list(map(int, c)) for c in zip(*bs.last_copies)] == [[1, 2, 2]]
    assert bs.candidates[0].trie_node.parent == bs.candidates[1].trie_node.parent


def test_fused_decode_inputs_match_separate_calls():
    """be_beam_decode_inputs (one call per step) writes exactly what
    step_inputs + cascade_levels + the cascade planner produce separately."""
    import ctypes as C
    from beam_engine_b200.cascade import cascade_plan_host
    rng = np.random.default_rng(3)
    pt = cpu_table(8, 4096)
    bs = BeamState(6, pt)
    bs.defer_copies = True
    for p in range(3):
        bs.add_root_sequence(rng.integers(0, 500, 40 + 13 * p).tolist())
    W = 6
    bs.update_native(bs.leaves, np.arange(4, dtype=np.int32) * W,
                     rng.integers(0, 500, 3 * W).astype(np.int32), -rng.random(3 * W))
    for step in range(12):
        n = len(bs.leaves)
        q, wp, wpos, pos = bs.step_inputs()
        info_ref, plan_ref = cascade_plan_host(bs.cascade_levels(), n, 8, 32, 8)
        off = -(-4 * n // 32) * 32
        buf = np.full(off + (1 << 16), -7, np.int32)
        info = _lib.AttnPlanInfo()
        leaves = np.ascontiguousarray(bs.leaves, np.int32)
        rc = _lib.lib().be_beam_decode_inputs(pt._trie, n, _lib.ptr32(leaves), 32, 8, 148,
                                              C.c_void_p(buf.ctypes.data), len(buf), off,
                                              C.byref(info))
        assert rc == _lib.BE_OK
        assert buf[:n].tolist() == list(q) and buf[n:2 * n].tolist() == list(pos)
        assert buf[2 * n:3 * n].tolist() == list(wp) and buf[3 * n:4 * n].tolist() == list(wpos)
        assert info.total_ints == info_ref.total_ints and info.n_work == info_ref.n_work
        assert buf[off:off + info.total_ints].tolist() == plan_ref[:info.total_ints].tolist()
        # three prompts' beams, selected together and one prompt at a time
        seg = np.array([0, n // 3, 2 * n // 3, n], np.int32)
        k = 2 * W
        tok = rng.integers(0, 500, (n, k)).astype(np.int32)
        lp = np.sort(-rng.random((n, k)) * 3, axis=1)[:, ::-1].copy()
        ptr, ct, cs, ns = VanillaBeamSearchStrategy().select_segments(seg, bs.scores, tok, lp, W)
        acc_p, acc_t, acc_s, acc_n = [0], [], [], [0]
        for s in range(3):
            a, b = seg[s], seg[s + 1]
            p1, t1, s1 = vanilla_select_arrays(bs.scores[a:b], tok[a:b], lp[a:b], W)
            acc_p += (p1[1:] + len(acc_t)).tolist()
            acc_t += t1.tolist()
            acc_s += s1.tolist()
            acc_n.append(acc_n[-1] + int(p1[-1]))
        assert ptr.tolist() == acc_p and ct.tolist() == acc_t and cs.tolist() == acc_s
        assert ns.tolist() == acc_n
        bs.update_native(bs.leaves, ptr, ct, cs)


def test_picker_exactness_and_cost(cascade_trees):
    """kernel_type "auto": an uneven tree (whose cascade levels list pages twice)
    goes to the tree plan; otherwise the cheaper plan by the launch model."""
    from beam_engine_b200.picker import PickerModel, cascade_counts_pages_twice, choose
    assert cascade_counts_pages_twice(cascade_trees["uneven"]["expect"]["levels"])
    assert not cascade_counts_pages_twice(cascade_trees["example"]["expect"]["levels"])
    assert not cascade_counts_pages_twice(cascade_trees["swapped"]["expect"]["levels"])

    def info(**kw):
        i = _lib.AttnPlanInfo()
        for k, v in kw.items():
            setattr(i, k, v)
        return i
    lv = cascade_trees["example"]["expect"]["levels"]
    shared = info(n_work=40, n_work_wide=8, total_tokens=9000, n_parts=200)
    tree_dup = info(n_work=300, n_work_wide=0, total_tokens=9000, n_parts=900)
    assert choose(lv, shared, tree_dup, 8, 32, 128) == "cascade"
    # a cascade that re-reads much more KV than the tree loses
    heavy = info(n_work=400, n_work_wide=300, total_tokens=400000, n_parts=3000)
    light = info(n_work=60, n_work_wide=0, total_tokens=20000, n_parts=200)
    assert choose(lv, heavy, light, 8, 32, 128) == "fasttree"
    m = PickerModel()
    assert m.cascade_us(shared, 8, 32, 128) < m.tree_us(tree_dup, 8, 32, 128)
    assert choose(cascade_trees["uneven"]["expect"]["levels"], shared, tree_dup, 8, 32, 128) == \
        "fasttree"
    # on the beam-tile kernel an exact cascade always wins; exactness still comes first
    assert choose(lv, heavy, light, 8, 32, 128, cascade_tiles=True) == "cascade"
    assert choose(cascade_trees["uneven"]["expect"]["levels"], shared, tree_dup, 8, 32, 128,
                  cascade_tiles=True) == "fasttree"


@pytest.mark.parametrize("case", ["ps16_w8", "ps8_w6_churn", "ps16_w16"])
def test_compressed_tree_plans_attend_the_same_tokens(trajectories, case):
    """Chains of single-child trie nodes merged into one tree node give vnode
    plans with fewer nodes and the same attention (oracle two-stage FastTree
    attention, float64) as one node per trie node."""
    from oracle.attention import fasttree_attention
    rec = trajectories[case]
    cs = rec["case"]
    pt = cpu_table(cs["ps"], cs["pages"])
    bs = BeamState(cs["W"], pt)
    bs.add_root_sequence(rec["prompt"])
    toks, sc = rec["root_children"]
    bs.update_native(bs.leaves, np.array([0, len(toks)]), np.array(toks), np.array(sc))
    rng = np.random.default_rng(4)
    hq, hkv, d = 8, 2, 16
    pool_k = rng.standard_normal((cs["pages"] * cs["ps"], hkv, d))
    pool_v = rng.standard_normal((cs["pages"] * cs["ps"], hkv, d))
    for si, step in enumerate(rec["steps"][:12]):
        B = len(bs.leaves)
        outs, sizes = [], []
        for comp in (False, True):
            par, seql, kids, rptr, rl, r2t = bs.tree_arrays(per_node=True, compress=comp)
            v = plan_vnodes(par, seql, kids, rptr, np.ascontiguousarray(rl) if len(rl) else
                            np.zeros(1, np.int32), r2t.shape[1], B, hq, hkv)
            v = {k: ([int(x) for x in a] if isinstance(a, np.ndarray) else a) for k, a in v.items()}
            q = np.random.default_rng(si).standard_normal((B, hq, d))
            outs.append(fasttree_attention(q, pool_k, pool_v, v, r2t.reshape(-1), d ** -0.5))
            sizes.append(len(par))
        assert sizes[1] <= sizes[0]
        np.testing.assert_allclose(outs[1], outs[0], atol=1e-12, rtol=0)
        kid_t = np.array([c[0] for c in step["children"]], np.int32)
        kid_l = np.array([c[1] for c in step["children"]], np.float64)
        ptr, ct, csc = vanilla_select_arrays(bs.scores, kid_t, kid_l, cs["W"])
        bs.update_native(bs.leaves, ptr, ct, csc)


def test_tree_plans_of_several_prompts_attend_each_request_exactly():
    """Several prompts decoded together make a forest: every request's vnodes
    must cover exactly its own tokens (oracle two-stage attention against dense
    attention over the request's token slots, float64)."""
    from oracle.attention import fasttree_attention
    rng = np.random.default_rng(5)
    W, ps, hq, hkv, d = 6, 16, 8, 2, 16
    pt = cpu_table(ps, 1024)
    bs = BeamState(W, pt)
    for p in range(3):
        bs.add_root_sequence(rng.integers(0, 1000, 40 + 9 * p).tolist())
    bs.update_native(bs.leaves, np.arange(4, dtype=np.int32) * W,
                     rng.integers(0, 1000, 3 * W).astype(np.int32), -rng.random(3 * W))
    kpool = rng.standard_normal((1024 * ps, hkv, d))
    vpool = rng.standard_normal((1024 * ps, hkv, d))
    for step in range(8):
        n = len(bs.leaves)
        lens = [len(bs.sequence(int(l))) for l in bs.leaves]
        for comp in (False, True):
            par, seql, kids, rptr, rl, r2t = bs.tree_arrays(per_node=True, compress=comp)
            v = plan_vnodes(par, seql, kids, rptr, np.ascontiguousarray(rl) if len(rl) else
                            np.zeros(1, np.int32), r2t.shape[1], n, hq, hkv)
            v = {k: ([int(x) for x in a] if isinstance(a, np.ndarray) else a) for k, a in v.items()}
            q = np.random.default_rng(step).standard_normal((n, hq, d))
            got = fasttree_attention(q, kpool, vpool, v, [int(x) for x in r2t.reshape(-1)], d ** -0.5)
            for c in range(n):
                sl = r2t[c, :lens[c]].astype(np.int64)
                K = np.repeat(kpool[sl], hq // hkv, axis=1)
                V = np.repeat(vpool[sl], hq // hkv, axis=1)
                s = np.einsum("hd,thd->ht", q[c], K) * d ** -0.5
                pr = np.exp(s - s.max(-1, keepdims=True))
                pr /= pr.sum(-1, keepdims=True)
                np.testing.assert_allclose(got[c], np.einsum("ht,thd->hd", pr, V), atol=1e-10)
        cnt = np.zeros(n, np.int32)
        for p in range(3):
            c = np.zeros(W, np.int32)
            c[: W // 2] = 2
            rng.shuffle(c)
            cnt[p * W:(p + 1) * W] = c
        ptr = np.concatenate([[0], np.cumsum(cnt)]).astype(np.int32)
        bs.update_native(bs.leaves, ptr, rng.integers(0, 1000, int(ptr[-1])).astype(np.int32),
                         -rng.random(int(ptr[-1])))


@pytest.mark.parametrize("seed", range(30))
def test_vanilla_select_matches_oracle_with_ties(seed):
    """be_vanilla_select against the oracle's stable sort on rows with many ties:
    rows in top-k order (the row-merge path) and rows in arbitrary order (the
    partial-sort path)."""
    from oracle.beam_state import vanilla_select
    rng = np.random.default_rng(seed)
    n, k = int(rng.integers(1, 20)), int(rng.integers(1, 40))
    W = int(rng.integers(1, 2 * n * k + 2))
    ps = np.round(rng.uniform(-3, 0, n) * 2) / 2
    lp = np.round(rng.uniform(-3, 0, (n, k)) * 4) / 4
    if seed % 2 == 0:
        lp = -np.sort(-lp, axis=1)
    toks = rng.integers(0, 1000, (n, k)).astype(np.int32)
    ptr, ct, cs = vanilla_select_arrays(ps, toks, lp, W)
    want = vanilla_select(ps.tolist(), toks.tolist(), lp.tolist(), W)
    got = [[(int(ct[j]), float(cs[j])) for j in range(ptr[i], ptr[i + 1])] for i in range(n)]
    assert got == want


def plan_token_sets(plan, info, ps, slots=None):
    """Per query: the sorted list of (slot id) tokens every work item of a plan
    makes it attend (slot = page * ps + i), from the plan buffer itself."""
    wk = plan[info.off_work:info.off_work + 8 * info.n_work].reshape(-1, 8)
    ql = plan[info.off_qlist:]
    kv = plan[info.off_kvlist:]
    out = {}
    for q_off, q_len, kv_off, b, e, kv_total, _, flags in wk:
        toks = []
        for t in range(b, e):
            if flags & 2:
                toks.append(int(slots[kv_off + t]))
            else:
                toks.append(int(kv[kv_off + t // ps]) * ps + t % ps)
        for i in range(q_len):
            lim = kv_total - q_len + i + 1 if flags & 1 else e   # causal: t < lim
            out.setdefault(int(ql[q_off + i]), []).extend(toks[:max(0, min(e, lim) - b)])
    return {q: sorted(v) for q, v in out.items()}


@pytest.mark.parametrize("case", ["ps4_w4", "ps16_w8", "ps8_w6_churn", "ps16_w16"])
def test_tree_page_plans_attend_what_slot_plans_attend(trajectories, case):
    """be_tree_plan_pages (page lists for the tensor-core kernels) makes every
    request attend exactly the tokens of the slot-list plan, each once, along
    a whole trajectory (forks, frees, merged single-child chains)."""
    from beam_engine_b200.fasttree import build_tree_page_plan, build_tree_plan
    rec = trajectories[case]
    cs = rec["case"]
    ps = cs["ps"]
    pt = cpu_table(ps, cs["pages"])
    bs = BeamState(cs["W"], pt)
    bs.add_root_sequence(rec["prompt"])
    toks, sc = rec["root_children"]
    bs.update_native(bs.leaves, np.array([0, len(toks)]), np.array(toks), np.array(sc))
    hq, hkv = 32, 8
    for step in rec["steps"]:
        B = len(bs.leaves)
        par, seql, kids, rptr, rl, r2t = bs.tree_arrays(per_node=True, compress=True)
        v = plan_vnodes(par, seql, kids, rptr, np.ascontiguousarray(rl) if len(rl) else
                        np.zeros(1, np.int32), r2t.shape[1], B, hq, hkv)
        slots = np.concatenate([r2t.reshape(-1), np.full(256, -1, np.int32)]).astype(np.int32)
        info_s, plan_s = build_tree_plan(v, B, ps, hq, hkv)
        got = build_tree_page_plan(v, slots, B, ps, hq, hkv)
        assert got is not None
        info_p, plan_p = got
        assert info_p.any_slots == 0 and info_p.max_wide_tokens <= 128
        want = plan_token_sets(plan_s, info_s, ps, slots)
        have = plan_token_sets(plan_p, info_p, ps)
        assert have == want
        for q, t in have.items():
            assert len(set(t)) == len(t)       # every token once
            assert len(t) == len(bs.sequence(int(bs.leaves[q])))   # the whole sequence
        kid_t = np.array([c[0] for c in step["children"]], np.int32)
        kid_l = np.array([c[1] for c in step["children"]], np.float64)
        ptr, ct, csc = vanilla_select_arrays(bs.scores, kid_t, kid_l, cs["W"])
        bs.update_native(bs.leaves, ptr, ct, csc)


@pytest.mark.parametrize("case", ["ps4_w4", "ps8_w6_churn", "ps16_w16"])
def test_fused_select_update_matches_reference_trajectory(trajectories, case):
    """be_beam_select_update (selection + trie update in one call) reproduces the
    reference trajectory: selections, copies, free list and final ranking."""
    rec = trajectories[case]
    cs = rec["case"]
    pt = cpu_table(cs["ps"], cs["pages"])
    bs = BeamState(cs["W"], pt)
    bs.add_root_sequence(rec["prompt"])
    toks, sc = rec["root_children"]
    bs.update_native(bs.leaves, np.array([0, len(toks)]), np.array(toks), np.array(sc))
    seg = np.array([0, len(bs.leaves)])
    for step in rec["steps"]:
        kid_t = np.array([c[0] for c in step["children"]], np.int32)
        kid_l = np.array([c[1] for c in step["children"]], np.float64)
        seg = bs.vanilla_step(seg, kid_t, kid_l, cs["W"])
        sel = step["selected"]
        cp = bs.last_child_ptr
        assert [int(cp[i + 1] - cp[i]) for i in range(len(sel))] == [len(s) for s in sel]
        assert sorted(bs.scores.tolist()) == sorted(x for s in sel for _, x in s)
        assert [list(map(int, c)) for c in zip(*bs.last_copies)] == step["copies"]
        assert pt.free_pages == step["free_after"]
        assert seg.tolist() == [0, len(bs.leaves)]
    final = bs.get_final_sequences(cs["W"], 1.0)
    assert [[s, x] for s, x in final] == rec["final"]


def test_native_pages_twice_check_matches_python(trajectories, cascade_trees):
    """be_cascade_pages_twice against the Python statement of the check, on the
    reference's cascade levels of every trajectory step and the known trees."""
    from beam_engine_b200.picker import cascade_counts_pages_twice, cascade_counts_pages_twice_py
    seen = set()
    for rec in trajectories.values():
        for step in rec["steps"]:
            lv = step["cascade"]["levels"]
            got = cascade_counts_pages_twice(lv)
            assert got == cascade_counts_pages_twice_py(lv)
            seen.add(got)
    for t in cascade_trees.values():
        lv = t["expect"]["levels"]
        assert cascade_counts_pages_twice(lv) == cascade_counts_pages_twice_py(lv)
    assert seen == {True, False}


def test_get_best_finished_ranks_active_by_score_per_token():
    pt = cpu_table(4, 32)
    bs = BeamState(3, pt)
    bs.add_root_sequence([1, 2, 3])
    bs.update_native(bs.leaves, np.array([0, 3], np.int32), np.array([7, 8, 9], np.int32),
                     np.array([-1.0, -2.0, -0.5]))
    best = bs.get_best_finished(2)
    # all sequences have 4 tokens: order by score
    assert [c.score for c in best] == [-0.5, -1.0]


_RUNS_ORDER_SCRIPT = r"""
import json, sys
import numpy as np
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[1] + '/tests')
from test_host_native import cpu_table, plan_token_sets
from beam_engine_b200.beam_state import BeamState
from beam_engine_b200.cascade import cascade_plan_host
rng = np.random.default_rng(0)
pt = cpu_table(16, 2048)
bs = BeamState(16, pt)
for _ in range(2):
    bs.add_root_sequence(rng.integers(0, 1000, 1000).tolist())
bs.update_native(bs.leaves, np.array([0, 16, 32], np.int32),
                 rng.integers(0, 1000, 32).astype(np.int32), -rng.random(32))
seg = np.array([0, 16, 32])
out = []
for step in range(6):
    n = len(bs.leaves)
    info, plan = cascade_plan_host(bs.cascade_levels(), n, 16, 32, 8, causal=True)
    wk = plan[info.off_work:info.off_work + 8 * info.n_work].reshape(-1, 8)
    out.append(dict(tokens={str(k): v for k, v in plan_token_sets(plan, info, 16).items()},
                    wide=[[int(x) for x in w] for w in wk[:info.n_work_wide]]))
    vals = -np.sort(rng.random((n, 32)) * 3, axis=1)
    idx = rng.integers(0, 1000, (n, 32)).astype(np.int32)
    seg = bs.vanilla_step(seg, idx, vals, 16)
print(json.dumps(out))
"""


def test_wide_runs_order_keeps_the_attention():
    """BE_ATTN_WIDE_RUNS=1 keeps wide items in creation order (each group's
    chunks adjacent): every query attends the same tokens as with the cost
    order, and consecutive wide items of one group have adjoining ranges."""
    import json
    import subprocess
    import sys
    runs = {}
    for flag in ("0", "1"):
        env = dict(os.environ, BE_ATTN_WIDE_RUNS=flag)
        r = subprocess.run([sys.executable, "-c", _RUNS_ORDER_SCRIPT, ROOT], env=env,
                           capture_output=True, text=True, timeout=300)
        assert r.returncode == 0, r.stderr[-2000:]
        runs[flag] = json.loads(r.stdout)
    adjoining = 0
    for a, b in zip(runs["0"], runs["1"]):
        assert a["tokens"] == b["tokens"]
        w = b["wide"]
        for x, y in zip(w, w[1:]):   # q_off, q_len, kv_off, kv_begin, kv_end, ...
            if x[0] == y[0] and x[2] == y[2] and x[4] == y[3]:
                adjoining += 1
    assert adjoining > 0


def test_ctypes_bindings_match_header_arities():
    """Every ctypes binding declares as many arguments as the header prototype
    (a mismatch passes garbage through the ABI without any error)."""
    src = open(os.path.join(ROOT, "include", "beam_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    protos = {}
    for m in re.finditer(r"\b(be_\w+)\s*\(([^;{]*?)\)\s*;", src, flags=re.S):
        args = m.group(2).strip()
        protos[m.group(1)] = 0 if args in ("", "void") else args.count(",") + 1
    sigs = _lib._SIGS
    checked = 0
    for name, (_, argtypes) in sigs.items():
        assert name in protos, name
        assert len(argtypes) == protos[name], (name, len(argtypes), protos[name])
        checked += 1
    assert checked > 30


def test_ctypes_return_types_match_header():
    import ctypes as C
    src = open(os.path.join(ROOT, "include", "beam_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    want = {"int": C.c_int, "int64_t": C.c_int64, "void*": C.c_void_p, "be_trie*": C.c_void_p,
            "be_comm*": C.c_void_p, "const char*": C.c_char_p, "void": None}
    for m in re.finditer(r"^\s*((?:const\s+)?\w+\s*\*?)\s*(be_\w+)\s*\(", src, flags=re.M):
        ret = re.sub(r"\s+", " ", m.group(1)).strip().replace(" *", "*")
        name = m.group(2)
        if name not in _lib._SIGS or ret == "typedef":
            continue
        assert ret in want, (name, ret)
        assert _lib._SIGS[name][0] is want[ret], (name, ret, _lib._SIGS[name][0])


_PREFILL_PLAN_SCRIPT = r"""
import json, sys
import numpy as np
sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[1] + '/tests')
from test_host_native import plan_token_sets
from beam_engine_b200.cascade import cascade_plan_host
rng = np.random.default_rng(1)
lens = [1000, 300, 1024, 77]
qo, kvp, kvi, last = [0], [0], [], []
perm = rng.permutation(4096).tolist()
for L in lens:
    m = -(-L // 16)
    kvi += perm[:m]; perm = perm[m:]
    kvp.append(len(kvi)); qo.append(qo[-1] + L); last.append(L - (m - 1) * 16)
lv = [dict(qo_indptr=qo, kv_indptr=kvp, kv_indices=kvi, kv_last_page_len=last)]
info, plan = cascade_plan_host(lv, qo[-1], 16, 32, 8, causal=True)
print(json.dumps(dict(max_wide=int(info.max_wide_tokens),
                      tokens={str(k): v for k, v in plan_token_sets(plan, info, 16).items()})))
"""


def test_causal_wide_chunk_cap_keeps_the_attention():
    """BE_PLAN_CAUSAL_WIDE_CHUNK=128 splits prefill (causal) wide groups into
    chunks the tcgen05 tile takes; every query still attends exactly its causal
    prefix."""
    import json
    import subprocess
    import sys
    res = {}
    for cap in ("0", "128"):
        env = dict(os.environ, BE_PLAN_CAUSAL_WIDE_CHUNK=cap)
        r = subprocess.run([sys.executable, "-c", _PREFILL_PLAN_SCRIPT, ROOT], env=env,
                           capture_output=True, text=True, timeout=300)
        assert r.returncode == 0, r.stderr[-2000:]
        res[cap] = json.loads(r.stdout)
    assert res["128"]["max_wide"] <= 128 < res["0"]["max_wide"]
    assert res["0"]["tokens"] == res["128"]["tokens"]
    # and each query's set is its own causal prefix: position j of a prompt sees j + 1 tokens
    t = res["128"]["tokens"]
    assert len(t["0"]) == 1 and len(t["999"]) == 1000 and len(t["1000"]) == 1


def test_new_entry_points_reject_bad_arguments():
    """Argument checks of the newer C entry points run before any device work:
    bad calls return BE_EINVAL with a message (no GPU needed)."""
    import ctypes as C
    L = _lib.lib()
    z = np.zeros(16, np.int32)
    # tree page plan: a vnode whose range does not start a page
    slots = np.arange(64, dtype=np.int32) + 3          # slot 3 is not a page start
    info = _lib.AttnPlanInfo()
    one, qlen, kvlen = (np.array([x], np.int32) for x in (0, 1, 20))
    rc = L.be_tree_plan_pages(1, _lib.addr(one), 1, _lib.addr(one), _lib.addr(qlen),
                              _lib.addr(one), _lib.addr(kvlen), _lib.addr(slots),
                              len(slots), 1, 16, 32, 8, 148, None, 0, C.byref(info))
    assert rc == _lib.BE_EINVAL and b"page aligned" in L.be_last_error()
    # peer all-reduce: no communicator / bad world
    h = (C.c_char * 64)()
    out = C.c_void_p()
    assert L.be_comm_create(9, 0, 1024, 2, 8, h, C.byref(out)) == _lib.BE_EINVAL
    assert L.be_comm_create(2, 2, 1024, 2, 8, h, C.byref(out)) == _lib.BE_EINVAL
    assert L.be_comm_allreduce_rmsnorm(None, 0, None, None, _lib.addr(z), 1, 8, 1e-6,
                                       _lib.BE_BF16, None) == _lib.BE_EINVAL
    assert L.be_comm_slot(None, 0) is None
    # fork list: null list
    assert L.be_fork_tail_copy_list(_lib.addr(z), 16, 1, 4, 16, 1, 8, _lib.BE_BF16, None, 4, 148,
                                    None) == _lib.BE_EINVAL
    # fused select + update: no beams
    seg = np.array([0, 0], np.int32)
    assert L.be_beam_select_update(None, 1, _lib.addr(seg), 2, None, None,
                                   None, None, 0, None, None, None, None, None, None, None, None,
                                   None) == _lib.BE_EINVAL
    # exactness check: negative level count
    assert L.be_cascade_pages_twice(-1, None, None, None, None, 0) == -_lib.BE_EINVAL


def test_picker_fit_recovers_a_known_model_and_drops_negative_terms():
    """fit_work_item_model: samples made by a known work-item model are fitted
    back to its per-launch and per-wave times and its bandwidth; a term the data contradicts
    (negative) is held at zero instead of crediting CTAs with negative time."""
    import random
    from types import SimpleNamespace
    from beam_engine_b200.picker import PickerModel, fit_work_item_model
    true = PickerModel(t_launch_us=2.5, t_wide_cta_us=13.0, t_narrow_cta_us=7.5)
    rnd = random.Random(0)
    samples = []
    for _ in range(16):
        nw = rnd.randint(8, 900)
        info = SimpleNamespace(n_work=nw, n_work_wide=rnd.randint(0, nw),
                               n_parts=rnd.randint(0, 4000), total_tokens=rnd.randint(500, 40000))
        samples.append(dict(us=true.cascade_us(info, 8, 32, 128), n_work=info.n_work,
                            n_work_wide=info.n_work_wide, n_parts=info.n_parts,
                            total_tokens=info.total_tokens, hkv=8, hq=32, d=128))
    fit = fit_work_item_model(samples)
    assert fit.t_launch_us == pytest.approx(2.5, abs=1e-6)
    assert fit.t_wide_cta_us == pytest.approx(13.0, abs=1e-6)
    assert fit.t_narrow_cta_us == pytest.approx(7.5, abs=1e-6)
    assert fit.hbm_gbs == pytest.approx(true.hbm_gbs, rel=1e-6)
    # times that fall as narrow waves grow: the narrow term is dropped, not negative
    for s in samples:
        s["us"] -= 5.0 * math.ceil((s["n_work"] - s["n_work_wide"]) / 148)
    fit = fit_work_item_model(samples)
    assert min(fit.t_launch_us, fit.t_wide_cta_us, fit.t_narrow_cta_us) >= 0.0
    with pytest.raises(ValueError):
        fit_work_item_model(samples[:3])


def test_diverse_select_device_argument_checks():
    """be_diverse_select_device refuses bad calls before any CUDA call (no GPU
    needed): null pointers, the cumulative penalty (host only), more entries
    per prompt than shared memory holds, more picks than the pick list holds."""
    L = _lib.lib()
    a = np.zeros(64, np.int64)
    p = a.ctypes.data

    def call(nseg=1, k=2, beam=4, groups=2, dtype=0, max_c=4, ptr=p):
        return L.be_diverse_select_device(nseg, ptr, k, p, p, p, p, beam, groups, 0.5, dtype, 1.0,
                                          max_c, p, p, p, p, None)
    assert call(ptr=None) == _lib.BE_EINVAL
    assert call(nseg=-1) == _lib.BE_EINVAL
    assert call(dtype=1) == _lib.BE_ENOTSUP
    assert b"hamming" in L.be_last_error()
    assert call(k=64, max_c=129) == _lib.BE_EINVAL
    assert call(beam=2048, groups=2048) == _lib.BE_EINVAL
    assert call(nseg=0) == _lib.BE_OK
