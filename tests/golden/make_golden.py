"""Generate the golden fixtures by running the UNMODIFIED reference engine.

Run in the build container (the reference tree is only present there):

    python tests/golden/make_golden.py      # BEAM_REF_SRC=<reference>/src if elsewhere

Writes ``tests/golden/*.json`` / ``*.npz``.  What each fixture pins:

* ``cascade_trees.json`` -- the hand-built trees of the reference's
  ``src/beam_engine/test_cascade.py`` (example :21-103, swapped :159-215,
  uneven :394-412) and the cascade indices ``BeamState.get_cascade_input``
  returns for them (the known-answer vectors of that test).
* ``trajectories.json`` (+ ``trajectory_pools.npz``) -- seeded beam-search
  trajectories driven through the reference ``PageTable`` + ``BeamState`` +
  ``VanillaBeamSearchStrategy`` on CPU: per step the cascade metadata,
  FastTree inputs, the reference FastTree planner's vnode metadata (as-is
  and with per-node ``seqlen``), the free list, the copy-on-write copies and
  the pool contents after the copies.
* ``fasttree_kernel.npz`` -- outputs of the reference Triton FastTree kernel
  (``attention/fasttree/kernel.py``) run by the Triton interpreter on a
  trajectory state with per-node metadata.
* ``diverse_trajectories.json`` -- seeded trajectories driven by the reference
  ``DiverseBeamSearchStrategy`` (hamming / cumulative / an unknown type string,
  1-5 groups, length penalty 0 / 0.7 / 1 / 2, tied log-probabilities, more
  groups than beams): parents' sequences, offered children, the selection,
  copies, free list and trie after each step, final ranking and groups.
* ``e2e_cfg1_diverse.json`` -- as ``e2e_cfg1.json`` with the diverse strategy
  (2 groups, hamming, penalty 0.5).
* ``e2e_cfg1.json`` -- the reference ``BeamSearchGenerator`` (cascade, vanilla
  strategy, fp32, CPU) on the tiny config: selected tokens per step and the
  final ranked sequences.  FlashInfer calls go through the CPU restatement in
  ``refshim.py``.
"""
from __future__ import annotations

import json
import os
import sys

os.environ.setdefault("TRITON_INTERPRET", "1")
HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import refshim  # noqa: E402

refshim.install()

import numpy as np  # noqa: E402
import torch  # noqa: E402

from beam_engine.page_table import PageTable  # noqa: E402
from beam_engine.beam_state import (BeamState, BeamCandidate, TrieNode,  # noqa: E402
                                    BeamGenerateInput, BeamTokenCandidate)
from beam_engine.beam_strategy import VanillaBeamSearchStrategy, DiverseBeamSearchStrategy  # noqa: E402
from beam_engine.attention.fasttree.preparation import prepare_fasttree_metadata_for_paged_cache  # noqa: E402
import logging  # noqa: E402

logging.disable(logging.WARNING)


def dump(name, obj):
    with open(os.path.join(HERE, name), "w") as f:
        json.dump(obj, f, separators=(",", ":"))
    print("wrote", name)


def tree_spec(bs):
    """Node list in BFS order from the root(s): (tokens, page, parent_index)."""
    roots = []
    for c in bs.candidates:
        n = c.trie_node
        while n.parent is not None:
            n = n.parent
        if all(n is not r for r in roots):
            roots.append(n)
    order, index = [], {}
    q = list(roots)
    while q:
        n = q.pop(0)
        if id(n) in index:
            continue
        index[id(n)] = len(order)
        order.append(n)
        q.extend(n.children)
    nodes = [dict(tokens=list(n.tokens), page=n.page_id,
                  parent=(index[id(n.parent)] if n.parent is not None else -1)) for n in order]
    cands = [index[id(c.trie_node)] for c in bs.candidates]
    return nodes, cands


def cascade_out(bs):
    out = bs.get_cascade_input()
    qo, kvp, kvi, last, q = out[:5]
    return dict(levels=[dict(qo_indptr=a.tolist(), kv_indptr=b.tolist(), kv_indices=c.tolist(),
                             kv_last_page_len=d.tolist()) for a, b, c, d in zip(qo, kvp, kvi, last)],
                query=q.tolist())


# ---------------------------------------------------------------------------
def make_cascade_trees():
    sys.path.insert(0, os.path.join(refshim.REF_SRC, "beam_engine"))
    import test_cascade as tc
    res = {}

    def table(P):
        return PageTable(layer_num=1, page_size=4, max_num_pages=P, head_num=2, head_dim=8,
                         device=torch.device("cpu"), store_dtype=torch.float32)

    for name, builder in (("example", tc.build_cascade_example_tree),
                          ("swapped", tc.build_cascade_swapped_tree)):
        bs = BeamState(beam_size=8, page_table=table(20))
        builder(bs)
        nodes, cands = tree_spec(bs)
        res[name] = dict(page_size=4, nodes=nodes, candidates=cands, expect=cascade_out(bs))
    # test_cascade.py:394-412 (uneven levels)
    bs = BeamState(beam_size=3, page_table=table(10))
    root = TrieNode(tokens=[1, 2], page_id=0, parent=None)
    a = TrieNode(tokens=[3, 4], page_id=1, parent=root)
    a1 = TrieNode(tokens=[5], page_id=2, parent=a)
    a2 = TrieNode(tokens=[6], page_id=3, parent=a)
    b = TrieNode(tokens=[7, 8, 9, 10], page_id=4, parent=root)
    b1 = TrieNode(tokens=[11], page_id=5, parent=b)
    bs.root = root
    bs.candidates = [BeamCandidate(trie_node=x, score=0.0) for x in (a1, a2, b1)]
    nodes, cands = tree_spec(bs)
    res["uneven"] = dict(page_size=4, nodes=nodes, candidates=cands, expect=cascade_out(bs))
    dump("cascade_trees.json", res)


# ---------------------------------------------------------------------------
def ft_meta(tree_nodes, r2t, B, hq, hkv, per_node, head_dim=16):
    from beam_engine.kv_tree_node import KVTreeNode
    nodes = []
    if per_node:
        # seqlen per node = own token count (cumulative minus parent's cumulative)
        cum = [t.seqlen for t in tree_nodes]
        for t in tree_nodes:
            n = KVTreeNode()
            n.parent, n.id, n.num_children = t.parent, t.id, t.num_children
            n.requests = list(t.requests)
            n.seqlen = cum[t.id] - (cum[t.parent] if t.parent >= 0 else 0)
            nodes.append(n)
    else:
        nodes = tree_nodes
    import contextlib
    import io
    with contextlib.redirect_stdout(io.StringIO()):
        m = prepare_fasttree_metadata_for_paged_cache(nodes, r2t, batch_size=B, num_qo_heads=hq,
                                                      num_kv_heads=hkv, head_dim=head_dim, device="cpu")
    n_v = m.phase_node_nums[0] + m.phase_node_nums[1]
    tot = int(m.req_to_vnode_lens[:B].sum())      # number of (vnode, request) entries
    return dict(
        vnode_to_q_entries=m.vnode_to_q_entries[:tot].tolist(),
        vnode_to_q_offs=m.vnode_to_q_offs[:n_v].tolist(),
        vnode_to_q_lens=m.vnode_to_q_lens[:n_v].tolist(),
        vnode_to_kv_offs=m.vnode_to_kv_offs[:n_v].tolist(),
        vnode_to_kv_lens=m.vnode_to_kv_lens[:n_v].tolist(),
        req_to_vnode_entries=m.req_to_vnode_entries[:tot].tolist(),
        req_to_vnode_offs=m.req_to_vnode_offs[:B].tolist(),
        req_to_vnode_lens=m.req_to_vnode_lens[:B].tolist(),
        phase_node_nums=list(m.phase_node_nums),
        phase_node_offsets=list(m.phase_node_offsets),
        phase_q_tile_sizes=list(m.phase_q_tile_sizes),
        phase_kv_tile_sizes=list(m.phase_kv_tile_sizes),
    ), m


def make_trajectories():
    cases = [
        dict(name="ps4_w4", seed=1, ps=4, pages=96, W=4, prompt=10, steps=14, temp=1.0, hq=4, hkv=2),
        dict(name="ps16_w8", seed=2, ps=16, pages=64, W=8, prompt=40, steps=24, temp=0.5, hq=8, hkv=2),
        dict(name="ps8_w6_churn", seed=3, ps=8, pages=128, W=6, prompt=8, steps=30, temp=3.0, hq=4, hkv=1),
        dict(name="ps16_w16", seed=4, ps=16, pages=200, W=16, prompt=33, steps=20, temp=2.0, hq=8, hkv=2),
    ]
    out, pools = {}, {}
    for cs in cases:
        g = torch.Generator().manual_seed(cs["seed"])
        L, H, D = 2, 2, 8
        pt = PageTable(layer_num=L, page_size=cs["ps"], max_num_pages=cs["pages"], head_num=H,
                       head_dim=D, device=torch.device("cpu"), store_dtype=torch.float32)
        for li in range(L):
            # the tests regenerate this initial pool from the same seed and draw order
            pt.kv_cache_at_layer[li].copy_(torch.randn(pt.kv_cache_at_layer[li].shape, generator=g))
        copies = []
        orig_copy = pt.copy_block

        def rec_copy(p, n, _orig=orig_copy, _c=copies):
            d = _orig(p, n)
            _c.append([p, d, n])
            return d

        pt.copy_block = rec_copy
        bs = BeamState(cs["W"], pt)
        strat = VanillaBeamSearchStrategy(length_penalty=1.0)
        prompt = torch.randint(0, 1000, (cs["prompt"],), generator=g).tolist()
        bs.add_root_sequence(prompt)
        from beam_engine.beam_state import BeamGenerateResult, BeamToken
        W = cs["W"]
        toks = torch.randperm(1000, generator=g)[:W].tolist()
        sc = sorted((-torch.rand(W, generator=g) * 3).tolist(), reverse=True)
        bs.add_filtered_results([BeamGenerateResult(candidate=bs.candidates[0],
                                                    children=[BeamToken(t, s) for t, s in zip(toks, sc)])])
        steps = []
        for step in range(cs["steps"]):
            rec = dict(spec=tree_spec(bs), scores=[c.score for c in bs.candidates])
            rec["cascade"] = cascade_out(bs)
            tree_nodes, r2t, qids, wpg, wpos = bs.get_fasttree_input()
            rec["tree"] = [dict(parent=t.parent, id=t.id, seqlen=t.seqlen, num_children=t.num_children,
                                requests=list(t.requests)) for t in tree_nodes]
            rec["req_to_token"] = r2t.tolist()
            rec["write_pages"], rec["write_pos"] = wpg.tolist(), wpos.tolist()
            B = len(bs.candidates)
            rec["ft_cumulative"], _ = ft_meta(tree_nodes, r2t, B, cs["hq"], cs["hkv"], False)
            rec["ft_per_node"], _ = ft_meta(tree_nodes, r2t, B, cs["hq"], cs["hkv"], True)
            # candidate children: 2W random tokens with sorted log-probs per beam
            inputs, kids = [], []
            for c in bs.candidates:
                t = torch.randperm(1000, generator=g)[:2 * W].tolist()
                lp = sorted((torch.log_softmax(torch.randn(2 * W, generator=g) * cs["temp"], 0)).tolist(),
                            reverse=True)
                kids.append([t, lp])
                inputs.append(BeamGenerateInput(candidate=c, children=[BeamTokenCandidate(a, b)
                                                                        for a, b in zip(t, lp)]))
            rec["children"] = kids
            res = strat.select_candidates(bs, inputs, step)
            rec["selected"] = [[[x.token_id, x.accumulated_score] for x in r.children] for r in res]
            ncopy = len(copies)
            bs.add_filtered_results(res)
            rec["copies"] = copies[ncopy:]
            rec["free_after"] = list(pt.free_pages)
            rec["allocated_after"] = sorted(pt.allocated_pages)
            steps.append(rec)
        final = bs.get_final_sequences(W, 1.0)
        pools[cs["name"] + "/final"] = np.stack([t.numpy() for t in pt.kv_cache_at_layer])
        out[cs["name"]] = dict(case=cs, prompt=prompt, root_children=[toks, sc], steps=steps,
                               final_spec=tree_spec(bs), final=[[s, float(x)] for s, x in final],
                               all_copies=copies)
    dump("trajectories.json", out)
    np.savez_compressed(os.path.join(HERE, "trajectory_pools.npz"), **pools)
    print("wrote trajectory_pools.npz")


# ---------------------------------------------------------------------------
def make_fasttree_kernel():
    from beam_engine.attention.fasttree.kernel import fasttree_decode
    with open(os.path.join(HERE, "trajectories.json")) as f:
        traj = json.load(f)
    out = {}
    for name, step_i, hq, hkv, D in (("ps16_w8", 10, 8, 2, 16), ("ps8_w6_churn", 20, 4, 1, 32)):
        rec = traj[name]["steps"][step_i]
        cs = traj[name]["case"]
        g = torch.Generator().manual_seed(100 + step_i)
        P, ps = cs["pages"], cs["ps"]
        pool = torch.randn((P, 2, ps, hkv, D), generator=g)
        B = len(rec["write_pages"])
        q = torch.randn((B, hq, D), generator=g)
        r2t = torch.tensor(rec["req_to_token"], dtype=torch.int32)
        from beam_engine.kv_tree_node import KVTreeNode
        nodes = []
        for t in rec["tree"]:
            n = KVTreeNode()
            n.parent, n.id, n.seqlen, n.num_children, n.requests = (t["parent"], t["id"], t["seqlen"],
                                                                    t["num_children"], list(t["requests"]))
            nodes.append(n)
        _, m = ft_meta(nodes, r2t, B, hq, hkv, True, head_dim=D)
        kbuf = pool[:, 0].reshape(P * ps, hkv, D).contiguous()
        vbuf = pool[:, 1].reshape(P * ps, hkv, D).contiguous()
        o = torch.empty_like(q)
        fasttree_decode(q, kbuf, vbuf, o, m.vnode_to_kv_entries, m.vnode_to_kv_offs, m.vnode_to_kv_lens,
                        m.vnode_to_q_entries, m.vnode_to_q_offs, m.vnode_to_q_lens,
                        m.req_to_vnode_entries, m.req_to_vnode_offs, m.req_to_vnode_lens,
                        m.mid_o, m.mid_lse, m.phase_node_nums, m.phase_node_offsets,
                        m.phase_q_tile_sizes, m.phase_kv_tile_sizes, D ** -0.5)
        out[f"{name}/pool"] = pool.numpy()
        out[f"{name}/q"] = q.numpy()
        out[f"{name}/o"] = o.numpy()
        out[f"{name}/meta"] = np.array([step_i, hq, hkv, D])
    np.savez_compressed(os.path.join(HERE, "fasttree_kernel.npz"), **out)
    print("wrote fasttree_kernel.npz")


# ---------------------------------------------------------------------------
CFG1 = dict(hidden_size=256, intermediate_size=688, num_hidden_layers=2, num_attention_heads=4,
            num_key_value_heads=2, head_dim=64, vocab_size=1024, rope_theta=10000.0, rms_norm_eps=1e-6)


E2E_DIVERSE = dict(num_groups=2, diversity_penalty=0.5, diversity_type="hamming", length_penalty=1.0)

DIVERSE_CASES = [
    dict(name="ham_w4_g2", seed=11, ps=4, pages=160, W=4, prompt=10, steps=14, vocab=12, quant=0.0,
         strat=dict(num_groups=2, diversity_penalty=0.5, diversity_type="hamming", length_penalty=1.0)),
    dict(name="ham_w8_g4_ties_nolp", seed=12, ps=8, pages=200, W=8, prompt=21, steps=12, vocab=20,
         quant=0.5, strat=dict(num_groups=4, diversity_penalty=1.5, diversity_type="hamming",
                               length_penalty=0.0)),
    dict(name="cum_w4_g4", seed=13, ps=4, pages=160, W=4, prompt=10, steps=14, vocab=10, quant=0.0,
         strat=dict(num_groups=4, diversity_penalty=0.3, diversity_type="cumulative",
                    length_penalty=1.0)),
    dict(name="cum_w6_g4_lp07_ties", seed=14, ps=16, pages=120, W=6, prompt=40, steps=12, vocab=14,
         quant=0.25, strat=dict(num_groups=4, diversity_penalty=0.8, diversity_type="cumulative",
                                length_penalty=0.7)),
    dict(name="ham_w3_g5_trunc", seed=15, ps=4, pages=120, W=3, prompt=7, steps=12, vocab=8, quant=0.0,
         strat=dict(num_groups=5, diversity_penalty=0.5, diversity_type="hamming", length_penalty=1.0)),
    dict(name="cum_w4_g1", seed=16, ps=8, pages=120, W=4, prompt=12, steps=10, vocab=10, quant=0.0,
         strat=dict(num_groups=1, diversity_penalty=0.5, diversity_type="cumulative",
                    length_penalty=1.0)),
    dict(name="other_type_w4_g2", seed=17, ps=4, pages=160, W=4, prompt=9, steps=10, vocab=10,
         quant=0.5, strat=dict(num_groups=2, diversity_penalty=0.4, diversity_type="overlap",
                               length_penalty=2.0)),
]


def make_diverse():
    """Seeded trajectories through the reference PageTable + BeamState +
    DiverseBeamSearchStrategy: per step the parents' sequences, the offered
    children, the selection and the allocator state after the fork."""
    from beam_engine.beam_state import BeamGenerateResult, BeamToken
    out = {}
    for cs in DIVERSE_CASES:
        g = torch.Generator().manual_seed(cs["seed"])
        pt = PageTable(layer_num=1, page_size=cs["ps"], max_num_pages=cs["pages"], head_num=1,
                       head_dim=4, device=torch.device("cpu"), store_dtype=torch.float32)
        copies = []
        orig_copy = pt.copy_block

        def rec_copy(p, n, _orig=orig_copy, _c=copies):
            d = _orig(p, n)
            _c.append([p, d, n])
            return d

        pt.copy_block = rec_copy
        bs = BeamState(cs["W"], pt)
        strat = DiverseBeamSearchStrategy(**cs["strat"])
        prompt = torch.randint(0, cs["vocab"], (cs["prompt"],), generator=g).tolist()
        bs.add_root_sequence(prompt)
        W = cs["W"]
        toks = torch.randperm(cs["vocab"], generator=g)[:W].tolist()
        sc = sorted((-torch.rand(W, generator=g) * 3).tolist(), reverse=True)
        bs.add_filtered_results([BeamGenerateResult(candidate=bs.candidates[0],
                                                    children=[BeamToken(t, s) for t, s in zip(toks, sc)])])
        steps = []
        for step in range(cs["steps"]):
            if not bs.candidates:
                break
            rec = dict(scores=[c.score for c in bs.candidates],
                       seqs=[strat._get_sequence_from_node(c.trie_node) for c in bs.candidates])
            inputs, kids = [], []
            k = min(2 * W, cs["vocab"])
            for c in bs.candidates:
                t = torch.randperm(cs["vocab"], generator=g)[:k].tolist()
                lp = torch.log_softmax(torch.randn(k, generator=g) * 2.0, 0)
                if cs["quant"]:
                    lp = torch.round(lp / cs["quant"]) * cs["quant"]
                lp = sorted(lp.tolist(), reverse=True)
                kids.append([t, lp])
                inputs.append(BeamGenerateInput(candidate=c, children=[BeamTokenCandidate(a, b)
                                                                        for a, b in zip(t, lp)]))
            rec["children"] = kids
            res = strat.select_candidates(bs, inputs, step)
            rec["selected"] = [[[x.token_id, x.accumulated_score] for x in r.children] for r in res]
            ncopy = len(copies)
            bs.add_filtered_results(res)
            rec["copies"] = copies[ncopy:]
            rec["free_after"] = list(pt.free_pages)
            rec["spec_after"] = tree_spec(bs)
            steps.append(rec)
        groups = [[c.score for c in grp] for grp in strat.get_diverse_groups(bs)]
        out[cs["name"]] = dict(case=cs, prompt=prompt, root_children=[toks, sc], steps=steps,
                               final=[[s, float(x)] for s, x in strat.get_final_sequences(bs)],
                               groups=groups)
    dump("diverse_trajectories.json", out)


def cfg1_weights(seed=0):
    """Seeded N(0, 0.02) weights (norms = 1) in a fixed generation order."""
    sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
    from beam_engine_b200.weights import random_llama_weights
    return random_llama_weights(CFG1, seed=seed, dtype=torch.float32, device="cpu")


def make_e2e(strategy="vanilla"):
    from beam_engine.models.configuration_llama import LlamaConfig
    import beam_engine.models.modeling_llama as ml
    from beam_engine.beam import BeamSearchGenerator
    ml.get_workspace_buffer = lambda: None
    ml.LlamaRotaryEmbedding.compute_default_rope_parameters = staticmethod(refshim.default_rope)
    cfg = LlamaConfig(vocab_size=CFG1["vocab_size"], hidden_size=CFG1["hidden_size"],
                      intermediate_size=CFG1["intermediate_size"],
                      num_hidden_layers=CFG1["num_hidden_layers"],
                      num_attention_heads=CFG1["num_attention_heads"],
                      num_key_value_heads=CFG1["num_key_value_heads"], head_dim=CFG1["head_dim"],
                      rope_theta=CFG1["rope_theta"], rms_norm_eps=CFG1["rms_norm_eps"],
                      max_position_embeddings=4096)
    model = ml.LlamaForCausalLM(cfg).float().eval()
    w = cfg1_weights(0)
    sd = {"model.embed_tokens.weight": w["embed"], "model.norm.weight": w["norm"], "lm_head.weight": w["lm_head"]}
    for i in range(CFG1["num_hidden_layers"]):
        p, q = f"model.layers.{i}.", f"layers.{i}."
        sd[p + "self_attn.q_proj.weight"] = w[q + "q"]
        sd[p + "self_attn.k_proj.weight"] = w[q + "k"]
        sd[p + "self_attn.v_proj.weight"] = w[q + "v"]
        sd[p + "self_attn.o_proj.weight"] = w[q + "o"]
        sd[p + "mlp.gate_proj.weight"] = w[q + "gate"]
        sd[p + "mlp.up_proj.weight"] = w[q + "up"]
        sd[p + "mlp.down_proj.weight"] = w[q + "down"]
        sd[p + "input_layernorm.weight"] = w[q + "input_norm"]
        sd[p + "post_attention_layernorm.weight"] = w[q + "post_norm"]
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not unexpected, unexpected
    assert all("rotary" in m for m in missing), missing

    class Tok:
        pad_token_id = 0
        eos_token_id = 1

        def __init__(self, ids):
            self.ids = ids

        def __call__(self, text, return_tensors="pt"):
            class R:
                pass
            r = R()
            r.input_ids = torch.tensor([self.ids])
            return r

        def decode(self, ids, skip_special_tokens=False):
            return " ".join(str(int(i)) for i in ids)

    prompt = torch.randint(0, 1024, (64,), generator=torch.Generator().manual_seed(0)).tolist()
    strat = (VanillaBeamSearchStrategy(length_penalty=1.0) if strategy == "vanilla" else
             DiverseBeamSearchStrategy(**E2E_DIVERSE))
    cls = type(strat)
    gen = BeamSearchGenerator(model, Tok(prompt), strat, page_size=16, kernel_type="cascade")
    gen.page_table = PageTable(layer_num=2, page_size=16, max_num_pages=256, head_num=2, head_dim=64,
                               device=torch.device("cpu"), store_dtype=torch.float32)
    trace = []
    orig = BeamState.add_filtered_results

    def traced(self, results):
        trace.append([[c.token_id for c in r.children] for r in results])
        return orig(self, results)

    BeamState.add_filtered_results = traced
    captured = {}
    orig_final = cls.get_final_sequences

    def fin(self, bs, num_return=None):
        r = orig_final(self, bs, num_return)
        captured["final"] = [[s, float(x)] for s, x in bs.get_final_sequences(len(bs.candidates), 1.0)]
        return r

    cls.get_final_sequences = fin
    with torch.no_grad():
        texts = gen.generate("x", beam_size=4, max_length=64 + 32, num_return_sequences=4)
    BeamState.add_filtered_results = orig
    cls.get_final_sequences = orig_final
    name = "e2e_cfg1.json" if strategy == "vanilla" else "e2e_cfg1_diverse.json"
    extra = {} if strategy == "vanilla" else dict(strategy=E2E_DIVERSE)
    dump(name, dict(config=CFG1, prompt=prompt, beam_size=4, max_length=96, page_size=16,
                    selections=trace, final=captured["final"], texts=texts, **extra))


if __name__ == "__main__":
    which = sys.argv[1:] or ["trees", "traj", "ftk", "e2e", "diverse", "e2e_diverse"]
    if "trees" in which:
        make_cascade_trees()
    if "traj" in which:
        make_trajectories()
    if "ftk" in which:
        make_fasttree_kernel()
    if "e2e" in which:
        make_e2e()
    if "diverse" in which:
        make_diverse()
    if "e2e_diverse" in which:
        make_e2e("diverse")
