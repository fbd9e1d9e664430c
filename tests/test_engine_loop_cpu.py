"""The engine's host loop (``BeamSearchGenerator.generate_ids``) on CPU with the
model replaced by a deterministic scorer: root expansion, per-step selection of
several prompts at once, trie updates, copy-on-write bookkeeping and the final
ranking must equal the oracle's restatement of the reference loop
(beam.py:48-352) run prompt by prompt on the same scorer.  The device step is
covered by the -m gpu tests; this pins everything around it."""
import hashlib

import numpy as np
import pytest
import torch

from beam_engine_b200.beam import BeamSearchGenerator
from beam_engine_b200.beam_strategy import DiverseBeamSearchStrategy, VanillaBeamSearchStrategy
from beam_engine_b200.page_table import PageTable
from oracle.beam_state import OracleBeamState, diverse_select, vanilla_select
from oracle.paging import OraclePageTable

VOCAB = 50


def fake_logprobs(seq):
    """Log-probabilities over VOCAB from the sequence alone (float32, like the
    device's scores), with frequent exact ties."""
    h = hashlib.sha256(np.asarray(seq, np.int64).tobytes()).digest()
    rng = np.random.default_rng(int.from_bytes(h[:8], "little"))
    x = np.round(rng.normal(0, 2, VOCAB) * 2) / 2
    x = x - x.max()
    lp = x - np.log(np.exp(x).sum())
    return lp.astype(np.float32)


def topk(lp, k):
    """Descending, ties by smaller token id (the device top-k's order)."""
    order = np.lexsort((np.arange(len(lp)), -lp.astype(np.float64)))[:k]
    return lp[order].astype(np.float64), order.astype(np.int32)


class FakeGenerator(BeamSearchGenerator):
    """BeamSearchGenerator with the device step replaced by fake_logprobs."""

    def __init__(self, strategy, page_size, pages):
        self.strategy = strategy
        self.page_table = PageTable(layer_num=1, page_size=page_size, max_num_pages=pages,
                                    head_num=1, head_dim=8, device="cpu",
                                    store_dtype=torch.bfloat16)
        self.model = type("M", (), {"vocab": VOCAB})()
        self.use_graph = True          # copies are deferred to the (fake) step graph
        self.use_graph_tree = False
        self._pending_fork = None
        self.forks = []
        self.steps = 0

    def prefill(self, state, prompts):
        for p in prompts:
            state.add_root_sequence(p)
        return np.stack([fake_logprobs(p) for p in prompts])

    def _topk(self, logits, k, temperature):
        out = [topk(row, k) for row in logits]
        return np.stack([v for v, _ in out]), np.stack([i for _, i in out])

    def decode_topk(self, state, k, temperature):
        self._take_fork_cpu()
        self.steps += 1
        return self._topk(np.stack([fake_logprobs(state.sequence(int(l))) for l in state.leaves]),
                          k, temperature)

    def _take_fork_cpu(self):
        if self._pending_fork is not None:
            self.forks.append(tuple(np.asarray(a).tolist() for a in self._pending_fork))
            self._pending_fork = None

    def _fork_now(self, copies):
        self.forks.append(tuple(np.asarray(a).tolist() for a in copies))


def oracle_generate(prompt, W, new_tokens, ps, strategy):
    """The reference loop on one prompt (oracle state, same scorer)."""
    st = OracleBeamState(W, OraclePageTable(1, ps, 4096, 1, 1, storage=False))
    st.add_root_sequence(prompt)
    k0 = min(2 * W, VOCAB)
    v, i = topk(fake_logprobs(prompt), k0)
    kw = min(W, k0)
    st.add_filtered_results([[(int(i[j]), float(v[j])) for j in range(kw)]])
    for _ in range(new_tokens - 1):
        if not st.cand_leaf:
            break
        k = min(2 * W, VOCAB) if W != 1 else 1
        kids = [topk(fake_logprobs(st.sequence(c)), k) for c in range(len(st.cand_leaf))]
        toks = [ki.tolist() for _, ki in kids]
        lps = [kv.tolist() for kv, _ in kids]
        if isinstance(strategy, DiverseBeamSearchStrategy):
            seqs = [st.sequence(c) for c in range(len(st.cand_leaf))]
            res = diverse_select(st.cand_score, seqs, toks, lps, W, strategy.num_groups,
                                 strategy.diversity_penalty, strategy.diversity_type,
                                 strategy.length_penalty)
        else:
            res = vanilla_select(st.cand_score, toks, lps, W)
        st.add_filtered_results(res)
    return st.final_sequences(W, strategy.length_penalty)


@pytest.mark.parametrize("strategy", [
    VanillaBeamSearchStrategy(length_penalty=1.0),
    DiverseBeamSearchStrategy(num_groups=2, diversity_penalty=0.5, diversity_type="hamming"),
    DiverseBeamSearchStrategy(num_groups=3, diversity_penalty=0.7, diversity_type="cumulative",
                              length_penalty=0.5),
], ids=["vanilla", "diverse_hamming", "diverse_cumulative"])
@pytest.mark.parametrize("W,ps", [(4, 16), (6, 4)])
def test_generate_ids_host_loop_matches_oracle(strategy, W, ps):
    rng = np.random.default_rng(W * 100 + ps)
    prompts = [rng.integers(0, VOCAB, n).tolist() for n in (9, 23, 16)]
    new_tokens = 12
    gen = FakeGenerator(strategy, ps, 2048)
    out = gen.generate_ids(prompts, W, max_new_tokens=new_tokens, num_return_sequences=W)
    gen._take_fork_cpu()
    assert gen.steps == new_tokens - 1
    for p, got in zip(prompts, out):
        want = oracle_generate(p, W, new_tokens, ps, strategy)
        assert [s for s, _ in got] == [s for s, _ in want]
        np.testing.assert_allclose([x for _, x in got], [x for _, x in want], rtol=0, atol=0)
    # every copy-on-write copy the updates asked for reached the (fake) device step
    assert all(len(a) == len(b) == len(c) for a, b, c in gen.forks)


@pytest.mark.parametrize("tree_pages,tiles", [(False, False), (True, False), (True, True)])
def test_pick_kernel_host_side(tree_pages, tiles):
    """kernel_type "auto": the per-step picker builds both plans on the host,
    returns a kind and stashes the tree plan for the step (page-list plan when
    tree_pages), along a trajectory with uneven beams.  With the beam-tile
    kernel every exact cascade step is a cascade step; a step whose cascade
    lists a page twice is always a tree step."""
    from types import SimpleNamespace
    from beam_engine_b200.picker import cascade_counts_pages_twice
    gen = FakeGenerator(VanillaBeamSearchStrategy(), 16, 2048)
    gen.use_tiles = tiles
    gen.model = SimpleNamespace(vocab=VOCAB, Hq=32, Hkv=8, D=128, Hq_total=32, Hkv_total=8)
    gen.attn = SimpleNamespace(plan=SimpleNamespace(num_sms=148))
    gen.picks, gen.tree_pages, gen._tree_stash = [], tree_pages, None
    from beam_engine_b200.beam_state import BeamState
    st = BeamState(8, gen.page_table)
    st.defer_copies = True
    rng = np.random.default_rng(5)
    gen.prefill(st, [rng.integers(0, VOCAB, 40).tolist(), rng.integers(0, VOCAB, 23).tolist()])
    st.update_native(st.leaves, np.array([0, 8, 16], np.int32),
                     rng.integers(0, VOCAB, 16).astype(np.int32), -rng.random(16))
    seg = np.array([0, 8, 16])
    kinds = []
    for _ in range(10):
        twice = cascade_counts_pages_twice(st.cascade_levels())
        kind = gen.pick_kernel(st)
        kinds.append(kind)
        if twice:
            assert kind == "fasttree"
        elif tiles:
            assert kind == "cascade"
        if kind == "fasttree":
            v, r2t, tinfo, tplan, pp = gen._tree_stash
            assert (pp is not None) == tree_pages
            assert (tplan is None) == tree_pages
            assert tinfo.n_work > 0
        else:
            assert gen._tree_stash is None
        vals, idx = gen.decode_topk(st, 16, 1.0)
        seg = st.vanilla_step(seg, idx, vals, 8)
    assert set(kinds) <= {"cascade", "fasttree"} and len(gen.picks) == 10


@pytest.mark.parametrize("ps", [16, 4])
@pytest.mark.parametrize("lens", [(37, 16, 5, 64), (1,), (16, 1, 17), (200,)])
def test_prefill_inputs(ps, lens):
    """The prefill's inputs and its plan: token ids, positions, each token's page
    and in-page slot along its prompt's root chain, the last row of every
    prompt, and the causal plan the native planner (be_cascade_plan, host code)
    builds from them.  Only the device copy and the model forward are stubbed,
    so every query of the plan must attend exactly positions 0..t of its own
    prompt (modeling_llama.py:213-283, prompt attention)."""
    from beam_engine_b200.beam_state import BeamState, TrieNode
    from beam_engine_b200.cascade import cascade_plan_host
    from test_host_native import plan_token_sets

    gen = FakeGenerator(VanillaBeamSearchStrategy(), ps, 4096)
    got = {}
    gen._to_device = lambda arrays: [torch.from_numpy(np.asarray(a).copy()) for a in arrays]

    class Attn:
        def plan_levels(self, levels, num_queries, causal=True, split_tokens=0):
            got["plan"] = cascade_plan_host(levels, num_queries, ps, 8, 2, causal=causal)
            got["num_queries"] = num_queries

    class Model:
        def forward(self, ids, pos, pt, wp, wpos, attn, logits_rows=None):
            got["a"] = [t.numpy() for t in (ids, pos, wp, wpos, logits_rows)]
            return "logits"

    gen.attn = Attn()
    gen.model = Model()
    st = BeamState(4, gen.page_table)
    rng = np.random.default_rng(1)
    prompts = [rng.integers(0, 1000, n).tolist() for n in lens]
    assert BeamSearchGenerator.prefill(gen, st, prompts) == "logits"
    ids, pos, wp, wpos, rows = got["a"]
    want = [[], [], [], []]
    want_sets = {}
    for leaf, pr in zip(st.leaves, prompts):
        chain = []
        node = TrieNode(trie=st._t, node_id=int(leaf), _owner=gen.page_table)
        while node is not None:
            chain.append(node.page_id)
            node = node.parent
        pages = chain[::-1]
        base = len(want[0])
        slots = [pages[i // ps] * ps + i % ps for i in range(len(pr))]
        for t in range(len(pr)):
            want_sets[base + t] = sorted(slots[:t + 1])
        want[0] += pr
        want[1] += list(range(len(pr)))
        want[2] += [pages[i // ps] for i in range(len(pr))]
        want[3] += [i % ps for i in range(len(pr))]
    assert [a.tolist() for a in (ids, pos, wp, wpos)] == want
    assert rows.tolist() == (np.cumsum([len(p) for p in prompts]) - 1).tolist()
    total = sum(lens)
    assert got["num_queries"] == total
    info, plan = got["plan"]
    assert info.n_queries == total
    assert plan_token_sets(plan, info, ps) == want_sets
