"""Diverse beam search selection on the device (be_diverse_select_device,
hamming penalty) against the host selection be_diverse_select, bit-exact:
the reference's recorded hamming trajectories (diverse_trajectories.json,
from DiverseBeamSearchStrategy, beam_strategy.py:173-317), randomized
prompts decoded together with ties, groups beyond the beam width, and a
cfg3-sized case (8 prompts x 16 beams x top-32)."""
import random

import numpy as np
import pytest
import torch

from conftest import load_json
from beam_engine_b200.beam_strategy import diverse_select_device, diverse_select_segments

pytestmark = pytest.mark.gpu


def _both(seg, scores, toks, lps, lens, W, groups, dpen, lpen):
    """(host, device) outputs as lists: child_ptr, tokens, scores, new_seg."""
    seg = np.asarray(seg, np.int32)
    toks = np.asarray(toks, np.int32)
    lps = np.asarray(lps, np.float64).reshape(toks.shape)
    sp = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    st = np.zeros(max(1, int(sp[-1])), np.int32)      # hamming reads no sequences
    host = diverse_select_segments(seg, scores, toks, lps, sp, st, W, groups, dpen, "hamming", lpen)
    dev = torch.device("cuda", 0)
    t = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a, dt)).to(dev)  # noqa: E731
    ptr, ct, cs, ns = diverse_select_device(t(seg, np.int32), t(scores, np.float64),
                                            t(toks, np.int32), t(lps, np.float64),
                                            t(sp, np.int32), W, groups, dpen, lpen)
    torch.cuda.synchronize()
    m = int(ns[-1].item())
    got = (ptr.cpu().tolist(), ct[:m].cpu().tolist(), cs[:m].cpu().tolist(), ns.cpu().tolist())
    want = (host[0].tolist(), host[1].tolist(), host[2].tolist(), host[3].tolist())
    return want, got


@pytest.mark.parametrize("case", ["ham_w4_g2", "ham_w8_g4_ties_nolp", "ham_w3_g5_trunc"])
def test_reference_trajectories(case):
    rec = load_json("diverse_trajectories.json")[case]
    strat, W = rec["case"]["strat"], rec["case"]["W"]
    for step in rec["steps"]:
        n = len(step["scores"])
        toks = [c[0] for c in step["children"]]
        lps = [c[1] for c in step["children"]]
        want, got = _both([0, n], step["scores"], toks, lps, [len(s) for s in step["seqs"]], W,
                          strat["num_groups"], strat["diversity_penalty"],
                          strat["length_penalty"])
        assert got == want


@pytest.mark.parametrize("seed", range(30))
def test_randomized_segments(seed):
    """Several prompts in one launch (one empty), ties in log-probability and in
    penalised score, lengths that differ per parent, more groups than beams."""
    rng = random.Random(seed)
    nseg = rng.randint(1, 4)
    k = rng.randint(1, 6)
    W = rng.randint(1, 8)
    vocab = rng.randint(k, k + 3)
    counts = [rng.randint(0, 6) for _ in range(nseg)]
    seg = np.concatenate([[0], np.cumsum(counts)])
    n = int(seg[-1])
    if n == 0:
        counts[0] = 1
        seg = np.concatenate([[0], np.cumsum(counts)])
        n = 1
    scores = [round(rng.uniform(-4, 0), 1) for _ in range(n)]
    toks = [rng.sample(range(vocab), k) for _ in range(n)]
    lps = [sorted((round(rng.uniform(-3, 0) * 4) / 4 for _ in range(k)), reverse=True)
           for _ in range(n)]
    lens = [rng.randint(1, 9) for _ in range(n)]
    want, got = _both(seg, scores, toks, lps, lens, W, rng.randint(1, 10),
                      rng.choice([0.0, 0.25, 0.5, 1.3]), rng.choice([0.0, 1.0]))
    assert got == want


def test_cfg3_sized():
    rng = np.random.default_rng(3)
    nseg, W, k = 8, 16, 32
    n = nseg * W
    seg = np.arange(nseg + 1) * W
    toks = np.stack([rng.choice(5000, k, replace=False) for _ in range(n)]).astype(np.int32)
    lps = -np.sort(rng.exponential(2.0, (n, k)).round(2), axis=1)   # rounded: ties
    for groups, dpen, lpen in ((4, 0.5, 1.0), (16, 2.0, 0.0), (1, 0.0, 1.0)):
        want, got = _both(seg, -rng.random(n) * 10, toks, lps, rng.integers(1000, 1100, n), W,
                          groups, dpen, lpen)
        assert got == want


def test_cumulative_is_refused():
    from beam_engine_b200 import _lib
    dev = torch.device("cuda", 0)
    z32 = torch.zeros(4, dtype=torch.int32, device=dev)
    z64 = torch.zeros(4, dtype=torch.float64, device=dev)
    rc = _lib.lib().be_diverse_select_device(1, z32.data_ptr(), 1, z64.data_ptr(), z32.data_ptr(),
                                             z64.data_ptr(), z32.data_ptr(), 2, 2, 0.5, 1, 1.0, 1,
                                             z32.data_ptr(), z32.data_ptr(), z64.data_ptr(),
                                             z32.data_ptr(), None)
    assert rc == _lib.BE_ENOTSUP


@pytest.mark.parametrize("groups,lpen", [(2, 1.0), (4, 0.0)])
def test_engine_with_device_diverse_selection_matches_host(monkeypatch, groups, lpen):
    """Three prompts, bf16 graph steps, diverse (hamming) strategy: the beams and
    scores of a search whose selection runs inside the step graph on the GPU
    equal the host-selection search's."""
    from beam_engine_b200.beam import BeamSearchGenerator
    from beam_engine_b200.beam_strategy import DiverseBeamSearchStrategy
    from beam_engine_b200.configs import TINY
    from beam_engine_b200.llama import BeamLlama
    cfg = dict(TINY, head_dim=128, num_attention_heads=4, num_key_value_heads=2, hidden_size=512)
    model = BeamLlama(cfg, None, dtype=torch.bfloat16, device=torch.device("cuda", 0), seed=3)
    g = torch.Generator().manual_seed(9)
    prompts = [torch.randint(0, 1024, (70,), generator=g).tolist() for _ in range(3)]
    outs = []
    for on in ("0", "1"):
        monkeypatch.setenv("BE_DEVICE_SELECT", on)
        strat = DiverseBeamSearchStrategy(num_groups=groups, diversity_penalty=0.75,
                                          diversity_type="hamming", length_penalty=lpen)
        gen = BeamSearchGenerator(model, None, strat, page_size=16, max_num_pages=512)
        outs.append(gen.generate_ids(prompts, 8, max_new_tokens=24, num_return_sequences=8))
        sg = gen.step_graph_tiles
        assert sg is not None
        assert (sg.select is not None and sg.select[3] is not None) == (on == "1")
    for a, b in zip(*outs):
        assert [s for s, _ in a] == [s for s, _ in b]
        assert [x for _, x in a] == [x for _, x in b]
