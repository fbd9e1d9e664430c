"""be_vanilla_select_device (global top-W of every prompt on the GPU,
VanillaBeamSearchStrategy.select_candidates, beam_strategy.py:433-488) against
the reference's stable sort on rows with many exact ties, several prompts per
launch, beam widths 1-32: parents, tokens and scores bit-identical.  Then a
whole beam search with the device selection equals one with the host
selection (be_vanilla_select_segments)."""
import numpy as np
import pytest
import torch

from test_select_device_form import rank_form

pytestmark = pytest.mark.gpu


def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    return torch.device("cuda:0")


@pytest.mark.parametrize("seed", range(8))
@pytest.mark.parametrize("W,k", [(1, 2), (4, 8), (16, 32), (32, 64), (5, 3)])
def test_device_selection_matches_reference_sort(seed, W, k):
    from beam_engine_b200 import _lib
    d = dev()
    rng = np.random.default_rng(seed * 100 + W)
    nseg = int(rng.integers(1, 9))
    counts = rng.integers(1, min(W, 8192 // k) + 1, nseg)
    seg = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    n = int(seg[-1])
    ps = np.round(rng.uniform(-6, 0, n) * 2) / 2
    lp = -np.sort(np.round(rng.uniform(0, 3, (n, k)) * 4) / 4, axis=1).astype(np.float32)
    toks = rng.integers(0, 128256, (n, k)).astype(np.int64)
    want = rank_form(seg, ps, toks, lp.astype(np.float64), W)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(d)   # noqa: E731
    seg_d, ps_d, lp_d, tok_d = t(seg), t(ps), t(lp), t(toks)
    sp = torch.full((nseg * W,), 7, dtype=torch.int32, device=d)
    st = torch.zeros(nseg * W, dtype=torch.int32, device=d)
    ss = torch.zeros(nseg * W, dtype=torch.float64, device=d)
    _lib.check(_lib.lib().be_vanilla_select_device(
        nseg, seg_d.data_ptr(), k, ps_d.data_ptr(), lp_d.data_ptr(), tok_d.data_ptr(), W,
        int(counts.max()), sp.data_ptr(), st.data_ptr(), ss.data_ptr(), None))
    torch.cuda.synchronize()
    got_p = sp.cpu().numpy()
    assert got_p.tolist() == want[0].tolist()
    ok = got_p >= 0
    assert st.cpu().numpy()[ok].tolist() == want[1][ok].tolist()
    assert ss.cpu().numpy()[ok].tolist() == want[2][ok].tolist()


def test_engine_with_device_selection_matches_host_selection(monkeypatch):
    """Three prompts, bf16 graph steps: the beams and scores of a search whose
    selection runs on the GPU equal the host-selection search's."""
    from beam_engine_b200.beam import BeamSearchGenerator
    from beam_engine_b200.beam_strategy import VanillaBeamSearchStrategy
    from beam_engine_b200.configs import TINY
    from beam_engine_b200.llama import BeamLlama
    cfg = dict(TINY, head_dim=128, num_attention_heads=4, num_key_value_heads=2, hidden_size=512)
    model = BeamLlama(cfg, None, dtype=torch.bfloat16, device=dev(), seed=3)
    g = torch.Generator().manual_seed(9)
    prompts = [torch.randint(0, 1024, (70,), generator=g).tolist() for _ in range(3)]
    outs = []
    for on in ("0", "1"):
        monkeypatch.setenv("BE_DEVICE_SELECT", on)
        gen = BeamSearchGenerator(model, None, VanillaBeamSearchStrategy(), page_size=16,
                                  max_num_pages=512)
        outs.append(gen.generate_ids(prompts, 8, max_new_tokens=24, num_return_sequences=8))
        assert gen.device_select == (on == "1")
    for a, b in zip(*outs):
        assert [s for s, _ in a] == [s for s, _ in b]
        assert [x for _, x in a] == [x for _, x in b]
