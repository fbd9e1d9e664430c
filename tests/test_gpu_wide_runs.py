"""The persistent wide kernel with run accumulation (BE_ATTN_WIDE_RUNS=1:
consecutive chunks of one group accumulate in the CTA before one partial row is
written) against the dense fp32 reference, on plans whose groups span many
chunks."""

import pytest
import torch

from test_gpu_wide import ATOL, LSE_ATOL, dense_reference, dev, prompts_with_beams, run_plan

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("prefixes,beams", [((1000, 37, 300), (16, 8, 5)),
                                            ((2048, 1024, 4000), (16, 16, 12))])
def test_wide_runs_match_dense(monkeypatch, dtype, prefixes, beams):
    monkeypatch.setenv("BE_ATTN_WIDE", "1")
    monkeypatch.setenv("BE_ATTN_WIDE_RUNS", "1")
    d = dev()
    ps, Hq, Hkv, D, P = 16, 32, 8, 128, 1024
    g = torch.Generator().manual_seed(sum(prefixes) + 1)
    levels = prompts_with_beams(g, P, ps, prefixes, beams)
    n = sum(beams)
    pool = torch.randn((P, 2, ps, Hkv, D), generator=g).to(dtype).to(d)
    q = torch.randn((n, Hq, D), generator=g).to(dtype).to(d)
    info, out, lse = run_plan(levels, q, pool, ps, causal=True)
    assert info.n_work_wide > 0 and info.max_wide_tokens <= 128
    ref, ref_lse = dense_reference(levels, q, pool, ps, D ** -0.5, True)
    assert (out.float() - ref).abs().max().item() < ATOL
    assert (lse - ref_lse).abs().max().item() < LSE_ATOL
