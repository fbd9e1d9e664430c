"""Wide (shared-prefix) tiles on the tensor cores: several prompts, beam counts
that leave the 64-row tile part empty, prefixes that end inside a page, causal
chunks, both 2-byte types.  Checked against a dense fp32 torch computation of
the same cascade (2e-2 absolute in bf16 / fp16), and
the natural-log LSE against the same reference (1e-2)."""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ATOL = 2e-2
LSE_ATOL = 1e-2


def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    return torch.device("cuda:0")


def dense_reference(levels, q, pool, ps, scale, causal_last):
    """Per query: concatenate the K/V of every level group it belongs to and
    run a plain softmax in fp32 (the last level causal when asked)."""
    n, Hq, D = q.shape
    Hkv = pool.shape[3]
    g = Hq // Hkv
    pf = pool.float()
    out = torch.empty((n, Hq, D), device=q.device)
    lse = torch.empty((n, Hq), device=q.device)
    for qi in range(n):
        ks, vs = [], []
        for li, lv in enumerate(levels):
            qo, kvp = lv["qo_indptr"], lv["kv_indptr"]
            for gi in range(len(qo) - 1):
                if not (qo[gi] <= qi < qo[gi + 1]):
                    continue
                pages = lv["kv_indices"][kvp[gi]:kvp[gi + 1]]
                if not pages:
                    continue
                L = (len(pages) - 1) * ps + lv["kv_last_page_len"][gi]
                if causal_last and li == len(levels) - 1:
                    L = min(L, L - (qo[gi + 1] - qo[gi]) + (qi - qo[gi]) + 1)
                pg = torch.tensor(pages, device=q.device)
                ks.append(pf[pg, 0].reshape(-1, Hkv, D)[:L])
                vs.append(pf[pg, 1].reshape(-1, Hkv, D)[:L])
        K = torch.cat(ks).repeat_interleave(g, dim=1)
        V = torch.cat(vs).repeat_interleave(g, dim=1)
        s = torch.einsum("hd,thd->ht", q[qi].float(), K) * scale
        out[qi] = torch.einsum("ht,thd->hd", torch.softmax(s, -1), V)
        lse[qi] = torch.logsumexp(s, -1)
    return out, lse


def run_plan(levels, q, pool, ps, causal, split_tokens=0):
    from beam_engine_b200 import _lib
    from beam_engine_b200.cascade import cascade_plan_host
    n, Hq, D = q.shape
    Hkv = pool.shape[3]
    info, plan = cascade_plan_host(levels, n, ps, Hq, Hkv, causal=causal, split_tokens=split_tokens)
    d = q.device
    pd = torch.from_numpy(plan).to(d)
    mo = torch.empty(max(1, info.n_parts) * Hq * D, dtype=torch.float32, device=d)
    ml = torch.empty(max(1, info.n_parts) * Hq, dtype=torch.float32, device=d)
    out = torch.full_like(q, float("nan"))
    lse = torch.full((n, Hq), float("nan"), dtype=torch.float32, device=d)
    dt = _lib.BE_BF16 if q.dtype == torch.bfloat16 else _lib.BE_F16
    _lib.check(_lib.lib().be_attn_run(pd.data_ptr(), C.byref(info), q.data_ptr(), q.stride(0),
                                      pool.data_ptr(), pool.shape[0], Hq, Hkv, D, dt, D ** -0.5,
                                      out.data_ptr(), out.stride(0), lse.data_ptr(), mo.data_ptr(),
                                      ml.data_ptr(), None, None))
    torch.cuda.synchronize()
    st = np.zeros(1, np.int32)
    _lib.check(_lib.lib().be_device_status(_lib.ptr32(st), None))
    assert st[0] == 0, st[0]
    return info, out, lse


def prompts_with_beams(g, P, ps, prefixes, beams, smax=70):
    """Level 0: one group per prompt (its prefix); level 1: one group per beam."""
    perm = torch.randperm(P, generator=g).tolist()
    off = 0
    lv0 = dict(qo_indptr=[0], kv_indptr=[0], kv_indices=[], kv_last_page_len=[])
    lv1 = dict(qo_indptr=[0], kv_indptr=[0], kv_indices=[], kv_last_page_len=[])
    for pre, W in zip(prefixes, beams):
        n = -(-pre // ps)
        lv0["kv_indices"] += perm[off:off + n]
        off += n
        lv0["kv_indptr"].append(len(lv0["kv_indices"]))
        lv0["kv_last_page_len"].append(pre - (n - 1) * ps)
        lv0["qo_indptr"].append(lv0["qo_indptr"][-1] + W)
        for L in torch.randint(1, smax, (W,), generator=g).tolist():
            m = -(-L // ps)
            lv1["kv_indices"] += perm[off:off + m]
            off += m
            lv1["kv_indptr"].append(len(lv1["kv_indices"]))
            lv1["kv_last_page_len"].append(L - (m - 1) * ps)
            lv1["qo_indptr"].append(lv1["qo_indptr"][-1] + 1)
    return [lv0, lv1]


@pytest.fixture(params=["0", "1"], ids=["per_cta_kernel", "persistent_kernel"])
def wide_kernel(request, monkeypatch):
    """Both tcgen05 kernels for wide tiles: one task per CTA, and persistent."""
    monkeypatch.setenv("BE_ATTN_WIDE", request.param)
    return request.param


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("prefixes,beams", [((1000, 37, 300), (16, 8, 5)),
                                            ((129, 128, 2048), (16, 16, 12))])
def test_wide_tiles_several_prompts(wide_kernel, dtype, prefixes, beams):
    d = dev()
    ps, Hq, Hkv, D, P = 16, 32, 8, 128, 1024
    g = torch.Generator().manual_seed(sum(prefixes))
    levels = prompts_with_beams(g, P, ps, prefixes, beams)
    n = sum(beams)
    pool = torch.randn((P, 2, ps, Hkv, D), generator=g).to(dtype).to(d)
    q = torch.randn((n, Hq, D), generator=g).to(dtype).to(d)
    info, out, lse = run_plan(levels, q, pool, ps, causal=True)
    assert info.n_work_wide > 0 and info.max_wide_tokens <= 128
    ref, ref_lse = dense_reference(levels, q, pool, ps, D ** -0.5, True)
    assert (out.float() - ref).abs().max().item() < ATOL
    assert (lse - ref_lse).abs().max().item() < LSE_ATOL


@pytest.mark.parametrize("n", [200, 77])
def test_wide_tiles_causal_chunks(wide_kernel, n):
    """A causal prefill split into <= 64-token chunks: tiles of 16 queries with
    rows that see none, part or all of a chunk."""
    d = dev()
    ps, Hq, Hkv, D, P = 16, 32, 8, 128, 64
    g = torch.Generator().manual_seed(n)
    npg = -(-n // ps)
    pages = torch.randperm(P, generator=g)[:npg].tolist()
    levels = [dict(qo_indptr=[0, n], kv_indptr=[0, npg], kv_indices=pages,
                   kv_last_page_len=[n - (npg - 1) * ps])]
    pool = torch.randn((P, 2, ps, Hkv, D), generator=g).to(torch.bfloat16).to(d)
    q = torch.randn((n, Hq, D), generator=g).to(torch.bfloat16).to(d)
    info, out, lse = run_plan(levels, q, pool, ps, causal=True, split_tokens=64)
    assert info.n_work_wide > 0 and info.max_wide_tokens <= 128
    ref, ref_lse = dense_reference(levels, q, pool, ps, D ** -0.5, True)
    assert (out.float() - ref).abs().max().item() < ATOL
    assert (lse - ref_lse).abs().max().item() < LSE_ATOL
