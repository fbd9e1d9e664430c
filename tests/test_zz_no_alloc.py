"""be_attn_run_noalloc: attention for callers that cannot allocate device memory.

Hosts such as a serving process whose device pool is fixed at start-up, or a
plugin that may only use the tensors it is given, cannot hand be_attn_run the
two scratch buffers it needs for partial rows.  be_attn_run_noalloc keeps those
rows in an array built into the library instead.  This test calls it through
the C ABI and checks it against be_attn_run (caller-provided scratch) on two
calls in a row, with the attention tolerance the other tests use (2e-2 in
bf16), and both against the fp64 cascade oracle (the reference's
MultiLevelCascadeAttentionWrapper semantics, modeling_llama.py:321-367).  It lives in its own file, collected last, and needs nothing from the
other tests, so it also passes alone in a fresh process."""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

BF16_ATOL = 2e-2


def _levels(g, P, W=16, prefix=512, ps=16):
    perm = torch.randperm(P, generator=g)
    npre = prefix // ps
    off, kvp, kvi, last = npre, [0], [], []
    for L in torch.randint(1, 97, (W,), generator=g).tolist():
        n = -(-L // ps)
        kvi += perm[off:off + n].tolist()
        off += n
        kvp.append(len(kvi))
        last.append(L - (n - 1) * ps)
    return [dict(qo_indptr=[0, W], kv_indptr=[0, npre], kv_indices=perm[:npre].tolist(),
                 kv_last_page_len=[ps]),
            dict(qo_indptr=list(range(W + 1)), kv_indptr=kvp, kv_indices=kvi,
                 kv_last_page_len=last)]


def test_noalloc_matches_caller_scratch_twice():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from beam_engine_b200 import _lib
    from beam_engine_b200.cascade import cascade_plan_host
    d = torch.device("cuda:0")
    L = _lib.lib()
    Hq, Hkv, D, ps, P, W = 32, 8, 128, 16, 1024, 16
    g = torch.Generator().manual_seed(21)
    pool = torch.randn((P, 2, ps, Hkv, D), generator=g).to(torch.bfloat16).to(d)
    from oracle.attention import cascade_attention
    levels = _levels(g, P, W)
    info, plan = cascade_plan_host(levels, W, ps, Hq, Hkv, causal=True)
    used = sorted({p for x in levels for p in x["kv_indices"]})   # compacted pool for the oracle
    at = {p: i for i, p in enumerate(used)}
    pool_c = pool[torch.tensor(used, device=d)].double().cpu().numpy()
    lv_c = [dict(x, kv_indices=[at[p] for p in x["kv_indices"]]) for x in levels]
    assert info.n_parts > 0 and info.n_merge > 0          # the path that needs scratch
    plan_dev = torch.from_numpy(plan).to(d)
    mid_o = torch.empty(info.n_parts * Hq * D, dtype=torch.float32, device=d)
    mid_lse = torch.empty(info.n_parts * Hq, dtype=torch.float32, device=d)
    for call in range(2):
        q = torch.randn((W, Hq, D), generator=g).to(torch.bfloat16).to(d)
        ref = torch.empty_like(q)
        got = torch.full_like(q, float("nan"))
        _lib.check(L.be_attn_run(plan_dev.data_ptr(), C.byref(info), q.data_ptr(), q.stride(0),
                                 pool.data_ptr(), P, Hq, Hkv, D, _lib.BE_BF16, D ** -0.5,
                                 ref.data_ptr(), ref.stride(0), None, mid_o.data_ptr(),
                                 mid_lse.data_ptr(), None, None))
        _lib.check(L.be_attn_run_noalloc(plan_dev.data_ptr(), C.byref(info), q.data_ptr(),
                                         q.stride(0), pool.data_ptr(), P, Hq, Hkv, D, _lib.BE_BF16,
                                         D ** -0.5, got.data_ptr(), got.stride(0), None, None,
                                         None))
        torch.cuda.synchronize()
        err = (got.float() - ref.float()).abs().max().item()
        assert err <= BF16_ATOL, (call, err)
        want = cascade_attention(q.double().cpu().numpy(), pool_c, lv_c, ps, D ** -0.5)
        err_o = float(np.abs(got.float().cpu().numpy() - want).max())
        assert err_o <= BF16_ATOL, (call, err_o)


def test_noalloc_rejects_plans_beyond_its_scratch():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from beam_engine_b200 import _lib
    L = _lib.lib()
    info = _lib.AttnPlanInfo()
    info.n_parts = 100000                          # 100k rows x 32 heads x 129 floats >> 16 MiB
    info.group_size = 4
    info.page_size = 16
    buf = torch.zeros(64, dtype=torch.int32, device="cuda:0")
    rc = L.be_attn_run_noalloc(buf.data_ptr(), C.byref(info), buf.data_ptr(), 128, buf.data_ptr(),
                               1, 32, 8, 128, _lib.BE_BF16, 0.1, buf.data_ptr(), 4096, None,
                               None, None)
    assert rc == _lib.BE_ECAPACITY
    assert b"built-in scratch" in L.be_last_error()
