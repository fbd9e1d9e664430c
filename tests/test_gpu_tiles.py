"""The beam-tile attention kernel (be_attn_tiles_run, tcgen05) against the fp64
cascade oracle -- the restatement of MultiLevelCascadeAttentionWrapper.run
(modeling_llama.py:321-367; FlashInfer cascade: per level, LSE-merged) -- on
cascade levels of the BASELINE cfg2 shape, of the reference's trajectories
(uneven trees with pages listed twice), of several prompts per launch, with
both tile heights (64 / 128 rows), one piece or many, bf16 and f16.
Tolerance: 2e-2 abs on outputs (bf16 / f16 pools), 2e-3 on the LSE."""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle.attention import cascade_attention

pytestmark = pytest.mark.gpu

ATOL = 2e-2
LSE_ATOL = 2e-3


def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    return torch.device("cuda:0")


def compact(pool, levels):
    """The pages the levels name, as a small float64 pool + remapped levels."""
    used = sorted({int(p) for lv in levels for p in lv["kv_indices"]})
    at = {p: i for i, p in enumerate(used)}
    idx = torch.tensor(used, dtype=torch.long, device=pool.device)
    small = pool[idx].double().cpu().numpy() if used else np.zeros((1,) + tuple(pool.shape[1:]))
    lv = [dict(lv, kv_indices=[at[int(p)] for p in lv["kv_indices"]]) for lv in levels]
    return small, lv


def run_tiles(levels, nq, q, pool, hq, hkv, tile_rows=None, pieces=None, lse=False, repeat=1,
              cluster=0):
    """Plan with be_tile_plan, run be_attn_tiles_run through the C ABI."""
    from beam_engine_b200 import _lib
    from beam_engine_b200.cascade import tile_plan_host
    from beam_engine_b200.page_table import dtype_code
    d = q.device
    got = tile_plan_host(levels, nq, 16, hq, hkv, tile_rows=tile_rows, pieces=pieces,
                         cluster=cluster)
    assert got is not None
    info, plan = got
    plan_d = torch.from_numpy(np.ascontiguousarray(plan)).to(d)
    slots = max(1, info.n_part_pieces) * hkv * info.tile_rows
    part_o = torch.empty(slots * 128, dtype=pool.dtype, device=d)
    part_l = torch.empty(slots, dtype=torch.float32, device=d)
    outs = []
    for _ in range(repeat):
        out = torch.full_like(q, float("nan"))
        l = torch.full((nq, hq), float("nan"), dtype=torch.float32, device=d) if lse else None
        rc = _lib.lib().be_attn_tiles_run(
            plan_d.data_ptr(), info.n_pieces, info.n_tiles, info.n_part_pieces, info.tile_rows,
            16, q.data_ptr(), q.stride(0), pool.data_ptr(), pool.shape[0], hq, hkv, 128,
            dtype_code(pool.dtype), 128 ** -0.5, out.data_ptr(), out.stride(0),
            l.data_ptr() if lse else None, part_o.data_ptr(), part_l.data_ptr(), info.cluster, 0,
            None)
        _lib.check(rc, "be_attn_tiles_run")
        torch.cuda.synchronize()
        outs.append((out, l))
    st = C.c_int(0)
    _lib.check(_lib.lib().be_device_status(C.byref(st), None))
    assert st.value == 0, f"device status {st.value}"
    return info, outs


def cfg2_levels(g, P, W=16, prefix=2048, max_suffix=256):
    perm = torch.randperm(P, generator=g).tolist()
    suf = torch.randint(1, max_suffix + 1, (W,), generator=g).tolist()
    npre = prefix // 16
    kvp, kvi, last, off = [0], [], [], npre
    for n_tok in suf:
        n = -(-n_tok // 16)
        kvi += perm[off:off + n]
        off += n
        kvp.append(len(kvi))
        last.append(n_tok - (n - 1) * 16)
    return [dict(qo_indptr=[0, W], kv_indptr=[0, npre], kv_indices=perm[:npre],
                 kv_last_page_len=[16]),
            dict(qo_indptr=list(range(W + 1)), kv_indptr=kvp, kv_indices=kvi,
                 kv_last_page_len=last)]


def check(out, levels, q, pool, lse=None):
    small, lv = compact(pool, levels)
    want, want_lse = cascade_attention(q.double().cpu().numpy(), small, lv, 16, 128 ** -0.5,
                                       return_lse=True)
    err = float(np.abs(out.float().cpu().numpy() - want).max())
    assert err <= ATOL, err
    if lse is not None:
        got = lse.cpu().numpy()
        fin = np.isfinite(want_lse)
        assert (np.isfinite(got) == fin).all()
        assert float(np.abs(got[fin] - want_lse[fin]).max()) <= LSE_ATOL
    return err


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("pieces,cluster", [(None, 0), (1, 0), (64, 0), (None, 2), (None, 7),
                                            (None, 16)])
def test_cfg2_shape_matches_oracle(dtype, pieces, cluster):
    """Partial rows merged by the merge kernel (cluster 0) or on chip by clusters
    of 2 / 7 / 16 CTAs through distributed shared memory."""
    d = dev()
    g = torch.Generator().manual_seed(7)
    P = 8192
    levels = cfg2_levels(g, P)
    pool = torch.randn((P, 2, 16, 8, 128), generator=g).to(dtype).to(d)
    q = torch.randn((16, 32, 128), generator=g).to(dtype).to(d)
    info, outs = run_tiles(levels, 16, q, pool, 32, 8, pieces=pieces, lse=True, repeat=2,
                           cluster=cluster)
    assert info.cluster == (cluster if cluster > 1 else 0)
    assert info.tile_rows == 64
    for out, l in outs:
        check(out, levels, q, pool, l)
    assert torch.equal(outs[0][0], outs[1][0])      # the rerun over the same scratch is identical


@pytest.mark.parametrize("case", ["ps16_w8", "ps16_w16"])
@pytest.mark.parametrize("hq,hkv", [(32, 8), (64, 8), (128, 8)])
def test_reference_trajectory_levels(trajectories, case, hq, hkv):
    """Every step of a reference trajectory (forks, uneven trees listing pages
    twice); 128 q heads over 8 KV heads makes 16-row groups, so 16 beams need
    two 128-row tiles."""
    d = dev()
    rec = trajectories[case]
    P = rec["case"]["pages"]
    g = torch.Generator().manual_seed(1)
    pool = torch.randn((P, 2, 16, hkv, 128), generator=g).to(torch.bfloat16).to(d)
    for step in rec["steps"][::3]:
        levels = step["cascade"]["levels"]
        nq = len(step["cascade"]["query"])
        q = torch.randn((nq, hq, 128), generator=g).to(torch.bfloat16).to(d)
        for pieces, cluster in ((None, 0), (3, 0), (None, 4), (64, -1)):
            _, outs = run_tiles(levels, nq, q, pool, hq, hkv, pieces=pieces, lse=True,
                                cluster=cluster)
            check(outs[0][0], levels, q, pool, outs[0][1])


def test_several_prompts_through_the_wrapper():
    """Three prompts of 12 beams (g = 8, so a prompt's 96 rows use a 128-row tile)
    through MultiLevelCascadeAttentionWrapper.plan / .run, which picks the tile
    kernel, along a beam trajectory with forks."""
    from beam_engine_b200.beam_state import BeamState
    from beam_engine_b200.cascade import MultiLevelCascadeAttentionWrapper
    from beam_engine_b200.page_table import PageTable
    d = dev()
    rng = np.random.default_rng(4)
    W, hq, hkv = 12, 64, 8
    pt = PageTable(1, 16, 2048, hkv, 128, device=d, store_dtype=torch.bfloat16)
    pt.kv_cache.normal_(generator=torch.Generator(device=d).manual_seed(3))
    bs = BeamState(W, pt)
    for p in range(3):
        bs.add_root_sequence(rng.integers(0, 500, 100 + 37 * p).tolist())
    bs.update_native(bs.leaves, np.arange(4, dtype=np.int32) * W,
                     rng.integers(0, 500, 3 * W).astype(np.int32), -rng.random(3 * W))
    ws = torch.empty(64 << 20, dtype=torch.uint8, device=d)
    for step in range(12):
        n = len(bs.leaves)
        levels = bs.cascade_levels()
        w = MultiLevelCascadeAttentionWrapper(len(levels), ws)
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.int32))  # noqa: E731
        w.plan([t(x["qo_indptr"]) for x in levels], [t(x["kv_indptr"]) for x in levels],
               [t(x["kv_indices"]) for x in levels], [t(x["kv_last_page_len"]) for x in levels],
               hq, hkv, 128, 16, causal=True, sm_scale=128 ** -0.5)
        assert w.tiles
        q = torch.from_numpy(rng.standard_normal((n, hq, 128))).to(torch.bfloat16).to(d)
        o, l = w.run(q, pt.kv_cache_at_layer[0], return_lse=True)
        torch.cuda.synchronize()
        lv = [{k: [int(x) for x in v] for k, v in x.items()} for x in levels]
        check(o, lv, q, pt.kv_cache_at_layer[0], l)
        cnt = np.zeros(n, np.int32)
        for p in range(3):
            c = np.zeros(W, np.int32)
            c[: W // 2] = 2
            rng.shuffle(c)
            cnt[p * W:(p + 1) * W] = c
        ptr = np.concatenate([[0], np.cumsum(cnt)]).astype(np.int32)
        bs.update_native(bs.leaves, ptr, rng.integers(0, 500, int(ptr[-1])).astype(np.int32),
                         -rng.random(int(ptr[-1])))


def test_empty_queries_and_non_finite_stale_slots():
    """Queries without pages get 0 and LSE -inf; NaN in page slots past the valid
    tokens (never written) must not reach any output."""
    d = dev()
    g = torch.Generator().manual_seed(5)
    P = 64
    pool = torch.randn((P, 2, 16, 2, 128), generator=g).to(torch.bfloat16)
    pool[11, :, 3:] = float("nan")          # slots past last_page_len 3
    pool[12, :, 5:] = float("inf")          # slots past last_page_len 5
    pool = pool.to(d)
    levels = [dict(qo_indptr=[0, 2, 4], kv_indptr=[0, 0, 2], kv_indices=[7, 9],
                   kv_last_page_len=[0, 16]),
              dict(qo_indptr=[0, 1, 2, 3, 4], kv_indptr=[0, 1, 1, 2, 3],
                   kv_indices=[11, 12, 13], kv_last_page_len=[3, 0, 5, 0])]
    q = torch.randn((4, 8, 128), generator=g).to(torch.bfloat16).to(d)
    for cluster in (0, 3):
        _, outs = run_tiles(levels, 4, q, pool, 8, 2, lse=True, cluster=cluster)
        out, l = outs[0]
        assert torch.isfinite(out).all()
        assert (out[1] == 0).all() and torch.isinf(l[1]).all() and (l[1] < 0).all()
        check(out, levels, q, pool, l)
    _, outs = run_tiles(levels, 4, q, pool, 8, 2, lse=True)
    out, l = outs[0]
    assert torch.isfinite(out).all()
    assert (out[1] == 0).all() and torch.isinf(l[1]).all() and (l[1] < 0).all()
    check(out, levels, q, pool, l)


@pytest.mark.parametrize("hq", [32, 64])
@pytest.mark.parametrize("cluster", [0, 4])
def test_large_logits_rescale_paths(hq, cluster):
    """Scores of large spread (q x 12, keys growing along the sequence) make the
    running maximum jump by more than 2^8 inside a piece, so the lazy O rescale
    in TMEM runs often; M = 64 and M = 128 rows, merged by kernel or cluster."""
    d = dev()
    g = torch.Generator().manual_seed(11)
    P = 4096
    levels = cfg2_levels(g, P, prefix=1024, max_suffix=200)
    pool = torch.randn((P, 2, 16, 8, 128), generator=g)
    ramp = torch.linspace(0.2, 3.0, P).view(P, 1, 1, 1, 1)      # later pages score higher
    pool[:, 0:1] = pool[:, 0:1] * ramp
    pool = pool.to(torch.bfloat16).to(d)
    q = (torch.randn((16, hq, 128), generator=g) * 12).to(torch.bfloat16).to(d)
    info, outs = run_tiles(levels, 16, q, pool, hq, 8, lse=True, cluster=cluster, pieces=8)
    check(outs[0][0], levels, q, pool, outs[0][1])
