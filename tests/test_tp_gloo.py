"""Tensor parallelism on CPU ranks (gloo, world sizes 2 and 4): the sharding of
:class:`BeamLlama` and the vocab-parallel log-softmax / top-k reproduce the
unsharded model.  The decoder layer is run here in plain torch (fp32, causal
dense attention with RoPE) on each rank's weight shards, with the same
all-reduces the GPU forward issues; the GPU kernels themselves are covered by
the -m gpu tests."""
import os
import socket

import torch
import torch.distributed as dist
import pytest
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rope(x, pos, theta):
    from beam_engine_b200.llama import inv_freq_table
    d = x.shape[-1]
    f = torch.outer(pos.float(), inv_freq_table(d, theta, "cpu"))
    cos, sin = torch.cat([f.cos(), f.cos()], -1), torch.cat([f.sin(), f.sin()], -1)
    x1, x2 = x[..., : d // 2], x[..., d // 2:]
    rot = torch.cat([-x2, x1], -1)
    return x * cos[:, None, :] + rot * sin[:, None, :]


def _rms(x, w, eps):
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def _forward(m, ids, tp):
    """Plain-torch decoder forward on the (possibly sharded) weights of m."""
    c = m.config
    D, Hq, Hkv, F = m.D, m.Hq, m.Hkv, m.F
    n = ids.shape[0]
    pos = torch.arange(n)
    x = m.embed[ids].float()
    for i in range(m.L):
        h = _rms(x, m.n_in[i].float(), m.eps)
        qkv = h @ m.w_qkv[i].float().t()
        q = qkv[:, :Hq * D].view(n, Hq, D)
        k = qkv[:, Hq * D:(Hq + Hkv) * D].view(n, Hkv, D)
        v = qkv[:, (Hq + Hkv) * D:].view(n, Hkv, D)
        q, k = _rope(q, pos, c["rope_theta"]), _rope(k, pos, c["rope_theta"])
        g = Hq // Hkv
        k, v = k.repeat_interleave(g, 1), v.repeat_interleave(g, 1)
        s = torch.einsum("ihd,jhd->hij", q, k) * D ** -0.5
        s = s.masked_fill(torch.triu(torch.ones(n, n, dtype=torch.bool), 1), float("-inf"))
        att = torch.einsum("hij,jhd->ihd", torch.softmax(s, -1), v).reshape(n, Hq * D)
        delta = att @ m.w_o[i].float().t()
        if tp is not None:
            tp.all_reduce(delta)
        x = x + delta
        h = _rms(x, m.n_post[i].float(), m.eps)
        gu = h @ m.w_gu[i].float().t()
        act = torch.nn.functional.silu(gu[:, :F]) * gu[:, F:]
        delta = act @ m.w_down[i].float().t()
        if tp is not None:
            tp.all_reduce(delta)
        x = x + delta
    h = _rms(x, m.norm.float(), m.eps)
    return h @ m.lm_head.float().t()


def _worker(rank, port, q, WORLD):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        from beam_engine_b200.configs import TINY as T0
        # 4 ranks: one KV head and two query heads per rank (the 8B shape at TP = 8 has
        # one KV head per rank too)
        TINY = T0 if WORLD == 2 else dict(T0, num_attention_heads=8, num_key_value_heads=4,
                                          head_dim=32)
        from beam_engine_b200.llama import BeamLlama
        from beam_engine_b200.parallel import TensorParallel, vocab_parallel_log_softmax_topk
        torch.manual_seed(0)
        tp = TensorParallel()
        assert (tp.size, tp.rank) == (WORLD, rank)
        full = BeamLlama(TINY, None, dtype=torch.float32, device="cpu", seed=7)
        part = BeamLlama(TINY, None, dtype=torch.float32, device="cpu", seed=7, tp=tp)
        assert part.Hq * WORLD == full.Hq and part.Hkv * WORLD == full.Hkv
        assert part.F * WORLD == full.F
        ids = torch.randint(0, TINY["vocab_size"], (12,), generator=torch.Generator().manual_seed(3))
        ref_logits = _forward(full, ids, None)
        loc_logits = _forward(part, ids, tp)
        # the vocabulary slices, gathered, are the full logits
        got = tp.all_gather_cat(loc_logits.contiguous(), dim=1)
        err = (got - ref_logits).abs().max().item()
        # the distributed log-softmax / top-k equals the single-rank one
        k = 8
        rv, ri = vocab_parallel_log_softmax_topk(ref_logits, k, 0, None)
        tv, ti = vocab_parallel_log_softmax_topk(loc_logits, k, part.v0, tp)
        q.put((rank, err, (tv - rv).abs().max().item(), bool(torch.equal(ti, ri))))
    except Exception:   # report instead of leaving the parent waiting
        import traceback
        q.put((rank, traceback.format_exc(), None, None))
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("WORLD", [2, 4])
def test_tensor_parallel_matches_unsharded_gloo(WORLD):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q, WORLD)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(WORLD)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, err, verr, same_ids in res:
        assert not isinstance(err, str), err
        assert err < 1e-4, (rank, err)
        assert verr < 1e-5, (rank, verr)
        assert same_ids, rank


def test_vocab_parallel_topk_uneven_slices():
    """Single process, three simulated ranks with uneven vocabulary slices: the
    merge of per-slice top-k with the global log-sum-exp is the full top-k."""
    from beam_engine_b200.parallel import vocab_parallel_log_softmax_topk

    g = torch.Generator().manual_seed(1)
    logits = torch.randn((5, 1000), generator=g) * 4
    ref_v, ref_i = torch.topk(torch.log_softmax(logits, -1), 12, -1)
    cuts = [0, 301, 650, 1000]
    m = logits.amax(-1)
    lse = m + torch.log(torch.exp(logits - m[:, None]).sum(-1))
    vs, is_ = [], []
    for a, b in zip(cuts[:-1], cuts[1:]):
        v, i = torch.topk(logits[:, a:b], 12, -1)
        vs.append(v)
        is_.append(i + a)
    v2, sel = torch.topk(torch.cat(vs, 1), 12, -1)
    assert torch.allclose(v2 - lse[:, None], ref_v, atol=1e-5)
    assert torch.equal(torch.gather(torch.cat(is_, 1), 1, sel), ref_i)
    # and the size-1 path is the plain one
    v1, i1 = vocab_parallel_log_softmax_topk(logits, 12, 0, None)
    assert torch.equal(i1, ref_i) and torch.allclose(v1, ref_v)


def _failing_worker(rank, port, q):
    """Rank 1 dies before the step's first collective; rank 0 must get an error
    from the collective within the process group's timeout, not hang."""
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2,
                            timeout=datetime.timedelta(seconds=4))
    from beam_engine_b200.parallel import TensorParallel, vocab_parallel_log_softmax_topk
    tp = TensorParallel()
    tp.all_reduce(torch.ones(8))         # one good step: the ranks' connections are up
    def say(msg):                        # flush the queue before the hard exit
        q.put((rank, msg))
        q.close()
        q.join_thread()

    if rank == 1:
        say("left")
        os._exit(0)                      # a rank that disappears between steps
    import time
    t0 = time.time()
    try:
        logits = torch.randn(4, 100)
        vocab_parallel_log_softmax_topk(logits, 4, 0, tp)
        say("no error")
    except Exception as e:   # the collective reports the dead peer
        say(f"error after {time.time() - t0:.1f}s: {type(e).__name__}")
    os._exit(0)


def test_rank_failure_surfaces_as_an_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert res[1] == "left"
    assert res[0].startswith("error after"), res[0]
    assert float(res[0].split()[2].rstrip("s:")) < 60
