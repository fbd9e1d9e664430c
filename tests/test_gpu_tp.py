"""Tensor parallelism on GPUs (NCCL, 2 ranks as child processes): the cfg1
model sharded over two GPUs selects the same beams as the unsharded model on
one GPU, in fp32 (eager step) and in bf16 (CUDA-graph step, NCCL all-reduces
captured in the graph; scores within 2e-2).  Skipped on boxes with fewer than
two GPUs.  NVLS is switched off: a rank dying while bound to a multicast
object has faulted peers on this kind of box."""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
WORLD = 2


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(dtype_name, tp_rank, world, port, q):
    import torch.distributed as dist
    from beam_engine_b200.beam import BeamSearchGenerator
    from beam_engine_b200.beam_strategy import VanillaBeamSearchStrategy
    from beam_engine_b200.configs import TINY
    from beam_engine_b200.llama import BeamLlama
    from beam_engine_b200.parallel import TensorParallel
    try:
        dtype = getattr(torch, dtype_name)
        torch.cuda.set_device(tp_rank)
        tp = None
        if world > 1:
            os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
            dist.init_process_group("nccl", rank=tp_rank, world_size=world,
                                    device_id=torch.device("cuda", tp_rank),
                                    timeout=__import__("datetime").timedelta(seconds=120))
            tp = TensorParallel()
        cfg = dict(TINY, head_dim=128, num_attention_heads=4, num_key_value_heads=2,
                   hidden_size=512)
        model = BeamLlama(cfg, None, dtype=dtype, device=torch.device("cuda", tp_rank), seed=5,
                          tp=tp)
        g = torch.Generator().manual_seed(2)
        prompts = [torch.randint(0, 1024, (40,), generator=g).tolist() for _ in range(2)]
        gen = BeamSearchGenerator(model, None, VanillaBeamSearchStrategy(), page_size=16,
                                  max_num_pages=512)
        out = gen.generate_ids(prompts, 4, max_new_tokens=12, num_return_sequences=4)
        q.put((tp_rank, [[(list(s), float(x)) for s, x in o] for o in out], gen.use_graph))
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
    except Exception:
        import traceback
        q.put((tp_rank, traceback.format_exc(), None))
        raise


@pytest.mark.parametrize("dtype_name,tol", [("float32", 1e-4), ("bfloat16", 2e-2)])
def test_tp2_matches_single_gpu(dtype_name, tol):
    if not torch.cuda.is_available() or torch.cuda.device_count() < WORLD:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    single = ctx.Process(target=_run, args=(dtype_name, 0, 1, 0, q), daemon=True)
    single.start()
    ref = q.get(timeout=300)
    single.join(timeout=60)
    assert not isinstance(ref[1], str), ref[1]
    port = _port()
    procs = [ctx.Process(target=_run, args=(dtype_name, r, WORLD, port, q), daemon=True)
             for r in range(WORLD)]
    for p in procs:
        p.start()
    try:
        res = [q.get(timeout=300) for _ in range(WORLD)]
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():      # a rank stuck in a collective: end it, do not hang the run
                p.kill()
    for rank, out, graph in res:
        assert not isinstance(out, str), out
        assert graph == (dtype_name != "float32")
        for a, b in zip(out, ref[1]):
            if dtype_name == "float32":
                assert [s for s, _ in a] == [s for s, _ in b]
            np.testing.assert_allclose([x for _, x in a], [x for _, x in b], atol=tol, rtol=0)
