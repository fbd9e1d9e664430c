"""Tensor parallelism for the beam-decode model step (one process per GPU).

The reference runs one GPU and has no parallel runtime; its config only
carries HF's TP plan metadata (``configuration_llama.py:146-154``).  Here the
decoder is sharded the Megatron way inside :class:`beam_engine_b200.llama.BeamLlama`:
q/k/v heads and gate/up columns are split across ranks, the O and down
projections are row-parallel and followed by one all-reduce each.  The paged
KV cache is sharded by KV head (each rank's pool holds its Hkv / TP heads), so
attention itself needs no exchange; the block tables, the allocator and the
beam trie are replicated -- every rank runs the same deterministic host
scheduler on the same top-k results.

The lm_head is vocab-parallel.  ``log_softmax -> topk(k)`` over the full
vocabulary (``beam.py:266-317``) becomes: per rank the row max and sum of
exponentials of its slice (two all-reduces give the global log-sum-exp) and
its local top-k with global ids; one all-gather of the k candidates per rank
and a top-k over the gathered ``TP * k`` gives the global top-k.  The result
equals the single-GPU one up to the order of floating-point summation in the
log-sum-exp.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class TensorParallel:
    """A tensor-parallel group over ``torch.distributed`` (NCCL on GPUs, gloo on
    CPU for tests).  ``size == 1`` makes every collective a no-op."""

    def __init__(self, group=None):
        self.group = group
        if dist.is_available() and dist.is_initialized():
            self.size = dist.get_world_size(group)
            self.rank = dist.get_rank(group)
        else:
            self.size, self.rank = 1, 0

    def all_reduce(self, t: torch.Tensor, op=None):
        if self.size > 1:
            dist.all_reduce(t, op=op or dist.ReduceOp.SUM, group=self.group)
        return t

    def all_gather_cat(self, t: torch.Tensor, dim: int) -> torch.Tensor:
        """Concatenate every rank's ``t`` along ``dim`` (rank order)."""
        if self.size == 1:
            return t
        t = t.contiguous()
        out = torch.empty((self.size * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype,
                          device=t.device)
        dist.all_gather_into_tensor(out, t, group=self.group)
        return torch.cat(out.view((self.size,) + tuple(t.shape)).unbind(0), dim=dim)


class PeerAllReduce:
    """All-reduce of the row-parallel projections over peer memory, fused with
    the residual add + RMSNorm after it (``be_comm_allreduce_rmsnorm``).

    Each rank's GEMM writes its partial into its own slot of a buffer the other
    ranks map through CUDA IPC (handles exchanged once with an all-gather);
    the fused kernel signals / waits per CTA over peer flags and sums every
    rank's slot with plain loads.  Two slots, alternated call by call.  Only
    for one process per GPU on one node."""

    def __init__(self, tp: TensorParallel, slot_bytes: int, device, max_ctas: int = 1024):
        import ctypes as C
        from ._lib import check, lib
        self.tp = tp
        self.device = torch.device(device)
        self.slot_bytes = int(slot_bytes)
        h = (C.c_char * 64)()
        ptr = C.c_void_p()
        # slots 0 / 1 alternate between the all-reduces; slot 2 holds the
        # vocabulary-parallel scoring exchange
        check(lib().be_comm_create(tp.size, tp.rank, self.slot_bytes, 3, max_ctas, h,
                                   C.byref(ptr)), "be_comm_create")
        self.ptr = ptr
        handles = [None] * tp.size
        dist.all_gather_object(handles, bytes(h), group=tp.group)
        check(lib().be_comm_open(ptr, b"".join(handles)), "be_comm_open")
        dist.barrier(group=tp.group)          # every rank mapped before anyone signals
        self.next_slot = 0

    def slot_view(self, slot: int, shape, dtype) -> torch.Tensor:
        """This rank's slot as a tensor (non-owning) to be used as a GEMM output."""
        from ._lib import lib
        addr = lib().be_comm_slot(self.ptr, slot)
        n = 1
        for d in shape:
            n *= d
        nbytes = n * torch.empty(0, dtype=dtype).element_size()
        if nbytes > self.slot_bytes:
            raise ValueError("partial larger than the all-reduce slot")
        st = torch._C._construct_storage_from_data_pointer(addr, self.device, nbytes)
        stride = [1] * len(shape)
        for i in range(len(shape) - 2, -1, -1):
            stride[i] = stride[i + 1] * shape[i + 1]
        return torch.empty(0, dtype=dtype, device=self.device).set_(st, 0, tuple(shape),
                                                                   tuple(stride))

    def fits(self, rows: int, hidden: int, elt: int) -> bool:
        return rows * hidden * elt <= self.slot_bytes

    TOPK_SLOT = 2

    def topk_addresses(self, rows: int, k: int):
        """Device addresses (ids, values, row max, row sum) in this rank's scoring
        slot for ``be_logsoftmax_topk``'s slice outputs, or None if they do not fit."""
        import ctypes as C
        from ._lib import check, lib
        if k > 64 or rows * (12 * k + 8) > self.slot_bytes:
            return None
        off = (C.c_int64 * 4)()
        check(lib().be_comm_topk_layout(rows, k, off), "be_comm_topk_layout")
        base = lib().be_comm_slot(self.ptr, self.TOPK_SLOT)
        return [base + off[i] for i in range(4)]

    def topk_merge(self, rows: int, k: int, out_val: torch.Tensor, out_idx: torch.Tensor,
                   stream) -> None:
        from ._lib import check, lib
        check(lib().be_comm_topk_merge(self.ptr, self.TOPK_SLOT, rows, k, out_val.data_ptr(),
                                       out_idx.data_ptr(), stream), "be_comm_topk_merge")

    def close(self):
        """Collective teardown: unmap the peers, wait for every rank, free."""
        from ._lib import lib
        if getattr(self, "ptr", None):
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.tp.group)
            lib().be_comm_close_peers(self.ptr)
            dist.barrier(group=self.tp.group)
            lib().be_comm_destroy(self.ptr)
            self.ptr = None


def vocab_parallel_log_softmax_topk(logits: torch.Tensor, k: int, vocab_offset: int,
                                    tp: TensorParallel | None, temperature: float = 1.0,
                                    comm: "PeerAllReduce | None" = None):
    """``topk(log_softmax(logits_full / temperature), k)`` from a vocabulary
    slice per rank.

    ``logits`` is [n, V_local] float32 holding columns [vocab_offset,
    vocab_offset + V_local) of the full logits.  Returns (values [n, k] f32,
    global ids [n, k] int64), identical on every rank.  CUDA tensors go through
    the fused ``be_logsoftmax_topk`` kernel, and with a peer communicator
    (``comm``) the ranks' slices meet in one ``be_comm_topk_merge`` launch
    instead of NCCL collectives; CPU tensors (gloo tests) go through torch."""
    sharded = tp is not None and tp.size > 1
    if logits.is_cuda:
        return _fused(logits, k, vocab_offset, tp if sharded else None, temperature,
                      comm if sharded else None)
    if temperature != 1.0:
        logits = logits / temperature
    if not sharded:
        lp = torch.log_softmax(logits, dim=-1)
        return torch.topk(lp, k, dim=-1)
    m = logits.amax(dim=-1)
    tp.all_reduce(m, op=dist.ReduceOp.MAX)
    s = torch.exp(logits - m[:, None]).sum(dim=-1)
    tp.all_reduce(s)
    lse = m + torch.log(s)
    kl = min(k, logits.shape[1])
    v, i = torch.topk(logits, kl, dim=-1)
    i = i + vocab_offset
    vg = tp.all_gather_cat(v, dim=1)           # [n, TP * kl], rank-major = vocabulary order
    ig = tp.all_gather_cat(i, dim=1)
    v2, sel = torch.topk(vg, k, dim=-1)
    return v2 - lse[:, None], torch.gather(ig, 1, sel)


def _fused(logits, k, vocab_offset, tp, temperature, comm=None):
    import ctypes as C
    from ._lib import check, lib
    if logits.dtype != torch.float32 or logits.stride(1) != 1:
        raise ValueError("be_logsoftmax_topk takes row-major float32 logits")
    n, v = logits.shape
    dev = logits.device
    kl = min(k, v)
    vals = torch.empty((n, kl), dtype=torch.float32, device=dev)
    idx = torch.empty((n, kl), dtype=torch.int64, device=dev)
    st = C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    if tp is None:
        check(lib().be_logsoftmax_topk(logits.data_ptr(), logits.stride(0), n, v, float(temperature),
                                       kl, vocab_offset, 1, vals.data_ptr(), idx.data_ptr(), None,
                                       None, st), "be_logsoftmax_topk")
        return vals, idx
    addr = comm.topk_addresses(n, kl) if comm is not None and kl == k else None
    if addr is not None:
        # the slice's top-k, max and sum go straight into this rank's scoring slot
        check(lib().be_logsoftmax_topk(logits.data_ptr(), logits.stride(0), n, v,
                                       float(temperature), kl, vocab_offset, 0, addr[1], addr[0],
                                       addr[2], addr[3], st), "be_logsoftmax_topk")
        comm.topk_merge(n, k, vals, idx, st)
        return vals, idx
    m = torch.empty(n, dtype=torch.float32, device=dev)
    s = torch.empty(n, dtype=torch.float32, device=dev)
    check(lib().be_logsoftmax_topk(logits.data_ptr(), logits.stride(0), n, v, float(temperature), kl,
                                   vocab_offset, 0, vals.data_ptr(), idx.data_ptr(), m.data_ptr(),
                                   s.data_ptr(), st), "be_logsoftmax_topk")
    gm = m.clone()
    tp.all_reduce(gm, op=dist.ReduceOp.MAX)
    gs = s * torch.exp(m - gm)
    tp.all_reduce(gs)
    lse = gm + torch.log(gs)
    vg = tp.all_gather_cat(vals, dim=1)
    ig = tp.all_gather_cat(idx, dim=1)
    v2, sel = torch.topk(vg, k, dim=-1)
    return v2 - lse[:, None], torch.gather(ig, 1, sel)
