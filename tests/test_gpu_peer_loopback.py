"""The peer all-reduce kernel on one GPU through loopback mapping (every
"peer" is this process's own buffer): the fused sum + residual add + RMSNorm
against torch when the other rank's flag is preset, and the bounded flag wait
when nothing ever sets it (BE_EDEVICE_TIMEOUT after ~2 s, context still
usable)."""
import ctypes as C
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def _comm(world=2, slot_bytes=1 << 20, max_ctas=64):
    from beam_engine_b200._lib import check, lib
    h = (C.c_char * 64)()
    ptr = C.c_void_p()
    check(lib().be_comm_create(world, 0, slot_bytes, 2, max_ctas, h, C.byref(ptr)), "create")
    check(lib().be_comm_open(ptr, bytes(h) * world), "open (loopback)")
    return ptr


def _view(addr, n, dtype, dev):
    nbytes = n * torch.empty(0, dtype=dtype).element_size()
    st = torch._C._construct_storage_from_data_pointer(addr, dev, nbytes)
    return torch.empty(0, dtype=dtype, device=dev).set_(st, 0, (n,), (1,))


def _status():
    from beam_engine_b200._lib import check, lib
    s = C.c_int(-1)
    check(lib().be_device_status(C.byref(s), None), "status")
    return s.value


def test_loopback_sum_matches_torch():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from beam_engine_b200 import _lib
    from beam_engine_b200._lib import check, lib
    dev = torch.device("cuda:0")
    comm = _comm()
    try:
        n, H, eps = 7, 512, 1e-6
        g = torch.Generator().manual_seed(0)
        part = torch.randn(n, H, generator=g).to(dev, torch.bfloat16)
        x = torch.randn(n, H, generator=g).to(dev, torch.bfloat16)
        w = torch.randn(H, generator=g).to(dev, torch.bfloat16)
        _view(lib().be_comm_slot(comm, 0), n * H, torch.bfloat16, dev).copy_(part.reshape(-1))
        flags = _view(lib().be_comm_flags(comm), 64 * 8, torch.int32, dev)
        flags.view(64, 8)[:n, 1] = 1          # "rank 1" has signalled call 1 for every CTA
        s = part.float() + part.float()
        xr = (x.float() + s.to(torch.bfloat16).float()).to(torch.bfloat16)
        hr = w.float() * (xr.float() * torch.rsqrt(xr.float().pow(2).mean(-1, keepdim=True) + eps)
                          ).to(torch.bfloat16).float()
        h = torch.empty_like(x)
        torch.cuda.synchronize()
        check(lib().be_comm_allreduce_rmsnorm(comm, 0, x.data_ptr(), w.data_ptr(), h.data_ptr(), n,
                                              H, eps, _lib.BE_BF16, None), "allreduce")
        torch.cuda.synchronize()
        assert _status() == 0
        assert torch.equal(x, xr)
        assert (h.float() - hr).abs().max().item() < 5e-2
        assert flags.view(64, 8)[:n, 0].tolist() == [1] * n    # this rank signalled call 1
    finally:
        lib().be_comm_destroy(comm)


def test_loopback_wait_times_out_with_a_status():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    from beam_engine_b200 import _lib
    from beam_engine_b200._lib import check, lib
    dev = torch.device("cuda:0")
    comm = _comm()
    try:
        n, H = 3, 256
        x = torch.zeros(n, H, dtype=torch.bfloat16, device=dev)
        w = torch.ones(H, dtype=torch.bfloat16, device=dev)
        h = torch.empty_like(x)
        torch.cuda.synchronize()
        t0 = time.time()
        check(lib().be_comm_allreduce_rmsnorm(comm, 0, x.data_ptr(), w.data_ptr(), h.data_ptr(), n,
                                              H, 1e-6, _lib.BE_BF16, None), "allreduce")
        torch.cuda.synchronize()               # nothing sets rank 1's flag: bounded wait
        assert time.time() - t0 < 30
        assert _status() == _lib.BE_EDEVICE_TIMEOUT
        check(lib().be_device_status_clear(None), "clear")
        assert _status() == 0
        torch.ones(4, device=dev).sum().item()  # the context still works
    finally:
        lib().be_comm_destroy(comm)
