"""be_rope_qkv_append (RoPE on the fused QKV rows, K and V written into their
KV pages) against a plain torch fp32 restatement of the reference's
apply_rotary_pos_emb + append_paged_kv_cache (modeling_llama.py:68-103,
428-470).  Both launch forms are covered: the CTA-per-row kernel (aligned
rows, D / 2 a multiple of the vector width) and the warp-per-head kernel
(an odd row stride).  Tolerance: one rounding of the stored dtype (bf16 2e-2,
fp32 1e-5), applied to outputs of magnitude ~1."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    return torch.device("cuda:0")


def torch_rope(x, pos, inv_freq):
    # the angle in fp32, as the reference forms it (inv_freq @ positions in fp32)
    ang = (pos.float()[:, None] * inv_freq.float()[None, :]).double()
    c, s = torch.cos(ang)[:, None, :], torch.sin(ang)[:, None, :]
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h].double(), x[..., h:].double()
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1)


@pytest.mark.parametrize("dtype,atol", [(torch.bfloat16, 2e-2), (torch.float32, 1e-5)])
@pytest.mark.parametrize("hq,hkv,D,pad", [(32, 8, 128, 0), (8, 2, 64, 0), (32, 8, 128, 1),
                                          (12, 4, 256, 0)])
@pytest.mark.parametrize("in_place", [0, 1])
def test_rope_append_matches_torch(dtype, atol, hq, hkv, D, pad, in_place):
    from beam_engine_b200 import _lib
    from beam_engine_b200.page_table import dtype_code
    d = dev()
    g = torch.Generator(device=d).manual_seed(hq + D + pad)
    n, P, ps = 37, 64, 16
    width = (hq + 2 * hkv) * D
    stride = width + pad            # pad = 1: rows off the 16-byte grid -> warp-per-head form
    buf = torch.randn((n, stride), generator=g, device=d).to(dtype)
    qkv0 = buf[:, :width].clone()
    pool = torch.zeros((P, 2, ps, hkv, D), dtype=dtype, device=d)
    slots = torch.randperm(P * ps, generator=g, device=d)[:n]
    wp = (slots // ps).int()
    wpos = (slots % ps).int()
    pos = torch.randint(0, 100000, (n,), generator=g, device=d).int()
    inv_freq = 1.0 / (500000.0 ** (torch.arange(0, D, 2, device=d).float() / D))
    st = _lib.lib().be_rope_qkv_append(buf.data_ptr(), stride, n, hq, hkv, D, pos.data_ptr(),
                                       inv_freq.data_ptr(), pool.data_ptr(), P, ps,
                                       wp.data_ptr(), wpos.data_ptr(), in_place,
                                       dtype_code(dtype), None)
    _lib.check(st, "be_rope_qkv_append")
    torch.cuda.synchronize()
    q0 = qkv0[:, :hq * D].view(n, hq, D)
    k0 = qkv0[:, hq * D:(hq + hkv) * D].view(n, hkv, D)
    v0 = qkv0[:, (hq + hkv) * D:].view(n, hkv, D)
    want_q = torch_rope(q0, pos, inv_freq)
    want_k = torch_rope(k0, pos, inv_freq)
    got = buf[:, :width]
    assert (got[:, :hq * D].view(n, hq, D).double() - want_q).abs().max().item() <= atol
    got_k_row = got[:, hq * D:(hq + hkv) * D].view(n, hkv, D)
    if in_place:
        assert (got_k_row.double() - want_k).abs().max().item() <= atol
    else:
        assert torch.equal(got_k_row, k0)
    assert torch.equal(got[:, (hq + hkv) * D:], qkv0[:, (hq + hkv) * D:])
    pk = pool[wp.long(), 0, wpos.long()]
    pv = pool[wp.long(), 1, wpos.long()]
    assert (pk.double() - want_k).abs().max().item() <= atol
    assert torch.equal(pv, v0)
    if in_place:
        assert torch.equal(pk, got_k_row)
    # slots nobody wrote stay zero
    mask = torch.ones(P * ps, dtype=torch.bool, device=d)
    mask[slots] = False
    rest = pool.permute(0, 2, 1, 3, 4).reshape(P * ps, -1)[mask]
    assert not rest.any()
