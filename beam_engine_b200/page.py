"""``append_paged_kv_cache`` with FlashInfer's signature, on the native kernel.

Replaces ``flashinfer.page.append_paged_kv_cache`` as the reference calls it
from ``PageTable.write_blocks_vectorized`` (src/beam_engine/page_table.py:199-209):
entry ``i`` lands in page ``kv_indices[kv_indptr[batch_indices[i]] +
positions[i] // page_size]`` at slot ``positions[i] % page_size``
(``kv_last_page_len`` is accepted and unused, as in FlashInfer's append).
"""
from __future__ import annotations

import torch

from ._lib import check, lib
from .page_table import dtype_code, require_cuda, stream_ptr


def append_paged_kv_cache(append_key: torch.Tensor, append_value: torch.Tensor,
                          batch_indices: torch.Tensor, positions: torch.Tensor,
                          paged_kv_cache: torch.Tensor, kv_indices: torch.Tensor,
                          kv_indptr: torch.Tensor, kv_last_page_len: torch.Tensor = None,
                          kv_layout: str = "NHD") -> None:
    if kv_layout != "NHD":
        raise ValueError("only the NHD layout is supported")
    if paged_kv_cache.dim() != 5 or paged_kv_cache.shape[1] != 2:
        raise ValueError("paged_kv_cache must be [pages, 2, page_size, kv_heads, head_dim]")
    require_cuda(append_key, append_value, paged_kv_cache, batch_indices, positions, kv_indices,
                 kv_indptr)
    P, _, ps, H, D = paged_kv_cache.shape
    if not paged_kv_cache.is_contiguous():
        raise ValueError("paged_kv_cache must be contiguous")
    k = append_key.to(paged_kv_cache.dtype)
    v = append_value.to(paged_kv_cache.dtype)
    if k.stride(-1) != 1 or k.stride(-2) != D:
        k = k.contiguous()
    if v.stride(-1) != 1 or v.stride(-2) != D or v.stride(0) != k.stride(0):
        k, v = k.contiguous(), v.contiguous()
    ints = [t.to(torch.int32) for t in (batch_indices, positions, kv_indices, kv_indptr)]
    rc = lib().be_append_paged_kv(k.data_ptr(), v.data_ptr(), k.stride(0), 0, ints[0].data_ptr(),
                                  ints[1].data_ptr(), ints[2].data_ptr(), ints[3].data_ptr(),
                                  k.shape[0], paged_kv_cache.data_ptr(), 0, 1, P, ps, H, D,
                                  dtype_code(paged_kv_cache.dtype),
                                  stream_ptr(paged_kv_cache.device))
    check(rc, "append_paged_kv_cache")
