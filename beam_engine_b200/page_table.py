"""PageTable: the paged KV-cache manager, same interface as the reference's
``src/beam_engine/page_table.py`` (``PageTable`` :18-241).

* The FIFO free list and allocation bookkeeping live in the native host page
  manager (``be_trie``), shared with :class:`BeamState`'s trie.
* Storage is ONE tensor ``[layers, pages, 2, page_size, kv_heads, head_dim]``;
  ``kv_cache_at_layer[l]`` are views of it (the reference's per-layer list), so
  kernels can address every layer in one launch.
* ``copy_block`` / ``copy_blocks`` / ``write_block`` / ``write_blocks_vectorized``
  run the CUDA kernels of ``libbeam_b200.so``; ``get_k_buffer``/``get_v_buffer``
  return zero-copy views ``[pages, page_size, kv_heads, head_dim]`` (the
  reference reshapes, i.e. copies, both pools every layer and step).
Allocation works on any device (it is host bookkeeping); data movement needs
CUDA tensors and raises otherwise.
"""
from __future__ import annotations

import ctypes as C
import logging
from typing import List, Optional

import numpy as np
import torch

from . import _lib
from ._lib import check, lib

logger = logging.getLogger(__name__)

_DT = {torch.float32: _lib.BE_F32, torch.float16: _lib.BE_F16, torch.bfloat16: _lib.BE_BF16}


def dtype_code(dt):
    if dt not in _DT:
        raise ValueError(f"unsupported KV dtype {dt}")
    return _DT[dt]


def stream_ptr(device):
    return C.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def require_cuda(*tensors):
    for t in tensors:
        if not t.is_cuda:
            raise RuntimeError("beam_engine_b200 kernels need CUDA tensors (no CPU fallback)")


class PageTable:
    def __init__(self, layer_num: int, page_size: int = 8, max_num_pages: int = 1024,
                 head_num: int = 32, head_dim: int = 128, v_head_dim: Optional[int] = None,
                 device: torch.device = None, store_dtype: torch.dtype = torch.float16):
        if v_head_dim is not None and v_head_dim != head_dim:
            raise ValueError("v_head_dim different from head_dim is not supported")
        self.layer_num = layer_num
        self.page_size = page_size
        self.max_num_pages = max_num_pages
        self.head_num = head_num
        self.head_dim = head_dim
        self.v_head_dim = head_dim
        self.device = torch.device(device) if device is not None else torch.device("cuda")
        self.store_dtype = store_dtype
        self._trie = lib().be_trie_create(page_size, max_num_pages)
        if not self._trie:
            check(_lib.BE_EINVAL, "be_trie_create")
        self.kv_cache = torch.zeros((layer_num, max_num_pages, 2, page_size, head_num, head_dim),
                                    dtype=store_dtype, device=self.device)
        self.kv_cache_at_layer: List[torch.Tensor] = [self.kv_cache[i] for i in range(layer_num)]
        self._pages_buf = np.zeros(0, np.int32)
        logger.info("Initialized PageTable: %d layers, %d pages of size %d", layer_num,
                    max_num_pages, page_size)

    def __del__(self):
        t = getattr(self, "_trie", None)
        if t:
            try:
                lib().be_trie_destroy(t)
            except Exception:   # interpreter shutdown: the library may already be gone
                pass
            self._trie = None

    # -- allocator (page_table.py:77-124) ---------------------------------
    @property
    def free_pages(self) -> List[int]:
        n = lib().be_num_free_pages(self._trie)
        buf = np.zeros(max(n, 1), np.int32)
        lib().be_free_list(self._trie, _lib.ptr32(buf), n)
        return buf[:n].tolist()

    @property
    def allocated_pages(self) -> set:
        free = set(self.free_pages)
        return {p for p in range(self.max_num_pages) if p not in free}

    def allocate_block(self) -> int:
        out = C.c_int32()
        rc = lib().be_alloc_page(self._trie, C.byref(out))
        if rc == _lib.BE_ENOMEM:
            raise MemoryError("No free pages available")
        check(rc, "allocate_block")
        return out.value

    def free_block(self, page_idx: int):
        rc = lib().be_free_page(self._trie, int(page_idx))
        if rc == _lib.BE_ENOT_ALLOCATED:
            logger.warning("Page %d is not allocated", page_idx)
            return
        check(rc, "free_block")

    def is_allocated(self, page_idx: int) -> bool:
        return bool(lib().be_is_allocated(self._trie, int(page_idx)))

    # -- data movement ------------------------------------------------------
    def _layer_stride(self):
        return self.kv_cache.stride(0)

    def copy_blocks(self, src, dst, lens):
        """Batched copy-on-write tail copies (tokens [0, len) of K and V, every layer)
        in ONE kernel launch.  src/dst/lens: int sequences or int32 CUDA tensors."""
        if len(src) == 0:
            return
        require_cuda(self.kv_cache)
        dev = self.kv_cache.device

        def as_dev(x):
            if isinstance(x, torch.Tensor) and x.is_cuda and x.dtype == torch.int32:
                return x
            return torch.as_tensor(np.asarray(x, np.int32)).to(dev, non_blocking=True)
        s, d, n = as_dev(src), as_dev(dst), as_dev(lens)
        rc = lib().be_fork_tail_copy(self.kv_cache.data_ptr(), self._layer_stride(), self.layer_num,
                                     self.max_num_pages, self.page_size, self.head_num,
                                     self.head_dim, dtype_code(self.store_dtype), s.data_ptr(),
                                     d.data_ptr(), n.data_ptr(), len(src), stream_ptr(dev))
        check(rc, "copy_blocks")

    def copy_block(self, page_idx: int, length: int) -> int:
        """page_table.py:96-106: new page holding the first `length` tokens of `page_idx`."""
        if length > self.page_size:
            raise ValueError("length cannot be larger than page size")
        if page_idx > self.max_num_pages:
            raise ValueError("page idx out of bound")
        new_page = self.allocate_block()
        self.copy_blocks([page_idx], [new_page], [length])
        return new_page

    def write_block(self, layer: int, page_idx: int, key: torch.Tensor, value: torch.Tensor,
                    index: int):
        """page_table.py:126-165: write key/value [n, H, D] at slots index..index+n-1."""
        assert key.shape == value.shape
        assert key.shape[0] + index <= self.page_size, \
            f"Cannot fit {key.shape[0]} tokens at index {index} in page size {self.page_size}"
        if layer >= self.layer_num:
            raise ValueError(f"Layer {layer} out of range (max: {self.layer_num - 1})")
        if not self.is_allocated(page_idx):
            raise ValueError(f"Page {page_idx} is not allocated")
        if index > self.page_size:
            raise ValueError(f"Index {index} exceeds page size {self.page_size}")
        n = key.shape[0]
        if n == 0:
            return
        dev = self.kv_cache.device
        pos = torch.arange(index, index + n, dtype=torch.int32, device=dev)
        zeros = torch.zeros(n, dtype=torch.int32, device=dev)
        pages = torch.tensor([page_idx], dtype=torch.int32, device=dev)
        indptr = torch.tensor([0, 1], dtype=torch.int32, device=dev)
        self._append(layer, key, value, zeros, pos, pages, indptr)

    def write_blocks_vectorized(self, layer: int, page_indices: torch.Tensor, keys: torch.Tensor,
                                values: torch.Tensor, indices: torch.Tensor,
                                batch_indices: torch.Tensor, kv_indptr: torch.Tensor):
        """page_table.py:167-209: one append kernel for all candidates."""
        self._append(layer, keys, values, batch_indices, indices, page_indices, kv_indptr)

    def _append(self, layer, keys, values, batch_indices, positions, kv_indices, kv_indptr,
                num_layers=1):
        require_cuda(keys, values, self.kv_cache)
        if keys.dtype != self.store_dtype or values.dtype != self.store_dtype:
            keys = keys.to(self.store_dtype)
            values = values.to(self.store_dtype)
        if keys.stride(-1) != 1 or keys.stride(-2) != self.head_dim:
            keys = keys.contiguous()
        if values.stride(-1) != 1 or values.stride(-2) != self.head_dim:
            values = values.contiguous()
        if keys.stride(0) != values.stride(0):
            keys, values = keys.contiguous(), values.contiguous()
        ints = [t if t.dtype == torch.int32 else t.to(torch.int32)
                for t in (batch_indices, positions, kv_indices, kv_indptr)]
        rc = lib().be_append_paged_kv(keys.data_ptr(), values.data_ptr(), keys.stride(0), 0,
                                      ints[0].data_ptr(), ints[1].data_ptr(), ints[2].data_ptr(),
                                      ints[3].data_ptr(), keys.shape[0],
                                      self.kv_cache_at_layer[layer].data_ptr(), self._layer_stride(),
                                      num_layers, self.max_num_pages, self.page_size, self.head_num,
                                      self.head_dim, dtype_code(self.store_dtype),
                                      stream_ptr(self.kv_cache.device))
        check(rc, "append_paged_kv")

    # -- flat slot views (page_table.py:211-241), zero copy -----------------
    def get_k_buffer(self, layer: int) -> torch.Tensor:
        return self.kv_cache_at_layer[layer][:, 0]

    def get_v_buffer(self, layer: int) -> torch.Tensor:
        return self.kv_cache_at_layer[layer][:, 1]
