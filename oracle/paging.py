"""Oracle: FIFO page allocator and per-layer paged KV pools (test infrastructure).

Restates ``src/beam_engine/page_table.py`` of the reference:
  * pool layout ``[pages, 2, page_size, kv_heads, head_dim]`` per layer, K at
    plane 0, V at plane 1 (page_table.py:62-72);
  * allocation pops the FRONT of the free list, freeing appends to the BACK
    (page_table.py:77-94, 110-124); freeing a page that is not allocated is a
    warning and a no-op;
  * ``copy_block`` allocates a fresh page and copies the first ``length``
    tokens of K and V for every layer (page_table.py:96-106);
  * ``write_block`` writes ``n`` tokens starting at ``index``
    (page_table.py:126-165);
  * the decode append restates ``flashinfer.page.append_paged_kv_cache`` as the
    reference calls it (page_table.py:167-209): with ``kv_indptr = arange`` and
    ``batch_indices = arange`` entry ``i`` lands in page ``kv_indices[i]`` at
    in-page slot ``positions[i]``.
"""
from __future__ import annotations

from collections import deque
import numpy as np


class OraclePageTable:
    def __init__(self, layer_num, page_size, max_num_pages, head_num, head_dim,
                 dtype=np.float32, storage=True):
        self.layer_num = layer_num
        self.page_size = page_size
        self.max_num_pages = max_num_pages
        self.head_num = head_num
        self.head_dim = head_dim
        self.free_pages = deque(range(max_num_pages))
        self.allocated = set()
        self.warnings = 0
        self.kv = None
        if storage:
            self.kv = [np.zeros((max_num_pages, 2, page_size, head_num, head_dim), dtype)
                       for _ in range(layer_num)]

    # page_table.py:77-94
    def allocate_block(self) -> int:
        if not self.free_pages:
            raise MemoryError("No free pages available")
        p = self.free_pages.popleft()
        self.allocated.add(p)
        return p

    # page_table.py:110-124
    def free_block(self, p: int) -> None:
        if p not in self.allocated:
            self.warnings += 1
            return
        self.allocated.discard(p)
        self.free_pages.append(p)

    # page_table.py:96-106
    def copy_block(self, p: int, length: int) -> int:
        if length > self.page_size:
            raise ValueError("length cannot be larger than page size")
        if p > self.max_num_pages:
            raise ValueError("page idx out of bound")
        q = self.allocate_block()
        if self.kv is not None:
            for layer in self.kv:
                layer[q, :, :length] = layer[p, :, :length]
        return q

    # page_table.py:126-165
    def write_block(self, layer, p, key, value, index):
        n = key.shape[0]
        if n + index > self.page_size:
            raise ValueError("does not fit in page")
        if p not in self.allocated:
            raise ValueError(f"Page {p} is not allocated")
        self.kv[layer][p, 0, index:index + n] = key
        self.kv[layer][p, 1, index:index + n] = value

    # page_table.py:199-209 (flashinfer.page.append_paged_kv_cache semantics)
    def append(self, layer, keys, values, page_ids, positions):
        for i in range(len(page_ids)):
            self.kv[layer][int(page_ids[i]), 0, int(positions[i])] = keys[i]
            self.kv[layer][int(page_ids[i]), 1, int(positions[i])] = values[i]


def append_paged_kv(pool, keys, values, page_ids, positions):
    """Stand-alone form of the decode append on one layer's pool array."""
    pool = pool.copy()
    for i in range(len(page_ids)):
        pool[int(page_ids[i]), 0, int(positions[i])] = keys[i]
        pool[int(page_ids[i]), 1, int(positions[i])] = values[i]
    return pool


def fork_tail_copy(pools, src, dst, lens):
    """Copy-on-write tail copies for a batch of forks, all layers.

    Each triple (src[i], dst[i], lens[i]) is one ``copy_block`` data movement
    (page_table.py:102-104): tokens ``[0, len)`` of K and V.  Copies are applied
    in order, so a later copy reads what an earlier one wrote.
    """
    out = [p.copy() for p in pools]
    for s, d, n in zip(src, dst, lens):
        for layer in out:
            layer[int(d), :, :int(n)] = layer[int(s), :, :int(n)]
    return out
