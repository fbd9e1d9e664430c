"""Cascade and paged-prefill attention wrappers with FlashInfer's plan/run API.

Drop-in for the two wrappers the reference drives:
  * ``MultiLevelCascadeAttentionWrapper`` (modeling_llama.py:733-755 plan,
    :362 run): level ``l`` group ``g`` attends queries ``qo_indptr[l][g]..[g+1]``
    to its pages; only the last level is causal (FlashInfer's cascade plan sets
    ``causal`` on the last level only); levels merge by log-sum-exp.
  * ``BatchPrefillWithPagedKVCacheWrapper`` (modeling_llama.py:775-798, :266):
    causal prompt attention over each request's pages.
``plan`` runs the native host planner (``be_cascade_plan``) and copies the
work list into the caller's workspace buffer with one async H2D copy;
``run`` launches the attention kernel (+ the LSE merge when a query has several
partial states) of ``libbeam_b200.so`` on the current stream.  The workspace
holds the plan followed by the fp32 partial (o, lse) rows.

Decode plans (no causal group of more than one query) with head_dim 128 and
page size 16 run as beam-tile plans (``be_tile_plan`` / ``be_attn_tiles_run``:
one launch, each page read once per KV head, partial rows merged inside the
kernel); ``BE_ATTN_TILES=0`` keeps the work-item kernels.
"""
from __future__ import annotations

import ctypes as C
import os
from typing import List, Optional

import numpy as np
import torch

from . import _lib
from ._lib import AttnPlanInfo, TilePlanInfo, check, lib
from .page_table import dtype_code, require_cuda, stream_ptr


def _i32(x):
    if isinstance(x, torch.Tensor):
        return np.ascontiguousarray(x.detach().cpu().numpy().astype(np.int32, copy=False))
    return np.ascontiguousarray(np.asarray(x, dtype=np.int32))


def tiles_enabled():
    return os.environ.get("BE_ATTN_TILES", "1") != "0"


def tiles_eligible(head_dim, page_size, num_qo_heads, num_kv_heads):
    """Shapes the beam-tile kernel serves (the pool dtype is checked at run)."""
    return (tiles_enabled() and head_dim == 128 and page_size == 16 and num_kv_heads > 0
            and num_qo_heads % num_kv_heads == 0 and num_qo_heads // num_kv_heads <= 128)


def tile_rows_for(rows):
    """Tile height (tcgen05 M) for tiles of up to `rows` query-head rows."""
    return 64 if rows <= 64 else 128


def target_pieces(num_sms, num_kv_heads):
    """About two CTAs per SM over all KV heads."""
    return max(1, -(-2 * num_sms // max(1, num_kv_heads)))


def _level_arrays(levels):
    L = len(levels)
    keys = ("qo_indptr", "kv_indptr", "kv_indices", "kv_last_page_len")
    arrs = [[_i32(lv[k] if isinstance(lv, dict) else lv[i]) for lv in levels]
            for i, k in enumerate(keys)]
    ng = np.asarray([len(a) - 1 for a in arrs[0]], np.int32)
    ptrs = [(_lib.P32 * max(L, 1))(*[_lib.ptr32(a) for a in group]) for group in arrs]
    return L, arrs, ng, ptrs


def level0_rows(levels, group_size):
    """Largest level-0 group (query-head rows): the tile height a plan needs."""
    if not levels:
        return group_size
    qo = _i32(levels[0]["qo_indptr"] if isinstance(levels[0], dict) else levels[0][0])
    return int(np.max(np.diff(qo))) * group_size if len(qo) > 1 else group_size


def tile_plan_host(levels, num_queries, page_size, num_qo_heads, num_kv_heads, causal=True,
                   tile_rows=None, num_sms=148, pieces=None, cluster=-1):
    """be_tile_plan on python/numpy level arrays: (info, plan ints), or None when the
    levels are not a decode shape (BE_ENOTSUP).  cluster -1 lets the planner choose."""
    L, arrs, ng, ptrs = _level_arrays(levels)
    g = num_qo_heads // num_kv_heads
    rows = tile_rows or tile_rows_for(level0_rows(levels, g))
    tp = pieces or target_pieces(num_sms, num_kv_heads)
    info = TilePlanInfo()

    def call(buf, cap):
        return lib().be_tile_plan(L, *ptrs, _lib.ptr32(ng), num_queries, page_size, num_qo_heads,
                                  num_kv_heads, 1 if causal else 0, rows, tp, cluster, buf, cap,
                                  C.byref(info))
    buf = np.empty(4096, np.int32)
    rc = call(_lib.ptr32(buf), buf.size)
    if rc == _lib.BE_ECAPACITY:
        buf = np.empty(info.total_ints + 64, np.int32)
        rc = call(_lib.ptr32(buf), buf.size)
    if rc == _lib.BE_ENOTSUP:
        return None
    check(rc, "be_tile_plan")
    return info, buf[:info.total_ints]


class _Plan:
    """Host staging + device placement of one attention plan."""

    def __init__(self, workspace: torch.Tensor):
        if workspace is None or workspace.dtype != torch.uint8 or not workspace.is_cuda:
            raise ValueError("workspace must be a CUDA uint8 tensor")
        self.ws = workspace
        self.host = torch.empty(0, dtype=torch.int32).pin_memory()
        self.info = AttnPlanInfo()
        self.tinfo = None             # TilePlanInfo of a placed beam-tile plan, else None
        self.copied = None
        self.device = workspace.device
        self.num_sms = torch.cuda.get_device_properties(self.device).multi_processor_count

    def build(self, fn):
        """fn(host_ptr, capacity, info_ref) -> status; grows the pinned buffer on
        BE_ECAPACITY."""
        if self.copied is not None:
            self.copied.synchronize()          # previous H2D still reading the buffer
        cap = self.host.numel()
        rc = fn(self.host.data_ptr(), cap, C.byref(self.info))
        if rc == _lib.BE_ECAPACITY:
            self.host = torch.empty(int(self.info.total_ints * 1.25) + 1024,
                                    dtype=torch.int32).pin_memory()
            rc = fn(self.host.data_ptr(), self.host.numel(), C.byref(self.info))
        check(rc, "attention plan")

    def place(self, num_qo_heads, head_dim):
        """Copy the plan to the front of the workspace; carve mid_o / mid_lse."""
        n = self.info.total_ints
        plan_bytes = (n * 4 + 255) // 256 * 256
        parts = self.info.n_parts
        mo = parts * num_qo_heads * head_dim * 4
        ml = parts * num_qo_heads * 4
        need = plan_bytes + (mo + 255) // 256 * 256 + ml
        if need > self.ws.numel():
            raise ValueError(f"workspace too small: plan needs {need} bytes, "
                             f"buffer has {self.ws.numel()}")
        base = self.ws.data_ptr()
        self.plan_dev = base
        self.mid_o = base + plan_bytes
        self.mid_lse = base + plan_bytes + (mo + 255) // 256 * 256
        dst = self.ws[: n * 4].view(torch.int32)
        stream = torch.cuda.current_stream(self.device)
        dst.copy_(self.host[:n], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(stream)
        self.copied = ev

    # -- beam-tile plans ----------------------------------------------------
    def build_tiles(self, fn):
        """fn(host_ptr, capacity, tile_info_ref) -> status.  False on BE_ENOTSUP."""
        if self.copied is not None:
            self.copied.synchronize()
        self.tinfo = TilePlanInfo()
        rc = fn(self.host.data_ptr(), self.host.numel(), C.byref(self.tinfo))
        if rc == _lib.BE_ECAPACITY:
            self.host = torch.empty(int(self.tinfo.total_ints * 1.25) + 1024,
                                    dtype=torch.int32).pin_memory()
            rc = fn(self.host.data_ptr(), self.host.numel(), C.byref(self.tinfo))
        if rc == _lib.BE_ENOTSUP:
            self.tinfo = None
            return False
        check(rc, "tile plan")
        return True

    def place_tiles(self, num_kv_heads, head_dim):
        """Copy the tile plan to the workspace; carve the partial rows."""
        ti = self.tinfo
        n = ti.total_ints
        plan_bytes = (n * 4 + 255) // 256 * 256
        slots = ti.n_part_pieces * num_kv_heads * ti.tile_rows
        mo = slots * head_dim * 2          # partial rows in the pool's 2-byte type
        need = plan_bytes + (mo + 255) // 256 * 256 + slots * 4
        if need > self.ws.numel():
            raise ValueError(f"workspace too small: tile plan needs {need} bytes, "
                             f"buffer has {self.ws.numel()}")
        base = self.ws.data_ptr()
        self.plan_dev = base
        self.mid_o = base + plan_bytes
        self.mid_lse = base + plan_bytes + (mo + 255) // 256 * 256
        dst = self.ws[: n * 4].view(torch.int32)
        stream = torch.cuda.current_stream(self.device)
        dst.copy_(self.host[:n], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(stream)
        self.copied = ev

    def run_tiles(self, q, kv, num_qo_heads, num_kv_heads, head_dim, sm_scale, out, lse=None):
        require_cuda(q, kv, out)
        if q.stride(-1) != 1 or q.stride(-2) != head_dim:
            q = q.contiguous()
        ti = self.tinfo
        rc = lib().be_attn_tiles_run(
            C.c_void_p(self.plan_dev), ti.n_pieces, ti.n_tiles, ti.n_part_pieces, ti.tile_rows,
            ti.page_size, q.data_ptr(), q.stride(0), kv.data_ptr(), kv.shape[0], num_qo_heads,
            num_kv_heads, head_dim, dtype_code(kv.dtype), float(sm_scale), out.data_ptr(),
            out.stride(0), lse.data_ptr() if lse is not None else None, C.c_void_p(self.mid_o),
            C.c_void_p(self.mid_lse), ti.cluster, 0, stream_ptr(q.device))
        check(rc, "be_attn_tiles_run")

    def run(self, q, kv, num_qo_heads, num_kv_heads, head_dim, sm_scale, out, lse=None,
            kv_list=None):
        require_cuda(q, kv, out)
        if q.stride(-1) != 1 or q.stride(-2) != head_dim:
            q = q.contiguous()
        rc = lib().be_attn_run(
            C.c_void_p(self.plan_dev), C.byref(self.info), q.data_ptr(), q.stride(0),
            kv.data_ptr(), kv.shape[0], num_qo_heads, num_kv_heads, head_dim,
            dtype_code(kv.dtype), float(sm_scale), out.data_ptr(), out.stride(0),
            lse.data_ptr() if lse is not None else None, C.c_void_p(self.mid_o),
            C.c_void_p(self.mid_lse), kv_list.data_ptr() if kv_list is not None else None,
            stream_ptr(q.device))
        check(rc, "be_attn_run")


_plan_cap = 4096     # int32 capacity of the next host plan buffer (grows on demand)


def cascade_plan_host(levels, num_queries, page_size, num_qo_heads, num_kv_heads, causal=True,
                      split_tokens=0, num_sms=148, plan_buf=None):
    """Host planner call on python/numpy level arrays; returns (info, plan ints)."""
    L = len(levels)
    keys = ("qo_indptr", "kv_indptr", "kv_indices", "kv_last_page_len")
    arrs = [[_i32(lv[k] if isinstance(lv, dict) else lv[i]) for lv in levels]
            for i, k in enumerate(keys)]
    ng = np.asarray([len(a) - 1 for a in arrs[0]], np.int32)
    ptrs = [(_lib.P32 * max(L, 1))(*[_lib.ptr32(a) for a in group]) for group in arrs]
    info = AttnPlanInfo()

    def call(buf, cap):
        return lib().be_cascade_plan(L, *ptrs, _lib.ptr32(ng), num_queries, page_size,
                                     num_qo_heads, num_kv_heads, 1 if causal else 0,
                                     split_tokens, num_sms, buf, cap, C.byref(info))
    global _plan_cap
    buf = np.empty(_plan_cap, np.int32)       # one call at the last plan's size
    rc = call(_lib.ptr32(buf), buf.size)
    if rc == _lib.BE_ECAPACITY:
        _plan_cap = int(info.total_ints * 1.25) + 1024
        buf = np.empty(_plan_cap, np.int32)
        rc = call(_lib.ptr32(buf), buf.size)
    check(rc, "be_cascade_plan")
    return info, buf[:info.total_ints]


class MultiLevelCascadeAttentionWrapper:
    def __init__(self, num_levels: int, float_workspace_buffer: torch.Tensor,
                 kv_layout: str = "NHD", **_):
        if kv_layout != "NHD":
            raise ValueError("only the NHD layout is supported")
        self.num_levels = num_levels
        self._plan = _Plan(float_workspace_buffer)

    def plan(self, qo_indptr_arr: List[torch.Tensor], paged_kv_indptr_arr: List[torch.Tensor],
             paged_kv_indices_arr: List[torch.Tensor], paged_kv_last_page_len: List[torch.Tensor],
             num_qo_heads: int, num_kv_heads: int, head_dim: int, page_size: int,
             causal: bool = False, pos_encoding_mode: str = "NONE", sm_scale: Optional[float] = None,
             q_data_type=None, split_tokens: int = 0, **_):
        if pos_encoding_mode != "NONE":
            raise ValueError("only pos_encoding_mode='NONE' is supported")
        if len(qo_indptr_arr) != self.num_levels:
            raise ValueError(f"expected {self.num_levels} levels, got {len(qo_indptr_arr)}")
        levels = list(zip(qo_indptr_arr, paged_kv_indptr_arr, paged_kv_indices_arr,
                          paged_kv_last_page_len))
        arrs = [[_i32(lv[k]) for lv in levels] for k in range(4)]
        nq = int(arrs[0][-1][-1]) if levels else 0
        ng = np.asarray([len(a) - 1 for a in arrs[0]], np.int32)
        L = len(levels)
        ptrs = [(_lib.P32 * max(L, 1))(*[_lib.ptr32(a) for a in group]) for group in arrs]
        ps = self._plan
        self._levels_args = (L, ptrs, ng, nq, page_size, num_qo_heads, num_kv_heads, causal,
                             split_tokens, head_dim, arrs)
        self.tiles = False
        if split_tokens == 0 and tiles_eligible(head_dim, page_size, num_qo_heads, num_kv_heads):
            g = num_qo_heads // num_kv_heads
            qo0 = arrs[0][0] if L else np.zeros(1, np.int32)
            rows = tile_rows_for(int(np.max(np.diff(qo0))) * g if len(qo0) > 1 else g)
            tp = target_pieces(ps.num_sms, num_kv_heads)

            def tfn(buf, cap, info):
                return lib().be_tile_plan(L, *ptrs, _lib.ptr32(ng), nq, page_size, num_qo_heads,
                                          num_kv_heads, 1 if causal else 0, rows, tp, -1,
                                          C.cast(buf, _lib.P32), cap, info)
            if ps.build_tiles(tfn):
                ps.place_tiles(num_kv_heads, head_dim)
                self.tiles = True
        if not self.tiles:
            self._plan_items()
        self.num_queries = nq
        self.hq, self.hkv, self.d = num_qo_heads, num_kv_heads, head_dim
        self.sm_scale = sm_scale if sm_scale is not None else head_dim ** -0.5

    def _plan_items(self):
        """The work-item plan (be_cascade_plan) of the last plan() call's levels."""
        (L, ptrs, ng, nq, page_size, hq, hkv, causal, split_tokens, head_dim, _) = \
            self._levels_args
        ps = self._plan

        def fn(buf, cap, info):
            return lib().be_cascade_plan(L, *ptrs, _lib.ptr32(ng), nq, page_size, hq, hkv,
                                         1 if causal else 0, split_tokens, ps.num_sms,
                                         C.cast(buf, _lib.P32), cap, info)
        ps.build(fn)
        ps.place(hq, head_dim)
        ps.tinfo = None
        self.tiles = False

    def run(self, q: torch.Tensor, paged_kv_cache: torch.Tensor, return_lse: bool = False,
            out: Optional[torch.Tensor] = None):
        if q.shape[0] != self.num_queries:
            raise ValueError(f"q has {q.shape[0]} rows, plan has {self.num_queries} queries")
        if out is None:
            out = torch.empty((q.shape[0], self.hq, self.d), dtype=q.dtype, device=q.device)
        lse = torch.empty((q.shape[0], self.hq), dtype=torch.float32,
                          device=q.device) if return_lse else None
        if self.tiles and paged_kv_cache.dtype == torch.float32:
            self._plan_items()               # fp32 pools run on the work-item kernels
        if self.tiles:
            self._plan.run_tiles(q, paged_kv_cache, self.hq, self.hkv, self.d, self.sm_scale, out,
                                 lse)
            return (out, lse) if return_lse else out
        self._plan.run(q, paged_kv_cache, self.hq, self.hkv, self.d, self.sm_scale, out, lse)
        return (out, lse) if return_lse else out

    forward = run


class BatchPrefillWithPagedKVCacheWrapper:
    def __init__(self, float_workspace_buffer: torch.Tensor, kv_layout: str = "NHD", **_):
        if kv_layout != "NHD":
            raise ValueError("only the NHD layout is supported")
        self._inner = MultiLevelCascadeAttentionWrapper(1, float_workspace_buffer)

    def plan(self, qo_indptr, paged_kv_indptr, paged_kv_indices, paged_kv_last_page_len,
             num_qo_heads, num_kv_heads, head_dim_qk, page_size, causal=False,
             pos_encoding_mode="NONE", sm_scale=None, **kw):
        self._inner.plan([qo_indptr], [paged_kv_indptr], [paged_kv_indices],
                         [paged_kv_last_page_len], num_qo_heads, num_kv_heads, head_dim_qk,
                         page_size, causal=causal, pos_encoding_mode=pos_encoding_mode,
                         sm_scale=sm_scale, **kw)

    def run(self, q, paged_kv_cache, return_lse=False, out=None):
        return self._inner.run(q, paged_kv_cache, return_lse=return_lse, out=out)

    forward = run
