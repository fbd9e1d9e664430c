"""Tree (FastTree) attention with the reference's API, on the native planner + kernels.

Same names and arguments as the reference's vendored FastTree package
(``src/beam_engine/attention/fasttree``) and ``kv_tree_node.py``:

* :class:`KVTreeNode` -- ``parent, id, seqlen, num_children, requests``;
* :func:`prepare_fasttree_metadata_for_paged_cache` (preparation.py:11-225):
  the SplitK/SplitQ cost model, vnode emission, req->vnode lists and two-phase
  order, run by ``be_fasttree_prepare`` in C++; the result keeps the
  reference's attribute names plus a ready work-item plan (``be_tree_plan``);
* :func:`fasttree_decode` (kernel.py:288-348): the work items run on the same
  paged attention kernel as the cascade path and the per-request LSE merge.

Differences, all deliberate: K/V are read in place from the page pool (pass
``PageTable.get_k_buffer(layer)`` / ``get_v_buffer(layer)``, zero-copy views),
the partial buffers are sized to the plan (the reference preallocates 81 920
rows), and no message is printed.
"""
from __future__ import annotations

import ctypes as C
from typing import List

import numpy as np
import torch

from . import _lib
from ._lib import AttnPlanInfo, check, lib
from .page_table import dtype_code, require_cuda, stream_ptr


class KVTreeNode:
    """kv_tree_node.py:3-19."""

    def __init__(self):
        self.parent: int = -1
        self.id: int = 0
        self.seqlen: int = 0
        self.num_children: int = 0
        self.requests: list = []


class FastTreeMetadata:
    """metadata.py:5-66 (parameters alpha/beta/gamma, TSQs, TSKs, kv split sizes)."""

    def __init__(self, num_qo_heads, num_kv_heads, head_dim, device="cuda", alpha=0.6, beta=0.3,
                 gamma=0.1, TSQs=None, TSKs=(32, 32), kv_split_sizes=(1024, 128), **_):
        self.num_qo_heads = num_qo_heads
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.kv_group_num = num_qo_heads // num_kv_heads
        self.device = device
        self.alpha, self.beta, self.gamma = alpha, beta, gamma
        self.TSQs = TSQs or (64 // self.kv_group_num, 16 // self.kv_group_num)
        self.TSKs = TSKs
        self.kv_split_sizes = kv_split_sizes
        self.phase_node_nums = None
        self.phase_node_offsets = None
        self.phase_q_tile_sizes = None
        self.phase_kv_tile_sizes = None


_PLANS = {}   # vnode_to_kv_offs.data_ptr() -> (info, plan_dev tensor, mid_o, mid_lse)


def _np32(x):
    return np.ascontiguousarray(np.asarray(x, dtype=np.int32))


def tree_arrays(tree_info: List[KVTreeNode]):
    n = len(tree_info)
    parent = _np32([t.parent for t in tree_info])
    seqlen = _np32([t.seqlen for t in tree_info])
    kids = _np32([t.num_children for t in tree_info])
    ptr = np.zeros(n + 1, np.int32)
    for i, t in enumerate(tree_info):
        ptr[i + 1] = ptr[i] + len(t.requests)
    reqs = _np32([r for t in tree_info for r in t.requests] or [0])
    return parent, seqlen, kids, ptr, reqs


def plan_vnodes(parent, seqlen, kids, ptr, reqs, r2t_stride, batch_size, num_qo_heads,
                num_kv_heads):
    """Host FastTree planner -> dict of int32 numpy arrays (reference names)."""
    n = len(parent)
    cap_v = max(64, 4 * (n + 1) * 8)
    cap_e = max(256, int(ptr[-1]) * 8 + 64)
    while True:
        out = {k: np.zeros(cap_v, np.int32) for k in
               ("vnode_to_q_offs", "vnode_to_q_lens", "vnode_to_kv_offs", "vnode_to_kv_lens")}
        qe = np.zeros(cap_e, np.int32)
        r2v = np.zeros(cap_e, np.int32)
        r2v_offs = np.zeros(max(batch_size, 1), np.int32)
        r2v_lens = np.zeros(max(batch_size, 1), np.int32)
        counts = np.zeros(4, np.int32)
        rc = lib().be_fasttree_prepare(
            n, _lib.ptr32(parent), _lib.ptr32(seqlen), _lib.ptr32(kids), _lib.ptr32(ptr),
            _lib.ptr32(reqs), r2t_stride, batch_size, num_qo_heads, num_kv_heads, cap_v, cap_e,
            _lib.ptr32(qe), _lib.ptr32(out["vnode_to_q_offs"]), _lib.ptr32(out["vnode_to_q_lens"]),
            _lib.ptr32(out["vnode_to_kv_offs"]), _lib.ptr32(out["vnode_to_kv_lens"]),
            _lib.ptr32(r2v), _lib.ptr32(r2v_offs), _lib.ptr32(r2v_lens), _lib.ptr32(counts))
        if rc == _lib.BE_ECAPACITY:
            cap_v, cap_e = int(counts[0]) + 16, int(counts[1]) + 16
            continue
        check(rc, "be_fasttree_prepare")
        break
    nv, ne = int(counts[0]), int(counts[1])
    res = {k: v[:nv] for k, v in out.items()}
    res["vnode_to_q_entries"] = qe[:ne]
    res["req_to_vnode_entries"] = r2v[:ne]
    res["req_to_vnode_offs"] = r2v_offs[:batch_size]
    res["req_to_vnode_lens"] = r2v_lens[:batch_size]
    res["phase_node_nums"] = (int(counts[2]), int(counts[3]))
    res["phase_node_offsets"] = (0, int(counts[2]))
    g = num_qo_heads // num_kv_heads
    res["phase_q_tile_sizes"] = (64 // g, 16 // g)
    res["phase_kv_tile_sizes"] = (32, 32)
    return res


def build_tree_plan(v, batch_size, page_size, num_qo_heads, num_kv_heads):
    info = AttnPlanInfo()
    args = [len(v["vnode_to_q_offs"]), _lib.ptr32(v["vnode_to_q_entries"]),
            len(v["vnode_to_q_entries"]), _lib.ptr32(v["vnode_to_q_offs"]),
            _lib.ptr32(v["vnode_to_q_lens"]), _lib.ptr32(v["vnode_to_kv_offs"]),
            _lib.ptr32(v["vnode_to_kv_lens"]), _lib.ptr32(v["req_to_vnode_entries"]),
            _lib.ptr32(v["req_to_vnode_offs"]), _lib.ptr32(v["req_to_vnode_lens"]), batch_size,
            page_size, num_qo_heads, num_kv_heads]
    rc = lib().be_tree_plan(*args, None, 0, C.byref(info))
    if rc not in (_lib.BE_OK, _lib.BE_ECAPACITY):
        check(rc, "be_tree_plan")
    buf = np.zeros(max(info.total_ints, 1), np.int32)
    check(lib().be_tree_plan(*args, _lib.ptr32(buf), buf.size, C.byref(info)), "be_tree_plan")
    return info, buf


def build_tree_page_plan(v, slots, batch_size, page_size, num_qo_heads, num_kv_heads, num_sms=148):
    """The vnodes as a page-list plan (``be_tree_plan_pages``) for the tensor-core
    decode kernels; ``slots`` is the flat slot table the vnodes index.  Returns
    (info, plan) or None when the tree is not page aligned (use build_tree_plan)."""
    slots = np.ascontiguousarray(slots, np.int32)
    info = AttnPlanInfo()
    keep = [np.ascontiguousarray(v[k], np.int32) for k in
            ("vnode_to_q_entries", "vnode_to_q_offs", "vnode_to_q_lens", "vnode_to_kv_offs",
             "vnode_to_kv_lens")]
    args = [len(keep[1]), _lib.addr(keep[0]), len(keep[0]), _lib.addr(keep[1]), _lib.addr(keep[2]),
            _lib.addr(keep[3]), _lib.addr(keep[4]), _lib.addr(slots), len(slots), batch_size,
            page_size, num_qo_heads, num_kv_heads, num_sms]
    rc = lib().be_tree_plan_pages(*args, None, 0, C.byref(info))
    if rc == _lib.BE_EINVAL:
        return None
    if rc not in (_lib.BE_OK, _lib.BE_ECAPACITY):
        check(rc, "be_tree_plan_pages")
    buf = np.zeros(max(info.total_ints, 1), np.int32)
    check(lib().be_tree_plan_pages(*args, _lib.addr(buf), buf.size, C.byref(info)),
          "be_tree_plan_pages")
    return info, buf


def prepare_fasttree_metadata_for_paged_cache(tree_info: List[KVTreeNode], req_to_token: torch.Tensor,
                                              batch_size: int, num_qo_heads: int, num_kv_heads: int,
                                              head_dim: int, device="cuda", page_size: int = None):
    """preparation.py:11-225.  ``page_size`` is needed only to decode slot ids
    when the plan runs; it defaults to the pool's page size at decode time."""
    md = FastTreeMetadata(num_qo_heads, num_kv_heads, head_dim, device)
    parent, seqlen, kids, ptr, reqs = tree_arrays(tree_info)
    v = plan_vnodes(parent, seqlen, kids, ptr, reqs, int(req_to_token.stride(0)), batch_size,
                    num_qo_heads, num_kv_heads)
    dev = torch.device(device)
    for k in ("vnode_to_q_entries", "vnode_to_q_offs", "vnode_to_q_lens", "vnode_to_kv_offs",
              "vnode_to_kv_lens", "req_to_vnode_entries", "req_to_vnode_offs",
              "req_to_vnode_lens"):
        setattr(md, k, torch.from_numpy(v[k].copy()).to(dev))
    md.phase_node_nums = v["phase_node_nums"]
    md.phase_node_offsets = v["phase_node_offsets"]
    md.phase_q_tile_sizes = tuple(md.TSQs)
    md.phase_kv_tile_sizes = tuple(md.TSKs)
    flat = req_to_token.reshape(-1).to(torch.int32)
    md.vnode_to_kv_entries = torch.nn.functional.pad(flat, (0, 256), value=-1).to(dev)
    md._host = v
    md.batch_size = batch_size
    ne = len(v["vnode_to_q_entries"])
    md.mid_o = torch.empty((max(ne, 1), num_qo_heads, head_dim), dtype=torch.float32, device=dev)
    md.mid_lse = torch.empty((max(ne, 1), num_qo_heads), dtype=torch.float32, device=dev)
    md._plans = {}
    _PLANS[md.vnode_to_kv_offs.data_ptr()] = md
    return md


def _plan_for(md, page_size):
    if page_size not in md._plans:
        info, buf = build_tree_plan(md._host, md.batch_size, page_size, md.num_qo_heads,
                                    md.num_kv_heads)
        md._plans[page_size] = (info, torch.from_numpy(buf).to(md.vnode_to_kv_offs.device))
    return md._plans[page_size]


def _pool_from_views(k_buffer, v_buffer):
    """k/v views [pages, page_size, H, D] of one [pages, 2, page_size, H, D] pool."""
    if k_buffer.dim() != 4:
        raise ValueError("k_buffer/v_buffer must be the pool views returned by "
                         "PageTable.get_k_buffer/get_v_buffer ([pages, page_size, H, D])")
    P, ps, H, D = k_buffer.shape
    elt = k_buffer.element_size()
    if (k_buffer.stride() != (2 * ps * H * D, H * D, D, 1) or v_buffer.stride() != k_buffer.stride()
            or v_buffer.data_ptr() != k_buffer.data_ptr() + ps * H * D * elt):
        raise ValueError("k_buffer/v_buffer are not the K/V planes of one paged pool")
    return P, ps, H, D


def fasttree_decode(q, k_buffer, v_buffer, o, vnode_to_kv_entries, vnode_to_kv_offs,
                    vnode_to_kv_lens, vnode_to_q_entries, vnode_to_q_offs, vnode_to_q_lens,
                    req_to_vnode_entries, req_to_vnode_offs, req_to_vnode_lens, mid_o, mid_lse,
                    phase_node_nums, phase_node_offsets, phase_q_tile_sizes, phase_kv_tile_sizes,
                    sm_scale, logit_cap=-1):
    """kernel.py:288-348 on the native kernels (K/V read in place from the pool)."""
    require_cuda(q, k_buffer, o)
    P, ps, H, D = _pool_from_views(k_buffer, v_buffer)
    Hq = q.shape[1]
    md = _PLANS.get(vnode_to_kv_offs.data_ptr())
    if md is None:   # metadata built elsewhere: read it back once (synchronises)
        host = {k: t.detach().cpu().numpy().astype(np.int32) for k, t in (
            ("vnode_to_q_entries", vnode_to_q_entries), ("vnode_to_q_offs", vnode_to_q_offs),
            ("vnode_to_q_lens", vnode_to_q_lens), ("vnode_to_kv_offs", vnode_to_kv_offs),
            ("vnode_to_kv_lens", vnode_to_kv_lens), ("req_to_vnode_entries", req_to_vnode_entries),
            ("req_to_vnode_offs", req_to_vnode_offs), ("req_to_vnode_lens", req_to_vnode_lens))}
        nv = int(sum(phase_node_nums))
        for k in ("vnode_to_q_offs", "vnode_to_q_lens", "vnode_to_kv_offs", "vnode_to_kv_lens"):
            host[k] = host[k][:nv]
        B = q.shape[0]
        host["req_to_vnode_offs"] = host["req_to_vnode_offs"][:B]
        host["req_to_vnode_lens"] = host["req_to_vnode_lens"][:B]
        ne = int(host["req_to_vnode_lens"].sum())
        host["vnode_to_q_entries"] = host["vnode_to_q_entries"][:ne]
        host["req_to_vnode_entries"] = host["req_to_vnode_entries"][:ne]
        info, buf = build_tree_plan(host, B, ps, Hq, H)
        plan_dev = torch.from_numpy(buf).to(q.device)
    else:
        info, plan_dev = _plan_for(md, ps)
    if mid_o.shape[0] < info.n_parts or mid_o.dtype != torch.float32:
        raise ValueError("mid_o too small for the plan")
    if q.stride(-1) != 1 or q.stride(-2) != D:
        q = q.contiguous()
    rc = lib().be_attn_run(plan_dev.data_ptr(), C.byref(info), q.data_ptr(), q.stride(0),
                           k_buffer.data_ptr(), P, Hq, H, D, dtype_code(k_buffer.dtype),
                           float(sm_scale), o.data_ptr(), o.stride(0), None, mid_o.data_ptr(),
                           mid_lse.data_ptr(), vnode_to_kv_entries.data_ptr(),
                           stream_ptr(q.device))
    check(rc, "fasttree_decode")
    return o
