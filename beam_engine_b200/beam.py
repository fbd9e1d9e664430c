"""BeamSearchGenerator: the reference's engine loop (src/beam_engine/beam.py:17-352)
on the B200 path.

Same constructor and ``generate`` signature as the reference.  One decode step:
  host (C++): cascade levels of the trie -> work-item plan; decode inputs
  device: one forward over all beams (fused RoPE/append, paged attention,
          cuBLAS GEMMs), log-softmax + top-2W per beam
  host (C++): global top-W per prompt, trie update; device: ONE batched
          copy-on-write kernel for every fork of the step (all layers).
Per step there is one H2D copy of the step's metadata + plan and one D2H copy
of the [beams, 2W] top-k (the reference makes W*2W ``.item()`` syncs).
``generate_ids`` runs several prompts at once (each with its own W beams) in
the same forward; the trie holds one root chain per prompt.
"""
from __future__ import annotations

import ctypes as C
import logging
import os
import time
from typing import List, Optional, Sequence

import numpy as np
import torch

from . import _lib
from ._lib import check, lib
from .beam_state import BeamState
from .beam_strategy import VanillaBeamSearchStrategy
from .cascade import _Plan, target_pieces, tile_rows_for, tiles_eligible
from .page_table import PageTable, stream_ptr
from .parallel import vocab_parallel_log_softmax_topk

logger = logging.getLogger(__name__)
UMMA_MAX_TOKENS = 128   # BE_UMMA_MAX_TOKENS in include/beam_b200.h
_NVTX = os.environ.get("BE_NVTX", "0") == "1"   # NVTX ranges per generation phase


class _Range:
    """NVTX range (BE_NVTX=1) around a phase of generation, for nsys / ncu timelines."""
    __slots__ = ("name",)

    def __init__(self, name):
        self.name = name

    def __enter__(self):
        if _NVTX:
            torch.cuda.nvtx.range_push(self.name)

    def __exit__(self, *exc):
        if _NVTX:
            torch.cuda.nvtx.range_pop()


def _i32(a):
    return np.ascontiguousarray(a, dtype=np.int32)


class PlannedAttention:
    """Paged attention for every layer of one forward, from one plan."""

    def __init__(self, model, page_table, workspace):
        self.m = model
        self.pt = page_table
        self.plan = _Plan(workspace)
        self.scale = model.D ** -0.5
        self.kv_list = None
        self.timer = None          # optional (start_event, end_event) list collector

    def plan_levels(self, levels, num_queries, causal=True, split_tokens=0):
        L = len(levels)
        arrs = [[_i32(lv[k]) for lv in levels] for k in
                ("qo_indptr", "kv_indptr", "kv_indices", "kv_last_page_len")]
        ng = _i32([len(a) - 1 for a in arrs[0]])
        ptrs = [(_lib.P32 * max(L, 1))(*[_lib.ptr32(a) for a in grp]) for grp in arrs]
        m, ps, p = self.m, self.pt.page_size, self.plan
        self.kv_list = None
        if (split_tokens == 0 and self.pt.store_dtype != torch.float32
                and tiles_eligible(m.D, ps, m.Hq, m.Hkv)):
            g = m.Hq // m.Hkv
            qo0 = arrs[0][0] if L else np.zeros(1, np.int32)
            rows = tile_rows_for(int(np.max(np.diff(qo0))) * g if len(qo0) > 1 else g)
            tp = target_pieces(p.num_sms, m.Hkv)

            def tfn(buf, cap, info):
                return lib().be_tile_plan(L, *ptrs, _lib.ptr32(ng), num_queries, ps, m.Hq, m.Hkv,
                                          1 if causal else 0, rows, tp, -1,
                                          C.cast(buf, _lib.P32), cap, info)
            if p.build_tiles(tfn):
                p.place_tiles(m.Hkv, m.D)
                return

        def fn(buf, cap, info):
            return lib().be_cascade_plan(L, *ptrs, _lib.ptr32(ng), num_queries, ps, m.Hq, m.Hkv,
                                         1 if causal else 0, split_tokens, p.num_sms,
                                         C.cast(buf, _lib.P32), cap, info)
        p.build(fn)
        p.place(m.Hq, m.D)
        p.tinfo = None

    def plan_prebuilt(self, info, buf):
        """Place a plan built elsewhere (a page-list tree plan)."""
        p = self.plan
        p.tinfo = None
        p.info = info
        host = torch.from_numpy(np.ascontiguousarray(buf[:info.total_ints]))
        if p.copied is not None:          # previous H2D still reading the staging buffer
            p.copied.synchronize()
        if p.host.numel() < host.numel():
            p.host = torch.empty(host.numel(), dtype=torch.int32).pin_memory()
        p.host[:host.numel()].copy_(host)
        p.place(self.m.Hq, self.m.D)
        self.kv_list = None

    def plan_tree(self, vnodes, batch_size, kv_entries_dev):
        from .fasttree import build_tree_plan
        info, buf = build_tree_plan(vnodes, batch_size, self.pt.page_size, self.m.Hq, self.m.Hkv)
        p = self.plan
        p.tinfo = None
        p.info = info
        host = torch.from_numpy(buf)
        if p.copied is not None:          # previous H2D still reading the staging buffer
            p.copied.synchronize()
        if p.host.numel() < host.numel():
            p.host = torch.empty(host.numel(), dtype=torch.int32).pin_memory()
        p.host[:host.numel()].copy_(host)
        p.place(self.m.Hq, self.m.D)
        self.kv_list = kv_entries_dev

    def run(self, layer, qkv, out):
        m = self.m
        t = self.timer
        if t is not None:
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
        if self.plan.tinfo is not None:
            self.plan.run_tiles(qkv[:, :m.Hq * m.D].view(-1, m.Hq, m.D), self.pt.kv_cache[layer],
                                m.Hq, m.Hkv, m.D, self.scale, out.view(-1, m.Hq, m.D))
            if t is not None:
                e.record()
                t.append((s, e))
            return
        rc = lib().be_attn_run(
            C.c_void_p(self.plan.plan_dev), C.byref(self.plan.info), qkv.data_ptr(), qkv.stride(0),
            self.pt.kv_cache[layer].data_ptr(), self.pt.max_num_pages, m.Hq, m.Hkv, m.D,
            m.dt, self.scale, out.data_ptr(), out.stride(0), None,
            C.c_void_p(self.plan.mid_o), C.c_void_p(self.plan.mid_lse),
            self.kv_list.data_ptr() if self.kv_list is not None else None, stream_ptr(qkv.device))
        check(rc, "be_attn_run")
        if t is not None:
            e.record()
            t.append((s, e))


def step_sel_offsets(n):
    """Offsets (int32 units) of the device-selection inputs in a step buffer of n
    beams: prompt ranges seg_ptr [<= n + 1] after the fork list, then the
    parents' accumulated scores as n doubles (8-byte aligned)."""
    seg_off = 7 * n + 1
    scores_off = (seg_off + n + 2) // 2 * 2
    return seg_off, scores_off


def step_lens_offset(n):
    """Offset (int32 units) of the parents' sequence offsets [n + 1] (their
    lengths, for the device diverse selection's length penalty), after the
    scores."""
    return step_sel_offsets(n)[1] + 2 * n


def step_plan_offset(n):
    """Offset (int32 units) of the attention plan in a step buffer of n beams."""
    return -(-(step_lens_offset(n) + n + 1) // 32) * 32


def _pool_dtype(pt):
    return (_lib.BE_F32 if pt.store_dtype == torch.float32 else
            (_lib.BE_BF16 if pt.store_dtype == torch.bfloat16 else _lib.BE_F16))


class DeviceSelection:
    """A step's vanilla selection made on the device (be_vanilla_select_device):
    per prompt, beam_size (parent candidate, token, accumulated score) in rank
    order, parent -1 past the prompt's entries."""
    __slots__ = ("parent", "token", "score")

    def __init__(self, parent, token, score):
        self.parent, self.token, self.score = parent, token, score


class DiverseSelection:
    """A step's diverse selection (hamming) made on the device
    (be_diverse_select_device): children per parent as be_diverse_select
    returns them -- child_ptr [candidates + 1], tokens and scores, and the new
    prompt ranges."""
    __slots__ = ("child_ptr", "tokens", "scores", "new_seg")

    def __init__(self, child_ptr, tokens, scores, new_seg):
        m = int(new_seg[-1])
        self.child_ptr, self.tokens, self.scores, self.new_seg = (child_ptr, tokens[:m],
                                                                  scores[:m], new_seg)


class StepGraph:
    """One beam decode step (forward over all layers, log-softmax, top-k, D2H
    of the top-k) recorded once as a CUDA graph and replayed every step.

    Everything that changes per step lives in one static device buffer
    [query ids | positions | append pages | append slots | fork copy list
    | attention plan | slot list (tree plans)] filled by one H2D copy before
    the replay; the step's first launch performs the copy-on-write tail copies
    of the previous selection (``be_fork_tail_copy_list``);
    attention runs through ``be_attn_run_fixed_2s``, whose launch shape depends
    only on the capacities (the kernels read the plan's counts from its
    device-side header).  ``kind`` is "cascade" (page-list plans, tensor-core
    prefix and suffix kernels) or "fasttree" (slot-list plans, general kernel)."""

    def __init__(self, gen, n, k, temperature, caps, kind="cascade"):
        self.gen, self.n, self.k, self.temp = gen, n, k, temperature
        self.kind = kind
        m = gen.model
        self.caps = dict(caps)
        self.caps.setdefault("slots", 0)
        dev = gen.device
        # [q | pos | pages | slots] then the fork list [count | src[n] | dst[n] | len[n]]
        self.fork_off = 4 * n
        self.plan_off = step_plan_offset(n)
        self.slots_off = self.plan_off + -(-self.caps["ints"] // 32) * 32
        self.total = self.slots_off + self.caps["slots"]
        self.dev_buf = torch.zeros(self.total, dtype=torch.int32, device=dev)
        self.host_buf = torch.empty(self.total, dtype=torch.int32).pin_memory()
        if kind == "tiles":
            # partial rows [part pieces][kv heads][tile rows][D] + LSE
            slots = max(1, self.caps["part_pieces"]) * m.Hkv * self.caps["rows"]
            self.mid_o = torch.empty(slots * m.D, dtype=m.dtype, device=dev)
            self.mid_lse = torch.empty(slots, dtype=torch.float32, device=dev)
        else:
            self.mid_o = torch.empty(max(1, self.caps["parts"]) * m.Hq * m.D,
                                     dtype=torch.float32, device=dev)
            self.mid_lse = torch.empty(max(1, self.caps["parts"]) * m.Hq, dtype=torch.float32,
                                       device=dev)
        self.vals_h = torch.empty(n * k, dtype=torch.float32).pin_memory()
        self.idx_h = torch.empty(n * k, dtype=torch.int64).pin_memory()
        # global top-W on the device (vanilla strategy): nseg prompts of beam width W
        # None or (nseg, W, max candidates per prompt, diverse): diverse is None for the
        # vanilla selection, else (num_groups, diversity_penalty, length_penalty)
        self.select = caps.get("select")
        if self.select is not None and self.select[3] is not None:
            nseg, W, _, (groups, _, _) = self.select
            self.seg_off, self.scores_off = step_sel_offsets(n)
            self.lens_off = step_lens_offset(n)
            cap = max(1, nseg * max(W, groups))
            self.sel_d = (torch.empty(n + 1, dtype=torch.int32, device=dev),
                          torch.empty(cap, dtype=torch.int32, device=dev),
                          torch.empty(cap, dtype=torch.float64, device=dev),
                          torch.empty(nseg + 1, dtype=torch.int32, device=dev))
            self.sel_h = tuple(torch.empty(x.numel(), dtype=x.dtype).pin_memory()
                               for x in self.sel_d)
        elif self.select is not None:
            nseg, W, _, _ = self.select
            self.seg_off, self.scores_off = step_sel_offsets(n)
            self.sel_d = (torch.empty(nseg * W, dtype=torch.int32, device=dev),
                          torch.empty(nseg * W, dtype=torch.int32, device=dev),
                          torch.empty(nseg * W, dtype=torch.float64, device=dev))
            self.sel_h = (torch.empty(nseg * W, dtype=torch.int32).pin_memory(),
                          torch.empty(nseg * W, dtype=torch.int32).pin_memory(),
                          torch.empty(nseg * W, dtype=torch.float64).pin_memory())
        if kind != "tiles":
            self.ccaps = _lib.AttnCaps(self.caps["work"], self.caps["wide"], self.caps["merge"], 1,
                                       _lib.BE_CAPS_SLOTS if kind == "fasttree" else 0)
        # suffix tiles on a second stream, overlapping the shared-prefix tiles
        self.side = (torch.cuda.Stream(dev) if os.environ.get("BE_ATTN_TWO_STREAMS", "1") != "0"
                     else None)
        self.graph = None
        # optional per-layer attention timing inside the graph (external event nodes)
        self.timing = bool(getattr(gen, "time_attention", False))
        self.events = None
        if self.timing:
            from cuda.bindings import runtime as rt
            self._rt = rt
            self.events = []
            for _ in range(2 * m.L):
                err, ev = rt.cudaEventCreate()
                self.events.append(ev)

    def fits(self, n, k, temperature, info, n_slots=0):
        c = self.caps
        if self.kind == "tiles":
            return (n == self.n and k == self.k and temperature == self.temp
                    and info.n_pieces <= c["pieces"] and info.n_tiles <= c["tiles"]
                    and info.n_part_pieces <= c["part_pieces"] and info.total_ints <= c["ints"]
                    and info.tile_rows == c["rows"] and info.cluster == c["cluster"])
        return (n == self.n and k == self.k and temperature == self.temp
                and info.n_work <= c["work"] and info.n_work_wide <= c["wide"]
                and info.n_merge <= c["merge"] and info.n_parts <= c["parts"]
                and info.total_ints <= c["ints"] and n_slots <= c["slots"]
                and (self.kind != "cascade" or info.max_wide_tokens <= UMMA_MAX_TOKENS))

    def _mark(self, idx, qkv):
        if self.timing and torch.cuda.is_current_stream_capturing():
            self._rt.cudaEventRecordWithFlags(self.events[idx],
                                              torch.cuda.current_stream(qkv.device).cuda_stream,
                                              self._rt.cudaEventRecordExternal)

    def attention_ms(self):
        """Per-layer attention durations (ms) of the last replay."""
        out = []
        for i in range(len(self.events) // 2):
            err, ms = self._rt.cudaEventElapsedTime(self.events[2 * i], self.events[2 * i + 1])
            out.append(float(ms))
        return out

    def run(self, layer, qkv, out):  # attention of one layer (the model calls this)
        m, pt = self.gen.model, self.gen.page_table
        self._mark(2 * layer, qkv)
        if self.kind == "tiles":
            c = self.caps
            rc = lib().be_attn_tiles_run(
                self.dev_buf.data_ptr() + 4 * self.plan_off, c["pieces"], c["tiles"],
                c["part_pieces"], c["rows"], pt.page_size, qkv.data_ptr(), qkv.stride(0),
                pt.kv_cache[layer].data_ptr(), pt.max_num_pages, m.Hq, m.Hkv, m.D, m.dt,
                m.D ** -0.5, out.data_ptr(), out.stride(0), None, self.mid_o.data_ptr(),
                self.mid_lse.data_ptr(), c["cluster"], 1, stream_ptr(qkv.device))
            check(rc, "be_attn_tiles_run")
            self._mark(2 * layer + 1, qkv)
            return
        rc = lib().be_attn_run_fixed_2s(
            self.dev_buf.data_ptr() + 4 * self.plan_off, C.byref(self.ccaps), pt.page_size,
            qkv.data_ptr(), qkv.stride(0), pt.kv_cache[layer].data_ptr(), pt.max_num_pages, m.Hq,
            m.Hkv, m.D, m.dt, m.D ** -0.5, out.data_ptr(), out.stride(0), None,
            self.mid_o.data_ptr(), self.mid_lse.data_ptr(),
            (self.dev_buf.data_ptr() + 4 * self.slots_off) if self.kind == "fasttree" else None,
            stream_ptr(qkv.device),
            C.c_void_p(self.side.cuda_stream) if self.side is not None else None)
        check(rc, "be_attn_run_fixed_2s")
        self._mark(2 * layer + 1, qkv)

    def set_fork(self, copies):
        """Write the pending copy-on-write list (src, dst, len arrays; None = none)."""
        h = self.host_buf.numpy()
        n, o = self.n, self.fork_off
        if copies is None or len(copies[0]) == 0:
            h[o] = 0
            return
        c = len(copies[0])
        h[o] = c
        h[o + 1:o + 1 + c] = copies[0]
        h[o + 1 + n:o + 1 + n + c] = copies[1]
        h[o + 1 + 2 * n:o + 1 + 2 * n + c] = copies[2]

    def _body(self):
        n = self.n
        d = self.dev_buf
        pt = self.gen.page_table
        check(lib().be_fork_tail_copy_list(pt.kv_cache.data_ptr(), pt.kv_cache.stride(0),
                                           pt.layer_num, pt.max_num_pages, pt.page_size,
                                           pt.head_num, pt.head_dim, _pool_dtype(pt),
                                           d.data_ptr() + 4 * self.fork_off, n,
                                           self.gen.attn.plan.num_sms,
                                           stream_ptr(self.gen.device)), "fork list")
        logits = self.gen.model.forward(d[0:n], d[n:2 * n], self.gen.page_table, d[2 * n:3 * n],
                                        d[3 * n:4 * n], self)
        v, i = self.gen._logprob_topk(logits, self.k, self.temp)
        if self.select is not None and self.select[3] is not None:
            # diverse selection (hamming) on the device; only the children leave it
            nseg, W, maxc, (groups, dpen, lpen) = self.select
            v64 = v.to(torch.float64).contiguous()
            i32 = i.to(torch.int32).contiguous()
            cp, ct, cs, ns = self.sel_d
            check(lib().be_diverse_select_device(
                nseg, d.data_ptr() + 4 * self.seg_off, self.k, d.data_ptr() + 4 * self.scores_off,
                i32.data_ptr(), v64.data_ptr(), d.data_ptr() + 4 * self.lens_off, W, groups,
                dpen, 0, lpen, maxc, cp.data_ptr(), ct.data_ptr(), cs.data_ptr(), ns.data_ptr(),
                stream_ptr(self.gen.device)), "device diverse selection")
            for h, x in zip(self.sel_h, self.sel_d):
                h.copy_(x, non_blocking=True)
            return
        if self.select is not None:
            # selection on the device; only beam_size (parent, token, score) per prompt leave it
            nseg, W, maxc, _ = self.select
            v, i = v.contiguous(), i.contiguous()
            sp, st, ss = self.sel_d
            check(lib().be_vanilla_select_device(
                nseg, d.data_ptr() + 4 * self.seg_off, self.k, d.data_ptr() + 4 * self.scores_off,
                v.data_ptr(), i.data_ptr(), W, maxc, sp.data_ptr(), st.data_ptr(), ss.data_ptr(),
                stream_ptr(self.gen.device)), "device selection")
            for h, x in zip(self.sel_h, self.sel_d):
                h.copy_(x, non_blocking=True)
            return
        self.vals_h.copy_(v.reshape(-1), non_blocking=True)
        self.idx_h.copy_(i.reshape(-1), non_blocking=True)

    def step_filled(self, used):
        """Replay with host_buf[:used] already holding [q | pos | pages | slots | fork | plan]."""
        n = self.n
        self.dev_buf[:used].copy_(self.host_buf[:used], non_blocking=True)
        self.gen.h2d_bytes += 4 * used
        if self.graph is None:
            t0 = time.perf_counter()
            if not self.gen._graph_warm:   # first capture of the generator: warm libraries up
                cur = torch.cuda.current_stream(self.gen.device)
                side = torch.cuda.Stream(self.gen.device)
                side.wait_stream(cur)
                with torch.cuda.stream(side):
                    self._body()            # warm-up (writes the same K/V the replay will)
                cur.wait_stream(side)
                self.gen._graph_warm = True
            g = torch.cuda.CUDAGraph()
            # thread-local capture: other threads (NCCL's watchdog polling its
            # events) may keep making CUDA calls while this one records
            with torch.cuda.graph(g, capture_error_mode="thread_local"):
                self._body()
            self.graph = g
            self.gen.graph_captures.append(time.perf_counter() - t0)
        self.graph.replay()
        torch.cuda.current_stream(self.gen.device).synchronize()
        if self.timing and self.gen.attn_times is not None:
            self.gen.attn_times.extend(self.attention_ms())
        k = self.k
        if self.select is not None:
            self.gen.d2h_bytes += sum(h.numel() * h.element_size() for h in self.sel_h)
            if self.select[3] is not None:
                return DiverseSelection(*(h.numpy().copy() for h in self.sel_h))
            return DeviceSelection(*(h.numpy().copy() for h in self.sel_h))
        self.gen.d2h_bytes += n * k * (4 + 8)
        return (self.vals_h.numpy()[:n * k].reshape(n, k).astype(np.float64),
                self.idx_h.numpy()[:n * k].reshape(n, k).astype(np.int32))

    def set_selection_inputs(self, seg, scores, seq_ptr=None):
        """Prompt ranges and parent scores of this step for the device selection
        (and, for the diverse selection, the parents' sequence offsets)."""
        h = self.host_buf.numpy()
        h[self.seg_off:self.seg_off + len(seg)] = seg
        h[self.scores_off:self.scores_off + 2 * len(scores)].view(np.float64)[:] = scores
        if seq_ptr is not None:
            h[self.lens_off:self.lens_off + len(seq_ptr)] = seq_ptr


class BeamSearchGenerator:
    """beam.py:17-352.  ``model`` is a :class:`BeamLlama`."""

    def __init__(self, model, tokenizer, strategy, page_size: int = 8, kernel_type: str = "cascade",
                 max_num_pages: int = 1024, store_dtype: Optional[torch.dtype] = None,
                 workspace_bytes: int = 128 << 20, use_graph: bool = True):
        if kernel_type not in ("cascade", "fasttree", "auto"):
            raise ValueError(f"Unknown kernel_type: {kernel_type}. "
                             "Must be 'cascade', 'fasttree' or 'auto'.")
        self.model = model
        self.tokenizer = tokenizer
        self.strategy = strategy
        self.device = model.device
        self.page_size = page_size
        self.kernel_type = kernel_type
        c = model.config
        self.page_table = PageTable(layer_num=c["num_hidden_layers"], page_size=page_size,
                                    max_num_pages=max_num_pages, head_num=model.Hkv,
                                    head_dim=model.D, device=self.device,
                                    store_dtype=store_dtype or model.dtype)
        self.workspace = torch.empty(workspace_bytes, dtype=torch.uint8, device=self.device)
        self.attn = PlannedAttention(model, self.page_table, self.workspace)
        self.meta_host = torch.empty(0, dtype=torch.int32).pin_memory()
        self.topk_host = None
        self.step_timer = None
        # cascade decode steps replay one CUDA graph (bf16/fp16 pools, page size 16)
        self.use_graph = (use_graph and kernel_type in ("cascade", "auto") and page_size == 16
                          and self.page_table.store_dtype != torch.float32)
        # tree steps replay their own graph (slot-list plans, any page size, 2-byte pools)
        self.use_graph_tree = (use_graph and kernel_type in ("fasttree", "auto")
                               and self.page_table.store_dtype != torch.float32)
        self.step_graph = None
        self.step_graph_tree = None
        self._tree_stash = None       # the picker's tree plan, reused by the same step
        self.time_attention = False   # record per-layer attention events in the step graph
        self.attn_times = None        # list to collect them into (ms per launch) when set
        self.plan_hook = None         # called with (queries, plan info) per graph step
        self.picks = []               # kernel_type "auto": the choice of every decode step
        self.graph_captures = []      # seconds spent recording each step graph
        self.graph_regrowth = []      # why a step graph was recorded again
        self._graph_warm = False
        self._pending_fork = None     # copies of the last selection, run by the next graph step
        # tree steps as page-list plans on the tensor-core kernels (default; BE_TREE_PAGES=0 keeps
        # the slot-list plan of the general kernel, which also serves trees that are not page
        # aligned)
        self.tree_pages = (os.environ.get("BE_TREE_PAGES", "1") == "1" and page_size == 16
                           and self.page_table.store_dtype != torch.float32)
        self.step_graph_tpages = None
        self.step_graph_tiles = None
        # cascade steps on the beam-tile kernel (BE_ATTN_TILES=0: the work-item kernels)
        self.use_tiles = (self.page_table.store_dtype != torch.float32
                          and tiles_eligible(model.D, page_size, model.Hq, model.Hkv))
        self._beam_width = 1
        # vanilla selection on the device inside the tile step graph (BE_DEVICE_SELECT=0: host)
        self.device_select = os.environ.get("BE_DEVICE_SELECT", "1") == "1"
        self._sel_ctx = None          # (prompt ranges, beam width) of the step being run
        self.h2d_bytes = 0
        self.d2h_bytes = 0            # device -> host bytes of the scoring / selection results            # host -> device bytes copied by the engine (inputs, plans)

    # ------------------------------------------------------------------
    def generate(self, input_text: str, beam_size: int = 4, max_length: int = 50,
                 num_return_sequences: int = 1, temperature: float = 1.0,
                 pad_token_id: Optional[int] = None, eos_token_id: Optional[int] = None) -> List[str]:
        inputs = self.tokenizer(input_text, return_tensors="pt")
        ids = inputs.input_ids[0].tolist()
        final = self.generate_ids([ids], beam_size, max_length=max_length,
                                  num_return_sequences=num_return_sequences,
                                  temperature=temperature)[0]
        return [self.tokenizer.decode(t, skip_special_tokens=True) for t, _ in final]

    def _to_device(self, arrays: Sequence[np.ndarray]):
        """One pinned staging buffer, one H2D copy -> list of int32 device views."""
        n = sum(len(a) for a in arrays)
        # the previous copy out of the staging buffer must finish before the
        # buffer is reused -- or dropped for a larger one
        if getattr(self, "_meta_ev", None) is not None:
            self._meta_ev.synchronize()
        if self.meta_host.numel() < n:
            self.meta_host = torch.empty(max(n, 1024) * 2, dtype=torch.int32).pin_memory()
        hv = self.meta_host.numpy()
        off = 0
        for a in arrays:
            hv[off:off + len(a)] = a
            off += len(a)
        dev = torch.empty(n, dtype=torch.int32, device=self.device)
        dev.copy_(self.meta_host[:n], non_blocking=True)
        self.h2d_bytes += 4 * n
        self._meta_ev = torch.cuda.Event()
        self._meta_ev.record()
        out, off = [], 0
        for a in arrays:
            out.append(dev[off:off + len(a)])
            off += len(a)
        return out

    def _logprob_topk(self, logits, k, temperature):
        """log_softmax over the full vocabulary, then top-k (beam.py:266-317);
        vocab-parallel across the tensor-parallel group when the model is sharded."""
        m = self.model
        return vocab_parallel_log_softmax_topk(logits, k, getattr(m, "v0", 0), getattr(m, "tp", None),
                                               temperature, getattr(m, "comm", None))

    def _topk(self, logits, k, temperature):
        vals, idx = self._logprob_topk(logits, k, temperature)
        n = vals.shape[0]
        if self.topk_host is None or self.topk_host[0].shape[0] < n * k:
            self.topk_host = (torch.empty(n * k * 2, dtype=torch.float32).pin_memory(),
                              torch.empty(n * k * 2, dtype=torch.int64).pin_memory())
        hv, hi = self.topk_host
        hv[:n * k].copy_(vals.reshape(-1), non_blocking=True)
        hi[:n * k].copy_(idx.reshape(-1), non_blocking=True)
        self.d2h_bytes += n * k * (4 + 8)
        torch.cuda.current_stream(self.device).synchronize()
        return (hv[:n * k].numpy().reshape(n, k).astype(np.float64),
                hi[:n * k].numpy().reshape(n, k).astype(np.int32))

    def prefill(self, state: BeamState, prompts: List[List[int]]):
        """Allocate each prompt's pages, run the causal prompt forward, return the
        last-position logits of each prompt [P, vocab]."""
        ps = self.page_table.page_size
        pages_all, qo, kvp, last = [], [0], [0], []
        ids, pos, wpage, wpos = [], [], [], []
        for pr in prompts:
            chain = state.add_root_sequence(pr)
            pages = np.asarray([n.page_id for n in chain], np.int32)
            pages_all.extend(pages.tolist())
            kvp.append(kvp[-1] + len(pages))
            last.append(len(chain[-1].tokens))
            qo.append(qo[-1] + len(pr))
            ids.append(np.asarray(pr, np.int32))
            t = np.arange(len(pr), dtype=np.int32)
            pos.append(t)
            wpage.append(pages[t // ps])
            wpos.append(t % ps)
        rows = np.asarray(qo[1:], np.int32) - 1
        cat = lambda xs: np.concatenate(xs).astype(np.int32) if xs else np.zeros(0, np.int32)
        d_ids, d_pos, d_wp, d_wpos, d_rows = self._to_device(
            [cat(ids), cat(pos), cat(wpage), cat(wpos), rows])
        self.attn.plan_levels([dict(qo_indptr=qo, kv_indptr=kvp, kv_indices=pages_all,
                                    kv_last_page_len=last)], qo[-1], causal=True)
        logits = self.model.forward(d_ids.long(), d_pos, self.page_table, d_wp, d_wpos, self.attn,
                                    logits_rows=d_rows.long())
        return logits

    def _tree_page_plan(self, v, r2t, n):
        """(info, plan) of the vnodes as a page-list plan, or None."""
        from .fasttree import build_tree_page_plan
        if not self.tree_pages:
            return None
        m = self.model
        got = build_tree_page_plan(v, np.ascontiguousarray(r2t, np.int32).reshape(-1), n,
                                   self.page_table.page_size, m.Hq, m.Hkv, self.attn.plan.num_sms)
        if got is None or got[0].max_wide_tokens > UMMA_MAX_TOKENS:
            return None
        return got

    def _tree_vnodes(self, state: BeamState, n: int):
        from .fasttree import plan_vnodes
        par, seql, kids, rptr, rl, r2t = state.tree_arrays(per_node=True, compress=True)
        v = plan_vnodes(par, seql, kids, rptr, np.ascontiguousarray(rl) if len(rl) else
                        np.zeros(1, np.int32), r2t.shape[1], n, self.model.Hq_total,
                        self.model.Hkv_total)
        return v, r2t

    def pick_kernel(self, state: BeamState) -> str:
        """kernel_type "auto": cascade or tree attention for this step (picker.py)."""
        from .cascade import cascade_plan_host
        from .fasttree import build_tree_plan
        from .picker import choose
        from .picker import cascade_counts_pages_twice
        m, ps = self.model, self.page_table.page_size
        n = len(state.leaves)
        levels = state.cascade_levels()
        if getattr(self, "use_tiles", False) and not cascade_counts_pages_twice(levels):
            # an exact cascade step runs on the beam-tile kernel (picker.py)
            self.picks.append("cascade")
            self._tree_stash = None
            return "cascade"
        cinfo, _ = cascade_plan_host(levels, n, ps, m.Hq, m.Hkv, causal=True,
                                     num_sms=self.attn.plan.num_sms)
        v, r2t = self._tree_vnodes(state, n)
        pp = self._tree_page_plan(v, r2t, n)
        tinfo, tplan = (pp[0], None) if pp is not None else build_tree_plan(v, n, ps, m.Hq, m.Hkv)
        elt = 4 if self.page_table.store_dtype == torch.float32 else 2
        kind = choose(levels, cinfo, tinfo, m.Hkv, m.Hq, m.D, elt=elt, tree_pages=pp is not None)
        self.picks.append(kind)
        self._tree_stash = (v, r2t, tinfo, tplan, pp) if kind == "fasttree" else None
        return kind

    def _tree_graph_step(self, state: BeamState, k: int, temperature: float):
        """A tree-attention decode step replayed from its own CUDA graph."""
        from .fasttree import build_tree_plan
        m = self.model
        n = len(state.leaves)
        q, wp, wpos, pos = state.step_inputs()
        if self._tree_stash is not None:
            v, r2t, info, plan, pp = self._tree_stash
            self._tree_stash = None
        else:
            v, r2t = self._tree_vnodes(state, n)
            pp = self._tree_page_plan(v, r2t, n)
            info = plan = None
        if pp is not None:
            return self._tree_pages_graph_step(state, n, k, temperature, q, pos, wp, wpos, *pp)
        if plan is None:
            info, plan = build_tree_plan(v, n, self.page_table.page_size, m.Hq, m.Hkv)
        slots = np.concatenate([r2t.reshape(-1), np.full(256, -1, np.int32)])
        sg = self.step_graph_tree
        if not (sg is not None and sg.fits(n, k, temperature, info, len(slots))):
            caps = dict(work=3 * info.n_work + 2 * n + 64, wide=2 * info.n_work_wide + 16,
                        merge=max(n, 1), parts=3 * info.n_parts + 4 * n + 256,
                        ints=3 * info.total_ints + 64 * n + 4096,
                        slots=2 * len(slots) + 64 * n + 4096)
            if sg is not None and sg.n == n and sg.k == k and sg.temp == temperature:
                for key in caps:
                    caps[key] = max(caps[key], sg.caps[key] * 3 // 2)
            self.step_graph_tree = sg = StepGraph(self, n, k, temperature, caps, kind="fasttree")
        if self.plan_hook is not None:
            self.plan_hook(n, info)
        h = sg.host_buf.numpy()
        h[0:n], h[n:2 * n], h[2 * n:3 * n], h[3 * n:4 * n] = q, pos, wp, wpos
        self._take_fork(sg)
        h[sg.plan_off:sg.plan_off + info.total_ints] = plan[:info.total_ints]
        h[sg.slots_off:sg.slots_off + len(slots)] = slots
        return sg.step_filled(sg.slots_off + len(slots))

    def _tree_pages_graph_step(self, state, n, k, temperature, q, pos, wp, wpos, info, plan):
        """A tree step whose plan is a page list: replayed from a page-list step graph."""
        sg = self.step_graph_tpages
        if not (sg is not None and sg.fits(n, k, temperature, info)):
            caps = dict(work=3 * info.n_work + 2 * n + 64, wide=2 * info.n_work_wide + 16,
                        merge=max(n, 1), parts=3 * info.n_parts + 4 * n + 256,
                        ints=3 * info.total_ints + 64 * n + 4096)
            if sg is not None and sg.n == n and sg.k == k and sg.temp == temperature:
                for key in caps:
                    caps[key] = max(caps[key], sg.caps[key] * 3 // 2)
            self.step_graph_tpages = sg = StepGraph(self, n, k, temperature, caps, kind="cascade")
        if self.plan_hook is not None:
            self.plan_hook(n, info)
        h = sg.host_buf.numpy()
        h[0:n], h[n:2 * n], h[2 * n:3 * n], h[3 * n:4 * n] = q, pos, wp, wpos
        self._take_fork(sg)
        h[sg.plan_off:sg.plan_off + info.total_ints] = plan[:info.total_ints]
        return sg.step_filled(sg.plan_off + info.total_ints)

    def decode_step(self, state: BeamState, kind: Optional[str] = None):
        """One beam step's forward: returns logits [beams, vocab]."""
        if kind is None:
            kind = self.pick_kernel(state) if self.kernel_type == "auto" else self.kernel_type
        self._flush_fork()
        q, wp, wpos, pos = state.step_inputs()
        if kind == "cascade":
            levels = state.cascade_levels()
            self.attn.plan_levels(levels, len(q), causal=True)
        else:
            v, r2t = self._tree_vnodes(state, len(q))
            flat = np.concatenate([r2t.reshape(-1), np.full(256, -1, np.int32)])
            pp = self._tree_page_plan(v, r2t, len(q))
            if pp is not None:              # page-list tree plan on the tensor-core kernels
                self.attn.plan_prebuilt(*pp)
                kind = "cascade"
        arrays = [q, pos, wp, wpos]
        if kind != "cascade":
            arrays.append(_i32(flat))
        dev = self._to_device(arrays)
        if kind != "cascade":
            self.attn.plan_tree(v, len(q), dev[4])
        return self.model.forward(dev[0].long(), dev[1], self.page_table, dev[2], dev[3], self.attn)

    def decode_topk(self, state: BeamState, k: int, temperature: float):
        """One decode step through to the host: (log-prob top-k [beams, k], ids)."""
        kind = self.pick_kernel(state) if self.kernel_type == "auto" else self.kernel_type
        if kind == "fasttree" and self.use_graph_tree:
            return self._tree_graph_step(state, k, temperature)
        self._tree_stash = None
        if not self.use_graph or kind != "cascade":
            return self._topk(self.decode_step(state, kind), k, temperature)
        if self.use_tiles:
            got = self._tiles_graph_step(state, k, temperature)
            if got is not None:
                return got
        m = self.model
        n = len(state.leaves)
        leaves = np.ascontiguousarray(state.leaves, np.int32)
        info = _lib.AttnPlanInfo()
        sg = self.step_graph

        def fill(buf_ptr, cap, plan_off):
            rc = lib().be_beam_decode_inputs(self.page_table._trie, n, _lib.addr(leaves), m.Hq,
                                             m.Hkv, self.attn.plan.num_sms, C.c_void_p(buf_ptr),
                                             cap, plan_off, C.byref(info))
            if rc not in (_lib.BE_OK, _lib.BE_ECAPACITY):
                check(rc, "be_beam_decode_inputs")
            return rc == _lib.BE_OK

        if not (sg is not None and sg.n == n and sg.k == k and sg.temp == temperature
                and fill(sg.host_buf.data_ptr(), sg.total, sg.plan_off)
                and sg.fits(n, k, temperature, info)):
            # size a new graph from this step's plan (grow the probe buffer until it fits)
            off = step_plan_offset(n)
            size = off + 65536
            while True:
                probe = np.empty(size, np.int32)
                if fill(probe.ctypes.data, size, off):
                    break
                size *= 4
            if info.max_wide_tokens > UMMA_MAX_TOKENS:   # outside the fixed kernels' range
                return self._topk(self.decode_step(state, "cascade"), k, temperature)
            # headroom: the suffix items (and their partial rows) keep growing with the
            # beams' suffixes; the shared-prefix items hardly do.  Surplus suffix CTAs exit
            # at once on the side stream, a re-record costs tens of ms (more under TP)
            # (the first decode step has no suffix items yet: allow ~2 per beam)
            caps = dict(work=3 * info.n_work + 2 * n + 64, wide=2 * info.n_work_wide + 16,
                        merge=max(n, 1), parts=3 * info.n_parts + 4 * n + 256,
                        ints=3 * info.total_ints + 64 * n + 4096)
            if sg is not None and sg.n == n and sg.k == k and sg.temp == temperature:
                # outgrown: the plan keeps growing with the suffixes, leave more room
                got = dict(work=info.n_work, wide=info.n_work_wide, merge=info.n_merge,
                           parts=info.n_parts, ints=info.total_ints)
                self.graph_regrowth.append({key: (got[key], sg.caps[key]) for key in got
                                            if got[key] > sg.caps[key]})
                for key in caps:
                    caps[key] = max(caps[key], sg.caps[key] * 3 // 2)
            elif sg is not None:
                self.graph_regrowth.append({"shape": (sg.n, n, sg.k, k)})
            self.step_graph = sg = StepGraph(self, n, k, temperature, caps)
            if not fill(sg.host_buf.data_ptr(), sg.total, sg.plan_off):
                raise RuntimeError("decode step graph sized too small for its own plan")
        if self.plan_hook is not None:
            self.plan_hook(n, info)
        self._take_fork(sg)
        return sg.step_filled(sg.plan_off + info.total_ints)

    def _tiles_graph_step(self, state: BeamState, k: int, temperature: float):
        """A cascade decode step on the beam-tile kernel, replayed from its graph.
        None when the step's plan is not a decode shape (the caller plans work items)."""
        m = self.model
        n = len(state.leaves)
        leaves = np.ascontiguousarray(state.leaves, np.int32)
        info = _lib.TilePlanInfo()
        rows = tile_rows_for(self._beam_width * (m.Hq // m.Hkv))
        tp = target_pieces(self.attn.plan.num_sms, m.Hkv)
        sg = self.step_graph_tiles

        want_sel = None
        if self._sel_ctx is not None:
            seg, W, div = self._sel_ctx
            want_sel = (len(seg) - 1, W, div)
        have_sel = (None if sg is None or sg.select is None else
                    (sg.select[0], sg.select[1], sg.select[3]))
        same = (sg is not None and sg.n == n and sg.k == k and sg.temp == temperature
                and have_sel == want_sel
                and (want_sel is None or int(np.max(np.diff(self._sel_ctx[0]))) <= sg.select[2]))

        def fill(buf_ptr, cap, plan_off, cluster):
            rc = lib().be_beam_decode_tiles(self.page_table._trie, n, _lib.addr(leaves), m.Hq,
                                            m.Hkv, rows, tp, cluster, C.c_void_p(buf_ptr), cap,
                                            plan_off, C.byref(info))
            if rc == _lib.BE_ENOTSUP:
                return None
            if rc not in (_lib.BE_OK, _lib.BE_ECAPACITY):
                check(rc, "be_beam_decode_tiles")
            return rc == _lib.BE_OK

        # the graph's cluster size is part of its recorded launch: keep it while the
        # shape stays (the planner chooses it for a new graph)
        ok = same and fill(sg.host_buf.data_ptr(), sg.total, sg.plan_off, sg.caps["cluster"])
        if ok is None:
            return None
        if not (ok and sg.fits(n, k, temperature, info)):
            off = step_plan_offset(n)
            size = off + 65536
            # BE_ATTN_CLUSTER: cluster size of new step graphs (-1: the planner's
            # choice, 0: the merge kernel, 2..16)
            cl = sg.caps["cluster"] if same else int(os.environ.get("BE_ATTN_CLUSTER", "-1"))
            while True:
                probe = np.empty(size, np.int32)
                got = fill(probe.ctypes.data, size, off, cl)
                if got is None:
                    return None
                if got:
                    break
                size *= 4
            # headroom: entries grow with the beams' suffixes; pieces and tiles hardly change
            cl = info.cluster
            sel = None
            if self._sel_ctx is not None:
                seg, W, div = self._sel_ctx
                sel = (len(seg) - 1, W, int(np.max(np.diff(seg))), div)
            if cl > 1:   # one cluster per (tile, KV head): pieces = tiles x cluster
                caps = dict(pieces=info.n_pieces, tiles=info.n_tiles, part_pieces=0,
                            ints=3 * info.total_ints + 64 * n + 4096, rows=info.tile_rows,
                            cluster=cl)
            else:
                caps = dict(pieces=info.n_pieces + 2 * info.n_tiles + tp // 4 + 16,
                            tiles=2 * info.n_tiles + 8,
                            part_pieces=info.n_pieces + 2 * info.n_tiles + tp // 4 + 16,
                            ints=3 * info.total_ints + 64 * n + 4096, rows=info.tile_rows,
                            cluster=0)
            caps["select"] = sel
            # the kernel reads piece records up to max_pieces before the piece count
            caps["ints"] = max(caps["ints"], 32 + 24 * caps["pieces"] + 64)
            if sg is not None and sg.n == n and sg.k == k and sg.temp == temperature:
                got = dict(pieces=info.n_pieces, tiles=info.n_tiles,
                           part_pieces=info.n_part_pieces, ints=info.total_ints)
                self.graph_regrowth.append({key: (got[key], sg.caps[key]) for key in got
                                            if got[key] > sg.caps[key]})
                for key in ("pieces", "tiles", "part_pieces", "ints"):
                    if cl <= 1 or key == "ints":
                        caps[key] = max(caps[key], sg.caps[key] * 3 // 2)
                caps["ints"] = max(caps["ints"], 32 + 24 * caps["pieces"] + 64)
            elif sg is not None:
                self.graph_regrowth.append({"shape": (sg.n, n, sg.k, k)})
            self.step_graph_tiles = sg = StepGraph(self, n, k, temperature, caps, kind="tiles")
            if not fill(sg.host_buf.data_ptr(), sg.total, sg.plan_off, cl):
                raise RuntimeError("decode step graph sized too small for its own plan")
        if self.plan_hook is not None:
            self.plan_hook(n, info)
        self._take_fork(sg)
        if sg.select is not None:
            seg, W, div = self._sel_ctx
            sg.set_selection_inputs(seg, state.scores,
                                    state.leaf_sequences()[0] if div is not None else None)
        return sg.step_filled(sg.plan_off + info.total_ints)

    def generate_ids(self, prompts: List[List[int]], beam_size: int = 4,
                     max_length: Optional[int] = None, max_new_tokens: Optional[int] = None,
                     num_return_sequences: int = 1, temperature: float = 1.0, on_step=None):
        """Beam search over several prompts at once.  ``max_length`` is per-prompt
        total length as in the reference (new tokens = max_length - len(prompt));
        ``max_new_tokens`` sets the same for every prompt.  Returns, per prompt,
        the ranked [(tokens, score)] list.  ``on_step(i)`` (optional) is called
        before decode step i and once more with the step count after the last."""
        if max_new_tokens is None:
            if max_length is None:
                raise ValueError("give max_length or max_new_tokens")
            steps_left = [max_length - len(p) - 1 for p in prompts]
            if len(set(steps_left)) != 1:
                raise ValueError("prompts of different lengths need max_new_tokens")
            n_steps = steps_left[0]
        else:
            n_steps = max_new_tokens - 1
        W = beam_size
        self._beam_width = W
        self._pending_fork = None    # copies left by an interrupted earlier call are void
        state = BeamState(W, self.page_table)
        state.defer_copies = True
        V = self.model.vocab
        with torch.no_grad():
            with _Range("prefill"):
                logits = self.prefill(state, prompts)
            k0 = min(2 * W, V)
            vals, idx = self._topk(logits, k0, temperature)
            kw = min(W, k0)
            ptr = np.arange(len(prompts) + 1, dtype=np.int32) * kw
            self._apply(state, ptr, idx[:, :kw].reshape(-1), vals[:, :kw].reshape(-1))
            seg = np.arange(len(prompts) + 1) * kw          # candidates per prompt
            for step in range(n_steps):
                if self.strategy.should_stop(state, 10 ** 9, step):
                    break
                if on_step is not None:
                    on_step(step)
                k = min(2 * W, V) if W != 1 else 1
                vanilla = type(self.strategy) is VanillaBeamSearchStrategy
                div = self._device_diverse_params(W)
                self._sel_ctx = ((np.asarray(seg, np.int32), W, div)
                                 if (vanilla or div is not None)
                                 and getattr(self, "device_select", False) and k <= 64
                                 and int(np.max(np.diff(seg))) * k <= 8192 else None)
                with _Range("decode_step"):
                    res = self.decode_topk(state, k, temperature)
                self._sel_ctx = None
                with _Range("select"):
                    if isinstance(res, DiverseSelection):
                        self._apply(state, res.child_ptr, res.tokens, res.scores)
                        seg = np.asarray(res.new_seg)
                        continue
                    if isinstance(res, DeviceSelection):
                        new_seg = state.vanilla_step_selected(seg, res.parent, res.token,
                                                              res.score, W)
                        self._after_update(state)
                        seg = np.asarray(new_seg)
                        continue
                    vals, idx = res
                    if vanilla:
                        # selection + trie update in one native call
                        new_seg = state.vanilla_step(seg, idx, vals, W)
                        self._after_update(state)
                    elif getattr(self.strategy, "needs_state", False):
                        cp, ct, cs, new_seg = self.strategy.select_segments(seg, state.scores, idx, vals, W,
                                                                            state=state)
                        self._apply(state, cp, ct, cs)
                    elif hasattr(self.strategy, "select_segments"):
                        cp, ct, cs, new_seg = self.strategy.select_segments(seg, state.scores, idx, vals, W)
                        self._apply(state, cp, ct, cs)
                    else:
                        ptr_all, tok_all, sc_all = [0], [], []
                        new_seg = [0]
                        for p in range(len(prompts)):
                            a, b = seg[p], seg[p + 1]
                            cp, ct, cs = self.strategy.select_arrays(state.scores[a:b], idx[a:b],
                                                                     vals[a:b], W)
                            ptr_all.extend((cp[1:] + len(tok_all)).tolist())
                            tok_all.extend(ct.tolist())
                            sc_all.extend(cs.tolist())
                            new_seg.append(new_seg[-1] + int(cp[-1]))
                        self._apply(state, np.asarray(ptr_all, np.int32), np.asarray(tok_all, np.int32),
                                    np.asarray(sc_all, np.float64))
                seg = np.asarray(new_seg)
            self._flush_fork()
            if getattr(self.model, "comm", None) is not None:
                # a peer exchange whose bounded wait ran out returns without writing
                # its rows: report it instead of returning beams from undefined states
                st = C.c_int(0)
                check(lib().be_device_status(C.byref(st), None), "be_device_status")
                if st.value != 0:
                    raise RuntimeError(
                        f"device status {st.value} during a tensor-parallel generation (a peer "
                        "exchange timed out or a page id was out of range); its beams are undefined")
            if on_step is not None:
                on_step(n_steps)
        out = []
        for p in range(len(prompts)):
            sub = BeamState(W, self.page_table)
            sub.set_state(state.leaves[seg[p]:seg[p + 1]], state.scores[seg[p]:seg[p + 1]])
            out.append(self.strategy.get_final_sequences(sub, num_return_sequences))
        self.last_state = state
        return out

    def _device_diverse_params(self, W):
        """(num_groups, diversity_penalty, length_penalty) when this step's
        diverse selection can run on the device (hamming penalty, within
        be_diverse_select_device's pick limit), else None."""
        from .beam_strategy import _DIVERSITY_TYPES, DiverseBeamSearchStrategy
        st = self.strategy
        if type(st) is not DiverseBeamSearchStrategy or _DIVERSITY_TYPES.get(st.diversity_type, 1):
            return None
        groups = int(st.num_groups)
        if groups < 1 or groups * max(1, W // groups) > 1024:
            return None
        return (groups, float(st.diversity_penalty), float(st.length_penalty))

    def _apply(self, state, child_ptr, child_tokens, child_scores):
        state.update_native(state.leaves, child_ptr, child_tokens, child_scores)
        self._after_update(state)

    def _after_update(self, state):
        """Hand the update's copy-on-write copies to the next step (or run them)."""
        self._flush_fork()
        cs, cd, cl = state.last_copies
        if len(cs):
            if self.use_graph or self.use_graph_tree:
                self._pending_fork = (cs, cd, cl)   # the next step graph's first launch
            else:
                self._fork_now((cs, cd, cl))

    def _fork_now(self, copies):
        cs, cd, cl = copies
        d = self._to_device([cs, cd, cl])
        pt = self.page_table
        check(lib().be_fork_tail_copy(pt.kv_cache.data_ptr(), pt.kv_cache.stride(0),
                                      pt.layer_num, pt.max_num_pages, pt.page_size,
                                      pt.head_num, pt.head_dim, _pool_dtype(pt),
                                      d[0].data_ptr(), d[1].data_ptr(), d[2].data_ptr(), len(cs),
                                      stream_ptr(self.device)), "fork")

    def _flush_fork(self):
        """Run pending copy-on-write copies now (a path without a step graph)."""
        if self._pending_fork is not None:
            copies, self._pending_fork = self._pending_fork, None
            self._fork_now(copies)

    def _take_fork(self, sg):
        """Hand the pending copies to the step graph about to replay."""
        copies, self._pending_fork = self._pending_fork, None
        if copies is not None and len(copies[0]) > sg.n:   # more than the list holds
            self._fork_now(copies)
            copies = None
        sg.set_fork(copies)
