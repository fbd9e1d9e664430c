"""Llama decoder for beam decode on the paged KV cache (the reference's patched HF
Llama, ``src/beam_engine/models/modeling_llama.py``), B200 layout.

Per layer: fused residual-add + RMSNorm -> one QKV GEMM -> fused RoPE + K/V
append into the pages -> paged attention (cascade / prefill / tree plan) ->
O GEMM -> fused add + RMSNorm -> one gate|up GEMM -> SiLU*up -> down GEMM.
GEMMs run on cuBLASLt through ``be_gemm_lt`` (pre-fused weights, the fastest
of cuBLASLt's candidates timed once per shape; BE_GEMM=0 selects torch.mm);
BE_GEMM=1 routes the ones with at most 128 rows to ``be_gemm_tn``, the
library's weight-streaming tcgen05 GEMM (correct, not yet faster than cuBLAS
on these shapes).  Every other op is a kernel of ``libbeam_b200.so``.  Tensor parallelism (``tp``) shards q/k/v heads, the
O-projection rows, gate/up columns and down rows, with one all-reduce after
the O and down projections.
"""
from __future__ import annotations

import ctypes as C
import os
from typing import Optional

import torch

from . import _lib

from ._lib import check, lib
from .page_table import dtype_code, stream_ptr
from .weights import iter_random_llama_weights


def inv_freq_table(head_dim, theta, device):
    """HF default RoPE inverse frequencies (float32), modeling_llama.py:89-110."""
    return (1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
            ).to(device)


class BeamLlama:
    def __init__(self, cfg: dict, weights: Optional[dict] = None, dtype=torch.bfloat16,
                 device="cuda", seed=0, tp=None):
        self.config = dict(cfg)
        self.device = torch.device(device)
        self.dtype = dtype
        self.tp = tp
        ts, tr = (tp.size, tp.rank) if tp is not None else (1, 0)
        c = self.config
        self.L = c["num_hidden_layers"]
        self.D = c["head_dim"]
        self.Hq_total, self.Hkv_total = c["num_attention_heads"], c["num_key_value_heads"]
        if self.Hq_total % ts or self.Hkv_total % ts or c["intermediate_size"] % ts:
            raise ValueError(f"heads / ffn not divisible by tensor-parallel size {ts}")
        self.Hq, self.Hkv = self.Hq_total // ts, self.Hkv_total // ts
        self.F = c["intermediate_size"] // ts
        self.H = c["hidden_size"]
        self.eps = float(c["rms_norm_eps"])
        self.vocab = c["vocab_size"]
        D, Hq, Hkv, F = self.D, self.Hq, self.Hkv, self.F

        def shard_rows(w, n_per, idx):   # output-feature shard
            return w[idx * n_per:(idx + 1) * n_per]

        def prep(t):
            return t.to(device=self.device, dtype=dtype).contiguous()

        # vocab-parallel lm_head under TP (each rank scores its vocabulary slice)
        V = self.vocab
        self.v0, self.v1 = (tr * V) // ts, ((tr + 1) * V) // ts

        def shard(name, w):
            """This rank's part of one tensor, in storage of its own (a view would keep
            the full tensor alive)."""
            x = _shard(name, w)
            if x.untyped_storage().nbytes() > x.numel() * x.element_size():
                x = x.clone()
            return x

        def _shard(name, w):
            m = name.rsplit(".", 1)[-1]
            if m == "q":
                return prep(shard_rows(w, Hq * D, tr))
            if m in ("k", "v"):
                return prep(shard_rows(w, Hkv * D, tr))
            if m == "o":
                return prep(w[:, tr * Hq * D:(tr + 1) * Hq * D])
            if m in ("gate", "up"):
                return prep(shard_rows(w, F, tr))
            if m == "down":
                return prep(w[:, tr * F:(tr + 1) * F])
            if name == "lm_head":
                return prep(w[self.v0:self.v1])
            return prep(w)

        # random init streams one tensor at a time (never the whole model on a rank)
        items = (weights.items() if weights is not None else
                 iter_random_llama_weights(c, seed=seed, dtype=dtype, device=self.device))
        parts = {}
        for name, w in items:
            parts[name] = shard(name, w)
            del w
        self.w_qkv, self.w_o, self.w_gu, self.w_down, self.n_in, self.n_post = [], [], [], [], [], []
        for i in range(self.L):
            p = f"layers.{i}."
            self.w_qkv.append(torch.cat([parts.pop(p + "q"), parts.pop(p + "k"),
                                         parts.pop(p + "v")], 0).contiguous())
            self.w_o.append(parts.pop(p + "o"))
            self.w_gu.append(torch.cat([parts.pop(p + "gate"), parts.pop(p + "up")], 0).contiguous())
            self.w_down.append(parts.pop(p + "down"))
            self.n_in.append(parts.pop(p + "input_norm"))
            self.n_post.append(parts.pop(p + "post_norm"))
        self.embed = parts.pop("embed")
        self.norm = parts.pop("norm")
        self.lm_head = parts.pop("lm_head")
        self.inv_freq = inv_freq_table(D, float(c["rope_theta"]), self.device)
        self.dt = dtype_code(dtype)
        self.qkv_width = (Hq + 2 * Hkv) * D
        mode = os.environ.get("BE_GEMM", "lt")
        cuda_bf16 = dtype == torch.bfloat16 and self.device.type == "cuda"
        self.use_gemm = mode == "1" and cuda_bf16          # tcgen05 weight-streaming GEMM
        self.use_lt = mode == "lt" and cuda_bf16           # cuBLASLt, per-shape tuned
        self._gemm_ws = None
        self._lt_ws = None
        self.comm = None          # PeerAllReduce: fused all-reduce + add + RMSNorm under TP
        self._slot_views = {}
        del weights

    def enable_peer_allreduce(self, max_rows: int = 512):
        """Route the row-parallel all-reduces of forwards with <= max_rows rows
        through ``be_comm_allreduce_rmsnorm`` (peer memory, fused with the
        residual add and the next RMSNorm) instead of NCCL + add_rmsnorm."""
        from .parallel import PeerAllReduce
        if self.tp is None or self.tp.size < 2:
            return None
        elt = torch.empty(0, dtype=self.dtype).element_size()
        self.comm = PeerAllReduce(self.tp, max_rows * self.H * elt, self.device)
        return self.comm

    def _slots(self, n):
        v = self._slot_views.get(n)
        if v is None:
            v = self._slot_views[n] = [self.comm.slot_view(i, (n, self.H), self.dtype)
                                       for i in (0, 1)]
        return v

    def _mm(self, a: torch.Tensor, w: torch.Tensor, out: torch.Tensor):
        """out = a @ w.T (a [T, K], w [N, K] row-major, out [T, N])."""
        T, K = a.shape
        N = w.shape[0]
        if (self.use_gemm and T <= 128 and N >= 128 and K % 64 == 0 and a.stride(1) == 1
                and a.stride(0) % 8 == 0 and w.is_contiguous() and out.stride(1) == 1
                and out.dtype in (torch.bfloat16, torch.float32)):
            if self._gemm_ws is None:   # split-K partials: 8 M floats (32 MB)
                self._gemm_ws = torch.empty(8 << 20, dtype=torch.float32, device=self.device)
            check(lib().be_gemm_tn(a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0),
                                   out.data_ptr(), out.stride(0), T, N, K,
                                   _lib.BE_BF16 if out.dtype == torch.bfloat16 else _lib.BE_F32,
                                   0, self._gemm_ws.data_ptr(), self._gemm_ws.numel(),
                                   stream_ptr(self.device)), "be_gemm_tn")
            return out
        if (self.use_lt and a.stride(1) == 1 and w.is_contiguous() and out.stride(1) == 1
                and out.dtype in (torch.bfloat16, torch.float32)):
            if self._lt_ws is None:   # split-K scratch for cuBLASLt
                self._lt_ws = torch.empty(32 << 20, dtype=torch.uint8, device=self.device)
            check(lib().be_gemm_lt(a.data_ptr(), a.stride(0), w.data_ptr(), w.stride(0),
                                   out.data_ptr(), out.stride(0), T, N, K,
                                   _lib.BE_BF16 if out.dtype == torch.bfloat16 else _lib.BE_F32,
                                   self._lt_ws.data_ptr(), self._lt_ws.numel(),
                                   stream_ptr(self.device)), "be_gemm_lt")
            return out
        if out.dtype == a.dtype:
            return torch.mm(a, w.t(), out=out)
        out.copy_(torch.mm(a, w.t()))
        return out

    def parameters(self):
        yield self.embed

    # ------------------------------------------------------------------
    def forward(self, ids: torch.Tensor, positions: torch.Tensor, page_table, write_pages,
                write_pos, attention, logits_rows: Optional[torch.Tensor] = None,
                layer_hook=None) -> torch.Tensor:
        """ids [n] (device), positions/write_pages/write_pos [n] int32 (device).
        attention.run(layer, qkv, out) computes paged attention for one layer.
        Returns logits [len(logits_rows) or n, vocab slice] in float32."""
        n = ids.shape[0]
        dev, dt = self.device, self.dtype
        st = stream_ptr(dev)
        L = lib()
        x = self.embed.index_select(0, ids)                     # residual stream [n, H]
        h = torch.empty_like(x)
        qkv = torch.empty((n, self.qkv_width), dtype=dt, device=dev)
        att = torch.empty((n, self.Hq * self.D), dtype=dt, device=dev)
        gu = torch.empty((n, 2 * self.F), dtype=dt, device=dev)
        act = torch.empty((n, self.F), dtype=dt, device=dev)
        delta = torch.empty_like(x)
        pool = page_table.kv_cache
        P, ps = page_table.max_num_pages, page_table.page_size
        have_delta = False
        # fused peer all-reduce: the O / down GEMMs write into this rank's slots and
        # one kernel sums the ranks' slots, adds the residual and applies the next norm
        fused = self.comm is not None and self.comm.fits(n, self.H, x.element_size())
        slots = self._slots(n) if fused else None
        for i in range(self.L):
            if not fused or i == 0:
                check(L.be_add_rmsnorm(x.data_ptr(), delta.data_ptr() if have_delta else None,
                                       self.n_in[i].data_ptr(), h.data_ptr(), n, self.H, self.eps,
                                       self.dt, st), "add_rmsnorm")
            self._mm(h, self.w_qkv[i], qkv)
            check(L.be_rope_qkv_append(qkv.data_ptr(), self.qkv_width, n, self.Hq, self.Hkv, self.D,
                                       positions.data_ptr(), self.inv_freq.data_ptr(),
                                       pool[i].data_ptr(), P, ps, write_pages.data_ptr(),
                                       write_pos.data_ptr(), 0, self.dt, st), "rope_append")
            attention.run(i, qkv, att)
            if layer_hook is not None:
                layer_hook(i)
            if fused:
                self._mm(att, self.w_o[i], slots[0])
                check(L.be_comm_allreduce_rmsnorm(self.comm.ptr, 0, x.data_ptr(),
                                                  self.n_post[i].data_ptr(), h.data_ptr(), n,
                                                  self.H, self.eps, self.dt, st), "allreduce o")
            else:
                self._mm(att, self.w_o[i], delta)
                self._all_reduce(delta)
                check(L.be_add_rmsnorm(x.data_ptr(), delta.data_ptr(), self.n_post[i].data_ptr(),
                                       h.data_ptr(), n, self.H, self.eps, self.dt, st), "add_rmsnorm")
            self._mm(h, self.w_gu[i], gu)
            check(L.be_silu_mul(gu.data_ptr(), act.data_ptr(), n, self.F, self.dt, st), "silu_mul")
            if fused:
                nxt = self.n_in[i + 1] if i + 1 < self.L else self.norm
                self._mm(act, self.w_down[i], slots[1])
                check(L.be_comm_allreduce_rmsnorm(self.comm.ptr, 1, x.data_ptr(), nxt.data_ptr(),
                                                  h.data_ptr(), n, self.H, self.eps, self.dt, st),
                      "allreduce down")
            else:
                self._mm(act, self.w_down[i], delta)
                self._all_reduce(delta)
            have_delta = True
        if not fused:
            check(L.be_add_rmsnorm(x.data_ptr(), delta.data_ptr(), self.norm.data_ptr(),
                                   h.data_ptr(), n, self.H, self.eps, self.dt, st), "final norm")
        hs = h if logits_rows is None else h.index_select(0, logits_rows)
        logits = torch.empty((hs.shape[0], self.lm_head.shape[0]), dtype=torch.float32, device=dev)
        return self._mm(hs, self.lm_head, logits)

    def _all_reduce(self, t):
        if self.tp is not None and self.tp.size > 1:
            self.tp.all_reduce(t)
