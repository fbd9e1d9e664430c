"""Import the unmodified reference engine on a CPU-only container.

Used only by ``make_golden.py`` in the build container (the reference source
tree is not present on GPU boxes).  Everything here is a run-time shim around
the reference, never an edit of it:

* transformers 5.5 vs the pinned 4.57.3: ``check_model_inputs`` must work as
  ``@check_model_inputs()``, ``ROPE_INIT_FUNCTIONS['default']`` is gone (and
  5.5's weight init asks the rotary module for
  ``compute_default_rope_parameters``), and
  ``create_causal_mask`` renamed a keyword (the FlashInfer paths ignore the
  mask, so it is stubbed to ``None``);
* FlashInfer is CUDA-only, so ``flashinfer.page.append_paged_kv_cache``,
  ``flashinfer.cascade.MultiLevelCascadeAttentionWrapper`` and
  ``flashinfer.BatchPrefillWithPagedKVCacheWrapper`` are replaced by CPU
  restatements (the oracle's) with FlashInfer's published semantics.
"""
from __future__ import annotations

import os
import sys
import types

import numpy as np
import torch

# the reference checkout's ``src`` directory (BEAM_REF_SRC); a sibling
# ``reference`` checkout of this repository's parent directory by default
REF_SRC = os.environ.get(
    "BEAM_REF_SRC",
    os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.dirname(
        os.path.abspath(__file__))))), "reference", "src"))


def _np(t):
    return t.detach().cpu().double().numpy()


def default_rope(config, device=None, **_):
    """HF's default RoPE init: inv_freq = theta^(-2i/D), attention scaling 1."""
    d = getattr(config, "head_dim", None) or config.hidden_size // config.num_attention_heads
    base = getattr(config, "rope_theta", 10000.0)
    inv = 1.0 / (base ** (torch.arange(0, d, 2, dtype=torch.int64).float() / d))
    return inv, 1.0


def install():
    if REF_SRC not in sys.path:
        sys.path.insert(0, REF_SRC)
    here = os.path.dirname(os.path.abspath(__file__))
    repo = os.path.dirname(os.path.dirname(here))
    if repo not in sys.path:
        sys.path.insert(0, repo)
    from oracle import attention as oatt

    import transformers.utils.generic as gen
    gen.check_model_inputs = lambda *a, **k: (lambda f: f)
    import transformers.masking_utils as mu
    mu.create_causal_mask = lambda *a, **k: None
    from transformers.modeling_rope_utils import ROPE_INIT_FUNCTIONS

    ROPE_INIT_FUNCTIONS["default"] = default_rope

    fi = types.ModuleType("flashinfer")
    page = types.ModuleType("flashinfer.page")
    casc = types.ModuleType("flashinfer.cascade")

    def append_paged_kv_cache(append_key, append_value, batch_indices, positions, paged_kv_cache,
                              kv_indices, kv_indptr, kv_last_page_len, kv_layout="NHD"):
        ps = paged_kv_cache.shape[2]
        for i in range(append_key.shape[0]):
            b = int(batch_indices[i])
            pos = int(positions[i])
            pg = int(kv_indices[int(kv_indptr[b]) + pos // ps])
            paged_kv_cache[pg, 0, pos % ps] = append_key[i]
            paged_kv_cache[pg, 1, pos % ps] = append_value[i]

    class MultiLevelCascadeAttentionWrapper:
        def __init__(self, num_levels, workspace, kv_layout="NHD"):
            self.num_levels = num_levels

        def plan(self, qo_indptr_arr, paged_kv_indptr_arr, paged_kv_indices_arr,
                 paged_kv_last_page_len, num_qo_heads, num_kv_heads, head_dim, page_size,
                 causal=True, pos_encoding_mode="NONE", sm_scale=None, q_data_type=None, **_):
            self.levels = [dict(qo_indptr=a.tolist(), kv_indptr=b.tolist(), kv_indices=c.tolist(),
                                kv_last_page_len=d.tolist())
                           for a, b, c, d in zip(qo_indptr_arr, paged_kv_indptr_arr,
                                                 paged_kv_indices_arr, paged_kv_last_page_len)]
            self.ps = page_size
            self.scale = sm_scale if sm_scale is not None else head_dim ** -0.5

        def run(self, q, kv):
            o = oatt.cascade_attention(_np(q), _np(kv), self.levels, self.ps, self.scale)
            return torch.from_numpy(o).to(q.dtype)

    class BatchPrefillWithPagedKVCacheWrapper:
        def __init__(self, workspace, kv_layout="NHD"):
            pass

        def plan(self, qo_indptr, paged_kv_indptr, paged_kv_indices, paged_kv_last_page_len,
                 num_qo_heads, num_kv_heads, head_dim_qk, page_size, causal=True, **_):
            self.pages = paged_kv_indices.tolist()
            self.last = int(paged_kv_last_page_len[0])
            self.ps = page_size
            self.scale = head_dim_qk ** -0.5

        def run(self, q, kv):
            o = oatt.paged_prefill(_np(q), _np(kv), self.pages, self.last, self.ps, self.scale)
            return torch.from_numpy(o).to(q.dtype)

    page.append_paged_kv_cache = append_paged_kv_cache
    casc.MultiLevelCascadeAttentionWrapper = MultiLevelCascadeAttentionWrapper
    fi.page = page
    fi.cascade = casc
    fi.BatchPrefillWithPagedKVCacheWrapper = BatchPrefillWithPagedKVCacheWrapper
    sys.modules["flashinfer"] = fi
    sys.modules["flashinfer.page"] = page
    sys.modules["flashinfer.cascade"] = casc
