"""Oracle: numpy Llama decoder and beam-search loop (test infrastructure).

Restates the reference's model runner and engine for the cascade path:
  * ``LlamaRMSNorm`` (modeling_llama.py:68-86): ``w * (x * rsqrt(mean(x^2) + eps))``;
  * RoPE as HF's default rotary embedding (modeling_llama.py:89-157);
  * ``LlamaAttention.forward`` (modeling_llama.py:428-562): q/k/v projections,
    RoPE, K/V written into the pages BEFORE attention, prefill = causal paged
    attention over the prompt pages, decode = multi-level cascade attention,
    ``o_proj``;
  * SwiGLU MLP (modeling_llama.py:160-173) and the pre-norm residual layer
    (modeling_llama.py:577-621); final norm and ``lm_head``;
  * ``BeamSearchGenerator.generate`` (beam.py:48-352) with the vanilla
    strategy: prefill -> log_softmax -> top-2W -> first W children of the
    root; then ``max_length - len(prompt) - 1`` decode steps of
    cascade metadata -> forward -> log_softmax -> top-2W per beam ->
    global top-W -> trie update; final ranking with the length penalty.
Weights come in as a dict of numpy float32 arrays (names as in
``random_weight_names``), so the same seeded tensors feed every checker.
"""
from __future__ import annotations

import numpy as np

from .attention import apply_rope, cascade_attention, paged_prefill, rope_cos_sin
from .beam_state import OracleBeamState, vanilla_select
from .paging import OraclePageTable


def rmsnorm(x, w, eps):
    x = x.astype(np.float32)
    var = np.mean(x * x, axis=-1, keepdims=True, dtype=np.float32)
    return (w * (x / np.sqrt(var + np.float32(eps)))).astype(np.float32)


def silu(x):
    return x / (1.0 + np.exp(-x))


def log_softmax(x):
    x = x.astype(np.float64)
    m = x.max(axis=-1, keepdims=True)
    return x - m - np.log(np.exp(x - m).sum(axis=-1, keepdims=True))


class OracleLlama:
    def __init__(self, cfg, weights):
        self.cfg = cfg
        self.w = weights
        self.D = cfg["head_dim"]
        self.Hq = cfg["num_attention_heads"]
        self.Hkv = cfg["num_key_value_heads"]
        self.scale = self.D ** -0.5

    def forward(self, ids, positions, table, mode, write=None, levels=None, prefill=None):
        """ids [n]; returns logits [n, vocab] (float32)."""
        c, w = self.cfg, self.w
        x = w["embed"][np.asarray(ids)].astype(np.float32)
        cos, sin = rope_cos_sin(positions, self.D, c["rope_theta"])
        n = len(ids)
        for li in range(c["num_hidden_layers"]):
            p = f"layers.{li}."
            h = rmsnorm(x, w[p + "input_norm"], c["rms_norm_eps"])
            q = (h @ w[p + "q"].T).reshape(n, self.Hq, self.D)
            k = (h @ w[p + "k"].T).reshape(n, self.Hkv, self.D)
            v = (h @ w[p + "v"].T).reshape(n, self.Hkv, self.D)
            q = apply_rope(q, cos, sin).astype(np.float32)
            k = apply_rope(k, cos, sin).astype(np.float32)
            if mode == "prefill":
                pages, last = prefill
                ps = table.page_size
                for i, pg in enumerate(pages):
                    seg = slice(i * ps, min(n, (i + 1) * ps))
                    table.write_block(li, pg, k[seg], v[seg], 0)
                a = paged_prefill(q, table.kv[li], pages, last, ps, self.scale)
            else:
                table.append(li, k, v, write[0], write[1])
                a = cascade_attention(q, table.kv[li], levels, table.page_size, self.scale)
            a = a.astype(np.float32).reshape(n, -1)
            x = x + a @ w[p + "o"].T
            h = rmsnorm(x, w[p + "post_norm"], c["rms_norm_eps"])
            m = silu(h @ w[p + "gate"].T) * (h @ w[p + "up"].T)
            x = (x + m.astype(np.float32) @ w[p + "down"].T).astype(np.float32)
        x = rmsnorm(x, w["norm"], c["rms_norm_eps"])
        return (x @ w["lm_head"].T).astype(np.float32)


def topk(row, k):
    """Descending top-k of a 1-D array (ties broken by lower index)."""
    idx = np.argsort(-row, kind="stable")[:k]
    return row[idx], idx


def generate(model, prompt, beam_size, max_length, page_size, max_pages,
             length_penalty=1.0, temperature=1.0, num_return=None, trace=None):
    """Beam search restated from beam.py:48-352 (cascade kernel, vanilla strategy).

    Returns (final [(seq, score)], state).  ``trace`` (a list) receives one
    dict per step with the selected parents/tokens when given."""
    c = model.cfg
    table = OraclePageTable(c["num_hidden_layers"], page_size, max_pages,
                            c["num_key_value_heads"], c["head_dim"])
    st = OracleBeamState(beam_size, table)
    made = st.add_root_sequence(list(prompt))
    pages = [st.nodes[m].page for m in made]
    last = len(st.nodes[made[-1]].tokens)
    logits = model.forward(prompt, list(range(len(prompt))), table, "prefill",
                           prefill=(pages, last))
    lp = log_softmax(logits[-1] / temperature if temperature != 1.0 else logits[-1])
    k = min(2 * beam_size, lp.shape[0])
    vals, idx = topk(lp, k)
    st.add_filtered_results([[(int(idx[i]), float(vals[i])) for i in range(min(beam_size, k))]])
    for step in range(max_length - len(prompt) - 1):
        if not st.cand_leaf:
            break
        levels, qtok = st.cascade_input()
        wp, wpos = st.write_targets()
        logits = model.forward(qtok, st.position_ids(), table, "decode",
                               write=(wp, wpos), levels=levels)
        lp = log_softmax(logits / temperature if temperature != 1.0 else logits)
        kk = min(2 * beam_size, lp.shape[1]) if beam_size != 1 else 1
        toks, lps = [], []
        for r in range(lp.shape[0]):
            v_, i_ = topk(lp[r], kk)
            toks.append(i_.tolist())
            lps.append([float(np.float32(x)) for x in v_])
        sel = vanilla_select(st.cand_score, toks, lps, beam_size)
        if trace is not None:
            trace.append(dict(step=step, sel=[[t for t, _ in s] for s in sel]))
        st.add_filtered_results(sel)
    final = st.final_sequences(num_return or beam_size, length_penalty)
    return final, st
