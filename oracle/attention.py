"""Oracle: attention semantics of the decode path (test infrastructure).

* ``cascade_attention`` restates ``MultiLevelCascadeAttentionWrapper`` as the
  reference drives it (modeling_llama.py:733-755 plan, :362 run): level ``l``
  is a batch paged prefill in which group ``g`` owns queries
  ``qo_indptr[g]:qo_indptr[g+1]`` and pages ``kv_indices[kv_indptr[g]:
  kv_indptr[g+1]]`` with ``kv_len = (npages - 1) * page_size + last_len``;
  only the LAST level is causal (bottom-right aligned: query ``i`` of a group
  of ``qo_len`` sees the first ``kv_len - qo_len + i + 1`` keys); each level
  yields ``(o, lse)`` with natural-log LSE and an empty key set gives
  ``lse = -inf``; levels are merged by LSE weights.  GQA: query head ``h``
  reads KV head ``h // (Hq / Hkv)``.
* ``paged_prefill`` restates the causal prompt attention of
  ``BatchPrefillWithPagedKVCacheWrapper`` (modeling_llama.py:213-283, 775-798).
* ``fasttree_plan`` restates ``prepare_fasttree_metadata_for_paged_cache``
  (attention/fasttree/preparation.py:11-225, parameters metadata.py:12-38):
  the SplitK/SplitQ edge cost model, merged request sets, vnode emission with
  KV splits, req->vnode lists and the two-phase reorder.
* ``fasttree_attention`` restates the two Triton stages
  (attention/fasttree/kernel.py:5-119 per-vnode partial softmax, 188-252
  per-(request, head) LSE merge).
All math runs in float64.
"""
from __future__ import annotations

import math
import numpy as np


def _attend(q, k, v, scale):
    """q [n, D], k/v [m, D] -> (o [n, D], lse [n]) with natural-log LSE."""
    if k.shape[0] == 0:
        return np.zeros((q.shape[0], v.shape[1])), np.full(q.shape[0], -np.inf)
    s = (q @ k.T) * scale
    m = s.max(axis=1, keepdims=True)
    p = np.exp(s - m)
    l = p.sum(axis=1, keepdims=True)
    return (p @ v) / l, (m + np.log(l))[:, 0]


def gather_pages(pool, pages, kv_len, plane):
    """pool [P, 2, ps, Hkv, D] -> [kv_len, Hkv, D] for the listed pages."""
    if len(pages) == 0 or kv_len <= 0:
        return np.zeros((0,) + pool.shape[3:], pool.dtype)
    x = pool[np.asarray(pages, np.int64), plane]          # [np, ps, Hkv, D]
    return x.reshape(-1, *pool.shape[3:])[:kv_len]


def merge_states(os_, lses):
    """LSE-merge a list of (o [.., D], lse [..]) states."""
    lse = np.stack(lses)                                   # [L, ...]
    m = lse.max(axis=0)
    safe = np.where(np.isfinite(m), m, 0.0)
    w = np.exp(lse - safe[None])
    w = np.where(np.isfinite(lse), w, 0.0)
    den = w.sum(axis=0)
    num = sum(w[i][..., None] * os_[i] for i in range(len(os_)))
    o = np.where(den[..., None] > 0, num / np.where(den > 0, den, 1.0)[..., None], 0.0)
    out_lse = np.where(den > 0, safe + np.log(np.where(den > 0, den, 1.0)), -np.inf)
    return o, out_lse


def level_attention(q, pool, lvl, page_size, scale, causal):
    """One cascade level.  q [N, Hq, D]; returns (o [N, Hq, D], lse [N, Hq])."""
    q = q.astype(np.float64)
    pool = pool.astype(np.float64)
    N, Hq, D = q.shape
    Hkv = pool.shape[3]
    g = Hq // Hkv
    o = np.zeros((N, Hq, D))
    lse = np.full((N, Hq), -np.inf)
    qo, kvp, kvi, last = (lvl["qo_indptr"], lvl["kv_indptr"], lvl["kv_indices"],
                          lvl["kv_last_page_len"])
    for gi in range(len(qo) - 1):
        pages = kvi[kvp[gi]:kvp[gi + 1]]
        kv_len = (len(pages) - 1) * page_size + last[gi] if len(pages) else 0
        K = gather_pages(pool, pages, kv_len, 0)
        V = gather_pages(pool, pages, kv_len, 1)
        qlen = qo[gi + 1] - qo[gi]
        for i in range(qlen):
            r = qo[gi] + i
            vis = kv_len if not causal else max(0, min(kv_len, kv_len - qlen + i + 1))
            for h in range(Hq):
                kh = h // g
                oo, ll = _attend(q[r, h][None], K[:vis, kh], V[:vis, kh], scale)
                o[r, h], lse[r, h] = oo[0], ll[0]
    return o, lse


def cascade_attention(q, pool, levels, page_size, scale, return_lse=False):
    """MultiLevelCascadeAttentionWrapper.run restated (causal on the last level)."""
    outs, lses = [], []
    for i, lvl in enumerate(levels):
        o, l = level_attention(q, pool, lvl, page_size, scale, causal=(i == len(levels) - 1))
        outs.append(o)
        lses.append(l)
    o, lse = merge_states(outs, lses)
    return (o, lse) if return_lse else o


def paged_prefill(q, pool, pages, last_len, page_size, scale):
    """Causal attention of n prompt queries over their own pages."""
    n = q.shape[0]
    lvl = dict(qo_indptr=[0, n], kv_indptr=[0, len(pages)], kv_indices=list(pages),
               kv_last_page_len=[last_len])
    o, _ = level_attention(q, pool, lvl, page_size, scale, causal=True)
    return o


def dense_attention(q, k, v, scale):
    """q [Hq, D]; k/v [T, Hkv, D] -> o [Hq, D] (plain softmax attention, GQA)."""
    Hq = q.shape[0]
    g = Hq // k.shape[1]
    out = np.zeros(q.shape)
    for h in range(Hq):
        out[h] = _attend(q[h][None].astype(np.float64), k[:, h // g].astype(np.float64),
                         v[:, h // g].astype(np.float64), scale)[0][0]
    return out


# ---------------------------------------------------------------------------
# FastTree (attention/fasttree/preparation.py, metadata.py, kernel.py)
# ---------------------------------------------------------------------------
FT_ALPHA, FT_BETA, FT_GAMMA = 0.6, 0.3, 0.1
FT_TSK = (32, 32)
FT_KV_SPLIT = (1024, 128)


def fasttree_plan(tree, r2t_stride, batch_size, num_qo_heads, num_kv_heads):
    """Returns a dict of int lists with the reference's vnode metadata."""
    g = num_qo_heads // num_kv_heads
    tsq = (64 // g, 16 // g)
    tsk = FT_TSK
    split = [FT_KV_SPLIT[0], FT_KV_SPLIT[0]]          # preparation.py:39 uses split[0] twice

    def pad_q(ts, n):
        return ts - ((n - 1) % ts + 1)

    def pad_k(ts, n):
        return max(0, ts - n)

    def cmm(nq, nk):
        ph = 0 if nq > tsq[1] else 1
        return FT_ALPHA * pad_q(tsq[ph], nq) * g * nk + FT_BETA * pad_k(tsk[ph], nk) * nq * g

    n = len(tree)
    kids = [[] for _ in range(n)]
    for i in range(n):
        if tree[i]["parent"] != -1:
            kids[tree[i]["parent"]].append(i)
    L = [t["seqlen"] for t in tree]
    merged = [0] * n
    fifo = [0]
    while fifo:
        v = fifo.pop(0)
        nq_cur = len(tree[v]["requests"])
        lenv = L[v]
        for c in kids[v]:
            nql = len(tree[c]["requests"])
            lenl = L[c]
            split_k = cmm(nq_cur, lenv) + cmm(nql, lenl) + FT_GAMMA * nql
            split_q = cmm(nq_cur - nql, lenv) + cmm(nql, lenl + lenv)
            if split_k > split_q:
                merged[c] = 1
                nq_cur -= nql
                L[c] = lenl + lenv
            fifo.append(c)
    node_reqs = [[] for _ in range(n)]
    fifo = []
    for i in range(n):
        if tree[i]["num_children"] == 0:
            fifo.append(i)
            node_reqs[i] = list(tree[i]["requests"])
    vkids = [t["num_children"] for t in tree]
    while fifo:
        v = fifo.pop(0)
        par = tree[v]["parent"]
        if merged[v] == 0 and v != 0:
            node_reqs[par] += tree[v]["requests"]
        vkids[par] -= 1                               # note: par == -1 touches the last entry
        if par >= 0 and vkids[par] == 0:
            fifo.append(par)
    tok_off = [0] * n
    for i in range(1, n):
        p = tree[i]["parent"]
        tok_off[i] = tok_off[p] + tree[p]["seqlen"]
    kv_offs, kv_lens, q_entries, q_offs, q_lens = [], [], [], [], []
    for i in range(n):
        reqs = node_reqs[i]
        if not reqs:
            continue
        kv_len = tree[i]["seqlen"]
        v = i
        while merged[v] == 1:
            v = tree[v]["parent"]
            kv_len += tree[v]["seqlen"]
        ph = 0 if len(reqs) > tsq[1] else 1
        kv_split, q_split = split[ph], tsq[ph]
        kv_start = r2t_stride * reqs[0] + tok_off[v]
        for ks in range((kv_len - 1) // kv_split + 1):
            q0 = len(q_entries)
            q_entries.extend(reqs)
            koff = ks * kv_split
            klen = min(koff + kv_split, kv_len) - koff
            for qs in range((len(reqs) - 1) // q_split + 1):
                qoff = qs * q_split
                kv_offs.append(kv_start + koff)
                kv_lens.append(klen)
                q_offs.append(q0 + qoff)
                q_lens.append(min(qoff + q_split, len(reqs)) - qoff)
    r2v = [[] for _ in range(batch_size)]
    for i, r in enumerate(q_entries):
        r2v[r].append(i)
    r2v_offs, r2v_lens, off = [], [], 0
    for b in range(batch_size):
        r2v_offs.append(off)
        r2v_lens.append(len(r2v[b]))
        off += len(r2v[b])
    above = [i for i, x in enumerate(q_lens) if x > tsq[1]]
    below = [i for i, x in enumerate(q_lens) if x <= tsq[1]]
    order = above + below
    return dict(
        vnode_to_q_entries=q_entries,
        vnode_to_q_offs=[q_offs[i] for i in order],
        vnode_to_q_lens=[q_lens[i] for i in order],
        vnode_to_kv_offs=[kv_offs[i] for i in order],
        vnode_to_kv_lens=[kv_lens[i] for i in order],
        req_to_vnode_entries=[x for lst in r2v for x in lst],
        req_to_vnode_offs=r2v_offs,
        req_to_vnode_lens=r2v_lens,
        phase_node_nums=(len(above), len(below)),
        phase_node_offsets=(0, len(above)),
        phase_q_tile_sizes=tsq,
        phase_kv_tile_sizes=tsk,
    )


def fasttree_attention(q, k_flat, v_flat, plan, kv_entries, scale):
    """Two-stage FastTree decode.  q [B, Hq, D]; k/v_flat [slots, Hkv, D];
    kv_entries = flattened req_to_token.  Stage 1 writes one (o, lse) per
    (vnode q-entry, head); stage 2 merges each request's entries."""
    q = q.astype(np.float64)
    B, Hq, D = q.shape
    g = Hq // k_flat.shape[1]
    nq = len(plan["vnode_to_q_entries"])
    mid_o = np.zeros((max(nq, 1), Hq, D))
    mid_lse = np.full((max(nq, 1), Hq), -np.inf)
    for v in range(len(plan["vnode_to_q_offs"])):
        qo, ql = plan["vnode_to_q_offs"][v], plan["vnode_to_q_lens"][v]
        ko, kl = plan["vnode_to_kv_offs"][v], plan["vnode_to_kv_lens"][v]
        slots = np.asarray(kv_entries[ko:ko + kl], np.int64)
        K = k_flat[slots].astype(np.float64)
        V = v_flat[slots].astype(np.float64)
        for j in range(ql):
            e = qo + j
            r = plan["vnode_to_q_entries"][e]
            for h in range(Hq):
                o, l = _attend(q[r, h][None], K[:, h // g], V[:, h // g], scale)
                mid_o[e, h], mid_lse[e, h] = o[0], l[0]
    out = np.zeros((B, Hq, D))
    for b in range(B):
        ents = plan["req_to_vnode_entries"][plan["req_to_vnode_offs"][b]:
                                            plan["req_to_vnode_offs"][b] + plan["req_to_vnode_lens"][b]]
        if not ents:
            out[b] = np.nan        # the reference kernel divides 0 by 0 here
            continue
        o, _ = merge_states([mid_o[e] for e in ents], [mid_lse[e] for e in ents])
        out[b] = o
    return out


def rope_cos_sin(positions, head_dim, theta):
    """HF default RoPE tables in float32 (modeling_llama.py:89-123)."""
    inv = 1.0 / (theta ** (np.arange(0, head_dim, 2, dtype=np.int64).astype(np.float32) / head_dim))
    f = np.outer(np.asarray(positions, np.float32), inv.astype(np.float32)).astype(np.float32)
    emb = np.concatenate([f, f], axis=-1)
    return np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)


def apply_rope(x, cos, sin):
    """x [n, H, D]; cos/sin [n, D]: x*cos + rotate_half(x)*sin."""
    h = x.shape[-1] // 2
    rot = np.concatenate([-x[..., h:], x[..., :h]], axis=-1)
    return x * cos[:, None, :] + rot * sin[:, None, :]


def safe_log(x):
    return math.log(x) if x > 0 else -math.inf
