"""The arithmetic of the persistent kernel's run accumulation (attention_wide.cu,
BE_ATTN_WIDE_RUNS): per-chunk unnormalised rows with the chunk's own base-2
maximum, merged as M = max(M, m_c), acc = acc * 2^(M_old - M) + O_c * 2^(m_c - M),
L = L * 2^(M_old - M) + l_c * 2^(m_c - M), out = acc / L, LSE = (M + log2 L) ln 2.
Checked in float64 against one softmax over all chunks (CPU, no device code)."""
import numpy as np
import pytest


def chunk_state(s_scaled, v):
    """What one task leaves: chunk max (base 2, scaled scores), row sum, O rows."""
    m = s_scaled.max(axis=1)
    p = np.exp2(s_scaled - m[:, None])
    return m, p.sum(axis=1), p @ v


@pytest.mark.parametrize("seed", range(5))
def test_run_merge_equals_full_softmax(seed):
    rng = np.random.default_rng(seed)
    rows, d = 64, 128
    chunks = [int(x) for x in rng.integers(1, 129, rng.integers(1, 9))]
    scale_log2 = d ** -0.5 * np.log2(np.e)
    q = rng.standard_normal((rows, d))
    ks = [rng.standard_normal((n, d)) * rng.uniform(0.5, 3) for n in chunks]
    vs = [rng.standard_normal((n, d)) for n in chunks]
    M = np.full(rows, -np.inf)
    L = np.zeros(rows)
    acc = np.zeros((rows, d))
    for k, v in zip(ks, vs):
        m_c, l_c, o_c = chunk_state(q @ k.T * scale_log2, v)
        m_new = np.maximum(M, m_c)
        a = np.where(M == -np.inf, 0.0, np.exp2(M - m_new))
        b = np.where(m_c == -np.inf, 0.0, np.exp2(m_c - m_new))
        acc = acc * a[:, None] + o_c * b[:, None]
        L = L * a + l_c * b
        M = m_new
    out = acc / L[:, None]
    lse = (M + np.log2(L)) * np.log(2)
    K, V = np.concatenate(ks), np.concatenate(vs)
    s = q @ K.T * d ** -0.5
    ref_lse = np.log(np.exp(s - s.max(1, keepdims=True)).sum(1)) + s.max(1)
    ref = np.exp(s - ref_lse[:, None]) @ V
    np.testing.assert_allclose(out, ref, rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(lse, ref_lse, rtol=1e-12, atol=1e-12)
