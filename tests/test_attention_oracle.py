"""CPU: the attention oracle (direct softmax in fp64) against a literal
restatement of the reference kernel's per-row loop (lold3344/ARIA
src/kernels.cu :1340-1436: running max from -1e30, per-key online update of
the sum and the output, causal skip, final 1/l and lse = m + ln l), on small
cases; and the packed-QKV view against the [NH][T][dh] one."""
import numpy as np


def _reference_loop(q, k, v, scale):
    NH, T, dh = q.shape
    out = np.zeros((NH, T, dh))
    lse = np.zeros((NH, T))
    for h in range(NH):
        for qi in range(T):
            m, l, o = -1e30, 0.0, np.zeros(dh)
            for ki in range(T):
                if ki > qi:
                    continue
                s = float(q[h, qi] @ k[h, ki]) * scale
                m_new = max(m, s)
                e, ed = np.exp(s - m_new), np.exp(m - m_new)
                l = l * ed + e
                o = o * ed + v[h, ki] * e
                m = m_new
            out[h, qi] = o / l
            lse[h, qi] = m + np.log(l)
    return out, lse


def test_oracle_equals_reference_loop():
    from oracle.attention_np import flash_attn_fwd
    rng = np.random.default_rng(0)
    for NH, T, dh in [(1, 1, 4), (2, 7, 8), (3, 13, 16)]:
        q, k, v = (rng.standard_normal((NH, T, dh)) for _ in range(3))
        a_out, a_lse = flash_attn_fwd(q, k, v, 0.3)
        b_out, b_lse = _reference_loop(q, k, v, 0.3)
        assert np.allclose(a_out, b_out, atol=1e-12) and np.allclose(a_lse, b_lse, atol=1e-12)


def test_packed_view_matches_head_major():
    from oracle.attention_np import attention_prefill, flash_attn_fwd
    rng = np.random.default_rng(1)
    B, T, d, H = 2, 9, 24, 3
    qkv = rng.standard_normal((B * T, 3 * d))
    out, lse = attention_prefill(qkv, B, T, d, H)
    dh = d // H
    for b in range(B):
        for h in range(H):
            rows = qkv[b * T:(b + 1) * T]
            q, k, v = (rows[:, c * d + h * dh:c * d + (h + 1) * dh][None] for c in range(3))
            o, l = flash_attn_fwd(q, k, v, 1 / np.sqrt(dh))
            assert np.allclose(out[b * T:(b + 1) * T, h * dh:(h + 1) * dh], o[0])
            assert np.allclose(lse[b, h], l[0])
