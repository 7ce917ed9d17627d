"""numpy restatement of the reference's causal attention forward.  TEST INFRASTRUCTURE ONLY.

Follows lold3344/ARIA src/kernels.cu `flash_attn_fwd` :1298-1437: q, k, v, out
[NH][T][dh], lse [NH][T]; for query t of head h, the scores scale * q[t].k[s]
over keys s <= t (causal mask, :1378), an online softmax with running max m and
sum l (:1413-1424), out = sum_s softmax_s * v[s] normalised by 1/l (:1433-1434)
and lse = m + ln(l) (:1435).  The online form equals the plain
softmax; this restatement computes it directly in fp64.  Only tests/ may import
it.

Parity status: pinned by the reference's code above, not by executed reference
output (the reference is Rust + a CUDA C kernel built by its own build script,
not runnable here).
"""
from __future__ import annotations

import numpy as np


def flash_attn_fwd(q, k, v, scale: float):
    """q, k, v: [NH][T][dh] (any float dtype).  Returns (out [NH][T][dh] f64,
    lse [NH][T] f64)."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    NH, T, dh = q.shape
    s = np.einsum("htd,hsd->hts", q, k) * scale
    mask = np.triu(np.ones((T, T), dtype=bool), 1)  # s > t
    s = np.where(mask[None], -np.inf, s)
    m = s.max(axis=-1, keepdims=True)
    e = np.exp(s - m)
    l = e.sum(axis=-1, keepdims=True)
    out = np.einsum("hts,hsd->htd", e / l, v)
    lse = (m + np.log(l))[..., 0]
    return out, lse


def attention_prefill(qkv, B: int, T: int, d: int, heads: int):
    """The same attention on the packed QKV projection output [B*T][3d]:
    returns (out [B*T][d] f64, lse [B][heads][T])."""
    qkv = np.asarray(qkv, dtype=np.float64).reshape(B, T, 3, heads, d // heads)
    q = qkv[:, :, 0].transpose(0, 2, 1, 3).reshape(B * heads, T, -1)
    k = qkv[:, :, 1].transpose(0, 2, 1, 3).reshape(B * heads, T, -1)
    v = qkv[:, :, 2].transpose(0, 2, 1, 3).reshape(B * heads, T, -1)
    out, lse = flash_attn_fwd(q, k, v, 1.0 / np.sqrt(d // heads))
    out = out.reshape(B, heads, T, -1).transpose(0, 2, 1, 3).reshape(B * T, d)
    return out, lse.reshape(B, heads, T)


__all__ = ["flash_attn_fwd", "attention_prefill"]
