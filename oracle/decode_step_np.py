"""numpy restatement of the reference's cached decode step.  TEST INFRASTRUCTURE ONLY.

Follows lold3344/ARIA src/transformer_cuda.rs:
  `step`               :1286-1324  embedding + position, layers, final LayerNorm, tied LM head
  `cpu_layer_forward`  :1059-1166  LayerNorm1, QKV + bias, K/V appended to the cache, per-head
                                    softmax(q.k / sqrt(dh)) over positions 0..pos, attn_out + bias,
                                    residual, LayerNorm2, ffn_up + bias, GELU, ffn_down + bias, residual
  `cpu_layernorm`      :3271-3293  eps 1e-5, population variance
  `gelu`               :3258-3261  tanh form

The reference computes in f32 with f16 weights.  This oracle computes in fp64
with the exact dequantisation of the Q4_0 weights (the product of the device
path) and rounds to f16 exactly where the GPU decode step stores f16 (LayerNorm
outputs, q/k/v and the caches, the attention output, the GELU output); the
residual stream stays unrounded (f32 on the GPU).  Only tests/ may import it.

Parity status: the arithmetic is pinned by the reference's code above, not by
executed reference output (Rust cannot run here).
"""
from __future__ import annotations

import numpy as np

from oracle.q4_oracle_np import LAYOUT_KN, LAYOUT_NK, gelu_tanh

LN_EPS = 1e-5


def f16(a) -> np.ndarray:
    return np.asarray(a, dtype=np.float64).astype(np.float16).astype(np.float64)


def layernorm(x, g, b, eps=LN_EPS) -> np.ndarray:
    x = np.asarray(x, dtype=np.float64)
    mu = x.mean(axis=-1, keepdims=True)
    var = ((x - mu) ** 2).mean(axis=-1, keepdims=True)
    return (x - mu) / np.sqrt(var + eps) * g + b


class DecodeOracle:
    """Holds dequantised weights [K][N] (f64) and the K/V caches of M sequences."""

    def __init__(self, coracle, params: dict, cfg, max_seq: int, M: int):
        """params: f16 numpy arrays keyed like aria_b200.decoder.DecoderWeights.f16
        ('{i}.qkv' [d][3d], '{i}.out', '{i}.up', '{i}.down', 'embed' [V][d]) plus
        biases / LayerNorm parameters ('{i}.b_qkv', ..., '{i}.ln1_g', ..., 'lnf_g',
        'lnf_b') and 'pos' [max_seq][d]."""
        self.cfg, self.max_seq, self.M = cfg, max_seq, M
        self.p = {k: np.asarray(v, dtype=np.float16).astype(np.float64) for k, v in params.items()}
        self.W = {}
        for key, v in params.items():
            if key.split(".")[-1] in ("qkv", "out", "up", "down") or key == "embed":
                w = np.asarray(v, dtype=np.float16)
                K, N = (w.shape[0], w.shape[1]) if key != "embed" else (w.shape[1], w.shape[0])
                blocks = coracle.quantize_q4_0_f16(w.reshape(-1))
                wd = coracle.dequantize_q4_0(blocks, K * N).astype(np.float64).reshape(w.shape)
                self.W[key] = wd if key != "embed" else wd.T  # [K][N]
        d = cfg.d_model
        self.k = [np.zeros((M, max_seq, d)) for _ in range(cfg.num_layers)]
        self.v = [np.zeros((M, max_seq, d)) for _ in range(cfg.num_layers)]

    def step(self, tokens, positions) -> np.ndarray:
        cfg, p = self.cfg, self.p
        d, H = cfg.d_model, cfg.num_heads
        dh = d // H
        V = cfg.vocab_size
        tok = np.clip(np.asarray(tokens), 0, V - 1)
        pos = np.clip(np.asarray(positions), 0, self.max_seq - 1)
        h = p["embed"][tok] + p["pos"][pos]  # f16 tables, exact f32 sum
        for i in range(cfg.num_layers):
            xn = f16(layernorm(h, p[f"{i}.ln1_g"], p[f"{i}.ln1_b"]))
            qkv = f16(xn @ self.W[f"{i}.qkv"] + p[f"{i}.b_qkv"])
            att = np.zeros((self.M, d))
            for m in range(self.M):
                t = pos[m]
                self.k[i][m, t] = qkv[m, d:2 * d]
                self.v[i][m, t] = qkv[m, 2 * d:]
                for hh in range(H):
                    q = qkv[m, hh * dh:(hh + 1) * dh]
                    Kc = self.k[i][m, :t + 1, hh * dh:(hh + 1) * dh]
                    Vc = self.v[i][m, :t + 1, hh * dh:(hh + 1) * dh]
                    s = Kc @ q / np.sqrt(dh)
                    e = np.exp(s - s.max())
                    att[m, hh * dh:(hh + 1) * dh] = (e / e.sum()) @ Vc
            att = f16(att)
            h = h + att @ self.W[f"{i}.out"] + p[f"{i}.b_out"]
            xn = f16(layernorm(h, p[f"{i}.ln2_g"], p[f"{i}.ln2_b"]))
            u = f16(gelu_tanh(xn @ self.W[f"{i}.up"] + p[f"{i}.b_up"]))
            h = h + u @ self.W[f"{i}.down"] + p[f"{i}.b_down"]
        xn = f16(layernorm(h, p["lnf_g"], p["lnf_b"]))
        return xn @ self.W["embed"]


__all__ = ["DecodeOracle", "layernorm", "f16", "LAYOUT_KN", "LAYOUT_NK"]
