"""GPU decode step with KV cache for the Efkolos decoder (Q4_0 projections).

Host mirror of the reference's cached inference step (lold3344/ARIA
src/transformer_cuda.rs `step` :1286-1324 over `cpu_layer_forward`
:1059-1166, with `KVCache` :144-155), which there runs on the CPU in f32.  Here
every operation runs on the GPU through libaria_q4.so:

    h  = embed[token] + pos_embed[pos]                      aria_embed_f16
    per layer:
      qkv = LayerNorm1(h) @ w_qkv + b_qkv                   aria_q4_0_matmul_ln (LayerNorm prologue)
      att = attention(q; K, V cache with this k, v added)   aria_attention_decode
      h  += att @ w_out + b_out                             aria_q4_0_matmul_ws, beta = 1 into the f32 residual
      u  = GELU(LayerNorm2(h) @ w_ff1 + b_ff1)              aria_q4_0_matmul_ln, GELU in the epilogue
      h  += u @ w_ff2 + b_ff2
    logits = LayerNorm_f(h) @ embed^T                       aria_layernorm_f32 + the tied LM head (Q4_0)

(above 64 sequences the LayerNorms run as aria_layernorm_f32 launches before
the projections).  `prefill` runs a whole prompt per sequence at once -- the
reference's forward_gpu -- with causal attention on the tensor cores
(aria_attention_prefill) and fills the caches for the steps that follow.

The residual stream h is f32; the LayerNorm outputs, q/k/v, the attention
output, the FFN hidden activation and the caches are f16 (the activation type
of the reference's GPU path).  M independent sequences decode together, each
at its own position with its own cache rows.  Weights are seeded synthetic (no
checkpoint is available): projections N(0, 0.02) (x 1/sqrt(2L) for attn_out and
ffn_down), biases N(0, 0.02), LayerNorm gains 1 + N(0, 0.1) and shifts
N(0, 0.1), the sinusoidal position table of the reference's initialiser
(:896-903).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import call
from .efkolos import EfkolosConfig, synth_f16
from .q4 import LAYOUT_KN, LAYOUT_NK, Q4Weight, matmul, matmul_ln

LN_EPS = 1e-5  # cpu_layernorm_stats (:3277)


def sinusoidal_positions(max_seq: int, d: int, device="cuda") -> torch.Tensor:
    """The reference's position table (:896-903): angle = pos / 10000^(2 (i/2) / d),
    sin for even i, cos for odd i, stored f16."""
    pos = torch.arange(max_seq, dtype=torch.float32).unsqueeze(1)
    i = torch.arange(d)
    angle = pos / torch.pow(torch.tensor(10000.0), (2 * (i // 2)).float() / d)
    table = torch.where(i % 2 == 0, torch.sin(angle), torch.cos(angle))
    return table.to(torch.float16).to(device)


@dataclass
class LayerParams:
    qkv: Q4Weight
    out: Q4Weight
    up: Q4Weight
    down: Q4Weight
    b_qkv: torch.Tensor
    b_out: torch.Tensor
    b_up: torch.Tensor
    b_down: torch.Tensor
    ln1_g: torch.Tensor
    ln1_b: torch.Tensor
    ln2_g: torch.Tensor
    ln2_b: torch.Tensor


class DecoderWeights:
    """Every parameter the decode step reads: Q4_0 projections, f16 biases,
    LayerNorm parameters, the f16 embedding table (token lookup) and its
    Q4_0 form (the tied LM head)."""

    def __init__(self, cfg: EfkolosConfig, max_seq: int = 512, seed: int = 0, device="cuda"):
        self.cfg, self.max_seq = cfg, max_seq
        d, ff, V, L = cfg.d_model, cfg.ffn_dim, cfg.vocab_size, cfg.num_layers
        s, sd = 0.02, 0.02 / math.sqrt(2 * L)
        self.f16 = {}  # the f16 tensors the Q4_0 weights were quantised from (for the oracle)
        self.layers: list[LayerParams] = []

        def w(name, shape, sigma, tag):
            t = synth_f16(shape, sigma, seed * 1000003 + tag, device)
            self.f16[name] = t
            return t

        def ln(tag, n):
            g = (1.0 + synth_f16((n,), 0.1, seed * 1000003 + tag, device).float()).half()
            return g, synth_f16((n,), 0.1, seed * 1000003 + tag + 1, device)

        for i in range(L):
            b = 100 * (i + 1)
            qkv = Q4Weight.from_f16(w(f"{i}.qkv", (d, 3 * d), s, b + 1), LAYOUT_KN)
            out = Q4Weight.from_f16(w(f"{i}.out", (d, d), sd, b + 2), LAYOUT_KN)
            up = Q4Weight.from_f16(w(f"{i}.up", (d, ff), s, b + 3), LAYOUT_KN)
            down = Q4Weight.from_f16(w(f"{i}.down", (ff, d), sd, b + 4), LAYOUT_KN)
            g1, b1 = ln(b + 10, d)
            g2, b2 = ln(b + 20, d)
            self.layers.append(LayerParams(
                qkv, out, up, down,
                synth_f16((3 * d,), 0.02, seed * 1000003 + b + 5, device),
                synth_f16((d,), 0.02, seed * 1000003 + b + 6, device),
                synth_f16((ff,), 0.02, seed * 1000003 + b + 7, device),
                synth_f16((d,), 0.02, seed * 1000003 + b + 8, device), g1, b1, g2, b2))
        self.embed = w("embed", (V, d), s, 7)
        self.head = Q4Weight.from_f16(self.embed, LAYOUT_NK)
        self.lnf_g, self.lnf_b = ln(9, d)
        self.pos_embed = sinusoidal_positions(max_seq, d, device)

    @property
    def q4_bytes(self) -> int:
        return sum(p.qkv.nbytes + p.out.nbytes + p.up.nbytes + p.down.nbytes for p in self.layers) + self.head.nbytes


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


class Decoder:
    """M sequences decoding together, one token each per `step`, with their
    KV caches ([layer] f16 [M][max_seq][d], K and V) on the device."""

    def __init__(self, weights: DecoderWeights, M: int = 1, device="cuda"):
        cfg = weights.cfg
        self.w, self.cfg, self.M = weights, cfg, M
        d, ff, V = cfg.d_model, cfg.ffn_dim, cfg.vocab_size
        self.k_cache = [torch.zeros(M, weights.max_seq, d, dtype=torch.float16, device=device)
                        for _ in range(cfg.num_layers)]
        self.v_cache = [torch.zeros_like(k) for k in self.k_cache]
        self.h = torch.empty(M, d, dtype=torch.float32, device=device)
        self.xn = torch.empty(M, d, dtype=torch.float16, device=device)
        self.qkv = torch.empty(M, 3 * d, dtype=torch.float16, device=device)
        self.att = torch.empty(M, d, dtype=torch.float16, device=device)
        self.u = torch.empty(M, ff, dtype=torch.float16, device=device)
        self.logits = torch.empty(M, V, dtype=torch.float32, device=device)
        self.tokens = torch.zeros(M, dtype=torch.int32, device=device)
        self.positions = torch.zeros(M, dtype=torch.int32, device=device)

    def _layernorm(self, g, b):
        call("aria_layernorm_f32", self.h.data_ptr(), self.M, self.cfg.d_model, g.data_ptr(), b.data_ptr(),
             LN_EPS, self.xn.data_ptr(), self.cfg.d_model, _stream())

    def run(self) -> torch.Tensor:
        """One decode step for the tokens and positions already in
        self.tokens / self.positions (device int32 [M]); returns self.logits."""
        cfg, w = self.cfg, self.w
        d = cfg.d_model
        call("aria_embed_f16", w.embed.data_ptr(), w.pos_embed.data_ptr(), cfg.vocab_size, w.max_seq, d,
             self.tokens.data_ptr(), self.positions.data_ptr(), self.M, self.h.data_ptr(), _stream())
        fused_ln = self.M <= 64  # LayerNorm as the prologue of QKV / ffn_up (register-fed kernel)
        for i, p in enumerate(w.layers):
            if fused_ln:
                matmul_ln(self.h, p.ln1_g, p.ln1_b, p.qkv, self.qkv, eps=LN_EPS, bias=p.b_qkv, const_weights=True)
            else:
                self._layernorm(p.ln1_g, p.ln1_b)
                matmul(self.xn, p.qkv, self.qkv, bias=p.b_qkv, const_weights=True)
            call("aria_attention_decode", self.qkv.data_ptr(), self.M, d, cfg.num_heads,
                 self.k_cache[i].data_ptr(), self.v_cache[i].data_ptr(), w.max_seq, self.positions.data_ptr(),
                 self.att.data_ptr(), _stream())
            matmul(self.att, p.out, self.h, bias=p.b_out, beta=1.0, const_weights=True)
            if fused_ln:
                matmul_ln(self.h, p.ln2_g, p.ln2_b, p.up, self.u, eps=LN_EPS, bias=p.b_up, activation="gelu",
                          const_weights=True)
            else:
                self._layernorm(p.ln2_g, p.ln2_b)
                matmul(self.xn, p.up, self.u, bias=p.b_up, activation="gelu", const_weights=True)
            matmul(self.u, p.down, self.h, bias=p.b_down, beta=1.0, const_weights=True)
        self._layernorm(w.lnf_g, w.lnf_b)
        matmul(self.xn, w.head, self.logits, const_weights=True)
        return self.logits

    def step(self, tokens, positions) -> torch.Tensor:
        """The reference's `step(token, kv)` for M sequences: tokens and
        positions are length-M sequences of ints (each sequence's cache must hold
        its positions 0..pos-1 already)."""
        self.tokens.copy_(torch.as_tensor(tokens, dtype=torch.int32))
        self.positions.copy_(torch.as_tensor(positions, dtype=torch.int32))
        return self.run()

    @property
    def launches(self) -> int:
        return 1 + (5 if self.M <= 64 else 7) * self.cfg.num_layers + 2

    # ------------------------------------------------------------------ prefill
    def _prefill_buffers(self, T: int) -> dict:
        buf = getattr(self, "_pbuf", None)
        if buf is not None and buf["T"] == T:
            return buf
        cfg, n, dev = self.cfg, self.M * T, self.h.device
        d = cfg.d_model
        buf = {"T": T,
               "h": torch.empty(n, d, dtype=torch.float32, device=dev),
               "xn": torch.empty(n, d, dtype=torch.float16, device=dev),
               "qkv": torch.empty(n, 3 * d, dtype=torch.float16, device=dev),
               "att": torch.empty(n, d, dtype=torch.float16, device=dev),
               "u": torch.empty(n, cfg.ffn_dim, dtype=torch.float16, device=dev),
               "logits": torch.empty(n, cfg.vocab_size, dtype=torch.float16, device=dev),
               "tok": torch.zeros(n, dtype=torch.int32, device=dev),
               "pos": torch.arange(T, dtype=torch.int32, device=dev).repeat(self.M)}
        self._pbuf = buf
        return buf

    def run_prefill(self, T: int, fill_cache: bool = True) -> torch.Tensor:
        """The reference's whole-prompt forward (forward_gpu,
        src/transformer_cuda.rs:1518-1873) for the M sequences of T tokens
        already in the prefill token buffer (`prefill` fills it): embedding +
        position, per layer LayerNorm -> QKV -> causal attention over the
        prompt (aria_attention_prefill) -> attn_out into the f32 residual ->
        LayerNorm -> ffn_up + GELU -> ffn_down into the residual, then the final
        LayerNorm and the LM head over every token (f16 logits [M*T][vocab]).
        With fill_cache, each layer's attention launch also stores its k and v
        rows into the KV caches at positions 0..T-1, so `step` continues at
        position T."""
        from .attention import attention_prefill
        cfg, w, b = self.cfg, self.w, self._prefill_buffers(T)
        d, n = cfg.d_model, self.M * T
        if T > w.max_seq:
            raise ValueError(f"T={T} exceeds the cache length {w.max_seq}")
        call("aria_embed_f16", w.embed.data_ptr(), w.pos_embed.data_ptr(), cfg.vocab_size, w.max_seq, d,
             b["tok"].data_ptr(), b["pos"].data_ptr(), n, b["h"].data_ptr(), _stream())

        def ln(g, bb):
            call("aria_layernorm_f32", b["h"].data_ptr(), n, d, g.data_ptr(), bb.data_ptr(), LN_EPS,
                 b["xn"].data_ptr(), d, _stream())

        for i, p in enumerate(w.layers):
            ln(p.ln1_g, p.ln1_b)
            matmul(b["xn"], p.qkv, b["qkv"], bias=p.b_qkv, const_weights=True)
            # the attention launch also stores this layer's k, v rows into the caches
            attention_prefill(b["qkv"], self.M, T, cfg.num_heads, out=b["att"],
                              k_cache=self.k_cache[i] if fill_cache else None,
                              v_cache=self.v_cache[i] if fill_cache else None)
            matmul(b["att"], p.out, b["h"], bias=p.b_out, beta=1.0, const_weights=True)
            ln(p.ln2_g, p.ln2_b)
            matmul(b["xn"], p.up, b["u"], bias=p.b_up, activation="gelu", const_weights=True)
            matmul(b["u"], p.down, b["h"], bias=p.b_down, beta=1.0, const_weights=True)
        ln(w.lnf_g, w.lnf_b)
        matmul(b["xn"], w.head, b["logits"], const_weights=True)
        return b["logits"]

    def prefill(self, tokens, fill_cache: bool = True) -> torch.Tensor:
        """tokens: [M][T] ints (one prompt per sequence).  Returns the f16
        logits [M*T][vocab] of every position (row m*T + t)."""
        tok = torch.as_tensor(tokens, dtype=torch.int32)
        if tok.dim() != 2 or tok.shape[0] != self.M:
            raise ValueError(f"tokens must be [{self.M}][T]")
        T = tok.shape[1]
        b = self._prefill_buffers(T)
        b["tok"].copy_(tok.reshape(-1))
        return self.run_prefill(T, fill_cache)

    def prefill_launches(self, fill_cache: bool = True) -> int:
        """Kernels of one run_prefill."""
        return 1 + 7 * self.cfg.num_layers + 2


__all__ = ["Decoder", "DecoderWeights", "sinusoidal_positions", "LN_EPS"]
_ = _lib  # the C ABI binding is loaded through `call`
