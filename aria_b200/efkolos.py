"""The Efkolos decoder's Q4_0 projection stack (the shapes the kernels serve).

Mirrors the projection-owning part of ARIA's TransformerModel
(lold3344/ARIA src/transformer_cuda.rs:261-271 TransformerLayer.w_*, :314 embed,
:717-776 make_layer init, :1483-1490 enable_int4 / int4_quantized) for the
quantised inference path only: attention, LayerNorm and GELU are outside this
library's scope, so a decode step here is the ordered chain of the five
projections per layer plus the LM head that forward_gpu runs
(:1583, :1686, :1753, :1805, :1864).

Weights are seeded synthetic N(0, sigma) (no checkpoints are available): sigma =
0.02, times 1/sqrt(2L) for attn_out and ffn_down as the reference's depth
scaling does (:719).  They are generated on the device in f16 and quantised
with the bit-exact device packer.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from .q4 import LAYOUT_KN, LAYOUT_NK, Q4Weight, matmul


@dataclass(frozen=True)
class EfkolosConfig:
    num_layers: int = 20
    d_model: int = 896
    num_heads: int = 14
    ffn_dim: int = 3584
    vocab_size: int = 31500

    @property
    def head_dim(self) -> int:
        return self.d_model // self.num_heads

    def projections(self):
        """(name, layout, K, N, sigma) per layer, in forward_gpu order."""
        d, ff = self.d_model, self.ffn_dim
        s = 0.02
        sd = s / math.sqrt(2 * self.num_layers)
        return [("attn_qkv", LAYOUT_KN, d, 3 * d, s), ("attn_out", LAYOUT_KN, d, d, sd),
                ("ffn_up", LAYOUT_KN, d, ff, s), ("ffn_down", LAYOUT_KN, ff, d, sd)]

    def lm_head(self):
        return ("lm_head", LAYOUT_NK, self.d_model, self.vocab_size, 0.02)

    def all_projections(self):
        out = []
        for i in range(self.num_layers):
            for (name, lay, K, N, s) in self.projections():
                out.append((f"blk.{i}.{name}", lay, K, N, s))
        out.append(self.lm_head())
        return out

    def weight_bytes(self) -> int:
        return sum(K * N // 32 * 18 for (_, _, K, N, _) in self.all_projections())

    def flops_per_token(self) -> int:
        return sum(2 * K * N for (_, _, K, N, _) in self.all_projections())


EFKOLOS = EfkolosConfig()
SCALED = EfkolosConfig(num_layers=32, d_model=4096, num_heads=32, ffn_dim=16384, vocab_size=31500)


def synth_f16(shape, sigma: float, seed: int, device="cuda") -> torch.Tensor:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return (torch.randn(shape, generator=g, device=device, dtype=torch.float32) * sigma).to(torch.float16)


@dataclass
class Q4Stack:
    """One replica of every projection weight of a config, Q4_0 on the device."""

    cfg: EfkolosConfig
    weights: list = field(default_factory=list)  # [(name, Q4Weight)]
    int4_quantized: bool = True

    @classmethod
    def build(cls, cfg: EfkolosConfig, seed: int = 0, device="cuda", chunk_rows: int = 0) -> "Q4Stack":
        st = cls(cfg)
        for idx, (name, lay, K, N, s) in enumerate(cfg.all_projections()):
            shape = (K, N) if lay == LAYOUT_KN else (N, K)
            w = synth_f16(shape, s, seed * 100003 + idx, device)
            st.weights.append((name, Q4Weight.from_f16(w, lay)))
            del w
        return st

    def enable_int4(self) -> None:
        """Reference flag (transformer_cuda.rs:1483-1490); the weights are Q4_0 already."""
        self.int4_quantized = True

    @property
    def nbytes(self) -> int:
        return sum(w.nbytes for _, w in self.weights)


class DecodeProgram:
    """One decode (or prefill) step's chain of projections over preallocated buffers.

    The data flow follows the reference's layer (src/transformer_cuda.rs:1059-1166
    and forward_gpu :1583-:1864): the residual stream h [M, d] feeds QKV; attn_out
    adds into h (the reference's residual add, fused as beta = 1); h feeds ffn_up,
    whose GELU is fused into its epilogue; ffn_down adds into h; after the last
    layer h feeds the LM head.  Attention and LayerNorm are outside this library:
    attn_out reads the first d_model columns of the QKV output in place of the
    attention output, and h is not normalised.  Every projection therefore
    consumes the output of the one before it, and every launch waits for the
    previous one on the stream (programmatic dependent launch) before it reads
    its activations.  A step starts by copying the input h0 into h."""

    def __init__(self, stack: Q4Stack, M: int, device="cuda", seed: int = 1):
        cfg = stack.cfg
        self.stack = stack
        self.M = M
        d = cfg.d_model
        self.h0 = synth_f16((M, d), 1.0, seed * 7919, device)
        self.h = torch.empty(M, d, dtype=torch.float16, device=device)
        self.y_qkv = torch.empty(M, 3 * d, dtype=torch.float16, device=device)
        self.u = torch.empty(M, cfg.ffn_dim, dtype=torch.float16, device=device)
        self.logits = torch.empty(M, cfg.vocab_size, dtype=torch.float16, device=device)

    def run(self, stack: Q4Stack | None = None) -> None:
        st = stack or self.stack
        d = st.cfg.d_model
        w = [q for _, q in st.weights]
        self.h.copy_(self.h0)
        for i in range(st.cfg.num_layers):
            qkv, out, up, down = w[4 * i:4 * i + 4]
            # model weights are never written inside a step: const-weights flag
            matmul(self.h, qkv, self.y_qkv, const_weights=True)
            matmul(self.y_qkv[:, :d], out, self.h, beta=1.0, const_weights=True)
            matmul(self.h, up, self.u, activation="gelu", const_weights=True)
            matmul(self.u, down, self.h, beta=1.0, const_weights=True)
        matmul(self.h, w[-1], self.logits, const_weights=True)

    @property
    def launches(self) -> int:
        return len(self.stack.weights)

    def algorithmic_bytes(self) -> int:
        """Q4_0 weights + f16 activations read + f16 outputs written, once each."""
        b = self.stack.nbytes
        for (_, w) in self.stack.weights:
            b += self.M * w.K * 2 + self.M * w.N * 2
        return b

    def input_bytes(self) -> int:
        return self.h0.numel() * 2

    def output_bytes(self) -> int:
        return self.logits.numel() * 2
