"""the scaled-up Q4_0 stack on 1..8 B200s.

32 layers, d_model 4096, 32 heads x 128, FFN 16384, vocab 31,500, seeded
N(0, 0.02) weights (x 1/sqrt(64) for attn_out and ffn_down), Q4_0-packed on the
device.  Two programs:

* `ColumnSplitDecode` -- decode at batch 64.  QKV and attn_out are replicated;
  ffn_up is column-split across the ranks (its GELU fused into the epilogue)
  and ffn_down is split along K with the same ranges, so each rank multiplies
  the ffn_up slice it produced by its rows of ffn_down, and one reduction per
  layer sums the partial products into the residual stream: a kernel reading
  the peers' partials over NVLink (aria_b200.p2p, the default) or an NCCL
  all-reduce.  The LM head is
  column-split (vocabulary rows of `embed`) and all-gathered once per step.
  Each rank quantises only its slices.
* batch-sharded prefill -- every rank holds the full replica and runs its own
  sequences (aria_b200.efkolos.DecodeProgram over the SCALED config).

The data flow between projections follows the reference's layer
(lold3344/ARIA src/transformer_cuda.rs:1059-1166): the residual stream h feeds
QKV and ffn_up, attn_out and ffn_down add into h.  Attention and LayerNorm are
outside this library: attn_out reads the first d_model columns of the QKV
output in place of the attention output, and h is not normalised.
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist

from . import dist as adist
from .efkolos import SCALED, EfkolosConfig, synth_f16
from .q4 import LAYOUT_KN, LAYOUT_NK, Q4Weight, matmul

FFN_ALIGN = 128  # ffn_up column / ffn_down row ranges: whole 128-k groups of the device layout


class ColumnSplitDecode:
    def __init__(self, cfg: EfkolosConfig = SCALED, M: int = 64, world: int = 1, rank: int = 0, group=None,
                 seed: int = 0, device="cuda", reduction: str = "p2p"):
        """reduction (world > 1): "p2p" -- one kernel per layer adds every rank's
        ffn_down partial into the residual stream, read over NVLink from the
        peers' memory (aria_b200.p2p); "nccl" -- NCCL all-reduce of the
        partials, then the residual add."""
        if reduction not in ("p2p", "nccl"):
            raise ValueError("reduction must be 'p2p' or 'nccl'")
        self.cfg, self.M, self.world, self.rank, self.group = cfg, M, world, rank, group
        self.reduction = reduction
        d, ff, V, L = cfg.d_model, cfg.ffn_dim, cfg.vocab_size, cfg.num_layers
        s, sd = 0.02, 0.02 / math.sqrt(2 * L)
        self.layers = []
        for i in range(L):
            base = seed * 1000003 + 10 * i
            qkv = Q4Weight.from_f16(synth_f16((d, 3 * d), s, base + 1, device), LAYOUT_KN)
            out = Q4Weight.from_f16(synth_f16((d, d), sd, base + 2, device), LAYOUT_KN)
            up_s = adist.ColumnSplit(LAYOUT_KN, d, ff, world, rank, align_to=FFN_ALIGN)
            dn_s = adist.RowSplit(LAYOUT_KN, ff, d, world, rank, align=FFN_ALIGN)
            assert up_s.cols == dn_s.rows
            # the full tensor is generated identically on every rank; each quantises its slice
            up = dn = None
            if up_s.cols[1] > up_s.cols[0]:
                up = Q4Weight.from_f16(up_s.slice_weight(synth_f16((d, ff), s, base + 3, device)), LAYOUT_KN)
                dn = Q4Weight.from_f16(dn_s.slice_weight(synth_f16((ff, d), sd, base + 4, device)), LAYOUT_KN)
            self.layers.append((qkv, out, up, dn))
        self.up_cols = adist.ColumnSplit(LAYOUT_KN, d, ff, world, rank, align_to=FFN_ALIGN).cols
        self.head_s = adist.ColumnSplit(LAYOUT_NK, d, V, world, rank)
        self.head = Q4Weight.from_f16(self.head_s.slice_weight(synth_f16((V, d), s, seed * 1000003 + 7, device)),
                                      LAYOUT_NK)
        self.h0 = synth_f16((M, d), 1.0, seed + 5, device)  # the step's input residual stream
        self.h = torch.empty(M, d, dtype=torch.float16, device=device)
        self.y_qkv = torch.empty(M, 3 * d, dtype=torch.float16, device=device)
        self.u = torch.empty(M, max(1, self.up_cols[1] - self.up_cols[0]), dtype=torch.float16, device=device)
        self.part = torch.empty(M, d, dtype=torch.float32, device=device)
        self.logits_l = torch.empty(M, self.head_s.cols[1] - self.head_s.cols[0], dtype=torch.float16, device=device)
        self.logits = torch.empty(M, V, dtype=torch.float16, device=device)
        self.p2p = None
        if world > 1 and reduction == "p2p":
            from .p2p import PeerReduction
            self.p2p = PeerReduction(M * d, L, group)
            self.parts = [self.p2p.part_tensor(i, (M, d)) for i in range(L)]

    def run(self) -> None:
        d = self.cfg.d_model
        self.h.copy_(self.h0)
        for i, (qkv, out, up, dn) in enumerate(self.layers):
            matmul(self.h, qkv, self.y_qkv, const_weights=True)
            matmul(self.y_qkv[:, :d], out, self.h, beta=1.0, const_weights=True)
            if self.world == 1:
                matmul(self.h, up, self.u, activation="gelu", const_weights=True)
                matmul(self.u, dn, self.h, beta=1.0, const_weights=True)
                continue
            part = self.parts[i] if self.p2p is not None else self.part
            if up is not None:
                matmul(self.h, up, self.u, activation="gelu", const_weights=True)
                matmul(self.u, dn, part, out_dtype=torch.float32, const_weights=True)
            else:
                part.zero_()
            if self.p2p is not None:
                self.p2p.reduce_into(i, self.h)  # h += every rank's partial, over peer memory
            else:
                dist.all_reduce(part, group=self.group)  # sum of the ranks' ffn_down partials (f32)
                self.h.add_(part)  # residual add, rounded once to f16
        matmul(self.h, self.head, self.logits_l, const_weights=True)
        if self.world == 1:
            self.logits.copy_(self.logits_l)
        else:
            adist.gather_columns(self.logits_l, self.cfg.vocab_size, self.world, self.head_s.align, self.group,
                                 out=self.logits)

    def weight_bytes(self) -> int:
        """Q4_0 bytes this rank streams per step."""
        b = 0
        for (q, o, u, dn) in self.layers:
            b += q.nbytes + o.nbytes + (u.nbytes + dn.nbytes if u is not None else 0)
        return b + self.head.nbytes

    def close(self) -> None:
        """Unmaps the peers' regions and frees this rank's (p2p reduction)."""
        if self.p2p is not None:
            self.parts = []
            self.p2p.close()
            self.p2p = None

    def collective_bytes(self) -> int:
        """Bytes each rank contributes to the collectives per step: one f32
        [M, d_model] reduction per layer and the f16 logits slice's all-gather."""
        if self.world == 1:
            return 0
        cfg = self.cfg
        W = adist.col_width(cfg.vocab_size, self.world, self.head_s.align)
        return cfg.num_layers * self.M * cfg.d_model * 4 + self.M * W * 2

    @property
    def collectives_per_step(self) -> int:
        return 0 if self.world == 1 else self.cfg.num_layers + 1
