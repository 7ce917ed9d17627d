"""the scaled-up Q4_0 stack on 1..8 B200s.

32 layers, d_model 4096, 32 heads x 128, FFN 16384, vocab 31,500, seeded
N(0, 0.02) weights (x 1/sqrt(64) for attn_out and ffn_down), Q4_0-packed on the
device.  Two programs:

* `ColumnSplitDecode` -- decode at batch 64 with ffn_up, ffn_down and the LM
  head column-split across the ranks (each rank quantises only its slice) and
  an NCCL all-gather reassembling every split output, which the next split
  projection consumes (ffn_up -> ffn_down); QKV and attn_out are replicated.
* batch-sharded prefill -- every rank holds the full replica and runs its own
  sequences (aria_b200.efkolos.DecodeProgram over the SCALED config).
"""
from __future__ import annotations

import math

import torch

from . import dist as adist
from .efkolos import SCALED, EfkolosConfig, synth_f16
from .q4 import LAYOUT_KN, LAYOUT_NK, Q4Weight, matmul


class ColumnSplitDecode:
    def __init__(self, cfg: EfkolosConfig = SCALED, M: int = 64, world: int = 1, rank: int = 0, group=None,
                 seed: int = 0, device="cuda"):
        self.cfg, self.M, self.world, self.rank, self.group = cfg, M, world, rank, group
        d, ff, V, L = cfg.d_model, cfg.ffn_dim, cfg.vocab_size, cfg.num_layers
        s, sd = 0.02, 0.02 / math.sqrt(2 * L)
        self.layers = []
        for i in range(L):
            base = seed * 1000003 + 10 * i
            qkv = Q4Weight.from_f16(synth_f16((d, 3 * d), s, base + 1, device), LAYOUT_KN)
            out = Q4Weight.from_f16(synth_f16((d, d), sd, base + 2, device), LAYOUT_KN)
            up_s = adist.ColumnSplit(LAYOUT_KN, d, ff, world, rank)
            dn_s = adist.ColumnSplit(LAYOUT_KN, ff, d, world, rank)
            # the full tensor is generated identically on every rank; each quantises its slice
            up = Q4Weight.from_f16(up_s.slice_weight(synth_f16((d, ff), s, base + 3, device)), LAYOUT_KN)
            dn = Q4Weight.from_f16(dn_s.slice_weight(synth_f16((ff, d), sd, base + 4, device)), LAYOUT_KN)
            self.layers.append((qkv, out, (up, up_s), (dn, dn_s)))
        self.head_s = adist.ColumnSplit(LAYOUT_NK, d, V, world, rank)
        self.head = Q4Weight.from_f16(self.head_s.slice_weight(synth_f16((V, d), s, seed * 1000003 + 7, device)),
                                      LAYOUT_NK)
        # activations: attention/LayerNorm/GELU are out of scope, so the inputs of
        # QKV and attn_out are synthetic; ffn_down consumes the gathered ffn_up output
        self.x = synth_f16((M, d), 1.0, seed + 5, device)
        self.y_qkv = torch.empty(M, 3 * d, dtype=torch.float16, device=device)
        self.y_out = torch.empty(M, d, dtype=torch.float16, device=device)
        self.y_up_l = torch.empty(M, up_s.cols[1] - up_s.cols[0], dtype=torch.float16, device=device)
        self.y_up = torch.empty(M, ff, dtype=torch.float16, device=device)
        self.y_dn_l = torch.empty(M, dn_s.cols[1] - dn_s.cols[0], dtype=torch.float16, device=device)
        self.y_dn = torch.empty(M, d, dtype=torch.float16, device=device)
        self.logits_l = torch.empty(M, self.head_s.cols[1] - self.head_s.cols[0], dtype=torch.float16, device=device)
        self.logits = torch.empty(M, V, dtype=torch.float16, device=device)

    def gather(self, y_local, N, align, out):
        if self.world == 1:
            out.copy_(y_local)
        else:
            adist.gather_columns(y_local, N, self.world, align, self.group, out=out)

    def run(self) -> None:
        cfg = self.cfg
        for (qkv, out, (up, up_s), (dn, dn_s)) in self.layers:
            matmul(self.x, qkv, self.y_qkv, const_weights=True)
            matmul(self.x, out, self.y_out, const_weights=True)
            matmul(self.x, up, self.y_up_l, const_weights=True)
            self.gather(self.y_up_l, cfg.ffn_dim, up_s.align, self.y_up)
            matmul(self.y_up, dn, self.y_dn_l, const_weights=True)
            self.gather(self.y_dn_l, cfg.d_model, dn_s.align, self.y_dn)
        matmul(self.y_dn, self.head, self.logits_l, const_weights=True)
        self.gather(self.logits_l, cfg.vocab_size, self.head_s.align, self.logits)

    def weight_bytes(self) -> int:
        """Q4_0 bytes this rank streams per step."""
        b = sum(q.nbytes + o.nbytes + u.nbytes + d.nbytes for (q, o, (u, _), (d, _)) in self.layers)
        return b + self.head.nbytes

    def gathered_bytes(self) -> int:
        """Bytes this rank receives from its peers per step through the all-gathers."""
        if self.world == 1:
            return 0
        cfg = self.cfg
        f = (self.world - 1) / self.world
        per_layer = self.M * (cfg.ffn_dim + cfg.d_model) * 2
        return int(f * (cfg.num_layers * per_layer + self.M * cfg.vocab_size * 2))
