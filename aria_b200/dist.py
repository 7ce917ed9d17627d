"""Multi-GPU layout of the Q4_0 projections: batch sharding and column splits.

One process per GPU (torch.distributed, NCCL over NVLink/NVSwitch on B200;
gloo in the CPU tests).  The reference runs on one device only
(lold3344/ARIA src/transformer_cuda.rs:83-103); these are the splits BASELINE
configs[2-4] ask for:

* batch sharding -- every rank holds a full weight replica and runs its own
  rows (sequences); no data-path collective;
* column split -- a projection's output columns are divided among ranks (each
  rank quantises only its slice), every rank computes its [M, N_r] part and an
  all-gather reassembles [M, N] in column order.  KN slices are aligned to the
  32-column Q4_0 blocks, so a rank's blocks are exactly the corresponding blocks
  of the full tensor; NK (LM head) slices are whole rows of `embed`;
* row split -- a projection's input features are divided among ranks and an
  all-reduce sums the partial products; after a column-split projection with
  the same ranges (ffn_up -> ffn_down) each rank already holds its input slice.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


def batch_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous rows [r0, r1) of `total` for `rank`; sizes differ by at most one."""
    base, extra = divmod(total, world)
    r0 = rank * base + min(rank, extra)
    return r0, r0 + base + (1 if rank < extra else 0)


def col_width(N: int, world: int, align: int) -> int:
    """Columns per rank (the last rank may hold fewer), a multiple of `align`."""
    w = -(-N // world)
    return -(-w // align) * align


def col_range(N: int, world: int, rank: int, align: int) -> tuple[int, int]:
    w = col_width(N, world, align)
    n0 = min(N, rank * w)
    return n0, min(N, n0 + w)


def assemble_columns(gathered: torch.Tensor, M: int, N: int, world: int, align: int) -> torch.Tensor:
    """[M, N] in column order from the rank-major result of an all-gather of
    every rank's [M, W] column slice (W = col_width; the last rank zero-padded)."""
    W = col_width(N, world, align)
    return gathered.view(world, M, W).permute(1, 0, 2).reshape(M, world * W)[:, :N]


def gather_columns(y_local: torch.Tensor, N: int, world: int, align: int, group=None,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """All-gather column slices [M, N_r] of every rank into [M, N] (column order).

    Each rank contributes a [M, W] buffer (W = col_width, zero-padded on the last
    rank) so the collective moves equal chunks; the rank-major result is
    reassembled by one strided copy."""
    M = y_local.shape[0]
    W = col_width(N, world, align)
    if y_local.shape[1] != W:
        padded = torch.zeros((M, W), dtype=y_local.dtype, device=y_local.device)
        padded[:, :y_local.shape[1]] = y_local
        y_local = padded
    gathered = torch.empty((world * M, W), dtype=y_local.dtype, device=y_local.device)
    dist.all_gather_into_tensor(gathered, y_local.contiguous(), group=group)
    full = assemble_columns(gathered, M, N, world, align)
    if out is None:
        return full.contiguous()
    out.copy_(full)
    return out


@dataclass
class ColumnSplit:
    """One rank's share of a column-split projection (its output features)."""

    layout: int
    K: int
    N: int
    world: int
    rank: int
    align_to: int = 0  # a coarser alignment than the block rule (0: none)

    @property
    def align(self) -> int:
        # KN: Q4_0 blocks run along n, so slices keep whole 32-column blocks.
        # NK: blocks run along k; any row split works, 16 keeps MMA tiles full.
        return max(32 if self.layout == 0 else 16, self.align_to)

    @property
    def cols(self) -> tuple[int, int]:
        return col_range(self.N, self.world, self.rank, self.align)

    def slice_weight(self, w_full: torch.Tensor) -> torch.Tensor:
        """This rank's part of the reference-oriented f16 weight: KN w[k][n] -> w[:, n0:n1],
        NK embed[n][k] -> embed[n0:n1, :]."""
        n0, n1 = self.cols
        return (w_full[:, n0:n1] if self.layout == 0 else w_full[n0:n1, :]).contiguous()


@dataclass
class RowSplit:
    """One rank's share of a projection split along K (its input features).

    Each rank multiplies its slice of the input by its rows of the weight and
    the ranks' partial products are summed (all-reduce).  Paired with a column
    split of the preceding projection (same ranges), the input slice is exactly
    what that rank produced, so the pair needs one collective instead of two.
    Ranges are multiples of `align` (a multiple of 128: the device layout pads K
    to 128, and NK blocks run along k)."""

    layout: int
    K: int
    N: int
    world: int
    rank: int
    align: int = 128

    @property
    def rows(self) -> tuple[int, int]:
        return col_range(self.K, self.world, self.rank, self.align)

    def slice_weight(self, w_full: torch.Tensor) -> torch.Tensor:
        """KN w[k][n] -> w[k0:k1, :], NK embed[n][k] -> embed[:, k0:k1]."""
        k0, k1 = self.rows
        return (w_full[k0:k1, :] if self.layout == 0 else w_full[:, k0:k1]).contiguous()
