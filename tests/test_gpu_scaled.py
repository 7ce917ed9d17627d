"""GPU parity of the multi-GPU layouts of BASELINE configs[4], on one GPU.

* `ColumnSplitDecode` at world = 1 (the program the scaled bench runs) on a
  reduced stack, its logits against the fp64 oracle chain with the same f16
  rounding points (QKV out, residual adds, GELU(ffn_up) out, logits);
* every rank's share of the ffn_up column split / ffn_down K split and of the
  LM-head column split for world = 2, 4 and 8, each run on this GPU: the summed
  ffn_down partials and the reassembled logits (the all-gather's index math,
  aria_b200.dist.assemble_columns) against the full projections.

Reference: dequantise-then-matmul of the Q4_0 blocks (lold3344/ARIA
src/transformer_cuda.rs:549-575 inverted, :3322-3333); tolerance max-abs 1e-2,
relative L2 1e-3."""
import math

import numpy as np
import pytest
import torch

from tests.gpu_helpers import LAYOUT_KN, LAYOUT_NK, check_close, sample_columns, sampled_ref

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]


def _f16(a):
    return np.asarray(a, dtype=np.float64).astype(np.float16).astype(np.float64)


def _dequant(coracle, w16, layout):
    """(blocks, W[K][N] f64) of an f16 weight in the reference orientation."""
    blocks = coracle.quantize_q4_0_f16(w16.reshape(-1))
    K, N = (w16.shape[0], w16.shape[1]) if layout == LAYOUT_KN else (w16.shape[1], w16.shape[0])
    wd = coracle.dequantize_q4_0(blocks, K * N).astype(np.float64).reshape(w16.shape)
    return blocks, (wd if layout == LAYOUT_KN else wd.T)


@pytest.mark.parametrize("M", [8, 64])
def test_column_split_decode_world1_chain(coracle, M):
    from oracle.q4_oracle_np import gelu_tanh
    from aria_b200.efkolos import EfkolosConfig, synth_f16
    from aria_b200.scaled import ColumnSplitDecode
    cfg = EfkolosConfig(num_layers=2, d_model=512, num_heads=8, ffn_dim=2048, vocab_size=1000)
    seed = 3
    prog = ColumnSplitDecode(cfg, M=M, world=1, rank=0, seed=seed)
    prog.run()
    torch.cuda.synchronize()
    got = prog.logits.cpu().to(torch.float64).numpy()
    # the same synthetic tensors, regenerated on the device and brought to the host
    d, ff, V, L = cfg.d_model, cfg.ffn_dim, cfg.vocab_size, cfg.num_layers
    s, sd = 0.02, 0.02 / math.sqrt(2 * L)
    h = prog.h0.cpu().numpy().astype(np.float64)
    for i in range(L):
        base = seed * 1000003 + 10 * i
        Wq = _dequant(coracle, synth_f16((d, 3 * d), s, base + 1).cpu().numpy(), LAYOUT_KN)[1]
        Wo = _dequant(coracle, synth_f16((d, d), sd, base + 2).cpu().numpy(), LAYOUT_KN)[1]
        Wu = _dequant(coracle, synth_f16((d, ff), s, base + 3).cpu().numpy(), LAYOUT_KN)[1]
        Wd = _dequant(coracle, synth_f16((ff, d), sd, base + 4).cpu().numpy(), LAYOUT_KN)[1]
        qkv = _f16(h @ Wq)
        h = _f16(h + qkv[:, :d] @ Wo)
        u = _f16(gelu_tanh(h @ Wu))
        h = _f16(h + u @ Wd)
    E = _dequant(coracle, synth_f16((V, d), s, seed * 1000003 + 7).cpu().numpy(), LAYOUT_NK)[1]
    check_close(got, h @ E, what=f"column-split program, world 1, M={M}")


@pytest.mark.parametrize("world", [2, 4, 8])
def test_rank_slices_reassemble(coracle, world):
    """Each rank's slices computed on this GPU; partial sums and gathered
    columns must equal the full projections."""
    from oracle.q4_oracle_np import gelu_tanh
    from aria_b200 import dist as adist
    from aria_b200.q4 import Q4Weight, matmul
    from aria_b200.scaled import FFN_ALIGN
    d, ff, V, M = 1024, 4096, 31500, 64
    rng = np.random.default_rng(world)
    up = (rng.standard_normal((d, ff), dtype=np.float32) * 0.02).astype(np.float16)
    dn = (rng.standard_normal((ff, d), dtype=np.float32) * 0.02).astype(np.float16)
    emb = (rng.standard_normal((V, d), dtype=np.float32) * 0.02).astype(np.float16)
    h = rng.standard_normal((M, d), dtype=np.float32).astype(np.float16)
    ht = torch.from_numpy(h).cuda()
    part_sum = torch.zeros(M, d, dtype=torch.float32, device="cuda")
    hs = adist.ColumnSplit(LAYOUT_NK, d, V, world, 0)
    W = adist.col_width(V, world, hs.align)
    gathered = torch.zeros(world * M, W, dtype=torch.float16, device="cuda")
    for r in range(world):
        us = adist.ColumnSplit(LAYOUT_KN, d, ff, world, r, align_to=FFN_ALIGN)
        ds = adist.RowSplit(LAYOUT_KN, ff, d, world, r, align=FFN_ALIGN)
        assert us.cols == ds.rows
        wu = Q4Weight.from_f16(us.slice_weight(torch.from_numpy(up).cuda()), LAYOUT_KN)
        wd = Q4Weight.from_f16(ds.slice_weight(torch.from_numpy(dn).cuda()), LAYOUT_KN)
        u_r = matmul(ht, wu, activation="gelu")
        part_sum += matmul(u_r, wd, out_dtype=torch.float32)
        hr = adist.ColumnSplit(LAYOUT_NK, d, V, world, r)
        n0, n1 = hr.cols
        we = Q4Weight.from_f16(hr.slice_weight(torch.from_numpy(emb).cuda()), LAYOUT_NK)
        gathered[r * M:(r + 1) * M, :n1 - n0] = matmul(ht, we)
    logits = adist.assemble_columns(gathered, M, V, world, hs.align)
    torch.cuda.synchronize()
    Wu = _dequant(coracle, up, LAYOUT_KN)[1]
    Wd = _dequant(coracle, dn, LAYOUT_KN)[1]
    u_ref = _f16(gelu_tanh(h.astype(np.float64) @ Wu))
    check_close(part_sum.cpu().numpy(), u_ref @ Wd, what=f"ffn pair, world {world}")
    cols = sample_columns(V, 512, seed=world)
    eblocks = coracle.quantize_q4_0_f16(emb.reshape(-1))
    check_close(logits.cpu().to(torch.float64).numpy()[:, cols], sampled_ref(eblocks, LAYOUT_NK, d, V, h, cols),
                what=f"LM head gather, world {world}")
