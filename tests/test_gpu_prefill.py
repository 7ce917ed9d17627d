"""GPU parity of the prefill path (M > 32 tokens -> tcgen05 kernel).

Reference: the oracle's exact dequantisation of the GGUF Q4_0 blocks
(lold3344/ARIA src/transformer_cuda.rs:549-575 inverted), multiplied in fp64.
Tolerance: max-abs 1e-2 and relative L2 1e-3."""
import numpy as np
import pytest
import torch

from tests.gpu_helpers import LAYOUT_KN, LAYOUT_NK, check_close

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]


@pytest.fixture(scope="module")
def q4():
    from aria_b200 import q4 as q4mod
    return q4mod


def _weights(coracle, layout, K, N, seed, sigma=0.02):
    rng = np.random.default_rng(seed)
    shape = (K, N) if layout == LAYOUT_KN else (N, K)
    w = (rng.standard_normal(shape) * sigma).astype(np.float16)
    blocks = coracle.quantize_q4_0_f16(w.reshape(-1))
    wd = coracle.dequantize_q4_0(blocks, K * N).astype(np.float64).reshape(shape)
    W = wd if layout == LAYOUT_KN else wd.T  # [K][N]
    return w, blocks, W


def _run(q4, w, layout, x, out_dtype=torch.float16, bias=None, alpha=1.0, beta=0.0, y0=None, kernel="auto"):
    wq = q4.Q4Weight.from_f16(torch.from_numpy(w).cuda(), layout)
    xt = torch.from_numpy(x).cuda()
    out = torch.from_numpy(y0).to(out_dtype).cuda() if y0 is not None else None
    bt = torch.from_numpy(bias).cuda() if bias is not None else None
    y = q4.matmul(xt, wq, out, bias=bt, alpha=alpha, beta=beta, out_dtype=out_dtype, kernel=kernel)
    torch.cuda.synchronize()
    return y.cpu().to(torch.float64).numpy()


EFKOLOS = [("qkv", LAYOUT_KN, 896, 2688), ("attn_out", LAYOUT_KN, 896, 896), ("ffn_up", LAYOUT_KN, 896, 3584),
           ("ffn_down", LAYOUT_KN, 3584, 896), ("lm_head", LAYOUT_NK, 896, 31500)]


@pytest.mark.parametrize("name,layout,K,N", EFKOLOS)
@pytest.mark.parametrize("M", [33, 64, 100, 256, 300])
def test_prefill_projections(q4, coracle, name, layout, K, N, M):
    w, blocks, W = _weights(coracle, layout, K, N, seed=K + N + M)
    rng = np.random.default_rng(M)
    x = rng.standard_normal((M, K)).astype(np.float16)
    b = (rng.standard_normal(N) * 0.1).astype(np.float16)
    y = _run(q4, w, layout, x, bias=b)
    ref = x.astype(np.float64) @ W + b.astype(np.float64)
    check_close(y, ref, what=f"{name} M={M}")


@pytest.mark.parametrize("layout,K,N,M", [(LAYOUT_KN, 32, 32, 40), (LAYOUT_KN, 160, 64, 129), (LAYOUT_NK, 96, 37, 65),
                                          (LAYOUT_NK, 224, 130, 257), (LAYOUT_KN, 4096, 256, 70),
                                          (LAYOUT_NK, 1056, 200, 33)])
def test_prefill_odd_shapes(q4, coracle, layout, K, N, M):
    w, blocks, W = _weights(coracle, layout, K, N, seed=7 * K + N)
    x = np.random.default_rng(1).standard_normal((M, K)).astype(np.float16)
    y = _run(q4, w, layout, x, out_dtype=torch.float32)
    check_close(y, x.astype(np.float64) @ W, what=f"odd {layout} {K}x{N} M={M}")


def test_prefill_alpha_beta(q4, coracle):
    w, blocks, W = _weights(coracle, LAYOUT_NK, 896, 640, seed=3)
    rng = np.random.default_rng(4)
    x = rng.standard_normal((96, 896)).astype(np.float16)
    y0 = rng.standard_normal((96, 640)).astype(np.float32)
    y = _run(q4, w, LAYOUT_NK, x, out_dtype=torch.float32, alpha=0.5, beta=0.25, y0=y0)
    check_close(y, 0.5 * (x.astype(np.float64) @ W) + 0.25 * y0, what="alpha/beta")


@pytest.mark.parametrize("name,layout,K,N", [EFKOLOS[2], EFKOLOS[3], EFKOLOS[4]])
def test_prefill_full_size_sampled_rows(q4, coracle, name, layout, K, N):
    """BASELINE config 3 (M = 4096 tokens): every output row computed on the GPU,
    a seeded sample of 48 rows checked against fp64."""
    M = 4096
    w, blocks, W = _weights(coracle, layout, K, N, seed=11)
    x = np.random.default_rng(12).standard_normal((M, K)).astype(np.float16)
    y = _run(q4, w, layout, x)
    rows = np.random.default_rng(13).choice(M, 48, replace=False)
    rows[:2] = [0, M - 1]
    check_close(y[rows], x[rows].astype(np.float64) @ W, what=f"{name} M=4096 sampled")
    assert np.isfinite(y).all()


@pytest.mark.parametrize("layout,K,N,M", [
    (LAYOUT_KN, 256, 1152, 4096),   # 9 row tiles: 256-token tiles fit one round of CTAs (single accumulator)
    (LAYOUT_NK, 320, 896, 4096),    # 7 row tiles: 224-token tiles (single accumulator)
    (LAYOUT_KN, 224, 896, 8192),    # two rounds of 224-token tiles
    (LAYOUT_NK, 256, 3584, 4096),   # 192-token tiles, double-buffered accumulators
    (LAYOUT_KN, 192, 640, 128),     # 128-token tiles
])
def test_prefill_token_tile_variants(q4, coracle, layout, K, N, M):
    """Every token-tile height the launcher can choose, with sampled rows
    (first, last and a seeded sample) checked against fp64."""
    w, blocks, W = _weights(coracle, layout, K, N, seed=K + 3 * N + M)
    x = np.random.default_rng(M + N).standard_normal((M, K)).astype(np.float16)
    y = _run(q4, w, layout, x, out_dtype=torch.float32)
    rows = np.random.default_rng(5).choice(M, min(M, 64), replace=False)
    rows[:2] = [0, M - 1]
    check_close(y[rows], x[rows].astype(np.float64) @ W, what=f"BT variant {layout} {K}x{N} M={M}")


@pytest.mark.parametrize("M", [1, 8, 33, 64])
@pytest.mark.parametrize("layout,K,N", [(LAYOUT_KN, 896, 2688), (LAYOUT_NK, 1056, 300)])
def test_tensor_kernel_small_m(q4, coracle, layout, K, N, M):
    """ARIA_Q4_FLAG_KERNEL_TENSOR: the tcgen05 kernel at decode-sized M (token
    rows past M are zero-filled by the tensor map and never stored)."""
    w, blocks, W = _weights(coracle, layout, K, N, seed=M + 17)
    x = np.random.default_rng(M).standard_normal((M, K)).astype(np.float16)
    b = (np.random.default_rng(M + 1).standard_normal(N) * 0.1).astype(np.float16)
    y = _run(q4, w, layout, x, bias=b, kernel="tensor")
    check_close(y, x.astype(np.float64) @ W + b.astype(np.float64), what=f"tensor M={M}")


@pytest.mark.parametrize("layout,K,N,M", [
    (LAYOUT_KN, 16384, 512, 64),    # 4 row tiles, 128 groups of k: deep K split
    (LAYOUT_NK, 3584, 896, 64),     # the Efkolos ffn_down shape at batch 64
    (LAYOUT_KN, 3584, 896, 40),
    (LAYOUT_NK, 4096, 300, 100),    # ragged N, 128-token tiles
    (LAYOUT_KN, 8224, 256, 50),     # K % 128 != 0: the last slice holds the padded tail
])
def test_split_k_through_workspace(q4, coracle, layout, K, N, M):
    """aria_q4_0_matmul_ws: few output tiles, long K -> work units over K
    slices, partials in the workspace, the last unit of each tile adds them in
    slice order.  Two calls in a row (the second relies on the first leaving its
    counters at zero) give identical bits; both are within tolerance of fp64."""
    from aria_b200 import _lib
    assert _lib.lib().aria_q4_0_workspace_bytes(K, N, M) > 0, "shape should split K"
    w, blocks, W = _weights(coracle, layout, K, N, seed=K + N + 5 * M)
    x = np.random.default_rng(M + 7).standard_normal((M, K)).astype(np.float16)
    b = (np.random.default_rng(M + 8).standard_normal(N) * 0.1).astype(np.float16)
    wq = q4.Q4Weight.from_f16(torch.from_numpy(w).cuda(), layout)
    xt, bt = torch.from_numpy(x).cuda(), torch.from_numpy(b).cuda()
    ws = torch.zeros(int(_lib.lib().aria_q4_0_workspace_bytes(K, N, M)), dtype=torch.uint8, device="cuda")
    y1 = q4.matmul(xt, wq, bias=bt, out_dtype=torch.float32, kernel="tensor", workspace=ws)
    y2 = q4.matmul(xt, wq, bias=bt, out_dtype=torch.float32, kernel="tensor", workspace=ws)
    y0 = q4.matmul(xt, wq, bias=bt, out_dtype=torch.float32, kernel="tensor", workspace=None)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2)
    ref = x.astype(np.float64) @ W + b.astype(np.float64)
    check_close(y1.cpu().numpy(), ref, what=f"split-K {layout} {K}x{N} M={M}")
    check_close(y0.cpu().numpy(), ref, what=f"unsplit {layout} {K}x{N} M={M}")


def test_one_workspace_serves_any_shape_sequence(q4, coracle):
    """Auto workspace (one cached buffer per device and stream) across shapes
    with different tile counts and splits, in both orders."""
    shapes = [(LAYOUT_KN, 896, 2688, 40), (LAYOUT_KN, 896, 896, 33), (LAYOUT_KN, 16384, 512, 64),
              (LAYOUT_NK, 3584, 896, 64), (LAYOUT_KN, 896, 896, 33), (LAYOUT_KN, 896, 2688, 40)]
    for layout, K, N, M in shapes:
        w, blocks, W = _weights(coracle, layout, K, N, seed=N + M)
        x = np.random.default_rng(M).standard_normal((M, K)).astype(np.float16)
        y = _run(q4, w, layout, x, out_dtype=torch.float32)
        check_close(y, x.astype(np.float64) @ W, what=f"sequence {layout} {K}x{N} M={M}")


def test_no_device_error_recorded(q4):
    from aria_b200 import _lib
    assert _lib.lib().aria_q4_take_device_error() == 0


CONFIG4 = [("ffn_up", LAYOUT_KN, 4096, 16384), ("ffn_down", LAYOUT_KN, 16384, 4096),
           ("lm_head", LAYOUT_NK, 4096, 31500)]


@pytest.mark.parametrize("name,layout,K,N", CONFIG4)
@pytest.mark.parametrize("M", [64, 4096])
def test_config4_full_shape_sampled(q4, coracle, name, layout, K, N, M):
    """BASELINE config 4 projections at their full shapes: M = 4096 (prefill,
    tcgen05 kernel) and M = 64 (batched decode through the auto workspace, so
    K is split where the planner splits it).  The weight is uploaded as GGUF
    blocks (repack at full size).  The GPU computes every output; a seeded
    sample of rows x columns (first and last of each included) is checked
    against the fp64 oracle."""
    from aria_b200 import _lib
    from tests.gpu_helpers import sample_columns, sampled_ref
    rng = np.random.default_rng(K + N + M)
    shape = (K, N) if layout == LAYOUT_KN else (N, K)
    w = (rng.standard_normal(shape, dtype=np.float32) * 0.02).astype(np.float16)
    blocks = coracle.quantize_q4_0_f16(w.reshape(-1))
    del w
    x = rng.standard_normal((M, K), dtype=np.float32).astype(np.float16)
    wq = q4.Q4Weight.from_gguf_blocks(torch.from_numpy(blocks).cuda(), layout, K, N)
    if M == 64:
        ws = int(_lib.lib().aria_q4_0_workspace_bytes(K, N, M))
        assert _lib.lib().aria_q4_0_kernel_choice(layout, K, N, M, ws, 0) == 3  # tcgen05
    y = q4.matmul(torch.from_numpy(x).cuda(), wq)
    torch.cuda.synchronize()
    rows = np.unique(np.concatenate([[0, M - 1], np.random.default_rng(M).choice(M, min(M, 48), replace=False)]))
    cols = sample_columns(N, 512, seed=N)
    got = y[torch.from_numpy(rows).cuda()][:, torch.from_numpy(cols).cuda()].cpu().to(torch.float64).numpy()
    check_close(got, sampled_ref(blocks, layout, K, N, x[rows], cols), what=f"config4 {name} M={M}")
    assert bool(torch.isfinite(y).all())
