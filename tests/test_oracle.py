"""The oracle itself: C restatement, numpy twin and golden vectors must agree.

These run without a GPU.  They pin the checker before it is used to judge the
CUDA kernels (reference: lold3344/ARIA src/transformer_cuda.rs:549-575)."""
import numpy as np
import pytest

from oracle import q4_oracle_np as npo


def _decode_input(case):
    raw = bytes.fromhex(case["input_hex"])
    if case["dtype"] == "f32":
        return np.frombuffer(raw, dtype=">u4").astype("<u4").view(np.float32)
    return np.frombuffer(raw, dtype=">u2").astype("<u2").view(np.float16)


def test_kat_numpy_twin(kat):
    for case in kat:
        x = _decode_input(case)
        got = npo.quantize_q4_0(x.astype(np.float32)).tobytes().hex()
        assert got == case["expected_hex"], case["name"]


def test_kat_c_oracle(kat, coracle):
    for case in kat:
        x = _decode_input(case)
        if case["dtype"] == "f16":
            got = coracle.quantize_q4_0_f16(x).tobytes().hex()
        else:
            got = coracle.quantize_q4_0(x).tobytes().hex()
        assert got == case["expected_hex"], case["name"]


def test_f16_conversion_matches_numpy(coracle):
    """The oracle's RNE f32->f16 equals numpy's IEEE conversion on edge values."""
    rng = np.random.default_rng(7)
    special = np.array([0.0, -0.0, 1.0, 65504.0, 65519.99, 65520.0, 1e9, -1e9, 2.0**-24,
                        2.0**-25, 2.0**-25 * 1.0001, 3 * 2.0**-26, 6.1e-5, 5.96e-8, np.inf, -np.inf],
                       dtype=np.float32)
    vals = np.concatenate([special, (rng.standard_normal(20000) * np.float32(10.0) ** rng.integers(-9, 6, 20000))
                           .astype(np.float32)])
    ref = vals.astype(np.float16).view(np.uint16)
    got = np.array([coracle.lib.q4o_f32_to_f16(float(v)) for v in vals], dtype=np.uint16)
    assert np.array_equal(got, ref)
    back = np.array([coracle.lib.q4o_f16_to_f32(int(h)) for h in ref[:4000]], dtype=np.float32)
    assert np.array_equal(back, ref[:4000].view(np.float16).astype(np.float32))


@pytest.mark.parametrize("n,sigma", [(1, 1.0), (31, 0.5), (32 * 1000 + 7, 0.02), (3584 * 896, 0.02)])
def test_c_vs_numpy_random(coracle, n, sigma):
    rng = np.random.default_rng(n)
    w = (rng.standard_normal(n) * sigma).astype(np.float16)
    a = coracle.quantize_q4_0_f16(w)
    b = npo.quantize_q4_0_f16(w)
    assert a.size == npo.packed_bytes(n)
    assert np.array_equal(a, b)
    # dequantisation agrees too
    assert np.array_equal(coracle.dequantize_q4_0(a, n), npo.dequantize_q4_0(b, n))


def test_c_vs_numpy_f32_extremes(coracle):
    rng = np.random.default_rng(11)
    x = (rng.standard_normal(32 * 64) * np.float32(10.0) ** rng.integers(-30, 30, 32 * 64)).astype(np.float32)
    x[::97] = np.nan
    x[5::131] = np.inf
    x[7::211] = -np.inf
    assert np.array_equal(coracle.quantize_q4_0(x), npo.quantize_q4_0(x))


def test_projection_fixtures(projection_fixtures, coracle):
    for c in projection_fixtures:
        w = np.frombuffer(bytes.fromhex(c["w_f16_hex"]), dtype="<u2").view(np.float16)
        x = np.frombuffer(bytes.fromhex(c["x_f16_hex"]), dtype="<u2").view(np.float16)
        blocks = npo.quantize_q4_0_f16(w)
        assert blocks.tobytes().hex() == c["blocks_hex"]
        y_np = npo.matmul_ref(blocks, c["layout"], c["K"], c["N"], x)
        y_c = coracle.matmul_ref(blocks, c["layout"], c["K"], c["N"], x)
        y_gold = np.array(c["y_f64"]).reshape(c["M"], c["N"])
        np.testing.assert_allclose(y_np, y_gold, rtol=1e-12, atol=1e-12)
        np.testing.assert_allclose(y_c, y_gold, rtol=1e-12, atol=1e-12)


def test_baseline_projection_matches_reference(coracle):
    """The timed CPU baseline (f32, i-p-j) stays within tolerance of the fp64 reference."""
    for layout in (0, 1):
        K, N, M = 256, 192, 2
        rng = np.random.default_rng(layout)
        w = (rng.standard_normal(K * N) * 0.02).astype(np.float16)
        x = rng.standard_normal((M, K)).astype(np.float16)
        blocks = coracle.quantize_q4_0_f16(w)
        y = np.zeros((M, N), dtype=np.float32)
        ws = np.zeros(K * N, dtype=np.float32)
        xs = np.zeros(M * K, dtype=np.float32)
        coracle.baseline_projection(blocks, layout, K, N, x, ws, xs, y, 2)
        ref = coracle.matmul_ref(blocks, layout, K, N, x)
        np.testing.assert_allclose(y, ref, rtol=1e-4, atol=1e-5)


def test_gelu_tanh_restatement():
    """The oracle's GELU is the reference's tanh form (src/kernels.cu:574-583)."""
    import math
    from oracle.q4_oracle_np import gelu_tanh
    xs = np.array([-6.0, -3.0, -1.0, -0.5, 0.0, 0.25, 1.0, 2.0, 8.0])
    want = [0.5 * v * (1.0 + math.tanh(0.7978845608 * (v + 0.044715 * v ** 3))) for v in xs]
    assert np.allclose(gelu_tanh(xs), want, rtol=0, atol=1e-15)
    assert gelu_tanh(0.0) == 0.0 and abs(gelu_tanh(8.0) - 8.0) < 1e-12 and abs(gelu_tanh(-8.0)) < 1e-12
    # within 1e-3 of the exact erf GELU over [-4, 4] (the approximation's published accuracy)
    grid = np.linspace(-4, 4, 801)
    exact = np.array([0.5 * v * (1.0 + math.erf(v / math.sqrt(2.0))) for v in grid])
    assert np.max(np.abs(gelu_tanh(grid) - exact)) < 1e-3


@pytest.mark.parametrize("layout,K,N", [(npo.LAYOUT_KN, 96, 64), (npo.LAYOUT_KN, 256, 352),
                                        (npo.LAYOUT_NK, 128, 37), (npo.LAYOUT_NK, 64, 300)])
def test_dequantize_columns_matches_full_dequantisation(coracle, layout, K, N):
    """The column-sampling dequantiser used by the sampled parity tests equals
    slicing the full dequantisation, in both orientations."""
    rng = np.random.default_rng(K + N)
    shape = (K, N) if layout == npo.LAYOUT_KN else (N, K)
    w = (rng.standard_normal(shape) * 0.05).astype(np.float16)
    blocks = coracle.quantize_q4_0_f16(w.reshape(-1))
    full = npo.dequantize_q4_0(blocks, K * N).reshape(shape)
    W = full if layout == npo.LAYOUT_KN else full.T
    cols = rng.choice(N, min(N, 29), replace=False)
    cols[0] = N - 1
    assert np.array_equal(npo.dequantize_columns(blocks, layout, K, N, cols), W[:, cols])
