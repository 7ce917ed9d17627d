"""GPU parity tests: the CUDA kernels behind the C ABI against the CPU oracle.

Bit-exact for packed bytes (lold3344/ARIA src/transformer_cuda.rs:549-575);
projection outputs within max-abs 1e-2 and relative L2 1e-3 of the fp64
dequantise-then-matmul reference (:3322-3333, :1864)."""
import numpy as np
import pytest
import torch

from oracle import q4_oracle_np as npo
from tests.gpu_helpers import (LAYOUT_KN, LAYOUT_NK, check_close, run_projection, sample_columns, tiled_from_aos,
                               tiled_regions)

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]


@pytest.fixture(scope="module")
def q4():
    from aria_b200 import q4 as q4mod
    return q4mod


def _decode_input(case):
    raw = bytes.fromhex(case["input_hex"])
    if case["dtype"] == "f32":
        return np.frombuffer(raw, dtype=">u4").astype("<u4").view(np.float32)
    return np.frombuffer(raw, dtype=">u2").astype("<u2").view(np.float16)


# ------------------------------------------------------------------ packer

def test_pack_known_answers(q4, kat):
    for case in kat:
        x = _decode_input(case).copy()
        got = q4.quantize_q4_0(torch.from_numpy(x).cuda()).cpu().numpy().tobytes().hex()
        assert got == case["expected_hex"], case["name"]
        if case["dtype"] == "f16":  # the f32 entry point on the widened values too
            got32 = q4.quantize_q4_0(torch.from_numpy(x.astype(np.float32)).cuda()).cpu().numpy()
            assert got32.tobytes().hex() == case["expected_hex"], case["name"] + " (f32)"


@pytest.mark.parametrize("n", [1, 31, 32, 33, 32 * 1000 + 7, 3584 * 896, 896 * 2688 + 5])
def test_pack_random_bit_exact(q4, coracle, n):
    rng = np.random.default_rng(n)
    w = (rng.standard_normal(n) * 0.02).astype(np.float16)
    got = q4.quantize_q4_0(torch.from_numpy(w).cuda()).cpu().numpy()
    ref = coracle.quantize_q4_0_f16(w)
    assert got.size == ref.size == npo.packed_bytes(n)
    assert np.array_equal(got, ref)


def test_pack_f32_extremes_bit_exact(q4, coracle):
    rng = np.random.default_rng(5)
    x = (rng.standard_normal(32 * 4096) * np.float32(10.0) ** rng.integers(-40, 38, 32 * 4096)).astype(np.float32)
    x[::97] = np.nan
    x[5::131] = np.inf
    x[7::211] = -np.inf
    x[64:96] = 0.0
    x[96:128] = -0.0
    got = q4.quantize_q4_0(torch.from_numpy(x).cuda()).cpu().numpy()
    assert np.array_equal(got, coracle.quantize_q4_0(x))


def test_unpack_exact(q4, coracle):
    n = 32 * 777 + 13
    rng = np.random.default_rng(9)
    w = (rng.standard_normal(n) * 0.3).astype(np.float16)
    blocks = coracle.quantize_q4_0_f16(w)
    got = q4.dequantize_q4_0(torch.from_numpy(blocks).cuda(), n).cpu().numpy()
    assert np.array_equal(got, coracle.dequantize_q4_0(blocks, n))


# ------------------------------------------------------------------ device form

SHAPES = [(LAYOUT_KN, 32, 32), (LAYOUT_KN, 64, 96), (LAYOUT_KN, 160, 64), (LAYOUT_KN, 896, 2688),
          (LAYOUT_KN, 3584, 896), (LAYOUT_NK, 32, 1), (LAYOUT_NK, 96, 37), (LAYOUT_NK, 224, 40),
          (LAYOUT_NK, 896, 3584), (LAYOUT_NK, 896, 31500)]


@pytest.mark.parametrize("layout,K,N", SHAPES)
def test_repack_and_quantize_tiled(q4, coracle, layout, K, N):
    rng = np.random.default_rng(K * 7 + N)
    shape = (K, N) if layout == LAYOUT_KN else (N, K)
    w = (rng.standard_normal(shape) * 0.02).astype(np.float16)
    blocks = coracle.quantize_q4_0_f16(w.reshape(-1))
    expect = tiled_from_aos(blocks, layout, K, N)
    wq = q4.Q4Weight.from_gguf_blocks(torch.from_numpy(blocks).cuda(), layout, K, N)
    assert wq.buf.numel() == expect.size
    eq, es = tiled_regions(expect, K, N)
    gq, gs = tiled_regions(wq.buf.cpu().numpy(), K, N)
    assert np.array_equal(gq, eq), "repack codes"
    assert np.array_equal(gs, es), "repack scales"
    wq2 = q4.Q4Weight.from_f16(torch.from_numpy(w).cuda(), layout)
    gq2, gs2 = tiled_regions(wq2.buf.cpu().numpy(), K, N)
    assert np.array_equal(gq2, eq), "quantize_tiled codes"
    assert np.array_equal(gs2, es), "quantize_tiled scales"


# ------------------------------------------------------------------ projections

_run = run_projection


def test_config0_single_projection(q4, coracle):
    """ffn_up-shaped W[3584x896] NK, x[896] -> y[3584] fp32."""
    y, ref = _run(q4, coracle, LAYOUT_NK, 896, 3584, 1)
    check_close(y, ref, what="config0")


EFKOLOS = [("qkv", LAYOUT_KN, 896, 2688), ("attn_out", LAYOUT_KN, 896, 896), ("ffn_up", LAYOUT_KN, 896, 3584),
           ("ffn_down", LAYOUT_KN, 3584, 896), ("lm_head", LAYOUT_NK, 896, 31500)]


@pytest.mark.parametrize("name,layout,K,N", EFKOLOS)
@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 8, 16, 24, 32, 40, 64])
def test_efkolos_projections(q4, coracle, name, layout, K, N, M):
    """Every Efkolos projection through the default kernel routing.  The LM head
    (31,500 outputs) at M > 4 is checked on a seeded sample of 384 output columns
    (first and last included): the GPU computes all of them, the fp64 oracle only
    the sample."""
    cols = sample_columns(N, 384, seed=M) if (name == "lm_head" and M > 4) else None
    y, ref = _run(q4, coracle, layout, K, N, M, out_dtype=torch.float16, bias=True, cols=cols)
    check_close(y, ref, what=f"{name} M={M}")


@pytest.mark.parametrize("layout,K,N,M", [(LAYOUT_KN, 32, 32, 1), (LAYOUT_KN, 32, 32, 3), (LAYOUT_KN, 32, 32, 17),
                                          (LAYOUT_NK, 32, 1, 1), (LAYOUT_NK, 64, 33, 17), (LAYOUT_NK, 1056, 5, 2),
                                          (LAYOUT_KN, 4096, 64, 3), (LAYOUT_NK, 4096, 100, 1)])
def test_odd_shapes(q4, coracle, layout, K, N, M):
    y, ref = _run(q4, coracle, layout, K, N, M)
    check_close(y, ref, what=f"odd {layout} {K}x{N} M={M}")


@pytest.mark.parametrize("layout,K,N,M", [(LAYOUT_KN, 32, 1056, 64), (LAYOUT_KN, 128, 1056, 33),
                                          (LAYOUT_KN, 256, 1056, 64), (LAYOUT_KN, 384, 2048, 48),
                                          (LAYOUT_NK, 128, 1057, 64), (LAYOUT_NK, 640, 1301, 40),
                                          (LAYOUT_KN, 4096, 2048, 64)])
def test_tensor_path_group_parities(q4, coracle, layout, K, N, M):
    """64-token tiles take two MMA issuers, each accumulating the 128-k groups of
    one parity; the epilogue adds both, or reads the only one present when a
    work unit holds a single group.  Units of one, two and three groups, odd N
    (NK), and a K split, all on the tensor-core kernel."""
    from aria_b200 import _lib
    lib = _lib.lib()
    ws = int(lib.aria_q4_0_workspace_bytes(K, N, M))
    assert lib.aria_q4_0_kernel_choice(layout, K, N, M, ws, 0) == 3
    y, ref = _run(q4, coracle, layout, K, N, M, out_dtype=torch.float16, bias=True)
    check_close(y, ref, what=f"tensor {layout} {K}x{N} M={M}")


def test_alpha_beta(q4, coracle):
    y, ref = _run(q4, coracle, LAYOUT_KN, 896, 896, 2, alpha=0.5, beta=0.25)
    check_close(y, ref, what="alpha/beta")
    y, ref = _run(q4, coracle, LAYOUT_NK, 896, 640, 1, out_dtype=torch.float16, alpha=1 / 29.93, beta=1.0, bias=True)
    check_close(y, ref, what="alpha/beta f16")


def test_golden_projection_fixtures(q4, projection_fixtures):
    for c in projection_fixtures:
        K, N, M, layout = c["K"], c["N"], c["M"], c["layout"]
        blocks = np.frombuffer(bytes.fromhex(c["blocks_hex"]), dtype=np.uint8).copy()
        x = np.frombuffer(bytes.fromhex(c["x_f16_hex"]), dtype="<u2").view(np.float16).reshape(M, K).copy()
        wq = q4.Q4Weight.from_gguf_blocks(torch.from_numpy(blocks).cuda(), layout, K, N)
        y = q4.matmul(torch.from_numpy(x).cuda(), wq, out_dtype=torch.float32).cpu().numpy()
        check_close(y, np.array(c["y_f64"]).reshape(M, N), what=f"golden {layout} {K}x{N}")


def test_errors_are_raised(q4):
    from aria_b200._lib import AriaQ4Error
    w = q4.Q4Weight.from_f16(torch.zeros(64, 64, dtype=torch.float16, device="cuda"), LAYOUT_KN)
    x = torch.zeros(1, 72, dtype=torch.float16, device="cuda")[:, 1:65]  # 2-byte offset: misaligned
    with pytest.raises(AriaQ4Error) as ei:
        q4.matmul(x, w)
    assert ei.value.status == 3
    with pytest.raises(AriaQ4Error) as ei:
        q4.Q4Weight.from_f16(torch.zeros(64, 48, dtype=torch.float16, device="cuda"), LAYOUT_KN)
    assert ei.value.status == 2


@pytest.mark.parametrize("name,layout,K,N", EFKOLOS)
def test_const_weights_flag_same_result(q4, name, layout, K, N):
    """aria_q4_0_matmul_ex with ARIA_Q4_FLAG_CONST_WEIGHTS computes exactly what
    aria_q4_0_matmul computes (only the load schedule differs)."""
    from aria_b200.efkolos import synth_f16
    shape = (K, N) if layout == LAYOUT_KN else (N, K)
    wq = q4.Q4Weight.from_f16(synth_f16(shape, 0.02, 3), layout)
    for M in (1, 3, 16):
        x = synth_f16((M, K), 1.0, 4)
        torch.cuda.synchronize()
        a = q4.matmul(x, wq, out_dtype=torch.float32)
        b = q4.matmul(x, wq, out_dtype=torch.float32, const_weights=True)
        torch.cuda.synchronize()
        assert torch.equal(a, b), (name, M)


def test_matmul_ex_rejects_unknown_flags(q4):
    from aria_b200._lib import lib
    w = q4.Q4Weight.from_f16(torch.zeros(64, 64, dtype=torch.float16, device="cuda"), LAYOUT_KN)
    x = torch.zeros(1, 64, dtype=torch.float16, device="cuda")
    y = torch.zeros(1, 64, dtype=torch.float16, device="cuda")
    rc = lib().aria_q4_0_matmul_ex(w.buf.data_ptr(), 0, 64, 64, x.data_ptr(), 1, 64, y.data_ptr(), 1, 64, None,
                                   1.0, 0.0, 32, None)
    assert rc == 1


# (kernel flag, layout, K, N, M): every kernel's epilogue, tensor-core cases with
# and without a K split through the workspace
GELU_CASES = [(2, LAYOUT_NK, 4096, 1001, 1), (2, LAYOUT_KN, 3584, 896, 8), (4, LAYOUT_KN, 896, 3584, 4),
              (4, LAYOUT_NK, 896, 1001, 32), (8, LAYOUT_KN, 896, 2688, 300), (8, LAYOUT_NK, 3584, 896, 64)]


@pytest.mark.parametrize("kflag,layout,K,N,M", GELU_CASES)
@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32])
def test_gelu_epilogue(q4, coracle, kflag, layout, K, N, M, out_dtype):
    """ARIA_Q4_FLAG_EPILOGUE_GELU: y = gelu(alpha x.W + bias) + beta y against the
    fp64 reference with the reference's tanh-form GELU (src/kernels.cu:574-583)."""
    y, ref = run_projection(q4, coracle, layout, K, N, M, out_dtype=out_dtype, bias=True, alpha=0.75, beta=0.5,
                            flags=kflag, gelu=True, wscale=0.05)
    check_close(y, ref, what=f"gelu kernel={kflag} {layout} {K}x{N} M={M}")


def test_gelu_python_mirror(q4, coracle):
    """q4.matmul(..., activation="gelu") through the auto workspace (split K)."""
    from oracle.q4_oracle_np import gelu_tanh
    from aria_b200.efkolos import synth_f16
    K, N, M = 3584, 896, 64
    w16 = synth_f16((K, N), 0.05, 31)
    wq = q4.Q4Weight.from_f16(w16, LAYOUT_KN)
    x = synth_f16((M, K), 1.0, 32)
    b = synth_f16((N,), 0.1, 33)
    y = q4.matmul(x, wq, bias=b, out_dtype=torch.float32, activation="gelu")
    blocks = coracle.quantize_q4_0_f16(w16.cpu().numpy().reshape(-1))
    ref = gelu_tanh(coracle.matmul_ref(blocks, LAYOUT_KN, K, N, x.cpu().numpy(), b.cpu().numpy(), 1.0))
    check_close(y.cpu().numpy(), ref, what="q4.matmul gelu")
