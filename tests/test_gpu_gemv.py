"""GPU parity of the streaming GEMV (M <= 8 token rows) against the fp64 oracle.

The shapes are chosen so that every kind of launch plan of the kernel runs (see
PLANS), with up to 8 token rows, a gap after each activation row (ldx > K,
filled with NaN that must never be read), f16 and f32 outputs, bias, alpha and
beta.  Reference: dequantise-then-matmul of the
GGUF Q4_0 blocks (lold3344/ARIA src/transformer_cuda.rs:549-575 inverted,
:3322-3333), tolerance max-abs 1e-2 and relative L2 1e-3."""
import pytest
import torch

from tests.gpu_helpers import LAYOUT_KN, LAYOUT_NK, check_close, run_projection

STREAM = 2  # ARIA_Q4_FLAG_KERNEL_STREAM: these tests pin the streaming kernel

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]


@pytest.fixture(scope="module")
def q4():
    from aria_b200 import q4 as q4mod
    return q4mod


# (layout, K, N, M) chosen so that, on a 148-SM B200, the launch plans cover 16-
# and 32-row tiles, chunks of one and two 128-k groups (and a warp slice of odd
# length, whose last chunk holds one group), cluster K splits of 1, 2 and 4, one
# and several row tiles per CTA or cluster (so both 8-warp teams of a CTA run),
# 7 of 8 warps busy (K = 896), odd N with a ragged last tile (NK), and K % 128 != 0.
PLANS = [
    (LAYOUT_KN, 896, 2688, 1), (LAYOUT_KN, 896, 2688, 3), (LAYOUT_KN, 896, 2688, 8),
    (LAYOUT_KN, 3584, 896, 1), (LAYOUT_KN, 3584, 4096, 8),
    (LAYOUT_KN, 8192, 4096, 3),
    (LAYOUT_KN, 6144, 4096, 8), (LAYOUT_KN, 12288, 4096, 8),
    (LAYOUT_KN, 16384, 4096, 1), (LAYOUT_KN, 16384, 4096, 8),
    (LAYOUT_KN, 16384, 2048, 8),
    (LAYOUT_NK, 128, 12000, 1),
    (LAYOUT_NK, 1056, 12000, 1),
    (LAYOUT_NK, 8192, 2048, 1),
    (LAYOUT_NK, 9216, 2048, 8), (LAYOUT_NK, 12288, 1001, 8),
    (LAYOUT_NK, 16384, 640, 8),
    (LAYOUT_NK, 4096, 12000, 1),
    (LAYOUT_NK, 4096, 1001, 1), (LAYOUT_NK, 4096, 1001, 3), (LAYOUT_NK, 4096, 1001, 8),
    (LAYOUT_NK, 1056, 300, 1), (LAYOUT_NK, 1056, 300, 8),
    (LAYOUT_NK, 896, 31500, 1),
    # kinds the launch planner reaches on other shapes: 2-CTA clusters holding
    # several tiles each, 16-row one-group chunks (also single-token NK, and with
    # 4-CTA clusters), and a warp slice of odd length under two-group chunks
    (LAYOUT_KN, 10240, 12000, 8), (LAYOUT_NK, 10240, 12000, 8),
    (LAYOUT_KN, 128, 32, 1), (LAYOUT_NK, 128, 32, 1), (LAYOUT_NK, 128, 32, 3),
    (LAYOUT_KN, 3072, 32, 8), (LAYOUT_NK, 12288, 32, 1),
    (LAYOUT_KN, 4608, 32, 1), (LAYOUT_NK, 4608, 32, 1),
]


@pytest.mark.parametrize("layout,K,N,M", PLANS)
def test_gemv_plans(q4, coracle, layout, K, N, M):
    y, ref = run_projection(q4, coracle, layout, K, N, M, bias=True, flags=STREAM)
    check_close(y, ref, what=f"gemv {layout} {K}x{N} M={M}")


@pytest.mark.parametrize("layout,K,N,M", [(LAYOUT_KN, 896, 896, 8), (LAYOUT_NK, 4096, 1001, 5),
                                          (LAYOUT_KN, 3584, 896, 2)])
def test_gemv_ldx_gap_f16_out(q4, coracle, layout, K, N, M):
    y, ref = run_projection(q4, coracle, layout, K, N, M, out_dtype=torch.float16, bias=True, ldx=K + 24,
                            flags=STREAM)
    check_close(y, ref, what=f"gemv ldx gap {layout} {K}x{N} M={M}")


def test_gemv_alpha_beta(q4, coracle):
    y, ref = run_projection(q4, coracle, LAYOUT_NK, 4096, 1001, 4, alpha=0.5, beta=0.25, flags=STREAM)
    check_close(y, ref, what="gemv alpha/beta NK")
    y, ref = run_projection(q4, coracle, LAYOUT_KN, 3584, 896, 1, out_dtype=torch.float16, alpha=1 / 29.93,
                            beta=1.0, bias=True, flags=STREAM)
    check_close(y, ref, what="gemv alpha/beta KN f16")


@pytest.mark.parametrize("layout,K,N", [(LAYOUT_KN, 3584, 896), (LAYOUT_KN, 16384, 4096), (LAYOUT_NK, 4096, 12000),
                                        (LAYOUT_NK, 1056, 300)])
def test_gemv_deterministic_and_const_weights(q4, layout, K, N):
    """Fixed-order reductions: repeated calls, with and without
    ARIA_Q4_FLAG_CONST_WEIGHTS, return identical bits."""
    from aria_b200.efkolos import synth_f16
    shape = (K, N) if layout == LAYOUT_KN else (N, K)
    wq = q4.Q4Weight.from_f16(synth_f16(shape, 0.02, 21), layout)
    for M in (1, 8):
        x = synth_f16((M, K), 1.0, 22)
        a = q4.matmul(x, wq, out_dtype=torch.float32, kernel="stream")
        b = q4.matmul(x, wq, out_dtype=torch.float32, kernel="stream")
        c = q4.matmul(x, wq, out_dtype=torch.float32, const_weights=True, kernel="stream")
        torch.cuda.synchronize()
        assert torch.equal(a, b) and torch.equal(a, c), (layout, K, N, M)


@pytest.mark.parametrize("layout,K,N", [(LAYOUT_KN, 896, 3584), (LAYOUT_NK, 4096, 1001)])
def test_stream_and_register_kernels_agree_with_oracle(q4, coracle, layout, K, N):
    """The same projections through both decode kernels (selected by flag),
    each within tolerance of the fp64 reference."""
    for flags in (2, 4):
        for M in (1, 8):
            y, ref = run_projection(q4, coracle, layout, K, N, M, seed=5, flags=flags)
            check_close(y, ref, what=f"flags={flags} M={M}")


def test_kernel_flags_errors(q4):
    from aria_b200._lib import lib
    w = q4.Q4Weight.from_f16(torch.zeros(64, 64, dtype=torch.float16, device="cuda"), LAYOUT_KN)
    x = torch.zeros(80, 64, dtype=torch.float16, device="cuda")
    y = torch.zeros(80, 64, dtype=torch.float16, device="cuda")
    L = lib()

    def rc(M, flags):
        return L.aria_q4_0_matmul_ex(w.buf.data_ptr(), 0, 64, 64, x.data_ptr(), M, 64, y.data_ptr(), 1, 64, None,
                                     1.0, 0.0, flags, None)
    assert rc(1, 2 | 4) == 1   # two kernels requested: EINVAL
    assert rc(1, 4 | 8) == 1
    assert rc(1, 8) == 0       # the tcgen05 kernel takes any M
    assert rc(9, 2) == 2       # streaming GEMV takes M <= 8: EUNSUPPORTED
    assert rc(65, 4) == 2      # register-fed kernel takes M <= 64: EUNSUPPORTED
    assert rc(8, 2) == 0 and rc(64, 4) == 0
    torch.cuda.synchronize()


@pytest.mark.parametrize("layout,K,N", [(LAYOUT_KN, 4096, 16384), (LAYOUT_NK, 4096, 31500), (LAYOUT_KN, 3584, 896)])
def test_chained_launches_bit_identical(q4, layout, K, N):
    """One token through a CUDA graph of back-to-back launches over four copies
    of the weight (programmatic dependent launch, const-weights flag: each
    launch streams its first chunks while the previous one runs), every launch
    into its own NaN-filled output: every output of every launch must equal a
    single standalone launch's bits (no unwritten element, no dependence on a
    neighbouring launch)."""
    g_ = torch.Generator(device="cuda")
    g_.manual_seed(K + N)
    shape = (K, N) if layout == LAYOUT_KN else (N, K)
    w0 = q4.Q4Weight.from_f16((torch.randn(shape, generator=g_, device="cuda") * 0.02).half(), layout)
    pool = [w0] + [q4.Q4Weight(w0.buf.clone(), layout, K, N) for _ in range(3)]
    x = torch.randn(1, K, generator=g_, device="cuda").half()
    ref = torch.empty(1, N, dtype=torch.float16, device="cuda")
    s = torch.cuda.Stream()
    ys = [torch.empty(1, N, dtype=torch.float16, device="cuda") for _ in range(16)]
    s.wait_stream(torch.cuda.current_stream())  # the weights and inputs were made on the current stream
    with torch.cuda.stream(s):
        q4.matmul(x, w0, ref, const_weights=True, kernel="stream")
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            for j, y in enumerate(ys):
                q4.matmul(x, pool[j % 4], y, const_weights=True, kernel="stream")
        for _ in range(5):
            for y in ys:
                y.fill_(float("nan"))
            graph.replay()
            torch.cuda.synchronize()
            for j, y in enumerate(ys):
                assert torch.equal(y, ref), f"launch {j}"
    del graph


def test_no_device_error_recorded(q4):
    from aria_b200 import _lib
    assert _lib.lib().aria_q4_take_device_error() == 0
