"""aria_q4_0_matmul_static_ws: the projection for callers that cannot allocate
device memory (inside another framework's memory pool or a captured graph, or
a foreign-language host with no allocator), using the library's own static
device scratch in place of a caller workspace.

Compared with aria_q4_0_matmul_ws (a caller-owned, zero-filled workspace) on
two calls in a row each: bit for bit on shapes whose K split fits in the 8 MiB
scratch (the same plan runs), and on shapes that need no scratch.  A shape
whose best split would need more than 8 MiB runs with a smaller split; it is
checked against the fp64 oracle (and against aria_q4_0_matmul_ws within the
projection tolerance).  The file name sorts last, so the suite runs it after
every other test (and it also passes alone in a fresh process)."""
import numpy as np
import pytest
import torch

from tests.gpu_helpers import LAYOUT_KN, LAYOUT_NK, check_close, sample_columns, sampled_ref

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]

STATIC_BYTES = 8 << 20
TENSOR = 3  # ARIA_Q4_KERNEL_TENSOR


@pytest.fixture(scope="module")
def q4():
    from aria_b200 import q4 as q4mod
    return q4mod


def _call(lib, name, wq, x, y, bias, extra):
    from aria_b200.q4 import _stream
    M, K = x.shape
    args = (wq.buf.data_ptr(), wq.layout, wq.K, wq.N, x.data_ptr(), M, K, y.data_ptr(), 0, wq.N,
            bias.data_ptr(), 1.0, 0.0) + extra + (0, _stream())
    return getattr(lib, name)(*args)


def _setup(q4, coracle, layout, K, N, M):
    rng = np.random.default_rng(K + N + M)
    shape = (K, N) if layout == LAYOUT_KN else (N, K)
    w = (rng.standard_normal(shape, dtype=np.float32) * 0.02).astype(np.float16)
    x = rng.standard_normal((M, K), dtype=np.float32).astype(np.float16)
    b = (rng.standard_normal(N) * 0.1).astype(np.float16)
    blocks = coracle.quantize_q4_0_f16(w.reshape(-1))
    wq = q4.Q4Weight.from_f16(torch.from_numpy(w).cuda(), layout)
    return blocks, wq, torch.from_numpy(x).cuda(), torch.from_numpy(b).cuda(), x, b


@pytest.mark.parametrize("layout,K,N,M,splits", [
    (LAYOUT_KN, 16384, 1536, 64, True),  # K split over the scratch
    (LAYOUT_NK, 3584, 1536, 64, True),
    (LAYOUT_KN, 8224, 1280, 50, True),
    (LAYOUT_KN, 896, 2688, 64, False),   # no split: no scratch used
    (LAYOUT_NK, 3584, 896, 64, False),   # register-fed kernel (few row tiles): no scratch
    (LAYOUT_NK, 4096, 1001, 1, False),
])
def test_static_scratch_matches_caller_workspace(q4, coracle, layout, K, N, M, splits):
    from aria_b200 import _lib
    lib = _lib.lib()
    need = int(lib.aria_q4_0_workspace_bytes(K, N, M))
    if splits:
        # the planner splits K for this shape, within the static scratch
        assert 0 < need <= STATIC_BYTES
        assert lib.aria_q4_0_kernel_choice(layout, K, N, M, STATIC_BYTES, 0) == TENSOR
    else:  # no split, or a kernel other than the tensor-core one (which alone uses scratch)
        assert need == 0 or lib.aria_q4_0_kernel_choice(layout, K, N, M, STATIC_BYTES, 0) != TENSOR
    blocks, wq, x, bias, xh, bh = _setup(q4, coracle, layout, K, N, M)
    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device="cuda")
    outs = []
    for _ in range(2):
        y = torch.empty(M, N, dtype=torch.float32, device="cuda")
        assert _call(lib, "aria_q4_0_matmul_ws", wq, x, y, bias, (ws.data_ptr(), need)) == 0
        outs.append(y)
    for _ in range(2):
        y = torch.empty(M, N, dtype=torch.float32, device="cuda")
        assert _call(lib, "aria_q4_0_matmul_static_ws", wq, x, y, bias, ()) == 0
        outs.append(y)
    torch.cuda.synchronize()
    for y in outs[1:]:
        assert torch.equal(outs[0], y)
    cols = sample_columns(N, 256, seed=N)
    check_close(outs[-1].cpu().numpy()[:, cols], sampled_ref(blocks, layout, K, N, xh, cols, bh),
                what=f"static scratch {layout} {K}x{N} M={M}")


def test_static_scratch_larger_plan_uses_smaller_split(q4, coracle):
    """The best split of this shape needs just over 8 MiB; the static-scratch
    call runs it with a split that fits (twice in a row) and stays within the
    projection tolerance of the fp64 oracle and of the caller-workspace call."""
    from aria_b200 import _lib
    lib = _lib.lib()
    layout, K, N, M = LAYOUT_KN, 16384, 4096, 128
    need = int(lib.aria_q4_0_workspace_bytes(K, N, M))
    assert need > STATIC_BYTES
    assert lib.aria_q4_0_kernel_choice(layout, K, N, M, STATIC_BYTES, 0) == TENSOR
    blocks, wq, x, bias, xh, bh = _setup(q4, coracle, layout, K, N, M)
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    y_ws = torch.empty(M, N, dtype=torch.float32, device="cuda")
    assert _call(lib, "aria_q4_0_matmul_ws", wq, x, y_ws, bias, (ws.data_ptr(), need)) == 0
    ys = []
    for _ in range(2):
        y = torch.empty(M, N, dtype=torch.float32, device="cuda")
        assert _call(lib, "aria_q4_0_matmul_static_ws", wq, x, y, bias, ()) == 0
        ys.append(y)
    torch.cuda.synchronize()
    assert torch.equal(ys[0], ys[1])
    cols = sample_columns(N, 256, seed=3)
    ref = sampled_ref(blocks, layout, K, N, xh, cols, bh)
    check_close(ys[1].cpu().numpy()[:, cols], ref, what="static scratch, smaller split")
    check_close(ys[1].cpu().numpy(), y_ws.cpu().numpy().astype(np.float64), what="static vs caller workspace")
    assert lib.aria_q4_take_device_error() == 0
