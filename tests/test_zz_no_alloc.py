"""aria_q4_0_matmul_static_ws: the projection with the library's own static
device scratch in place of a caller workspace.

Compared bit for bit with aria_q4_0_matmul_ws (a caller-owned, zero-filled
workspace) on two calls in a row each, on shapes whose tensor-core plan splits
K over the scratch and on shapes that need none; a shape whose split needs more
than the 8 MiB of static scratch is rejected with ARIA_Q4_ESIZE.  The file name
sorts last, so the suite runs it after every other test (and it also passes
alone)."""
import numpy as np
import pytest
import torch

from tests.gpu_helpers import LAYOUT_KN, LAYOUT_NK

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]

ESIZE = 6


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


@pytest.mark.parametrize("layout,K,N,M", [
    (LAYOUT_KN, 16384, 512, 64),   # K split over the scratch
    (LAYOUT_NK, 3584, 896, 64),
    (LAYOUT_KN, 8224, 256, 50),
    (LAYOUT_KN, 896, 2688, 64),    # no split: no scratch used
    (LAYOUT_NK, 4096, 1001, 1),
])
def test_static_scratch_matches_caller_workspace(q4, layout, K, N, M):
    from aria_b200 import _lib
    from aria_b200.efkolos import synth_f16
    lib = _lib.lib()
    shape = (K, N) if layout == LAYOUT_KN else (N, K)
    wq = q4.Q4Weight.from_f16(synth_f16(shape, 0.02, K + N), layout)
    x = synth_f16((M, K), 1.0, M)
    bias = synth_f16((N,), 0.1, 3)
    need = int(lib.aria_q4_0_workspace_bytes(K, N, M))
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
    assert np.isfinite(outs[0].cpu().numpy()).all()


def test_static_scratch_rejects_oversize(q4):
    from aria_b200 import _lib
    lib = _lib.lib()
    K, N, M = 16384, 4096, 128  # the split plan needs just over 8 MiB
    assert int(lib.aria_q4_0_workspace_bytes(K, N, M)) > 8 << 20
    wq = q4.Q4Weight.empty(LAYOUT_KN, K, N, torch.device("cuda"))
    x = torch.zeros(M, K, dtype=torch.float16, device="cuda")
    y = torch.zeros(M, N, dtype=torch.float32, device="cuda")
    bias = torch.zeros(N, dtype=torch.float16, device="cuda")
    assert _call(lib, "aria_q4_0_matmul_static_ws", wq, x, y, bias, ()) == ESIZE
    torch.cuda.synchronize()
    assert not y.any()  # nothing was launched
