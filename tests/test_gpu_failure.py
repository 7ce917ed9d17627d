"""The failure path of the tensor-core kernel, driven without faulting the GPU.

Every wait inside gemm_tc_kernel is bounded: when one runs out the kernel
records an error code, the other warps of the CTA stop waiting, tensor memory is
released and the kernel returns (the reference has no such path: it aborts the
process on any CUDA error, lold3344/ARIA Cargo.toml:24).  The test hook
aria_q4_test_tensor_stall launches the kernel with its activation-tile producer
issuing no copies and a short wait limit, so the MMA issuer's first wait can
never complete.  The test checks the recorded code, that the kernel returned
within a few limits, and that the next ordinary call on the same context is
correct and records nothing."""
import time

import numpy as np
import pytest
import torch

from tests.gpu_helpers import LAYOUT_KN, LAYOUT_NK, check_close

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]

DEVERR_TIMEOUT_FULL = 1  # ARIA_Q4_DEVERR_TIMEOUT_FULL


@pytest.mark.parametrize("layout,K,N,M", [(LAYOUT_KN, 896, 128, 64), (LAYOUT_NK, 1024, 96, 200)])
def test_expired_wait_reported_then_next_call_correct(coracle, layout, K, N, M):
    from aria_b200 import _lib, q4
    from aria_b200.q4 import _stream
    lib = _lib.lib()
    torch.cuda.synchronize()
    assert lib.aria_q4_take_device_error() == 0
    rng = np.random.default_rng(K + N + M)
    shape = (K, N) if layout == LAYOUT_KN else (N, K)
    w = (rng.standard_normal(shape) * 0.02).astype(np.float16)
    x = rng.standard_normal((M, K)).astype(np.float16)
    blocks = coracle.quantize_q4_0_f16(w.reshape(-1))
    wq = q4.Q4Weight.from_f16(torch.from_numpy(w).cuda(), layout)
    xt = torch.from_numpy(x).cuda()
    y = torch.zeros(M, N, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    rc = lib.aria_q4_test_tensor_stall(wq.buf.data_ptr(), layout, K, N, xt.data_ptr(), M, K, y.data_ptr(), 0, N,
                                       20000, _stream())
    assert rc == 0
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    # one CTA per output tile here; its issuer's wait (20 ms) runs out first and
    # every other wait returns at once on the abort flag
    assert lib.aria_q4_take_device_error() == DEVERR_TIMEOUT_FULL
    assert elapsed < 2.0, elapsed
    # the context is still usable: the next ordinary call is correct
    y2 = q4.matmul(xt, wq, out_dtype=torch.float32, kernel="tensor")
    torch.cuda.synchronize()
    check_close(y2.cpu().numpy(), coracle.matmul_ref(blocks, layout, K, N, x), what="after the expired wait")
    assert lib.aria_q4_take_device_error() == 0


def test_stall_hook_rejects_bad_limits():
    from aria_b200 import _lib, q4
    lib = _lib.lib()
    wq = q4.Q4Weight.from_f16(torch.zeros(64, 64, dtype=torch.float16, device="cuda"), LAYOUT_KN)
    x = torch.zeros(1, 64, dtype=torch.float16, device="cuda")
    y = torch.zeros(1, 64, dtype=torch.float32, device="cuda")
    for limit in (0, 1000001):
        assert lib.aria_q4_test_tensor_stall(wq.buf.data_ptr(), LAYOUT_KN, 64, 64, x.data_ptr(), 1, 64,
                                             y.data_ptr(), 0, 64, limit, None) == 1
