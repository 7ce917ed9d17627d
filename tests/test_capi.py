"""CPU-side checks of the C ABI: the library loads, exports every declared
symbol, and its pure-host functions answer without a GPU."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "aria_q4.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\bARIA_Q4_API\s+[\w\s\*]*?\b(aria_\w*)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from aria_b200 import _lib
    return _lib.lib()


def test_header_lists_functions():
    names = declared_functions()
    assert "aria_q4_0_matmul" in names and "aria_q4_0_pack_f16" in names
    assert len(names) >= 10


def test_every_declared_symbol_is_exported(lib):
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared in aria_q4.h but not exported"


def test_binding_covers_header():
    from aria_b200._lib import SIGNATURES
    assert set(SIGNATURES) == set(declared_functions())


def test_host_only_functions(lib):
    assert lib.aria_q4_abi_version() == 1
    assert lib.aria_q4_0_packed_bytes(0) == 0
    assert lib.aria_q4_0_packed_bytes(1) == 18
    assert lib.aria_q4_0_packed_bytes(33) == 36
    assert lib.aria_q4_0_packed_bytes(3584 * 896) == 1806336
    assert lib.aria_q4_0_tiled_bytes(0, 5) == 0
    K, N = 896, 2688
    assert lib.aria_q4_0_tiled_bytes(K, N) >= K * N // 32 * 18
    assert lib.aria_q4_strerror(0) == b"ok"
    assert b"multiple of 32" in lib.aria_q4_strerror(2)


def test_argument_errors_need_no_gpu(lib):
    # shape / pointer validation happens before any CUDA call
    P = ctypes.c_void_p
    assert lib.aria_q4_0_matmul(P(256), 0, 33, 64, P(256), 1, 64, P(256), 1, 64, None, 1.0, 0.0, None) == 2
    assert lib.aria_q4_0_matmul(P(256), 0, 64, 48, P(256), 1, 64, P(256), 1, 64, None, 1.0, 0.0, None) == 2
    assert lib.aria_q4_0_matmul(P(256), 7, 64, 64, P(256), 1, 64, P(256), 1, 64, None, 1.0, 0.0, None) == 1
    assert lib.aria_q4_0_matmul(None, 0, 64, 64, P(256), 1, 64, P(256), 1, 64, None, 1.0, 0.0, None) == 1
    assert lib.aria_q4_0_matmul(P(256), 0, 64, 64, P(256), -1, 64, P(256), 1, 64, None, 1.0, 0.0, None) == 1
    assert lib.aria_q4_0_matmul(P(256), 0, 64, 64, P(256), 0, 64, P(256), 1, 64, None, 1.0, 0.0, None) == 0
    assert lib.aria_q4_0_matmul(P(256), 0, 64, 64, P(258), 1, 64, P(256), 1, 64, None, 1.0, 0.0, None) == 3
    assert lib.aria_q4_0_repack(P(256), 1, 64, 64, P(256), 10, None) == 6
    assert lib.aria_q4_0_repack(P(256), 1, 64, 64, P(260), 1 << 20, None) == 3
    assert lib.aria_q4_0_pack_f16(None, 0, None, None) == 0
    assert lib.aria_q4_0_pack_f16(None, 5, None, None) == 1


def test_kernel_choice_routing():
    """aria_q4_0_kernel_choice (no GPU needed: the planners fall back to 148 SMs)."""
    from aria_b200._lib import lib
    L = lib()
    STREAM, REGISTER, TENSOR = 1, 2, 3
    KN, NK = 0, 1
    assert L.aria_q4_0_kernel_choice(KN, 896, 2688, 1, 0, 0) == REGISTER    # small weight: latency-bound
    assert L.aria_q4_0_kernel_choice(NK, 896, 31500, 1, 0, 0) == STREAM     # 15.9 MB: bandwidth-bound
    assert L.aria_q4_0_kernel_choice(KN, 4096, 16384, 8, 0, 0) == STREAM
    assert L.aria_q4_0_kernel_choice(KN, 896, 2688, 16, 0, 0) == REGISTER
    assert L.aria_q4_0_kernel_choice(KN, 3584, 896, 1, 0, 0) == STREAM      # tall K
    assert L.aria_q4_0_kernel_choice(KN, 896, 2688, 64, 0, 0) == TENSOR     # no K split needed
    assert L.aria_q4_0_workspace_bytes(3584, 896, 64) > 0
    assert L.aria_q4_0_kernel_choice(NK, 3584, 896, 64, 0, 0) == REGISTER   # few row tiles (N <= 1024)
    assert L.aria_q4_0_kernel_choice(NK, 3584, 896, 64, 1 << 20, 0) == REGISTER
    assert L.aria_q4_0_kernel_choice(KN, 896, 896, 40, 1 << 20, 0) == REGISTER
    assert L.aria_q4_0_kernel_choice(KN, 896, 896, 65, 1 << 20, 0) == TENSOR   # above the register kernel's 64
    assert L.aria_q4_0_workspace_bytes(16384, 4096, 64) > 0
    assert L.aria_q4_0_kernel_choice(KN, 16384, 4096, 64, 0, 0) == REGISTER  # would split K, no workspace
    assert L.aria_q4_0_kernel_choice(KN, 16384, 4096, 64, 64 << 20, 0) == TENSOR
    assert L.aria_q4_0_kernel_choice(KN, 896, 896, 4096, 0, 0) == TENSOR
    assert L.aria_q4_0_kernel_choice(KN, 896, 896, 1, 0, 2) == STREAM       # forced
    assert L.aria_q4_0_kernel_choice(KN, 896, 896, 9, 0, 2) == -2           # stream takes M <= 8
    assert L.aria_q4_0_kernel_choice(KN, 896, 896, 65, 0, 4) == -2          # register takes M <= 64
    assert L.aria_q4_0_kernel_choice(KN, 896, 896, 1, 0, 2 | 4) == -1       # two kernels requested
    assert L.aria_q4_0_kernel_choice(KN, 896, 896, 1, 0, 8) == TENSOR
    assert L.aria_q4_0_kernel_choice(KN, 896, 48, 1, 0, 0) == -2            # KN needs N % 32 == 0
    for M in (1, 16, 4096):  # the GELU epilogue flag does not change the routing
        assert L.aria_q4_0_kernel_choice(KN, 896, 3584, M, 0, 16) == L.aria_q4_0_kernel_choice(KN, 896, 3584, M, 0, 0)
    assert L.aria_q4_0_kernel_choice(KN, 896, 896, 1, 0, 32) == -1          # unknown flag



def test_static_scratch_validation_needs_no_gpu(lib):
    """aria_q4_0_matmul_static_ws validates its arguments before touching the
    device, and no longer rejects shapes by the unlimited plan's scratch size:
    a forced register-kernel call at M = 64 on a tall K (whose tensor-core plan
    would want more than the 8 MiB scratch) and a plan that only fits with a
    smaller split both get past validation to the device check (which fails on
    a host without a GPU with ECUDA or ENODEVICE, never ESIZE)."""
    P = ctypes.c_void_p
    args = lambda K, N, M: (P(256), 0, K, N, P(256), M, K, P(256), 0, N, None, 1.0, 0.0)  # noqa: E731
    assert lib.aria_q4_0_matmul_static_ws(*args(64, 64, 1), 64, None) == 1         # unknown flag
    assert lib.aria_q4_0_matmul_static_ws(*args(64, 64, 1), 2 | 4, None) == 1      # two kernels
    assert lib.aria_q4_0_matmul_static_ws(*args(64, 48, 1), 0, None) == 2          # KN needs N % 32 == 0
    assert lib.aria_q4_0_matmul_static_ws(*args(64, 64, 0), 0, None) == 0          # M == 0: nothing to do
    assert lib.aria_q4_0_matmul_static_ws(*args(64, 64, 9), 2, None) == 2          # stream takes M <= 8
    assert lib.aria_q4_0_workspace_bytes(16384, 4096, 64) > 0
    for flags in (4, 0):
        rc = lib.aria_q4_0_matmul_static_ws(*args(16384, 4096, 64), flags, None)
        assert rc in (4, 5), rc
    assert lib.aria_q4_0_workspace_bytes(16384, 4096, 128) > 8 << 20
    assert lib.aria_q4_0_kernel_choice(0, 16384, 4096, 128, 8 << 20, 0) == 3
    assert lib.aria_q4_0_matmul_static_ws(*args(16384, 4096, 128), 0, None) in (4, 5)
    assert lib.aria_q4_0_workspace_counter_bytes() > 0


def test_stall_hook_validates_without_gpu(lib):
    P = ctypes.c_void_p
    assert lib.aria_q4_test_tensor_stall(P(256), 0, 64, 64, P(256), 1, 64, P(256), 0, 64, 0, None) == 1
    assert lib.aria_q4_test_tensor_stall(P(256), 0, 64, 48, P(256), 1, 64, P(256), 0, 64, 100, None) == 2
    assert lib.aria_q4_test_tensor_stall(P(256), 0, 64, 64, P(256), 1, 64, P(256), 0, 64, 100, None) in (4, 5)
