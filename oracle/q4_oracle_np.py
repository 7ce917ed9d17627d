"""numpy twin of the Q4_0 oracle.  TEST INFRASTRUCTURE ONLY.

A second, independent restatement of ARIA's CPU Q4_0 packer and of the
dequantise-then-matmul arithmetic, written vectorised so that it shares no code
with q4_oracle.c.  Tests require the two to agree byte for byte before either is
used to judge the CUDA kernels.  Only tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py may import this module.

Parity status: UNPINNED against executed reference output (the reference is
Rust, which cannot be built here, and it ships no golden vectors).

Reference lines followed (lold3344/ARIA):
  src/transformer_cuda.rs:548-575    quantize_q4_0
  src/transformer_cuda.rs:3214-3218  push_q4!: f16 -> f32 -> quantize_q4_0
  src/transformer_cuda.rs:3322-3333  cpu_matmul (KN orientation)
  src/transformer_cuda.rs:1318-1321  LM-head dot products (NK orientation)
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

BLOCK = 32
BLOCK_BYTES = 18
LAYOUT_KN = 0
LAYOUT_NK = 1

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "libq4oracle.so")


def packed_bytes(n: int) -> int:
    return (n + BLOCK - 1) // BLOCK * BLOCK_BYTES


def _round_half_away(v: np.ndarray) -> np.ndarray:
    """f32::round: ties away from zero, computed exactly in f32."""
    a = np.abs(v)
    fl = np.floor(a)
    up = (a - fl) >= np.float32(0.5)  # a - floor(a) is exact for |a| < 2**23
    r = fl + up.astype(np.float32)
    return np.copysign(r, v).astype(np.float32)


def _as_i32_saturating(r: np.ndarray) -> np.ndarray:
    out = np.zeros(r.shape, dtype=np.int64)
    finite = ~np.isnan(r)
    out[finite] = np.clip(r[finite], -2147483648.0, 2147483647.0).astype(np.int64)
    return out


def quantize_q4_0(data) -> np.ndarray:
    """quantize_q4_0(&[f32]) -> Vec<u8>, vectorised over blocks."""
    x = np.ascontiguousarray(np.asarray(data, dtype=np.float32).reshape(-1))
    n = x.size
    nb = (n + BLOCK - 1) // BLOCK
    if nb == 0:
        return np.zeros(0, dtype=np.uint8)
    padded = np.zeros(nb * BLOCK, dtype=np.float32)
    padded[:n] = x
    blocks = padded.reshape(nb, BLOCK)
    # fold(0, f32::max) over |x| of the *real* elements; the zero padding cannot
    # change a max that starts from 0, and fmax ignores NaN like f32::max.
    absmax = np.fmax.reduce(np.abs(blocks), axis=1, initial=np.float32(0.0))
    absmax = np.fmax(absmax, np.float32(0.0)).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        scale = np.where(absmax > 0, absmax / np.float32(7.0), np.float32(1.0)).astype(np.float32)
        scale_f16 = scale.astype(np.float16)
        v = (blocks / scale[:, None]).astype(np.float32)
    q = _as_i32_saturating(_round_half_away(v))
    q = (q + 8 + 2**31) % 2**32 - 2**31  # i32 wrapping add
    q = np.clip(q, 0, 15).astype(np.uint8)
    nib = (q[:, 0::2] | (q[:, 1::2] << 4)).astype(np.uint8)
    out = np.empty((nb, BLOCK_BYTES), dtype=np.uint8)
    out[:, 0:2] = scale_f16.view(np.uint8).reshape(nb, 2)
    out[:, 2:] = nib
    return out.reshape(-1)


def quantize_q4_0_f16(data_f16) -> np.ndarray:
    """push_q4!: the f16 weight is widened to f32 exactly, then packed."""
    return quantize_q4_0(np.asarray(data_f16, dtype=np.float16).astype(np.float32))


def dequantize_q4_0(blocks, n: int) -> np.ndarray:
    """w = (q - 8) * f32(scale_f16), the exact inverse of the packer's encoding."""
    b = np.asarray(blocks, dtype=np.uint8).reshape(-1, BLOCK_BYTES)
    scale = b[:, 0:2].copy().view(np.float16).astype(np.float32).reshape(-1)
    nib = b[:, 2:]
    q = np.empty((b.shape[0], BLOCK), dtype=np.int32)
    q[:, 0::2] = nib & 0xF
    q[:, 1::2] = nib >> 4
    w = (q - 8).astype(np.float32) * scale[:, None]
    return w.reshape(-1)[:n]


def dequantize_columns(blocks, layout: int, K: int, N: int, cols) -> np.ndarray:
    """Exact (q - 8) * scale of the output columns `cols` of a K x N projection
    stored as GGUF Q4_0 blocks in the reference's flat order, as f32 [K][len(cols)].

    KN (w[k][n], blocks along n): element (k, n) sits in block (k*N + n) // 32
    at position (k*N + n) % 32.  NK (embed[n][k], blocks along k): column n is
    row n of the stored tensor, blocks n*K/32 .. (n+1)*K/32 - 1.  Lets a parity
    test check a seeded sample of the outputs of a projection too large to
    dequantise whole."""
    b = np.asarray(blocks, dtype=np.uint8).reshape(-1, BLOCK_BYTES)
    cols = np.asarray(cols, dtype=np.int64).reshape(-1)
    if layout == LAYOUT_NK:
        nb = K // BLOCK
        idx = (cols[:, None] * nb + np.arange(nb)[None, :]).reshape(-1)
        rows = dequantize_q4_0(b[idx].reshape(-1), idx.size * BLOCK).reshape(cols.size, K)
        return np.ascontiguousarray(rows.T)
    flat = np.arange(K, dtype=np.int64)[:, None] * N + cols[None, :]
    blk, pos = flat // BLOCK, flat % BLOCK
    scale = b[:, 0:2].copy().view(np.float16).astype(np.float32).reshape(-1)[blk]
    byte = b[blk, 2 + pos // 2].astype(np.int32)
    q = (byte >> (4 * (pos % 2))) & 0xF
    return ((q - 8).astype(np.float32) * scale).astype(np.float32)


def matmul_ref(blocks, layout: int, K: int, N: int, x_f16, bias_f16=None, alpha: float = 1.0) -> np.ndarray:
    """fp64 parity reference: y[M,N] = alpha * x[M,K] @ W(K,N) (+ bias)."""
    w = dequantize_q4_0(blocks, K * N).astype(np.float64)
    w = w.reshape(K, N) if layout == LAYOUT_KN else w.reshape(N, K).T
    x = np.asarray(x_f16, dtype=np.float16).astype(np.float64).reshape(-1, K)
    y = alpha * (x @ w)
    if bias_f16 is not None:
        y = y + np.asarray(bias_f16, dtype=np.float16).astype(np.float64)[None, :]
    return y


def gelu_tanh(y) -> np.ndarray:
    """GELU in its tanh form, fp64, as the reference's gelu_fwd states it
    (lold3344/ARIA src/kernels.cu:574-583): 0.5 y (1 + tanh(0.7978845608 (y + 0.044715 y^3)))."""
    y = np.asarray(y, dtype=np.float64)
    return 0.5 * y * (1.0 + np.tanh(0.7978845608 * (y + 0.044715 * y ** 3)))


# ------------------------------------------------------------ C oracle binding

def build_c_oracle() -> str:
    """Compile q4_oracle.c with the committed Makefile (gcc is on both hosts)."""
    src = os.path.join(_HERE, "q4_oracle.c")
    if not os.path.exists(_SO) or os.path.getmtime(_SO) < os.path.getmtime(src):
        subprocess.run(["make", "-C", _HERE, "CC=gcc"], check=True, capture_output=True)
    return _SO


class COracle:
    """ctypes view of oracle/_build/libq4oracle.so."""

    def __init__(self):
        self.lib = ctypes.CDLL(build_c_oracle())
        L = self.lib
        P = ctypes.c_void_p
        L.q4o_f32_to_f16.restype = ctypes.c_uint16
        L.q4o_f32_to_f16.argtypes = [ctypes.c_float]
        L.q4o_f16_to_f32.restype = ctypes.c_float
        L.q4o_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.q4o_quantize_q4_0.argtypes = [P, ctypes.c_size_t, P]
        L.q4o_quantize_q4_0_f16.argtypes = [P, ctypes.c_size_t, P]
        L.q4o_dequantize_q4_0.argtypes = [P, ctypes.c_size_t, P]
        L.q4o_matmul_ref_f64.restype = ctypes.c_int
        L.q4o_matmul_ref_f64.argtypes = [P, ctypes.c_int, ctypes.c_int, ctypes.c_int, P,
                                         ctypes.c_int, ctypes.c_int, P, ctypes.c_double, P]
        L.q4o_cpu_matmul_f32.argtypes = [P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int, P]
        L.q4o_baseline_projection.argtypes = [P, ctypes.c_int, ctypes.c_int, ctypes.c_int, P,
                                              ctypes.c_int, P, P, P, ctypes.c_int]
        L.q4o_max_threads.restype = ctypes.c_int

    @staticmethod
    def _p(a: np.ndarray):
        return a.ctypes.data_as(ctypes.c_void_p)

    def quantize_q4_0(self, data) -> np.ndarray:
        x = np.ascontiguousarray(np.asarray(data, dtype=np.float32).reshape(-1))
        out = np.zeros(packed_bytes(x.size), dtype=np.uint8)
        self.lib.q4o_quantize_q4_0(self._p(x), x.size, self._p(out))
        return out

    def quantize_q4_0_f16(self, data_f16) -> np.ndarray:
        x = np.ascontiguousarray(np.asarray(data_f16, dtype=np.float16).reshape(-1))
        out = np.zeros(packed_bytes(x.size), dtype=np.uint8)
        self.lib.q4o_quantize_q4_0_f16(self._p(x), x.size, self._p(out))
        return out

    def dequantize_q4_0(self, blocks, n: int) -> np.ndarray:
        b = np.ascontiguousarray(np.asarray(blocks, dtype=np.uint8))
        out = np.zeros(n, dtype=np.float32)
        self.lib.q4o_dequantize_q4_0(self._p(b), n, self._p(out))
        return out

    def matmul_ref(self, blocks, layout, K, N, x_f16, bias_f16=None, alpha=1.0) -> np.ndarray:
        b = np.ascontiguousarray(np.asarray(blocks, dtype=np.uint8))
        x = np.ascontiguousarray(np.asarray(x_f16, dtype=np.float16).reshape(-1, K))
        M = x.shape[0]
        y = np.zeros((M, N), dtype=np.float64)
        bias = None
        if bias_f16 is not None:
            bias = np.ascontiguousarray(np.asarray(bias_f16, dtype=np.float16))
        rc = self.lib.q4o_matmul_ref_f64(self._p(b), layout, K, N, self._p(x), M, K,
                                         self._p(bias) if bias is not None else None,
                                         float(alpha), self._p(y))
        if rc != 0:
            raise MemoryError("q4o_matmul_ref_f64 failed")
        return y

    def baseline_projection(self, blocks, layout, K, N, x_f16, w_scratch, x_scratch, y, threads):
        self.lib.q4o_baseline_projection(self._p(blocks), layout, K, N, self._p(x_f16),
                                         x_f16.shape[0], self._p(y), self._p(w_scratch),
                                         self._p(x_scratch), int(threads))

    def max_threads(self) -> int:
        return int(self.lib.q4o_max_threads())
