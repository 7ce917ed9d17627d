"""Host-side mirror of ARIA's Q4_0 call surface, backed by libaria_q4.so.

Reference surface (lold3344/ARIA, src/transformer_cuda.rs):
  quantize_q4_0(&[f32]) -> Vec<u8>                           :549-575
  gemm(blas, a, b, c, m, k, n, transa, transb, alpha, beta)  :615-640
  TransformerLayer.w_qkv / w_out / w_ff1 / w_ff2, embed      :261-271, :314

Names and argument meaning follow the reference: `quantize_q4_0` returns the
GGUF Q4_0 bytes, `gemm_q4` takes (a, b, c, m, k, n, transb, alpha, beta) with b
a Q4_0 weight.  Where the reference panics (`.unwrap()` on a CUDA error) these
raise AriaQ4Error.  torch supplies device memory and the current stream only.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import F16, F32, LAYOUT_KN, LAYOUT_NK, call

__all__ = ["quantize_q4_0", "packed_bytes", "dequantize_q4_0", "Q4Weight", "gemm_q4", "matmul", "matmul_ln",
           "LAYOUT_KN", "LAYOUT_NK"]


def _stream(device=None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def packed_bytes(n: int) -> int:
    return int(_lib.lib().aria_q4_0_packed_bytes(n))


def quantize_q4_0(data) -> torch.Tensor:
    """GPU twin of quantize_q4_0: flat f16/f32 -> uint8 GGUF Q4_0 blocks on the device.

    Accepts a CUDA tensor, or a CPU tensor / numpy array (copied to the current device).
    """
    if isinstance(data, np.ndarray):
        data = torch.from_numpy(np.ascontiguousarray(data))
    if not data.is_cuda:
        data = data.cuda()
    data = data.contiguous().reshape(-1)
    out = torch.empty(packed_bytes(data.numel()), dtype=torch.uint8, device=data.device)
    if data.dtype == torch.float16:
        call("aria_q4_0_pack_f16", data.data_ptr(), data.numel(), out.data_ptr(), _stream(data.device))
    elif data.dtype == torch.float32:
        call("aria_q4_0_pack_f32", data.data_ptr(), data.numel(), out.data_ptr(), _stream(data.device))
    else:
        raise TypeError(f"quantize_q4_0 takes f16 or f32, got {data.dtype}")
    return out


def dequantize_q4_0(blocks: torch.Tensor, n: int) -> torch.Tensor:
    """Exact (q-8)*scale of the first n elements of GGUF Q4_0 blocks, as f32."""
    _require_cuda(blocks, "blocks")
    if blocks.numel() < packed_bytes(n):
        raise ValueError("blocks too short")
    out = torch.empty(n, dtype=torch.float32, device=blocks.device)
    call("aria_q4_0_unpack_f32", blocks.data_ptr(), n, out.data_ptr(), _stream(blocks.device))
    return out


@dataclass
class Q4Weight:
    """A projection weight resident on the GPU in the library's tiled form.

    layout KN: the reference tensor is w[k][n] (w_qkv, w_out, w_ff1, w_ff2);
    layout NK: the reference tensor is w[n][k] (tied LM head `embed`).
    y = x @ W(k, n) in both cases; W has K inputs and N outputs.
    """

    buf: torch.Tensor
    layout: int
    K: int
    N: int

    @property
    def nbytes(self) -> int:
        """Q4_0 bytes the kernels stream per full pass (0.5625 B per weight)."""
        return self.K * self.N // 32 * 18

    @staticmethod
    def tiled_bytes(K: int, N: int) -> int:
        return int(_lib.lib().aria_q4_0_tiled_bytes(K, N))

    @classmethod
    def empty(cls, layout: int, K: int, N: int, device=None) -> "Q4Weight":
        nb = cls.tiled_bytes(K, N)
        if nb == 0:
            raise ValueError(f"bad shape K={K} N={N}")
        buf = torch.empty(nb, dtype=torch.uint8, device=device or "cuda")
        return cls(buf, layout, K, N)

    @classmethod
    def from_f16(cls, w: torch.Tensor, layout: int) -> "Q4Weight":
        """Quantise an f16 weight in the reference orientation: [K][N] for KN, [N][K] for NK."""
        _require_cuda(w, "w")
        if w.dtype != torch.float16 or w.dim() != 2:
            raise TypeError("w must be a 2-D f16 CUDA tensor")
        K, N = (w.shape[0], w.shape[1]) if layout == LAYOUT_KN else (w.shape[1], w.shape[0])
        q = cls.empty(layout, K, N, w.device)
        call("aria_q4_0_quantize_tiled", w.data_ptr(), layout, K, N, q.buf.data_ptr(), q.buf.numel(),
             _stream(w.device))
        return q

    @classmethod
    def from_gguf_blocks(cls, blocks: torch.Tensor, layout: int, K: int, N: int) -> "Q4Weight":
        """Upload a Q4_0 GGUF tensor (K*N/32*18 bytes in the reference's flat order)."""
        if not isinstance(blocks, torch.Tensor):
            blocks = torch.from_numpy(np.frombuffer(bytes(blocks), dtype=np.uint8).copy())
        if not blocks.is_cuda:
            blocks = blocks.cuda()
        blocks = blocks.contiguous()
        if blocks.numel() != K * N // 32 * 18:
            raise ValueError(f"expected {K * N // 32 * 18} bytes, got {blocks.numel()}")
        q = cls.empty(layout, K, N, blocks.device)
        call("aria_q4_0_repack", blocks.data_ptr(), layout, K, N, q.buf.data_ptr(), q.buf.numel(),
             _stream(blocks.device))
        return q


_KERNEL_FLAGS = {"auto": 0, "stream": _lib.FLAG_KERNEL_STREAM, "register": _lib.FLAG_KERNEL_REGISTER,
                 "tensor": _lib.FLAG_KERNEL_TENSOR}
_ACT_FLAGS = {None: 0, "gelu": _lib.FLAG_EPILOGUE_GELU}


_WORKSPACES: dict = {}


def workspace_for(K: int, N: int, M: int, device: torch.device) -> torch.Tensor | None:
    """Zero-filled device workspace for aria_q4_0_matmul_ws on `device` and the
    current stream (one per pair, grown on demand; every call leaves its
    counters zero, so it is reused as is).  None when no K split would help."""
    nbytes = int(_lib.lib().aria_q4_0_workspace_bytes(K, N, M))
    if nbytes == 0:
        return None
    key = (device.index if device.index is not None else torch.cuda.current_device(),
           torch.cuda.current_stream(device).cuda_stream)
    ws = _WORKSPACES.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 2 * (ws.numel() if ws is not None else 0)), dtype=torch.uint8, device=device)
        _WORKSPACES[key] = ws
    return ws


def matmul(x: torch.Tensor, w: Q4Weight, out: torch.Tensor | None = None, *, bias: torch.Tensor | None = None,
           alpha: float = 1.0, beta: float = 0.0, out_dtype: torch.dtype = torch.float16,
           const_weights: bool = False, kernel: str = "auto", workspace="auto",
           activation: str | None = None) -> torch.Tensor:
    """y[M, N] = act(alpha * x[M, K] @ W + bias) + beta * out, through aria_q4_0_matmul_ws.

    activation: None, or "gelu" for the reference's tanh-form GELU fused into the
    epilogue (its add_bias + gelu_fwd after ffn_up, src/transformer_cuda.rs:1789-1794).

    const_weights: the weight buffer is not written by the kernel preceding this
    call on the stream (model weights), so the kernel may start reading it early.
    kernel: "auto" (the library chooses), "stream" (streaming GEMV, M <= 8),
    "register" (register-fed decode kernel, M <= 64) or "tensor" (tcgen05 kernel).
    workspace: "auto" (a cached per-device/stream buffer sized by
    aria_q4_0_workspace_bytes), None (no K split) or a zero-initialised uint8
    CUDA tensor owned by the caller."""
    if not x.is_cuda:
        raise ValueError("x must be a CUDA tensor")
    if x.dtype != torch.float16:
        raise TypeError("x must be f16 (the reference's activation dtype)")
    x2 = x.reshape(-1, x.shape[-1])
    if x2.shape[1] != w.K:
        raise ValueError(f"x has K={x2.shape[1]}, weight has K={w.K}")
    if x2.stride(1) != 1:
        raise ValueError("x rows must be contiguous (a row stride of ldx >= K elements is allowed)")
    M = x2.shape[0]
    if out is None:
        out = torch.empty((M, w.N), dtype=out_dtype, device=x.device)
    _require_cuda(out, "out")
    ydt = {torch.float16: F16, torch.float32: F32}.get(out.dtype)
    if ydt is None:
        raise TypeError("out must be f16 or f32")
    if bias is not None:
        _require_cuda(bias, "bias")
        if bias.dtype != torch.float16 or bias.numel() != w.N:
            raise ValueError("bias must be f16 [N]")
    if isinstance(workspace, str):
        if workspace != "auto":
            raise ValueError("workspace must be 'auto', None or a uint8 CUDA tensor")
        workspace = workspace_for(w.K, w.N, M, x.device) if M > 32 else None
    if workspace is not None:
        _require_cuda(workspace, "workspace")
    call("aria_q4_0_matmul_ws", w.buf.data_ptr(), w.layout, w.K, w.N, x2.data_ptr(), M, x2.stride(0),
         out.data_ptr(), ydt, out.reshape(-1, w.N).stride(0),
         bias.data_ptr() if bias is not None else None, float(alpha), float(beta),
         workspace.data_ptr() if workspace is not None else None,
         workspace.numel() * workspace.element_size() if workspace is not None else 0,
         (_lib.FLAG_CONST_WEIGHTS if const_weights else 0) | _KERNEL_FLAGS[kernel] | _ACT_FLAGS[activation],
         _stream(x.device))
    return out


def matmul_ln(h: torch.Tensor, gamma: torch.Tensor, beta_ln: torch.Tensor, w: Q4Weight,
              out: torch.Tensor | None = None, *, eps: float = 1e-5, bias: torch.Tensor | None = None,
              beta: float = 0.0, out_dtype: torch.dtype = torch.float16, const_weights: bool = False,
              activation: str | None = None) -> torch.Tensor:
    """y = act(LayerNorm(h) @ W + bias) + beta * out through aria_q4_0_matmul_ln:
    the reference's LayerNorm followed by a projection (cpu_layer_forward,
    src/transformer_cuda.rs:1092-1096, :1145-1150) in one launch.  h is f32
    [M, K] (M <= 64), gamma / beta_ln f16 [K]."""
    _require_cuda(h, "h")
    if h.dtype != torch.float32 or h.dim() != 2 or h.shape[1] != w.K:
        raise ValueError("h must be f32 [M, K]")
    M = h.shape[0]
    if out is None:
        out = torch.empty((M, w.N), dtype=out_dtype, device=h.device)
    ydt = {torch.float16: F16, torch.float32: F32}[out.dtype]
    call("aria_q4_0_matmul_ln", w.buf.data_ptr(), w.layout, w.K, w.N, h.data_ptr(), M, h.stride(0),
         gamma.data_ptr(), beta_ln.data_ptr(), float(eps), out.data_ptr(), ydt, out.stride(0),
         bias.data_ptr() if bias is not None else None, 1.0, float(beta),
         (_lib.FLAG_CONST_WEIGHTS if const_weights else 0) | _ACT_FLAGS[activation], _stream(h.device))
    return out


def gemm_q4(a: torch.Tensor, b: Q4Weight, c: torch.Tensor, m: int, k: int, n: int,
            transa: bool = False, transb: bool | None = None, alpha: float = 1.0, beta: float = 0.0) -> None:
    """The reference's `gemm()` (transformer_cuda.rs:615-640) with a Q4_0 `b`.

    C[m,n] = alpha * A[m,k] @ op(B) + beta * C.  transb=False pairs with a KN
    weight (w_* tensors), transb=True with an NK weight (the tied `embed`).
    transa=True (used only by the reference's backward pass) is not supported.
    """
    if transa:
        raise NotImplementedError("transa=True is a training-path GEMM; Q4_0 weights are inference-only")
    want = LAYOUT_NK if transb else LAYOUT_KN
    if transb is not None and b.layout != want:
        raise ValueError("transb does not match the weight's layout")
    if (b.K, b.N) != (k, n):
        raise ValueError(f"gemm_q4: weight is {b.K}x{b.N}, call says k={k} n={n}")
    matmul(a.reshape(m, k), b, c.reshape(m, n), alpha=alpha, beta=beta)
