"""Causal attention over whole prompts (prefill) through libaria_q4.so.

Host mirror of the reference's flash-attention forward (lold3344/ARIA
src/kernels.cu `flash_attn_fwd` :1298-1437): same tensors, layouts and outputs,
computed by the tcgen05 kernel behind `aria_flash_attn_fwd`.  `attention_prefill`
reads the packed output of the QKV projection directly (the layout the Q4_0
prefill step produces) and writes the [tokens][d] input of attn_out.  There is
no fallback: without the library or a B200 every call raises.
"""
from __future__ import annotations

import math

import torch

from ._lib import call


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _check(t: torch.Tensor, name: str, shape=None) -> None:
    if not t.is_cuda or t.dtype != torch.float16 or not t.is_contiguous():
        raise TypeError(f"{name} must be a contiguous f16 CUDA tensor")
    if shape is not None and tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name} must have shape {tuple(shape)}, got {tuple(t.shape)}")


def flash_attn_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float | None = None,
                   out: torch.Tensor | None = None, want_lse: bool = True):
    """q, k, v: f16 [NH][T][dh] (dh 64 or 128).  Returns (out [NH][T][dh] f16,
    lse [NH][T] f32 or None) like the reference kernel (causal; lse = max +
    ln(sum of exp) per query row)."""
    _check(q, "q")
    NH, T, dh = q.shape
    _check(k, "k", q.shape)
    _check(v, "v", q.shape)
    if scale is None:
        scale = 1.0 / math.sqrt(dh)
    if out is None:
        out = torch.empty_like(q)
    _check(out, "out", q.shape)
    lse = torch.empty(NH, T, dtype=torch.float32, device=q.device) if want_lse else None
    call("aria_flash_attn_fwd", q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
         lse.data_ptr() if lse is not None else None, NH, T, dh, float(scale), _stream(q.device))
    return out, lse


def attention_prefill(qkv: torch.Tensor, B: int, T: int, heads: int, out: torch.Tensor | None = None,
                      want_lse: bool = False, k_cache: torch.Tensor | None = None,
                      v_cache: torch.Tensor | None = None):
    """qkv: f16 [B*T][3d] (the QKV projection of B sequences of T tokens).
    Returns (out f16 [B*T][d] with the heads side by side, lse [B][heads][T] or
    None); scale 1/sqrt(d / heads), causal within each sequence.  k_cache,
    v_cache (f16 [B][max_seq][d], both or neither): positions 0..T-1 of the
    keys and values are written there in the same launch."""
    _check(qkv, "qkv")
    if qkv.dim() != 2 or qkv.shape[0] != B * T or qkv.shape[1] % 3 != 0:
        raise ValueError("qkv must be [B*T][3d]")
    d = qkv.shape[1] // 3
    if out is None:
        out = torch.empty(B * T, d, dtype=torch.float16, device=qkv.device)
    _check(out, "out", (B * T, d))
    lse = torch.empty(B, heads, T, dtype=torch.float32, device=qkv.device) if want_lse else None
    max_seq = 0
    if (k_cache is None) != (v_cache is None):
        raise ValueError("k_cache and v_cache go together")
    if k_cache is not None:
        _check(k_cache, "k_cache")
        _check(v_cache, "v_cache", k_cache.shape)
        if k_cache.dim() != 3 or k_cache.shape[0] != B or k_cache.shape[2] != d:
            raise ValueError("caches must be [B][max_seq][d]")
        max_seq = k_cache.shape[1]
    call("aria_attention_prefill", qkv.data_ptr(), B, T, d, heads, out.data_ptr(),
         lse.data_ptr() if lse is not None else None,
         k_cache.data_ptr() if k_cache is not None else None,
         v_cache.data_ptr() if v_cache is not None else None, max_seq, _stream(qkv.device))
    return out, lse


__all__ = ["flash_attn_fwd", "attention_prefill"]
