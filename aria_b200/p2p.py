"""Host side of the peer-memory reduction of the column-split FFN
(aria_p2p_allreduce_add, p2p_allreduce.cu).

One process per GPU.  Each rank allocates one zero-filled device region
(aria_p2p_alloc) holding one f32 partial buffer per layer, a block of 8 flag
words and a 2-word state block; the 64-byte IPC handles of the regions are
exchanged over the process group (all_gather_object: any backend) and the
peers' regions mapped with aria_p2p_ipc_open.  `reduce_into(layer, h)` then
adds every rank's partial of that layer into this rank's f16 residual stream
in one kernel, waiting on the GPU (bounded) for the peers' partials.  The
partial buffer of a layer is written by the caller's ffn_down projection
through `part_ptr(layer)`.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from ._lib import call

_FLAG_BYTES = 64    # 8 flag words (one per possible rank), 64-byte block
_STATE_BYTES = 64   # [epoch, blocks finished]


class _DeviceArray:
    """A device buffer of this library seen through __cuda_array_interface__."""

    def __init__(self, ptr: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


def exchange_handles(handle: bytes, group=None) -> list[bytes]:
    """Every rank's 64-byte handle, in rank order (host-side collective)."""
    world = dist.get_world_size(group)
    out: list = [None] * world
    dist.all_gather_object(out, bytes(handle), group=group)
    return [bytes(h) for h in out]


class PeerReduction:
    def __init__(self, n: int, layers: int, group=None, wait_limit_us: int = 2_000_000):
        if n % 8 != 0:
            raise ValueError("n must be a multiple of 8")
        self.n, self.layers, self.group = n, layers, group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if self.world > 8:
            raise ValueError("at most 8 ranks")
        self.wait_limit_us = wait_limit_us
        self.part_bytes = (n * 4 + 255) // 256 * 256
        self.region_bytes = _FLAG_BYTES + _STATE_BYTES + 128 + layers * self.part_bytes
        lib = _lib.lib()
        ptr = ctypes.c_void_p()
        _lib.check("aria_p2p_alloc", lib.aria_p2p_alloc(self.region_bytes, ctypes.byref(ptr)))
        self.base = ptr.value
        self.bases = [0] * self.world
        self.bases[self.rank] = self.base
        self._opened = []
        if self.world > 1:
            h = ctypes.create_string_buffer(64)
            _lib.check("aria_p2p_ipc_handle", lib.aria_p2p_ipc_handle(ctypes.c_void_p(self.base), h))
            handles = exchange_handles(h.raw, group)
            for r, hr in enumerate(handles):
                if r == self.rank:
                    continue
                pr = ctypes.c_void_p()
                _lib.check("aria_p2p_ipc_open", lib.aria_p2p_ipc_open(ctypes.create_string_buffer(hr, 64),
                                                                      ctypes.byref(pr)))
                self.bases[r] = pr.value
                self._opened.append(pr.value)
            dist.barrier(group)  # every mapping exists before any rank's first reduction
        self.flags = [b for b in self.bases]                      # flag block at offset 0
        self.state = self.base + _FLAG_BYTES                      # this rank's state block
        self._flag_arr = (ctypes.c_void_p * self.world)(*self.flags)

    def _part(self, base: int, layer: int) -> int:
        return base + _FLAG_BYTES + _STATE_BYTES + 128 + layer * self.part_bytes

    def part_ptr(self, layer: int) -> int:
        """Device pointer of this rank's f32 partial buffer of `layer` ([n])."""
        return self._part(self.base, layer)

    def part_tensor(self, layer: int, shape) -> torch.Tensor:
        """This rank's partial buffer of `layer` as an f32 CUDA tensor (no copy)."""
        numel = 1
        for s in shape:
            numel *= int(s)
        if numel != self.n:
            raise ValueError("shape must hold n elements")
        return torch.as_tensor(_DeviceArray(self.part_ptr(layer), tuple(int(s) for s in shape), "<f4"),
                               device=torch.device("cuda", torch.cuda.current_device()))

    def reduce_into(self, layer: int, h: torch.Tensor) -> None:
        """h (f16, n elements, contiguous) += sum over ranks of their partial of `layer`."""
        if h.dtype != torch.float16 or h.numel() != self.n or not h.is_contiguous():
            raise ValueError("h must be a contiguous f16 tensor of n elements")
        parts = (ctypes.c_void_p * self.world)(*[self._part(b, layer) for b in self.bases])
        call("aria_p2p_allreduce_add", parts, self._flag_arr, self.state, self.world, self.rank, h.data_ptr(),
             self.n, self.wait_limit_us, torch.cuda.current_stream(h.device).cuda_stream)

    def close(self) -> None:
        lib = _lib.lib()
        for p in self._opened:
            lib.aria_p2p_ipc_close(ctypes.c_void_p(p))
        self._opened = []
        if self.base:
            lib.aria_p2p_free(ctypes.c_void_p(self.base))
            self.base = 0


__all__ = ["PeerReduction", "exchange_handles"]
