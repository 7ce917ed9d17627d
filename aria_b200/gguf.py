"""GGUF v3 container in ARIA's dialect: writer (byte-identical) and Q4_0 reader.

Writer: `write_gguf_file` reproduces lold3344/ARIA src/transformer_cuda.rs:463-546
byte for byte (magic, version 3, u64 counts, the fixed KV set with types
8/5/4/7, 1-D tensor descriptors whose dim[0] is the tensor's BYTE length, data
aligned to 32 bytes).  `save_gguf_inference` follows :3209-3252: the four
projection matrices of each layer as Q4_0 (dtype 2, packed on the GPU by the
bit-exact packer), everything else as F16 (dtype 1), no tokenizer, is_checkpoint
false.

Reader: the reference cannot read its own Q4_0 export (load_checkpoint_internal
ignores the dtype and reads dim[0] elements of f16, :3046-3065, and requires a
tokenizer, :3198-3202).  `read_gguf` parses the container without those
assumptions: it accepts dim[0] as either the byte length (ARIA's writer) or the
element count (standard GGUF) and takes shapes from the aria.* metadata.
`load_q4_projections` uploads the Q4_0 tensors into the kernels' tiled form.
"""
from __future__ import annotations

import io
import os
import struct
from dataclasses import dataclass, field

import numpy as np

GGUF_F32, GGUF_F16, GGUF_Q4_0 = 0, 1, 2
_T_U32, _T_I32, _T_BOOL, _T_STR = 4, 5, 7, 8  # reference uses 5 for u32 and 4 for i32 (:501, :506)
ALIGN = 32


def _wstr(w, s: str) -> None:
    b = s.encode()
    w.write(struct.pack("<Q", len(b)))
    w.write(b)


def write_gguf_file(path, tensors, vocab_size: int, d_model: int, num_heads: int, num_layers: int,
                    ffn_dim: int, max_seq_len: int, adam_step: int = 0, is_checkpoint: bool = False,
                    tokenizer_json: str | None = None) -> None:
    """tensors: list of (name, bytes-like data, dtype) in file order."""
    kv_u32 = [("aria.vocab_size", vocab_size), ("aria.embedding_length", d_model),
              ("aria.attention.head_count", num_heads), ("aria.block_count", num_layers),
              ("aria.feed_forward_length", ffn_dim), ("aria.context_length", max_seq_len)]
    n_kv = 2 + len(kv_u32) + 2 + (1 if tokenizer_json is not None else 0)
    w = io.BytesIO()
    w.write(b"GGUF")
    w.write(struct.pack("<I", 3))
    w.write(struct.pack("<Q", len(tensors)))
    w.write(struct.pack("<Q", n_kv))
    for k, v in (("general.architecture", "aria"), ("general.name", "ARIA")):
        _wstr(w, k)
        w.write(struct.pack("<I", _T_STR))
        _wstr(w, v)
    for k, v in kv_u32:
        _wstr(w, k)
        w.write(struct.pack("<I", _T_I32))  # the reference tags its u32 values with type id 5
        w.write(struct.pack("<I", int(v) & 0xFFFFFFFF))
    _wstr(w, "aria.adam_step")
    w.write(struct.pack("<I", _T_U32))
    w.write(struct.pack("<i", int(adam_step)))
    _wstr(w, "aria.is_checkpoint")
    w.write(struct.pack("<I", _T_BOOL))
    w.write(bytes([1 if is_checkpoint else 0]))
    if tokenizer_json is not None:
        _wstr(w, "tokenizer.aria.data")
        w.write(struct.pack("<I", _T_STR))
        _wstr(w, tokenizer_json)
    offsets, cur = [], 0
    datas = []
    for (_, data, _) in tensors:
        b = bytes(memoryview(data).cast("B")) if not isinstance(data, (bytes, bytearray)) else bytes(data)
        datas.append(b)
        offsets.append(cur)
        cur += (len(b) + ALIGN - 1) // ALIGN * ALIGN
    for (name, _, dtype), b, off in zip(tensors, datas, offsets):
        _wstr(w, name)
        w.write(struct.pack("<I", 1))        # n_dims
        w.write(struct.pack("<Q", len(b)))   # dim[0] = byte length, as the reference writes it
        w.write(struct.pack("<I", dtype))
        w.write(struct.pack("<Q", off))
    w.write(b"\0" * ((ALIGN - w.tell() % ALIGN) % ALIGN))
    for b in datas:
        w.write(b)
        w.write(b"\0" * ((ALIGN - len(b) % ALIGN) % ALIGN))
    tmp = str(path) + ".tmp"
    with open(tmp, "wb") as f:
        f.write(w.getvalue())
    os.replace(tmp, path)


@dataclass
class GgufTensor:
    name: str
    dtype: int
    dims: tuple
    offset: int
    nbytes: int


@dataclass
class GgufFile:
    path: str
    version: int
    kv: dict = field(default_factory=dict)
    tensors: dict = field(default_factory=dict)
    data_start: int = 0

    def raw(self, name: str) -> bytes:
        t = self.tensors[name]
        with open(self.path, "rb") as f:
            f.seek(self.data_start + t.offset)
            b = f.read(t.nbytes)
        if len(b) != t.nbytes:
            raise ValueError(f"{name}: truncated file")
        return b


def _rstr(r) -> str:
    (n,) = struct.unpack("<Q", r.read(8))
    if n > 1 << 32:
        raise ValueError("implausible string length")
    return r.read(n).decode("utf-8", errors="replace")


_SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<B", 10: "<Q", 11: "<q", 12: "<d"}


def _rvalue(r, t: int):
    if t == _T_STR:
        return _rstr(r)
    if t in _SCALAR:
        fmt = _SCALAR[t]
        return struct.unpack(fmt, r.read(struct.calcsize(fmt)))[0]
    if t == 9:  # array
        (et,) = struct.unpack("<I", r.read(4))
        (n,) = struct.unpack("<Q", r.read(8))
        return [_rvalue(r, et) for _ in range(n)]
    raise ValueError(f"unknown GGUF value type {t}")


def _elem_bytes(dtype: int, n: int) -> int:
    if dtype == GGUF_F32:
        return 4 * n
    if dtype == GGUF_F16:
        return 2 * n
    if dtype == GGUF_Q4_0:
        return (n + 31) // 32 * 18
    raise ValueError(f"unsupported dtype {dtype}")


def expected_shape(name: str, kv: dict):
    """(K, N, layout) of a projection tensor from the aria.* metadata, or None."""
    d = kv.get("aria.embedding_length")
    ff = kv.get("aria.feed_forward_length")
    v = kv.get("aria.vocab_size")
    tail = name.split(".", 2)[-1] if name.startswith("blk.") else name
    if tail == "attn_qkv.weight":
        return (d, 3 * d, 0)
    if tail == "attn_out.weight":
        return (d, d, 0)
    if tail == "ffn_up.weight":
        return (d, ff, 0)
    if tail == "ffn_down.weight":
        return (ff, d, 0)
    if tail == "token_embd.weight":
        return (d, v, 1)
    return None


def read_gguf(path) -> GgufFile:
    with open(path, "rb") as r:
        if r.read(4) != b"GGUF":
            raise ValueError("not a GGUF file")
        (ver,) = struct.unpack("<I", r.read(4))
        if ver != 3:
            raise ValueError(f"GGUF version {ver} unsupported")
        n_t, n_kv = struct.unpack("<QQ", r.read(16))
        g = GgufFile(str(path), ver)
        for _ in range(n_kv):
            k = _rstr(r)
            (t,) = struct.unpack("<I", r.read(4))
            g.kv[k] = _rvalue(r, t)
        descs = []
        for _ in range(n_t):
            name = _rstr(r)
            (nd,) = struct.unpack("<I", r.read(4))
            dims = struct.unpack("<" + "Q" * nd, r.read(8 * nd))
            dtype, off = struct.unpack("<IQ", r.read(12))
            descs.append((name, dtype, dims, off))
        pos = r.tell()
        g.data_start = (pos + ALIGN - 1) // ALIGN * ALIGN
        r.seek(0, 2)
        size = r.tell()
    for name, dtype, dims, off in descs:
        shape = expected_shape(name, g.kv)
        if len(dims) == 1:
            if shape is not None and dims[0] == shape[0] * shape[1]:
                nbytes = _elem_bytes(dtype, dims[0])  # standard GGUF: element count
            elif shape is not None and dims[0] == _elem_bytes(dtype, shape[0] * shape[1]):
                nbytes = dims[0]                      # ARIA's writer: byte length
            else:
                nbytes = dims[0]                      # ARIA: bytes for every tensor it writes
        else:
            nbytes = _elem_bytes(dtype, int(np.prod(dims)))
        if g.data_start + off + nbytes > size:
            raise ValueError(f"{name}: descriptor points past the end of the file")
        g.tensors[name] = GgufTensor(name, dtype, tuple(dims), off, nbytes)
    return g


# ------------------------------------------------------------------ GPU export / import

def save_gguf_inference(path, weights: dict, cfg, max_seq_len: int = 2048, adam_step: int = 0) -> None:
    """TransformerModel::save_gguf_inference (transformer_cuda.rs:3209-3252).

    `weights` maps the reference's parameter names to f16 tensors (CUDA or CPU):
    embed, pos_embed, ln_f_g, ln_f_b and layers[i] dicts with w_qkv, b_qkv, w_out,
    b_out, w_ff1, b_ff1, w_ff2, b_ff2, ln1_g, ln1_b, ln2_g, ln2_b.  The four w_*
    matrices are packed to Q4_0 on the GPU (byte-identical to quantize_q4_0)."""
    import torch
    from .q4 import quantize_q4_0

    def f16(t):
        t = t.detach()
        if t.dtype != torch.float16:
            raise TypeError("F16 tensors expected")
        return t.contiguous().cpu().numpy().tobytes()

    def q4(t):
        return quantize_q4_0(t.detach().contiguous()).cpu().numpy().tobytes()

    tensors = [("token_embd.weight", f16(weights["embed"]), GGUF_F16),
               ("position_embd.weight", f16(weights["pos_embed"]), GGUF_F16),
               ("output_norm.weight", f16(weights["ln_f_g"]), GGUF_F16),
               ("output_norm.bias", f16(weights["ln_f_b"]), GGUF_F16)]
    for i, l in enumerate(weights["layers"]):
        tensors += [(f"blk.{i}.attn_qkv.weight", q4(l["w_qkv"]), GGUF_Q4_0),
                    (f"blk.{i}.attn_out.weight", q4(l["w_out"]), GGUF_Q4_0),
                    (f"blk.{i}.ffn_up.weight", q4(l["w_ff1"]), GGUF_Q4_0),
                    (f"blk.{i}.ffn_down.weight", q4(l["w_ff2"]), GGUF_Q4_0),
                    (f"blk.{i}.attn_qkv.bias", f16(l["b_qkv"]), GGUF_F16),
                    (f"blk.{i}.attn_out.bias", f16(l["b_out"]), GGUF_F16),
                    (f"blk.{i}.ffn_up.bias", f16(l["b_ff1"]), GGUF_F16),
                    (f"blk.{i}.ffn_down.bias", f16(l["b_ff2"]), GGUF_F16),
                    (f"blk.{i}.attn_norm.weight", f16(l["ln1_g"]), GGUF_F16),
                    (f"blk.{i}.attn_norm.bias", f16(l["ln1_b"]), GGUF_F16),
                    (f"blk.{i}.ffn_norm.weight", f16(l["ln2_g"]), GGUF_F16),
                    (f"blk.{i}.ffn_norm.bias", f16(l["ln2_b"]), GGUF_F16)]
    write_gguf_file(path, tensors, cfg.vocab_size, cfg.d_model, cfg.num_heads, cfg.num_layers, cfg.ffn_dim,
                    max_seq_len, adam_step, False, None)


def load_q4_projections(path, device="cuda") -> dict:
    """Every Q4_0 projection of an ARIA inference GGUF as a device Q4Weight (tiled)."""
    import torch
    from .q4 import Q4Weight
    g = read_gguf(path)
    out = {}
    for name, t in g.tensors.items():
        if t.dtype != GGUF_Q4_0:
            continue
        shape = expected_shape(name, g.kv)
        if shape is None:
            raise ValueError(f"{name}: Q4_0 tensor with no known shape")
        K, N, layout = shape
        b = torch.frombuffer(bytearray(g.raw(name)), dtype=torch.uint8).to(device)
        out[name] = Q4Weight.from_gguf_blocks(b, layout, K, N)
    return out
