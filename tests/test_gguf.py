"""GGUF container: byte layout of ARIA's writer (transformer_cuda.rs:463-546),
read-back, and the Q4_0 export path (:3209-3252).  CPU tests use the oracle
packer; the GPU test exports with the device packer."""
import struct

import numpy as np
import pytest

from aria_b200 import gguf
from oracle import q4_oracle_np as npo


def _hand_built(tensors, meta):
    """Independent byte-by-byte assembly following the reference writer's lines."""
    out = bytearray()

    def s(x):
        b = x.encode()
        return struct.pack("<Q", len(b)) + b

    out += b"GGUF" + struct.pack("<I", 3) + struct.pack("<Q", len(tensors)) + struct.pack("<Q", 10)
    out += s("general.architecture") + struct.pack("<I", 8) + s("aria")
    out += s("general.name") + struct.pack("<I", 8) + s("ARIA")
    for k in ("aria.vocab_size", "aria.embedding_length", "aria.attention.head_count", "aria.block_count",
              "aria.feed_forward_length", "aria.context_length"):
        out += s(k) + struct.pack("<I", 5) + struct.pack("<I", meta[k])
    out += s("aria.adam_step") + struct.pack("<I", 4) + struct.pack("<i", meta["adam_step"])
    out += s("aria.is_checkpoint") + struct.pack("<I", 7) + b"\x00"
    off = 0
    for name, data, dt in tensors:
        out += s(name) + struct.pack("<I", 1) + struct.pack("<Q", len(data)) + struct.pack("<I", dt)
        out += struct.pack("<Q", off)
        off += (len(data) + 31) // 32 * 32
    out += b"\0" * ((32 - len(out) % 32) % 32)
    for _, data, _ in tensors:
        out += data + b"\0" * ((32 - len(data) % 32) % 32)
    return bytes(out)


META = {"aria.vocab_size": 40, "aria.embedding_length": 32, "aria.attention.head_count": 2,
        "aria.block_count": 1, "aria.feed_forward_length": 64, "aria.context_length": 16, "adam_step": 7}


def _tiny_tensors():
    rng = np.random.default_rng(0)
    d, ff, v = 32, 64, 40
    f = lambda *sh: (rng.standard_normal(sh) * 0.02).astype(np.float16)
    q = lambda a: npo.quantize_q4_0_f16(a.reshape(-1)).tobytes()
    return [("token_embd.weight", f(v, d).tobytes(), 1), ("output_norm.bias", f(d).tobytes(), 1),
            ("blk.0.attn_qkv.weight", q(f(d, 3 * d)), 2), ("blk.0.attn_out.weight", q(f(d, d)), 2),
            ("blk.0.ffn_up.weight", q(f(d, ff)), 2), ("blk.0.ffn_down.weight", q(f(ff, d)), 2),
            ("blk.0.ffn_down.bias", f(d).tobytes(), 1)]


def test_writer_matches_reference_layout(tmp_path):
    tensors = _tiny_tensors()
    p = tmp_path / "m.gguf"
    gguf.write_gguf_file(p, tensors, 40, 32, 2, 1, 64, 16, adam_step=7)
    assert p.read_bytes() == _hand_built(tensors, META)


def test_reader_round_trip(tmp_path):
    tensors = _tiny_tensors()
    p = tmp_path / "m.gguf"
    gguf.write_gguf_file(p, tensors, 40, 32, 2, 1, 64, 16, adam_step=7)
    g = gguf.read_gguf(p)
    assert g.kv["general.architecture"] == "aria"
    assert g.kv["aria.embedding_length"] == 32 and g.kv["aria.feed_forward_length"] == 64
    assert g.kv["aria.adam_step"] == 7 and g.kv["aria.is_checkpoint"] == 0
    assert list(g.tensors) == [t[0] for t in tensors]
    for name, data, dt in tensors:
        assert g.tensors[name].dtype == dt
        assert g.raw(name) == data
    # Q4_0 tensors decode back to the packer's dequantisation
    qkv = np.frombuffer(g.raw("blk.0.attn_qkv.weight"), dtype=np.uint8)
    assert gguf.expected_shape("blk.0.attn_qkv.weight", g.kv) == (32, 96, 0)
    assert npo.dequantize_q4_0(qkv, 32 * 96).shape == (32 * 96,)


def test_reader_rejects_bad_files(tmp_path):
    p = tmp_path / "bad.gguf"
    p.write_bytes(b"GGUG" + b"\0" * 40)
    with pytest.raises(ValueError):
        gguf.read_gguf(p)
    tensors = _tiny_tensors()
    good = tmp_path / "m.gguf"
    gguf.write_gguf_file(good, tensors, 40, 32, 2, 1, 64, 16)
    trunc = tmp_path / "t.gguf"
    trunc.write_bytes(good.read_bytes()[:-200])
    with pytest.raises(ValueError):
        gguf.read_gguf(trunc)


@pytest.mark.gpu
@pytest.mark.skipif(not __import__("torch").cuda.is_available(), reason="needs a CUDA device")
def test_export_and_load_on_gpu(tmp_path, coracle):
    """save_gguf_inference with the device packer: Q4_0 bytes equal the oracle's,
    and the loaded projections compute what quantize-on-device computes."""
    import torch
    from aria_b200 import q4
    from aria_b200.efkolos import EfkolosConfig, synth_f16
    cfg = EfkolosConfig(num_layers=2, d_model=128, num_heads=2, ffn_dim=256, vocab_size=300)
    d, ff = cfg.d_model, cfg.ffn_dim
    layers = []
    for i in range(cfg.num_layers):
        sd = lambda *sh, k=[0]: synth_f16(sh, 0.02, 1000 * i + len(sh) * 17 + sh[-1])
        layers.append({"w_qkv": sd(d, 3 * d), "b_qkv": sd(3 * d), "w_out": sd(d, d), "b_out": sd(d),
                       "w_ff1": sd(d, ff), "b_ff1": sd(ff), "w_ff2": sd(ff, d), "b_ff2": sd(d),
                       "ln1_g": sd(d), "ln1_b": sd(d), "ln2_g": sd(d), "ln2_b": sd(d)})
    weights = {"embed": synth_f16((cfg.vocab_size, d), 0.02, 5), "pos_embed": synth_f16((64, d), 0.02, 6),
               "ln_f_g": synth_f16((d,), 0.02, 7), "ln_f_b": synth_f16((d,), 0.02, 8), "layers": layers}
    p = tmp_path / "inf.gguf"
    gguf.save_gguf_inference(p, weights, cfg, max_seq_len=64)
    g = gguf.read_gguf(p)
    for i, l in enumerate(layers):
        for key, name in (("w_qkv", "attn_qkv"), ("w_out", "attn_out"), ("w_ff1", "ffn_up"), ("w_ff2", "ffn_down")):
            ref = coracle.quantize_q4_0_f16(l[key].cpu().numpy().reshape(-1)).tobytes()
            assert g.raw(f"blk.{i}.{name}.weight") == ref
    loaded = gguf.load_q4_projections(p)
    x = synth_f16((3, d), 1.0, 9)
    for i, l in enumerate(layers):
        a = q4.matmul(x, loaded[f"blk.{i}.attn_qkv.weight"], out_dtype=torch.float32)
        b = q4.matmul(x, q4.Q4Weight.from_f16(l["w_qkv"], q4.LAYOUT_KN), out_dtype=torch.float32)
        assert torch.equal(a, b)
