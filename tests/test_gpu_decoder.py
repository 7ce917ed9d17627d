"""GPU decode step with KV cache (aria_b200.decoder) against the numpy oracle.

The reference's cached step runs on the CPU (lold3344/ARIA
src/transformer_cuda.rs `step` :1286-1324, `cpu_layer_forward` :1059-1166);
oracle/decode_step_np.py restates it in fp64 on the exactly dequantised Q4_0
weights, rounding to f16 where the GPU stores f16.  Checked here:

* the LayerNorm kernel (cpu_layernorm :3271-3293) and the single-token
  attention kernel (cache append + softmax over positions 0..pos, :1098-1137)
  on their own, against numpy;
* whole decode steps of several sequences over several positions (the caches
  filled by earlier steps), logits against the oracle.

Tolerance on logits and kernel outputs: max-abs 1e-2 and relative L2 1e-3
(the projection bar); the f16 outputs of the single kernels (magnitudes up to
~6): max-abs 4e-3, one f16 ulp at that size."""
import numpy as np
import pytest
import torch

from tests.gpu_helpers import check_close

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]


def _stream():
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("M,d", [(1, 896), (3, 896), (2, 4096), (5, 200)])
def test_layernorm_kernel(M, d):
    from aria_b200 import _lib
    from oracle.decode_step_np import layernorm
    rng = np.random.default_rng(d + M)
    x = (rng.standard_normal((M, d)) * 3 + 0.5).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(d)).astype(np.float16)
    b = (0.1 * rng.standard_normal(d)).astype(np.float16)
    xt, gt, bt = (torch.from_numpy(a).cuda() for a in (x, g, b))
    y = torch.zeros(M, d + 8, dtype=torch.float16, device="cuda")
    _lib.call("aria_layernorm_f32", xt.data_ptr(), M, d, gt.data_ptr(), bt.data_ptr(), 1e-5, y.data_ptr(), d + 8,
              _stream())
    torch.cuda.synchronize()
    ref = layernorm(x, g.astype(np.float64), b.astype(np.float64))
    got = y.cpu().numpy().astype(np.float64)
    assert np.abs(got[:, :d] - ref).max() <= 4e-3
    assert not got[:, d:].any()  # the row gap is not written


@pytest.mark.parametrize("M,d,heads,positions", [(1, 896, 14, [0]), (2, 896, 14, [5, 63]),
                                                   (3, 4096, 32, [1, 100, 255]), (1, 256, 8, [255])])
def test_attention_kernel(M, d, heads, positions):
    from aria_b200 import _lib
    rng = np.random.default_rng(d + M)
    max_seq, dh = 256, d // heads
    qkv = rng.standard_normal((M, 3 * d)).astype(np.float16)
    kc = rng.standard_normal((M, max_seq, d)).astype(np.float16)
    vc = rng.standard_normal((M, max_seq, d)).astype(np.float16)
    q_t, k_t, v_t = (torch.from_numpy(a).cuda() for a in (qkv, kc, vc))
    pos_t = torch.tensor(positions, dtype=torch.int32, device="cuda")
    out = torch.empty(M, d, dtype=torch.float16, device="cuda")
    _lib.call("aria_attention_decode", q_t.data_ptr(), M, d, heads, k_t.data_ptr(), v_t.data_ptr(), max_seq,
              pos_t.data_ptr(), out.data_ptr(), _stream())
    torch.cuda.synchronize()
    kc2, vc2 = k_t.cpu().numpy(), v_t.cpu().numpy()
    ref = np.zeros((M, d))
    for m, p in enumerate(positions):
        kc[m, p], vc[m, p] = qkv[m, d:2 * d], qkv[m, 2 * d:]
        for h in range(heads):
            q = qkv[m, h * dh:(h + 1) * dh].astype(np.float64)
            K = kc[m, :p + 1, h * dh:(h + 1) * dh].astype(np.float64)
            V = vc[m, :p + 1, h * dh:(h + 1) * dh].astype(np.float64)
            s = K @ q / np.sqrt(dh)
            e = np.exp(s - s.max())
            ref[m, h * dh:(h + 1) * dh] = (e / e.sum()) @ V
    assert np.array_equal(kc2, kc) and np.array_equal(vc2, vc)  # only the new rows changed
    assert np.abs(out.cpu().numpy().astype(np.float64) - ref).max() <= 4e-3


def test_embed_kernel_clamps():
    from aria_b200 import _lib
    V, S, d = 50, 16, 64
    rng = np.random.default_rng(3)
    emb = rng.standard_normal((V, d)).astype(np.float16)
    pos = rng.standard_normal((S, d)).astype(np.float16)
    tok = np.array([0, 7, 49, 120], dtype=np.int32)    # 120 -> 49
    ps = np.array([0, 15, 3, 40], dtype=np.int32)      # 40 -> 15
    e_t, p_t, tk_t, ps_t = (torch.from_numpy(a).cuda() for a in (emb, pos, tok, ps))
    h = torch.empty(4, d, dtype=torch.float32, device="cuda")
    _lib.call("aria_embed_f16", e_t.data_ptr(), p_t.data_ptr(), V, S, d, tk_t.data_ptr(), ps_t.data_ptr(), 4,
              h.data_ptr(), _stream())
    torch.cuda.synchronize()
    ref = emb[np.minimum(tok, V - 1)].astype(np.float32) + pos[np.minimum(ps, S - 1)].astype(np.float32)
    assert np.array_equal(h.cpu().numpy(), ref)


@pytest.mark.parametrize("layout,K,N,M", [(0, 896, 2688, 1), (0, 896, 3584, 5), (0, 4096, 1024, 16),
                                          (1, 896, 1000, 40), (0, 256, 512, 64), (1, 896, 2048, 3),
                                          (0, 800, 1024, 2), (0, 896, 896, 8), (0, 4096, 4096, 1)])
def test_layernorm_prologue(coracle, layout, K, N, M):
    """aria_q4_0_matmul_ln against the fp64 oracle of LayerNorm (rounded to f16,
    as the projection reads it) followed by the projection, with bias and the
    GELU epilogue; and against the separate LayerNorm kernel + projection."""
    from aria_b200 import _lib, q4
    from oracle.decode_step_np import f16, layernorm
    from oracle.q4_oracle_np import gelu_tanh
    rng = np.random.default_rng(K + N + M)
    h = (rng.standard_normal((M, K)) * 2 + 0.3).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(K)).astype(np.float16)
    b = (0.1 * rng.standard_normal(K)).astype(np.float16)
    bias = (0.05 * rng.standard_normal(N)).astype(np.float16)
    shape = (K, N) if layout == 0 else (N, K)
    w = (rng.standard_normal(shape) * 0.02).astype(np.float16)
    blocks = coracle.quantize_q4_0_f16(w.reshape(-1))
    wq = q4.Q4Weight.from_f16(torch.from_numpy(w).cuda(), layout)
    ht, gt, bt, biast = (torch.from_numpy(a).cuda() for a in (h, g, b, bias))
    y = q4.matmul_ln(ht, gt, bt, wq, bias=biast, out_dtype=torch.float32, activation="gelu")
    xn = torch.empty(M, K, dtype=torch.float16, device="cuda")
    _lib.call("aria_layernorm_f32", ht.data_ptr(), M, K, gt.data_ptr(), bt.data_ptr(), 1e-5, xn.data_ptr(), K,
              _stream())
    y2 = q4.matmul(xn, wq, bias=biast, out_dtype=torch.float32, activation="gelu", kernel="register")
    torch.cuda.synchronize()
    xref = f16(layernorm(h, g.astype(np.float64), b.astype(np.float64)))
    ref = gelu_tanh(coracle.matmul_ref(blocks, layout, K, N, xref.astype(np.float16), bias))
    check_close(y.cpu().numpy(), ref, what=f"LayerNorm prologue {layout} {K}x{N} M={M}")
    check_close(y.cpu().numpy(), y2.cpu().numpy().astype(np.float64), what="prologue vs separate LayerNorm")


def _oracle_params(w):
    p = {k: v.cpu().numpy() for k, v in w.f16.items()}
    for i, lp in enumerate(w.layers):
        for name in ("b_qkv", "b_out", "b_up", "b_down", "ln1_g", "ln1_b", "ln2_g", "ln2_b"):
            p[f"{i}.{name}"] = getattr(lp, name).cpu().numpy()
    p["lnf_g"], p["lnf_b"] = w.lnf_g.cpu().numpy(), w.lnf_b.cpu().numpy()
    p["pos"] = w.pos_embed.cpu().numpy()
    return p


@pytest.mark.parametrize("cfg_kw,M,steps", [
    (dict(num_layers=2, d_model=256, num_heads=4, ffn_dim=1024, vocab_size=1000), 2, 6),
    (dict(num_layers=3, d_model=896, num_heads=14, ffn_dim=3584, vocab_size=31500), 1, 4),
])
def test_decode_steps_against_oracle(coracle, cfg_kw, M, steps):
    from aria_b200.decoder import Decoder, DecoderWeights
    from aria_b200.efkolos import EfkolosConfig
    from oracle.decode_step_np import DecodeOracle
    cfg = EfkolosConfig(**cfg_kw)
    w = DecoderWeights(cfg, max_seq=64, seed=11)
    dec = Decoder(w, M=M)
    orc = DecodeOracle(coracle, _oracle_params(w), cfg, 64, M)
    rng = np.random.default_rng(5)
    pos0 = [2 * m for m in range(M)]  # sequences at different positions (earlier cache rows stay zero in both)
    for t in range(steps):
        tokens = rng.integers(0, cfg.vocab_size, M)
        positions = [p + t for p in pos0]
        got = dec.step(tokens, positions).cpu().numpy().astype(np.float64)
        ref = orc.step(tokens, positions)
        check_close(got, ref, what=f"decode step {t} (d_model {cfg.d_model})")
    # the caches hold the oracle's f16 k and v rows of every step (to f16 rounding)
    last = max(pos0) + steps
    for i in range(cfg.num_layers):
        got_k = dec.k_cache[i][:, :last].cpu().numpy().astype(np.float64)
        got_v = dec.v_cache[i][:, :last].cpu().numpy().astype(np.float64)
        assert np.abs(got_k - orc.k[i][:, :last]).max() <= 2e-2
        assert np.abs(got_v - orc.v[i][:, :last]).max() <= 2e-2


@pytest.mark.parametrize("cfg_kw,M,T", [
    (dict(num_layers=2, d_model=256, num_heads=4, ffn_dim=1024, vocab_size=1000), 2, 40),
    (dict(num_layers=1, d_model=896, num_heads=14, ffn_dim=3584, vocab_size=3000), 1, 130),
])
def test_prefill_then_decode_against_oracle(coracle, cfg_kw, M, T):
    """Decoder.prefill (whole prompts: tensor-core projections and causal
    attention) gives, at every position, the logits the oracle's cached step
    gives when fed the prompt token by token; the caches it fills let `step`
    continue at position T."""
    from aria_b200.decoder import Decoder, DecoderWeights
    from aria_b200.efkolos import EfkolosConfig
    from oracle.decode_step_np import DecodeOracle
    cfg = EfkolosConfig(**cfg_kw)
    w = DecoderWeights(cfg, max_seq=256, seed=12)
    dec = Decoder(w, M=M)
    orc = DecodeOracle(coracle, _oracle_params(w), cfg, 256, M)
    rng = np.random.default_rng(9)
    prompt = rng.integers(0, cfg.vocab_size, (M, T))
    got = dec.prefill(prompt).cpu().numpy().astype(np.float64).reshape(M, T, -1)
    for t in range(T):
        ref = orc.step(prompt[:, t], [t] * M)
        if t % 13 == 0 or t == T - 1:
            check_close(got[:, t], ref, what=f"prefill logits at position {t}")
    for s in range(2):
        tokens = rng.integers(0, cfg.vocab_size, M)
        out = dec.step(tokens, [T + s] * M).cpu().numpy().astype(np.float64)
        check_close(out, orc.step(tokens, [T + s] * M), what=f"decode step {s} after prefill")
