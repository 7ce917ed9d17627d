"""Prefill attention (aria_flash_attn_fwd, aria_attention_prefill) against the
fp64 oracle of the reference's flash_attn_fwd (lold3344/ARIA src/kernels.cu
:1298-1437; oracle/attention_np.py).

Cases: head sizes 64 (Efkolos) and 128 (the scaled config), T = 1, T not a
multiple of the 128-position tile, several tiles (causal blocks up to the
diagonal), several sequences packed in one QKV buffer (no attention across
sequences).  Tolerance: outputs max-abs 4e-3 (values up to ~4: one f16 ulp
plus the f16 rounding of the softmax weights), lse max-abs 2e-3."""
import numpy as np
import pytest
import torch

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]


def _rand(shape, seed, sigma=1.0):
    return (np.random.default_rng(seed).standard_normal(shape) * sigma).astype(np.float16)


@pytest.mark.parametrize("NH,T,dh", [(2, 1, 64), (3, 100, 64), (2, 128, 64), (1, 129, 64), (2, 300, 128),
                                     (4, 512, 64), (1, 257, 128), (2, 640, 64)])
def test_flash_attn_fwd_matches_oracle(NH, T, dh):
    from aria_b200.attention import flash_attn_fwd
    from oracle.attention_np import flash_attn_fwd as ref_fwd
    q, k, v = (_rand((NH, T, dh), 10 * T + dh + i) for i in range(3))
    scale = 1.0 / np.sqrt(dh)
    out, lse = flash_attn_fwd(*(torch.from_numpy(a).cuda() for a in (q, k, v)), scale=scale)
    torch.cuda.synchronize()
    ro, rl = ref_fwd(q, k, v, scale)
    got = out.cpu().numpy().astype(np.float64)
    assert np.abs(got - ro).max() <= 4e-3, np.abs(got - ro).max()
    assert np.abs(lse.cpu().numpy() - rl).max() <= 2e-3


@pytest.mark.parametrize("B,T,d,heads", [(3, 200, 896, 14), (1, 130, 256, 2), (2, 512, 896, 14), (2, 64, 512, 4)])
def test_attention_prefill_packed_qkv(B, T, d, heads):
    from aria_b200 import _lib
    from aria_b200.attention import attention_prefill
    from oracle.attention_np import attention_prefill as ref
    qkv = _rand((B * T, 3 * d), B + T + d)
    out_t = torch.full((B * T, d), float("nan"), dtype=torch.float16, device="cuda")
    out, lse = attention_prefill(torch.from_numpy(qkv).cuda(), B, T, heads, out=out_t, want_lse=True)
    torch.cuda.synchronize()
    ro, rl = ref(qkv, B, T, d, heads)
    got = out.cpu().numpy().astype(np.float64)
    assert np.isfinite(got).all()  # every output element written
    assert np.abs(got - ro).max() <= 4e-3
    assert np.abs(lse.cpu().numpy() - rl).max() <= 2e-3
    assert _lib.lib().aria_q4_take_device_error() == 0


@pytest.mark.parametrize("B,T,d,heads,max_seq", [(3, 200, 896, 14, 256), (2, 128, 256, 2, 300), (1, 5, 512, 8, 5)])
def test_attention_prefill_fills_kv_cache(B, T, d, heads, max_seq):
    """With caches, the same launch stores positions 0..T-1 of k and v into
    [B][max_seq][d] (bit-exact copies of the QKV columns) and leaves the rest of
    the caches untouched; the attention output is unchanged."""
    from aria_b200.attention import attention_prefill
    qkv = torch.from_numpy(_rand((B * T, 3 * d), 7 * T + d)).cuda()
    kc = torch.full((B, max_seq, d), 3.0, dtype=torch.float16, device="cuda")
    vc = torch.full((B, max_seq, d), -3.0, dtype=torch.float16, device="cuda")
    out_a, _ = attention_prefill(qkv, B, T, heads)
    out_b, _ = attention_prefill(qkv, B, T, heads, k_cache=kc, v_cache=vc)
    torch.cuda.synchronize()
    assert torch.equal(out_a, out_b)
    q3 = qkv.view(B, T, 3 * d)
    assert torch.equal(kc[:, :T], q3[:, :, d:2 * d]) and torch.equal(vc[:, :T], q3[:, :, 2 * d:])
    assert bool((kc[:, T:] == 3.0).all()) and bool((vc[:, T:] == -3.0).all())


def test_attention_rejects_bad_arguments():
    from aria_b200 import _lib
    lib = _lib.lib()
    x = torch.zeros(4, 3 * 96, dtype=torch.float16, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert lib.aria_attention_prefill(x.data_ptr(), 1, 4, 96, 3, x.data_ptr(), None, None, None, 0,
                                      s) == _lib.EUNSUPPORTED  # dh 32
    assert lib.aria_attention_prefill(x.data_ptr(), 1, 4, 96, 5, x.data_ptr(), None, None, None, 0,
                                      s) == _lib.EINVAL  # d % heads
    assert lib.aria_attention_prefill(x.data_ptr(), 1, 4, 128, 2, x.data_ptr(), None, x.data_ptr(), None, 8,
                                      s) == _lib.EINVAL  # one cache without the other
    assert lib.aria_attention_prefill(x.data_ptr(), 1, 4, 128, 2, x.data_ptr(), None, x.data_ptr(), x.data_ptr(), 3,
                                      s) == _lib.ESIZE  # cache shorter than the prompt
    assert lib.aria_flash_attn_fwd(x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), None, 1, 4, 48, 0.1,
                                   s) == _lib.EUNSUPPORTED
    assert lib.aria_flash_attn_fwd(x.data_ptr() + 2, x.data_ptr(), x.data_ptr(), x.data_ptr(), None, 1, 4, 64, 0.1,
                                   s) == _lib.EALIGN
    assert lib.aria_flash_attn_fwd(x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), None, 0, 4, 64, 0.1,
                                   s) == _lib.OK  # nothing to do
