"""CPU checks of the tiled-layout restatement used by the GPU tests."""
import numpy as np

from oracle import q4_oracle_np as npo
from tests.gpu_helpers import LAYOUT_KN, LAYOUT_NK, dev_pos, k_of_word, tiled_from_aos, tiled_regions


def test_word_map_is_a_permutation():
    ks = sorted(k_of_word(w) for w in range(16 * 3))
    assert ks == list(range(0, 128 * 3, 8))
    assert sorted(dev_pos(i) for i in range(8)) == list(range(8))


def _decode_tiled(buf, layout, K, N):
    """Inverse of tiled_from_aos: recover (q, scale) per element of W(k, n)."""
    Kp = (K + 127) // 128 * 128
    qs, sc = tiled_regions(buf, K, N)
    words = qs.view("<u4").reshape(N, Kp // 8)
    q = np.zeros((N, Kp), dtype=np.int64)
    for w in range(Kp // 8):
        for e in range(8):
            q[:, k_of_word(w) + e] = (words[:, w] >> (4 * dev_pos(e))) & 0xF
    s = sc.view("<u2").view(np.float16).astype(np.float32)
    if layout == LAYOUT_NK:
        s = np.repeat(s.reshape(Kp // 128, N, 4).transpose(1, 0, 2).reshape(N, Kp // 32), 32, axis=1)
    else:
        s = np.repeat(s.reshape(N // 32, Kp), 32, axis=0)
    return ((q - 8) * s)[:, :K]


def test_tiled_roundtrip_matches_dequant():
    rng = np.random.default_rng(3)
    for layout, K, N in [(LAYOUT_KN, 160, 64), (LAYOUT_NK, 224, 40), (LAYOUT_NK, 128, 3)]:
        shape = (K, N) if layout == LAYOUT_KN else (N, K)
        w = (rng.standard_normal(shape) * 0.02).astype(np.float16)
        blocks = npo.quantize_q4_0_f16(w.reshape(-1))
        wd = npo.dequantize_q4_0(blocks, K * N).reshape(shape)
        wt = wd.T if layout == LAYOUT_KN else wd  # [N][K]
        got = _decode_tiled(tiled_from_aos(blocks, layout, K, N), layout, K, N)
        assert np.array_equal(got, wt)
