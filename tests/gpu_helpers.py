"""Helpers shared by the GPU parity tests (test side only)."""
import numpy as np

LAYOUT_KN, LAYOUT_NK = 0, 1


def dev_pos(i: int) -> int:
    return (i >> 1) + 4 * (i & 1)


def k_of_word(w: int) -> int:
    return 128 * (w >> 4) + 32 * (w & 3) + 8 * ((w >> 2) & 3)


def tiled_from_aos(blocks: np.ndarray, layout: int, K: int, N: int) -> np.ndarray:
    """numpy restatement of the device tiled form built from GGUF Q4_0 blocks.

    K is padded to Kp = roundup(K, 128) with code 8 and scale 0.
    qs: [N][Kp/2] bytes, row n = output feature n; word w of a row holds the 8
    consecutive k starting at 128*(w//16) + 32*(w%4) + 8*((w//4)%4), nibbles in
    the order e0 e2 e4 e6 e1 e3 e5 e7.  scales at align256(N*Kp/2):
    NK -> [Kp/128][N][4] (group-major), KN -> [N/32][Kp]."""
    Kp = (K + 127) // 128 * 128
    b = blocks.reshape(-1, 18)
    sc = b[:, 0:2].copy().view(np.uint16).reshape(-1)
    nib = b[:, 2:]
    q = np.empty((b.shape[0], 32), dtype=np.uint32)
    q[:, 0::2] = nib & 0xF
    q[:, 1::2] = nib >> 4
    flat = q.reshape(-1)
    qd = np.full((N, Kp), 8, dtype=np.uint32)
    if layout == LAYOUT_NK:
        qd[:, :K] = flat.reshape(N, K)
        rows = np.zeros((N, Kp // 32), dtype=np.uint16)
        rows[:, :K // 32] = sc.reshape(N, K // 32)
        sdev = rows.reshape(N, Kp // 128, 4).transpose(1, 0, 2)  # group-major [Kp/128][N][4]
    else:
        qd[:, :K] = flat.reshape(K, N).T
        sdev = np.zeros((N // 32, Kp), dtype=np.uint16)
        sdev[:, :K] = sc.reshape(K, N // 32).T
    words = np.zeros((N, Kp // 8), dtype=np.uint32)
    for w in range(Kp // 8):
        k0 = k_of_word(w)
        for e in range(8):
            words[:, w] |= qd[:, k0 + e] << np.uint32(4 * dev_pos(e))
    qs_bytes = words.astype("<u4").view(np.uint8).reshape(-1)
    off = (N * Kp // 2 + 255) // 256 * 256
    out = np.zeros(off + N * Kp // 16, dtype=np.uint8)
    out[:qs_bytes.size] = qs_bytes
    out[off:] = np.ascontiguousarray(sdev).astype("<u2").view(np.uint8).reshape(-1)
    return out


def tiled_regions(buf: np.ndarray, K: int, N: int):
    """(qs bytes, scale bytes) of a tiled buffer, skipping the alignment gap."""
    Kp = (K + 127) // 128 * 128
    off = (N * Kp // 2 + 255) // 256 * 256
    return buf[:N * Kp // 2], buf[off:off + N * Kp // 16]


def check_close(y, ref, max_abs=1e-2, rel_l2=1e-3, what=""):
    """Projection tolerance of the task: max-abs 1e-2 and relative L2 1e-3 vs fp64."""
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert y.shape == ref.shape, (y.shape, ref.shape)
    err = np.abs(y - ref)
    mx = float(err.max()) if err.size else 0.0
    den = float(np.linalg.norm(ref))
    rl2 = float(np.linalg.norm(y - ref) / den) if den > 0 else float(np.linalg.norm(y - ref))
    assert mx <= max_abs, f"{what}: max-abs {mx:.3e} > {max_abs}"
    assert rl2 <= rel_l2, f"{what}: rel-L2 {rl2:.3e} > {rel_l2}"
    return mx, rl2
