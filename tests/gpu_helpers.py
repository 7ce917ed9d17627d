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


def sampled_ref(blocks, layout, K, N, x_f16, cols, bias_f16=None, alpha=1.0):
    """fp64 reference of the output columns `cols` only (for projections too
    large to dequantise whole in a test): alpha * x @ W[:, cols] (+ bias[cols])."""
    from oracle.q4_oracle_np import dequantize_columns
    W = dequantize_columns(blocks, layout, K, N, cols).astype(np.float64)
    y = alpha * (np.asarray(x_f16, dtype=np.float16).astype(np.float64).reshape(-1, K) @ W)
    if bias_f16 is not None:
        y = y + np.asarray(bias_f16, dtype=np.float16).astype(np.float64)[cols][None, :]
    return y


def sample_columns(N, n, seed):
    """A seeded sample of n output columns of N, always holding the first and last."""
    cols = np.sort(np.random.default_rng(seed).choice(N, min(N, n), replace=False))
    cols[0], cols[-1] = 0, N - 1
    return np.unique(cols)


def run_projection(q4, coracle, layout, K, N, M, out_dtype=None, bias=False, alpha=1.0, beta=0.0, seed=0,
                   wscale=0.02, ldx=None, flags=0, gelu=False, cols=None):
    """One aria_q4_0_matmul call on seeded inputs, checked for canary damage;
    returns (y, fp64 reference).  ldx > K leaves a gap after each x row.  gelu:
    request the GELU epilogue (ARIA_Q4_FLAG_EPILOGUE_GELU) and apply it to the
    reference before the beta term.  cols: check only these output columns (the
    GPU still computes all N; y and the reference are returned for cols)."""
    import torch
    if out_dtype is None:
        out_dtype = torch.float32
    ldx = K if ldx is None else ldx
    rng = np.random.default_rng(seed + 1000 * M + K + N)
    shape = (K, N) if layout == LAYOUT_KN else (N, K)
    w = (rng.standard_normal(shape) * wscale).astype(np.float16)
    x = rng.standard_normal((M, K)).astype(np.float16)
    b = (rng.standard_normal(N) * 0.1).astype(np.float16) if bias else None
    blocks = coracle.quantize_q4_0_f16(w.reshape(-1))
    if cols is None:
        ref = coracle.matmul_ref(blocks, layout, K, N, x, b, alpha)
    else:
        ref = sampled_ref(blocks, layout, K, N, x, cols, b, alpha)
    if gelu:
        from oracle.q4_oracle_np import gelu_tanh
        ref = gelu_tanh(ref)
        flags |= 16  # ARIA_Q4_FLAG_EPILOGUE_GELU
    wq = q4.Q4Weight.from_f16(torch.from_numpy(w).cuda(), layout)
    # canaries: extra rows and columns around the output must stay untouched
    ldy = N + 8
    y0 = (rng.standard_normal((M + 2, ldy))).astype(np.float32)
    yt = torch.from_numpy(y0).to(out_dtype).cuda()
    view = yt[1:M + 1, :N]
    from aria_b200._lib import call
    from aria_b200.q4 import _stream
    xpad = np.full((M, ldx), np.float16(np.nan), dtype=np.float16)  # the gap must never be read
    xpad[:, :K] = x
    xt = torch.from_numpy(xpad).cuda()
    bt = torch.from_numpy(b).cuda() if b is not None else None
    args = (wq.buf.data_ptr(), layout, K, N, xt.data_ptr(), M, ldx, view.data_ptr(),
            0 if out_dtype == torch.float32 else 1, ldy, bt.data_ptr() if bt is not None else None,
            float(alpha), float(beta))
    if flags:
        call("aria_q4_0_matmul_ex", *args, flags, _stream())
    else:
        call("aria_q4_0_matmul", *args, _stream())
    out = yt.cpu().to(torch.float64).numpy()
    y_init = torch.from_numpy(y0).to(out_dtype).to(torch.float64).numpy()
    sel = slice(None) if cols is None else cols
    if beta != 0.0:
        ref = ref + beta * y_init[1:M + 1, :N][:, sel]
    # canaries
    assert np.array_equal(out[0], y_init[0]) and np.array_equal(out[M + 1], y_init[M + 1]), "row canary"
    assert np.array_equal(out[1:M + 1, N:], y_init[1:M + 1, N:]), "column canary"
    assert np.isfinite(out[1:M + 1, :N]).all()
    return out[1:M + 1, :N][:, sel], ref
