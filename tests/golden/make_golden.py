"""Generates tests/golden/*.json -- known-answer vectors for the Q4_0 path.

Run from the repo root:  python tests/golden/make_golden.py

Three sources of truth are combined here so that no single restatement of the
reference packer (lold3344/ARIA src/transformer_cuda.rs:549-575) is trusted alone:

1. HAND cases: inputs chosen to pin one rule each (zero block, f32 scale used
   for the division, half-away-from-zero rounding, interleaved nibble order, the
   short tail block, an f16-subnormal scale, NaN/Inf, f16 overflow of the scale,
   the f16 maximum).  Their expected bytes were worked out by hand and are
   written literally below.
2. An exact-rational restatement in pure Python (fractions.Fraction): IEEE f32
   division and f32->f16 conversion are evaluated as exact rationals and rounded
   to nearest-even by hand.  Every hand case must equal it.
3. Random cases whose bytes come from (2) and are re-checked against the C and
   numpy oracles by tests/test_oracle.py.

The projection fixture (small KN and NK matmuls) stores the fp64 output of the
dequantise-then-matmul reference computed with exact rationals of the inputs.
"""
from __future__ import annotations

import json
import math
import os
import struct
from fractions import Fraction

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


# ----------------------------------------------------------- exact IEEE helpers

def f32_from_bits(b: int) -> float:
    return struct.unpack("<f", struct.pack("<I", b))[0]


def f32_bits(x: float) -> int:
    return struct.unpack("<I", struct.pack("<f", x))[0]


def round_to_format(v: Fraction, p: int, emin: int, emax: int):
    """Round an exact nonzero rational to the binary format with precision p.

    Returns (is_inf, exp_field, mant_field, sign)."""
    sign = 1 if v < 0 else 0
    a = -v if v < 0 else v
    # exact floor(log2(a))
    e = a.numerator.bit_length() - a.denominator.bit_length()
    if Fraction(2) ** e > a:
        e -= 1
    if Fraction(2) ** (e + 1) <= a:
        e += 1
    if e < emin:
        e = emin
    quantum = Fraction(2) ** (e - (p - 1))
    m = a / quantum
    M = m.numerator // m.denominator
    rem = m - M
    if rem > Fraction(1, 2) or (rem == Fraction(1, 2) and M % 2 == 1):
        M += 1
    if M == 2 ** p:
        M = 2 ** (p - 1)
        e += 1
    bias = emax
    if e > emax:
        return True, 0, 0, sign
    if M < 2 ** (p - 1):
        return False, 0, M, sign  # subnormal (e == emin)
    return False, e + bias, M - 2 ** (p - 1), sign


def exact_f32(v: Fraction) -> Fraction | float:
    """RN-even rounding of an exact rational to f32, returned as an exact rational."""
    if v == 0:
        return Fraction(0)
    inf, ef, mf, s = round_to_format(v, 24, -126, 127)
    if inf:
        return -math.inf if s else math.inf
    if ef == 0:
        val = Fraction(mf) * Fraction(2) ** (-126 - 23)
    else:
        val = (1 + Fraction(mf, 2 ** 23)) * Fraction(2) ** (ef - 127)
    return -val if s else val


def f16_bits_of(v) -> int:
    """f16::from_f32 for a finite-or-infinite f32 value given exactly."""
    if isinstance(v, float):
        if math.isnan(v):
            return 0x7E00
        if math.isinf(v):
            return 0xFC00 if v < 0 else 0x7C00
        v = Fraction(v)
    if v == 0:
        return 0
    inf, ef, mf, s = round_to_format(v, 11, -14, 15)
    if inf:
        return (s << 15) | 0x7C00
    return (s << 15) | (ef << 10) | mf


def pack_block_exact(vals: list[float]) -> bytes:
    """One block of the reference packer, evaluated with exact rationals."""
    n = len(vals)
    # abs_max = fold(0, f32::max) over |x|: NaN ignored
    absmax: float | Fraction = Fraction(0)
    for v in vals:
        if math.isnan(v):
            continue
        av = abs(v)
        if math.isinf(av):
            absmax = math.inf
        elif absmax != math.inf and Fraction(av) > absmax:
            absmax = Fraction(av)
    if absmax == math.inf:
        scale = math.inf
    elif absmax > 0:
        scale = exact_f32(absmax / 7)
    else:
        scale = Fraction(1)
    out = bytearray(struct.pack("<H", f16_bits_of(scale)))
    qs = []
    for i in range(32):
        val = vals[i] if i < n else 0.0
        if math.isnan(val):
            q32 = 0
        elif scale == math.inf:
            q32 = 0 if not math.isinf(val) else 0  # finite/Inf = 0, Inf/Inf = NaN -> 0
        else:
            quo = exact_f32(Fraction(val) / scale)
            if isinstance(quo, float):  # overflow to Inf: saturating cast
                q32 = 2**31 - 1 if quo > 0 else -(2**31)
            else:
                aq = abs(quo)
                r = math.floor(aq + Fraction(1, 2))  # half away from zero
                r = -r if quo < 0 else r
                q32 = max(-(2**31), min(2**31 - 1, r))
        q = ((q32 + 8 + 2**31) % 2**32) - 2**31  # wrapping i32 add
        qs.append(max(0, min(15, q)))
    for j in range(16):
        out.append(qs[2 * j] | (qs[2 * j + 1] << 4))
    return bytes(out)


def quantize_exact(vals: list[float]) -> bytes:
    out = b""
    for b in range(0, max(len(vals), 0), 32):
        out += pack_block_exact(vals[b:b + 32])
    return out


def f32_list(vals) -> list[float]:
    return [f32_from_bits(f32_bits(float(v))) if not (isinstance(v, float) and math.isnan(v)) else v
            for v in vals]


# ----------------------------------------------------------- hand cases

NAN = float("nan")
INF = float("inf")
Z31 = [0.0] * 31

HAND = [
    # name, dtype, values, expected hex (worked out by hand)
    ("zero_block", "f32", [0.0] * 32, "003c" + "88" * 16),
    ("neg_zero_block", "f32", [-0.0] * 32, "003c" + "88" * 16),
    ("seven_then_zeros", "f32", [7.0] + Z31, "003c" + "8f" + "88" * 15),
    ("half_away_from_zero", "f32",
     [7.0, 0.5, -0.5, 1.5, -1.5, 2.5, -2.5, 3.5, -3.5] + [0.0] * 23,
     "003c" + "9fa7b6c584" + "88" * 11),
    ("tail_block_33", "f32", [1.0] * 33, "9230" + "ff" * 16 + "9230" + "8f" + "88" * 15),
    ("f16_subnormal_scale", "f32", [2.0 ** -20] + Z31, "0200" + "8f" + "88" * 15),
    ("nan_ignored_by_absmax", "f32", [NAN, 1.0] + [0.0] * 30, "9230" + "f8" + "88" * 15),
    ("inf_scale", "f32", [INF, 1.0, -INF] + [0.0] * 29, "007c" + "88" * 16),
    ("f16_scale_overflow", "f32", [1e38] + Z31, "007c" + "8f" + "88" * 15),
    ("f16_max", "f16", [65504.0, -65504.0, 1.0] + [0.0] * 29, "9270" + "1f" + "88" * 15),
]


def hexbits(vals, dtype):
    if dtype == "f32":
        return "".join(f"{f32_bits(v) if not math.isnan(v) else 0x7FC00000:08x}" for v in vals)
    return np.asarray(vals, dtype=np.float16).view(np.uint16).astype(">u2").tobytes().hex()


def main():
    cases = []
    for name, dtype, vals, exp_hex in HAND:
        vals = f32_list(vals)
        got = quantize_exact(vals).hex()
        assert got == exp_hex, f"{name}: exact restatement {got} != hand {exp_hex}"
        cases.append({"name": name, "dtype": dtype, "n": len(vals),
                      "input_hex": hexbits(vals, dtype), "expected_hex": exp_hex, "source": "hand"})

    # ramp -16..15: exercises every code, q = round(v*7/16) under f32 division
    ramp = [float(v) for v in range(-16, 16)]
    cases.append({"name": "ramp_-16_15", "dtype": "f32", "n": 32, "input_hex": hexbits(ramp, "f32"),
                  "expected_hex": quantize_exact(ramp).hex(), "source": "exact-rational"})

    rng = np.random.default_rng(20261201)
    for i, (n, sigma) in enumerate([(32, 1.0), (100, 0.02), (257, 3.0), (1024, 0.02)]):
        v = (rng.standard_normal(n) * sigma).astype(np.float16)
        vals = [float(t) for t in v.astype(np.float32)]
        cases.append({"name": f"random_f16_{i}_n{n}", "dtype": "f16", "n": n,
                      "input_hex": hexbits(vals, "f16"),
                      "expected_hex": quantize_exact(vals).hex(), "source": "exact-rational"})
    with open(os.path.join(HERE, "kat_q4_0.json"), "w") as f:
        json.dump({"generator": "tests/golden/make_golden.py",
                   "reference": "lold3344/ARIA src/transformer_cuda.rs:549-575",
                   "cases": cases}, f, indent=1)

    # ---- projection fixtures: y = x @ W for both layouts, exact in rationals
    proj = []
    for (layout, K, N, M, seed) in [(0, 64, 96, 3, 1), (1, 96, 64, 2, 2), (0, 32, 32, 1, 3), (1, 128, 40, 5, 4)]:
        r = np.random.default_rng(seed)
        w = (r.standard_normal(K * N) * 0.02).astype(np.float16)
        x = r.standard_normal(M * K).astype(np.float16)
        blocks = quantize_exact([float(t) for t in w.astype(np.float32)])
        # exact dequant + exact products, rounded to double once
        wq = []
        for b in range(0, len(blocks), 18):
            s = Fraction(float(np.frombuffer(blocks[b:b + 2], dtype=np.float16)[0]))
            for j in range(16):
                byte = blocks[b + 2 + j]
                wq.append((byte & 0xF) - 8)
                wq.append((byte >> 4) - 8)
            wq[-32:] = [Fraction(q) * s for q in wq[-32:]]
        xf = [Fraction(float(t)) for t in x.astype(np.float32)]
        y = []
        for m in range(M):
            for n_ in range(N):
                acc = Fraction(0)
                for k in range(K):
                    wk = wq[k * N + n_] if layout == 0 else wq[n_ * K + k]
                    acc += xf[m * K + k] * wk
                y.append(float(acc))
        proj.append({"layout": layout, "K": K, "N": N, "M": M,
                     "w_f16_hex": w.view(np.uint16).astype("<u2").tobytes().hex(),
                     "x_f16_hex": x.view(np.uint16).astype("<u2").tobytes().hex(),
                     "blocks_hex": blocks.hex(), "y_f64": y})
    with open(os.path.join(HERE, "projection_small.json"), "w") as f:
        json.dump({"generator": "tests/golden/make_golden.py",
                   "reference": "lold3344/ARIA src/transformer_cuda.rs:549-575,3322-3333,1864",
                   "cases": proj}, f)
    print("wrote", len(cases), "packer cases and", len(proj), "projection cases")


if __name__ == "__main__":
    main()
