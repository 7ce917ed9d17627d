"""Single-projection runs for profiling (ncu) and quick timing.

    python -m aria_b200.profile_cases --case lm_head --M 1 --launches 3
    python -m aria_b200.profile_cases --case ffn_up --M 4096 --launches 3 --time

Cases are the Efkolos projections (lold3344/ARIA src/transformer_cuda.rs:1583,
:1686, :1753, :1805, :1864) and their scaled-up (d_model 4096) counterparts,
with seeded synthetic weights quantised on the device.  Each launch goes
through the public C ABI (aria_q4_0_matmul).  With --time, launches are
captured in a CUDA graph over weight copies larger than 4x L2 and timed with
CUDA events.
"""
from __future__ import annotations

import argparse
import json

import torch

from . import q4
from .efkolos import EFKOLOS, SCALED, synth_f16


def case_shape(name: str):
    cfg = SCALED if name.startswith("scaled_") else EFKOLOS
    base = name.replace("scaled_", "")
    for (n, lay, K, N, s) in cfg.projections() + [cfg.lm_head()]:
        if n.endswith(base) or n == base:
            return lay, K, N, s
    raise SystemExit(f"unknown case {name}")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", default="lm_head")
    ap.add_argument("--M", type=int, default=1)
    ap.add_argument("--launches", type=int, default=3)
    ap.add_argument("--time", action="store_true")
    args = ap.parse_args()
    lay, K, N, sigma = case_shape(args.case)
    shape = (K, N) if lay == q4.LAYOUT_KN else (N, K)
    w = q4.Q4Weight.from_f16(synth_f16(shape, sigma, 1), lay)
    x = synth_f16((args.M, K), 1.0, 2)
    y = torch.empty(args.M, N, dtype=torch.float16, device="cuda")
    for _ in range(args.launches):
        q4.matmul(x, w, y)
    torch.cuda.synchronize()
    out = {"case": args.case, "K": K, "N": N, "M": args.M}
    if args.time:
        l2 = torch.cuda.get_device_properties(0).L2_cache_size
        ncopy = max(4, -(-4 * l2 // w.nbytes))
        pool = [q4.Q4Weight(w.buf.clone(), lay, K, N) for _ in range(ncopy)]
        n = max(32, min(256, ncopy))
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                for j in range(n):
                    q4.matmul(x, pool[j % ncopy], y)
            g.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            for _ in range(5):
                g.replay()
            e1.record(s)
            torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1000 / (5 * n)
        out.update({"us_per_launch": us, "GBs": (w.nbytes + args.M * (K + N) * 2) / us / 1e3,
                    "TFLOPs": 2 * args.M * K * N / us / 1e6})
    print(json.dumps(out))


if __name__ == "__main__":
    main()
