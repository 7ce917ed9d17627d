#!/usr/bin/env python
"""Benchmark of the B200 Q4_0 projection path (driver contract: one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: one Efkolos decode step at batch 1 -- the
81 Q4_0 projections of a token (20 layers x QKV 896->2688, attn_out 896->896,
ffn_up 896->3584, ffn_down 3584->896, plus the LM head 896->31500) in model
order with the reference layer's data flow (the residual stream feeds QKV and
ffn_up, attn_out and ffn_down add into it, GELU after ffn_up), each projection
consuming the previous one's output; launched through the C ABI, each waiting
on the previous (programmatic dependent launch), captured once in a CUDA graph
per weight replica.  Metric: algorithmic HBM GB/s = (Q4_0 weight bytes + f16
activations in + f16 outputs out) / step time.  The weight set (124 MB) is as
large as B200's L2, so steps rotate over weight replicas totalling > 4x L2;
inputs are therefore never L2-resident between timed steps.

Under torchrun (N > 1) every rank decodes its own sequence on a full weight
replica (batch-sharded weak scaling, no data-path collective); value = bytes
all ranks streamed / max-over-ranks time.

--impl reference times the reference's CPU arithmetic on the same workload:
the whole 81-projection step, chained the same way, each projection a
dequantise + f32 i-p-j matmul (the oracle restatement of
transformer_cuda.rs:549-575 and :3322-3333), on all host cores, rank 0 only.

--case NAME runs a single projection kind a few times (for ncu captures) and,
with --time, times it over weight copies larger than 4x L2.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Q4_0 GEMV HBM GB/s (decode)"
UNIT = "GB/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-cublas", action="store_true", help="skip the cuBLAS fp16 same-box reference point")
    ap.add_argument("--prefill", type=lambda v: [int(t) for t in v.split(",") if t], default=[4096, 8192])
    ap.add_argument("--batched", type=lambda v: [int(t) for t in v.split(",") if t], default=[16, 64, 256])
    ap.add_argument("--scaled", type=int, default=1, help="1: also run BASELINE configs[4] (d_model 4096)")
    ap.add_argument("--scaled-prefill-tokens", type=int, default=4096)
    ap.add_argument("--prefill-forward", type=int, default=1,
                    help="1: also time the whole-prompt forward with causal attention (8x512, 4x2048 tokens)")
    ap.add_argument("--case", default=None,
                    help="single projection kind (qkv, attn_out, ffn_up, ffn_down, lm_head; prefix scaled_ for "
                         "BASELINE configs[4]) or attention / scaled_attention, instead of the benchmark")
    ap.add_argument("--M", type=int, default=1, help="--case: token rows (attention: positions per sequence)")
    ap.add_argument("--seqs", type=int, default=8, help="--case attention: sequences")
    ap.add_argument("--epilogue", default="plain", choices=["plain", "gelu", "residual", "gelu_residual"],
                    help="--case: the projection's epilogue (GELU, residual add with beta = 1)")
    ap.add_argument("--launches", type=int, default=3, help="--case: launches before exiting")
    ap.add_argument("--kernel", default="auto", help="--case: auto, stream, register or tensor")
    ap.add_argument("--time", action="store_true", help="--case: also time the kind over weight copies")
    ap.add_argument("--program", default=None, choices=["decode_step", "decode_kv", "prefill_fwd"],
                    help="run one whole program --launches times (for ncu launch lists): the 81-projection "
                         "step (decode_step, --M token rows), the decode step with KV cache (decode_kv) or the "
                         "whole-prompt forward (prefill_fwd, --seqs x --M tokens)")
    return ap.parse_args()


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi sampling of SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()
        time.sleep(0.25)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.t:
            self.t.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ CPU baseline

class CpuDecodeStep:
    """The reference's CPU arithmetic for one Efkolos decode step at batch 1.

    All 81 projections with the same data flow as the GPU step (residual
    stream h, attn_out on the first d_model QKV columns, GELU after ffn_up,
    residual adds, LM head on the final h); each projection dequantises its
    Q4_0 blocks to f32 and runs the f32 i-p-j matmul of the reference's
    cpu_matmul (the oracle's restatement of transformer_cuda.rs:549-575 and
    :3322-3333), as the reference's CPU step re-reads its weights every step
    (:1059-1166, :1286-1324).  Weights are the oracle packer's blocks of
    seeded N(0, sigma) f16 weights."""

    def __init__(self, threads: int):
        import numpy as np
        from oracle.q4_oracle_np import COracle
        from aria_b200.efkolos import EFKOLOS
        self.np = np
        self.orc = COracle()
        self.threads = threads
        self.cfg = EFKOLOS
        rng = np.random.default_rng(0)
        self.items = []
        for (name, lay, K, N, sg) in EFKOLOS.all_projections():
            w = (rng.standard_normal(K * N, dtype=np.float32) * sg).astype(np.float16)
            self.items.append((self.orc.quantize_q4_0_f16(w), lay, K, N))
        big = max(K * N for (_, _, K, N) in self.items)
        self.ws = np.zeros(big, np.float32)
        self.xs = np.zeros(max(K for (_, _, K, _) in self.items), np.float32)
        self.h0 = rng.standard_normal((1, EFKOLOS.d_model)).astype(np.float16)
        self.bytes_per_step = sum(K * N // 32 * 18 + K * 2 + N * 2 for (_, _, K, N) in self.items)

    def _proj(self, i, x16):
        blocks, lay, K, N = self.items[i]
        y = self.np.zeros((1, N), self.np.float32)
        self.orc.baseline_projection(blocks, lay, K, N, self.np.ascontiguousarray(x16), self.ws, self.xs, y,
                                     self.threads)
        return y

    def step(self):
        from oracle.q4_oracle_np import gelu_tanh
        np = self.np
        d = self.cfg.d_model
        h = self.h0.astype(np.float32)
        for li in range(self.cfg.num_layers):
            qkv = self._proj(4 * li, h.astype(np.float16))
            h = h + self._proj(4 * li + 1, qkv[:, :d].astype(np.float16))
            u = gelu_tanh(self._proj(4 * li + 2, h.astype(np.float16)))
            h = h + self._proj(4 * li + 3, u.astype(np.float16))
        return self._proj(len(self.items) - 1, h.astype(np.float16))

    def rate(self, steps: int) -> tuple[float, float]:
        """(GB/s, seconds) over `steps` whole steps."""
        t0 = time.perf_counter()
        for _ in range(steps):
            self.step()
        el = time.perf_counter() - t0
        return self.bytes_per_step * steps / el / 1e9, el


def cpu_baseline_record(seconds: float = 12.0) -> dict:
    """CPU baseline for the JSON line: whole decode steps on all host threads for
    about `seconds`, and one step on a single thread (the reference's cpu_matmul
    is serial)."""
    threads = os.cpu_count() or 1
    cs = CpuDecodeStep(threads)
    _, one = cs.rate(1)
    n = max(1, int(seconds / max(one, 1e-3)))
    v, el = cs.rate(n)
    cs1 = CpuDecodeStep(1)
    cs1.items, cs1.ws, cs1.xs, cs1.h0 = cs.items, cs.ws, cs.xs, cs.h0
    v1, el1 = cs1.rate(1)
    return {"value": v, "unit": UNIT, "cores": threads, "kind": "port", "seconds": el,
            "sample": f"{n} whole decode steps (81 chained projections at M=1, dequantise + f32 i-p-j matmul, "
                      f"{threads} OpenMP threads)",
            "single_thread": {"value": v1, "unit": UNIT, "cores": 1, "seconds": el1,
                              "sample": "1 whole decode step on one thread"},
            "cpu_model": cpu_model(), "nproc": os.cpu_count()}


def cpu_model() -> str:
    """Host CPU model name (for the CPU-baseline record)."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def run_reference(args, rank: int) -> None:
    """The reference arm: the reference's CPU arithmetic on our workload (whole
    Efkolos decode steps at batch 1), all host threads; each step is one whole
    decode step (tens of ms on a 16-core host)."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    cs = CpuDecodeStep(threads)
    for _ in range(min(args.warmup, 3)):
        cs.step()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        cs.step()
        times.append(time.perf_counter() - t0)
    ms = statistics.median(times) * 1e3
    v = cs.bytes_per_step / (ms * 1e-3) / 1e9
    cs1 = CpuDecodeStep(1)
    cs1.items, cs1.ws, cs1.xs, cs1.h0 = cs.items, cs.ws, cs.xs, cs.h0
    v1, el1 = cs1.rate(1)
    cb = {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
          "sample": f"{args.steps} whole decode steps (81 chained projections at M=1, dequantise + f32 i-p-j "
                    f"matmul, {threads} OpenMP threads), median step",
          "single_thread": {"value": v1, "unit": UNIT, "cores": 1, "seconds": el1,
                            "sample": "1 whole decode step on one thread"},
          "cpu_model": cpu_model(), "nproc": os.cpu_count()}
    rec = {"impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
           "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
           "config": {"workload": "efkolos_decode_b1 (BASELINE configs[1]): 20 layers x (QKV, attn_out, ffn_up, "
                                  "ffn_down) + LM head, M=1, model-order chain", "M": 1,
                      "alg_bytes_per_step": cs.bytes_per_step},
           "cpu_baseline": cb, "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(rec), flush=True)


def case_shape(name: str):
    from aria_b200.efkolos import EFKOLOS, SCALED
    cfg = SCALED if name.startswith("scaled_") else EFKOLOS
    base = name.replace("scaled_", "")
    for (n, lay, K, N, s) in cfg.projections() + [cfg.lm_head()]:
        if n.endswith(base) or n == base:
            return lay, K, N, s
    raise SystemExit(f"unknown case {name}")


def run_program(args) -> None:
    """A whole step, --launches times, on fresh seeded weights (for ncu launch
    lists of the kernels a step runs and their shares)."""
    import torch
    from aria_b200.efkolos import EFKOLOS, DecodeProgram, Q4Stack
    if args.program == "decode_step":
        prog = DecodeProgram(Q4Stack.build(EFKOLOS, seed=1), M=args.M, seed=2)
        run = prog.run
    elif args.program == "prefill_fwd":
        # whole-prompt forward of --seqs sequences x --M tokens
        from aria_b200.decoder import Decoder, DecoderWeights
        dec = Decoder(DecoderWeights(EFKOLOS, max_seq=max(512, args.M), seed=3), M=args.seqs)
        tokens = torch.randint(0, EFKOLOS.vocab_size, (args.seqs, args.M), generator=torch.Generator().manual_seed(5))
        dec.prefill(tokens)
        run = lambda: dec.run_prefill(args.M)  # noqa: E731
    else:
        from aria_b200.decoder import Decoder, DecoderWeights
        dec = Decoder(DecoderWeights(EFKOLOS, max_seq=512, seed=3), M=args.M)
        dec.positions.fill_(255)
        run = dec.run
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("aria_program")
    for _ in range(args.launches):
        run()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    print(json.dumps({"program": args.program, "M": args.M, "seqs": args.seqs, "runs": args.launches}), flush=True)


def run_case(args) -> None:
    """One projection kind, `--launches` times through the C ABI (small enough
    for an ncu capture); with --time, chained over weight copies > 4x L2 in a
    CUDA graph and timed with CUDA events."""
    import torch
    from aria_b200 import q4
    from aria_b200.efkolos import EFKOLOS, SCALED, synth_f16
    if args.case in ("attention", "scaled_attention"):
        # causal prefill attention over the packed QKV output of --seqs
        # sequences x --M positions (Efkolos: 14 heads x 64; scaled: 32 x 128)
        from aria_b200.attention import attention_prefill
        cfg = SCALED if args.case.startswith("scaled_") else EFKOLOS
        B, T, d = args.seqs, args.M, cfg.d_model
        qkv = synth_f16((B * T, 3 * d), 1.0, 3)
        att = torch.empty(B * T, d, dtype=torch.float16, device="cuda")
        for _ in range(args.launches):
            attention_prefill(qkv, B, T, cfg.num_heads, out=att)
        torch.cuda.synchronize()
        out = {"case": args.case, "seqs": B, "T": T, "d": d, "heads": cfg.num_heads}
        if args.time:
            s = torch.cuda.Stream()
            with torch.cuda.stream(s):
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(s)
                for _ in range(20):
                    attention_prefill(qkv, B, T, cfg.num_heads, out=att)
                e1.record(s)
                torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1000 / 20
            fl = 4 * (d // cfg.num_heads) * cfg.num_heads * B * T * (T + 1) // 2
            out.update({"us_per_launch": us, "TFLOPs": fl / us / 1e6})
        print(json.dumps(out), flush=True)
        return
    lay, K, N, sigma = case_shape(args.case)
    shape = (K, N) if lay == q4.LAYOUT_KN else (N, K)
    w = q4.Q4Weight.from_f16(synth_f16(shape, sigma, 1), lay)
    x = synth_f16((args.M, K), 1.0, 2)
    y = torch.empty(args.M, N, dtype=torch.float16, device="cuda")
    act = "gelu" if args.epilogue in ("gelu", "gelu_residual") else None
    beta = 1.0 if args.epilogue in ("residual", "gelu_residual") else 0.0
    for _ in range(args.launches):
        q4.matmul(x, w, y, kernel=args.kernel, activation=act, beta=beta)
    torch.cuda.synchronize()
    out = {"case": args.case, "K": K, "N": N, "M": args.M, "kernel": kernel_name(w, args.M, flags_for(args.kernel)),
           "epilogue": args.epilogue}
    if args.time:
        l2 = torch.cuda.get_device_properties(0).L2_cache_size
        ncopy = max(4, -(-4 * l2 // w.nbytes))
        pool = [q4.Q4Weight(w.buf.clone(), lay, K, N) for _ in range(ncopy)]
        n = max(32, min(256, ncopy))
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            q4.matmul(x, pool[0], y, kernel=args.kernel, const_weights=True)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                for j in range(n):
                    q4.matmul(x, pool[j % ncopy], y, kernel=args.kernel, const_weights=True)
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
    print(json.dumps(out), flush=True)


# ------------------------------------------------------------------ GPU arm

def scaled_section(args, rank, world, local_rank, stream, timed, peaks):
    """decode batch 64 with column-split FFN / LM head and NCCL
    all-gathers, and batch-sharded prefill (4096 tokens per rank per step)."""
    import torch
    from aria_b200.efkolos import SCALED, DecodeProgram, Q4Stack
    from aria_b200.scaled import ColumnSplitDecode
    out = {"workload": "BASELINE configs[4]: 32 layers, d_model 4096, FFN 16384, vocab 31500"}
    for red in (("p2p", "nccl") if world > 1 else ("p2p",)):
        prog = ColumnSplitDecode(SCALED, M=64, world=world, rank=rank, reduction=red)
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            prog.run()
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                prog.run()
        steps = max(5, args.steps // 10)
        ms = timed(lambda i: g.replay(), steps, 3, f"aria_scaled_decode_{red}") / steps
        wb = prog.weight_bytes()
        key = "decode_b64_colsplit" if red == "p2p" else "decode_b64_colsplit_nccl"
        out[key] = {
            "ms_per_step": ms, "tokens_per_s": 64 / (ms * 1e-3),
            "weight_GBs_per_rank": wb / (ms * 1e-3) / 1e9, "weight_GBs_total": wb * world / (ms * 1e-3) / 1e9,
            "collective_bytes_per_rank": prog.collective_bytes(), "collectives_per_step": prog.collectives_per_step,
            "split": "ffn_up column-split and ffn_down split along K, LM head column-split + NCCL all-gather; "
                     "QKV, attn_out replicated",
            "reduction": ("one kernel per layer reading the peers' f32 partials over NVLink and adding them into "
                          "the residual stream" if red == "p2p" else "NCCL all-reduce + residual add per layer")
            if world > 1 else "none (one GPU)"}
        del g
        prog.close()
        del prog
        torch.cuda.empty_cache()
    stack = Q4Stack.build(SCALED, seed=rank * 1000 + 77)
    M = args.scaled_prefill_tokens
    pprog = DecodeProgram(stack, M=M, seed=rank + 31)
    with torch.cuda.stream(stream):
        pprog.run()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            pprog.run()
    pms = timed(lambda i: g.replay(), 3, 2, "aria_scaled_prefill") / 3
    tf = M * SCALED.flops_per_token() * world / (pms * 1e-3) / 1e12
    out["prefill_batch_sharded"] = {
        "tokens_per_rank_per_step": M, "ms_per_step": pms, "tokens_per_s": M * world / (pms * 1e-3),
        "TFLOPs": tf, "frac_of_measured_bf16_peak": tf / world / float(peaks.get("bf16_tflops", 1590.0)),
        "job": "256 x 512 tokens split by batch; each step is a bounded sample of M tokens per rank"}
    del g, pprog, stack
    torch.cuda.empty_cache()
    return out


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch of each
# decode-step projection kind as its kernel runs in the step, from one ncu
# capture of `bench.py --case <kind> --M 1` (cold launch)
NCU_TRAFFIC = {"attn_qkv": 1376256, "attn_out": 472832, "ffn_up": 1828096, "ffn_down": 1851904}


def flags_for(kernel: str) -> int:
    from aria_b200 import _lib
    return {"auto": 0, "stream": _lib.FLAG_KERNEL_STREAM, "register": _lib.FLAG_KERNEL_REGISTER,
            "tensor": _lib.FLAG_KERNEL_TENSOR}[kernel]


def decode_kv_section(rank, world, stream, timed, steps: int) -> dict:
    """The whole decode step with KV cache on the GPU (aria_b200.decoder: the
    reference's cached `step`, src/transformer_cuda.rs:1286-1324, with LayerNorm,
    attention over the cache and the Q4_0 projections), Efkolos config, one new
    token per sequence at position 255 (256 positions attended), M = 1 and 16
    sequences.  Caches hold random f16 keys and values."""
    import torch
    from aria_b200.decoder import Decoder, DecoderWeights
    from aria_b200.efkolos import EFKOLOS
    w = DecoderWeights(EFKOLOS, max_seq=512, seed=rank + 3)
    out = {"workload": "Efkolos decode step with KV cache (LayerNorm, QKV, attention over 256 cached positions, "
                       "attn_out, LayerNorm, ffn_up+GELU, ffn_down, final LayerNorm, LM head)",
           "q4_weight_bytes": w.q4_bytes}
    for M in (1, 16):
        dec = Decoder(w, M=M)
        gen = torch.Generator(device="cuda")
        gen.manual_seed(rank + M)
        for kc, vc in zip(dec.k_cache, dec.v_cache):
            kc.copy_(torch.randn(kc.shape, generator=gen, device="cuda", dtype=torch.float16))
            vc.copy_(torch.randn(vc.shape, generator=gen, device="cuda", dtype=torch.float16))
        dec.tokens.copy_(torch.arange(M, dtype=torch.int32) * 997 % EFKOLOS.vocab_size)
        dec.positions.fill_(255)
        with torch.cuda.stream(stream):
            dec.run()
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                dec.run()
        n = max(10, steps // 4)
        ms = timed(lambda i: g.replay(), n, 3, f"aria_decode_kv_M{M}") / n
        out[f"M{M}"] = {"ms_per_step": ms, "tokens_per_s": M * world / (ms * 1e-3), "context_positions": 256,
                        "launches_per_step": dec.launches,
                        "q4_weight_GBs": w.q4_bytes * world / (ms * 1e-3) / 1e9}
        del g, dec
    del w
    torch.cuda.empty_cache()
    return out


def prefill_forward_section(rank, world, stream, timed, bf16_peak: float) -> dict:
    """The whole-prompt forward on the GPU (aria_b200.decoder.Decoder.prefill:
    the reference's forward_gpu, src/transformer_cuda.rs:1518-1873) on the
    Efkolos config at BASELINE configs[3]'s shapes, 8 x 512 and 4 x 2048
    tokens: embedding, 20 x (LayerNorm, QKV, causal attention on the tensor
    cores, attn_out, LayerNorm, ffn_up + GELU, ffn_down, KV-cache fill), final
    LayerNorm, LM head over every token.  Also the attention kernel alone
    (aria_attention_prefill on the step's QKV output), TFLOP/s over the causal
    (unmasked) query-key pairs, 4 dh flops each."""
    import torch
    from aria_b200.attention import attention_prefill
    from aria_b200.decoder import Decoder, DecoderWeights
    from aria_b200.efkolos import EFKOLOS
    cfg = EFKOLOS
    w = DecoderWeights(cfg, max_seq=2048, seed=rank + 5)
    out = {"workload": "Efkolos whole-prompt forward (BASELINE configs[3] token counts) with causal attention",
           "q4_weight_bytes": w.q4_bytes}
    dh = cfg.d_model // cfg.num_heads
    for B, T in ((8, 512), (4, 2048)):
        dec = Decoder(w, M=B)
        gen = torch.Generator()
        gen.manual_seed(rank * 7 + T)
        tokens = torch.randint(0, cfg.vocab_size, (B, T), generator=gen)
        dec.prefill(tokens)  # fills the token buffer, warms the path
        with torch.cuda.stream(stream):
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                dec.run_prefill(T)
        ms = timed(lambda i: g.replay(), 3, 3, f"aria_prefill_forward_{B}x{T}") / 3
        del g
        n_tok = B * T
        attn_flops = 4 * dh * cfg.num_heads * B * T * (T + 1) // 2
        qkv = dec._pbuf["qkv"]
        att = dec._pbuf["att"]
        with torch.cuda.stream(stream):
            attention_prefill(qkv, B, T, cfg.num_heads, out=att)
            torch.cuda.synchronize()
            ga = torch.cuda.CUDAGraph()
            with torch.cuda.graph(ga, stream=stream):
                for _ in range(cfg.num_layers):
                    attention_prefill(qkv, B, T, cfg.num_heads, out=att)
        ams = timed(lambda i: ga.replay(), 3, 2, f"aria_attention_prefill_{B}x{T}") / (3 * cfg.num_layers)
        del ga
        total_flops = n_tok * cfg.flops_per_token() + cfg.num_layers * attn_flops
        out[f"{B}x{T}"] = {"ms_per_step": ms, "tokens_per_s": n_tok * world / (ms * 1e-3),
                           "TFLOPs": total_flops * world / (ms * 1e-3) / 1e12,
                           "launches_per_step": dec.prefill_launches(),
                           "attention_us_per_layer": ams * 1e3,
                           "attention_TFLOPs": attn_flops / (ams * 1e-3) / 1e12,
                           "attention_frac_of_measured_bf16_peak": attn_flops / (ams * 1e-3) / 1e12 / bf16_peak,
                           "attention_share_of_step": cfg.num_layers * ams / ms}
        del dec
        torch.cuda.empty_cache()
    del w
    torch.cuda.empty_cache()
    return out


def kernel_name(w, M: int, flags: int = 0, workspace_bytes: int = 0) -> str:
    """The kernel the library routes this projection to (aria_q4_0_kernel_choice)."""
    from aria_b200._lib import lib
    k = lib().aria_q4_0_kernel_choice(w.layout, w.K, w.N, M, workspace_bytes, flags)
    return {1: "gemv_stream_kernel", 2: "decode_mma_kernel", 3: "gemm_tc_kernel"}.get(k, f"status {-k}")


def gemv_config4_b1(stream, timed, l2: int, hbm_peak: float) -> dict:
    """Each config-4 projection kind alone at M=1, launched as a chain with the
    const-weights flag over weight copies totalling > 4x L2."""
    import torch
    from aria_b200.efkolos import SCALED, synth_f16
    from aria_b200.q4 import Q4Weight, matmul
    out = {"workload": "BASELINE configs[4] projections, one token, each kind chained over copies > 4x L2"}
    for (name, lay, K, N, sigma) in SCALED.projections()[:4] + [SCALED.lm_head()]:
        kind = name.split(".")[-1]
        shape = (K, N) if lay == 0 else (N, K)
        w0 = Q4Weight.from_f16(synth_f16(shape, sigma, 3), lay)
        ncopy = max(4, -(-4 * l2 // w0.nbytes))
        pool = [w0] + [Q4Weight(w0.buf.clone(), lay, K, N) for _ in range(ncopy - 1)]
        x = synth_f16((1, K), 1.0, 4)
        y = torch.empty(1, N, dtype=torch.float16, device=x.device)
        n = max(32, ncopy)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            matmul(x, pool[0], y, const_weights=True)
            torch.cuda.synchronize()
            with torch.cuda.graph(g, stream=stream):
                for j in range(n):
                    matmul(x, pool[j % ncopy], y, const_weights=True)
        us = timed(lambda i: g.replay(), 5, 3, f"aria_gemv4_{kind}") * 1e3 / (5 * n)
        abytes = w0.nbytes + K * 2 + N * 2
        out[kind] = {"K": K, "N": N, "kernel": kernel_name(w0, 1), "us_per_launch": round(us, 3),
                     "GBs": abytes / (us * 1e-6) / 1e9, "frac_of_measured_hbm": abytes / (us * 1e-6) / 1e9 / hbm_peak}
        del g, pool, w0
        torch.cuda.empty_cache()
    return out


def cublas_fp16_section(stream, timed, l2: int, q4_decode_ms: float, q4_prefill_ms: dict) -> dict:
    """The reference's own GPU op on the same box and shapes, as a reference
    point: cuBLAS fp16 GEMM on f16 weights (the reference's gemm(),
    lold3344/ARIA src/transformer_cuda.rs:615-640, reached here through
    torch.matmul / addmm), with no Q4_0 kernel involved.  Efkolos decode step
    at M = 1 (the 81 projections with the step's data flow -- residual adds and
    GELU -- in a CUDA graph, weight replicas > 4x L2 rotated), the config-4 LM
    head at M = 1 (copies > 4x L2), and the Efkolos prefill step at M = 4096."""
    import torch
    from aria_b200.efkolos import EFKOLOS, SCALED
    gen = torch.Generator(device="cuda")
    gen.manual_seed(7)

    def f16(shape, sigma):
        return torch.randn(shape, generator=gen, device="cuda", dtype=torch.float16) * sigma

    projs = EFKOLOS.all_projections()
    f16_bytes = sum(K * N * 2 for (_, _, K, N, _) in projs)
    reps = max(2, -(-4 * l2 // f16_bytes))
    # weights as the reference holds them: KN w[k][n] (x @ w), NK embed[n][k] (x @ embed^T)
    replicas = [[f16((K, N) if lay == 0 else (N, K), sg) for (_, lay, K, N, sg) in projs] for _ in range(reps)]
    out = {"op": "torch.matmul / addmm (beta = 1 residual) -> cuBLAS fp16 GEMM on f16 weights (the reference's "
                 "gemm()), torch tanh GELU; the Q4_0 step's data flow"}

    def chain(ws, M):
        """The same data flow as the Q4_0 step (DecodeProgram): h feeds QKV,
        attn_out adds into h (cuBLAS with beta = 1), GELU after ffn_up (torch's
        tanh GELU, a separate kernel as the reference's gelu_fwd), ffn_down
        adds into h, the LM head reads the final h."""
        d = EFKOLOS.d_model
        h0 = f16((M, d), 1.0)
        h = torch.empty_like(h0)
        qkv = torch.empty(M, 3 * d, device="cuda", dtype=torch.float16)
        u = torch.empty(M, EFKOLOS.ffn_dim, device="cuda", dtype=torch.float16)
        logits = torch.empty(M, EFKOLOS.vocab_size, device="cuda", dtype=torch.float16)

        def run():
            h.copy_(h0)
            for li in range(EFKOLOS.num_layers):
                w_qkv, w_out, w_up, w_down = ws[4 * li:4 * li + 4]
                torch.matmul(h, w_qkv, out=qkv)
                h.addmm_(qkv[:, :d], w_out)
                torch.matmul(h, w_up, out=u)
                u.copy_(torch.nn.functional.gelu(u, approximate="tanh"))
                h.addmm_(u, w_down)
            torch.matmul(h, ws[-1].t(), out=logits)
        return run

    graphs = []
    with torch.cuda.stream(stream):
        for ws in replicas:
            run = chain(ws, 1)
            run()
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                run()
            graphs.append(g)
    ms = timed(lambda i: graphs[i % reps].replay(), 50, 5, "cublas_decode_step") / 50
    out["decode_b1"] = {"ms_per_step": ms, "weight_bytes_f16": f16_bytes,
                        "GBs": (f16_bytes + 2 * sum(K + N for (_, _, K, N, _) in projs)) / (ms * 1e-3) / 1e9,
                        "q4_step_speedup": ms / q4_decode_ms}
    del graphs
    # config-4 LM head at one token
    (_, _, K, N, sg) = SCALED.lm_head()
    ncopy = max(2, -(-4 * l2 // (K * N * 2)))
    embeds = [f16((N, K), sg) for _ in range(ncopy)]
    x = f16((1, K), 1.0)
    y = torch.empty(1, N, device="cuda", dtype=torch.float16)
    n = 16
    with torch.cuda.stream(stream):
        torch.matmul(x, embeds[0].t(), out=y)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for j in range(n):
                torch.matmul(x, embeds[j % ncopy].t(), out=y)
    us = timed(lambda i: g.replay(), 10, 3, "cublas_lm_head_config4") * 1e3 / (10 * n)
    out["lm_head_config4_b1"] = {"us_per_launch": us, "GBs": (K * N * 2 + 2 * (K + N)) / (us * 1e-6) / 1e9}
    del g, embeds
    # prefill step
    for M, q4_ms in q4_prefill_ms.items():
        with torch.cuda.stream(stream):
            run = chain(replicas[0], M)
            run()
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                run()
        pms = timed(lambda i: g.replay(), 5, 2, f"cublas_prefill_M{M}") / 5
        out[f"prefill_M{M}"] = {"ms_per_step": pms, "TFLOPs": M * EFKOLOS.flops_per_token() / (pms * 1e-3) / 1e12,
                                "q4_step_speedup": pms / q4_ms}
        del g
    del replicas
    torch.cuda.empty_cache()
    return out


def run_ours(args, rank: int, world: int, local_rank: int) -> None:
    import torch
    import torch.distributed as dist
    from aria_b200.efkolos import EFKOLOS, DecodeProgram, Q4Stack, synth_f16

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    props = torch.cuda.get_device_properties(dev)
    l2 = getattr(props, "L2_cache_size", 126 * 2**20) or 126 * 2**20
    cfg = EFKOLOS
    stack0 = Q4Stack.build(cfg, seed=rank * 1000)
    reps = max(2, -(-4 * l2 // stack0.nbytes) + 0)
    stacks = [stack0] + [Q4Stack.build(cfg, seed=rank * 1000 + r) for r in range(1, reps)]
    prog = DecodeProgram(stack0, M=1, seed=rank + 1)
    torch.cuda.synchronize()

    stream = torch.cuda.Stream(dev)
    graphs = []
    with torch.cuda.stream(stream):
        for st in stacks:  # warm the path once outside capture
            prog.run(st)
        torch.cuda.synchronize()
        for st in stacks:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                prog.run(st)
            graphs.append(g)
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    def timed(fn, steps, warmup, tag="aria_timed"):
        with torch.cuda.stream(stream):
            for i in range(warmup):
                fn(i)
            torch.cuda.synchronize()
            barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.nvtx.range_push(tag)  # lets an ncu launch list select exactly the timed work
            e0.record(stream)
            for i in range(steps):
                fn(i)
            e1.record(stream)
            torch.cuda.nvtx.range_pop()
            torch.cuda.synchronize()
            barrier()
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except OSError:
        pass
    sampler = ClockSampler(local_rank)
    sampler.start()
    ms = timed(lambda i: graphs[i % reps].replay(), args.steps, args.warmup, "aria_decode_step")
    ms_step = ms / args.steps
    bytes_step = prog.algorithmic_bytes()
    value = bytes_step * world / (ms_step * 1e-3) / 1e9

    # ---- dominant kernel: time each projection kind alone, chained like the step,
    # rotating over copies of its weight that total > 4x L2 so no launch hits L2
    from aria_b200.q4 import Q4Weight, matmul
    kinds = {}
    for idx, (name, w) in enumerate(stack0.weights):
        kinds.setdefault(name.split(".")[-1], []).append(idx)
    per_kind = {}
    for kind, idxs in kinds.items():
        w0 = stack0.weights[idxs[0]][1]
        ncopy = max(4, -(-4 * l2 // w0.nbytes))
        pool = [Q4Weight(w0.buf.clone(), w0.layout, w0.K, w0.N) for _ in range(ncopy)]
        x_ = synth_f16((1, w0.K), 1.0, 17 + idxs[0])
        y_ = torch.empty(1, w0.N, dtype=torch.float16, device=dev)
        n_launch = max(64, min(512, ncopy))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            matmul(x_, pool[0], y_, const_weights=True)
            torch.cuda.synchronize()
            with torch.cuda.graph(g, stream=stream):
                for j in range(n_launch):  # launched as in the step (model weights: const-weights flag)
                    matmul(x_, pool[j % ncopy], y_, const_weights=True)
        kms = timed(lambda i: g.replay(), 3, 2, f"aria_kind_{kind}") / (3 * n_launch)
        abytes = w0.nbytes + w0.K * 2 + w0.N * 2
        per_kind[kind] = {"us_per_launch": round(kms * 1e3, 3), "launches_per_step": len(idxs),
                          "share_est": kms * len(idxs), "alg_bytes": abytes,
                          "gbs": abytes / (kms * 1e-3) / 1e9}
        del g, pool
        torch.cuda.empty_cache()
    for k in per_kind:
        w_k = stack0.weights[kinds[k][0]][1]
        per_kind[k]["kernel"] = kernel_name(w_k, 1)
    # the dominant kernel: the one with the largest share of the step (summed
    # over the kinds it runs); achieved = its algorithmic bytes per launch over
    # its mean launch time, traffic = its ncu DRAM bytes per launch (mean)
    by_kernel = {}
    for k, r in per_kind.items():
        by_kernel.setdefault(r["kernel"], []).append(k)
    dom_kernel = max(by_kernel, key=lambda kk: sum(per_kind[k]["share_est"] for k in by_kernel[kk]))
    dk = by_kernel[dom_kernel]
    n_l = sum(per_kind[k]["launches_per_step"] for k in dk)
    b_l = sum(per_kind[k]["launches_per_step"] * per_kind[k]["alg_bytes"] for k in dk) / n_l
    t_l = sum(per_kind[k]["launches_per_step"] * per_kind[k]["us_per_launch"] for k in dk) / n_l
    traffic = (sum(per_kind[k]["launches_per_step"] * NCU_TRAFFIC[k] for k in dk) / n_l
               if all(k in NCU_TRAFFIC for k in dk) else None)
    hbm_peak = float(peaks.get("hbm_gbs", 6650.0))
    achieved = b_l / (t_l * 1e-6) / 1e9
    roof = {"bound": "hbm", "kernel": f"{dom_kernel} ({', '.join(dk)})", "achieved": achieved,
            "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak,
            "traffic": traffic, "alg_bytes_per_launch": b_l, "us_per_launch": t_l,
            "traffic_source": "ncu dram bytes per launch of each kind (cold), mean over the kernel's launches",
            "peak_source": "MEASURED_PEAKS.json hbm_gbs" if peaks else "fallback 6650",
            "share_of_step": sum(per_kind[k]["share_est"] for k in dk) / ms_step,
            "per_kind": per_kind}

    # ---- the streaming GEMV on BASELINE configs[4] weights (d_model 4096) at one
    # token: bandwidth-bound projections large enough to show the kernel's
    # streaming rate (the Efkolos layers are latency-bound)
    gemv_large = gemv_config4_b1(stream, timed, l2, hbm_peak)

    # ---- end to end through the public API with host buffers
    x_host = torch.empty_like(prog.h0, device="cpu").pin_memory()
    x_host.copy_(prog.h0)
    out_host = torch.empty_like(prog.logits, device="cpu").pin_memory()

    def e2e_step(i):
        prog.h0.copy_(x_host, non_blocking=True)
        graphs[i % reps].replay()
        out_host.copy_(prog.logits, non_blocking=True)

    e2e_ms = timed(e2e_step, args.steps, args.warmup, "aria_e2e") / args.steps
    e2e_val = bytes_step * world / (e2e_ms * 1e-3) / 1e9
    del x_host, out_host

    # ---- batched decode and prefill: same weights, larger M.
    # Each projection reads its own activation buffer, so a prefill step's inputs
    # (>= 1 GB at M=4096) are never L2-resident; batched decode rotates replicas.
    flops_token = cfg.flops_per_token()
    bf16_peak = float(peaks.get("bf16_tflops", 1590.0))
    bf16_sus = float(peaks.get("bf16_tflops_sustained", 1420.0))
    batched = {}
    for M in args.batched:
        bprog = DecodeProgram(stack0, M=M, seed=rank + 11)
        bgraphs = []
        with torch.cuda.stream(stream):
            for st in stacks:
                bprog.run(st)
            torch.cuda.synchronize()
            for st in stacks:
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    bprog.run(st)
                bgraphs.append(g)
        bsteps = max(5, args.steps // 4)
        bms = timed(lambda i: bgraphs[i % reps].replay(), bsteps, max(3, args.warmup // 4), f"aria_batched_M{M}") / bsteps
        batched[f"M{M}"] = {"ms_per_step": bms, "GBs": bprog.algorithmic_bytes() * world / (bms * 1e-3) / 1e9,
                            "TFLOPs": M * flops_token * world / (bms * 1e-3) / 1e12,
                            "tokens_per_s": M * world / (bms * 1e-3)}
        del bgraphs, bprog
        torch.cuda.empty_cache()
    prefill = {}
    for M in args.prefill:
        pprog = DecodeProgram(stack0, M=M, seed=rank + 21)
        with torch.cuda.stream(stream):
            pprog.run()
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                pprog.run()
        psteps = max(3, args.steps // 20)
        pms = timed(lambda i: g.replay(), psteps, 3, f"aria_prefill_M{M}") / psteps
        tf = M * flops_token * world / (pms * 1e-3) / 1e12
        prefill[f"M{M}"] = {"ms_per_step": pms, "tokens_per_s": M * world / (pms * 1e-3), "TFLOPs": tf,
                            "frac_of_measured_bf16_peak": tf / world / bf16_peak,
                            "frac_of_measured_sustained_peak": tf / world / bf16_sus}
        del g, pprog
        torch.cuda.empty_cache()
    decode_kv = decode_kv_section(rank, world, stream, timed, args.steps)
    prefill_fwd = prefill_forward_section(rank, world, stream, timed, bf16_peak) if args.prefill_forward else None
    cublas = None
    if rank == 0 and world == 1 and not args.no_cublas:
        cublas = cublas_fp16_section(stream, timed, l2, ms_step,
                                     {4096: prefill["M4096"]["ms_per_step"]} if "M4096" in prefill else {})
    scaled = None
    if args.scaled:
        scaled = scaled_section(args, rank, world, local_rank, stream, timed, peaks)
    clocks = sampler.stop()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_record(12.0)

    rec = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
           "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
           "vs_baseline": None, "dtype": "q4_0 weights, f16 activations, f32 accumulate", "data": "synthetic",
           "config": {"workload": "efkolos_decode_b1 (BASELINE configs[1]): 20 layers x (QKV, attn_out, ffn_up, "
                                  "ffn_down) + LM head, M=1, model-order chain",
                      "M": 1, "weight_bytes": stack0.nbytes, "alg_bytes_per_step": bytes_step,
                      "l2_policy": f"rotate {reps} weight replicas ({reps * stack0.nbytes / 2**20:.0f} MiB > 4x L2)",
                      "parallelism": f"batch-sharded replicas x{world}"},
           "roofline": roof, "cpu_baseline": cpu, "clocks": clocks,
           "batched_decode": {"workload": "BASELINE configs[2]: same 81 projections, M tokens per step",
                              **batched},
           "prefill": {"workload": "BASELINE configs[3]: 81 projections of the 20 layers + LM head over M "
                                   "tokens (8x512 = 4096, 4x2048 = 8192), tcgen05 kernel",
                       "flops_per_token": flops_token, "peak_tflops_measured": bf16_peak,
                       "peak_tflops_sustained": bf16_sus, **prefill},
           "decode_step_kv": decode_kv,
           "prefill_forward": prefill_fwd,
           "scaled": scaled,
           "gemv_config4_b1": gemv_large,
           "cublas_fp16_same_box": cublas,
           "e2e": {"value": e2e_val, "unit": UNIT, "h2d_bytes_per_step": prog.input_bytes(),
                   "d2h_bytes_per_step": prog.output_bytes(), "ms_per_step": e2e_ms},
           "gpu_launches": prog.launches * args.steps}
    if rank == 0:
        print(json.dumps(rec), flush=True)
    for g in graphs:
        del g


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.case:
        run_case(args)
        return
    if args.program:
        run_program(args)
        return
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
