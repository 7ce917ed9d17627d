"""bench.py's reference arm (run by the driver as `bench.py --impl reference`)
prints one JSON line with the contract's keys; it needs no GPU.  The CPU
sampler is also checked at one thread."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_json_line():
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0"],
                       cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["e2e"]["value"] == d["value"] and d["e2e"]["unit"] == d["unit"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert cb["sample"] and cb["cpu_model"] and cb["nproc"] >= 1


def test_cpu_decode_step_chains_like_the_gpu_step():
    """The CPU step (reference arithmetic) runs the 81 projections in order, one
    thread, and its bytes per step are the GPU step's algorithmic bytes."""
    sys.path.insert(0, ROOT)
    import bench
    from aria_b200.efkolos import EFKOLOS
    cs = bench.CpuDecodeStep(threads=1)
    assert len(cs.items) == 4 * EFKOLOS.num_layers + 1
    assert cs.bytes_per_step == sum(K * N // 32 * 18 + 2 * (K + N) for (_, _, K, N, _) in EFKOLOS.all_projections())
    logits = cs.step()
    assert logits.shape == (1, EFKOLOS.vocab_size)
    import numpy as np
    assert np.isfinite(logits).all()
