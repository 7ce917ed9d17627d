"""Multi-rank host logic on CPU (gloo, world_size 2 and 3): batch shards cover
the batch exactly once, column-split projections reassemble to the full
projection, and the Q4_0 blocks of a rank's slice are the full tensor's blocks.
The per-rank arithmetic is the oracle's dequantise-then-matmul (the GPU
kernels are checked against the same oracle in the -m gpu tests)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from aria_b200 import dist as adist


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, layout, K, N, M, q):
    import torch.distributed as dist
    from oracle import q4_oracle_np as npo
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(0)  # same full weight on every rank
        shape = (K, N) if layout == 0 else (N, K)
        w = torch.from_numpy((rng.standard_normal(shape) * 0.02).astype(np.float16))
        x = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float16))
        cs = adist.ColumnSplit(layout, K, N, world, rank)
        n0, n1 = cs.cols
        w_local = cs.slice_weight(w)
        blocks = npo.quantize_q4_0_f16(w_local.numpy().reshape(-1))
        # the slice's blocks are the full tensor's blocks (KN: 32-aligned columns)
        full_blocks = npo.quantize_q4_0_f16(w.numpy().reshape(-1)).reshape(-1, 18)
        if layout == 0:
            idx = (np.arange(K)[:, None] * (N // 32) + np.arange(n0 // 32, n1 // 32)[None, :]).reshape(-1)
        else:
            idx = np.arange(n0 * K // 32, n1 * K // 32)
        ok_blocks = np.array_equal(blocks.reshape(-1, 18), full_blocks[idx])
        y_local = torch.from_numpy(npo.matmul_ref(blocks, layout, K, n1 - n0, x.numpy()).astype(np.float32))
        y = adist.gather_columns(y_local, N, world, cs.align)
        ref = npo.matmul_ref(npo.quantize_q4_0_f16(w.numpy().reshape(-1)), layout, K, N, x.numpy())
        err = float(np.abs(y.numpy() - ref).max())
        # batch shards
        rows = adist.batch_range(M, world, rank)
        allr = [None] * world
        dist.all_gather_object(allr, rows)
        covered = sorted(i for (a, b) in allr for i in range(a, b)) == list(range(M))
        q.put((rank, ok_blocks, err, tuple(y.shape), covered))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,layout,K,N,M", [(2, 0, 64, 160, 5), (3, 0, 96, 96, 4), (2, 1, 64, 75, 3),
                                                (3, 1, 128, 31, 7)])
def test_column_split_gloo(world, layout, K, N, M):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, layout, K, N, M, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = []
    import queue as _queue
    while len(res) < world:
        try:
            res.append(q.get(timeout=2))
        except _queue.Empty:
            dead = [p for p in procs if p.exitcode not in (None, 0)]
            assert not dead, "a rank failed"
            assert any(p.is_alive() for p in procs) or len(res) == world, "ranks exited without a result"
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ok_blocks, err, shape, covered in res:
        assert ok_blocks, f"rank {rank}: slice blocks differ from the full tensor's"
        assert shape == (M, N)
        assert err < 1e-5, f"rank {rank}: reassembled projection off by {err}"
        assert covered


def test_ranges_cover_exactly():
    for N in (31500, 16384, 4096, 100, 31):
        for world in (1, 2, 3, 4, 8):
            for align in (16, 32):
                spans = [adist.col_range(N, world, r, align) for r in range(world)]
                assert spans[0][0] == 0 and spans[-1][1] == N
                for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
                    assert a1 == b0
                    assert a0 % align == 0 or a0 == a1 == N  # trailing ranks may be empty
        for world in (1, 2, 3, 8):
            rs = [adist.batch_range(N, world, r) for r in range(world)]
            assert sum(b - a for a, b in rs) == N and rs[0][0] == 0 and rs[-1][1] == N


def _pair_worker(rank, world, port, d, ff, M, q):
    """ffn_up column slice -> ffn_down K slice -> all-reduce, oracle arithmetic."""
    import torch.distributed as dist
    from oracle import q4_oracle_np as npo
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(1)
        up = torch.from_numpy((rng.standard_normal((d, ff)) * 0.02).astype(np.float16))
        dn = torch.from_numpy((rng.standard_normal((ff, d)) * 0.02).astype(np.float16))
        h = rng.standard_normal((M, d)).astype(np.float16)
        us = adist.ColumnSplit(0, d, ff, world, rank, align_to=128)
        ds = adist.RowSplit(0, ff, d, world, rank, align=128)
        same = us.cols == ds.rows
        k0, k1 = ds.rows
        part = np.zeros((M, d))
        if k1 > k0:
            u = npo.gelu_tanh(npo.matmul_ref(npo.quantize_q4_0_f16(us.slice_weight(up).numpy().reshape(-1)), 0, d,
                                             k1 - k0, h)).astype(np.float16)
            part = npo.matmul_ref(npo.quantize_q4_0_f16(ds.slice_weight(dn).numpy().reshape(-1)), 0, k1 - k0, d, u)
        t = torch.from_numpy(part)
        dist.all_reduce(t)
        u_full = npo.gelu_tanh(npo.matmul_ref(npo.quantize_q4_0_f16(up.numpy().reshape(-1)), 0, d, ff, h))
        ref = npo.matmul_ref(npo.quantize_q4_0_f16(dn.numpy().reshape(-1)), 0, ff, d, u_full.astype(np.float16))
        q.put((rank, same, float(np.abs(t.numpy() - ref).max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,d,ff,M", [(2, 64, 512, 3), (3, 96, 640, 2)])
def test_ffn_pair_split_allreduce_gloo(world, d, ff, M):
    """ffn_up split by columns and ffn_down split along K on the same ranges:
    the all-reduced partial products equal the unsplit pair (the Q4_0 blocks of
    K-slices of a KN tensor are the full tensor's blocks, so only the f32
    summation order differs)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_pair_worker, args=(r, world, port, d, ff, M, q)) for r in range(world)]
    for p in procs:
        p.start()
    import queue as _queue
    res = []
    while len(res) < world:
        try:
            res.append(q.get(timeout=2))
        except _queue.Empty:
            assert not [p for p in procs if p.exitcode not in (None, 0)], "a rank failed"
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, same, err in res:
        assert same, f"rank {rank}: ffn_up columns and ffn_down rows differ"
        assert err < 1e-9, f"rank {rank}: all-reduced pair off by {err}"


def _handles_worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from aria_b200.p2p import exchange_handles
    got = exchange_handles(bytes([rank]) * 64)
    dist.destroy_process_group()
    q.put((rank, got))


def test_ipc_handle_exchange_gloo():
    """aria_b200.p2p.exchange_handles: every rank receives every 64-byte handle in rank order."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + os.getpid() % 200
    procs = [ctx.Process(target=_handles_worker, args=(r, 3, port, q)) for r in range(3)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, got in res:
        assert got == [bytes([r]) * 64 for r in range(3)]
