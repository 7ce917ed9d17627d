"""The peer-memory reduction of the column-split FFN (aria_p2p_allreduce_add).

On one GPU (the round-end suite): the kernel's arithmetic and its bounded wait,
with the "peer" played by buffers in the same GPU's memory -- a peer flag the
host has already raised (no waiting), or one that nothing ever raises (the wait
must run out within its limit, record ARIA_Q4_DEVERR_PEER_TIMEOUT and leave h
unchanged).  Only one kernel runs at a time; nothing waits on another launch.

On 2-8 GPUs (skipped with fewer): one process per GPU, NCCL for the set-up
and the logits all-gather, the column-split decode with the peer reduction
against the same program with NCCL's all-reduce, and a second step
(graph-free) to check that the per-call epochs stay in step."""
import ctypes
import os

import numpy as np
import pytest
import torch

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")]

PEER_TIMEOUT = 4


def _region(lib, nbytes):
    from aria_b200 import _lib
    p = ctypes.c_void_p()
    _lib.check("aria_p2p_alloc", lib.aria_p2p_alloc(nbytes, ctypes.byref(p)))
    return p.value


def test_single_rank_adds_partial():
    from aria_b200.p2p import PeerReduction
    n = 64 * 256
    red = PeerReduction(n, layers=3)
    rng = np.random.default_rng(0)
    h0 = torch.from_numpy(rng.standard_normal(n).astype(np.float16)).cuda()
    for layer in range(3):
        part = red.part_tensor(layer, (64, 256))
        part.copy_(torch.from_numpy(rng.standard_normal((64, 256)).astype(np.float32)).cuda())
        h = h0.clone()
        red.reduce_into(layer, h)
        torch.cuda.synchronize()
        ref = (h0.float() + part.reshape(-1)).half()
        assert torch.equal(h, ref)
    red.close()


def _two_rank_call(lib, base, n, h, rank, wait_us):
    part = [base + 256, base + 256 + n * 4]
    flags = [base, base + 128]  # rank 0's flag block, the "peer"'s flag block
    state = base + 64
    pa = (ctypes.c_void_p * 2)(*part)
    fa = (ctypes.c_void_p * 2)(*flags)
    return lib.aria_p2p_allreduce_add(pa, fa, ctypes.c_void_p(state), 2, rank, ctypes.c_void_p(h.data_ptr()), n,
                                      wait_us, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def _view(ptr, n, typestr):
    from aria_b200.p2p import _DeviceArray
    return torch.as_tensor(_DeviceArray(ptr, (n,), typestr), device="cuda")


def test_presignalled_peer_sums_in_rank_order():
    from aria_b200 import _lib
    lib = _lib.lib()
    n = 8192
    base = _region(lib, 256 + 2 * n * 4)
    rng = np.random.default_rng(1)
    own, peer = _view(base + 256, n, "<f4"), _view(base + 256 + n * 4, n, "<f4")
    own.copy_(torch.from_numpy(rng.standard_normal(n).astype(np.float32)))
    peer.copy_(torch.from_numpy(rng.standard_normal(n).astype(np.float32)))
    _view(base, 16, "<i4")[1] = 1 << 20  # the peer has published far ahead: no waiting
    h0 = torch.from_numpy(rng.standard_normal(n).astype(np.float16)).cuda()
    for _ in range(2):
        h = h0.clone()
        assert _two_rank_call(lib, base, n, h, 0, 20000) == 0
        torch.cuda.synchronize()
        assert torch.equal(h, (h0.float() + (own + peer)).half())
    assert int(_view(base + 64, 2, "<i4")[0]) == 2  # two calls counted
    assert int(_view(base + 128, 16, "<i4")[0]) == 2  # this rank's epoch published to the "peer"
    assert lib.aria_q4_take_device_error() == 0
    lib.aria_p2p_free(ctypes.c_void_p(base))


def test_peer_that_never_publishes_times_out():
    from aria_b200 import _lib
    lib = _lib.lib()
    assert lib.aria_q4_take_device_error() == 0
    n = 4096
    base = _region(lib, 256 + 2 * n * 4)
    h = torch.ones(n, dtype=torch.float16, device="cuda")
    import time
    t0 = time.time()
    assert _two_rank_call(lib, base, n, h, 0, 20000) == 0  # 20 ms limit
    torch.cuda.synchronize()
    assert time.time() - t0 < 5.0
    assert lib.aria_q4_take_device_error() == PEER_TIMEOUT
    assert bool((h == 1).all())  # left unchanged
    lib.aria_p2p_free(ctypes.c_void_p(base))


def _worker(rank, world, port, q):
    try:
        os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "RANK": str(rank),
                           "WORLD_SIZE": str(world), "NCCL_NVLS_ENABLE": "0"})
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=torch.device("cuda", rank))
        from aria_b200.efkolos import EfkolosConfig
        from aria_b200.scaled import ColumnSplitDecode
        cfg = EfkolosConfig(num_layers=4, d_model=1024, num_heads=8, ffn_dim=4096, vocab_size=2000)
        outs = {}
        for red in ("nccl", "p2p"):
            prog = ColumnSplitDecode(cfg, M=64, world=world, rank=rank, seed=3, reduction=red)
            prog.run()
            first = prog.logits.clone()
            prog.run()  # a second step: epochs and per-layer buffers reused
            torch.cuda.synchronize()
            assert torch.equal(first, prog.logits)
            outs[red] = prog.logits.float().cpu().numpy()
            prog.close()
            del prog
        assert torch.cuda.current_device() == rank
        from aria_b200 import _lib
        err = _lib.lib().aria_q4_take_device_error()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, None if err == 0 else f"device error {err}",
               float(np.abs(outs["p2p"] - outs["nccl"]).max()), float(np.abs(outs["nccl"]).max())))
    except Exception as e:  # reported to the parent
        q.put((rank, repr(e), None, None))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_multi_gpu_peer_reduction_matches_nccl():
    """Every visible GPU (2..8) as one rank."""
    import torch.multiprocessing as mp
    world = min(torch.cuda.device_count(), 8)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=600) for _ in procs]
    for p in procs:
        p.join(timeout=120)
    for rank, err, diff, mag in results:
        assert err is None, (rank, err)
        # f32 partial sums in rank order vs NCCL's order, one f16 rounding of h per layer
        assert diff <= 2e-2 * max(1.0, mag), (rank, diff, mag)
