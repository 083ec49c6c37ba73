"""GPU check of the peer-memory all-reduce (hyq_peer_allreduce) on two
GPUs: every rank gets the rank-ordered sum of all partials, bit for bit,
on consecutive calls and on calls replayed from a CUDA graph.  Each rank is
a child process on its own GPU; the group is gloo (it only carries the IPC
handles and barriers), so no NCCL or multicast memory is involved.
Skipped on machines with fewer than two GPUs."""
import os
import socket
import sys
from datetime import timedelta

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _partials(step, world, n):
    import torch

    return [torch.randn(n, generator=torch.Generator().manual_seed(1000 * step + q)) for q in range(world)]


def _rank_main(rank, world, port, q):
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    from hy_mt_rs_b200 import quant
    from hy_mt_rs_b200.peer import PeerAllReduce

    n = 4096 + 3  # float4 body plus a scalar tail
    ar = PeerAllReduce(n, device=dev)
    ok = True
    out = torch.empty(n, device=dev)
    # eager, three calls in a row
    for step in range(3):
        parts = _partials(step, world, n)
        ar.partial.copy_(parts[rank].to(dev))
        ar.allreduce(out)
        ref = torch.zeros(n)
        for p in parts:
            ref = ref + p
        ok &= torch.equal(out.cpu(), ref)
    # replayed from a CUDA graph: the epoch lives on the device
    stream = torch.cuda.Stream(dev)
    src = torch.empty(n, device=dev)
    with torch.cuda.stream(stream):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            ar.partial.copy_(src)
            ar.allreduce(out)
        for step in range(3, 6):
            parts = _partials(step, world, n)
            src.copy_(parts[rank].to(dev))
            g.replay()
            stream.synchronize()
            ref = torch.zeros(n)
            for p in parts:
                ref = ref + p
            ok &= torch.equal(out.cpu(), ref)
    ok &= quant.device_status(dev) == 0
    del g
    ar.close()
    q.put((rank, bool(ok)))
    dist.destroy_process_group()


def test_peer_allreduce_two_gpus():
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res == {0: True, 1: True}


def test_peer_wait_runs_out_and_reports(cuda):
    """Failure detection of a bounded device wait, on one GPU with no peer:
    rank 0 of a two-rank all-reduce whose second region is a local buffer
    that no rank ever flags.  The kernel's wait for that rank's ready flag
    must give up after the limit set by hyq_set_peer_timeout_ms (200 ms
    here), raise HYQ_DEV_TIMEOUT_PEER in the status word and return without
    writing `out`; the context stays usable (a product afterwards runs
    clean).  Both regions are this process's own device memory: no IPC
    mapping, no second GPU, no multicast."""
    import ctypes as C
    import time

    import torch
    from hy_mt_rs_b200 import quant, synth
    from hy_mt_rs_b200._native import check, lib

    n = 1024
    regions, handles = [], []
    for _ in range(2):
        r, h = C.c_void_p(), (C.c_uint8 * 64)()
        check(lib.hyq_peer_alloc(4 * n, C.byref(r), h))
        regions.append(r.value)
        handles.append(h)
    arr = (C.c_uint64 * 2)(*regions)
    out = torch.full((n,), float("nan"), device=cuda)
    stream = torch.cuda.current_stream(cuda)
    try:
        check(lib.hyq_set_peer_timeout_ms(200))
        t0 = time.perf_counter()
        check(lib.hyq_peer_allreduce(arr, 0, 2, n, C.c_void_p(out.data_ptr()), C.c_void_p(stream.cuda_stream)))
        status = quant.device_status(cuda)    # synchronizes: the kernel has returned
        waited = time.perf_counter() - t0
        assert status == 16, status           # HYQ_DEV_TIMEOUT_PEER
        assert 0.15 < waited < 5.0, waited
        assert torch.isnan(out).all()         # nothing written
        # the context still works
        w = quant.Weight(synth.random_packed(5, 256, 2048, seed=1, device=cuda), 5, [2048, 256])
        y = w.matmul(torch.randn(2048, device=cuda), 1)
        assert torch.isfinite(y).all() and quant.device_status(cuda) == 0
    finally:
        check(lib.hyq_set_peer_timeout_ms(5000))
        for r in regions:
            check(lib.hyq_peer_free(C.c_void_p(r)))
