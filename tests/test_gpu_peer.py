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
