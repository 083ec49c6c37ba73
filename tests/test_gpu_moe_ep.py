"""GPU check of expert parallelism for the MoE layer (MoeLayer with ep=...)
on two GPUs (and four where the box has them): each rank holds its share of
the experts and its own tokens; token
rows travel to the expert's rank and back by NCCL all-to-all or, with a
PeerExchange, by pushes into the other rank's peer-memory region.  Every
expert output row is computed as on one GPU, so each rank's layer output
equals the one-GPU layer on the same tokens bit for bit.  Each rank is a
child process on its own GPU; NVLS is off.  Skipped with fewer than two
GPUs."""
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


def _rank_main(rank, world, port, q, peer=False):
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    from hy_mt_rs_b200 import quant
    from hy_mt_rs_b200.moe import MoeConfig, MoeLayer, random_moe_weights
    from hy_mt_rs_b200.peer import PeerExchange

    ok = True
    xchgs = []
    for T, cfg in ((37, MoeConfig(hidden=512, experts=8, used=2, mid=256, shared_mid=256)),
                   (64, MoeConfig(hidden=2048, experts=16, used=4, mid=1024, shared_mid=1024))):
        w = random_moe_weights(cfg, dev, seed=11)
        full = MoeLayer(cfg, w)
        # the peer slots are sized for more tokens than this call has
        xchg = PeerExchange((2 * T * cfg.used + 1) * cfg.hidden, device=dev) if peer else None
        if xchg is not None:
            xchgs.append(xchg)
        ep = MoeLayer(cfg, w, ep=(rank, world, None), exchange=xchg)
        x = torch.randn(T, cfg.hidden, generator=torch.Generator().manual_seed(100 + rank)).to(dev)
        ref = full.forward(x, T).clone()
        for _ in range(2):
            got = ep.forward(x, T)
            ok &= torch.equal(got, ref)
        torch.cuda.synchronize(dev)
    if peer:
        # the plain exchange: block q of rank r is r * 1000 + q * 10 + row, the
        # first (q + 2) rows of it sent, and the block's last row with last_row
        H, rows = 64, 6
        X = PeerExchange(rows * H, device=dev)
        xchgs.append(X)
        send = torch.stack([torch.full((rows, H), float(rank * 1000 + q * 10)) + torch.arange(rows)[:, None]
                            for q in range(world)]).reshape(world * rows, H).to(dev)
        valid = torch.tensor([q + 2 for q in range(world)], dtype=torch.int32, device=dev)
        for _ in range(2):
            X.exchange(send, rows, valid, last_row=True)
            recv = X.recv(rows, H).view(world, rows, H).cpu()
            for s in range(world):
                for i in list(range(rank + 2)) + [rows - 1]:
                    ok &= bool((recv[s, i] == float(s * 1000 + rank * 10 + i)).all())
    ok &= quant.device_status(dev) == 0
    for xchg in xchgs:
        xchg.close()
    q.put((rank, bool(ok)))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,peer", [(2, False), (2, True), (4, True)])
def test_moe_expert_parallel_two_gpus(world, peer):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q, peer)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res == {r: True for r in range(world)}
