"""Host-side logic of bench.py's N-GPU runs, on CPU with two gloo ranks:
device-timed durations are reduced with MAX over ranks (the job ends with
its slowest replica), clock summaries are gathered from every rank, a
device-status failure on one rank reaches all of them through the same
collective, and the whole-job value counts the units of every replica."""
import os
import socket
import subprocess
import sys
from datetime import timedelta

import pytest

from conftest import ROOT


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch
    import torch.distributed as dist

    import bench

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        # rank r took 2 + r ms for the timed steps and 5 - r ms end to end;
        # only rank 1 saw a failed status word
        times, clocks = bench.reduce_over_ranks([2.0 + rank, 5.0 - rank, float(rank == 1)],
                                                {"sm_mhz": 1900 + rank, "reasons": [f"r{rank}"], "samples": 3},
                                                torch.device("cpu"))
        q.put((rank, times, clocks))
    finally:
        dist.destroy_process_group()


def test_reduce_over_ranks_two_gloo_ranks():
    import torch.multiprocessing as mp

    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, times, clocks = q.get(timeout=120)
        results[rank] = (times, clocks)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank in range(world):
        times, clocks = results[rank]
        assert times == [3.0, 5.0, 1.0]  # max over ranks, same on every rank
        assert [c["sm_mhz"] for c in clocks] == [1900, 1901]


def test_single_process_needs_no_process_group():
    import torch

    import bench

    times, clocks = bench.reduce_over_ranks([1.5, 2.5], {"sm_mhz": 1965}, torch.device("cpu"))
    assert times == [1.5, 2.5] and clocks == [{"sm_mhz": 1965}]


def test_job_rate_counts_every_replica():
    import bench

    # 100 units per step, 10 steps, 4 replicas, slowest rank 2 ms -> 2e6 units/s
    assert bench.job_rate(100, 10, 4, 2.0) == pytest.approx(2e6)
    assert bench.job_rate(100, 10, 1, 2.0) == pytest.approx(5e5)


def test_reference_arm_other_ranks_exit_without_work():
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--gpus", "2",
                        "--steps", "1", "--warmup", "0"], env=env, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0
    assert r.stdout.strip() == ""


def test_expert_major_permutation():
    """hy_mt_rs_b200.moe.expert_major: received rows (by source, then by
    expert) reordered expert-major, and the inverse."""
    import numpy as np
    from hy_mt_rs_b200.moe import expert_major

    counts = np.array([[2, 0, 1], [1, 3, 0]])       # 2 sources, 3 local experts
    # received order: s0:e0 e0 e2 | s1:e0 e1 e1 e1
    perm, inv, off = expert_major(counts)
    assert list(off) == [0, 3, 6, 7]
    assert list(perm) == [0, 1, 3, 4, 5, 6, 2]
    assert list(perm[inv]) == list(range(7))
    empty = expert_major(np.zeros((2, 2), dtype=np.int64))
    assert empty[0].size == 0 and list(empty[2]) == [0, 0, 0]


def test_ep_device_index_math_round_trip():
    """Expert parallelism without host round trips (hy_mt_rs_b200.moe
    ep_send_index / ep_recv_perm), simulated on the CPU for 3 ranks with
    random routing: the fixed-capacity all-to-all moved as blocks, the
    receivers' expert-major order equal to expert_major's (host version),
    and every row's result back at its own grouped position on its sender."""
    import numpy as np
    import torch

    from hy_mt_rs_b200.moe import ep_recv_perm, ep_send_index, expert_major

    W, El, T, used = 3, 4, 5, 2
    E, cap = W * El, T * used
    rng = np.random.default_rng(7)
    counts_src = [rng.multinomial(cap, [1.0 / E] * E) for _ in range(W)]
    offs = [torch.tensor(np.concatenate([[0], np.cumsum(c)]), dtype=torch.int32) for c in counts_src]
    # sender s's grouped row g carries the value 1000 s + g
    sends = []
    for s in range(W):
        idx, valid = ep_send_index(offs[s], W, El, cap)
        assert valid.sum().item() == cap
        for r in range(W):
            n = int(counts_src[s][r * El:(r + 1) * El].sum())
            assert valid[r].tolist() == [True] * n + [False] * (cap - n)
            assert idx[r, :n].tolist() == list(range(int(offs[s][r * El]), int(offs[s][r * El]) + n))
        sends.append((idx, valid, (1000 * s + idx).float()))           # [W, cap] values to each rank
    backs = [torch.zeros(W, cap) for _ in range(W)]
    for r in range(W):
        recv = torch.cat([sends[s][2][r] for s in range(W)])          # block s = what s sent to r
        counts = torch.tensor(np.stack([counts_src[s][r * El:(r + 1) * El] for s in range(W)]))
        perm, valid, off = ep_recv_perm(counts, cap)
        hp, _, hoff = expert_major(counts.numpy())
        base = np.concatenate([[0], np.cumsum(counts.numpy().sum(axis=1))[:-1]])
        src = np.searchsorted(np.cumsum(counts.numpy().sum(axis=1)), hp, side="right")
        assert perm[:len(hp)].tolist() == (src * cap + hp - base[src]).tolist()
        assert off.tolist() == hoff.tolist() and int(valid.sum()) == len(hp)
        y = recv[perm]                                                # "expert results" in expert-major order
        yr = torch.zeros(W * cap + 1)
        yr.index_copy_(0, torch.where(valid, perm, torch.full_like(perm, W * cap)), y)
        for s in range(W):
            backs[s][r] = yr[s * cap:(s + 1) * cap]
    for s in range(W):
        idx, valid, vals = sends[s]
        out = torch.full((cap + 1,), -1.0)
        out.index_copy_(0, torch.where(valid, idx, torch.full_like(idx, cap)).reshape(-1), backs[s].reshape(-1))
        assert out[:cap].tolist() == [1000.0 * s + g for g in range(cap)]


def test_ep_counts_travel_with_the_rows():
    """The expert-parallel send buffer carries each destination's per-expert
    counts in one extra row per block (hy_mt_rs_b200.moe ep_pack), so one
    all-to-all replaces two: simulated on the CPU for 3 ranks, every
    receiver recovers the counts bit for bit, and the packed row indices
    (ep_packed_rows) reach the same token rows as the unpacked layout."""
    import numpy as np
    import torch

    from hy_mt_rs_b200.moe import ep_pack, ep_packed_rows, ep_recv_perm, ep_send_index, ep_unpack_counts

    W, El, T, used, hidden = 3, 4, 5, 2, 8
    E, cap = W * El, T * used
    rng = np.random.default_rng(11)
    counts_src = [rng.multinomial(cap, [1.0 / E] * E) for _ in range(W)]
    xs = [torch.randn(T, hidden, generator=torch.Generator().manual_seed(s)) for s in range(W)]
    sends, plain = [], []
    for s in range(W):
        off = torch.tensor(np.concatenate([[0], np.cumsum(counts_src[s])]), dtype=torch.int32)
        per_expert = off[1:] - off[:-1]
        idx, _ = ep_send_index(off, W, El, cap)
        rows = (idx.reshape(-1) % T).long()       # grouped row -> token row (any map will do here)
        packed = ep_pack(xs[s], rows, per_expert, W, El, cap)
        assert packed.shape == (W * (cap + 1), hidden)
        sends.append(packed.view(W, cap + 1, hidden))
        plain.append(xs[s].index_select(0, rows).view(W, cap, hidden))
    for r in range(W):
        recv = torch.cat([sends[s][r] for s in range(W)])             # block s = what s sent to r
        counts = ep_unpack_counts(recv, W, El, cap)
        want = np.stack([counts_src[s][r * El:(r + 1) * El] for s in range(W)])
        assert counts.tolist() == want.tolist()
        perm, valid, _ = ep_recv_perm(counts, cap)
        unpacked = torch.cat([plain[s][r] for s in range(W)])         # the two-all-to-all layout
        assert torch.equal(recv[ep_packed_rows(perm, cap)][valid], unpacked[perm][valid])


def test_ep_peer_slot_layout():
    """The peer-memory exchange (hy_mt_rs_b200.peer.PeerExchange) leaves
    source s's block at row s * stride of the receiver's region, with only
    its valid rows and its count row written (the rest is whatever an
    earlier exchange left): simulated on the CPU for 3 ranks with a slot
    wider than one block, the counts and the packed row indices still reach
    the right rows."""
    import numpy as np
    import torch

    from hy_mt_rs_b200.moe import ep_pack, ep_packed_rows, ep_recv_perm, ep_send_index, ep_unpack_counts

    W, El, T, used, hidden = 3, 2, 4, 2, 4
    E, cap = W * El, T * used
    stride = cap + 1 + 3
    rng = np.random.default_rng(5)
    counts_src = [rng.multinomial(cap, [1.0 / E] * E) for _ in range(W)]
    regions = [torch.full((W * stride, hidden), float("nan")) for _ in range(W)]
    plain = []
    for s in range(W):
        off = torch.tensor(np.concatenate([[0], np.cumsum(counts_src[s])]), dtype=torch.int32)
        idx, valid = ep_send_index(off, W, El, cap)
        rows = (idx.reshape(-1) % T).long()
        x = torch.randn(T, hidden, generator=torch.Generator().manual_seed(10 + s))
        send = ep_pack(x, rows, off[1:] - off[:-1], W, El, cap).view(W, cap + 1, hidden)
        n = valid.sum(1)
        for q in range(W):   # what the push kernel writes into q's region, slot s
            regions[q][s * stride:s * stride + int(n[q])] = send[q, :int(n[q])]
            regions[q][s * stride + cap] = send[q, cap]
        plain.append(x.index_select(0, rows).view(W, cap, hidden))
    for r in range(W):
        counts = ep_unpack_counts(regions[r], W, El, cap, stride)
        assert counts.tolist() == np.stack([counts_src[s][r * El:(r + 1) * El] for s in range(W)]).tolist()
        perm, valid, _ = ep_recv_perm(counts, cap)
        unpacked = torch.cat([plain[s][r] for s in range(W)])
        got = regions[r][ep_packed_rows(perm, cap, stride)][valid]
        assert torch.equal(got, unpacked[perm][valid])
