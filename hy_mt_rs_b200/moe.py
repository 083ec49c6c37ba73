"""Mixture-of-experts feed-forward layer (Moe::forward, hy-mt-rs
src/model.rs:688-767) on the device, through libhyq.

The reference computes router logits, routes each token on the host, then
loops over experts (one small matmul per expert) and accumulates
`output[token] += weight * value`.  Here the routing, the per-expert token
lists, the expert products (tensor cores, all experts in one launch per
projection) and the combine are six launches over all tokens, with the
expert token lists kept in device memory: no host round trip per layer.

Weights are packed GGUF tensors: the router F32 [hidden, experts] (the
reference requires F32, model.rs:223-227), the expert gate/up [hidden, mid,
experts] and down [mid, hidden, experts] tensors (Weight::expert slices,
quant.rs:144-154) and the shared dense FFN (DenseFfn, model.rs:673-685).
"""
import ctypes as C
from dataclasses import dataclass

import torch

from . import quant
from ._native import check, lib


@dataclass
class MoeConfig:
    hidden: int = 2048
    experts: int = 64
    used: int = 8
    mid: int = 1024           # expert_feed_forward_length
    shared_mid: int = 1024    # expert_shared_feed_forward_length
    normalize: bool = True    # expert_weights_norm
    scale: float = 1.0        # expert_weights_scale
    dtype: int = 2            # Q4_K expert and shared weights


def random_moe_weights(cfg, device, seed=0):
    """Seeded random-init weights: an N(0, 1) F32 router (as the benchmark
    configuration asks), a small N(0, 0.1) router bias, N(0, 0.02) experts and
    shared FFN packed by hy_mt_rs_b200.synth."""
    from . import synth

    g = torch.Generator().manual_seed(seed)
    H, E, M, S = cfg.hidden, cfg.experts, cfg.mid, cfg.shared_mid
    router = torch.randn(E, H, generator=g).to(device)  # rows = experts, K = hidden contiguous
    bias = (0.1 * torch.randn(E, generator=g)).to(device)
    t = cfg.dtype
    return {
        "router": router.contiguous().view(torch.uint8).reshape(-1),
        "bias": bias,
        "gate": synth.random_packed(t, E * M, H, seed=seed + 1, device=device),
        "up": synth.random_packed(t, E * M, H, seed=seed + 2, device=device),
        "down": synth.random_packed(t, E * H, M, seed=seed + 3, device=device),
        "shared_gate": synth.random_packed(t, S, H, seed=seed + 4, device=device),
        "shared_up": synth.random_packed(t, S, H, seed=seed + 5, device=device),
        "shared_down": synth.random_packed(t, H, S, seed=seed + 6, device=device),
    }


def _p(t):
    return C.c_void_p(t.data_ptr()) if t is not None else C.c_void_p(0)


def expert_major(counts):
    """Expert parallelism: received rows arrive grouped by source rank, then by
    expert (each source sends its rows in its own expert-major order).
    counts[s][e] = rows from source s for local expert e.  Returns (perm,
    inv, off): perm[i] = received index of expert-major row i, inv its
    inverse, off the local experts' row offsets (experts + 1)."""
    import numpy as np

    counts = np.asarray(counts, dtype=np.int64)
    W, El = counts.shape
    recv_base = np.concatenate([[0], np.cumsum(counts.sum(axis=1))[:-1]])  # first row of each source
    src_off = np.concatenate([np.zeros((W, 1), np.int64), np.cumsum(counts, axis=1)[:, :-1]], axis=1)
    off = np.concatenate([[0], np.cumsum(counts.sum(axis=0))])
    perm = np.empty(int(counts.sum()), dtype=np.int64)
    i = 0
    for e in range(El):
        for s in range(W):
            n = int(counts[s, e])
            perm[i:i + n] = recv_base[s] + src_off[s, e] + np.arange(n)
            i += n
    inv = np.empty_like(perm)
    inv[perm] = np.arange(perm.size)
    return perm, inv, off


def ep_send_index(off, world, local_experts, cap):
    """Expert parallelism, sending side, on the device: this rank's grouped
    rows are expert-major, so the rows for rank r's experts are grouped rows
    off[r El] .. off[(r + 1) El].  Returns (idx [world, cap], valid [world,
    cap]): block r of the fixed-capacity send buffer holds grouped rows
    idx[r, :count_r] (the rest is padding, idx 0)."""
    r = torch.arange(world, device=off.device)
    starts = off[r * local_experts].long()
    n = off[(r + 1) * local_experts].long() - starts
    i = torch.arange(cap, device=off.device)
    valid = i[None, :] < n[:, None]
    return torch.where(valid, starts[:, None] + i[None, :], torch.zeros_like(starts)[:, None]), valid


def ep_recv_perm(counts, cap):
    """Expert parallelism, receiving side, on the device: counts [world,
    local experts] = rows source s sent for local expert e, each source's
    rows in its block s * cap .. in expert order.  Returns (perm [world cap],
    valid [world cap], off [experts + 1]): expert-major row t (expert e's
    rows from source 0, then 1, ...) is received row perm[t] for valid t, and
    local expert e owns expert-major rows off[e] .. off[e + 1] (the order of
    expert_major, without a host round trip)."""
    counts = counts.long()
    W, El = counts.shape
    dev = counts.device
    src_off = torch.cumsum(counts, 1) - counts                 # first row of (s, e) in source s's block
    seg = counts.t().reshape(-1)                               # segments in (e, s) order
    seg_end = torch.cumsum(seg, 0)
    seg_start = seg_end - seg
    t = torch.arange(W * cap, device=dev)
    k = torch.searchsorted(seg_end, t, right=True).clamp(max=W * El - 1)
    e, src = k // W, k % W
    perm = src * cap + src_off[src, e] + (t - seg_start[k])
    valid = t < seg_end[-1]
    off = torch.cat([torch.zeros(1, dtype=torch.long, device=dev), torch.cumsum(counts.sum(0), 0)])
    return torch.where(valid, perm, torch.zeros_like(perm)), valid, off


def ep_pack(x, rows, per_expert, world, local_experts, cap):
    """Expert parallelism, sending side: the send buffer of one all-to-all
    that carries, for each destination rank r, its cap rows (rows[r * cap ..],
    token rows of x) followed by one row whose first local_experts floats
    hold the int32 bit patterns of r's experts' row counts
    (per_expert[r El .. (r + 1) El]).  [world * (cap + 1), hidden]."""
    hidden = x.shape[1]
    if hidden < local_experts:
        raise ValueError("expert parallelism: hidden size below the experts per rank")
    ext = torch.cat([rows.view(world, cap), rows.new_zeros(world, 1)], 1).reshape(-1)
    send = x.index_select(0, ext)
    counts = per_expert.to(torch.int32).view(world, local_experts).view(torch.float32)
    send.view(world, cap + 1, hidden)[:, cap, :local_experts] = counts
    return send


def ep_unpack_counts(recv, world, local_experts, cap, stride=None):
    """Receiving side of ep_pack: counts [world, local experts] (int64) of
    the rows each source sent for this rank's experts.  Source s's block
    starts at row s * stride (cap + 1 by default: blocks back to back)."""
    hidden = recv.shape[1]
    stride = cap + 1 if stride is None else stride
    c = recv.view(world, stride, hidden)[:, cap, :local_experts].contiguous()
    return c.view(torch.int32).long()


def ep_packed_rows(perm, cap, stride=None):
    """Received row s * cap + i of the unpacked layout sits at row
    s * stride + i of a layout whose source blocks start `stride` rows apart
    (ep_pack's: cap + 1, one count row per block)."""
    stride = cap + 1 if stride is None else stride
    return (perm // cap) * stride + perm % cap


class MoeLayer:
    """Moe::forward for `tokens` rows of normalized activations.

    ep = (rank, world, process_group): expert parallelism over `world`
    ranks (one per GPU); this rank holds experts [rank * E / world, (rank +
    1) * E / world) and its own tokens.  Token rows travel to the rank of
    each chosen expert and back by NCCL all-to-all, or, with `exchange` (a
    hy_mt_rs_b200.peer.PeerExchange), by pushes into the other ranks'
    NVLink peer-memory regions (only the valid rows travel); routing, shared
    expert and combine stay local, so the result equals the one-GPU layer.
    The exchange has a fixed capacity (tokens * used rows per destination,
    the most a rank can send) and carries the per-expert counts in-band, so
    no count reaches the host and the layer can be captured in a CUDA graph.
    Every rank passes the same token count."""

    def __init__(self, cfg, weights, ep=None, exchange=None):
        self.cfg = cfg
        H, E, M, S, t = cfg.hidden, cfg.experts, cfg.mid, cfg.shared_mid, cfg.dtype
        self.ep = ep
        # expert parallelism over NVLink peer memory instead of NCCL: a
        # hy_mt_rs_b200.peer.PeerExchange whose slots hold (tokens * used +
        # 1) x hidden floats for the largest token count the layer will see
        self.xchg = exchange
        self.router = quant.Weight(weights["router"], quant.DType.F32, [H, E], name="ffn_gate_inp")
        self.bias = weights["bias"]
        gate, up, down, El = weights["gate"], weights["up"], weights["down"], E
        if ep is not None:
            rank, world, _ = ep
            if E % world:
                raise ValueError("experts must divide over the ranks")
            El = E // world
            gu = gate.numel() // E   # bytes of one expert's gate (or up) matrix
            dn = down.numel() // E
            gate = gate[rank * El * gu:(rank + 1) * El * gu]
            up = up[rank * El * gu:(rank + 1) * El * gu]
            down = down[rank * El * dn:(rank + 1) * El * dn]
        self.local_experts = El
        self.gate = quant.Weight(gate, t, [H, M, El], name="ffn_gate_exps")
        self.up = quant.Weight(up, t, [H, M, El], name="ffn_up_exps")
        self.down = quant.Weight(down, t, [M, H, El], name="ffn_down_exps")
        self.shared_gate = quant.Weight(weights["shared_gate"], t, [H, S], name="ffn_gate_shexp")
        self.shared_up = quant.Weight(weights["shared_up"], t, [H, S], name="ffn_up_shexp")
        self.shared_down = quant.Weight(weights["shared_down"], t, [S, H], name="ffn_down_shexp")
        self._bufs = {}

    def _buffers(self, T, device):
        b = self._bufs.get(T)
        if b is None:
            c = self.cfg
            R = T * c.used
            f = dict(device=device)
            b = {
                "logits": torch.empty(T, c.experts, **f),
                "idx": torch.empty(T, c.used, dtype=torch.int32, **f),
                "w": torch.empty(T, c.used, **f),
                "off": torch.empty(c.experts + 1, dtype=torch.int32, **f),
                "row_token": torch.empty(R, dtype=torch.int32, **f),
                "row_weight": torch.empty(R, **f),
                "token_rows": torch.empty(R, dtype=torch.int32, **f),
                "h": torch.empty(R, c.mid, **f),
                "y": torch.empty(R + 1, c.hidden, **f),   # + one row that absorbs padded returns
                "sh": torch.empty(T, c.shared_mid, **f),
                "shared": torch.empty(T, c.hidden, **f),
            }
            self._bufs[T] = b
        return b

    def forward(self, x, tokens, out=None):
        """x: [tokens, hidden] f32 on the device; returns [tokens, hidden]."""
        c = self.cfg
        T = int(tokens)
        b = self._buffers(T, x.device)
        st = C.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)
        if out is None:
            out = torch.empty(T, c.hidden, device=x.device)
        check(lib.hyq_moe_router(self.router.handle, _p(x), T, _p(b["logits"]), st))
        check(lib.hyq_moe_route(_p(b["logits"]), T, c.experts, _p(self.bias), c.used, 1 if c.normalize else 0,
                                c.scale, _p(b["idx"]), _p(b["w"]), st))
        check(lib.hyq_moe_group(_p(b["idx"]), _p(b["w"]), T, c.experts, c.used, _p(b["off"]), _p(b["row_token"]),
                                _p(b["row_weight"]), _p(b["token_rows"]), st))
        R = T * c.used
        if self.ep is None:
            check(lib.hyq_matmul_experts_gate_up_silu(self.gate.handle, self.up.handle, _p(x), _p(b["row_token"]),
                                                      R, _p(b["off"]), T, _p(b["h"]), st))
            check(lib.hyq_matmul_experts(self.down.handle, _p(b["h"]), None, R, _p(b["off"]), T, _p(b["y"]), st))
        else:
            self._experts_ep(x, b, st)
        # shared expert (DenseFfn::forward, model.rs:673-685)
        if T == 1:
            check(lib.hyq_matmul_gate_up_silu(self.shared_gate.handle, self.shared_up.handle, _p(x), _p(b["sh"]), st))
        else:
            check(lib.hyq_matmul_gate_up_silu_batch(self.shared_gate.handle, self.shared_up.handle, _p(x), T,
                                                    _p(b["sh"]), st))
        check(lib.hyq_matmul(self.shared_down.handle, _p(b["sh"]), T, _p(b["shared"]), st))
        check(lib.hyq_moe_combine(_p(b["shared"]), _p(b["y"]), T, c.hidden, _p(b["idx"]), _p(b["token_rows"]),
                                  _p(b["row_weight"]), c.used, _p(out), st))
        return out

    def _experts_ep(self, x, b, st):
        """The expert products of this rank's tokens under expert
        parallelism: b["y"] gets the same rows, in the same grouped order, as
        the one-GPU products would.  Two NCCL all-to-alls of equal splits:
        cap = tokens * used rows to every rank (the rows for its experts,
        padded) with the per-expert counts in one extra row per block
        (ep_pack), then the results back."""
        import torch.distributed as dist

        rank, world, group = self.ep
        c, El = self.cfg, self.local_experts
        T = x.shape[0]
        cap = T * c.used
        dev = x.device
        off = b["off"]
        if self.xchg is not None:
            self._experts_ep_peer(x, b, st)
            return
        per_expert = off[1:] - off[:-1]                        # [E] rows per expert, this rank's tokens
        send_idx, send_valid = ep_send_index(off, world, El, cap)
        rows = b["row_token"].long()[send_idx.reshape(-1)]
        send = ep_pack(x, rows, per_expert, world, El, cap)    # [world * (cap + 1), hidden]
        stride = cap + 1
        recv = torch.empty(world * stride, c.hidden, device=dev)
        dist.all_to_all_single(recv, send, group=group)
        counts = ep_unpack_counts(recv, world, El, cap, stride)
        perm, valid, loff = ep_recv_perm(counts, cap)
        perm_d, off_d = ep_packed_rows(perm, cap, stride).to(torch.int32), loff.to(torch.int32)
        Rr = world * cap
        h = torch.empty(Rr, c.mid, device=dev)
        y = torch.empty(Rr, c.hidden, device=dev)
        # any local expert sees at most every rank's tokens once
        check(lib.hyq_matmul_experts_gate_up_silu(self.gate.handle, self.up.handle, _p(recv), _p(perm_d), Rr,
                                                  _p(off_d), world * T, _p(h), st))
        check(lib.hyq_matmul_experts(self.down.handle, _p(h), None, Rr, _p(off_d), world * T, _p(y), st))
        # back into received order (padding rows go to a spare row), then home
        yr = torch.empty(Rr + 1, c.hidden, device=dev)
        yr.index_copy_(0, torch.where(valid, perm, torch.full_like(perm, Rr)), y)
        back = torch.empty(Rr, c.hidden, device=dev)
        dist.all_to_all_single(back, yr[:Rr], group=group)
        R = T * c.used
        dest = torch.where(send_valid, send_idx, torch.full_like(send_idx, R)).reshape(-1)
        b["y"].index_copy_(0, dest, back)

    def _experts_ep_peer(self, x, b, st):
        """_experts_ep over NVLink peer memory with the index work inside the
        library: dispatch (grouped rows gathered straight from x, counts
        in-band), plan (expert-major gather index and its inverse from the
        received counts), the expert products reading the region, return
        (outputs gathered by the inverse), home (into b["y"])."""
        rank, world, _ = self.ep
        c, El, X = self.cfg, self.local_experts, self.xchg
        T = x.shape[0]
        cap = T * c.used
        dev = x.device
        if X.slot < (cap + 1) * c.hidden or X.slot % c.hidden:
            raise ValueError("expert parallelism: the exchange's slots are too small for this token count")
        Rr = world * cap
        key = ("ep", T)
        e = self._bufs.get(key)
        if e is None:
            i32 = dict(dtype=torch.int32, device=dev)
            e = {"perm": torch.empty(Rr, **i32), "off": torch.empty(El + 1, **i32), "inv": torch.zeros(Rr, **i32),
                 "back": torch.empty(world, **i32), "h": torch.empty(Rr, c.mid, device=dev),
                 "y": torch.empty(Rr, c.hidden, device=dev)}
            self._bufs[key] = e
        regions, nbytes, slot = X._regions, X.data_bytes, X.slot
        check(lib.hyq_moe_ep_dispatch(regions, rank, world, nbytes, slot, _p(x), T, c.hidden, _p(b["off"]),
                                      _p(b["row_token"]), El, cap, st))
        check(lib.hyq_moe_ep_plan(regions, rank, world, nbytes, slot, c.hidden, cap, El, _p(e["perm"]),
                                  _p(e["off"]), _p(e["inv"]), _p(e["back"]), st))
        recv = X.recv(slot // c.hidden, c.hidden)
        check(lib.hyq_matmul_experts_gate_up_silu(self.gate.handle, self.up.handle, _p(recv), _p(e["perm"]), Rr,
                                                  _p(e["off"]), world * T, _p(e["h"]), st))
        check(lib.hyq_matmul_experts(self.down.handle, _p(e["h"]), None, Rr, _p(e["off"]), world * T, _p(e["y"]),
                                     st))
        check(lib.hyq_moe_ep_return(regions, rank, world, nbytes, slot, _p(e["y"]), c.hidden, _p(e["inv"]),
                                    _p(e["back"]), cap, st))
        check(lib.hyq_moe_ep_home(regions, rank, world, nbytes, slot, c.hidden, _p(b["off"]), El, cap, _p(b["y"]),
                                  st))

    def launches(self, tokens):
        """Kernel launches of the library in one forward (for the bench's
        count): router, route, group, 2 x (conversion + expert GEMM), shared
        FFN, combine; with the peer-memory exchange its dispatch and
        return (two launches each), plan and home."""
        return 3 + 4 + (2 if tokens == 1 else 4) + 1 + (6 if self.xchg is not None else 0)
