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


class MoeLayer:
    """Moe::forward for `tokens` rows of normalized activations.

    ep = (rank, world, process_group): expert parallelism over `world`
    ranks (one per GPU); this rank holds experts [rank * E / world, (rank +
    1) * E / world) and its own tokens.  Token rows travel to the rank of
    each chosen expert and back by NCCL all-to-all; routing, shared expert
    and combine stay local, so the result equals the one-GPU layer."""

    def __init__(self, cfg, weights, ep=None):
        self.cfg = cfg
        H, E, M, S, t = cfg.hidden, cfg.experts, cfg.mid, cfg.shared_mid, cfg.dtype
        self.ep = ep
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
                "y": torch.empty(R, c.hidden, **f),
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
        the one-GPU products would."""
        import torch.distributed as dist

        rank, world, group = self.ep
        c, El = self.cfg, self.local_experts
        off = b["off"].cpu()  # split sizes of the exchange live on the host
        per_expert = (off[1:] - off[:-1]).to(torch.int32)
        send_rows = [int(off[(r + 1) * El] - off[r * El]) for r in range(world)]
        # rows each source sends for each of this rank's experts
        recv_cnt = torch.empty(world * El, dtype=torch.int32, device=x.device)
        dist.all_to_all_single(recv_cnt, per_expert.to(x.device), group=group)
        counts = recv_cnt.cpu().view(world, El)
        recv_rows = [int(v) for v in counts.sum(dim=1)]
        xg = x.index_select(0, b["row_token"].long())           # this rank's rows, grouped by expert
        recv = torch.empty(sum(recv_rows), c.hidden, device=x.device)
        dist.all_to_all_single(recv, xg, recv_rows, send_rows, group=group)
        perm, inv, loff = expert_major(counts.numpy())
        Rr = int(perm.size)
        yr = torch.empty(Rr, c.hidden, device=x.device)
        if Rr:
            dev = x.device
            perm_d = torch.from_numpy(perm.astype("int32")).to(dev)
            off_d = torch.from_numpy(loff.astype("int32")).to(dev)
            h = torch.empty(Rr, c.mid, device=dev)
            y = torch.empty(Rr, c.hidden, device=dev)
            check(lib.hyq_matmul_experts_gate_up_silu(self.gate.handle, self.up.handle, _p(recv), _p(perm_d), Rr,
                                                      _p(off_d), Rr, _p(h), st))
            check(lib.hyq_matmul_experts(self.down.handle, _p(h), None, Rr, _p(off_d), Rr, _p(y), st))
            yr = y.index_select(0, torch.from_numpy(inv).to(dev))  # back in received order
        dist.all_to_all_single(b["y"][:sum(send_rows)], yr, send_rows, recv_rows, group=group)

    def launches(self, tokens):
        """Kernel launches of one forward (for the bench's count)."""
        # router, route, group, 2 x (conversion + expert GEMM), shared FFN, combine
        return 3 + 4 + (2 if tokens == 1 else 4) + 1
