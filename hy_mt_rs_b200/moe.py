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


class MoeLayer:
    """Moe::forward for `tokens` rows of normalized activations."""

    def __init__(self, cfg, weights):
        self.cfg = cfg
        H, E, M, S, t = cfg.hidden, cfg.experts, cfg.mid, cfg.shared_mid, cfg.dtype
        self.router = quant.Weight(weights["router"], quant.DType.F32, [H, E], name="ffn_gate_inp")
        self.bias = weights["bias"]
        self.gate = quant.Weight(weights["gate"], t, [H, M, E], name="ffn_gate_exps")
        self.up = quant.Weight(weights["up"], t, [H, M, E], name="ffn_up_exps")
        self.down = quant.Weight(weights["down"], t, [M, H, E], name="ffn_down_exps")
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
        check(lib.hyq_matmul_experts_gate_up_silu(self.gate.handle, self.up.handle, _p(x), _p(b["row_token"]), R,
                                                  _p(b["off"]), T, _p(b["h"]), st))
        check(lib.hyq_matmul_experts(self.down.handle, _p(b["h"]), None, R, _p(b["off"]), T, _p(b["y"]), st))
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

    def launches(self, tokens):
        """Kernel launches of one forward (for the bench's count)."""
        # router, route, group, 2 x (conversion + expert GEMM), shared FFN, combine
        return 3 + 4 + (2 if tokens == 1 else 4) + 1
