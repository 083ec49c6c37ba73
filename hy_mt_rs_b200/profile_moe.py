"""Run forwards of the MoE FFN layer (hy_mt_rs_b200.moe), for profiler
captures.

    python -m hy_mt_rs_b200.profile_moe --tokens 64 --iters 3

Config 5 shapes (64 experts, top-8, 2048->1024->2048 Q4_K, shared expert),
seeded random-init weights; every iteration is one forward of `--tokens`
rows, with the same launches in the same order.
"""
import argparse

import torch

from .moe import MoeConfig, MoeLayer, random_moe_weights


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=64)
    ap.add_argument("--iters", type=int, default=3)
    a = ap.parse_args()
    dev = torch.device("cuda", 0)
    cfg = MoeConfig()
    layer = MoeLayer(cfg, random_moe_weights(cfg, dev, seed=3))
    x = torch.randn(a.tokens, cfg.hidden, generator=torch.Generator().manual_seed(a.tokens)).to(dev)
    for _ in range(a.iters):
        layer.forward(x, a.tokens)
    torch.cuda.synchronize()
    print("ok")


if __name__ == "__main__":
    main()
