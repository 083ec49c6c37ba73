"""Run token steps of the Dense decoder (hy_mt_rs_b200.model), for profiler
captures.

    python -m hy_mt_rs_b200.profile_model --layers 32 --prompt 8 --steps 3

Builds the seeded random-init model with the 1.8B shapes (Q2_0C linears,
tied Q6_K embedding), captures one token step as a CUDA graph, feeds
`--prompt` tokens in one batched forward and then `--steps` greedy steps,
one graph replay each.
Every replay launches the same kernels in the same order (a launch list of
one replay is one token step).

    python -m hy_mt_rs_b200.profile_model --batch 64 --prompt 256 --steps 3

With --batch B: B concurrent requests (DenseBatch), every request starting
at position --prompt over zero caches (the step's work depends on the
positions only, so no prompt is fed), then --steps replays of the batch step.
"""
import argparse

import torch

from .model import DenseBatch, DenseConfig, DenseModel, random_weights


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--prompt", type=int, default=8)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--batch", type=int, default=0)
    ap.add_argument("--kv16", action="store_true", help="f16 KV cache")
    ap.add_argument("--precision", choices=["fp16", "f32"], default="fp16",
                    help="batched products: fp16 operands or split operands")
    a = ap.parse_args()
    dev = torch.device("cuda", 0)
    cfg = DenseConfig(layers=a.layers, positions=a.prompt + a.steps + 1)
    from . import quant
    prec = quant.GEMM_F32 if a.precision == "f32" else quant.GEMM_FP16
    model = DenseModel(cfg, random_weights(cfg, dev, seed=1), dev, kv16=a.kv16, gemm_precision=prec)
    torch.cuda.synchronize()
    stream = torch.cuda.Stream(dev)
    if a.batch:
        batch = DenseBatch(model, a.batch)
        batch.capture(stream)
        with torch.cuda.stream(stream):
            batch.pos.fill_(a.prompt)
            for _ in range(a.steps):
                batch.graph.replay()
        stream.synchronize()
        print("tokens", batch.tokens.cpu().tolist())
        return
    ids = model.generate(list(range(1, a.prompt + 1)), a.steps, stream, batched_prefill=True)
    print("tokens", ids)


if __name__ == "__main__":
    main()
