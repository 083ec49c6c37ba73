"""Run one product shape a few times, for profiler captures.

    python -m hy_mt_rs_b200.profile_gemv --dtype Q6_K --rows 120832 --cols 2048 \
        --path f32 --iters 3

Every iteration is one launch of the product kernel (plus one Q8 launch
with --path q8; --path int8 quantizes inside the product kernel, as the
bench's q8 decode chain does).  Weights are seeded synthetic (hy_mt_rs_b200.synth).
"""
import argparse

import torch

from . import quant, synth


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--dtype", default="Q6_K", choices=[d.name for d in quant.DType])
    ap.add_argument("--rows", type=int, default=120832)
    ap.add_argument("--cols", type=int, default=2048)
    ap.add_argument("--path", choices=["f32", "q8", "int8"], default="f32")
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--batch", type=int, default=1, help="> 1: batched product (tensor-core GEMM)")
    ap.add_argument("--gate-up", action="store_true",
                    help="batched: the fused gate/up-SiLU product of two such matrices (the 7B layer's FFN call)")
    ap.add_argument("--precision", choices=["fp16", "f32"], default="fp16",
                    help="batched: fp16 operands or split operands (hyq_set_gemm_precision)")
    a = ap.parse_args()
    dev = torch.device("cuda", 0)
    t = quant.DType[a.dtype]
    w = quant.Weight(synth.random_packed(t, a.rows, a.cols, seed=1, device=dev), t, [a.cols, a.rows])
    up = quant.Weight(synth.random_packed(t, a.rows, a.cols, seed=2, device=dev), t, [a.cols, a.rows]) \
        if a.gate_up else None
    x = torch.randn(a.batch * a.cols, generator=torch.Generator().manual_seed(0)).to(dev)
    q8 = quant.Q8(a.cols, dev)
    quant.set_gemm_precision(quant.GEMM_F32 if a.precision == "f32" else quant.GEMM_FP16)
    for _ in range(a.iters):
        if a.batch > 1 and up is not None:
            w.matmul_gate_up_silu_batch(up, x, a.batch)
        elif a.batch > 1:
            w.matmul(x, a.batch)
        elif a.path == "f32":
            w.matmul(x, 1)
        elif a.path == "int8":
            w.gemv_int8(x)
        else:
            q8.quantize_into(x)
            w.gemv_q8_fast(q8)
    torch.cuda.synchronize()
    assert quant.device_status() == 0
    print("ok")


if __name__ == "__main__":
    main()
