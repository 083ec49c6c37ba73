#!/usr/bin/env python
"""Benchmark of the block-quantized decode GEMV path (hy-mt-rs config 2).

Workload ("1.8B decoder-layer projections + lm_head, batch 1"): the
projections one Hy-MT2-1.8B decode step runs per layer (model.rs:403-538),
repeated for each low-bit format -- Q2_0C and STQ1_0 layers with
q 2048x2048, k/v 512x2048, o 2048x2048, gate/up 6144x2048 (fused SiLU),
down 2048x6144 -- followed by the Q6_K lm_head 120832x2048.  Weights are
seeded N(0, 0.02) packed by hy_mt_rs_b200.synth; activations N(0, 1).

A step is one pass of that chain.  The metric is quantized-GEMV HBM
throughput: algorithmic bytes (packed weights + f32 activations read + f32
outputs written) per second, whole job.  Every step reads the 203 MB lm_head,
which is larger than the 126 MB L2, and the layers rotate over `--copies`
distinct weight copies, so no step starts with its weights in L2.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--path f32|q8]
    python bench.py --impl reference ...   # the reference's CPU path

--path f32 (default) takes f32 activations like the reference's x86 path;
--path q8 quantizes activations per 256 values first, like the reference's
aarch64 decode loop (model.rs:404-533).
"""
import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

HIDDEN, FFN, KV, VOCAB = 2048, 6144, 512, 120832
# (name, rows N, input width K) of one decoder layer, in call order
LAYER = [("attn_q", HIDDEN, HIDDEN), ("attn_k", KV, HIDDEN), ("attn_v", KV, HIDDEN),
         ("attn_output", HIDDEN, HIDDEN), ("ffn_gate", FFN, HIDDEN), ("ffn_up", FFN, HIDDEN),
         ("ffn_down", HIDDEN, FFN)]
N_LAYERS_MODEL = 32


def args_parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["hyq", "reference"], default="hyq")
    ap.add_argument("--path", choices=["f32", "q8"], default="f32")
    ap.add_argument("--copies", type=int, default=4)
    ap.add_argument("--no-overlap", action="store_true",
                    help="decode: plain stream order instead of overlapped launches (hyq_set_launch_overlap)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU baseline sample budget")
    ap.add_argument("--workload", choices=["decode", "prefill", "gemv", "tp", "model", "moe", "moe-stack"],
                    default="decode",
                    help="decode: config 2 (default line); prefill: config 3 (7B layer GEMMs); "
                         "gemv: config 1 (one 6144x2048 product, L2 defeated by rotating copies)")
    ap.add_argument("--tp-mode", choices=["decode", "prefill"], default="decode",
                    help="tp: batch-1 layer chain (decode) or the layer's GEMMs at --tokens (prefill)")
    ap.add_argument("--tp-allreduce", choices=["peer", "nccl"], default="peer",
                    help="tp decode: all-reduce by hyq_peer_allreduce (NVLink peer memory) or NCCL")
    ap.add_argument("--ep-exchange", choices=["peer", "nccl"], default="peer",
                    help="moe at N > 1: expert-parallel row exchange by hyq_peer_exchange (NVLink peer memory) "
                         "or NCCL all-to-all")
    ap.add_argument("--sweep", action="store_true",
                    help="gemv: also measure every packed format at 6144x2048 and 120832x2048, both paths")
    ap.add_argument("--tokens", type=int, default=512, help="prefill: tokens M")
    ap.add_argument("--concurrency", type=int, default=1,
                    help="model: independent requests decoded together (config 4 asks for 1 and 64)")
    ap.add_argument("--model-fused", action="store_true",
                    help="model: run each token step as one persistent kernel (hyq_dense_step) instead of the "
                         "per-kernel graph (the default, which measures faster)")
    ap.add_argument("--gemm-precision", choices=["fp16", "f32"], default=None,
                    help="batched tensor-core products: fp16 operands, or split operands (f32-accurate, "
                         "hyq_set_gemm_precision); default fp16 for prefill, f32 for concurrent decode")
    ap.add_argument("--activations", choices=["f32", "q8"], default="f32",
                    help="model, one request: the single-token products' activations -- f32 (the reference's x86 "
                         "branch) or Q8 (its aarch64 SDOT branch, gemv_q8_fast and friends)")
    ap.add_argument("--kv16", action="store_true",
                    help="model: f16 KV cache (BASELINE config 4) instead of the reference's f32 cache")
    ap.add_argument("--no-suite", action="store_true",
                    help="decode: print the config-2 line alone, without the other configs' measurements")
    return ap.parse_args()


def row_bytes(dtype, K):
    bl = {0: 1, 1: 1, 2: 256, 3: 256, 4: 32, 5: 512, 6: 256}[int(dtype)]
    bb = {0: 4, 1: 2, 2: 144, 3: 210, 4: 34, 5: 130, 6: 42}[int(dtype)]
    return K // bl * bb


def gemv_bytes(dtype, N, K):
    """Algorithmic bytes of one batch-1 product: packed W + f32 x + f32 y."""
    return N * row_bytes(dtype, K) + 4 * K + 4 * N


def layer_bytes(dtype):
    b = 0
    for name, N, K in LAYER:
        b += N * row_bytes(dtype, K)
    # activations: qkv reads x once, writes q,k,v; o; gate/up reads x once, writes N; down
    b += 4 * (HIDDEN + HIDDEN + 2 * KV) + 4 * (HIDDEN + HIDDEN) + 4 * (HIDDEN + FFN) + 4 * (FFN + HIDDEN)
    return b


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profile_traffic(kernel_key):
    """DRAM bytes per launch of the dominant kernel from the committed ncu
    summary (profiles/ncu_traffic.json), or None."""
    p = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return d.get(kernel_key, {}).get("dram_bytes_per_launch")
    except Exception:
        return None


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------
class ClockSampler:
    """Samples SM clock and throttle reasons of one GPU through NVML (read-only)."""

    REASONS = [
        ("gpu_idle", 0x1), ("applications_clocks_setting", 0x2), ("sw_power_cap", 0x4),
        ("hw_slowdown", 0x8), ("sync_boost", 0x10), ("sw_thermal_slowdown", 0x20),
        ("hw_thermal_slowdown", 0x40), ("hw_power_brake_slowdown", 0x80), ("display_clock_setting", 0x100),
    ]

    def __init__(self, uuid, period=0.005):
        self.samples = []
        self.reasons = 0
        self.period = period
        self._stop = threading.Event()
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByUUID(uuid)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.max_mhz = None

    def _sample(self):
        try:
            self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
            self.reasons |= self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
        except Exception:
            pass

    def _run(self):
        while not self._stop.is_set():
            self._sample()
            time.sleep(self.period)

    def start(self):
        if self.ok:
            self._sample()
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()

    def stop(self):
        if self.ok:
            self._stop.set()
            self.t.join()
            self._sample()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["nvml_unavailable"], "samples": 0}
        reasons = [n for n, bit in self.REASONS if self.reasons & bit and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# CPU baseline / reference arm: the oracle port of the reference's x86 path
# ---------------------------------------------------------------------------
def cpu_workload(seed=0, lm_rows=None):
    import numpy as np

    from hy_mt_rs_b200 import synth

    layers = {}
    for fmt in (5, 6):
        layers[fmt] = [(name, N, K, synth.random_packed(fmt, N, K, seed=seed + 100 * fmt + i).numpy())
                       for i, (name, N, K) in enumerate(LAYER)]
    lm_rows = lm_rows or VOCAB
    lm = synth.random_packed(3, lm_rows, HIDDEN, seed=seed + 7).numpy()
    x = np.random.default_rng(seed).standard_normal(HIDDEN).astype(np.float32)
    return layers, lm, lm_rows, x


def cpu_step(layers, lm, lm_rows, x, threads=0):
    """One pass of the chain through the oracle (x86 f32 order)."""
    from oracle import oracle as O

    h = x
    for fmt in (5, 6):
        L = {name: (N, K, p) for name, N, K, p in layers[fmt]}
        q = O.matmul(fmt, L["attn_q"][2], HIDDEN, HIDDEN, h, 1, threads)[0]
        O.matmul(fmt, L["attn_k"][2], HIDDEN, KV, h, 1, threads)
        O.matmul(fmt, L["attn_v"][2], HIDDEN, KV, h, 1, threads)
        o = O.matmul(fmt, L["attn_output"][2], HIDDEN, HIDDEN, q, 1, threads)[0]
        g = O.gate_up_silu(fmt, L["ffn_gate"][2], L["ffn_up"][2], HIDDEN, FFN, o, threads)
        h = O.matmul(fmt, L["ffn_down"][2], FFN, HIDDEN, g, 1, threads)[0]
    return O.matmul(3, lm, HIDDEN, lm_rows, h, 1, threads)[0]


def cpu_step_bytes(lm_rows):
    return layer_bytes(5) + layer_bytes(6) + gemv_bytes(3, lm_rows, HIDDEN)


def host_threads():
    """Every host core this process may run on.  Set explicitly on each
    oracle call, because torchrun exports OMP_NUM_THREADS=1 to its ranks."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def run_cpu(seconds, lm_rows):
    layers, lm, lm_rows, x = cpu_workload(lm_rows=lm_rows)
    threads = host_threads()
    cpu_step(layers, lm, lm_rows, x, threads)  # warm
    n = 0
    t0 = time.perf_counter()
    while True:
        cpu_step(layers, lm, lm_rows, x, threads)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    gbs = n * cpu_step_bytes(lm_rows) / el / 1e9
    what = "the whole chain" if lm_rows == VOCAB else f"the chain with the lm_head cut to {lm_rows} of {VOCAB} rows"
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{n} passes of {what} ({el:.1f} s); oracle/hyq_oracle.c x86 f32 order, OpenMP"}


METRIC = "quantized GEMV HBM GB/s (1.8B layer projections Q2_0C+STQ1_0 + Q6_K lm_head, batch 1)"


def decode_config(a, world):
    """The `config` of the default line, shared verbatim by both arms."""
    return {"workload": "hy-mt-rs config 2: 1.8B decoder-layer projections (Q2_0C, STQ1_0) + "
                        "Q6_K lm_head 120832x2048, batch 1",
            "path": a.path, "layer_copies": max(1, a.copies),
            "step_bytes": layer_bytes(5) + layer_bytes(6) + gemv_bytes(3, VOCAB, HIDDEN),
            "launch_overlap": not a.no_overlap,
            "l2": "inputs larger than L2: every step streams the 203 MB lm_head; layers rotate copies",
            "step": "one CUDA graph per pass of the chain (one per weight copy)",
            "parallelism": f"replicas x{world} (rows are independent; no collective)"}


def reference_arm(a):
    """The reference's CPU path (the oracle port of its x86 f32 path, all host
    threads) on the default line's workload: every step is the whole chain,
    both layers and all 120832 lm_head rows.  Under torchrun rank 0 alone
    runs it.  Loads no GPU library."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return None
    layers, lm, lm_rows, x = cpu_workload()
    threads = host_threads()
    for _ in range(a.warmup):
        cpu_step(layers, lm, lm_rows, x, threads)
    t0 = time.perf_counter()
    for _ in range(a.steps):
        cpu_step(layers, lm, lm_rows, x, threads)
    el = time.perf_counter() - t0
    gbs = a.steps * cpu_step_bytes(lm_rows) / el / 1e9
    sample = (f"each step: the whole chain (both layers, all {VOCAB} lm_head rows), the CPU port of the "
              f"reference's x86 f32 path (oracle/hyq_oracle.c, OpenMP)")
    line = {
        "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": a.gpus, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": round(el / a.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "f32 activations x packed int weights (f32 accumulate)" if a.path == "f32"
                 else "int8 activations (Q8, per-256 scale) x packed int weights",
        "data": "synthetic (seeded N(0,0.02) weights packed by hy_mt_rs_b200.synth; N(0,1) activations)",
        "config": decode_config(a, world),
        "impl": "reference",
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    return line


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def build_weights(dev, copies, seed=0):
    from hy_mt_rs_b200 import quant, synth

    layers = {5: [], 6: []}
    for fmt in (5, 6):
        for c in range(copies):
            L = {}
            for i, (name, N, K) in enumerate(LAYER):
                packed = synth.random_packed(fmt, N, K, seed=seed + 1000 * c + 100 * fmt + i, device=dev)
                L[name] = quant.Weight(packed, fmt, [K, N], name=name)
            layers[fmt].append(L)
    lm = quant.Weight(synth.random_packed(3, VOCAB, HIDDEN, seed=seed + 7, device=dev), 3, [HIDDEN, VOCAB],
                      name="output")
    return layers, lm


def layer_chain(L, h, path, q8h=None, q8f=None):
    """Projections of one decoder layer (model.rs:403-538 order)."""
    from hy_mt_rs_b200.quant import Weight

    if path == "f32":
        q, k, v = Weight.gemv_qkv(L["attn_q"], L["attn_k"], L["attn_v"], h)
        o = L["attn_output"].matmul(q, 1)[0]  # attention output stands in as q (same width)
        g = L["ffn_gate"].matmul_gate_up_silu(L["ffn_up"], o)
        return L["ffn_down"].matmul(g, 1)[0]
    # int8 activations quantized inside each product kernel (one launch per
    # projection group, as the reference quantizes once per group)
    q, k, v = Weight.gemv_qkv_int8(L["attn_q"], L["attn_k"], L["attn_v"], h)
    o = L["attn_output"].gemv_int8(q)
    g = L["ffn_gate"].matmul_gate_up_silu_int8(L["ffn_up"], o)
    return L["ffn_down"].gemv_int8(g)


def lm_head(lm, h, path, q8h=None):
    if path == "f32":
        return lm.matmul(h, 1)[0]
    return lm.gemv_int8(h)


def reduce_over_ranks(times_ms, clocks, device):
    """Timing across replicas: every rank's device-timed durations reduced
    with MAX (the job ends when its slowest rank does) and every rank's clock
    summary gathered.  Same collectives, same order, on every rank."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return [float(t) for t in times_ms], [clocks]
    t = torch.tensor([float(x) for x in times_ms], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    clocks_all = [None] * dist.get_world_size()
    dist.all_gather_object(clocks_all, clocks)
    return [float(x) for x in t.tolist()], clocks_all


def device_failed(quant, dev):
    """1.0 when a kernel on this device reported an expired bounded wait (the
    status word), else 0.0; reduced with the timings so every rank raises
    together instead of leaving the others inside a collective."""
    try:
        return 0.0 if quant.device_status(dev) == 0 else 1.0
    except quant.HyqError:
        return 1.0


def job_rate(unit_per_step, steps, world, ms):
    """Whole-job throughput: the units all replicas processed over the
    max-over-ranks time, in units per second."""
    return unit_per_step * steps * world / (ms * 1e-3)


def finish_ranks():
    """End the process group once, after every arm of the run."""
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()


def sub_args(a, **kw):
    import copy

    b = copy.copy(a)
    b.__dict__.update(kw)
    return b


def run_suite(a):
    """The other BASELINE configs, measured in the same run after the config-2
    line (every rank runs every arm; rank 0 collects the lines).  Each keeps
    its own step count so that the whole run stays within a few minutes, and
    each reports its value, roofline, e2e, clocks and (one GPU) CPU baseline.
    At N > 1 config 3 is the tensor-parallel layer (NCCL all-reduce of the
    row-parallel partials) and config 5 expert-parallel (NCCL all-to-all)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    out = {"config1": gemv_arm(sub_args(a, sweep=False))}
    if world == 1:
        out["config3"] = {f"M{M}": prefill_arm(sub_args(a, tokens=M, steps=10, warmup=3, gemm_precision="fp16"))
                          for M in (128, 512, 2048)}
        out["config3"]["M2048_f32_products"] = prefill_arm(
            sub_args(a, tokens=2048, steps=5, warmup=3, gemm_precision="f32", cpu_seconds=0))
    else:
        out["config3"] = {"M2048_tp": tp_arm(sub_args(a, tp_mode="prefill", tokens=2048, steps=10, warmup=3))}
    # config 4 as BASELINE names it (f16 KV cache) with split-operand products
    # (the setting the token-stream tests pin), then labelled variants: the
    # reference's f32 cache, and fp16 tensor-core operands
    out["config4"] = {
        "concurrency_1": model_arm(sub_args(a, concurrency=1, model_fused=False, warmup=3, kv16=True)),
        "concurrency_64": model_arm(sub_args(a, concurrency=64, warmup=3, gemm_precision="f32", kv16=True)),
        "concurrency_1_f32_kv": model_arm(sub_args(a, concurrency=1, model_fused=False, warmup=3, kv16=False,
                                                   cpu_seconds=0)),
        "concurrency_1_q8_activations": model_arm(sub_args(a, concurrency=1, model_fused=False, warmup=3, kv16=True,
                                                           activations="q8", cpu_seconds=0)),
        "concurrency_64_f32_kv": model_arm(sub_args(a, concurrency=64, warmup=3, gemm_precision="f32", kv16=False,
                                                    cpu_seconds=0)),
        "concurrency_64_fp16_products": model_arm(sub_args(a, concurrency=64, warmup=3, gemm_precision="fp16",
                                                           kv16=True, cpu_seconds=0))}
    out["config5"] = {"moe_ffn": moe_arm(sub_args(a, steps=20, warmup=3)),
                      "layer_stack": moe_stack_arm(sub_args(a, warmup=3))}
    return out


def init_ranks():
    """One process per GPU (torchrun's RANK / LOCAL_RANK / WORLD_SIZE); NCCL
    only for the barriers and the max-over-ranks timing."""
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():   # the suite's arms share one process group
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local if world > 1 else 0)
    torch.cuda.set_device(dev)
    return world, rank, dev


def gpu_arm(a):
    import torch
    import torch.distributed as dist

    world, rank, dev = init_ranks()

    import hy_mt_rs_b200.quant  # noqa: F401  (loads libhyq.so or raises)
    from hy_mt_rs_b200 import quant

    copies = max(1, a.copies)
    layers, lm = build_weights(dev, copies)
    path = a.path
    # The weights are final before any product is issued, which is what
    # overlapped launches require of the caller.
    torch.cuda.synchronize(dev)
    quant.set_launch_overlap(not a.no_overlap)
    x_static = torch.randn(HIDDEN, generator=torch.Generator().manual_seed(0)).to(dev)
    q8h = quant.Q8(HIDDEN, dev)
    q8f = quant.Q8(FFN, dev)

    # One graph per (format, copy) for the layer chain, one for the lm_head.
    stream = torch.cuda.Stream(dev)
    h_mid = {}
    graphs = {}
    with torch.cuda.stream(stream):
        for _ in range(2):  # warm every path (plans, smem attributes, status word)
            h = x_static
            for fmt in (5, 6):
                for c in range(copies):
                    hh = layer_chain(layers[fmt][c], h, path, q8h, q8f)
                h = hh
            lm_head(lm, h, path, q8h)
        stream.synchronize()
        for c in range(copies):
            h = x_static
            for fmt in (5, 6):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    out = layer_chain(layers[fmt][c], h, path, q8h, q8f)
                graphs[(fmt, c)] = g
                h_mid[(fmt, c)] = out
                h = out
        # all copies end in the same buffer role; the lm_head reads copy 0's output
        h_last = h_mid[(6, 0)]
        g_lm = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_lm, stream=stream):
            logits = lm_head(lm, h_last, path, q8h)
        # The whole chain of one copy as one graph (the timed step): each
        # stage's first product then launches as a programmatic dependent of
        # the previous stage's last one, as inside a stage.  The per-stage
        # graphs above time the stages for the breakdown and the roofline.
        full, logits_full = [], []
        for c in range(copies):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                h = x_static
                for fmt in (5, 6):
                    h = layer_chain(layers[fmt][c], h, path, q8h, q8f)
                logits_full.append(lm_head(lm, h, path, q8h))
            full.append(g)
    launches_per_step = 4 * 2 + 1

    def step(i, evs=None):
        c = i % copies
        if evs is not None:
            evs[0].record(stream)
        graphs[(5, c)].replay()
        if evs is not None:
            evs[1].record(stream)
        graphs[(6, c)].replay()
        if evs is not None:
            evs[2].record(stream)
        g_lm.replay()
        if evs is not None:
            evs[3].record(stream)

    with torch.cuda.stream(stream):
        for i in range(a.warmup):
            step(i)
            full[i % copies].replay()
    stream.synchronize()

    sampler = ClockSampler("GPU-" + str(torch.cuda.get_device_properties(dev).uuid))
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(a.steps)]
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    sampler.start()
    with torch.cuda.stream(stream):
        start.record(stream)
        for i in range(a.steps):
            full[i % copies].replay()
        end.record(stream)
        for i in range(a.steps):   # the stage breakdown
            step(i, evs[i])
    stream.synchronize()
    torch.cuda.synchronize(dev)
    sampler.stop()
    if world > 1:
        dist.barrier()
    ms = start.elapsed_time(end)
    t_q2 = statistics.fmean(e[0].elapsed_time(e[1]) for e in evs)
    t_stq = statistics.fmean(e[1].elapsed_time(e[2]) for e in evs)
    t_lm = statistics.fmean(e[2].elapsed_time(e[3]) for e in evs)
    failed = device_failed(quant, dev)

    # ---- e2e: host buffers through the public API, copies inside the region
    x_host = torch.randn(HIDDEN, generator=torch.Generator().manual_seed(1)).pin_memory()
    logits_host = torch.empty(VOCAB, dtype=torch.float32).pin_memory()
    e2e_steps = a.steps
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        for i in range(3):
            x_static.copy_(x_host, non_blocking=True)
            full[i % copies].replay()
            logits_host.copy_(logits_full[i % copies], non_blocking=True)
        stream.synchronize()
        e0.record(stream)
        for i in range(e2e_steps):
            x_static.copy_(x_host, non_blocking=True)
            full[i % copies].replay()
            logits_host.copy_(logits_full[i % copies], non_blocking=True)
            stream.synchronize()  # a decode loop needs the logits on the host every token
        e1.record(stream)
    stream.synchronize()
    e2e_ms = e0.elapsed_time(e1)

    step_bytes = layer_bytes(5) + layer_bytes(6) + gemv_bytes(3, VOCAB, HIDDEN)
    (ms, e2e_ms, failed), clocks_all = reduce_over_ranks([ms, e2e_ms, failed + device_failed(quant, dev)],
                                                         sampler.summary(), dev)
    if failed:
        raise RuntimeError("a kernel reported an expired bounded wait (device status word) on some rank")

    if rank == 0:
        peak, peak_kind = measured_peaks()
        lm_bytes = gemv_bytes(3, VOCAB, HIDDEN)
        achieved = lm_bytes / (t_lm * 1e-3) / 1e9
        value = job_rate(step_bytes, a.steps, world, ms) / 1e9
        e2e_value = job_rate(step_bytes, e2e_steps, world, e2e_ms) / 1e9
        sm = [c["sm_mhz"] for c in clocks_all if c.get("sm_mhz")]
        reasons = sorted({r for c in clocks_all for r in c.get("reasons", [])})
        kernel_key = f"lm_head_{path}"
        line = {
            "metric": METRIC,
            "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": round(ms / a.steps, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f32 activations x packed int weights (f32 accumulate)" if path == "f32"
                     else "int8 activations (Q8, per-256 scale) x packed int weights",
            "data": "synthetic (seeded N(0,0.02) weights packed by hy_mt_rs_b200.synth; N(0,1) activations)",
            "config": decode_config(a, world),
            "roofline": {"bound": "hbm", "kernel": f"lm_head Q6_K {path} GEMV", "achieved": round(achieved, 1),
                         "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": profile_traffic(kernel_key),
                         "algorithmic_bytes_per_launch": lm_bytes, "avg_launch_ms": round(t_lm, 5)},
            "per_stage_ms": {"q2_0c_layer": round(t_q2, 5), "stq1_0_layer": round(t_stq, 5),
                             "q6k_lm_head": round(t_lm, 5)},
            "decode_tok_s_projection_only": {
                "q2_0c": round(1e3 / (N_LAYERS_MODEL * t_q2 + t_lm), 1),
                "stq1_0": round(1e3 / (N_LAYERS_MODEL * t_stq + t_lm), 1)},
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": 4 * HIDDEN,
                    "d2h_bytes_per_step": 4 * VOCAB, "ms_per_step": round(e2e_ms / e2e_steps, 5),
                    "how": "pinned host x -> device, graph-replayed public-API chain, logits -> pinned host, "
                           "stream sync per step"},
            "gpu_launches": launches_per_step * a.steps,
            "clocks": {"sm_mhz": statistics.median(sm) if sm else None,
                       "sm_max_mhz": clocks_all[0].get("sm_max_mhz"), "reasons": reasons,
                       "samples": sum(c.get("samples", 0) for c in clocks_all)},
        }
        if world == 1:
            line["cpu_baseline"] = run_cpu(a.cpu_seconds, VOCAB)
    for g in list(graphs.values()) + [g_lm] + full:
        del g
    graphs.clear()
    full.clear()
    return line if rank == 0 else None


# ---------------------------------------------------------------------------
# Prefill (config 3): one 7B decoder layer's projections at M tokens
# ---------------------------------------------------------------------------
LAYER_7B = [("attn_q", 4096, 4096, 2), ("attn_k", 1024, 4096, 2), ("attn_v", 1024, 4096, 2),
            ("attn_output", 4096, 4096, 2), ("ffn_gate", 14336, 4096, 2), ("ffn_up", 14336, 4096, 2),
            ("ffn_down", 4096, 14336, 3)]  # (name, N, K, dtype): Q4_K_M-style, Q6_K down


def gemm_launches(row_tiles, K, M, sms, dtype=2, split=False, pair=False):
    """Kernel launches of one batched product in libhyq (hyq_gemm.cu): the
    fp16 activation copy, the GEMM, and the split-K or tail reduction when
    it takes one (the library's rules, mirrored in hy_mt_rs_b200.quant)."""
    from hy_mt_rs_b200 import quant
    return quant.gemm_launches(row_tiles, K, M, dtype, sms, split=split, pair=pair)


def prefill_arm(a):
    import torch
    import torch.distributed as dist

    world, rank, dev = init_ranks()
    import hy_mt_rs_b200.quant  # noqa: F401  (loads libhyq.so or raises)
    from hy_mt_rs_b200 import quant, synth

    M = a.tokens
    ws = []
    for i, (name, N, K, t) in enumerate(LAYER_7B):
        ws.append(quant.Weight(synth.random_packed(t, N, K, seed=50 + i, device=dev), t, [K, N], name=name))
    xs = {K: torch.randn(M, K, generator=torch.Generator().manual_seed(K)).to(dev) for K in (4096, 14336)}
    flops = sum(2 * M * N * K for _, N, K, _ in LAYER_7B)
    wbytes = sum(N * row_bytes(t, K) for _, N, K, t in LAYER_7B)
    stream = torch.cuda.Stream(dev)
    outs = {}

    W = {w.name: w for w in ws}
    # the layer's calls as the reference makes them for a batch (model.rs:559-565
    # QKV, O, and DenseFfn::forward :678-683): QKV in one grouped launch, O,
    # gate/up with SiLU in one fused launch, down
    calls = {
        "attn_qkv": lambda: quant.Weight.matmul_qkv(W["attn_q"], W["attn_k"], W["attn_v"], xs[4096], M),
        "attn_output": lambda: W["attn_output"].matmul(xs[4096], M),
        "ffn_gate_up_silu": lambda: W["ffn_gate"].matmul_gate_up_silu_batch(W["ffn_up"], xs[4096], M),
        "ffn_down": lambda: W["ffn_down"].matmul(xs[14336], M),
    }

    def step():
        for name, f in calls.items():
            outs[name] = f()

    # fp16 operands (default), or split operands that agree with an f32 GEMM
    split = a.gemm_precision == "f32"
    quant.set_gemm_precision(quant.GEMM_F32 if split else quant.GEMM_FP16)
    sampler = ClockSampler("GPU-" + str(torch.cuda.get_device_properties(dev).uuid))
    with torch.cuda.stream(stream):
        for _ in range(a.warmup):
            step()
        stream.synchronize()
        # each call captured once and replayed, so that host-side work
        # (argument checks, tensor maps, workspace) stays out of the timing
        graphs = {}
        for name, f in calls.items():
            graphs[name] = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graphs[name], stream=stream):
                outs[name] = f()
        for g in graphs.values():
            g.replay()
        stream.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        sampler.start()
        per = {name: [] for name in calls}
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(a.steps):
            for name, g in graphs.items():
                b = torch.cuda.Event(enable_timing=True)
                c = torch.cuda.Event(enable_timing=True)
                b.record(stream)
                g.replay()
                c.record(stream)
                per[name].append((b, c))
        e1.record(stream)
    stream.synchronize()
    del graphs
    torch.cuda.synchronize(dev)
    sampler.stop()
    # e2e: every step copies its activations in from pinned host memory, runs
    # the layer's products through the public calls and reads the layer's
    # output (the down projection) back
    xh = {K: v.cpu().pin_memory() for K, v in xs.items()}
    yh = torch.empty(M, 4096).pin_memory()
    e2e_steps = max(5, a.steps // 2)
    with torch.cuda.stream(stream):
        for i in range(2 + e2e_steps):  # two untimed warm-up passes of the eager calls
            if i == 2:
                stream.synchronize()
                t0 = time.perf_counter()
            for K in xs:
                xs[K].copy_(xh[K], non_blocking=True)
            step()
            yh.copy_(outs["ffn_down"], non_blocking=True)
            stream.synchronize()
        e2e_s = (time.perf_counter() - t0) / e2e_steps
    h2d = sum(v.numel() * 4 for v in xs.values())
    quant.set_gemm_precision(quant.GEMM_FP16)
    if world > 1:
        dist.barrier()
    (ms_total, failed, e2e_s), clocks_all = reduce_over_ranks(
        [e0.elapsed_time(e1), device_failed(quant, dev), e2e_s], sampler.summary(), dev)
    if failed:
        raise RuntimeError("a kernel reported an expired bounded wait (device status word) on some rank")
    ms = ms_total / a.steps
    if rank != 0:
        return None
    sm = [c["sm_mhz"] for c in clocks_all if c.get("sm_mhz")]
    clocks = {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": clocks_all[0].get("sm_max_mhz"),
              "reasons": sorted({r for c in clocks_all for r in c.get("reasons", [])}),
              "samples": sum(c.get("samples", 0) for c in clocks_all)}
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    split = a.gemm_precision == "f32"
    pair = M >= 256 and not split  # O and down (single matrices, 4096 rows) on the 2-SM kernel
    launches = (gemm_launches(32 + 8 + 8, 4096, M, sms, split=split) + gemm_launches(32, 4096, M, sms, split=split,
                                                                                     pair=pair)
                + gemm_launches(14336 // 64, 4096, M, sms, split=split)
                + gemm_launches(32, 14336, M, sms, dtype=3, split=split, pair=pair)) * a.steps
    per_ms = {k: statistics.fmean(b.elapsed_time(c) for b, c in v) for k, v in per.items()}
    gate = per_ms["ffn_gate_up_silu"]
    gate_flops = 2 * 2 * M * 14336 * 4096
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except Exception:
        pass
    peak = float(peaks.get("bf16_tflops", 1590.0))
    line = {
        "metric": "prefill GEMM TFLOP/s (7B layer projections, Q4_K + Q6_K down, "
                  + ("split-operand f32-accurate tensor cores)" if split else "fp16 tensor cores)"),
        "value": round(job_rate(flops, 1, world, ms) / 1e12, 2), "unit": "TFLOP/s", "n_gpus": world,
        "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None,
        "dtype": "split fp16 operands (hi + lo / 2^11 of f32 weights and activations, 3 MMAs), f32 accumulate"
                 if split else "fp16 operands (decoded weights, activations), f32 accumulate",
        "data": "synthetic", "config": {"workload": f"hy-mt-rs config 3: 7B layer projections, M={M}",
                                        "tokens": M, "flops_per_step": flops, "weight_bytes": wbytes,
                                        "parallelism": f"replicas x{world} (independent token batches)"},
        "roofline": {"bound": "tensor", "kernel": "ffn gate/up + SiLU, Q4_K 2 x 14336x4096 GEMM",
                     "achieved": round(gate_flops / (gate * 1e-3) / 1e12, 2), "peak": peak,
                     "peak_kind": "measured" if peaks else "fallback", "unit": "TFLOP/s",
                     "frac": round(gate_flops / (gate * 1e-3) / 1e12 / peak, 4),
                     "traffic": profile_traffic(f"gemm_gate_up_m{M}" + ("_f32" if split else "")),
                     "avg_launch_ms": round(gate, 5)},
        "per_projection_ms": {k: round(v, 5) for k, v in per_ms.items()},
        "prefill_tok_s_layer": round(job_rate(M, 1, world, ms), 1),
        "e2e": {"value": round(job_rate(flops, 1, world, e2e_s * 1e3) / 1e12, 2), "unit": "TFLOP/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": M * 4096 * 4,
                "how": "each step: both activation matrices in from pinned host memory, the four layer calls, "
                       "the down projection's output back"},
        "gpu_launches": launches,
        "clocks": clocks,
    }
    if world == 1 and a.cpu_seconds > 0:
        line["cpu_baseline"] = prefill_cpu(M)
    return line


def prefill_cpu(M):
    """CPU baseline of config 3: the reference's batch >= 8 path
    (quant.rs:272-343) -- every projection's rows decoded to f32 (the oracle's
    decoders, all host threads), then an f32 GEMM (numpy's BLAS, all host
    threads, standing in for Candle's gemm crate) -- for the 7B layer's four
    calls at M tokens, once."""
    import numpy as np

    from hy_mt_rs_b200 import synth
    from oracle import oracle as O

    threads = host_threads()
    ws = [(N, K, t, synth.random_packed(t, N, K, seed=50 + i).numpy()) for i, (_, N, K, t) in enumerate(LAYER_7B)]
    xs = {K: np.random.default_rng(K).standard_normal((M, K)).astype(np.float32) for K in (4096, 14336)}
    flops = sum(2 * M * N * K for N, K, _, _ in ws)
    t0 = time.perf_counter()
    for N, K, t, w in ws:
        wd = O.decode_rows(t, w, K, N, threads)
        np.matmul(xs[K], wd.T)
    el = time.perf_counter() - t0
    return {"value": round(flops / el / 1e12, 4), "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"the 7B layer's seven products at M={M} once ({el:.2f} s): oracle decoders + numpy f32 "
                      f"GEMM (BLAS) in place of Candle's"}


# ---------------------------------------------------------------------------
# Single products (config 1, and every format at two sizes with --sweep)
# ---------------------------------------------------------------------------
FMT_NAMES = {2: "Q4_K", 3: "Q6_K", 4: "Q8_0", 5: "Q2_0C", 6: "STQ1_0"}


def time_products(dtype, N, K, path, dev, min_bytes=256 << 20, reps=1000, seed=0):
    """Batch-1 products over enough distinct weight copies that their bytes
    exceed L2 twice over, replayed from one CUDA graph (one launch per copy)
    until `reps` products ran.  Returns (bytes per product, mean ms per
    product, copies)."""
    import torch
    from hy_mt_rs_b200 import quant, synth

    one = gemv_bytes(dtype, N, K)
    copies = max(2, -(-min_bytes // (N * row_bytes(dtype, K))))
    ws = [quant.Weight(synth.random_packed(dtype, N, K, seed=seed + c, device=dev), dtype, [K, N])
          for c in range(copies)]
    x = torch.randn(K, generator=torch.Generator().manual_seed(seed)).to(dev)
    ys = [torch.empty(N, device=dev) for _ in range(copies)]
    torch.cuda.synchronize(dev)
    quant.set_launch_overlap(True)
    stream = torch.cuda.Stream(dev)

    def run():
        for w, y in zip(ws, ys):
            if path == "f32":
                quant.check(quant.lib.hyq_matmul(w.handle, quant._ptr(x), 1, quant._ptr(y), quant._stream(dev)))
            else:
                w.gemv_int8(x, out=y)

    with torch.cuda.stream(stream):
        run()
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            run()
        rounds = max(1, -(-reps // copies))
        for _ in range(3):
            g.replay()
        stream.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(rounds):
            g.replay()
        e1.record(stream)
        stream.synchronize()
    ms = e0.elapsed_time(e1) / (rounds * copies)
    if quant.device_status(dev) != 0:
        raise RuntimeError("device status word set")
    del g
    return one, ms, copies


def gemv_e2e(dev, n=300):
    """Config 1 through the public call with host buffers: every product
    copies x in from pinned host memory, runs hyq_matmul on the next of
    several weight copies (> L2 in total) and reads y back, synchronizing."""
    import torch
    from hy_mt_rs_b200 import quant, synth

    N, K = 6144, 2048
    copies = max(2, -(-(256 << 20) // (N * row_bytes(2, K))))
    ws = [quant.Weight(synth.random_packed(2, N, K, seed=c, device=dev), 2, [K, N]) for c in range(copies)]
    xh = torch.randn(K, generator=torch.Generator().manual_seed(5)).pin_memory()
    yh = torch.empty(N).pin_memory()
    xd, yd = torch.empty(K, device=dev), torch.empty(N, device=dev)
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        for i in range(3 + n):
            if i == 3:
                stream.synchronize()
                t0 = time.perf_counter()
            xd.copy_(xh, non_blocking=True)
            ws[i % copies].matmul(xd, 1, out=yd)
            yh.copy_(yd, non_blocking=True)
            stream.synchronize()
        el = time.perf_counter() - t0
    return {"value": round(n * gemv_bytes(2, N, K) / el / 1e9, 1), "unit": "GB/s", "h2d_bytes_per_step": 4 * K,
            "d2h_bytes_per_step": 4 * N, "ms_per_step": round(el / n * 1e3, 5),
            "how": "pinned host x -> device, hyq_matmul (batch 1) over rotating weight copies, y -> pinned host, "
                   "stream sync per product"}


def gemv_cpu(seconds=3.0):
    """The oracle port of the reference's x86 f32 Q4_K product on all host
    threads, for about `seconds`."""
    import numpy as np

    from hy_mt_rs_b200 import synth
    from oracle import oracle as O

    N, K = 6144, 2048
    w = synth.random_packed(2, N, K, seed=0).numpy()
    x = np.random.default_rng(0).standard_normal(K).astype(np.float32)
    threads = host_threads()
    O.matmul(2, w, K, N, x, 1, threads)
    n, t0 = 0, time.perf_counter()
    while n == 0 or time.perf_counter() - t0 < seconds:
        O.matmul(2, w, K, N, x, 1, threads)
        n += 1
    el = time.perf_counter() - t0
    return {"value": round(n * gemv_bytes(2, N, K) / el / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{n} Q4_K 6144x2048 products ({el:.1f} s); oracle/hyq_oracle.c x86 f32 order, OpenMP"}


def gemv_arm(a):
    import torch

    world, rank, dev = init_ranks()
    import hy_mt_rs_b200.quant  # noqa: F401  (loads libhyq.so or raises)

    peak, peak_kind = measured_peaks()
    sampler = ClockSampler("GPU-" + str(torch.cuda.get_device_properties(dev).uuid))
    sampler.start()
    res = {}
    for path in ("f32", "int8"):
        b, ms, copies = time_products(2, 6144, 2048, path, dev)
        res[path] = {"gb_s": round(b / (ms * 1e-3) / 1e9, 1), "us_per_product": round(ms * 1e3, 3),
                     "frac_of_hbm": round(b / (ms * 1e-3) / 1e9 / peak, 4), "copies": copies}
    sweep = {}
    if a.sweep:
        for t in (2, 3, 4, 5, 6):
            for N in (6144, 120832):
                for path in ("f32", "int8"):
                    b, ms, copies = time_products(t, N, 2048, path, dev, seed=10 * t)
                    sweep[f"{FMT_NAMES[t]} {N}x2048 {path}"] = {
                        "gb_s": round(b / (ms * 1e-3) / 1e9, 1), "us": round(ms * 1e3, 2),
                        "frac_of_hbm": round(b / (ms * 1e-3) / 1e9 / peak, 4)}
    sampler.stop()
    clocks = sampler.summary()
    f32 = res["f32"]
    b = gemv_bytes(2, 6144, 2048)
    line = {
        "metric": "quantized GEMV HBM GB/s (config 1: Q4_K 6144x2048, batch 1)",
        "value": f32["gb_s"], "unit": "GB/s", "n_gpus": 1, "steps": 1000, "warmup": 3,
        "ms_per_step": round(f32["us_per_product"] / 1e3, 6), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32 activations x packed int weights (exact int32 dp4a)",
        "data": "synthetic (seeded N(0,0.02) weights packed by hy_mt_rs_b200.synth; N(0,1) activations)",
        "config": {"workload": "hy-mt-rs config 1: Q4_K 6144x2048 batch-1 product, 1000 products",
                   "l2": f"{f32['copies']} distinct weight copies rotate (> 2 x L2), one CUDA graph",
                   "launch_overlap": True},
        "paths": res,
        "roofline": {"bound": "hbm", "kernel": "Q4_K 6144x2048 f32 GEMV", "achieved": f32["gb_s"], "peak": peak,
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": f32["frac_of_hbm"],
                     "traffic": profile_traffic("gemv_q4k_6144x2048_f32"),
                     "algorithmic_bytes_per_launch": b, "avg_launch_ms": round(f32["us_per_product"] / 1e3, 6)},
        "gpu_launches": 1000,
        "clocks": {"sm_mhz": clocks.get("sm_mhz"), "sm_max_mhz": clocks.get("sm_max_mhz"),
                   "reasons": clocks.get("reasons", []), "samples": clocks.get("samples", 0)},
    }
    if sweep:
        line["sweep"] = sweep
    line["e2e"] = gemv_e2e(dev)
    if rank == 0:
        if world == 1 and a.cpu_seconds > 0:
            line["cpu_baseline"] = gemv_cpu(min(a.cpu_seconds, 5.0))
        return line


# ---------------------------------------------------------------------------
# Tensor parallelism over the 7B layer (config 3 shapes), one process per GPU
# ---------------------------------------------------------------------------
TP_COL = ("attn_q", "attn_k", "attn_v", "ffn_gate", "ffn_up")  # split output rows
TP_ROW = ("attn_output", "ffn_down")                               # split input columns + all-reduce


def tp_arm(a):
    """Dense tensor parallelism of one 7B decoder layer's projections: QKV and
    gate/up column-parallel, O and down row-parallel with an all-reduce of the
    partial outputs (NCCL).  Every rank builds the full layer from the same
    seeds and keeps its shards, so the job equals the one-GPU layer."""
    import torch
    import torch.distributed as dist

    world, rank, dev = init_ranks()
    import hy_mt_rs_b200.quant  # noqa: F401  (loads libhyq.so or raises)
    from hy_mt_rs_b200 import quant, synth

    full = {}
    for i, (name, N, K, t) in enumerate(LAYER_7B):
        full[name] = quant.Weight(synth.random_packed(t, N, K, seed=50 + i, device=dev), t, [K, N], name=name)
    sh = {n: (w.shard(0, rank, world) if n in TP_COL else w.shard(1, rank, world)) for n, w in full.items()}
    for n in TP_ROW:
        del full[n]  # row shards are copies
    torch.cuda.synchronize(dev)
    quant.set_launch_overlap(a.tp_mode == "decode")
    H, F = 4096, 14336
    stream = torch.cuda.Stream(dev)
    ar = None
    if a.tp_mode == "decode":
        M = 1
        x = torch.randn(H, generator=torch.Generator().manual_seed(1)).to(dev)
        o = torch.empty(H, device=dev)
        h = torch.empty(H, device=dev)
        use_peer = world > 1 and a.tp_allreduce == "peer"
        if use_peer:
            from hy_mt_rs_b200.peer import PeerAllReduce
            ar = PeerAllReduce(H, device=dev)

        def step():
            q, k, v = quant.Weight.gemv_qkv(sh["attn_q"], sh["attn_k"], sh["attn_v"], x)
            # attention output stands in as q (same shard width); the
            # row-parallel partials go straight into the all-reduce buffer
            if use_peer:
                sh["attn_output"].matmul(q, 1, out=ar.partial)
                ar.allreduce(o)
            else:
                sh["attn_output"].matmul(q, 1, out=o)
                if world > 1:
                    dist.all_reduce(o)
            g = sh["ffn_gate"].matmul_gate_up_silu(sh["ffn_up"], o)
            if use_peer:
                sh["ffn_down"].matmul(g, 1, out=ar.partial)
                ar.allreduce(h)
            else:
                sh["ffn_down"].matmul(g, 1, out=h)
                if world > 1:
                    dist.all_reduce(h)
            return h
        flops = 2 * sum(N * K for _, N, K, _ in LAYER_7B)
    else:
        M = a.tokens
        xs = {H: torch.randn(M, H, generator=torch.Generator().manual_seed(H)).to(dev),
              F // world: torch.randn(M, F // world, generator=torch.Generator().manual_seed(F)).to(dev),
              H // world: torch.randn(M, H // world, generator=torch.Generator().manual_seed(7)).to(dev)}

        def step():
            for n in ("attn_q", "attn_k", "attn_v", "ffn_gate", "ffn_up"):
                sh[n].matmul(xs[H], M)
            o = sh["attn_output"].matmul(xs[H // world], M)
            d = sh["ffn_down"].matmul(xs[F // world], M)
            if world > 1:
                dist.all_reduce(o)
                dist.all_reduce(d)
            return d
        flops = 2 * M * sum(N * K for _, N, K, _ in LAYER_7B)
    wbytes = sum(N * row_bytes(t, K) for _, N, K, t in LAYER_7B)
    with torch.cuda.stream(stream):
        for _ in range(a.warmup):
            step()
        stream.synchronize()
        graph = None
        if a.tp_mode == "decode":
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                step()
            for _ in range(3):
                graph.replay()
            stream.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(a.steps):
            graph.replay() if graph is not None else step()
        e1.record(stream)
        stream.synchronize()
    failed = device_failed(quant, dev)
    (ms_total, failed), _ = reduce_over_ranks([e0.elapsed_time(e1), failed], {}, dev)
    if failed:
        raise RuntimeError("a kernel reported an expired bounded wait (device status word) on some rank")
    ms = ms_total / a.steps
    del graph
    if ar is not None:
        ar.close()
    if world > 1:
        dist.barrier()
    if rank != 0:
        return None
    if a.tp_mode == "decode":
        line = {"metric": "7B layer projections, batch-1 decode, tensor-parallel: weight GB/s",
                "value": round(wbytes / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "layer_us": round(ms * 1e3, 3), "dtype": "f32 activations x packed int weights"}
    else:
        line = {"metric": f"7B layer GEMMs at M={M}, tensor-parallel: TFLOP/s",
                "value": round(flops / (ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                "layer_us": round(ms * 1e3, 3), "dtype": "fp16 operands, f32 accumulate"}
    line.update({"n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms, 5),
                 "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "data": "synthetic",
                 "config": {"workload": f"hy-mt-rs config 3 shapes, TP={world} ({a.tp_mode})", "tokens": M,
                            "parallelism": f"tp{world}: QKV, gate/up column-parallel; O, down row-parallel "
                                           f"+ all-reduce ({'NCCL' if (a.tp_mode == 'prefill' or a.tp_allreduce == 'nccl') else 'hyq_peer_allreduce over NVLink peer memory'})",
                            "weight_bytes": wbytes}})
    return line


# ---------------------------------------------------------------------------
# Full-model greedy decode (config 4): random-init 1.8B architecture
# ---------------------------------------------------------------------------
def model_arm(a):
    if a.concurrency > 1:
        return batch_arm(a)
    import numpy as np
    import torch

    world, rank, dev = init_ranks()
    import hy_mt_rs_b200.quant  # noqa: F401  (loads libhyq.so or raises)
    from hy_mt_rs_b200 import quant
    from hy_mt_rs_b200.model import DenseConfig, DenseModel, random_weights

    n_prompt, n_new = 256, 256
    cfg = DenseConfig(layers=N_LAYERS_MODEL, positions=n_prompt + n_new)
    weights = random_weights(cfg, dev, seed=1)
    torch.cuda.synchronize(dev)
    # the prompt's batched products: split operands (f32-accurate, the
    # parity-tested setting) unless fp16 is asked for
    prec = quant.GEMM_FP16 if a.gemm_precision == "fp16" else quant.GEMM_F32
    kv16 = a.kv16 and not a.model_fused
    q8 = a.activations == "q8" and not a.model_fused
    model = DenseModel(cfg, weights, dev, fused=a.model_fused, gemm_precision=prec, kv16=kv16,
                       activations="q8" if q8 else "f32")
    stream = torch.cuda.Stream(dev)
    model.capture(stream)
    prompt = np.random.default_rng(0).integers(0, cfg.vocab, n_prompt).tolist()
    ids = torch.tensor(prompt, dtype=torch.int32).to(dev)
    sampler = ClockSampler("GPU-" + str(torch.cuda.get_device_properties(dev).uuid))
    e0, e1, e1b, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(4))
    with torch.cuda.stream(stream):
        for _ in range(max(3, a.warmup)):
            model.graph.replay()
        # the prompt's kernels once untimed (a kernel's first launch loads its module)
        model.reset()
        for c0 in range(0, n_prompt, model.chunk):
            model.prefill(ids[c0:c0 + model.chunk])
        model.reset()
        e0.record(stream)
        for c0 in range(0, n_prompt, model.chunk):  # the prompt: batched forwards (model.rs:549-646)
            model.prefill(ids[c0:c0 + model.chunk])
        e1.record(stream)
        stream.synchronize()
        sampler.start()
        e1b.record(stream)
        for _ in range(n_new - 1):
            model.graph.replay()
        e2.record(stream)
        stream.synchronize()
        sampler.stop()
        # e2e: the serving loop reads every new token back to the host
        model.reset()
        for c0 in range(0, n_prompt, model.chunk):
            model.prefill(ids[c0:c0 + model.chunk])
        # one step of lookahead: step i+1 is enqueued before the host waits
        # for token i, as a streaming server does (it stops on a token it
        # has read, one step late)
        tok_host = torch.empty(n_new, dtype=torch.int32).pin_memory()
        done = [torch.cuda.Event() for _ in range(n_new)]
        got = []
        stream.synchronize()  # the prompt steps are not part of the decode rate
        t0 = time.perf_counter()
        for i in range(n_new - 1):
            model.graph.replay()
            tok_host[i:i + 1].copy_(model.token, non_blocking=True)
            done[i].record(stream)
            if i:
                done[i - 1].synchronize()
                got.append(int(tok_host[i - 1]))
        done[n_new - 2].synchronize()
        got.append(int(tok_host[n_new - 2]))
        e2e_s = time.perf_counter() - t0
        # one whole request from the host: prompt ids in, batched prefill,
        # n_new - 1 greedy steps, every token read back
        ids_host = torch.tensor(prompt, dtype=torch.int32).pin_memory()
        ids_dev = torch.empty_like(ids_host, device=dev)
        stream.synchronize()
        t0 = time.perf_counter()
        model.reset()
        ids_dev.copy_(ids_host, non_blocking=True)
        for c0 in range(0, n_prompt, model.chunk):
            model.prefill(ids_dev[c0:c0 + model.chunk])
        for i in range(n_new - 1):
            model.graph.replay()
            tok_host[i:i + 1].copy_(model.token, non_blocking=True)
            done[i].record(stream)
            if i:
                done[i - 1].synchronize()
        done[n_new - 2].synchronize()
        request_s = time.perf_counter() - t0
    failed = device_failed(quant, dev)
    (ms_decode, ms_prompt, failed), clocks_all = reduce_over_ranks(
        [e1b.elapsed_time(e2), e0.elapsed_time(e1), failed + 0.0], sampler.summary(), dev)
    if failed:
        raise RuntimeError("a kernel reported an expired bounded wait (device status word) on some rank")
    model_launches = model.launches()
    model.graph = None
    if rank != 0:
        return None
    steps = n_new - 1
    tok_s = steps / (ms_decode * 1e-3) * world
    token_bytes = N_LAYERS_MODEL * sum(N * row_bytes(5, K) for _, N, K in LAYER) + VOCAB * row_bytes(3, HIDDEN)
    peak, peak_kind = measured_peaks()
    cpu = model_cpu(cfg, weights, prompt, "q8" if q8 else "f32") if world == 1 and a.cpu_seconds > 0 else None
    sm = [c["sm_mhz"] for c in clocks_all if c.get("sm_mhz")]
    line = {
        "metric": "decode tokens/s (random-init Hy-MT2-1.8B architecture, Q2_0C linears, Q6_K tied embedding, "
                  "batch 1, greedy)",
        "value": round(tok_s, 1), "unit": "tokens/s", "n_gpus": world, "steps": steps, "warmup": max(3, a.warmup),
        "ms_per_step": round(ms_decode / steps, 4), "higher_is_better": True, "scaling": "weak",
        # the reference's published 1.8B Q2_0C decode rate, one request on an M2 Pro
        # (docs/validation.md:70-71 of hy-mt-rs)
        "vs_baseline": round(tok_s / 86.86, 2), "vs_baseline_number": "86.86 tokens/s, 1.8B Q2_0C, 1 request",
        "dtype": ("Q8 activations (the reference's aarch64 SDOT branch)" if q8 else "f32 activations")
                 + " x packed int weights; " + ("f16" if kv16 else "f32") + " KV cache; prompt products "
                 + ("fp16 tensor-core operands" if prec == quant.GEMM_FP16 else "split-operand f32-accurate"),
        "data": "synthetic (seeded random-init weights, 256 seeded random prompt ids)",
        "config": {"workload": "hy-mt-rs config 4: 32 layers, hidden 2048, 16/4 heads x 128, SwiGLU 6144, "
                               "vocab 120832, RoPE 10000; 256-token prompt (batched prefill), 256 generated",
                   "concurrency": 1, "positions": cfg.positions, "launch_overlap": True,
                   "kv_cache": "f16" if kv16 else "f32",
                   "step": "one persistent kernel per token (hyq_dense_step)" if a.model_fused
                   else (f"per-kernel CUDA graph ({model_launches} launches per token, programmatic dependent "
                         "launch" + (", norms and residual adds inside the products)" if model.fuse_norms else ")")),
                   "parallelism": f"replicas x{world}"},
        "prompt_ms": round(ms_prompt, 2),
        "prompt": "256 tokens in one batched forward (tensor-core projections, causal attention)",
        "request_ms": round(request_s * 1e3, 2),
        "weight_gb_s": round(token_bytes / (ms_decode / steps * 1e-3) / 1e9, 1),
        "roofline": {"bound": "hbm", "kernel": "whole decode step (weights per token)", "unit": "GB/s",
                     "achieved": round(token_bytes / (ms_decode / steps * 1e-3) / 1e9, 1), "peak": peak,
                     "peak_kind": peak_kind, "frac": round(token_bytes / (ms_decode / steps * 1e-3) / 1e9 / peak, 4),
                     "traffic": None, "algorithmic_bytes_per_launch": token_bytes},
        "e2e": {"value": round(steps / e2e_s, 1), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 4, "how": "graph replay per token, each token read back to the host one step late"},
        "gpu_launches": steps * model_launches,
        "clocks": {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": clocks_all[0].get("sm_max_mhz"),
                   "reasons": sorted({r for c in clocks_all for r in c.get("reasons", [])}),
                   "samples": sum(c.get("samples", 0) for c in clocks_all)},
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    return line


def model_cpu(cfg, weights, prompt, activations="f32"):
    """CPU baseline of config 4: the oracle's single-token step (the
    reference's x86 decode path, or with activations "q8" its aarch64 SDOT
    path, oracle/model.py) of the same model on all host threads, a bounded
    sample of steps; one request (the reference serves concurrent requests
    as separate sessions on the same cores)."""
    import dataclasses

    from oracle.model import DenseOracle

    oracle = DenseOracle(dataclasses.replace(cfg, positions=8), weights, threads=host_threads(),
                         activations=activations)
    t0 = time.perf_counter()
    n = 0
    while n < 8 and (n == 0 or time.perf_counter() - t0 < 20.0):
        oracle.step(prompt[n], n)
        n += 1
    el = time.perf_counter() - t0
    return {"value": round(n / el, 3), "unit": "tokens/s", "cores": host_threads(), "kind": "port",
            "sample": f"{n} decode steps of one request of the same model through oracle/model.py ("
                      + ("Q8 activations, SDOT order" if activations == "q8" else "x86 f32 order")
                      + f", OpenMP over all host threads; {el:.1f} s)"}


def batch_arm(a):
    """Config 4 at concurrency B: B independent requests (256-token prompts,
    256 generated each) decoded together, one token of every request per
    step (DenseBatch, one CUDA graph per step)."""
    import numpy as np
    import torch

    world, rank, dev = init_ranks()
    import hy_mt_rs_b200.quant  # noqa: F401  (loads libhyq.so or raises)
    from hy_mt_rs_b200 import quant
    from hy_mt_rs_b200.model import DenseBatch, DenseConfig, DenseModel, random_weights

    B, n_prompt, n_new = a.concurrency, 256, 256
    cfg = DenseConfig(layers=N_LAYERS_MODEL, positions=n_prompt + n_new)
    weights = random_weights(cfg, dev, seed=1)
    torch.cuda.synchronize(dev)
    # the batched products: split operands (f32-accurate; the setting whose
    # token streams the parity tests pin to the oracle) unless fp16 is asked for
    prec = quant.GEMM_FP16 if a.gemm_precision == "fp16" else quant.GEMM_F32
    model = DenseModel(cfg, weights, dev, gemm_precision=prec, kv16=a.kv16)
    batch = DenseBatch(model, B)
    stream = torch.cuda.Stream(dev)
    batch.capture(stream)
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, cfg.vocab, n_prompt).tolist() for _ in range(B)]
    sampler = ClockSampler("GPU-" + str(torch.cuda.get_device_properties(dev).uuid))
    e0, e1, e1b, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(4))
    with torch.cuda.stream(stream):
        for _ in range(max(3, a.warmup)):
            batch.graph.replay()
        batch.reset()
        ids = [torch.tensor(p, dtype=torch.int32).to(dev) for p in prompts]
        stream.synchronize()
        e0.record(stream)
        for b in range(B):   # each request's prompt: batched forwards into its cache slice
            caches = [(k[b], v[b]) for k, v in batch.caches]
            for c0 in range(0, n_prompt, model.chunk):
                model.prefill(ids[b][c0:c0 + model.chunk], caches=caches, pos=batch.pos[b:b + 1],
                              token_out=batch.tokens[b:b + 1], logits=batch.logits[b])
        e1.record(stream)
        stream.synchronize()
        sampler.start()
        e1b.record(stream)
        for _ in range(n_new - 1):
            batch.graph.replay()
        e2.record(stream)
        stream.synchronize()
        sampler.stop()
        # e2e: every step's B tokens read back to the host, one step late
        batch.reset()
        batch.prefill_all(prompts)
        tok_host = torch.empty(n_new, B, dtype=torch.int32).pin_memory()
        done = [torch.cuda.Event() for _ in range(n_new)]
        stream.synchronize()
        t0 = time.perf_counter()
        for i in range(n_new - 1):
            batch.graph.replay()
            tok_host[i].copy_(batch.tokens, non_blocking=True)
            done[i].record(stream)
            if i:
                done[i - 1].synchronize()
        done[n_new - 2].synchronize()
        e2e_s = time.perf_counter() - t0
    failed = device_failed(quant, dev)
    (ms_decode, ms_prompt, failed), clocks_all = reduce_over_ranks(
        [e1b.elapsed_time(e2), e0.elapsed_time(e1), failed + 0.0], sampler.summary(), dev)
    if failed:
        raise RuntimeError("a kernel reported an expired bounded wait (device status word) on some rank")
    step_launches = batch.launches()
    batch.graph = None
    if rank != 0:
        return None
    steps = n_new - 1
    tok_s = B * steps / (ms_decode * 1e-3) * world
    weight_bytes = N_LAYERS_MODEL * sum(N * row_bytes(5, K) for _, N, K in LAYER) + VOCAB * row_bytes(3, HIDDEN)
    # KV cache bytes a step reads (K and V rows, f32 or f16, of every visible position
    # of every request) and writes (one row pair per request), per layer
    kv_row = 2 * cfg.kv_heads * cfg.head_dim * (2 if a.kv16 else 4)
    visible = sum(n_prompt + i + 1 for i in range(1, n_new)) / steps
    kv_bytes = N_LAYERS_MODEL * B * (visible + 1) * kv_row
    step_bytes = weight_bytes + kv_bytes
    step_s = ms_decode / steps * 1e-3
    peak, peak_kind = measured_peaks()
    sm = [c["sm_mhz"] for c in clocks_all if c.get("sm_mhz")]
    cpu = model_cpu(cfg, weights, prompts[0]) if world == 1 and a.cpu_seconds > 0 else None
    line = {
        "metric": f"decode tokens/s (random-init Hy-MT2-1.8B architecture, Q2_0C linears, Q6_K tied embedding, "
                  f"{B} concurrent requests, greedy)",
        "value": round(tok_s, 1), "unit": "tokens/s", "n_gpus": world, "steps": steps, "warmup": max(3, a.warmup),
        "ms_per_step": round(ms_decode / steps, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32 activations; "
                 + ("fp16 tensor-core operands" if prec == quant.GEMM_FP16
                    else "split-operand f32-accurate tensor-core products (3 MMAs per K chunk)")
                 + " of the dequantized weights; " + ("f16" if a.kv16 else "f32") + " KV cache",
        "data": f"synthetic (seeded random-init weights, {B} seeded random 256-token prompts)",
        "config": {"workload": "hy-mt-rs config 4: 32 layers, hidden 2048, 16/4 heads x 128, SwiGLU 6144, "
                               "vocab 120832, RoPE 10000; 256-token prompts (batched prefill), 256 generated each",
                   "concurrency": B, "positions": cfg.positions, "kv_cache": "f16" if a.kv16 else "f32",
                   "parallelism": f"replicas x{world}"},
        "prompt_ms": round(ms_prompt, 2),
        "prompt": f"{B} prompts of 256 tokens, one batched forward each",
        "roofline": {"bound": "hbm", "kernel": "whole decode step (weights + KV cache per step)", "unit": "GB/s",
                     "achieved": round(step_bytes / step_s / 1e9, 1), "peak": peak, "peak_kind": peak_kind,
                     "frac": round(step_bytes / step_s / 1e9 / peak, 4), "traffic": None,
                     "algorithmic_bytes_per_launch": int(step_bytes), "weight_bytes": weight_bytes,
                     "kv_bytes": int(kv_bytes)},
        "e2e": {"value": round(B * steps / e2e_s, 1), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 4 * B, "how": "graph replay per step, each step's tokens read back one step late"},
        "gpu_launches": steps * step_launches,
        "clocks": {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": clocks_all[0].get("sm_max_mhz"),
                   "reasons": sorted({r for c in clocks_all for r in c.get("reasons", [])}),
                   "samples": sum(c.get("samples", 0) for c in clocks_all)},
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    return line


# ---------------------------------------------------------------------------
# Mixture-of-experts FFN (config 5): decode batch 64, prefill M = 1024
# ---------------------------------------------------------------------------
MOE_DECODE_TOKENS, MOE_PREFILL_TOKENS = 64, 1024


def moe_graph(layer, x, T, out, stream, world, dev):
    """Capture layer.forward(x, T, out) as one CUDA graph on `stream`; None
    (and eager calls) unless every rank captured it."""
    import torch
    import torch.distributed as dist

    graph = torch.cuda.CUDAGraph()
    try:
        with torch.cuda.graph(graph, stream=stream):
            layer.forward(x, T, out)
        ok = 1.0
    except Exception:
        graph, ok = None, 0.0
    torch.cuda.synchronize(dev)
    if world > 1:
        flag = torch.tensor([ok], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        ok = float(flag.item())
    if ok < 1.0:
        return None
    graph.replay()
    stream.synchronize()
    return graph


def moe_arm(a):
    import numpy as np
    import torch

    world, rank, dev = init_ranks()
    import hy_mt_rs_b200.quant  # noqa: F401  (loads libhyq.so or raises)
    from hy_mt_rs_b200 import quant
    from hy_mt_rs_b200.moe import MoeConfig, MoeLayer, random_moe_weights

    cfg = MoeConfig()
    weights = random_moe_weights(cfg, dev, seed=3)
    # N > 1: expert parallelism (each rank E / N experts and its own tokens), rows
    # exchanged through NVLink peer memory (hyq_peer_exchange) or NCCL all-to-all
    xchg = None
    if world > 1 and getattr(a, "ep_exchange", "peer") == "peer":
        from hy_mt_rs_b200.peer import PeerExchange
        xchg = PeerExchange((MOE_PREFILL_TOKENS * cfg.used + 1) * cfg.hidden, device=dev)
    layer = MoeLayer(cfg, weights, ep=(rank, world, None) if world > 1 else None, exchange=xchg)
    H, E, M, S, U = cfg.hidden, cfg.experts, cfg.mid, cfg.shared_mid, cfg.used
    expert_bytes = 3 * M * row_bytes(cfg.dtype, H)  # gate + up + down of one expert (same byte count)
    shared_bytes = 3 * S * row_bytes(cfg.dtype, H)
    stream = torch.cuda.Stream(dev)
    sampler = ClockSampler("GPU-" + str(torch.cuda.get_device_properties(dev).uuid))
    res = {}
    # The experts one step reads (those the router picks, about 100 MB with
    # the saturated N(0, 1) router) fit in L2, so L2 is flushed between timed
    # steps by writing a buffer twice its size, outside the timed events.
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    graphed = {}
    for T in (MOE_DECODE_TOKENS, MOE_PREFILL_TOKENS):
        x = torch.randn(T, H, generator=torch.Generator().manual_seed(T)).to(dev)
        out = torch.empty(T, H, device=dev)
        with torch.cuda.stream(stream):
            for _ in range(max(3, a.warmup)):
                layer.forward(x, T, out)
            stream.synchronize()
            # the layer as one CUDA graph (routing, counts and the expert
            # exchange stay on the device, so it captures), replayed per step;
            # every rank must capture, else all run the calls eagerly
            graph = moe_graph(layer, x, T, out, stream, world, dev)
            if T == MOE_DECODE_TOKENS:
                sampler.start()
            evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                   for _ in range(a.steps)]
            for b, c in evs:
                flush.fill_(1)
                b.record(stream)
                graph.replay() if graph is not None else layer.forward(x, T, out)
                c.record(stream)
            stream.synchronize()
            if T == MOE_DECODE_TOKENS:
                sampler.stop()
            off = layer._buffers(T, dev)["off"].cpu().numpy()
            # e2e: host activations in (pinned), the layer, host result out, every step
            xh = x.cpu().pin_memory()
            oh = torch.empty(T, H).pin_memory()
            xd = torch.empty_like(x)
            torch.cuda.synchronize(dev)
            t0 = time.perf_counter()
            for _ in range(a.steps):
                (x if graph is not None else xd).copy_(xh, non_blocking=True)
                graph.replay() if graph is not None else layer.forward(xd, T, out)
                oh.copy_(out, non_blocking=True)
                stream.synchronize()
            e2e_s = (time.perf_counter() - t0) / a.steps
            graphed[T] = graph is not None
            del graph
        hit = int((np.diff(off) > 0).sum())
        res[T] = {"ms": statistics.fmean(b.elapsed_time(c) for b, c in evs), "e2e_s": e2e_s, "experts_hit": hit,
                  "bytes": hit * expert_bytes + shared_bytes + E * H * 4,
                  "flops": 2 * T * (U * 3 * M * H + 3 * S * H + E * H)}
    failed = device_failed(quant, dev)
    (ms_dec, ms_pre, failed), clocks_all = reduce_over_ranks(
        [res[MOE_DECODE_TOKENS]["ms"], res[MOE_PREFILL_TOKENS]["ms"], failed + 0.0], sampler.summary(), dev)
    if xchg is not None:
        xchg.close()  # every rank, after the graphs that use the regions are gone
    if failed:
        raise RuntimeError("a kernel reported an expired bounded wait (device status word) on some rank")
    launches = layer.launches(MOE_DECODE_TOKENS) * a.steps
    if rank != 0:
        return None
    dec, pre = res[MOE_DECODE_TOKENS], res[MOE_PREFILL_TOKENS]
    peak, peak_kind = measured_peaks()
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except Exception:
        pass
    tpeak = float(peaks.get("bf16_tflops", 1590.0))
    gbs = dec["bytes"] / (ms_dec * 1e-3) / 1e9
    cpu_tok_s = None
    if world == 1 and a.cpu_seconds > 0:
        # CPU baseline: the oracle port of the reference's Moe::forward on a sample
        from oracle.moe import moe_forward_port
        wn = {k: v.cpu().numpy() for k, v in weights.items()}
        xs = np.random.default_rng(0).standard_normal((8, H)).astype(np.float32)
        t0 = time.perf_counter()
        moe_forward_port(cfg, wn, xs, host_threads())
        cpu_tok_s = xs.shape[0] / (time.perf_counter() - t0)
    sm = [c["sm_mhz"] for c in clocks_all if c.get("sm_mhz")]
    line = {
        "metric": "MoE FFN decode tokens/s (config 5: 64 experts top-8, 2048->1024->2048 Q4_K, batch 64)",
        "value": round(MOE_DECODE_TOKENS / (ms_dec * 1e-3) * world, 1), "unit": "tokens/s", "n_gpus": world,
        "steps": a.steps, "warmup": max(3, a.warmup), "ms_per_step": round(ms_dec, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": "fp16 tensor-core operands, f32 accumulate; f32 router and routing",
        "data": "synthetic (seeded N(0,1) F32 router, N(0,0.1) bias, N(0,0.02) Q4_K experts; N(0,1) activations)",
        "config": {"workload": "hy-mt-rs config 5: one MoE FFN (router, sigmoid top-8 routing, 64 experts "
                               "2048->1024->2048 SwiGLU Q4_K, shared expert 2048->1024->2048), batch 64",
                   "experts": E, "used": U,
                   "parallelism": (f"expert parallel x{world} ("
                                   + ("NVLink peer-memory exchange" if xchg is not None else "NCCL all-to-all") + ")")
                                  if world > 1 else "1 GPU",
                   "l2": "L2 flushed between timed steps (256 MB written outside the timed events)",
                   "step": "one CUDA graph of the layer" if graphed.get(MOE_DECODE_TOKENS) else "eager calls"},
        "prefill": {"tokens": MOE_PREFILL_TOKENS, "ms_per_step": round(ms_pre, 4),
                    "tokens_per_s": round(MOE_PREFILL_TOKENS / (ms_pre * 1e-3) * world, 1),
                    "tflops": round(pre["flops"] / (ms_pre * 1e-3) / 1e12, 2),
                    "frac_of_bf16": round(pre["flops"] / (ms_pre * 1e-3) / 1e12 / tpeak, 4)},
        "roofline": {"bound": "hbm", "kernel": "whole decode step (router + experts hit + shared expert bytes)",
                     "unit": "GB/s", "achieved": round(gbs, 1), "peak": peak, "peak_kind": peak_kind,
                     "frac": round(gbs / peak, 4), "traffic": None,
                     "algorithmic_bytes_per_launch": dec["bytes"], "experts_hit": dec["experts_hit"]},
        "e2e": {"value": round(MOE_DECODE_TOKENS / dec["e2e_s"], 1), "unit": "tokens/s",
                "h2d_bytes_per_step": MOE_DECODE_TOKENS * H * 4, "d2h_bytes_per_step": MOE_DECODE_TOKENS * H * 4},
        "gpu_launches": launches,
        "clocks": {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": clocks_all[0].get("sm_max_mhz"),
                   "reasons": sorted({r for c in clocks_all for r in c.get("reasons", [])}),
                   "samples": sum(c.get("samples", 0) for c in clocks_all)},
    }
    if cpu_tok_s is not None:
        line["cpu_baseline"] = {"value": round(cpu_tok_s, 3), "unit": "tokens/s", "cores": host_threads(),
                                "kind": "port",
                                "sample": "8 tokens through oracle/moe.py moe_forward_port (the reference's expert "
                                          "loop, x86 f32 order; f64 accumulation in the batch >= 8 products)"}
    return line


MOE_STACK_LAYERS = 8


def moe_stack_arm(a):
    """Config 5's layer stack: a random-init HyV3 decoder (model.rs:210-231,
    684-726) of MOE_STACK_LAYERS layers -- hidden 2048, attention 16 / 4 heads
    of 128, layer 0 a dense SwiGLU FFN of 6144, layers 1.. the MoE FFN (64
    experts top 8, 2048 -> 1024 -> 2048, shared expert 1024), Q4_K linears and
    experts, Q6_K embedding and output of 120832 -- decoding 64 requests
    (64-token prompts, 64 steps) and prefilling 1024 tokens (four 256-token
    chunks).  Split-operand products (the setting the HyV3 parity tests pin)."""
    import numpy as np
    import torch

    world, rank, dev = init_ranks()
    import hy_mt_rs_b200.quant  # noqa: F401  (loads libhyq.so or raises)
    from hy_mt_rs_b200 import quant
    from hy_mt_rs_b200.model import DenseBatch, DenseConfig, DenseModel, random_weights

    B, n_prompt, n_new, M = 64, 64, 64, 1024
    cfg = DenseConfig(arch="hyv3", layers=MOE_STACK_LAYERS, ffn=6144, linear_dtype=2, embed_dtype=3,
                      positions=M + 8)
    weights = random_weights(cfg, dev, seed=5)
    torch.cuda.synchronize(dev)
    model = DenseModel(cfg, weights, dev, gemm_precision=quant.GEMM_F32)
    stream = torch.cuda.Stream(dev)
    sampler = ClockSampler("GPU-" + str(torch.cuda.get_device_properties(dev).uuid))
    # ---- prefill: 1024 tokens of one request, the reference's 256-token chunks
    ids = torch.from_numpy(np.random.default_rng(5).integers(0, cfg.vocab, M).astype(np.int32)).to(dev)
    with torch.cuda.stream(stream):
        for _ in range(max(2, a.warmup)):
            model.reset()
            for c0 in range(0, M, model.chunk):
                model.prefill(ids[c0:c0 + model.chunk])
        stream.synchronize()
        evs = []
        for _ in range(3):
            model.reset()
            b, c = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            b.record(stream)
            for c0 in range(0, M, model.chunk):
                model.prefill(ids[c0:c0 + model.chunk])
            c.record(stream)
            evs.append((b, c))
        stream.synchronize()
    ms_prefill = statistics.fmean(b.elapsed_time(c) for b, c in evs)
    # ---- decode: 64 requests
    batch = DenseBatch(model, B)
    rng = np.random.default_rng(6)
    prompts = [rng.integers(0, cfg.vocab, n_prompt).tolist() for _ in range(B)]
    with torch.cuda.stream(stream):
        batch.capture(stream)
        batch.reset()
        batch.prefill_all(prompts)
        for _ in range(3):
            batch.graph.replay()
        batch.reset()
        batch.prefill_all(prompts)
        stream.synchronize()
        sampler.start()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(n_new - 1):
            batch.graph.replay()
        e1.record(stream)
        stream.synchronize()
        sampler.stop()
        # experts each MoE layer read in the last step (its routing)
        hit = [int((torch.diff(W["moe"]._buffers(B, dev)["off"]) > 0).sum()) for W in model.layers if "moe" in W]
        # e2e: every step's tokens read back to the host, one step late
        batch.reset()
        batch.prefill_all(prompts)
        tok_host = torch.empty(n_new, B, dtype=torch.int32).pin_memory()
        done = [torch.cuda.Event() for _ in range(n_new)]
        stream.synchronize()
        t0 = time.perf_counter()
        for i in range(n_new - 1):
            batch.graph.replay()
            tok_host[i].copy_(batch.tokens, non_blocking=True)
            done[i].record(stream)
            if i:
                done[i - 1].synchronize()
        done[n_new - 2].synchronize()
        e2e_s = time.perf_counter() - t0
    failed = device_failed(quant, dev)
    steps = n_new - 1
    (ms_decode, ms_prefill, failed), clocks_all = reduce_over_ranks([e0.elapsed_time(e1), ms_prefill, failed + 0.0],
                                                                     sampler.summary(), dev)
    if failed:
        raise RuntimeError("a kernel reported an expired bounded wait (device status word) on some rank")
    launches = batch.launches()
    batch.graph = None
    if rank != 0:
        return None
    H, A, KV = cfg.hidden, cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim
    attn_bytes = (A + 2 * KV) * row_bytes(2, H) + H * row_bytes(2, A)
    mc = cfg.moe_config()
    expert_bytes = 3 * mc.mid * row_bytes(2, H)
    moe_fixed = 3 * mc.shared_mid * row_bytes(2, H) + mc.experts * H * 4     # shared expert + F32 router
    dense_ffn = 3 * cfg.ffn * row_bytes(2, H)
    out_bytes = cfg.vocab * row_bytes(3, H)
    kv_row = 2 * KV * 4
    kv_bytes = cfg.layers * B * (n_prompt + n_new / 2) * kv_row
    step_bytes = (cfg.layers * attn_bytes + dense_ffn + sum(h * expert_bytes + moe_fixed for h in hit) + out_bytes
                  + kv_bytes)
    step_s = ms_decode / steps * 1e-3
    peak, peak_kind = measured_peaks()
    moe_layers = cfg.layers - 1
    flops_tok = 2 * (cfg.layers * (A + 2 * KV) * H + cfg.layers * H * A + 3 * cfg.ffn * H
                     + moe_layers * (mc.used * 3 * mc.mid * H + 3 * mc.shared_mid * H + mc.experts * H))
    sm = [c["sm_mhz"] for c in clocks_all if c.get("sm_mhz")]
    line = {
        "metric": f"MoE layer-stack decode tokens/s (config 5: {cfg.layers} HyV3 layers, 64 experts top-8, "
                  f"16/4 x 128 attention; 64 requests)",
        "value": round(B / step_s * world, 1), "unit": "tokens/s", "n_gpus": world, "steps": steps,
        "warmup": 3, "ms_per_step": round(ms_decode / steps, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None,
        "dtype": "split-operand f32-accurate tensor-core products (experts, batched projections); f32 KV cache",
        "data": "synthetic (seeded random-init HyV3 weights, N(0,1) F32 routers; seeded prompts)",
        "config": {"workload": f"hy-mt-rs config 5 layer stack: {cfg.layers} HyV3 layers (layer 0 dense FFN 6144, "
                               "layers 1.. MoE 64 experts top 8 2048->1024->2048 + shared 1024), attention 16/4 x "
                               "128 Q4_K, Q6_K embedding and output 120832; decode 64 requests with 64-token "
                               "prompts, prefill 1024 tokens",
                   "layers": cfg.layers, "concurrency": B, "parallelism": f"replicas x{world}"},
        "prefill": {"tokens": M, "ms": round(ms_prefill, 3), "tokens_per_s": round(M / (ms_prefill * 1e-3), 1),
                    "tflops": round(flops_tok * M / (ms_prefill * 1e-3) / 1e12, 2),
                    "how": "four 256-token batched forwards (model.rs:640-646), CUDA events"},
        "roofline": {"bound": "hbm", "kernel": "whole decode step (weights read + experts hit + KV cache)",
                     "unit": "GB/s", "achieved": round(step_bytes / step_s / 1e9, 1), "peak": peak,
                     "peak_kind": peak_kind, "frac": round(step_bytes / step_s / 1e9 / peak, 4), "traffic": None,
                     "algorithmic_bytes_per_launch": int(step_bytes), "experts_hit_per_layer": hit},
        "e2e": {"value": round(B * steps / e2e_s, 1), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 4 * B, "how": "graph replay per step, each step's tokens read back one step late"},
        "gpu_launches": steps * launches,
        "clocks": {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": clocks_all[0].get("sm_max_mhz"),
                   "reasons": sorted({r for c in clocks_all for r in c.get("reasons", [])}),
                   "samples": sum(c.get("samples", 0) for c in clocks_all)},
    }
    if world == 1 and a.cpu_seconds > 0:
        line["cpu_baseline"] = model_cpu(cfg, weights, prompts[0])
    return line


def main():
    a = args_parse()
    if a.impl == "reference":
        line = reference_arm(a)
    else:
        arm = {"prefill": prefill_arm, "gemv": gemv_arm, "tp": tp_arm, "model": model_arm, "moe": moe_arm,
               "moe-stack": moe_stack_arm}.get(a.workload, gpu_arm)
        line = arm(a)
        if arm is gpu_arm and not a.no_suite:
            suite = run_suite(a)
            if line is not None:
                line["configs"] = suite
        finish_ranks()
    if line is not None:
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
