"""GPU parity: the tensor-core batched product (Weight::matmul, batch >= 16,
quant.rs:272-343) against an f64 oracle of the decoded weights.

Operands are fp16 on the tensor cores (weights decoded in f32 then rounded,
activations rounded), accumulation f32: the north-star bound is 1e-3
relative L2; each element is also held to 2e-3 of sum|w x|."""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

Q4_K, Q6_K, Q8_0, Q2_0C, STQ1_0 = 2, 3, 4, 5, 6


def to_dev(a, cuda):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def run_case(cuda, t, N, K, M, seed, split=False):
    """split: the split-operand products (hyq_set_gemm_precision(HYQ_GEMM_F32)),
    held to the per-element bound of the f32 batch-1 products, 1e-5 of
    sum|w x|, and to 1e-5 relative L2 (measured up to 5e-6 at K = 4096: the
    tensor core's f32 accumulation over K / 16 chained MMAs)."""
    from hy_mt_rs_b200 import quant, synth

    packed = synth.encode(t, synth.random_weights(N, K, seed)).numpy()
    w = quant.Weight(to_dev(packed, cuda), t, [K, N])
    x = np.random.default_rng(seed).standard_normal((M, K)).astype(np.float32)
    with quant.gemm_precision(quant.GEMM_F32 if split else quant.GEMM_FP16):
        y = w.matmul(to_dev(x, cuda), M).cpu().numpy()
    wd = O.decode(t, packed, N * K).reshape(N, K).astype(np.float64)
    ref = x.astype(np.float64) @ wd.T
    mag = np.abs(x.astype(np.float64)) @ np.abs(wd).T
    rel_l2 = np.linalg.norm(y - ref) / np.linalg.norm(ref)
    bound_l2, bound_el = (1e-5, 1e-5) if split else (1e-3, 2e-3)
    assert rel_l2 < bound_l2, rel_l2
    assert np.all(np.abs(y - ref) <= bound_el * mag + 1e-6), np.max(np.abs(y - ref) / (mag + 1e-9))
    assert quant.device_status() == 0
    return rel_l2


@pytest.mark.parametrize("t", [Q4_K, Q6_K])
@pytest.mark.parametrize("N,K,M", [(128, 256, 16), (300, 1024, 37), (128, 512, 130), (257, 2048, 200)])
def test_gemm_small(cuda, t, N, K, M):
    run_case(cuda, t, N, K, M, seed=N + K + M)


@pytest.mark.parametrize("t,N,K,M", [(Q4_K, 4096, 4096, 128), (Q6_K, 1024, 14336, 64), (Q4_K, 1024, 4096, 512)])
def test_gemm_7b_shapes(cuda, t, N, K, M):
    run_case(cuda, t, N, K, M, seed=7)


# 2-SM tiles (256 rows x 256 tokens per CTA pair): N a multiple of 256 and at
# least 256 tokens; a partial last token tile, a 2-row pitch (Q6_K, 4 blocks)
# and split-K slices of pairs.
PAIR_CASES = [(Q4_K, 512, 1024, 256), (Q6_K, 768, 1024, 300), (Q6_K, 2048, 7168, 512), (Q4_K, 1024, 4096, 1000)]


@pytest.mark.parametrize("pair", ["1", "0"])
def test_gemm_pair_tiles(cuda, pair):
    """Single-matrix Q4_K / Q6_K products from 256 tokens on the 2-SM kernel
    (the default) and, with HYQ_GEMM_PAIR=0, on the 1-SM kernel.  The switch
    is read once per process, so the cases run in a child process."""
    import os
    import subprocess
    import sys

    from conftest import ROOT

    code = ("import sys; sys.path.insert(0, %r); sys.path.insert(0, %r)\n"
            "import test_gpu_gemm as T, torch\n"
            "dev = torch.device('cuda', 0)\n"
            "for c in T.PAIR_CASES: T.run_case(dev, *c, seed=c[1] + c[3])\n"
            "print('ok')\n") % (ROOT, os.path.join(ROOT, "tests"))
    env = dict(os.environ, HYQ_GEMM_PAIR=pair)
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stderr[-3000:]


def test_gemm_matches_gemv_path(cuda):
    """Batch 16 (tensor cores) and batch-1 rows agree to fp16-operand accuracy."""
    import torch
    from hy_mt_rs_b200 import quant, synth

    K, N, M = 2048, 512, 16
    packed = synth.random_packed(Q4_K, N, K, seed=3, device=cuda)
    w = quant.Weight(packed, Q4_K, [K, N])
    x = torch.randn(M, K, generator=torch.Generator().manual_seed(4)).to(cuda)
    y = w.matmul(x, M)
    rows = torch.stack([w.matmul(x[i].contiguous(), 1)[0] for i in range(M)])
    assert (torch.linalg.norm(y - rows) / torch.linalg.norm(rows)).item() < 1e-3


def _w(cuda, t, N, K, seed):
    from hy_mt_rs_b200 import quant, synth
    return quant.Weight(synth.random_packed(t, N, K, seed=seed, device=cuda), t, [K, N])


def _rel(a, b):
    import torch
    return (torch.linalg.norm(a - b) / torch.linalg.norm(b)).item()


@pytest.mark.parametrize("t,K,Nq,Nkv,M", [(Q4_K, 4096, 4096, 1024, 512), (Q4_K, 2048, 1024, 256, 37),
                                          (Q6_K, 1024, 512, 128, 300), (Q4_K, 1024, 256, 128, 7)])
def test_matmul_qkv_matches_separate_products(cuda, t, K, Nq, Nkv, M):
    """One grouped launch (QKV share the input) equals three products; M=7
    takes the batch-1 path."""
    import torch
    from hy_mt_rs_b200 import quant

    q, k, v = _w(cuda, t, Nq, K, 1), _w(cuda, t, Nkv, K, 2), _w(cuda, t, Nkv, K, 3)
    x = torch.randn(M, K, generator=torch.Generator().manual_seed(4)).to(cuda)
    got = quant.Weight.matmul_qkv(q, k, v, x, M)
    for w, y in zip((q, k, v), got):
        ref = w.matmul(x, M)
        assert _rel(y, ref) < 1e-5, _rel(y, ref)
    assert quant.device_status() == 0


# Tail split (fp16 operands, at least one wave of tiles): the tiles past the
# last full wave run as K-slices summed by a second kernel.  A partial last
# row tile and token tile in the tail (Q8_0, 149 tiles at 50 tokens), a whole
# one (Q4_K at 128 tokens, 150 tiles), both against the f64 oracle.
TAIL_CASES = [(Q8_0, 148 * 128 + 37, 2048, 50), (Q4_K, 150 * 128, 4096, 128)]


@pytest.mark.parametrize("t,N,K,M", TAIL_CASES)
def test_gemm_tail_split(cuda, t, N, K, M):
    import torch
    from hy_mt_rs_b200 import quant

    sms = torch.cuda.get_device_properties(cuda).multi_processor_count
    assert quant.gemm_tail_slices(-(-N // 128), K, M, t, sms) > 1
    run_case(cuda, t, N, K, M, seed=N + M)


def test_matmul_qkv_tail_split_matches_separate_products(cuda):
    """A grouped QKV launch whose last tile (the v matrix's) falls past the
    first wave: it runs as K-slices, and the three outputs still equal three
    separate products (which take split-K or whole tiles)."""
    import torch
    from hy_mt_rs_b200 import quant

    t, K, Nq, Nkv, M = Q4_K, 2048, 133 * 128, 1024, 64
    assert quant.gemm_tail_slices(Nq // 128 + 2 * Nkv // 128, K, M, t) > 1
    q, k, v = _w(cuda, t, Nq, K, 1), _w(cuda, t, Nkv, K, 2), _w(cuda, t, Nkv, K, 3)
    x = torch.randn(M, K, generator=torch.Generator().manual_seed(4)).to(cuda)
    got = quant.Weight.matmul_qkv(q, k, v, x, M)
    for w, y in zip((q, k, v), got):
        ref = w.matmul(x, M)
        assert _rel(y, ref) < 1e-5, _rel(y, ref)
    assert quant.device_status() == 0


@pytest.mark.parametrize("t,N,K,M", [(Q4_K, 14336, 4096, 512), (Q4_K, 14336, 4096, 2048), (Q4_K, 1024, 2048, 64),
                                     (Q6_K, 768, 1024, 200), (Q4_K, 512, 1024, 9)])
def test_gate_up_silu_batch_matches_separate_products(cuda, t, N, K, M):
    """silu(gate) * up from one fused launch equals the reference's batched
    DenseFfn (two products, then the elementwise combination)."""
    import torch
    from hy_mt_rs_b200 import quant

    gate, up = _w(cuda, t, N, K, 5), _w(cuda, t, N, K, 6)
    x = torch.randn(M, K, generator=torch.Generator().manual_seed(7)).to(cuda)
    got = gate.matmul_gate_up_silu_batch(up, x, M)
    g, u = gate.matmul(x, M), up.matmul(x, M)
    ref = (g / (1.0 + torch.exp(-g))) * u
    assert _rel(got, ref) < 1e-5, _rel(got, ref)
    assert quant.device_status() == 0


# The other packed formats (Q8_0 in 4-block columns, Q2_0C in 512-weight
# blocks, STQ1_0 ternary through the codebook), at small and 1.8B shapes.
@pytest.mark.parametrize("t,N,K,M", [(Q8_0, 128, 256, 16), (Q8_0, 300, 1024, 37), (Q8_0, 2048, 2048, 512),
                                     (Q2_0C, 128, 512, 16), (Q2_0C, 300, 2048, 200), (Q2_0C, 2048, 6144, 512),
                                     (STQ1_0, 128, 256, 16), (STQ1_0, 257, 2048, 130), (STQ1_0, 6144, 2048, 256),
                                     (Q2_0C, 2048, 2048, 64), (Q2_0C, 2048, 6144, 64), (STQ1_0, 2048, 6144, 33),
                                     (Q2_0C, 1024, 2048, 65)])
def test_gemm_other_formats(cuda, t, N, K, M):
    run_case(cuda, t, N, K, M, seed=N + K + M + t)


@pytest.mark.parametrize("t,M", [(Q2_0C, 256), (STQ1_0, 256), (Q2_0C, 64), (Q2_0C, 20)])
def test_gemm_1p8b_layer_calls(cuda, t, M):
    """Grouped QKV and fused gate/up-SiLU on the 1.8B layer shapes (M <= 64:
    the 64-token tile)."""
    import torch
    from hy_mt_rs_b200 import quant

    q, k, v = _w(cuda, t, 2048, 2048, 1), _w(cuda, t, 512, 2048, 2), _w(cuda, t, 512, 2048, 3)
    x = torch.randn(M, 2048, generator=torch.Generator().manual_seed(8)).to(cuda)
    for w, y in zip((q, k, v), quant.Weight.matmul_qkv(q, k, v, x, M)):
        assert _rel(y, w.matmul(x, M)) < 1e-5
    gate, up = _w(cuda, t, 6144, 2048, 4), _w(cuda, t, 6144, 2048, 5)
    got = gate.matmul_gate_up_silu_batch(up, x, M)
    g, u = gate.matmul(x, M), up.matmul(x, M)
    assert _rel(got, (g / (1.0 + torch.exp(-g))) * u) < 1e-5
    assert quant.device_status() == 0


# Split-operand products (HYQ_GEMM_F32): every format, both token tiles (64,
# 128; 256-token batches run 128-token tiles), split-K slices and a partial
# last token tile.
SPLIT_CASES = [(Q4_K, 256, 2048, 16), (Q4_K, 4096, 4096, 300), (Q6_K, 1024, 14336, 64), (Q6_K, 384, 1024, 100),
               (Q8_0, 300, 1024, 37), (Q2_0C, 2048, 6144, 64), (Q2_0C, 512, 2048, 256), (STQ1_0, 257, 2048, 130),
               (STQ1_0, 2048, 2048, 64)]


@pytest.mark.parametrize("t,N,K,M", SPLIT_CASES)
def test_gemm_split_operands_f32_accuracy(cuda, t, N, K, M):
    run_case(cuda, t, N, K, M, seed=N + K + M + t, split=True)


@pytest.mark.parametrize("t,M", [(Q2_0C, 64), (Q2_0C, 256), (STQ1_0, 40), (Q4_K, 130)])
def test_gemm_split_layer_calls_match_batch1_products(cuda, t, M):
    """Grouped QKV and the fused gate/up-SiLU in the split-operand form agree
    with the f32 batch-1 products row by row (both f32-accurate): within 1e-5
    relative L2 (about 5e-6 measured, from the tensor core's accumulation)."""
    import torch
    from hy_mt_rs_b200 import quant

    K = 2048
    q, k, v = _w(cuda, t, 2048, K, 1), _w(cuda, t, 512, K, 2), _w(cuda, t, 512, K, 3)
    gate, up = _w(cuda, t, 6144, K, 4), _w(cuda, t, 6144, K, 5)
    x = torch.randn(M, K, generator=torch.Generator().manual_seed(8)).to(cuda)
    with quant.gemm_precision(quant.GEMM_F32):
        got_qkv = quant.Weight.matmul_qkv(q, k, v, x, M)
        got_gu = gate.matmul_gate_up_silu_batch(up, x, M)
    for w, y in zip((q, k, v), got_qkv):
        rows = torch.stack([w.matmul(x[i].contiguous(), 1)[0] for i in range(M)])
        assert _rel(y, rows) < 1e-5, _rel(y, rows)
    rows = torch.stack([gate.matmul_gate_up_silu(up, x[i].contiguous()) for i in range(M)])
    assert _rel(got_gu, rows) < 1e-5, _rel(got_gu, rows)
    assert quant.device_status() == 0


@pytest.mark.parametrize("t,M,split,delta", [(Q2_0C, 64, True, True), (Q2_0C, 64, False, False),
                                             (Q4_K, 40, True, False), (STQ1_0, 256, False, True),
                                             (Q2_0C, 5, True, True), (Q6_K, 1, False, True)])
def test_batched_norm_forms_match_separate_calls(cuda, t, M, split, delta):
    """hyq_matmul_qkv_norm / hyq_matmul_gate_up_silu_norm / hyq_matmul_norm
    (the residual add and the RMSNorm inside the tensor-core conversion from
    16 rows, the separate kernel below) = hyq_add_rms_norm (or hyq_rms_norm)
    followed by the plain batched product: outputs and the updated hidden
    rows bit-identical, both operand precisions."""
    import ctypes as C
    import torch
    from hy_mt_rs_b200 import quant, synth
    from hy_mt_rs_b200._native import lib

    def P(x):
        return C.c_void_p(x.data_ptr()) if x is not None else None

    def ok(rc):
        assert rc == 0, lib.hyq_last_error().decode()

    K, Nq, Nkv, F = 2048, 2048, 512, 1024

    def weight(N, seed):
        packed = synth.encode(t, synth.random_weights(N, K, seed))
        return quant.Weight(packed.to(cuda), t, [K, N])

    q, k, v, g, u, o = weight(Nq, 1), weight(Nkv, 2), weight(Nkv, 3), weight(F, 4), weight(F, 5), weight(Nq, 6)
    rng = np.random.default_rng(M)
    h0 = to_dev((rng.standard_normal((M, K)) * 2).astype(np.float32), cuda)
    d = to_dev(rng.standard_normal((M, K)).astype(np.float32), cuda) if delta else None
    w = to_dev(rng.standard_normal(K).astype(np.float32), cuda)
    st = C.c_void_p(torch.cuda.current_stream(cuda).cuda_stream)
    eps = 1e-6
    res = []
    with quant.gemm_precision(quant.GEMM_F32 if split else quant.GEMM_FP16):
        for fused in (False, True):
            outs = [torch.empty(M, n, device=cuda) for n in (Nq, Nkv, Nkv, F, Nq)]
            hids = [h0.clone() for _ in range(3)]
            for j in range(3):
                if fused:
                    if j == 0:
                        ok(lib.hyq_matmul_qkv_norm(q.handle, k.handle, v.handle, P(hids[0]), P(d), P(w), eps, M,
                                                   *map(P, outs[:3]), st))
                    elif j == 1:
                        ok(lib.hyq_matmul_gate_up_silu_norm(g.handle, u.handle, P(hids[1]), P(d), P(w), eps, M,
                                                            P(outs[3]), st))
                    else:
                        ok(lib.hyq_matmul_norm(o.handle, P(hids[2]), P(d), P(w), eps, M, P(outs[4]), st))
                else:
                    x = torch.empty(M, K, device=cuda)
                    if delta:
                        ok(lib.hyq_add_rms_norm(P(hids[j]), P(d), P(w), K, M, eps, P(x), st))
                    else:
                        ok(lib.hyq_rms_norm(P(hids[j]), P(w), K, M, eps, P(x), st))
                    if j == 0:
                        ok(lib.hyq_matmul_qkv(q.handle, k.handle, v.handle, P(x), M, *map(P, outs[:3]), st))
                    elif j == 1:
                        ok(lib.hyq_matmul_gate_up_silu_batch(g.handle, u.handle, P(x), M, P(outs[3]), st))
                    else:
                        ok(lib.hyq_matmul(o.handle, P(x), M, P(outs[4]), st))
            res.append(outs + hids)
    torch.cuda.synchronize()
    for a, b in zip(*res):
        assert torch.equal(a, b)
    if delta:
        assert torch.equal(res[1][5], h0 + d)
    else:
        assert torch.equal(res[1][5], h0)
    assert quant.device_status() == 0
