"""GPU parity: batch-1 products (f32 and int8 activations), fused QKV and
gate/up-SiLU, small batches, against the oracle (through the C ABI)."""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

F32, F16, Q4_K, Q6_K, Q8_0, Q2_0C, STQ1_0 = range(7)
PACKED = [Q4_K, Q6_K, Q8_0, Q2_0C, STQ1_0]
NAMES = {F32: "F32", F16: "F16", Q4_K: "Q4_K", Q6_K: "Q6_K", Q8_0: "Q8_0", Q2_0C: "Q2_0C", STQ1_0: "STQ1_0"}

# f32 activations: the CUDA path is f32-accurate; allow 1e-5 of the f64
# magnitude sum|w_i x_i| (the reference's own SDOT test uses the same bound).
REL = 1e-5


def to_dev(a, cuda):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def make(t, N, K, seed, cuda):
    from hy_mt_rs_b200 import quant, synth
    packed = synth.encode(t, synth.random_weights(N, K, seed)).numpy()
    return packed, quant.Weight(to_dev(packed, cuda), t, [K, N], name=f"{NAMES[t]}{N}x{K}")


def f64_ref(t, packed, N, K, x):
    w = O.decode(t, packed, N * K).reshape(N, K).astype(np.float64)
    x64 = x.astype(np.float64)
    return w @ x64, np.abs(w) @ np.abs(x64)


def check_close(got, ref, mag, rel=REL, what=""):
    err = np.abs(got.astype(np.float64) - ref)
    bad = err > rel * mag + 1e-6
    assert not bad.any(), f"{what}: {bad.sum()} rows off, worst {err.max()} (mag {mag[np.argmax(err)]})"


SHAPES = [(1, 512), (7, 1024), (16, 2048), (33, 2048), (100, 4096), (40, 6144), (9, 14336)]


@pytest.mark.parametrize("t", PACKED + [F32, F16])
@pytest.mark.parametrize("N,K", SHAPES)
def test_gemv_f32(cuda, t, N, K):
    from hy_mt_rs_b200 import quant

    packed, w = make(t, N, K, N + K, cuda)
    x = np.random.default_rng(K).standard_normal(K).astype(np.float32)
    y = w.matmul(to_dev(x, cuda), 1).cpu().numpy()[0]
    ref, mag = f64_ref(t, packed, N, K, x)
    check_close(y, ref, mag, what=f"{NAMES[t]} {N}x{K}")
    yo = O.matmul(t, packed, K, N, x, 1)[0]          # the reference's x86 order
    check_close(y, yo.astype(np.float64), mag, what="vs oracle order")
    assert quant.device_status() == 0


@pytest.mark.parametrize("t", PACKED)
@pytest.mark.parametrize("N,K", SHAPES)
def test_gemv_q8(cuda, t, N, K):
    from hy_mt_rs_b200 import quant

    packed, w = make(t, N, K, 2 * N + K, cuda)
    x = (np.random.default_rng(N).standard_normal(K) * 3).astype(np.float32)
    q8 = quant.Q8.quantize(to_dev(x, cuda))
    y = w.gemv_q8_fast(q8).cpu().numpy()
    vals, scales, q2c = O.q8_quantize(x)
    ref = O.gemv_q8(t, packed, K, N, vals, scales, q2c)
    wd = O.decode(t, packed, N * K).reshape(N, K).astype(np.float64)
    xa = vals.astype(np.float64) * scales[np.arange(K) // 256].astype(np.float64)
    mag = np.abs(wd) @ np.abs(xa)
    check_close(y, ref.astype(np.float64), mag, what=f"q8 {NAMES[t]} {N}x{K}")
    check_close(y, wd @ xa, mag, what="q8 vs f64")
    assert quant.device_status() == 0


@pytest.mark.parametrize("t", [Q2_0C, STQ1_0, Q6_K, Q4_K])
def test_gemv_qkv_and_gate_up(cuda, t):
    from hy_mt_rs_b200 import quant

    K = 2048
    pq, q = make(t, 2048, K, 1, cuda)
    pk, k = make(t, 512, K, 2, cuda)
    pv, v = make(t, 512, K, 3, cuda)
    x = np.random.default_rng(7).standard_normal(K).astype(np.float32)
    xd = to_dev(x, cuda)
    qo, ko, vo = quant.Weight.gemv_qkv(q, k, v, xd)
    for got, p, n in ((qo, pq, 2048), (ko, pk, 512), (vo, pv, 512)):
        ref, mag = f64_ref(t, p, n, K, x)
        check_close(got.cpu().numpy(), ref, mag, what="qkv")
    q8 = quant.Q8.quantize(xd)
    vals, scales, q2c = O.q8_quantize(x)
    qo, ko, vo = quant.Weight.gemv_qkv_fast(q, k, v, q8)
    for got, p, n in ((qo, pq, 2048), (ko, pk, 512), (vo, pv, 512)):
        ref = O.gemv_q8(t, p, K, n, vals, scales, q2c)
        wd = O.decode(t, p, n * K).reshape(n, K).astype(np.float64)
        mag = np.abs(wd) @ np.abs(vals.astype(np.float64) * scales[np.arange(K) // 256])
        check_close(got.cpu().numpy(), ref.astype(np.float64), mag, what="qkv q8")
    # gate/up with SiLU (quant.rs:724-841): compare g and u separately via the
    # plain products, then the fused value with the oracle's formula.
    N = 6144
    pg, g = make(t, N, K, 11, cuda)
    pu, u = make(t, N, K, 12, cuda)
    y = g.matmul_gate_up_silu(u, xd).cpu().numpy()
    ref = O.gate_up_silu(t, pg, pu, K, N, x)
    gref, gmag = f64_ref(t, pg, N, K, x)
    uref, umag = f64_ref(t, pu, N, K, x)
    # d(silu(g) u) <= |u| |dg| (|silu'| <= 1.1) + |silu(g)| |du|
    tol = 1.1 * np.abs(uref) * REL * gmag + np.abs(gref) * REL * umag + 1e-6
    assert np.all(np.abs(y - ref) <= tol + 1e-6 * np.abs(ref))
    y8 = g.matmul_gate_up_silu_fast(u, q8).cpu().numpy()
    ref8 = O.gate_up_silu_q8(t, pg, pu, K, N, vals, scales, q2c)
    assert np.all(np.abs(y8 - ref8) <= tol * 2 + 1e-5 * np.abs(ref8))
    assert quant.device_status() == 0


@pytest.mark.parametrize("batch", [2, 3, 7, 8, 9])
def test_matmul_small_batches(cuda, batch):
    from hy_mt_rs_b200 import quant

    K, N = 2048, 300
    for t in (Q4_K, Q6_K, Q2_0C, STQ1_0, Q8_0):
        packed, w = make(t, N, K, batch, cuda)
        x = np.random.default_rng(batch).standard_normal((batch, K)).astype(np.float32)
        y = w.matmul(to_dev(x, cuda), batch).cpu().numpy()
        ref = O.matmul(t, packed, K, N, x.ravel(), batch)
        wd = O.decode(t, packed, N * K).reshape(N, K).astype(np.float64)
        mag = (np.abs(x.astype(np.float64)) @ np.abs(wd).T)
        assert np.all(np.abs(y - ref) <= REL * mag + 1e-6)


def test_fallback_paths(cuda):
    """Shapes/pointers the streaming engine does not take still compute."""
    import torch
    from hy_mt_rs_b200 import quant, synth

    # Q8_0 with K = 96 (not a multiple of 256)
    K, N = 96, 50
    packed = synth.encode(Q8_0, synth.random_weights(N, K, 1)).numpy()
    w = quant.Weight(to_dev(packed, cuda), Q8_0, [K, N])
    x = np.random.default_rng(1).standard_normal(K).astype(np.float32)
    ref, mag = f64_ref(Q8_0, packed, N, K, x)
    check_close(w.matmul(to_dev(x, cuda), 1).cpu().numpy()[0], ref, mag, what="Q8_0 K=96")
    # weight bytes at a 2-byte offset inside a buffer (not 16-byte aligned)
    K, N = 2048, 64
    packed = synth.encode(Q2_0C, synth.random_weights(N, K, 2)).numpy()
    buf = torch.zeros(packed.size + 16, dtype=torch.uint8, device=cuda)
    buf[2:2 + packed.size] = to_dev(packed, cuda)
    w = quant.Weight(buf[2:2 + packed.size], Q2_0C, [K, N])
    x = np.random.default_rng(2).standard_normal(K).astype(np.float32)
    ref, mag = f64_ref(Q2_0C, packed, N, K, x)
    check_close(w.matmul(to_dev(x, cuda), 1).cpu().numpy()[0], ref, mag, what="unaligned")
    assert quant.device_status() == 0


def test_shape_errors(cuda):
    import torch
    from hy_mt_rs_b200 import quant

    _, w = make(Q2_0C, 8, 1024, 0, cuda)
    _, w3 = make(Q2_0C, 8, 512, 0, cuda)
    x = torch.zeros(1024, device=cuda)
    with pytest.raises(quant.HyqError):
        w.matmul(x, 2)
    with pytest.raises(quant.HyqError):
        quant.Weight.gemv_qkv(w, w3, w, x)
    with pytest.raises(quant.HyqError):
        w.matmul_gate_up_silu(w3, x)


def test_full_size_lm_head_properties(cuda):
    """Q6_K lm_head 120832 x 2048: rows spot-checked against the oracle, and
    the f32 path is exactly homogeneous under power-of-two scaling."""
    import torch
    from hy_mt_rs_b200 import quant, synth

    K, N = 2048, 120832
    packed_t = synth.random_packed(Q6_K, N, K, seed=42, device=cuda)
    w = quant.Weight(packed_t, Q6_K, [K, N])
    x = np.random.default_rng(3).standard_normal(K).astype(np.float32)
    xd = to_dev(x, cuda)
    y = w.matmul(xd, 1)[0]
    y4 = w.matmul(xd * 4.0, 1)[0]
    assert torch.equal(y4, y * 4.0)
    rows = np.r_[0:64, N - 64:N, np.random.default_rng(0).integers(0, N, 256)]
    packed = packed_t.cpu().numpy().reshape(N, -1)
    sub = np.ascontiguousarray(packed[rows]).ravel()
    ref, mag = f64_ref(Q6_K, sub, len(rows), K, x)
    check_close(y.cpu().numpy()[rows], ref, mag, what="lm_head rows")
    q8 = quant.Q8.quantize(xd)
    y8 = w.gemv_q8_fast(q8).cpu().numpy()
    vals, scales, q2c = O.q8_quantize(x)
    ref8 = O.gemv_q8(Q6_K, sub, K, len(rows), vals, scales, q2c)
    wd = O.decode(Q6_K, sub, len(rows) * K).reshape(len(rows), K).astype(np.float64)
    mag8 = np.abs(wd) @ np.abs(vals.astype(np.float64) * scales[np.arange(K) // 256])
    check_close(y8[rows], ref8.astype(np.float64), mag8, what="lm_head q8 rows")
    assert quant.device_status() == 0


@pytest.mark.parametrize("t", PACKED)
@pytest.mark.parametrize("N,K", [(16, 2048), (40, 6144), (9, 14336), (100, 4096), (7, 256)])
def test_int8_in_kernel_matches_two_step(cuda, t, N, K):
    """hyq_gemv_int8 (Q8 inside the kernel) == hyq_q8_quantize + hyq_gemv_q8,
    bit for bit, including a NaN group and an all-zero group."""
    import torch
    from hy_mt_rs_b200 import quant

    if K % O.block_len(t):
        pytest.skip("K is not a whole number of blocks")
    packed, w = make(t, N, K, 3 * N + K, cuda)
    x = (np.random.default_rng(K + N).standard_normal(K) * 2).astype(np.float32)
    if K >= 1024:
        x[256:512] = 0.0
        x[700] = np.nan
    xd = to_dev(x, cuda)
    y1 = w.gemv_int8(xd)
    y2 = w.gemv_q8_fast(quant.Q8.quantize(xd))
    assert torch.equal(torch.nan_to_num(y1, nan=123.0), torch.nan_to_num(y2, nan=123.0))
    vals, scales, q2c = O.q8_quantize(x)
    ref = O.gemv_q8(t, packed, K, N, vals, scales, q2c)
    wd = O.decode(t, packed, N * K).reshape(N, K).astype(np.float64)
    mag = np.abs(wd) @ np.abs(vals.astype(np.float64) * scales[np.arange(K) // 256])
    check_close(y1.cpu().numpy(), ref.astype(np.float64), mag, what=f"int8 {NAMES[t]} {N}x{K}")


@pytest.mark.parametrize("t", [Q2_0C, STQ1_0, Q6_K])
def test_fused_int8_entry_points(cuda, t):
    """gemv_qkv / matmul_gate_up_silu through in-kernel Q8 == their two-step forms."""
    import torch
    from hy_mt_rs_b200 import quant

    K = 2048
    _, q = make(t, 2048, K, 21, cuda)
    _, k = make(t, 512, K, 22, cuda)
    _, v = make(t, 512, K, 23, cuda)
    _, g = make(t, 6144, K, 24, cuda)
    _, u = make(t, 6144, K, 25, cuda)
    xd = to_dev(np.random.default_rng(9).standard_normal(K).astype(np.float32), cuda)
    q8 = quant.Q8.quantize(xd)
    for a, b in zip(quant.Weight.gemv_qkv_int8(q, k, v, xd), quant.Weight.gemv_qkv_fast(q, k, v, q8)):
        assert torch.equal(a, b)
    assert torch.equal(g.matmul_gate_up_silu_int8(u, xd), g.matmul_gate_up_silu_fast(u, q8))
    assert quant.device_status() == 0


@pytest.mark.parametrize("act", [0, 1])
@pytest.mark.parametrize("t", PACKED)
def test_fused_norm_and_residual_forms(cuda, t, act):
    """hyq_gemv_*_norm = hyq_rms_norm then the plain batch-1 product, and
    hyq_gemv_residual = the plain product then hyq_add, bit for bit (the
    decoder chain of model.rs:1007-1041 with the norm and the residual add
    inside the products); the norm itself equals the oracle's x86 order.
    act 1 (HYQ_ACT_Q8): the products are the in-kernel-Q8 forms (_int8)."""
    import ctypes as C
    import torch
    from hy_mt_rs_b200._native import lib

    def P(a):
        return C.c_void_p(a.data_ptr())

    def ok(rc):
        assert rc == 0, lib.hyq_last_error().decode()

    K, F, eps = 2048, 6144, 1e-6
    _, q = make(t, 2048, K, 31, cuda)
    _, k = make(t, 512, K, 32, cuda)
    _, v = make(t, 512, K, 33, cuda)
    _, g = make(t, F, K, 34, cuda)
    _, u = make(t, F, K, 35, cuda)
    _, down = make(t, K, F, 36, cuda)
    rng = np.random.default_rng(40 + t)
    h = (rng.standard_normal(K) * 3).astype(np.float32)
    nw = rng.standard_normal(K).astype(np.float32)
    hd, nwd = to_dev(h, cuda), to_dev(nw, cuda)
    st = C.c_void_p(torch.cuda.current_stream(cuda).cuda_stream)
    fus = C.c_int()
    for w in (q, k, v, g, u, down):
        ok(lib.hyq_gemv_fusable(w.handle, C.byref(fus)))
        assert fus.value == 1
    normalized = torch.empty(K, device=cuda)
    ok(lib.hyq_rms_norm(P(hd), P(nwd), K, 1, eps, P(normalized), st))
    a = [torch.empty(n, device=cuda) for n in (2048, 512, 512)]
    b = [torch.empty(n, device=cuda) for n in (2048, 512, 512)]
    qkv = lib.hyq_gemv_qkv_int8 if act else lib.hyq_gemv_qkv
    ok(qkv(q.handle, k.handle, v.handle, P(normalized), *map(P, a), st))
    ok(lib.hyq_gemv_qkv_norm(q.handle, k.handle, v.handle, P(hd), P(nwd), eps, act, *map(P, b), st))

    def gemv(w, x, y):
        return lib.hyq_gemv_int8(w.handle, P(x), P(y), st) if act else lib.hyq_matmul(w.handle, P(x), 1, P(y), st)

    y1, y2 = torch.empty(2048, device=cuda), torch.empty(2048, device=cuda)
    ok(gemv(q, normalized, y1))
    ok(lib.hyq_gemv_norm(q.handle, P(hd), P(nwd), eps, act, P(y2), st))
    s1, s2 = torch.empty(F, device=cuda), torch.empty(F, device=cuda)
    gate_up = lib.hyq_matmul_gate_up_silu_int8 if act else lib.hyq_matmul_gate_up_silu
    ok(gate_up(g.handle, u.handle, P(normalized), P(s1), st))
    ok(lib.hyq_gemv_gate_up_silu_norm(g.handle, u.handle, P(hd), P(nwd), eps, act, P(s2), st))
    xf = to_dev(rng.standard_normal(F).astype(np.float32), cuda)
    h1, h2, dy = hd.clone(), hd.clone(), torch.empty(K, device=cuda)
    ok(gemv(down, xf, dy))
    ok(lib.hyq_add(P(h1), P(dy), K, st))
    ok(lib.hyq_gemv_residual(down.handle, P(xf), act, P(h2), st))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(normalized.cpu().numpy(), O.rms_norm(h, nw, eps))
    for x, y in zip(a + [y1, s1, h1], b + [y2, s2, h2]):
        assert torch.equal(x, y)
    assert torch.equal(hd.cpu(), torch.from_numpy(h))   # the norm forms leave hidden as it was
    assert not torch.equal(h2, hd)


def test_fused_forms_refuse_unqualified_inputs(cuda):
    """The fused norm / residual forms run only on the streaming engine with
    staged activations: F32 weights, K off the 256 grid or above 6144, and an
    input that is not 16-byte aligned give HYQ_E_UNSUPPORTED, and
    hyq_gemv_fusable says so beforehand."""
    import ctypes as C
    import torch
    from hy_mt_rs_b200._native import lib

    st = C.c_void_p(torch.cuda.current_stream(cuda).cuda_stream)
    fus = C.c_int()
    for t, N, K in ((F32, 64, 2048), (Q8_0, 64, 2080), (Q4_K, 64, 6400)):
        _, w = make(t, N, K, 50, cuda)
        assert lib.hyq_gemv_fusable(w.handle, C.byref(fus)) == 0 and fus.value == 0
        x = torch.ones(K, device=cuda)
        y = torch.zeros(N, device=cuda)
        rc = lib.hyq_gemv_norm(w.handle, C.c_void_p(x.data_ptr()), C.c_void_p(x.data_ptr()), 1e-6, 0,
                               C.c_void_p(y.data_ptr()), st)
        assert rc == -6, (t, K, rc)
        assert lib.hyq_gemv_residual(w.handle, C.c_void_p(x.data_ptr()), 0, C.c_void_p(y.data_ptr()), st) == -6
    _, w = make(Q2_0C, 64, 2048, 51, cuda)
    buf = torch.ones(2048 + 4, device=cuda)
    y = torch.zeros(64, device=cuda)
    off = C.c_void_p(buf.data_ptr() + 4)   # 4-byte aligned, not 16
    assert lib.hyq_gemv_norm(w.handle, off, off, 1e-6, 0, C.c_void_p(y.data_ptr()), st) == -6
    assert lib.hyq_gemv_residual(w.handle, off, 0, C.c_void_p(y.data_ptr()), st) == -6
    aligned = C.c_void_p(buf.data_ptr())
    assert lib.hyq_gemv_residual(w.handle, aligned, 2, C.c_void_p(y.data_ptr()), st) == -1   # unknown mode
    torch.cuda.synchronize()
    assert torch.count_nonzero(y).item() == 0
