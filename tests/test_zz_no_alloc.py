"""GPU check of hyq_matmul_noalloc, the batched product for callers that may
not allocate device memory per call (its scratch is a fixed device array in
the library).  Called through the C ABI, it must give hyq_matmul's result
(same tolerance as the GEMM parity tests: 1e-3 relative L2, 2e-3 of the
largest magnitude per element) on consecutive calls that reuse the array,
and refuse a batch whose scratch would not fit.

Collected last so that it also runs after every other GPU test in the same
process; it passes on its own in a fresh process too."""
import ctypes as C

import pytest

pytestmark = pytest.mark.gpu

Q4_K, Q6_K = 2, 3
HYQ_E_SHAPE = -2
SCRATCH_BYTES = 64 << 20  # HYQ_NOALLOC_SCRATCH_BYTES


def make(cuda, t, N, K, M, seed):
    import torch
    from hy_mt_rs_b200 import quant, synth

    w = quant.Weight(synth.random_packed(t, N, K, seed=seed, device=cuda), t, [K, N])
    x = torch.randn(M, K, generator=torch.Generator().manual_seed(seed + 1)).to(cuda)
    return w, x


def noalloc(w, x, M):
    import torch
    from hy_mt_rs_b200 import _native, quant

    out = torch.full((M, w.rows), float("nan"), dtype=torch.float32, device=x.device)
    rc = _native.lib.hyq_matmul_noalloc(w.handle, C.c_void_p(x.data_ptr()), M, C.c_void_p(out.data_ptr()),
                                        quant._stream(x.device))
    return rc, out


def assert_close(y, ref):
    import torch

    assert torch.isfinite(y).all()
    rel = (torch.linalg.norm(y - ref) / torch.linalg.norm(ref)).item()
    assert rel < 1e-3, rel
    assert (y - ref).abs().max().item() <= 2e-3 * ref.abs().max().item() + 1e-5


# (dtype, N, K, M): split-K partials in the scratch, a single slice, and a
# batch below the tensor-core threshold (batch-1 products, no scratch).
CASES = [(Q6_K, 1024, 14336, 64), (Q4_K, 14336, 4096, 512), (Q4_K, 512, 2048, 5)]


def test_noalloc_matches_matmul_on_consecutive_calls(cuda):
    from hy_mt_rs_b200 import _native, quant

    # the first case must reach the partial-sum region of the array (more
    # than one split-K slice), the second must not, the third stays below
    # the tensor-core batch threshold
    assert quant.gemm_splits(CASES[0][1] // 128, CASES[0][2], CASES[0][3], CASES[0][0]) > 1
    assert quant.gemm_splits(CASES[1][1] // 128, CASES[1][2], CASES[1][3], CASES[1][0]) == 1
    assert CASES[2][3] < 16
    runs = []
    for i, (t, N, K, M) in enumerate(CASES):
        w, x = make(cuda, t, N, K, M, seed=11 + i)
        rc, y = noalloc(w, x, M)
        assert rc == 0, _native.last_error()
        runs.append((w, x, M, y))
    # the first case again, after the other calls overwrote the array
    w, x, M, _ = runs[0]
    rc, y_again = noalloc(w, x, M)
    assert rc == 0, _native.last_error()
    for w, x, M, y in runs:
        assert_close(y, w.matmul(x, M))
    assert_close(y_again, runs[0][3])
    assert quant.device_status() == 0


def test_noalloc_rejects_batch_beyond_scratch(cuda):
    from hy_mt_rs_b200 import _native

    K, N = 14336, 128
    # the fp16 activation copy alone exceeds the array; a whole number of
    # 256-token tiles, so the batch takes the tensor-core path for certain
    M = (SCRATCH_BYTES // (2 * K) // 256 + 1) * 256
    assert 2 * K * M > SCRATCH_BYTES
    w, x = make(cuda, Q6_K, N, K, M, seed=3)
    rc, _ = noalloc(w, x, M)
    assert rc == HYQ_E_SHAPE
    assert "HYQ_NOALLOC_SCRATCH_BYTES" in _native.last_error()
