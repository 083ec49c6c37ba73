"""GPU check of tensor-parallel shards (hyq_weight_shard): column-parallel
shards give the full product's rows, and the partial products of
row-parallel shards sum to the full product, for batch-1 products on both
activation paths and for the tensor-core GEMM."""
import pytest

pytestmark = pytest.mark.gpu

Q4_K, Q6_K, Q2_0C = 2, 3, 5


def _weight(cuda, t, N, K, seed):
    from hy_mt_rs_b200 import quant, synth

    return quant.Weight(synth.random_packed(t, N, K, seed=seed, device=cuda), t, [K, N])


def _close(a, b, tol):
    import torch

    err = (a - b).abs().max().item()
    scale = b.abs().max().item() + 1e-12
    assert err <= tol * scale, (err, scale)


@pytest.mark.parametrize("t,N,K,parts", [(Q4_K, 4096, 4096, 4), (Q6_K, 4096, 14336, 8), (Q2_0C, 2048, 6144, 4)])
@pytest.mark.parametrize("path", ["f32", "int8"])
def test_batch1_shards_rebuild_the_product(cuda, t, N, K, parts, path):
    import torch

    w = _weight(cuda, t, N, K, seed=N + K)
    x = torch.randn(K, generator=torch.Generator().manual_seed(5)).to(cuda)
    run = (lambda m, v: m.matmul(v, 1)[0]) if path == "f32" else (lambda m, v: m.gemv_int8(v))
    full = run(w, x)
    cols = torch.cat([run(w.shard(0, p, parts), x) for p in range(parts)])
    _close(cols, full, 1e-6)
    k = K // parts
    rows = sum(run(w.shard(1, p, parts), x[p * k:(p + 1) * k].contiguous()) for p in range(parts))
    _close(rows, full, 1e-5)


@pytest.mark.parametrize("t,N,K,parts", [(Q4_K, 1024, 4096, 2), (Q6_K, 1024, 14336, 8)])
def test_gemm_shards_rebuild_the_product(cuda, t, N, K, parts):
    import torch

    M = 64
    w = _weight(cuda, t, N, K, seed=3)
    x = torch.randn(M, K, generator=torch.Generator().manual_seed(6)).to(cuda)
    full = w.matmul(x, M)
    cols = torch.cat([w.shard(0, p, parts).matmul(x, M) for p in range(parts)], dim=1)
    _close(cols, full, 1e-4)  # split-K choices differ with the row count
    k = K // parts
    rows = sum(w.shard(1, p, parts).matmul(x[:, p * k:(p + 1) * k].contiguous(), M) for p in range(parts))
    _close(rows, full, 1e-3)
