"""GPU check of overlapped launches (hyq_set_launch_overlap): a chain of
batch-1 products in which every product consumes the previous one's output
gives bit-identical results with and without programmatic dependent launch,
eagerly and replayed from a CUDA graph.  A product that read its input before
the preceding kernel finished would break the equality."""
import pytest

pytestmark = pytest.mark.gpu

Q2_0C, STQ1_0, Q6_K = 5, 6, 3


def _layer(cuda, fmt, seed, H=2048, F=6144, KV=512):
    from hy_mt_rs_b200 import quant, synth

    shapes = {"q": (H, H), "k": (KV, H), "v": (KV, H), "o": (H, H), "gate": (F, H), "up": (F, H), "down": (H, F)}
    return {n: quant.Weight(synth.random_packed(fmt, N, K, seed=seed + i, device=cuda), fmt, [K, N], name=n)
            for i, (n, (N, K)) in enumerate(shapes.items())}


def _chain(layers, lm, x, path):
    from hy_mt_rs_b200.quant import Weight

    h = x
    for L in layers:
        if path == "f32":
            q, k, v = Weight.gemv_qkv(L["q"], L["k"], L["v"], h)
            o = L["o"].matmul(q, 1)[0]
            g = L["gate"].matmul_gate_up_silu(L["up"], o)
            h = L["down"].matmul(g, 1)[0]
        else:
            q, k, v = Weight.gemv_qkv_int8(L["q"], L["k"], L["v"], h)
            o = L["o"].gemv_int8(q)
            g = L["gate"].matmul_gate_up_silu_int8(L["up"], o)
            h = L["down"].gemv_int8(g)
    return lm.matmul(h, 1)[0] if path == "f32" else lm.gemv_int8(h)


@pytest.mark.parametrize("path", ["f32", "int8"])
def test_overlapped_chain_is_bit_identical(cuda, path):
    import torch
    from hy_mt_rs_b200 import quant, synth

    layers = [_layer(cuda, Q2_0C, 100), _layer(cuda, STQ1_0, 200)]
    lm = quant.Weight(synth.random_packed(Q6_K, 32768, 2048, seed=7, device=cuda), Q6_K, [2048, 32768])
    x = torch.randn(2048, generator=torch.Generator().manual_seed(1)).to(cuda)
    torch.cuda.synchronize()  # the weights are complete before any overlapped launch
    ref = _chain(layers, lm, x, path).clone()
    stream = torch.cuda.Stream(cuda)
    try:
        quant.set_launch_overlap(True)
        eager = _chain(layers, lm, x, path).clone()
        with torch.cuda.stream(stream):
            _chain(layers, lm, x, path)  # warm plans outside the capture
            stream.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                out = _chain(layers, lm, x, path)
            outs = []
            for _ in range(3):
                g.replay()
                outs.append(out.clone())
        torch.cuda.synchronize()
    finally:
        quant.set_launch_overlap(False)
    assert torch.equal(eager, ref)
    for o in outs:
        assert torch.equal(o, ref)
    assert quant.device_status() == 0
