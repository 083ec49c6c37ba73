"""GPU parity: block decoders and Q8 activation quantization, bit-exact
against the golden vectors and the oracle (through the C ABI)."""
import struct

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

F32, F16, Q4_K, Q6_K, Q8_0, Q2_0C, STQ1_0 = range(7)
ALL = [F32, F16, Q4_K, Q6_K, Q8_0, Q2_0C, STQ1_0]


def to_dev(a, cuda):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def test_golden_vectors_bit_exact(cuda, golden_cases):
    import torch
    from hy_mt_rs_b200 import quant

    for c in golden_cases:
        out = torch.empty(c["bits"].size, dtype=torch.float32, device=cuda)
        quant.decode(c["dtype"], to_dev(c["encoded"], cuda), out)
        got = out.cpu().numpy().view(np.uint32)
        assert np.array_equal(got, c["bits"]), c["name"]


def random_blocks(t, nblocks, rng, special_scales=True):
    bb = O.block_bytes(t)
    raw = rng.integers(0, 256, size=nblocks * bb, dtype=np.uint8).reshape(nblocks, bb)
    if t in (F32, F16):
        return raw.reshape(-1)
    scales = [0.0, -0.0, 1.5, -3.25, 6.1e-5, 5.96e-8, 65504.0, float("inf"), float("nan")]
    offs = {Q4_K: [0, 2], Q6_K: [208], Q8_0: [0], Q2_0C: [0], STQ1_0: [40]}[t]
    for i in range(nblocks):
        for o in offs:
            if special_scales and i < len(scales):
                v = scales[i]
            else:
                v = float(rng.standard_normal() * 0.05)
            raw[i, o:o + 2] = np.frombuffer(struct.pack("<e", v), np.uint8)
    return raw.reshape(-1)


@pytest.mark.parametrize("t", ALL)
def test_decode_matches_oracle_bits(cuda, t):
    import torch
    from hy_mt_rs_b200 import quant

    rng = np.random.default_rng(t)
    nblocks = 777 if t not in (F32, F16) else 5000
    blob = random_blocks(t, nblocks, rng)
    n = nblocks * O.block_len(t)
    ref = O.decode(t, blob, n)
    out = torch.empty(n, dtype=torch.float32, device=cuda)
    quant.decode(t, to_dev(blob, cuda), out)
    got = out.cpu().numpy()
    # Bit-exact for every non-NaN value.  NaN payloads are platform-defined
    # (the reference itself yields different NaN bits on x86 and aarch64;
    # GPU arithmetic returns the canonical NaN), so NaNs compare by position.
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got.view(np.uint32)[~nan], ref.view(np.uint32)[~nan])


def test_decode_shape_errors(cuda):
    import torch
    from hy_mt_rs_b200 import quant

    out = torch.empty(255, dtype=torch.float32, device=cuda)
    with pytest.raises(quant.HyqError):
        quant.decode(Q4_K, torch.zeros(144, dtype=torch.uint8, device=cuda), out)
    out = torch.empty(256, dtype=torch.float32, device=cuda)
    with pytest.raises(quant.HyqError):
        quant.decode(Q4_K, torch.zeros(143, dtype=torch.uint8, device=cuda), out)
    quant.decode(Q4_K, torch.zeros(0, dtype=torch.uint8, device=cuda),
                 torch.empty(0, dtype=torch.float32, device=cuda))


def test_row_into_and_to_vec(cuda):
    import torch
    from hy_mt_rs_b200 import quant, synth

    K, N = 2048, 37
    for t in (Q6_K, Q2_0C, STQ1_0, Q4_K, Q8_0, F32, F16):
        packed = synth.encode(t, synth.random_weights(N, K, 5)).numpy()
        w = quant.Weight(to_dev(packed, cuda), t, [K, N])
        full = O.decode(t, packed, N * K).reshape(N, K)
        assert np.array_equal(w.to_vec().cpu().numpy().reshape(N, K), full)
        for r in (0, 17, N - 1):
            assert np.array_equal(w.row(r).cpu().numpy(), full[r])
        with pytest.raises(quant.HyqError):
            w.row(N)


@pytest.mark.parametrize("n", [1, 15, 16, 17, 255, 256, 257, 1000, 2048, 6144, 6151])
def test_q8_quantize_bit_exact(cuda, n):
    from hy_mt_rs_b200 import quant

    rng = np.random.default_rng(n)
    x = (rng.standard_normal(n) * rng.uniform(0.1, 10)).astype(np.float32)
    if n > 300:
        x[256:512] = 0.0             # an all-zero group: scale 0, no division
        x[600] = 1e30
    q_ref, s_ref, q2_ref = O.q8_quantize(x)
    q8 = quant.Q8.quantize(to_dev(x, cuda))
    assert np.array_equal(q8.values.cpu().numpy(), q_ref)
    assert np.array_equal(q8.scales.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))
    assert np.array_equal(q8.values_q2c.cpu().numpy(), q2_ref)


def test_q8_quantize_special_values(cuda):
    from hy_mt_rs_b200 import quant

    x = np.linspace(-5, 5, 530).astype(np.float32)
    x[3] = np.nan          # vector part of group 0: NaN propagates into the max
    x[300] = np.inf        # group 1: infinite max -> inverse 0
    x[520] = np.nan        # tail of the last group (530 % 16 = 2 -> indices 528, 529)
    x[529] = np.nan
    x[528] = 2.5
    q_ref, s_ref, q2_ref = O.q8_quantize(x)
    q8 = quant.Q8.quantize(to_dev(x, cuda))
    assert np.array_equal(q8.values.cpu().numpy(), q_ref)
    assert np.array_equal(q8.scales.cpu().numpy().view(np.uint32), s_ref.view(np.uint32))
    assert np.array_equal(q8.values_q2c.cpu().numpy(), q2_ref)


def test_dot(cuda):
    from hy_mt_rs_b200 import quant

    for n in [0, 1, 3, 7, 16, 32, 127, 256, 512, 2049]:
        a = np.sin(np.arange(n, dtype=np.float32) * np.float32(0.7)).astype(np.float32)
        b = np.cos(np.arange(n, dtype=np.float32) * np.float32(0.9)).astype(np.float32)
        got = float(quant.dot(to_dev(a, cuda), to_dev(b, cuda)).cpu())
        assert abs(got - O.dot_scalar(a, b)) < 1e-4, n


@pytest.mark.parametrize("t", [2, 3, 4, 5, 6])
def test_synthetic_encoding_same_bytes_on_every_device(cuda, t):
    """hy_mt_rs_b200.synth packs the same bytes on the GPU as on the CPU (the
    config-4 fixture was made on the CPU and the GPU tests rebuild its model
    on the device; both are checked through the model's SHA-256)."""
    import torch
    from hy_mt_rs_b200 import synth

    K = 2048
    for seed in (1, 2):
        cpu = synth.random_packed(t, 300, K, seed=seed)
        gpu = synth.random_packed(t, 300, K, seed=seed, device=cuda).cpu()
        assert torch.equal(cpu, gpu), (t, seed)
