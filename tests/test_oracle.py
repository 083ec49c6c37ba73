"""CPU checks of the oracle: pinned to the reference's golden decoder vectors
and to ports of the reference's own unit-test known answers
(hy-mt-rs src/quant.rs:2598-3090, tests/quant_reference.rs)."""
import math
import struct

import numpy as np
import pytest

from oracle import oracle as O

F32, F16, Q4_K, Q6_K, Q8_0, Q2_0C, STQ1_0 = range(7)


def f16_bytes(v):
    return struct.pack("<e", v)


def test_golden_decoders_bit_exact(golden_cases):
    """tests/quant_reference.rs:12-50: exact f32 bits, then dot within
    1e-3 + 1e-4 |ref| of an f64 oracle."""
    assert {c["name"] for c in golden_cases} == {"Q8_0", "Q4_K", "Q6_K", "Q2_0C", "STQ1_0"}
    for c in golden_cases:
        out = O.decode(c["dtype"], c["encoded"], c["bits"].size)
        assert np.array_equal(out.view(np.uint32), c["bits"]), c["name"]
        x = np.sin(np.arange(out.size, dtype=np.float32) * np.float32(0.17)).astype(np.float32)
        ref = float(np.dot(c["bits"].view(np.float32).astype(np.float64), x.astype(np.float64)))
        got = O.dot(out, x)
        assert abs(ref - got) < 1e-3 + 1e-4 * abs(ref), c["name"]


def test_block_geometry_and_profiles():
    """quant.rs:30-62 and ambiguous_ids_need_the_matching_profile (:3081)."""
    assert [O.block_len(t) for t in range(7)] == [1, 1, 256, 256, 32, 512, 256]
    assert [O.block_bytes(t) for t in range(7)] == [4, 2, 144, 210, 34, 130, 42]
    assert O.dtype_from_id(40, 1) == -1
    assert O.dtype_from_id(42, 2) == -1
    assert O.dtype_from_id(42, 3) == STQ1_0
    assert O.dtype_from_id(40, 2) == Q2_0C
    assert [O.dtype_from_id(i, 1) for i in (0, 1, 8, 12, 14)] == [F32, F16, Q8_0, Q4_K, Q6_K]


def test_q2_codes_and_scale():
    """quant.rs:2602-2612."""
    block = bytearray([0b11100100] * 130)
    block[:2] = f16_bytes(0.5)
    out = O.decode(Q2_0C, np.frombuffer(bytes(block), np.uint8), 512)
    assert np.array_equal(out.reshape(-1, 4), np.tile([-1.5, -0.5, 0.5, 1.5], (128, 1)).astype(np.float32))


def stq_all_patterns_block():
    block = bytearray(42)
    block[40:42] = f16_bytes(2.0)
    for g in range(64):
        block[g // 2] |= (g % 16) << (4 * (g % 2))
        block[32 + g // 8] |= ((g // 16) % 2) << (g % 8)
    return np.frombuffer(bytes(block), np.uint8)


def stq_expected(g, p):
    zero = (g % 16) // 4
    tail = g % 4
    if p == zero:
        return 0.0
    nz = p if p < zero else p - 1
    sign = 1.0 if nz == 0 or (tail & (1 << (nz - 1))) == 0 else -1.0
    return sign * (2.0 if (g // 16) % 2 == 0 else -2.0)


def test_stq_all_patterns_and_stride():
    """quant.rs:2614-2644: every codebook entry and the stride-16 placement."""
    out = O.decode(STQ1_0, stq_all_patterns_block(), 256)
    for g in range(64):
        for p in range(4):
            assert out[g // 16 * 64 + g % 16 + 16 * p] == stq_expected(g, p), (g, p)


def test_dot_matches_scalar_with_tails():
    """quant.rs:2646-2654."""
    for n in [0, 1, 3, 7, 16, 32, 127, 256, 512, 2049]:
        a = np.sin(np.arange(n, dtype=np.float32) * np.float32(0.7)).astype(np.float32)
        b = np.cos(np.arange(n, dtype=np.float32) * np.float32(0.9)).astype(np.float32)
        assert abs(O.dot(a, b) - O.dot_scalar(a, b)) < 1e-4, n


def _seeded(seed, mul, step, n, skip=0, take=None):
    vals = [((seed * mul + i * step) & 0xFFFFFFFF) & 0xFF for i in range(n)]
    return vals


@pytest.mark.parametrize("seed", range(64))
def test_fused_row_dots_match_decode(seed):
    """quant.rs:2656-2711 (fused STQ / Q6_K / Q2_0C row dots vs decode + dot)."""
    # STQ (:2657-2672)
    blk = bytearray(42)
    for i in range(40):
        blk[i] = ((seed * 2654435761 + i * 7) & 0xFFFFFFFF) & 0xFF
    blk[40:42] = f16_bytes(1.0 + math.fmod(seed, 0.5))
    x = np.cos((np.arange(256, dtype=np.float32) + np.float32(seed)) * np.float32(0.31)).astype(np.float32)
    b = np.frombuffer(bytes(blk), np.uint8)
    dec = O.decode(STQ1_0, b, 256)
    assert abs(O.row_dot_f32(STQ1_0, b, x) - O.dot(dec, x)) < 1e-3
    # Q6_K (:2675-2690)
    blk = bytearray(210)
    for i in range(208):
        blk[i] = ((seed * 40503 + i * 13) & 0xFFFFFFFF) & 0xFF
    blk[208:210] = f16_bytes(0.25 + math.fmod(seed, 0.75))
    x = np.sin((np.arange(256, dtype=np.float32) + np.float32(seed)) * np.float32(0.17)).astype(np.float32)
    b = np.frombuffer(bytes(blk), np.uint8)
    assert abs(O.row_dot_f32(Q6_K, b, x) - O.dot(O.decode(Q6_K, b, 256), x)) < 1e-3
    # Q2_0C (:2693-2711)
    blk = bytearray(130)
    for i in range(2, 130):
        blk[i] = ((seed * 40503 + i * 13) & 0xFFFFFFFF) & 0xFF
    blk[0:2] = f16_bytes(0.25 + math.fmod(seed, 0.75))
    x = np.sin((np.arange(512, dtype=np.float32) + np.float32(seed)) * np.float32(0.17)).astype(np.float32)
    b = np.frombuffer(bytes(blk), np.uint8)
    assert abs(O.row_dot_f32(Q2_0C, b, x) - O.dot(O.decode(Q2_0C, b, 512), x)) < 1e-3


def test_int8_activation_groups_round_trip():
    """quant.rs:2955-2978."""
    values = (np.sin(np.arange(1024, dtype=np.float32) * np.float32(0.37)) * np.float32(3.0)).astype(np.float32)
    q, s, _ = O.q8_quantize(values)
    assert q.size == 1024 and s.size == 4
    for g in range(4):
        restored = q[g * 256:(g + 1) * 256].astype(np.float32) * s[g]
        assert np.all(np.abs(restored - values[g * 256:(g + 1) * 256]) <= s[g] * 0.5 + 1e-6)
    q, s, _ = O.q8_quantize(np.zeros(256, np.float32))
    assert s.tolist() == [0.0] and not q.any()


@pytest.mark.parametrize("seed", range(8))
def test_sdot_kernels_match_int8_reference(seed):
    """quant.rs:2980-3079: SDOT row dots within 1e-5 of the f64 magnitude."""
    x = (np.sin((np.arange(512, dtype=np.float32) + np.float32(seed)) * np.float32(0.11)) * np.float32(2.0))
    x = x.astype(np.float32)
    x[:256] *= np.float32(1.0)
    x[256:] *= np.float32(2.0)
    q, s, q2c = O.q8_quantize(x)

    def check(t, blob, n):
        b = np.frombuffer(bytes(blob), np.uint8)
        w = O.decode(t, b, n).astype(np.float64)
        terms = w * q[:n].astype(np.float64) * s[np.arange(n) // 256].astype(np.float64)
        got = O.row_dot_q8(t, b, n, q[:n], s, q2c[:n])
        assert abs(got - terms.sum()) <= np.abs(terms).sum() * 1e-5, (t, got, terms.sum())

    stq = bytearray(((seed * 2654435761 + i * 7) & 0xFFFFFFFF) & 0xFF for i in range(84))
    stq[40:42] = f16_bytes(0.5)
    stq[82:84] = f16_bytes(0.25)
    check(STQ1_0, stq, 512)
    q6 = bytearray(((seed * 40503 + i * 13) & 0xFFFFFFFF) & 0xFF for i in range(420))
    q6[208:210] = f16_bytes(0.125)
    q6[418:420] = f16_bytes(0.75)
    check(Q6_K, q6, 512)
    q2 = bytearray(((seed * 40503 + i * 13) & 0xFFFFFFFF) & 0xFF for i in range(130))
    q2[0:2] = f16_bytes(0.375)
    check(Q2_0C, q2, 512)


def test_q8_deinterleave_layout():
    """deinterleave_q2c (quant.rs:945-963): t[k*16+j] = s[4j+k] per full 64 chunk."""
    x = np.linspace(-3, 3, 200, dtype=np.float32)
    q, s, q2c = O.q8_quantize(x)
    for c in range(200 // 64):
        for k in range(4):
            for j in range(16):
                assert q2c[c * 64 + 16 * k + j] == q[c * 64 + 4 * j + k]
    assert np.array_equal(q2c[192:], q[192:])


def test_q8_tail_rounds_half_away():
    """Scalar tail of quantize_group_neon (quant.rs:987-989) uses round()
    half-away-from-zero; the vector part rounds to nearest even."""
    # max 127 -> inverse 1.0, so x * inverse is x itself.
    x = np.zeros(20, dtype=np.float32)
    x[0] = 127.0
    x[1] = 2.5   # vector part: rne -> 2
    x[17] = 2.5  # tail (index >= 16): half away -> 3
    x[18] = -2.5
    q, s, _ = O.q8_quantize(x)
    assert s[0] == np.float32(1.0)
    assert q[1] == 2 and q[17] == 3 and q[18] == -3


def test_decode_rejects_bad_shapes():
    """decode (quant.rs:1066-1079) errors."""
    with pytest.raises(ValueError):
        O.decode(Q4_K, np.zeros(144, np.uint8), 255)  # partial block
    with pytest.raises(ValueError):
        O.decode(Q4_K, np.zeros(143, np.uint8), 256)  # wrong byte count
    assert O.decode(Q4_K, np.zeros(0, np.uint8), 0).size == 0


def test_matmul_batch_paths_agree():
    """The three batch branches of Weight::matmul agree to f32 rounding."""
    from hy_mt_rs_b200 import synth  # host-only encoder (torch CPU)

    K, N = 512, 40
    for t in (Q4_K, Q6_K, Q2_0C, STQ1_0, Q8_0):
        w = synth.encode(t, synth.random_weights(N, K, 3)).numpy()
        x = np.random.default_rng(0).standard_normal((9, K)).astype(np.float32)
        y1 = np.stack([O.matmul(t, w, K, N, x[b], 1)[0] for b in range(9)])
        y3 = O.matmul(t, w, K, N, x[:3].ravel(), 3)
        y9 = O.matmul(t, w, K, N, x.ravel(), 9)
        mag = np.abs(O.decode(t, w, N * K).reshape(N, K)).sum(1) * np.abs(x).max()
        assert np.all(np.abs(y3 - y1[:3]) <= 1e-5 * mag + 1e-6)
        assert np.all(np.abs(y9 - y1) <= 1e-5 * mag + 1e-6)


def test_moe_route_matches_sort_semantics():
    """hyo_moe_route (route, model.rs:728-767) against a Python restatement
    with sorted(): total_cmp order of sigmoid + bias, ties to the lower
    index, normalized weights with the f16 MIN_POSITIVE floor."""
    import struct

    def total_key(v):
        b = struct.unpack("<i", struct.pack("<f", float(v)))[0]
        return b ^ ((b >> 31) & 0x7FFFFFFF)

    rng = np.random.default_rng(5)
    E, used = 64, 8
    logits = rng.standard_normal((20, E)).astype(np.float32) * 3
    logits[0, :] = 0.0                       # every key tied: lowest indices win
    logits[1, 5] = -100.0                    # sigmoid underflows toward 0
    bias = (rng.standard_normal(E) * 0.1).astype(np.float32)
    bias[7] = bias[9] = np.float32(0.0)
    for normalize, scale in ((True, 2.5), (False, 1.0)):
        idx, w = O.moe_route(logits, bias, used, normalize, scale)
        for t in range(logits.shape[0]):
            x = logits[t]
            sig = np.where(x >= 0, np.float32(1) / (np.float32(1) + np.exp(-x)),
                           np.exp(x) / (np.float32(1) + np.exp(x))).astype(np.float32)
            keys = (sig + bias).astype(np.float32)
            order = sorted(range(E), key=lambda i: (-total_key(keys[i]), i))[:used]
            assert list(idx[t]) == order, t
            s = np.float32(0)
            for i in order:
                s = np.float32(s + sig[i])
            s = max(s, np.float32(6.103515625e-05)) if normalize else np.float32(1)
            ref = np.array([np.float32(np.float32(sig[i] / s) * np.float32(scale)) for i in order], np.float32)
            np.testing.assert_allclose(w[t], ref, rtol=2e-7)
    idx0, _ = O.moe_route(logits[:1], np.zeros(E, np.float32), used, True, 1.0)
    assert list(idx0[0]) == list(range(used))
