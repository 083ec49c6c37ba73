"""Seeded synthetic weights in the packed GGUF formats.

hy-mt-rs has no weight quantizers (only the Q8 activation quantizer,
quant.rs:904), so these encoders are written for this library: they only
shape value distributions for tests and benchmarks.  Parity never depends on
them: kernels and oracle always consume the same packed bytes.

All encoders take f32 weights [N, K] (rows x input width) on any torch device
and return the packed rows as a flat uint8 tensor on the same device, laid
out exactly as the decoders of quant.rs:2405-2486 read them.
"""
import torch

__all__ = ["encode", "random_weights", "random_packed", "row_bytes"]

# DType values and their block geometry (quant.rs:19-27, 43-62), kept here so
# that synthesising weights needs no GPU library (the CPU benchmark arms and
# the fixture scripts import this module without loading libhyq.so).
F32, F16, Q4_K, Q6_K, Q8_0, Q2_0C, STQ1_0 = range(7)
_GEOMETRY = {F32: (1, 4), F16: (1, 2), Q4_K: (256, 144), Q6_K: (256, 210), Q8_0: (32, 34), Q2_0C: (512, 130),
             STQ1_0: (256, 42)}


def _block(dtype):
    if int(dtype) not in _GEOMETRY:
        raise ValueError(f"unsupported tensor type {dtype}")
    return _GEOMETRY[int(dtype)]


def row_bytes(dtype, K):
    bl, bb = _block(dtype)
    return K // bl * bb


def _f16_bytes(v):
    """f32 tensor [...] -> uint8 [..., 2] little-endian binary16."""
    return v.to(torch.float16).contiguous().view(torch.uint8).reshape(*v.shape, 2)


def _f16_round(v):
    return v.to(torch.float16).to(torch.float32)


def _div(a, c):
    """a / c, divided (IEEE) on every device: a CUDA tensor divided by a
    Python scalar is multiplied by the scalar's reciprocal instead, which
    rounds differently; a 0-dim tensor on a's device divides."""
    return a / torch.full((), c, dtype=a.dtype, device=a.device)


def _safe_div(a, b):
    return torch.where(b != 0, a / torch.where(b != 0, b, torch.ones_like(b)), torch.zeros_like(a))


def _q8_0(w):
    N, K = w.shape
    b = w.reshape(N, K // 32, 32)
    d = _f16_round(_div(b.abs().amax(-1), 127.0))
    q = torch.round(_safe_div(b, d[..., None])).clamp(-127, 127).to(torch.int8)
    out = torch.cat([_f16_bytes(d), q.view(torch.uint8)], dim=-1)
    return out.reshape(-1)


def _q2_0c(w):
    N, K = w.shape
    b = w.reshape(N, K // 512, 512)
    d = _f16_round(_div(b.abs().amax(-1), 3.0))
    c = torch.round(_div(_safe_div(b, d[..., None]) + 3.0, 2.0)).clamp(0, 3).to(torch.int32)
    c = c.reshape(N, K // 512, 128, 4)
    payload = (c[..., 0] | (c[..., 1] << 2) | (c[..., 2] << 4) | (c[..., 3] << 6)).to(torch.uint8)
    return torch.cat([_f16_bytes(d), payload], dim=-1).reshape(-1)


def _stq1_0(w):
    N, K = w.shape
    nb = K // 256
    b = w.reshape(N, nb, 4, 4, 16)  # [.., chunk, lane p, group-in-chunk j]; column 64c + 16p + j
    # summed in f64 so that the order of the device's reduction cannot change the f32 mean
    d = _f16_round(b.abs().double().mean(dim=(-1, -2, -3)).float())
    lanes = b.permute(0, 1, 2, 4, 3).reshape(N, nb, 64, 4)  # group g = 16c + j, lanes p
    z = lanes.abs().argmin(dim=-1)  # the zero lane
    neg = lanes < 0
    # signs of the three non-zero lanes in lane order
    order = torch.arange(4, device=w.device).expand(N, nb, 64, 4)
    keep = order != z[..., None]
    nz_neg = neg[keep].reshape(N, nb, 64, 3)
    s_global = nz_neg[..., 0]
    t0 = nz_neg[..., 1] ^ s_global
    t1 = nz_neg[..., 2] ^ s_global
    nib = (z.to(torch.int32) << 2) | (t1.to(torch.int32) << 1) | t0.to(torch.int32)
    sign = s_global.to(torch.int32)
    nib2 = nib.reshape(N, nb, 32, 2)
    codes = (nib2[..., 0] | (nib2[..., 1] << 4)).to(torch.uint8)
    s8 = sign.reshape(N, nb, 8, 8)
    shifts = torch.arange(8, device=w.device, dtype=torch.int32)
    sbytes = (s8 << shifts).sum(-1).to(torch.uint8)
    return torch.cat([codes, sbytes, _f16_bytes(d)], dim=-1).reshape(-1)


def _q4_k(w):
    N, K = w.shape
    nb = K // 256
    sub = w.reshape(N, nb, 8, 32)
    mn = sub.amin(-1).clamp(max=0.0)
    mx = sub.amax(-1)
    scale = _div(mx - mn, 15.0)
    minv = -mn
    d = _f16_round(_div(scale.amax(-1), 63.0))
    dmin = _f16_round(_div(minv.amax(-1), 63.0))
    s6 = torch.round(_safe_div(scale, d[..., None])).clamp(0, 63).to(torch.int32)
    m6 = torch.round(_safe_div(minv, dmin[..., None])).clamp(0, 63).to(torch.int32)
    eff_s = d[..., None] * s6.to(torch.float32)
    eff_m = dmin[..., None] * m6.to(torch.float32)
    q = torch.round(_safe_div(sub + eff_m[..., None], eff_s[..., None])).clamp(0, 15).to(torch.int32)
    sc = torch.zeros(N, nb, 12, dtype=torch.int32, device=w.device)
    sc[..., 0:4] = s6[..., 0:4] | ((s6[..., 4:8] >> 4) << 6)
    sc[..., 4:8] = m6[..., 0:4] | ((m6[..., 4:8] >> 4) << 6)
    sc[..., 8:12] = (s6[..., 4:8] & 15) | ((m6[..., 4:8] & 15) << 4)
    qg = q.reshape(N, nb, 4, 2, 32)  # group g: sub-block 2g (low nibble), 2g+1 (high)
    qs = (qg[..., 0, :] | (qg[..., 1, :] << 4)).reshape(N, nb, 128).to(torch.uint8)
    out = torch.cat([_f16_bytes(d), _f16_bytes(dmin), sc.to(torch.uint8), qs], dim=-1)
    return out.reshape(-1)


def _q6_k(w):
    N, K = w.shape
    nb = K // 256
    sub = w.reshape(N, nb, 16, 16)  # sub-block s covers outputs 16s..16s+15 -> scale sc[s]
    scale = _div(sub.abs().amax(-1), 31.0)
    d = _f16_round(_div(scale.abs().amax(-1), 127.0))
    sc = torch.round(_safe_div(scale, d[..., None])).clamp(-128, 127).to(torch.int32)
    eff = d[..., None] * sc.to(torch.float32)
    q = (torch.round(_safe_div(sub, eff[..., None])).clamp(-32, 31) + 32).to(torch.int32)
    q = q.reshape(N, nb, 2, 4, 2, 16)  # chunk, p, half, i
    lo = q & 15
    ql = lo[:, :, :, 0:2] | (lo[:, :, :, 2:4] << 4)  # [.., chunk, p&1, half, i]
    ql = ql.reshape(N, nb, 2, 64)
    hi = (q >> 4) & 3
    qh = hi[:, :, :, 0] | (hi[:, :, :, 1] << 2) | (hi[:, :, :, 2] << 4) | (hi[:, :, :, 3] << 6)  # [.., chunk, half, i]
    qh = qh.reshape(N, nb, 2, 32)
    out = torch.cat([ql.reshape(N, nb, 128).to(torch.uint8), qh.reshape(N, nb, 64).to(torch.uint8),
                     sc.to(torch.int8).view(torch.uint8), _f16_bytes(d)], dim=-1)
    return out.reshape(-1)


def encode(dtype, w):
    """Pack f32 weights [N, K] into `dtype` rows (flat uint8 tensor)."""
    dtype = int(dtype)
    bl = _block(dtype)[0]
    w = w.to(torch.float32).contiguous()
    N, K = w.shape
    if K % bl:
        raise ValueError(f"K={K} is not a multiple of {bl}")
    if dtype == F32:
        return w.view(torch.uint8).reshape(-1).clone()
    if dtype == F16:
        return w.to(torch.float16).view(torch.uint8).reshape(-1).clone()
    fn = {Q8_0: _q8_0, Q2_0C: _q2_0c, STQ1_0: _stq1_0, Q4_K: _q4_k, Q6_K: _q6_k}
    out = fn[dtype](w)
    assert out.numel() == N * row_bytes(dtype, K)
    return out


def random_weights(N, K, seed, std=0.02, device="cpu"):
    g = torch.Generator(device="cpu").manual_seed(int(seed))
    return (torch.randn(N, K, generator=g) * std).to(device)


def random_packed(dtype, N, K, seed, std=0.02, device="cpu", chunk_rows=16384):
    """Seeded N(0, std) weights packed as `dtype`; encoded in row chunks."""
    parts = []
    g = torch.Generator(device="cpu").manual_seed(int(seed))
    for r0 in range(0, N, chunk_rows):
        n = min(chunk_rows, N - r0)
        w = (torch.randn(n, K, generator=g) * std).to(device)
        parts.append(encode(dtype, w))
    return torch.cat(parts)
