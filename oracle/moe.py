"""CPU restatement of Moe::forward (hy-mt-rs src/model.rs:688-767) for the
parity tests.  Test infrastructure only: nothing in the product imports it.

Steps and their reference lines:
  router logits      self.router.matmul(input, batch) (model.rs:691); the
                     F32 branch of Weight::matmul (quant.rs:225-238), one x86
                     `dot` per (token, expert), here through the C oracle
  route              route (model.rs:728-767), restated in C (hyo_moe_route)
  assignments        experts ascending, tokens ascending (model.rs:693-701)
  shared + experts   DenseFfn::forward (model.rs:673-685) in f64 from the
                     decoded weights: silu(g) * u then down
  combine            output = shared; output[token] += weight * value in
                     expert order (model.rs:703-723), f32 roundings

The expert products of the reference's batched path go through Candle's CPU
GEMM (not in the reference tree), whose summation order is not restated, so
the products here are f64 and the comparison is within a tolerance.  The
routing and the combine are exact restatements.
"""
import numpy as np

from . import oracle as O

F32 = 0


def router_logits(router_bytes, hidden, experts, x):
    """[tokens, experts]: each logit the batch-1 F32 row product (x86 dot)."""
    x = np.ascontiguousarray(np.atleast_2d(x), dtype=np.float32)
    return np.stack([O.matmul(F32, router_bytes, hidden, experts, x[t], 1)[0] for t in range(x.shape[0])])


def _dense_f64(t, gate, up, down, K, mid, x):
    """DenseFfn::forward in f64: [tokens, K] -> [tokens, K]."""
    wg = O.decode(t, gate, mid * K).reshape(mid, K).astype(np.float64)
    wu = O.decode(t, up, mid * K).reshape(mid, K).astype(np.float64)
    wd = O.decode(t, down, K * mid).reshape(K, mid).astype(np.float64)
    x64 = np.atleast_2d(x).astype(np.float64)
    g = x64 @ wg.T
    u = x64 @ wu.T
    h = g / (1.0 + np.exp(-g)) * u
    return h @ wd.T


def moe_forward(cfg, w, x, routing=None):
    """Moe::forward of x [tokens, hidden] (numpy f32).  `w`: numpy copies of
    hy_mt_rs_b200.moe.random_moe_weights.  `routing` (indices, weights)
    replaces the routing step (to follow the device's choices at a near-tie).
    Returns (output [tokens, hidden] f32, indices, weights)."""
    H, E, M, S, t = cfg.hidden, cfg.experts, cfg.mid, cfg.shared_mid, cfg.dtype
    x = np.ascontiguousarray(np.atleast_2d(x), dtype=np.float32)
    T = x.shape[0]
    if routing is None:
        logits = router_logits(w["router"], H, E, x)
        idx, wt = O.moe_route(logits, w["bias"], cfg.used, cfg.normalize, cfg.scale)
    else:
        idx, wt = routing
    out = _dense_f64(t, w["shared_gate"], w["shared_up"], w["shared_down"], H, S, x).astype(np.float32)
    rb_gu = O.block_bytes(t) * H // O.block_len(t)      # bytes per gate/up row
    rb_d = O.block_bytes(t) * M // O.block_len(t)       # bytes per down row
    for e in range(E):
        tokens = [(tok, wt[tok, k]) for tok in range(T) for k in range(cfg.used) if idx[tok, k] == e]
        if not tokens:
            continue
        g = w["gate"][e * M * rb_gu:(e + 1) * M * rb_gu]
        u = w["up"][e * M * rb_gu:(e + 1) * M * rb_gu]
        d = w["down"][e * H * rb_d:(e + 1) * H * rb_d]
        rows = np.array([tok for tok, _ in tokens])
        res = _dense_f64(t, g, u, d, H, M, x[rows]).astype(np.float32)
        for (tok, weight), row in zip(tokens, res):
            out[tok] = (out[tok] + (np.float32(weight) * row).astype(np.float32)).astype(np.float32)
    return out, idx, wt


def moe_forward_port(cfg, w, x, threads=0):
    """Moe::forward with the reference's own structure at f32 (the CPU
    baseline): router matmul, host routing, then for each expert in order its
    tokens' DenseFfn::forward (gate and up matmuls, silu(g) * u, down matmul;
    quant.rs batch paths as restated in hyo_matmul), then the combine."""
    H, E, M, S, t = cfg.hidden, cfg.experts, cfg.mid, cfg.shared_mid, cfg.dtype
    x = np.ascontiguousarray(np.atleast_2d(x), dtype=np.float32)
    T = x.shape[0]

    def dense(g, u, d, K, mid, xs):
        n = xs.shape[0]
        gg = O.matmul(t, g, K, mid, xs, n, threads)
        uu = O.matmul(t, u, K, mid, xs, n, threads)
        h = (gg / (np.float32(1) + np.exp(-gg)) * uu).astype(np.float32)
        return O.matmul(t, d, mid, K, h, n, threads)

    logits = O.matmul(F32, w["router"], H, E, x, T, threads)
    idx, wt = O.moe_route(logits, w["bias"], cfg.used, cfg.normalize, cfg.scale)
    out = dense(w["shared_gate"], w["shared_up"], w["shared_down"], H, S, x)
    rb_gu = O.block_bytes(t) * H // O.block_len(t)
    rb_d = O.block_bytes(t) * M // O.block_len(t)
    for e in range(E):
        hits = [(tok, wt[tok, k]) for tok in range(T) for k in range(cfg.used) if idx[tok, k] == e]
        if not hits:
            continue
        rows = np.array([tok for tok, _ in hits])
        res = dense(w["gate"][e * M * rb_gu:(e + 1) * M * rb_gu], w["up"][e * M * rb_gu:(e + 1) * M * rb_gu],
                    w["down"][e * H * rb_d:(e + 1) * H * rb_d], H, M, x[rows])
        for (tok, weight), row in zip(hits, res):
            out[tok] = (out[tok] + (np.float32(weight) * row).astype(np.float32)).astype(np.float32)
    return out
