"""Single-token decode of the Dense architecture (Hy-MT2: model.rs:374-547)
on the device, through libhyq only: embedding row, per layer RMSNorm -> QKV
-> RoPE + q/k norm + KV append -> attention -> O + residual -> RMSNorm ->
gate/up-SiLU -> down + residual, then the output norm, the lm_head product
and the greedy argmax.  The position and the token live in device memory,
so one captured CUDA graph replays a whole token step.

The HyV3 architecture (hy_v3, model.rs:139-140, 210-231) runs through the
same runner: the q/k RMSNorm before RoPE (model.rs:425-428), the MoE FFN
(Moe::forward, model.rs:684-726; hy_mt_rs_b200.moe.MoeLayer) in every layer
but the first, and an output matrix of its own.

Weights are packed GGUF bytes (any hyq_dtype for the linears; the embedding
is tied to the lm_head as in the 1.8B model); norms are f32.  The KV cache is
f32, as in the reference (model.rs:116-120).
"""
import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from . import quant
from ._native import check, lib


@dataclass
class DenseConfig:
    layers: int = 32
    hidden: int = 2048
    heads: int = 16
    kv_heads: int = 4
    head_dim: int = 128
    ffn: int = 6144
    vocab: int = 120832
    rope_base: float = 10000.0
    eps: float = 1e-5
    positions: int = 512        # KV-cache capacity (prompt + generated tokens)
    linear_dtype: int = 5       # Q2_0C
    embed_dtype: int = 3        # Q6_K
    # "dense" (hunyuan-dense) or "hyv3" (hy_v3: MoE FFN from layer 1, q/k
    # norm before RoPE, separate output matrix); MoE shapes for hyv3
    arch: str = "dense"
    experts: int = 64
    experts_used: int = 8
    expert_ffn: int = 1024
    shared_ffn: int = 1024
    expert_scale: float = 1.0
    expert_normalize: bool = True
    expert_dtype: int = 2       # Q4_K

    def moe_config(self):
        from .moe import MoeConfig
        return MoeConfig(hidden=self.hidden, experts=self.experts, used=self.experts_used, mid=self.expert_ffn,
                         shared_mid=self.shared_ffn, normalize=self.expert_normalize, scale=self.expert_scale,
                         dtype=self.expert_dtype)


def random_weights(cfg, device, seed=0):
    """Seeded random-init weights of the architecture: N(0, 0.02) linears
    packed by hy_mt_rs_b200.synth, norms 1 + N(0, 0.02)."""
    from . import synth

    H, A, KV, F = cfg.hidden, cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim, cfg.ffn
    g = torch.Generator().manual_seed(seed)

    def norm(n):
        return (1.0 + 0.02 * torch.randn(n, generator=g)).to(device)

    shapes = {"q": (A, H), "k": (KV, H), "v": (KV, H), "o": (H, A), "gate": (F, H), "up": (F, H), "down": (H, F)}
    layers = []
    for i in range(cfg.layers):
        moe = cfg.arch == "hyv3" and i > 0   # HyV3: every layer but the first (model.rs:210)
        L = {n: synth.random_packed(cfg.linear_dtype, N, K, seed=seed + 1000 * i + j, device=device)
             for j, (n, (N, K)) in enumerate(shapes.items()) if not (moe and n in ("gate", "up", "down"))}
        if moe:
            from .moe import random_moe_weights
            L["moe"] = random_moe_weights(cfg.moe_config(), device, seed=seed + 1000 * i + 500)
        L.update(input_norm=norm(H), ffn_norm=norm(H), q_norm=norm(cfg.head_dim), k_norm=norm(cfg.head_dim))
        layers.append(L)
    embed = synth.random_packed(cfg.embed_dtype, cfg.vocab, H, seed=seed + 7, device=device)
    out = {"layers": layers, "embed": embed, "output_norm": norm(H), "shapes": shapes}
    if cfg.arch == "hyv3":   # HyV3 requires separate output weights (model.rs:198-201)
        out["output"] = synth.random_packed(cfg.embed_dtype, cfg.vocab, H, seed=seed + 9, device=device)
    return out


def weights_digest(weights):
    """SHA-256 over a random_weights() dict: every layer's packed linears
    (q, k, v, o, gate, up, down) and f32 norms in that order, then the
    embedding and the output norm.  Identifies the model bytes on any device
    (the parity fixtures record it)."""
    import hashlib

    h = hashlib.sha256()

    def add(t):
        h.update(t.detach().contiguous().cpu().numpy().tobytes())

    for L in weights["layers"]:
        for n in ("q", "k", "v", "o", "gate", "up", "down", "input_norm", "ffn_norm", "q_norm", "k_norm"):
            if n in L:
                add(L[n])
        for n in sorted(L.get("moe", {})):
            add(L["moe"][n])
    add(weights["embed"])
    if weights.get("output") is not None:
        add(weights["output"])
    add(weights["output_norm"])
    return h.hexdigest()


def _p(t):
    return C.c_void_p(t.data_ptr())


PREFILL_CHUNK = 256  # tokens per batched forward (model.rs:18, 353)
_F32, _Q8 = 0, 1     # HYQ_ACT_F32, HYQ_ACT_Q8
# weight types whose single-token products take Q8 activations on the
# reference's aarch64 SDOT branch (model.rs:403-404)
_SDOT_TYPES = (quant.DType.STQ1_0, quant.DType.Q6_K, quant.DType.Q2_0C)


class _DenseLayerDesc(C.Structure):
    """hyq_dense_layer (include/hyq.h)."""
    _fields_ = [(n, C.c_void_p) for n in ("q", "k", "v", "o", "gate", "up", "down", "input_norm", "ffn_norm",
                                          "q_norm", "k_norm", "k_cache", "v_cache")]


class _DenseStepDesc(C.Structure):
    """hyq_dense_step_desc (include/hyq.h)."""
    _fields_ = [("layers", C.c_int), ("hidden", C.c_int), ("heads", C.c_int), ("kv_heads", C.c_int),
                ("head_dim", C.c_int), ("ffn", C.c_int), ("positions", C.c_int64), ("eps", C.c_float),
                ("layer", C.c_void_p), ("embed", C.c_void_p), ("output_norm", C.c_void_p), ("cos_tab", C.c_void_p),
                ("sin_tab", C.c_void_p), ("hidden_state", C.c_void_p), ("q", C.c_void_p), ("k", C.c_void_p),
                ("v", C.c_void_p), ("attended", C.c_void_p), ("gate", C.c_void_p), ("logits", C.c_void_p),
                ("token", C.c_void_p), ("pos", C.c_void_p)]


# The batched forward's residual adds and RMSNorms (model.rs:569-616): with
# split-operand products inside the products' activation conversions
# (hyq_matmul_*_norm, one launch fewer each); with fp16 operands as the
# separate add + norm kernel, which measured faster there (fusing gate/up's
# norm added 0.38 ms to a 64-request step).  hidden += delta when delta is
# given (a pointer), then the product of RMSNorm(hidden) * norm_w; the same
# bits either way.
def _add_norm(hidden, delta, norm_w, K, M, eps, normalized, st):
    if delta is None:
        check(lib.hyq_rms_norm(hidden, norm_w, K, M, eps, normalized, st))
    else:
        check(lib.hyq_add_rms_norm(hidden, delta, norm_w, K, M, eps, normalized, st))


def _qkv_normed(fused, W, hidden, delta, norm_w, eps, M, normalized, outs, st):
    if fused:
        check(lib.hyq_matmul_qkv_norm(W["q"].handle, W["k"].handle, W["v"].handle, hidden, delta, norm_w, eps, M,
                                      *outs, st))
    else:
        _add_norm(hidden, delta, norm_w, W["q"].shape()[0], M, eps, normalized, st)
        check(lib.hyq_matmul_qkv(W["q"].handle, W["k"].handle, W["v"].handle, normalized, M, *outs, st))


def _gate_up_normed(fused, W, hidden, delta, norm_w, eps, M, normalized, out, st):
    if fused:
        check(lib.hyq_matmul_gate_up_silu_norm(W["gate"].handle, W["up"].handle, hidden, delta, norm_w, eps, M, out,
                                               st))
    else:
        _add_norm(hidden, delta, norm_w, W["gate"].shape()[0], M, eps, normalized, st)
        check(lib.hyq_matmul_gate_up_silu_batch(W["gate"].handle, W["up"].handle, normalized, M, out, st))


def _matmul_normed(fused, w, hidden, delta, norm_w, eps, M, normalized, out, st):
    if fused:
        check(lib.hyq_matmul_norm(w.handle, hidden, delta, norm_w, eps, M, out, st))
    else:
        _add_norm(hidden, delta, norm_w, w.shape()[0], M, eps, normalized, st)
        check(lib.hyq_matmul(w.handle, normalized, M, out, st))


class _Acts:
    """Activation buffers of a forward over M tokens (rows)."""

    def __init__(self, cfg, M, device):
        H, A, KV, F = cfg.hidden, cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim, cfg.ffn
        z = lambda *n: torch.zeros(*n, device=device)  # noqa: E731
        self.M = M
        self.hidden, self.normalized, self.attended = z(M, H), z(M, H), z(M, A)
        self.projected, self.ff, self.gate = z(M, H), z(M, H), z(M, F)
        self.q, self.k, self.v = z(M, A), z(M, KV), z(M, KV)


class DenseModel:
    """fused: run each token step as one persistent kernel
    (hyq_dense_step_enqueue) instead of 8 launches per layer.
    rope_in_attention: single-token steps run RoPE + q/k norm + KV append
    inside the attention launch (hyq_rope_attention, bit-identical to
    hyq_rope_qk + hyq_attention).  Off by default: every split CTA then
    repeats the query heads' norm and RoPE on its own critical path, which
    measured slower than the separate launch (1.318 vs 1.302 ms per token
    with one query head per CTA and f32 KV, 3.89 vs 3.69 ms per step of 64
    requests).
    gemm_precision: arithmetic of the batched products (prompt chunks of 16
    tokens and more, DenseBatch steps of 16 requests and more):
    quant.GEMM_FP16 (fp16 operands, the fastest) or quant.GEMM_F32 (split
    operands, f32-accurate like the batch-1 products).  Graphs keep the
    precision they were captured with.
    kv16: keep the KV cache in f16 (hyq_rope_qk(_seqs)_kv16 append rounds each
    key and value to binary16, hyq_attention(_seqs)_kv16 reads it), half the
    cache bytes of the reference's f32 cache; per-kernel steps only.
    fuse_norms: single-token steps of Dense layers run each RMSNorm in the
    activation prologue of the product that reads it and each residual add
    in the output step of the product that feeds it (hyq_gemv_*_norm,
    hyq_gemv_residual): two launches fewer per layer, bit-identical.  Used
    when every product weight qualifies (hyq_gemv_fusable).
    activations: "f32" (the reference's x86 branch of the single-token step)
    or "q8" (its aarch64 SDOT branch, model.rs:403-529: the products of
    STQ1_0, Q6_K and Q2_0C weights take their input quantized to Q8 --
    gemv_qkv_fast, gemv_q8_fast, matmul_gate_up_silu_fast -- under the
    reference's per-product conditions; other formats stay f32).
    Single-token steps only (the batched forward is f32 in both)."""

    def __init__(self, cfg, weights, device, prefill_chunk=PREFILL_CHUNK, fused=False, rope_in_attention=False,
                 gemm_precision=quant.GEMM_FP16, kv16=False, fuse_norms=True, activations="f32"):
        if activations not in ("f32", "q8"):
            raise ValueError(f"activations must be 'f32' or 'q8', not {activations!r}")
        if activations == "q8" and fused:
            raise ValueError("the persistent step kernel runs f32 activations")
        if kv16 and (fused or rope_in_attention):
            raise ValueError("the f16 KV cache runs with the per-kernel step (fused=False, rope_in_attention=False)")
        if cfg.arch not in ("dense", "hyv3"):
            raise ValueError(f"unknown architecture {cfg.arch}")
        if fused and cfg.arch != "dense":
            raise ValueError("the persistent step kernel runs the Dense architecture")
        self.norm_first = 1 if cfg.arch == "hyv3" else 0   # q/k norm before RoPE (model.rs:425-428)
        self.cfg = cfg
        self.rope_in_attention = rope_in_attention
        self.precision = gemm_precision
        self.kv16 = kv16
        self.kv_dtype = torch.float16 if kv16 else torch.float32
        self.device = device
        H, KV = cfg.hidden, cfg.kv_heads * cfg.head_dim
        sh = weights["shapes"]
        self.layers = []
        # packed bytes (wrapped with the configured dtypes) or ready device weights
        wrap = lambda v, t, dims, n: v if isinstance(v, quant.Weight) else quant.Weight(v, t, dims, name=n)  # noqa: E731
        for L in weights["layers"]:
            W = {n: wrap(L[n], cfg.linear_dtype, [sh[n][1], sh[n][0]], n) for n in sh if n in L}
            W.update({n: L[n] for n in ("input_norm", "ffn_norm", "q_norm", "k_norm")})
            if "moe" in L:
                from .moe import MoeLayer
                W["moe"] = L["moe"] if isinstance(L["moe"], MoeLayer) else MoeLayer(cfg.moe_config(), L["moe"])
            W["k_cache"] = torch.zeros(cfg.positions, KV, device=device, dtype=self.kv_dtype)
            W["v_cache"] = torch.zeros(cfg.positions, KV, device=device, dtype=self.kv_dtype)
            self.layers.append(W)
        self.embed = wrap(weights["embed"], cfg.embed_dtype, [H, cfg.vocab], "token_embd")
        # lm_head: the tied embedding (model.rs:194-202), or a separate output.weight
        out_w = weights.get("output")
        self.output = self.embed if out_w is None else wrap(out_w, cfg.embed_dtype, [H, cfg.vocab], "output")
        self.output_norm = weights["output_norm"]
        self.one = _Acts(cfg, 1, device)          # the graph-captured single-token step
        self.chunk = min(prefill_chunk, cfg.positions)
        self._prefill_acts = {}
        self.logits = torch.zeros(cfg.vocab, device=device)
        self.token = torch.zeros(1, dtype=torch.int32, device=device)
        self.pos = torch.zeros(1, dtype=torch.int32, device=device)
        half = cfg.head_dim // 2
        cos = np.empty(cfg.positions * half, dtype=np.float32)
        sin = np.empty_like(cos)
        check(lib.hyq_rope_table(cfg.positions, cfg.head_dim, cfg.rope_base, cos.ctypes.data_as(C.c_void_p),
                                 sin.ctypes.data_as(C.c_void_p)))
        self.cos = torch.from_numpy(cos).to(device)
        self.sin = torch.from_numpy(sin).to(device)
        ws = C.c_size_t()
        check(lib.hyq_attention_workspace_bytes(cfg.heads, cfg.head_dim, cfg.positions, self.chunk, C.byref(ws)))
        # split partials + per-(token, head) counters; zero once, every call leaves it zero
        self.attn_ws = torch.zeros(ws.value, dtype=torch.uint8, device=device)
        self.argmax_ws = torch.zeros(2, dtype=torch.int64, device=device)  # HYQ_ARGMAX_WORKSPACE_BYTES, zero
        self.graph = None
        self._step = None
        self.fuse_norms = fuse_norms and self._fusable()
        self.activations = activations
        self._acts = [self._sdot_modes(W) for W in self.layers]
        self._act_head = _Q8 if activations == "q8" and self.output.dtype in _SDOT_TYPES else _F32
        if fused:
            self._make_fused_step()

    def _sdot_modes(self, W):
        """(QKV, O, FFN) activation modes of a layer's single-token products:
        Q8 where the reference's aarch64 branch takes the SDOT kernel
        (model.rs:403-404, 462-466, 486-490), else f32."""
        if self.activations != "q8":
            return _F32, _F32, _F32
        qkv = _Q8 if W["q"].dtype in _SDOT_TYPES else _F32
        o = _Q8 if W["o"].dtype in _SDOT_TYPES else _F32
        ffn = _F32
        if "moe" not in W and W["gate"].dtype in _SDOT_TYPES and W["gate"].dtype == W["up"].dtype \
                and W["down"].dtype in _SDOT_TYPES:
            ffn = _Q8
        return qkv, o, ffn

    def _fusable(self):
        if any("moe" in W for W in self.layers):
            return False
        names = ("q", "k", "v", "o", "gate", "up", "down")
        ok = C.c_int()
        for w in [self.output] + [W[n] for W in self.layers for n in names]:
            check(lib.hyq_gemv_fusable(w.handle, C.byref(ok)))
            if not ok.value:
                return False
        return True

    def _make_fused_step(self):
        cfg, a = self.cfg, self.one
        if self.output is not self.embed:
            raise ValueError("the persistent step takes a tied lm_head only")
        arr = (_DenseLayerDesc * cfg.layers)()
        for i, W in enumerate(self.layers):
            arr[i] = _DenseLayerDesc(*(W[n].handle for n in ("q", "k", "v", "o", "gate", "up", "down")),
                                     *(W[n].data_ptr() for n in ("input_norm", "ffn_norm", "q_norm", "k_norm",
                                                                  "k_cache", "v_cache")))
        d = _DenseStepDesc(cfg.layers, cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.ffn, cfg.positions,
                           cfg.eps, C.cast(arr, C.c_void_p), self.embed.handle, self.output_norm.data_ptr(),
                           self.cos.data_ptr(), self.sin.data_ptr(), a.hidden.data_ptr(), a.q.data_ptr(),
                           a.k.data_ptr(), a.v.data_ptr(), a.attended.data_ptr(), a.gate.data_ptr(),
                           self.logits.data_ptr(), self.token.data_ptr(), self.pos.data_ptr())
        h = C.c_void_p()
        check(lib.hyq_dense_step_create(C.byref(d), C.byref(h)))
        self._step = h

    @classmethod
    def from_gguf(cls, path, device, positions=None, profile=0, fused=False):
        """Model::from_gguf (model.rs:131-284) for the Dense architecture
        (hunyuan-dense): configuration from the metadata, tensors uploaded
        unchanged from the mapped file.  positions caps the KV cache (at most
        the context length)."""
        from . import gguf

        g = gguf.Gguf(path, profile)
        md = g.metadata
        arch = md.get("general.architecture")
        if arch != "hunyuan-dense":
            raise ValueError(f"unsupported model architecture {arch} (the device runner takes hunyuan-dense)")
        key = lambda s: md[f"{arch}.{s}"]  # noqa: E731
        head_dim = int(key("attention.key_length"))
        if int(key("attention.value_length")) != head_dim:
            raise ValueError("different key/value dimensions are not supported")
        if md.get(f"{arch}.rope.scaling.type", "none") != "none":
            raise ValueError("GGUF must contain an effective RoPE base with no extra scaling")
        if f"{arch}.rope.dimension_count" in md and int(key("rope.dimension_count")) != head_dim:
            raise ValueError("partial rotary embeddings are not supported")
        heads, kv = int(key("attention.head_count")), int(key("attention.head_count_kv"))
        if heads <= 0 or kv <= 0 or heads % kv or head_dim % 2:
            raise ValueError("invalid head counts or head dimension")
        ctx = int(key("context_length"))
        t = g.tensors
        cfg = DenseConfig(layers=int(key("block_count")), hidden=int(key("embedding_length")), heads=heads,
                          kv_heads=kv, head_dim=head_dim, ffn=t["blk.0.ffn_gate.weight"].dims[1],
                          vocab=t["token_embd.weight"].dims[1], rope_base=float(key("rope.freq_base")),
                          eps=float(key("attention.layer_norm_rms_epsilon")),
                          positions=min(positions or ctx, ctx), linear_dtype=t["blk.0.attn_q.weight"].dtype,
                          embed_dtype=t["token_embd.weight"].dtype)
        names = {"q": "attn_q", "k": "attn_k", "v": "attn_v", "o": "attn_output", "gate": "ffn_gate",
                 "up": "ffn_up", "down": "ffn_down"}
        norms = {"input_norm": "attn_norm", "ffn_norm": "ffn_norm", "q_norm": "attn_q_norm",
                 "k_norm": "attn_k_norm"}
        to_dev = lambda n: torch.from_numpy(g.floats(n)).to(device)  # noqa: E731
        layers = []
        for i in range(cfg.layers):
            L = {k: g.tensor(f"blk.{i}.{n}.weight") for k, n in names.items()}
            L.update({k: to_dev(f"blk.{i}.{n}.weight") for k, n in norms.items()})
            layers.append(L)
        shapes = {k: (v.shape()[1], v.shape()[0]) for k, v in layers[0].items() if k in names}
        weights = {"layers": layers, "embed": g.tensor("token_embd.weight"),
                   "output": g.tensor("output.weight") if "output.weight" in t else None,
                   "output_norm": to_dev("output_norm.weight"), "shapes": shapes}
        model = cls(cfg, weights, device, fused=fused)
        model.gguf = g  # keeps the mapping (and its metadata) alive with the model
        return model

    def __del__(self):
        h = getattr(self, "_step", None)
        if h is not None:
            try:
                lib.hyq_dense_step_free(h)
            except Exception:
                pass
            self._step = None

    # ----------------------------------------------------------------- step
    def _stream(self):
        return C.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)

    def _enqueue(self, acts, tokens, caches=None, pos=None, token_out=None, logits=None):
        """Forward of acts.M tokens (device int32 `tokens`) at positions
        *pos ..: the layers of model.rs:374-547 (M = 1) or of the batched
        forward model.rs:549-646 (M > 1, projections on the tensor cores),
        then the lm_head of the last row and the greedy token; *pos += M.
        caches (per layer (k, v)), pos, token_out and logits default to the
        model's own (one request)."""
        with quant.gemm_precision(self.precision):
            self._enqueue_layers(acts, tokens, caches, pos, token_out, logits)

    def _enqueue_layers(self, acts, tokens, caches, pos, token_out, logits):
        cfg, st, a, M = self.cfg, self._stream(), acts, acts.M
        pos = self.pos if pos is None else pos
        token_out = self.token if token_out is None else token_out
        logits = self.logits if logits is None else logits
        check(lib.hyq_embed(self.embed.handle, _p(tokens), M, _p(a.hidden), st))
        if M > 1:
            self._enqueue_batched(a, caches, pos, token_out, logits)
        elif self.fuse_norms:
            self._enqueue_fused_norms(a, caches, pos, token_out, logits)
        else:
            self._enqueue_separate_norms(a, caches, pos, token_out, logits)

    def _enqueue_batched(self, a, caches, pos, token_out, logits):
        """The batched forward (model.rs:549-646) of a.M > 1 tokens at *pos ..:
        every residual add and RMSNorm runs in the activation conversion of
        the batched product that follows it (hyq_matmul_qkv_norm,
        hyq_matmul_gate_up_silu_norm, hyq_matmul_norm; bit-identical to the
        separate add + norm kernel), the MoE FFN takes the separate one."""
        cfg, st, M, H = self.cfg, self._stream(), a.M, self.cfg.hidden
        fused = self.precision == quant.GEMM_F32
        delta = None   # the residual add the next norm applies
        for i, W in enumerate(self.layers):
            kc, vc = (W["k_cache"], W["v_cache"]) if caches is None else caches[i]
            _qkv_normed(fused, W, _p(a.hidden), delta, _p(W["input_norm"]), cfg.eps, M, _p(a.normalized),
                        (_p(a.q), _p(a.k), _p(a.v)), st)
            rope = lib.hyq_rope_qk_kv16 if self.kv16 else lib.hyq_rope_qk
            attention = lib.hyq_attention_kv16 if self.kv16 else lib.hyq_attention
            check(rope(_p(a.q), _p(a.k), _p(a.v), cfg.heads, cfg.kv_heads, cfg.head_dim, _p(self.cos), _p(self.sin),
                       cfg.positions, _p(pos), M, _p(W["q_norm"]), _p(W["k_norm"]), cfg.eps, self.norm_first, _p(kc),
                       _p(vc), st))
            check(attention(_p(a.q), _p(kc), _p(vc), cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.positions, _p(pos),
                            M, _p(a.attended), _p(self.attn_ws), st))
            check(lib.hyq_matmul(W["o"].handle, _p(a.attended), M, _p(a.projected), st))
            if "moe" in W:      # Moe::forward (model.rs:688-726)
                check(lib.hyq_add_rms_norm(_p(a.hidden), _p(a.projected), _p(W["ffn_norm"]), H, M, cfg.eps,
                                           _p(a.normalized), st))
                W["moe"].forward(a.normalized, M, out=a.ff)
            else:
                _gate_up_normed(fused, W, _p(a.hidden), _p(a.projected), _p(W["ffn_norm"]), cfg.eps, M,
                                _p(a.normalized), _p(a.gate), st)
                check(lib.hyq_matmul(W["down"].handle, _p(a.gate), M, _p(a.ff), st))
            delta = _p(a.ff)
        # logits of the last token only (model.rs:619-622): its residual add
        # and norm, then the lm_head
        last = lambda t: C.c_void_p(t.data_ptr() + (M - 1) * t.stride(0) * t.element_size())  # noqa: E731
        _matmul_normed(fused, self.output, last(a.hidden), last(a.ff), _p(self.output_norm), cfg.eps, 1,
                       last(a.normalized), _p(logits), st)
        check(lib.hyq_argmax(_p(logits), cfg.vocab, _p(token_out), _p(pos), M, _p(self.argmax_ws), st))

    def _enqueue_separate_norms(self, a, caches, pos, token_out, logits):
        """The single-token step with each RMSNorm and residual add as its own
        launch (fuse_norms=False)."""
        cfg, st, H = self.cfg, self._stream(), self.cfg.hidden
        check(lib.hyq_rms_norm(_p(a.hidden), _p(self.layers[0]["input_norm"]), H, 1, cfg.eps, _p(a.normalized), st))
        for i, W in enumerate(self.layers):
            kc, vc = (W["k_cache"], W["v_cache"]) if caches is None else caches[i]
            act_qkv, act_o, act_ffn = self._acts[i]
            qkv = lib.hyq_gemv_qkv_int8 if act_qkv == _Q8 else lib.hyq_gemv_qkv
            check(qkv(W["q"].handle, W["k"].handle, W["v"].handle, _p(a.normalized), _p(a.q), _p(a.k), _p(a.v), st))
            self._attention_one(W, a, kc, vc, pos)
            if act_o == _Q8:
                check(lib.hyq_gemv_int8(W["o"].handle, _p(a.attended), _p(a.projected), st))
            else:
                check(lib.hyq_matmul(W["o"].handle, _p(a.attended), 1, _p(a.projected), st))
            # residual add fused with the norm that follows it
            check(lib.hyq_add_rms_norm(_p(a.hidden), _p(a.projected), _p(W["ffn_norm"]), H, 1, cfg.eps,
                                       _p(a.normalized), st))
            if "moe" in W:      # Moe::forward (model.rs:688-726)
                W["moe"].forward(a.normalized, 1, out=a.ff)
            else:
                gate_up = lib.hyq_matmul_gate_up_silu_int8 if act_ffn == _Q8 else lib.hyq_matmul_gate_up_silu
                check(gate_up(W["gate"].handle, W["up"].handle, _p(a.normalized), _p(a.gate), st))
                if act_ffn == _Q8:
                    check(lib.hyq_gemv_int8(W["down"].handle, _p(a.gate), _p(a.ff), st))
                else:
                    check(lib.hyq_matmul(W["down"].handle, _p(a.gate), 1, _p(a.ff), st))
            nxt = self.layers[i + 1]["input_norm"] if i + 1 < len(self.layers) else self.output_norm
            check(lib.hyq_add_rms_norm(_p(a.hidden), _p(a.ff), _p(nxt), H, 1, cfg.eps, _p(a.normalized), st))
        if self._act_head == _Q8:
            check(lib.hyq_gemv_int8(self.output.handle, _p(a.normalized), _p(logits), st))
        else:
            check(lib.hyq_matmul(self.output.handle, _p(a.normalized), 1, _p(logits), st))
        check(lib.hyq_argmax(_p(logits), cfg.vocab, _p(token_out), _p(pos), 1, _p(self.argmax_ws), st))

    def _attention_one(self, W, a, kc, vc, pos):
        cfg, st = self.cfg, self._stream()
        if self.rope_in_attention:
            check(lib.hyq_rope_attention(_p(a.q), _p(a.k), _p(a.v), cfg.heads, cfg.kv_heads, cfg.head_dim,
                                         _p(self.cos), _p(self.sin), cfg.positions, _p(pos), _p(W["q_norm"]),
                                         _p(W["k_norm"]), cfg.eps, self.norm_first, _p(kc), _p(vc), _p(a.attended),
                                         _p(self.attn_ws), st))
            return
        rope = lib.hyq_rope_qk_kv16 if self.kv16 else lib.hyq_rope_qk
        attention = lib.hyq_attention_kv16 if self.kv16 else lib.hyq_attention
        check(rope(_p(a.q), _p(a.k), _p(a.v), cfg.heads, cfg.kv_heads, cfg.head_dim, _p(self.cos), _p(self.sin),
                   cfg.positions, _p(pos), 1, _p(W["q_norm"]), _p(W["k_norm"]), cfg.eps, self.norm_first, _p(kc),
                   _p(vc), st))
        check(attention(_p(a.q), _p(kc), _p(vc), cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.positions, _p(pos), 1,
                        _p(a.attended), _p(self.attn_ws), st))

    def _enqueue_fused_norms(self, a, caches, pos, token_out, logits):
        """The single-token chain of Model::forward (model.rs:1007-1041) with
        every RMSNorm in the prologue of the product that reads it and every
        residual add in the output step of the product that feeds it; the
        hidden row is the only residual-stream buffer."""
        cfg, st = self.cfg, self._stream()
        for i, W in enumerate(self.layers):
            kc, vc = (W["k_cache"], W["v_cache"]) if caches is None else caches[i]
            act_qkv, act_o, act_ffn = self._acts[i]
            check(lib.hyq_gemv_qkv_norm(W["q"].handle, W["k"].handle, W["v"].handle, _p(a.hidden),
                                        _p(W["input_norm"]), cfg.eps, act_qkv, _p(a.q), _p(a.k), _p(a.v), st))
            self._attention_one(W, a, kc, vc, pos)
            check(lib.hyq_gemv_residual(W["o"].handle, _p(a.attended), act_o, _p(a.hidden), st))
            check(lib.hyq_gemv_gate_up_silu_norm(W["gate"].handle, W["up"].handle, _p(a.hidden),
                                                 _p(W["ffn_norm"]), cfg.eps, act_ffn, _p(a.gate), st))
            check(lib.hyq_gemv_residual(W["down"].handle, _p(a.gate), act_ffn, _p(a.hidden), st))
        check(lib.hyq_gemv_norm(self.output.handle, _p(a.hidden), _p(self.output_norm), cfg.eps, self._act_head,
                                _p(logits), st))
        check(lib.hyq_argmax(_p(logits), cfg.vocab, _p(token_out), _p(pos), 1, _p(self.argmax_ws), st))

    def enqueue_step(self):
        """One token: reads self.token / self.pos, leaves the logits, the next
        greedy token in self.token, and pos + 1."""
        if self._step is not None:
            check(lib.hyq_dense_step_enqueue(self._step, self._stream()))
        else:
            self._enqueue(self.one, self.token)

    def prefill(self, ids, **targets):
        """Feed a prompt chunk of at most self.chunk tokens (a device int32
        tensor) in one batched forward; leaves the logits of its last token,
        the next greedy token in self.token and pos += len(ids) (or in the
        caches / pos / token_out / logits given)."""
        M = int(ids.numel())
        if not 0 < M <= self.chunk:
            raise ValueError(f"prefill takes 1..{self.chunk} tokens")
        acts = self._prefill_acts.get(M)
        if acts is None:
            acts = self._prefill_acts[M] = _Acts(self.cfg, M, self.device)
        self._enqueue(acts, ids, **targets)

    # kernel launches of one enqueue_step
    def launches(self):
        if self._step is not None:
            return 1
        if self.fuse_norms:   # embed; QKV, (RoPE,) attention, O, gate/up, down per layer; lm_head, argmax
            return 3 + (5 if self.rope_in_attention else 6) * len(self.layers)
        per_layer = 7 if self.rope_in_attention else 8
        # a MoE layer runs MoeLayer's launches in place of gate/up and down
        return 4 + sum(per_layer + (W["moe"].launches(1) - 2 if "moe" in W else 0) for W in self.layers)

    def capture(self, stream):
        """Capture enqueue_step as one CUDA graph on `stream`."""
        quant.set_launch_overlap(True)  # the weights are final; see hyq_set_launch_overlap
        with torch.cuda.stream(stream):
            self.pos.zero_()
            self.enqueue_step()  # warm every path outside the capture
            stream.synchronize()
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=stream):
                self.enqueue_step()
            self.reset()
        return self.graph

    def reset(self):
        self.pos.zero_()
        for W in self.layers:
            W["k_cache"].zero_()
            W["v_cache"].zero_()

    def generate(self, prompt, n_new, stream, logits_out=None, batched_prefill=False):
        """Greedy decode: feed `prompt` (one graph step per token, or in
        batched chunks with batched_prefill), then `n_new` tokens.  Returns the
        generated ids (and fills logits_out[i] with the logits that chose
        token i when given)."""
        if self.graph is None:
            self.capture(stream)
        if len(prompt) + n_new > self.cfg.positions:
            raise ValueError("prompt + generated tokens exceed the KV-cache capacity")
        out = torch.empty(n_new, dtype=torch.int32, device=self.device)
        ids = torch.tensor(prompt, dtype=torch.int32).to(self.device)
        with torch.cuda.stream(stream):
            self.reset()
            # after the prompt, self.token holds generated token 0 and
            # self.logits the logits that chose it
            if batched_prefill:
                for c0 in range(0, len(prompt), self.chunk):
                    self.prefill(ids[c0:c0 + self.chunk])
            else:
                for i in range(len(prompt)):
                    self.token.copy_(ids[i:i + 1])
                    self.graph.replay()
            for i in range(n_new):
                out[i:i + 1].copy_(self.token)
                if logits_out is not None:
                    logits_out[i].copy_(self.logits)
                if i < n_new - 1:
                    self.graph.replay()
        stream.synchronize()
        return out.cpu().tolist()


class DenseBatch:
    """Concurrent greedy decoding of `batch` independent requests with one
    model: each step runs model.rs:374-547 for one token of every request,
    the projections as [batch, K] products (on the tensor cores from 16
    requests), RoPE, KV append and attention per request over its own cache
    (hyq_rope_qk_seqs, hyq_attention_seqs), and a greedy token per request
    (hyq_argmax_rows).  Prompts are fed per request with the batched
    forward, into that request's cache slice."""

    def __init__(self, model, batch):
        cfg, dev = model.cfg, model.device
        if batch > cfg.positions:
            raise ValueError("at most `positions` concurrent requests")
        self.m, self.B = model, batch
        KV = cfg.kv_heads * cfg.head_dim
        self.caches = [(torch.zeros(batch, cfg.positions, KV, device=dev, dtype=model.kv_dtype),
                        torch.zeros(batch, cfg.positions, KV, device=dev, dtype=model.kv_dtype)) for _ in model.layers]
        self.stride = cfg.positions * KV
        self.acts = _Acts(cfg, batch, dev)
        self.logits = torch.zeros(batch, cfg.vocab, device=dev)
        self.tokens = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(batch, dtype=torch.int32, device=dev)
        ws = C.c_size_t()
        check(lib.hyq_attention_workspace_bytes(cfg.heads, cfg.head_dim, cfg.positions, batch, C.byref(ws)))
        self.attn_ws = torch.zeros(ws.value, dtype=torch.uint8, device=dev)
        self.graph = None

    def enqueue_step(self):
        with quant.gemm_precision(self.m.precision):
            self._enqueue_step()

    def _enqueue_step(self):
        m, cfg, a, B = self.m, self.m.cfg, self.acts, self.B
        st, H = m._stream(), cfg.hidden
        check(lib.hyq_embed(m.embed.handle, _p(self.tokens), B, _p(a.hidden), st))
        # the residual adds and RMSNorms with the products (_qkv_normed and
        # friends; the MoE FFN takes the separate kernel)
        fused = m.precision == quant.GEMM_F32
        delta = None
        for i, W in enumerate(m.layers):
            kc, vc = self.caches[i]
            _qkv_normed(fused, W, _p(a.hidden), delta, _p(W["input_norm"]), cfg.eps, B, _p(a.normalized),
                        (_p(a.q), _p(a.k), _p(a.v)), st)
            if m.rope_in_attention:
                check(lib.hyq_rope_attention_seqs(_p(a.q), _p(a.k), _p(a.v), cfg.heads, cfg.kv_heads, cfg.head_dim,
                                                  _p(m.cos), _p(m.sin), cfg.positions, _p(self.pos), B,
                                                  _p(W["q_norm"]), _p(W["k_norm"]), cfg.eps, m.norm_first, _p(kc), _p(vc),
                                                  self.stride, _p(a.attended), _p(self.attn_ws), st))
            else:
                rope = lib.hyq_rope_qk_seqs_kv16 if m.kv16 else lib.hyq_rope_qk_seqs
                attention = lib.hyq_attention_seqs_kv16 if m.kv16 else lib.hyq_attention_seqs
                check(rope(_p(a.q), _p(a.k), _p(a.v), cfg.heads, cfg.kv_heads, cfg.head_dim, _p(m.cos), _p(m.sin),
                           cfg.positions, _p(self.pos), B, _p(W["q_norm"]), _p(W["k_norm"]), cfg.eps, m.norm_first,
                           _p(kc),
                           _p(vc), self.stride, st))
                check(attention(_p(a.q), _p(kc), _p(vc), cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.positions,
                                _p(self.pos), B, self.stride, _p(a.attended), _p(self.attn_ws), st))
            check(lib.hyq_matmul(W["o"].handle, _p(a.attended), B, _p(a.projected), st))
            if "moe" in W:      # Moe::forward over the requests' rows
                check(lib.hyq_add_rms_norm(_p(a.hidden), _p(a.projected), _p(W["ffn_norm"]), H, B, cfg.eps,
                                           _p(a.normalized), st))
                W["moe"].forward(a.normalized, B, out=a.ff)
            else:
                _gate_up_normed(fused, W, _p(a.hidden), _p(a.projected), _p(W["ffn_norm"]), cfg.eps, B,
                                _p(a.normalized), _p(a.gate), st)
                check(lib.hyq_matmul(W["down"].handle, _p(a.gate), B, _p(a.ff), st))
            delta = _p(a.ff)
        _matmul_normed(fused, m.output, _p(a.hidden), delta, _p(m.output_norm), cfg.eps, B, _p(a.normalized),
                       _p(self.logits), st)
        check(lib.hyq_argmax_rows(_p(self.logits), cfg.vocab, B, _p(self.tokens), _p(self.pos), st))

    def launches(self, sms=148):
        """Kernel launches of one step: QKV / O / gate-up / down / lm_head as
        batched products (on the tensor cores from 16 requests: activation
        conversion + GEMM + split-K reduction when the product splits;
        below 16, one batch-1 product per request)."""
        cfg, B = self.m.cfg, self.B
        t = cfg.linear_dtype
        KV = cfg.kv_heads * cfg.head_dim
        if B >= 16:
            # split operands: the norms run in the conversions of QKV,
            # gate/up and lm_head; fp16 operands: a separate norm kernel each
            split = self.m.precision == quant.GEMM_F32
            g = lambda tiles, K, dt=t: quant.gemm_launches(tiles, K, B, dt, sms, split=split)  # noqa: E731
            attn = g((cfg.heads * cfg.head_dim + 2 * KV) // 128, cfg.hidden) + g(cfg.hidden // 128, cfg.hidden)
            ffn = g(2 * cfg.ffn // 128, cfg.hidden) + g(cfg.hidden // 128, cfg.ffn)
            lm_head = g(-(-cfg.vocab // 128), cfg.hidden, cfg.embed_dtype)
            norm = 0 if self.m.precision == quant.GEMM_F32 else 1
        else:
            # batch-1 products; each fused form runs its add + norm kernel first
            attn, ffn, lm_head = 2 * B, 2 * B, B
            norm = 1
        ra = 1 if self.m.rope_in_attention else 2   # (RoPE +) attention
        # embedding; per layer QKV (+ norm), (RoPE,) attention, O, then gate/up
        # (+ norm) and down, or the MoE layer after its add + norm kernel;
        # lm_head (+ norm); argmax
        layers = sum(norm + ra + attn + (1 + W["moe"].launches(B) if "moe" in W else norm + ffn)
                     for W in self.m.layers)
        return 1 + layers + norm + lm_head + 1

    def capture(self, stream):
        quant.set_launch_overlap(True)
        with torch.cuda.stream(stream):
            saved = (self.tokens.clone(), self.pos.clone())
            self.enqueue_step()  # warm every path outside the capture
            stream.synchronize()
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=stream):
                self.enqueue_step()
            self.tokens.copy_(saved[0])
            self.pos.copy_(saved[1])
        return self.graph

    def reset(self):
        self.pos.zero_()
        for k, v in self.caches:
            k.zero_()
            v.zero_()

    def prefill_all(self, prompts):
        """Feed each request's prompt (batched forwards into its cache
        slice); leaves each request's first generated token in self.tokens."""
        m = self.m
        ids = [torch.tensor(p, dtype=torch.int32).to(m.device) for p in prompts]
        for b, t in enumerate(ids):
            caches = [(k[b], v[b]) for k, v in self.caches]
            for c0 in range(0, t.numel(), m.chunk):
                m.prefill(t[c0:c0 + m.chunk], caches=caches, pos=self.pos[b:b + 1],
                          token_out=self.tokens[b:b + 1], logits=self.logits[b])

    def generate(self, prompts, n_new, stream, logits_out=None):
        """Greedy decode of len(prompts) == batch requests: per request the
        n_new generated ids (and logits_out[i, b] the logits that chose
        request b's token i)."""
        if len(prompts) != self.B:
            raise ValueError("one prompt per request")
        if max(len(p) for p in prompts) + n_new > self.m.cfg.positions:
            raise ValueError("prompt + generated tokens exceed the KV-cache capacity")
        out = torch.empty(n_new, self.B, dtype=torch.int32, device=self.m.device)
        with torch.cuda.stream(stream):
            if self.graph is None:
                self.capture(stream)   # its warm-up step writes logits and caches: before the prompts
            self.reset()
            self.prefill_all(prompts)
            for i in range(n_new):
                out[i].copy_(self.tokens)
                if logits_out is not None:
                    logits_out[i].copy_(self.logits)
                if i < n_new - 1:
                    self.graph.replay()
        stream.synchronize()
        return out.t().cpu().tolist()
