"""CPU restatement of one single-token decoder step of the Dense
architecture (model.rs:374-547: the x86 branch, or with activations="q8"
the aarch64 SDOT branch), composed from the C oracle's
primitives.  Test infrastructure only: the parity tests and nothing else use
it.  Parity of these model-level steps is unpinned (the reference's logits
fixtures need its real GGUF files); the quantized products inside are pinned
through the oracle's decoders and dot orders.
"""
import numpy as np

from . import oracle as O

# STQ1_0, Q6_K, Q2_0C: the types the aarch64 branch sends to the SDOT kernels
# (model.rs:403-404)
_SDOT_TYPES = (6, 3, 5)


class DenseOracle:
    """Weights as numpy arrays (packed uint8 linears, f32 norms), from the same
    bytes the device model uploads."""

    def __init__(self, cfg, weights, threads=0, kv16=False, activations="f32"):
        """cfg.arch "hyv3": the q/k norm before RoPE (model.rs:425-428), the
        MoE FFN of layers with a "moe" entry (Moe::forward at batch 1 with
        the x86-order batch-1 products, oracle/moe.py moe_forward_port), and
        the separate output matrix."""
        """kv16: store every cached key and value rounded to the nearest
        binary16 (the device's f16 KV cache), everything else as the
        reference."""
        """activations "q8": the aarch64 SDOT branch of the single-token step
        (model.rs:403-529): products of STQ1_0 / Q6_K / Q2_0C weights take
        their input through Q8::quantize_into and the SDOT-order dot
        (gemv_qkv_fast, gemv_q8_fast, matmul_gate_up_silu_fast), under the
        branch's per-product conditions."""
        self.cfg = cfg
        self.q8 = activations == "q8"
        self.threads = threads
        self.kv16 = kv16
        self.layers = [{k: (v.cpu().numpy() if hasattr(v, "cpu") else v) for k, v in L.items()}
                       for L in weights["layers"]]
        self.embed = weights["embed"].cpu().numpy()
        self.output = weights["output"].cpu().numpy() if weights.get("output") is not None else self.embed
        self.moe_cfg = cfg.moe_config() if getattr(cfg, "arch", "dense") == "hyv3" else None
        for L in self.layers:
            if "moe" in L:
                L["moe"] = {k: v.cpu().numpy() for k, v in L["moe"].items()}
        self.output_norm = weights["output_norm"].cpu().numpy()
        kv = cfg.kv_heads * cfg.head_dim
        self.k_cache = [np.zeros((cfg.positions, kv), np.float32) for _ in range(cfg.layers)]
        self.v_cache = [np.zeros((cfg.positions, kv), np.float32) for _ in range(cfg.layers)]

    def _mm(self, w, K, N, x, t=None, q8=False):
        t = self.cfg.linear_dtype if t is None else t
        if q8:
            values, scales, q2c = O.q8_quantize(x)
            return O.gemv_q8(t, w, K, N, values, scales, q2c, self.threads)
        return O.matmul(t, w, K, N, x, 1, self.threads)[0]

    def _sdot(self, t):
        return self.q8 and t in _SDOT_TYPES

    def step(self, token, pos):
        """Logits after feeding `token` at position `pos`."""
        c = self.cfg
        H, A, KV, F = c.hidden, c.heads * c.head_dim, c.kv_heads * c.head_dim, c.ffn
        rb = H // 256 * 210 if c.embed_dtype == 3 else None
        hidden = O.decode(c.embed_dtype, self.embed[token * rb:(token + 1) * rb], H)  # row_into
        cos, sin = O.rope_table(pos, c.head_dim, c.rope_base)
        for i, L in enumerate(self.layers):
            normalized = O.rms_norm(hidden, L["input_norm"], c.eps)
            lin = self._sdot(c.linear_dtype)   # every linear has the configured type
            q = self._mm(L["q"], H, A, normalized, q8=lin)
            k = self._mm(L["k"], H, KV, normalized, q8=lin)
            v = self._mm(L["v"], H, KV, normalized, q8=lin)
            if self.moe_cfg is not None:   # HyV3: before RoPE (model.rs:425-428)
                q = O.rms_norm_rows(q, L["q_norm"], c.eps)
                k = O.rms_norm_rows(k, L["k_norm"], c.eps)
            q = O.rope(q, c.heads, c.head_dim, cos, sin)
            k = O.rope(k, c.kv_heads, c.head_dim, cos, sin)
            if self.moe_cfg is None:       # Dense: after RoPE (model.rs:443-446)
                q = O.rms_norm_rows(q, L["q_norm"], c.eps)
                k = O.rms_norm_rows(k, L["k_norm"], c.eps)
            if self.kv16:
                k = k.astype(np.float16).astype(np.float32)
                v = v.astype(np.float16).astype(np.float32)
            self.k_cache[i][pos] = k
            self.v_cache[i][pos] = v
            attended = O.attention(q, self.k_cache[i][:pos + 1], self.v_cache[i][:pos + 1], c.heads, c.kv_heads,
                                   c.head_dim, pos)
            hidden = (hidden + self._mm(L["o"], A, H, attended, q8=lin)).astype(np.float32)
            normalized = O.rms_norm(hidden, L["ffn_norm"], c.eps)
            if "moe" in L:
                from .moe import moe_forward_port
                ff = moe_forward_port(self.moe_cfg, L["moe"], normalized[None], self.threads)[0]
            elif lin:
                values, scales, q2c = O.q8_quantize(normalized)
                gate = O.gate_up_silu_q8(c.linear_dtype, L["gate"], L["up"], H, F, values, scales, q2c,
                                         self.threads)
                ff = self._mm(L["down"], F, H, gate, q8=True)
            else:
                gate = O.gate_up_silu(c.linear_dtype, L["gate"], L["up"], H, F, normalized, self.threads)
                ff = self._mm(L["down"], F, H, gate)
            hidden = (hidden + ff).astype(np.float32)
        hidden = O.rms_norm(hidden, self.output_norm, c.eps)
        return self._mm(self.output, H, c.vocab, hidden, t=c.embed_dtype, q8=self._sdot(c.embed_dtype))

    def generate(self, prompt, n_new):
        """Greedy ids and the logits that chose each (generation.rs:281-290)."""
        pos = 0
        logits = None
        for t in prompt:
            logits = self.step(int(t), pos)
            pos += 1
        ids, all_logits = [], []
        for i in range(n_new):
            tok = int(np.argmax(logits))  # first index of the maximum
            ids.append(tok)
            all_logits.append(logits)
            if i < n_new - 1:
                logits = self.step(tok, pos)
                pos += 1
        return ids, all_logits
