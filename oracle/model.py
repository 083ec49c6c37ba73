"""CPU restatement of one single-token decoder step of the Dense
architecture (model.rs:374-547, x86 branches), composed from the C oracle's
primitives.  Test infrastructure only: the parity tests and nothing else use
it.  Parity of these model-level steps is unpinned (the reference's logits
fixtures need its real GGUF files); the quantized products inside are pinned
through the oracle's decoders and dot orders.
"""
import numpy as np

from . import oracle as O


class DenseOracle:
    """Weights as numpy arrays (packed uint8 linears, f32 norms), from the same
    bytes the device model uploads."""

    def __init__(self, cfg, weights, threads=0, kv16=False):
        """cfg.arch "hyv3": the q/k norm before RoPE (model.rs:425-428), the
        MoE FFN of layers with a "moe" entry (Moe::forward at batch 1 with
        the x86-order batch-1 products, oracle/moe.py moe_forward_port), and
        the separate output matrix."""
        """kv16: store every cached key and value rounded to the nearest
        binary16 (the device's f16 KV cache), everything else as the
        reference."""
        self.cfg = cfg
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

    def _mm(self, w, K, N, x):
        return O.matmul(self.cfg.linear_dtype, w, K, N, x, 1, self.threads)[0]

    def step(self, token, pos):
        """Logits after feeding `token` at position `pos`."""
        c = self.cfg
        H, A, KV, F = c.hidden, c.heads * c.head_dim, c.kv_heads * c.head_dim, c.ffn
        rb = H // 256 * 210 if c.embed_dtype == 3 else None
        hidden = O.decode(c.embed_dtype, self.embed[token * rb:(token + 1) * rb], H)  # row_into
        cos, sin = O.rope_table(pos, c.head_dim, c.rope_base)
        for i, L in enumerate(self.layers):
            normalized = O.rms_norm(hidden, L["input_norm"], c.eps)
            q = self._mm(L["q"], H, A, normalized)
            k = self._mm(L["k"], H, KV, normalized)
            v = self._mm(L["v"], H, KV, normalized)
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
            hidden = (hidden + self._mm(L["o"], A, H, attended)).astype(np.float32)
            normalized = O.rms_norm(hidden, L["ffn_norm"], c.eps)
            if "moe" in L:
                from .moe import moe_forward_port
                ff = moe_forward_port(self.moe_cfg, L["moe"], normalized[None], self.threads)[0]
            else:
                gate = O.gate_up_silu(c.linear_dtype, L["gate"], L["up"], H, F, normalized, self.threads)
                ff = self._mm(L["down"], F, H, gate)
            hidden = (hidden + ff).astype(np.float32)
        hidden = O.rms_norm(hidden, self.output_norm, c.eps)
        return O.matmul(c.embed_dtype, self.output, H, c.vocab, hidden, 1, self.threads)[0]

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
