"""A random-init Dense model written as a Tencent Q2_0C legacy GGUF file
(type ids 0, 14, 40; hunyuan-dense metadata) and loaded back through
hyq_gguf_* / DenseModel.from_gguf (model.rs:131-284): the same greedy tokens
and the same logits, bit for bit, as the model built from the weights in
memory (the packed bytes travel unchanged)."""
import numpy as np
import pytest

from gguf_writer import gguf_bytes

pytestmark = pytest.mark.gpu


def _write_model(path, cfg, w):
    import torch

    arch = "hunyuan-dense"
    md = [("general.architecture", 8, arch), ("general.file_type", 4, 39),
          (f"{arch}.block_count", 4, cfg.layers), (f"{arch}.embedding_length", 4, cfg.hidden),
          (f"{arch}.attention.head_count", 4, cfg.heads), (f"{arch}.attention.head_count_kv", 4, cfg.kv_heads),
          (f"{arch}.attention.key_length", 4, cfg.head_dim), (f"{arch}.attention.value_length", 4, cfg.head_dim),
          (f"{arch}.context_length", 4, cfg.positions), (f"{arch}.rope.freq_base", 6, cfg.rope_base),
          (f"{arch}.attention.layer_norm_rms_epsilon", 6, cfg.eps)]
    raw = lambda t: t.cpu().numpy().tobytes()  # noqa: E731
    tensors = [("token_embd.weight", [cfg.hidden, cfg.vocab], 14, raw(w["embed"])),
               ("output_norm.weight", [cfg.hidden], 0, raw(w["output_norm"]))]
    names = {"q": "attn_q", "k": "attn_k", "v": "attn_v", "o": "attn_output", "gate": "ffn_gate", "up": "ffn_up",
             "down": "ffn_down"}
    norms = {"input_norm": "attn_norm", "ffn_norm": "ffn_norm", "q_norm": "attn_q_norm", "k_norm": "attn_k_norm"}
    for i, L in enumerate(w["layers"]):
        for k, n in names.items():
            N, K = w["shapes"][k]
            tensors.append((f"blk.{i}.{n}.weight", [K, N], 40, raw(L[k])))
        for k, n in norms.items():
            tensors.append((f"blk.{i}.{n}.weight", [L[k].numel()], 0, raw(L[k])))
    path.write_bytes(gguf_bytes(metadata=md, tensors=tensors))
    del torch


def test_dense_model_from_gguf(cuda, tmp_path):
    import torch
    from hy_mt_rs_b200 import quant
    from hy_mt_rs_b200.gguf import TENCENT_Q2_0C
    from hy_mt_rs_b200.model import DenseConfig, DenseModel, random_weights

    cfg = DenseConfig(layers=3, vocab=8192, positions=64)
    w = random_weights(cfg, cuda, seed=5)
    p = tmp_path / "dense.gguf"
    _write_model(p, cfg, w)
    loaded = DenseModel.from_gguf(p, cuda, profile=TENCENT_Q2_0C)
    assert loaded.gguf.profile == TENCENT_Q2_0C
    assert (loaded.cfg.layers, loaded.cfg.vocab, loaded.cfg.ffn, loaded.cfg.positions) == (3, 8192, 6144, 64)
    ref = DenseModel(cfg, w, cuda)
    prompt, n_new = [3, 1000, 77, 8000, 5], 6
    stream = torch.cuda.Stream(cuda)
    la = torch.zeros(n_new, cfg.vocab, device=cuda)
    lb = torch.zeros(n_new, cfg.vocab, device=cuda)
    try:
        ids_a = loaded.generate(prompt, n_new, stream, logits_out=la)
        ids_b = ref.generate(prompt, n_new, stream, logits_out=lb)
    finally:
        quant.set_launch_overlap(False)
    assert ids_a == ids_b
    np.testing.assert_array_equal(la.cpu().numpy(), lb.cpu().numpy())
    assert quant.device_status() == 0
