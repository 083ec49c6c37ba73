"""Concurrent decoding of independent requests (DenseBatch): every step
decodes one token of each request, the projections as [requests, K]
products, RoPE / KV append / attention per request over its own cache
(hyq_rope_qk_seqs, hyq_attention_seqs) and one greedy token per request
(hyq_argmax_rows).  Each request must decode exactly as it would alone
(DenseModel.generate with the batched prompt forward): bit-identical below
16 requests, where the products are the same f32 batch-1 products, and
within the fp16 tensor-core tolerance from 16 requests."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _alone(model, prompts, n_new, stream):
    import torch

    ids, logits = [], []
    for p in prompts:
        lg = torch.zeros(n_new, model.cfg.vocab, device=model.device)
        ids.append(model.generate(p, n_new, stream, logits_out=lg, batched_prefill=True))
        logits.append(lg.cpu().numpy())
    return ids, np.stack(logits, axis=1)   # [n_new, requests, vocab]


def test_batch_below_16_bit_exact(cuda):
    import torch
    from hy_mt_rs_b200 import quant
    from hy_mt_rs_b200.model import DenseBatch, DenseConfig, DenseModel, random_weights

    cfg = DenseConfig(layers=3, positions=48)
    weights = random_weights(cfg, cuda, seed=5)
    torch.cuda.synchronize()
    model = DenseModel(cfg, weights, cuda)
    rng = np.random.default_rng(5)
    prompts = [rng.integers(0, cfg.vocab, n).tolist() for n in (3, 9, 1, 6)]   # ragged prompts
    n_new = 7
    stream = torch.cuda.Stream(cuda)
    try:
        ref_ids, ref_logits = _alone(model, prompts, n_new, stream)
        batch = DenseBatch(model, len(prompts))
        logits = torch.zeros(n_new, len(prompts), cfg.vocab, device=cuda)
        ids = batch.generate(prompts, n_new, stream, logits_out=logits)
        again = batch.generate(prompts, n_new, stream)      # same graph, caches reset
    finally:
        quant.set_launch_overlap(False)
    assert ids == ref_ids
    assert np.array_equal(logits.cpu().numpy(), ref_logits)
    assert again == ids
    assert quant.device_status() == 0


def test_batch_64_tensor_cores(cuda):
    import torch
    from hy_mt_rs_b200 import quant
    from hy_mt_rs_b200.model import DenseBatch, DenseConfig, DenseModel, random_weights

    cfg = DenseConfig(layers=2, positions=96)
    weights = random_weights(cfg, cuda, seed=64)
    torch.cuda.synchronize()
    model = DenseModel(cfg, weights, cuda)
    rng = np.random.default_rng(64)
    B, n_new = 64, 4
    prompts = [rng.integers(0, cfg.vocab, int(n)).tolist() for n in rng.integers(1, 40, B)]
    stream = torch.cuda.Stream(cuda)
    try:
        ref_ids, ref_logits = _alone(model, prompts, n_new, stream)
        batch = DenseBatch(model, B)
        logits = torch.zeros(n_new, B, cfg.vocab, device=cuda)
        ids = batch.generate(prompts, n_new, stream, logits_out=logits)
    finally:
        quant.set_launch_overlap(False)
    got = logits.cpu().numpy()
    for b in range(B):
        for i in range(n_new):
            rel = np.linalg.norm(got[i, b] - ref_logits[i, b]) / np.linalg.norm(ref_logits[i, b])
            assert rel < 2e-2, (b, i, rel)
            if ids[b][i] != ref_ids[b][i]:
                top = np.sort(ref_logits[i, b])[-2:]
                err = float(np.abs(got[i, b] - ref_logits[i, b]).max())
                assert float(top[1] - top[0]) <= 2 * err, (b, i)
                break
    # token 0 comes from the prompt forward, the same call on both sides
    assert [r[0] for r in ids] == [r[0] for r in ref_ids]
    assert quant.device_status() == 0


def test_batch_64_split_operands_match_oracle(cuda):
    """64 concurrent requests with f32-accurate batched products
    (GEMM_F32: split fp16 operands on the tensor cores): requests 0, 21, 42
    and 63 against the CPU oracle model decoding each request on its own
    (oracle/model.py), not against the GPU: logits of every step within the
    1e-4 bound of the f32 single-request path, identical greedy tokens (a
    divergence only at a near-tie the numerics cannot order)."""
    import torch
    from hy_mt_rs_b200 import quant
    from hy_mt_rs_b200.model import DenseBatch, DenseConfig, DenseModel, random_weights
    from oracle.model import DenseOracle

    cfg = DenseConfig(layers=2, positions=96)
    weights = random_weights(cfg, cuda, seed=65)
    torch.cuda.synchronize()
    model = DenseModel(cfg, weights, cuda, gemm_precision=quant.GEMM_F32)
    rng = np.random.default_rng(65)
    B, n_new = 64, 5
    prompts = [rng.integers(0, cfg.vocab, int(n)).tolist() for n in rng.integers(1, 40, B)]
    stream = torch.cuda.Stream(cuda)
    try:
        batch = DenseBatch(model, B)
        logits = torch.zeros(n_new, B, cfg.vocab, device=cuda)
        ids = batch.generate(prompts, n_new, stream, logits_out=logits)
    finally:
        quant.set_launch_overlap(False)
    got = logits.cpu().numpy()
    for b in (0, 21, 42, 63):
        ref_ids, ref_logits = DenseOracle(cfg, weights).generate(prompts[b], n_new)
        for i in range(n_new):
            rel = np.linalg.norm(got[i, b] - ref_logits[i]) / np.linalg.norm(ref_logits[i])
            assert rel < 1e-4, (b, i, rel)
            if ids[b][i] != ref_ids[i]:
                top = np.sort(ref_logits[i])[-2:]
                err = float(np.abs(got[i, b] - ref_logits[i]).max())
                assert float(top[1] - top[0]) <= 2 * err, (b, i)
                break
    assert quant.device_status() == 0


def test_batch_64_kv16_matches_oracle(cuda):
    """64 concurrent requests with f16 KV caches and split-operand products:
    requests 0, 21, 42 and 63 against the oracle model with the same binary16
    rounding of its cache (DenseOracle(kv16=True)), within 3e-4 (see
    test_kv16_decode_matches_oracle), same tokens."""
    import torch
    from hy_mt_rs_b200 import quant
    from hy_mt_rs_b200.model import DenseBatch, DenseConfig, DenseModel, random_weights
    from oracle.model import DenseOracle

    cfg = DenseConfig(layers=2, positions=96)
    weights = random_weights(cfg, cuda, seed=66)
    torch.cuda.synchronize()
    model = DenseModel(cfg, weights, cuda, gemm_precision=quant.GEMM_F32, kv16=True)
    rng = np.random.default_rng(66)
    B, n_new = 64, 5
    prompts = [rng.integers(0, cfg.vocab, int(n)).tolist() for n in rng.integers(1, 40, B)]
    stream = torch.cuda.Stream(cuda)
    try:
        batch = DenseBatch(model, B)
        assert batch.caches[0][0].dtype == torch.float16
        logits = torch.zeros(n_new, B, cfg.vocab, device=cuda)
        ids = batch.generate(prompts, n_new, stream, logits_out=logits)
    finally:
        quant.set_launch_overlap(False)
    got = logits.cpu().numpy()
    for b in (0, 21, 42, 63):
        ref_ids, ref_logits = DenseOracle(cfg, weights, kv16=True).generate(prompts[b], n_new)
        for i in range(n_new):
            rel = np.linalg.norm(got[i, b] - ref_logits[i]) / np.linalg.norm(ref_logits[i])
            assert rel < 3e-4, (b, i, rel)
            if ids[b][i] != ref_ids[i]:
                top = np.sort(ref_logits[i])[-2:]
                assert float(top[1] - top[0]) <= 2 * float(np.abs(got[i, b] - ref_logits[i]).max()), (b, i)
                break
    assert quant.device_status() == 0
