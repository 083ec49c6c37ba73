"""Greedy token-stream identity at BASELINE config 4's full size, against
the CPU oracle model: the Hy-MT2-1.8B architecture (32 layers, Q2_0C
linears, tied Q6_K embedding, vocab 120832, f32 KV cache), random-init
weights (seed 1), 256-token prompts and 256 greedy tokens -- the workload
`bench.py --workload model` runs.  The oracle's streams are the committed
fixture tests/golden/dense_config4.npz (tests/golden/make_model_fixture.py,
about 8 CPU-minutes per request); the model bytes are checked against its
SHA-256 first, so both sides decode the same model.

Paths checked, each for identical 256-token streams:
  * one request, prompt fed token by token (f32 batch-1 products), through
    the per-kernel graph and through the persistent step kernel;
  * one request, prompt in one batched forward with f32-accurate
    split-operand tensor-core products (GEMM_F32);
  * 64 concurrent requests (DenseBatch, tensor-core products at 64 rows,
    GEMM_F32): requests 0, 21, 42 and 63 against their own oracle streams.
The logits of the first and last step of request 0 are also held to 1e-4
relative L2 of the oracle's."""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

FIXTURE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "dense_config4.npz")


@pytest.fixture(scope="module")
def c4(cuda):
    import torch
    from hy_mt_rs_b200.model import DenseConfig, random_weights, weights_digest

    fx = dict(np.load(FIXTURE))
    cfg = DenseConfig(layers=int(fx["layers"]), positions=int(fx["positions"]))
    weights = random_weights(cfg, cuda, seed=int(fx["seed"]))
    torch.cuda.synchronize()
    assert weights_digest(weights) == str(fx["digest"]), "the device model's bytes differ from the fixture's"
    return cfg, weights, fx


def assert_stream(ids, fx, k, what):
    """ids must equal the oracle's stream k; on a difference, report the step
    and the oracle's top-2 margin there."""
    ref = fx["tokens"][k].tolist()
    if ids != ref:
        i = next(j for j in range(len(ref)) if ids[j] != ref[j])
        pytest.fail(f"{what}: request {int(fx['requests'][k])} diverges at step {i} "
                    f"(got {ids[i]}, oracle {ref[i]}, oracle top-2 margin {float(fx['margins'][k][i]):.3g})")


def assert_logits(logits, fx):
    for j, step in enumerate(fx["logit_steps"].tolist()):
        ref = fx["logits"][j]
        rel = np.linalg.norm(logits[step] - ref) / np.linalg.norm(ref)
        assert rel < 1e-4, (step, rel)


def _generate(model, fx, n_new, **kw):
    import torch
    from hy_mt_rs_b200 import quant

    stream = torch.cuda.Stream(model.device)
    logits = torch.zeros(n_new, model.cfg.vocab, device=model.device)
    try:
        ids = model.generate(fx["prompts"][0].tolist(), n_new, stream, logits_out=logits, **kw)
    finally:
        quant.set_launch_overlap(False)
    assert quant.device_status() == 0
    return ids, logits.cpu().numpy()


def test_config4_one_request_token_by_token(c4):
    from hy_mt_rs_b200.model import DenseModel

    cfg, weights, fx = c4
    model = DenseModel(cfg, weights, weights["embed"].device)
    ids, logits = _generate(model, fx, fx["tokens"].shape[1])
    assert_stream(ids, fx, 0, "per-kernel graph")
    assert_logits(logits, fx)


def test_config4_one_request_persistent_step(c4):
    from hy_mt_rs_b200.model import DenseModel

    cfg, weights, fx = c4
    model = DenseModel(cfg, weights, weights["embed"].device, fused=True)
    ids, logits = _generate(model, fx, fx["tokens"].shape[1])
    assert_stream(ids, fx, 0, "persistent step kernel")
    assert_logits(logits, fx)


def test_config4_one_request_batched_prefill_f32_products(c4):
    from hy_mt_rs_b200 import quant
    from hy_mt_rs_b200.model import DenseModel

    cfg, weights, fx = c4
    model = DenseModel(cfg, weights, weights["embed"].device, gemm_precision=quant.GEMM_F32)
    ids, logits = _generate(model, fx, fx["tokens"].shape[1], batched_prefill=True)
    assert_stream(ids, fx, 0, "batched prefill, split-operand products")
    assert_logits(logits, fx)


def test_config4_64_requests_f32_products(c4):
    import torch
    from hy_mt_rs_b200 import quant
    from hy_mt_rs_b200.model import DenseBatch, DenseModel

    cfg, weights, fx = c4
    dev = weights["embed"].device
    B, n_prompt, n_new = int(fx["batch"]), fx["prompts"].shape[1], fx["tokens"].shape[1]
    rng = np.random.default_rng(0)     # the fixture's (and the bench's) prompts, in request order
    prompts = [rng.integers(0, cfg.vocab, n_prompt).tolist() for _ in range(B)]
    for k, r in enumerate(fx["requests"].tolist()):
        assert prompts[r] == fx["prompts"][k].tolist()
    model = DenseModel(cfg, weights, dev, gemm_precision=quant.GEMM_F32)
    stream = torch.cuda.Stream(dev)
    try:
        batch = DenseBatch(model, B)
        ids = batch.generate(prompts, n_new, stream)
    finally:
        quant.set_launch_overlap(False)
    assert quant.device_status() == 0
    for k, r in enumerate(fx["requests"].tolist()):
        assert_stream(ids[r], fx, k, "64 concurrent requests, split-operand products")
