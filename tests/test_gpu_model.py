"""GPU parity of the single-token decode of the Dense architecture
(model.rs:374-547) against the CPU oracle step (oracle/model.py): greedy
token streams and the logits of every step, on a random-init model with the
1.8B shapes (Q2_0C linears, tied Q6_K embedding) and fewer layers so the
CPU side stays fast.  Both sides share the packed bytes, the rotary tables
(glibc sinf/cosf) and the x86 dot order of the norms; the products and the
softmax exponential differ in the last bits, hence a logits tolerance."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_dense_decode_matches_oracle(cuda):
    import torch
    from hy_mt_rs_b200 import quant
    from hy_mt_rs_b200.model import DenseConfig, DenseModel, random_weights
    from oracle.model import DenseOracle

    cfg = DenseConfig(layers=4, positions=64)
    weights = random_weights(cfg, cuda, seed=3)
    torch.cuda.synchronize()
    model = DenseModel(cfg, weights, cuda)
    oracle = DenseOracle(cfg, weights)
    prompt = [11, 4093, 77, 120000, 5, 42]
    n_new = 12
    stream = torch.cuda.Stream(cuda)
    logits = torch.zeros(n_new, cfg.vocab, device=cuda)
    try:
        ids = model.generate(prompt, n_new, stream, logits_out=logits)
    finally:
        quant.set_launch_overlap(False)
    ref_ids, ref_logits = oracle.generate(prompt, n_new)
    got = logits.cpu().numpy()
    for i in range(n_new):
        rel = np.linalg.norm(got[i] - ref_logits[i]) / np.linalg.norm(ref_logits[i])
        assert rel < 1e-4, (i, rel)
        if ids[i] != ref_ids[i]:
            top = np.sort(ref_logits[i])[-2:]
            margin = float(top[1] - top[0])
            err = float(np.abs(got[i] - ref_logits[i]).max())
            # the only acceptable divergence: a near-tie the numerics cannot order
            assert margin <= 2 * err, (i, ids[i], ref_ids[i], margin, err)
            break
    assert quant.device_status() == 0
    # the same stream again from the same graph (KV caches and position reset)
    again = model.generate(prompt, n_new, stream)
    assert again == ids
