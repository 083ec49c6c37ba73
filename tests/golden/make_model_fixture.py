"""Writes tests/golden/dense_config4.npz: greedy token streams of the CPU
oracle model (oracle/model.py, composed from the pinned C primitives) for
BASELINE config 4, the workload `bench.py --workload model` runs:

  * the Hy-MT2-1.8B architecture at full size: 32 layers, hidden 2048,
    16/4 heads of 128, SwiGLU 6144, vocab 120832, Q2_0C linears, tied Q6_K
    embedding, f32 KV cache of 512 positions;
  * random-init weights hy_mt_rs_b200.model.random_weights(seed=1);
  * prompts of 256 seeded token ids (numpy default_rng(0), one draw of 256 per
    request in request order: request 0 is the single-request prompt) and
    256 greedy tokens each.

Requests 0, 21, 42 and 63 of the 64 concurrent ones are recorded.  For each:
the prompt, the 256 tokens, the top-1 minus top-2 logit margin and the L2
norm of the logits at every step; for request 0 also the full logits of the
first and last steps; and the SHA-256 of the model bytes (weights_digest),
so the GPU test can prove it decodes the same model.

Test infrastructure: run once on a CPU (about 6 minutes per request on 8
cores), `python tests/golden/make_model_fixture.py`.
"""
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

OUT = os.path.join(ROOT, "tests", "golden", "dense_config4.npz")
SEED, N_PROMPT, N_NEW, BATCH = 1, 256, 256, 64
REQUESTS = (0, 21, 42, 63)
LOGIT_STEPS = (0, N_NEW - 1)


def prompts(vocab):
    rng = np.random.default_rng(0)
    return [rng.integers(0, vocab, N_PROMPT).tolist() for _ in range(BATCH)]


def main():
    from hy_mt_rs_b200.model import DenseConfig, random_weights, weights_digest
    from oracle.model import DenseOracle

    cfg = DenseConfig(layers=32, positions=N_PROMPT + N_NEW)
    weights = random_weights(cfg, "cpu", seed=SEED)
    digest = weights_digest(weights)
    all_prompts = prompts(cfg.vocab)
    rec = {"prompts": [], "tokens": [], "margins": [], "norms": []}
    logits_keep = None
    for r in REQUESTS:
        t0 = time.time()
        oracle = DenseOracle(cfg, weights)
        ids, logits = oracle.generate(all_prompts[r], N_NEW)
        top2 = np.sort(np.stack(logits), axis=1)[:, -2:]
        rec["prompts"].append(all_prompts[r])
        rec["tokens"].append(ids)
        rec["margins"].append(top2[:, 1] - top2[:, 0])
        rec["norms"].append([float(np.linalg.norm(l)) for l in logits])
        if r == 0:
            logits_keep = np.stack([logits[i] for i in LOGIT_STEPS])
        print(f"request {r}: {time.time() - t0:.0f} s, min margin {float(np.min(rec['margins'][-1])):.3g}",
              flush=True)
    np.savez_compressed(
        OUT, requests=np.array(REQUESTS, np.int32), prompts=np.array(rec["prompts"], np.int32),
        tokens=np.array(rec["tokens"], np.int32), margins=np.array(rec["margins"], np.float32),
        norms=np.array(rec["norms"], np.float32), logit_steps=np.array(LOGIT_STEPS, np.int32),
        logits=logits_keep.astype(np.float32), digest=np.array(digest), seed=np.array(SEED),
        layers=np.array(cfg.layers), positions=np.array(cfg.positions), batch=np.array(BATCH))
    print("wrote", OUT)


if __name__ == "__main__":
    main()
