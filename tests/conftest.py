import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden", "quant.json")
DTYPES = {"F32": 0, "F16": 1, "Q4_K": 2, "Q6_K": 3, "Q8_0": 4, "Q2_0C": 5, "STQ1_0": 6}


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built libhyq.so")


@pytest.fixture(scope="session")
def golden_cases():
    with open(GOLDEN) as f:
        data = json.load(f)
    cases = []
    for c in data["cases"]:
        cases.append({
            "dtype": DTYPES[c["dtype"]],
            "name": c["dtype"],
            "encoded": np.frombuffer(bytes.fromhex(c["encoded_hex"]), dtype=np.uint8).copy(),
            "bits": np.array(c["expected_f32_bits"], dtype=np.uint32),
        })
    return cases


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import hy_mt_rs_b200.quant  # noqa: F401  (loads libhyq.so or raises)
    return torch.device("cuda", 0)
