"""Regenerate tests/golden/quant.json from the reference's decoder fixture.

The reference pins its block decoders with tests/fixtures/quant.json: three
synthetic blocks per packed type, with expected f32 bit patterns produced by
pinned C decoders (llama.cpp forks), read by tests/quant_reference.rs:12-50.
This script copies those vectors (dtype, encoded bytes, expected bits) into
this repository so that the tests can run where the reference tree is absent.
Run it where the reference checkout is mounted:

    python tests/golden/make_golden.py /path/to/hy-mt-rs
"""
import json
import os
import sys


def main(ref_root):
    src = os.path.join(ref_root, "tests", "fixtures", "quant.json")
    with open(src) as f:
        cases = json.load(f)
    out = []
    for case in cases:
        out.append({
            "dtype": case["dtype"],
            "encoded_hex": case["encoded_hex"],
            "expected_f32_bits": case["expected_f32_bits"],
            "oracle": case.get("oracle"),
        })
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "quant.json")
    with open(dst, "w") as f:
        json.dump({"source": "hy-mt-rs tests/fixtures/quant.json", "cases": out}, f, indent=1)
        f.write("\n")
    print(f"wrote {dst}: {len(out)} cases")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <reference checkout>")
    main(sys.argv[1])
