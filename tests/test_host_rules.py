"""Host-side rules mirrored in Python, on CPU: the tensor-core product's
split-K choice (hyq_gemm.cu choose_splits / token_tile) that the bench's
launch counts rely on, checked against the grids the ncu launch lists of
the 64-request decode step and of MoE decode recorded (grid.z = slices)."""
import pytest

from hy_mt_rs_b200.quant import DType, gemm_launches, gemm_splits, gemm_tail_slices

Q2C, Q4K, Q6K = DType.Q2_0C, DType.Q4_K, DType.Q6_K


@pytest.mark.parametrize("tiles,K,M,dtype,splits", [
    (24, 2048, 64, Q2C, 4),     # 1.8B QKV at 64 requests: grid (24, 1, 4)
    (16, 2048, 64, Q2C, 4),     # O: (16, 1, 4)
    (96, 2048, 64, Q2C, 1),     # gate/up pair tiles: (96, 1, 1)
    (16, 6144, 64, Q2C, 6),     # down: (16, 1, 6)
    (944, 2048, 64, Q6K, 1),    # lm_head, split operands: (944, 1, 1)
    (16, 2048, 64, Q4K, 8),     # MoE shared gate/up at 64 tokens: (16, 1, 8)
    (16, 1024, 64, Q4K, 4),     # MoE shared down: (16, 1, 4)
    (48, 4096, 2048, Q4K, 1),   # 7B QKV at 2048 tokens: 384 tiles, no split
    (32, 4096, 512, Q4K, 2),    # 7B O at 512 tokens: 64 tiles, two slices in one wave
])
def test_gemm_splits_match_recorded_grids(tiles, K, M, dtype, splits):
    assert gemm_splits(tiles, K, M, dtype) == splits
    if M <= 128:  # split operands take the same token tile here
        assert gemm_splits(tiles, K, M, dtype, split=True) == splits
        assert gemm_launches(tiles, K, M, dtype, split=True) == 2 + (splits > 1)
    tail = gemm_tail_slices(tiles, K, M, dtype) > 1  # fp16 lm_head at 64 rows: its last wave is split
    assert gemm_launches(tiles, K, M, dtype) == 2 + (splits > 1) + tail


@pytest.mark.parametrize("tiles,K,M,dtype,z", [
    (224, 4096, 512, Q4K, 16),   # 7B gate/up at 512 tokens: 448 tiles, 4 past three waves, 16 slices each
    (224, 4096, 2048, Q4K, 8),   # 7B gate/up at 2048: 1792 tiles, 16 past twelve waves, 9 -> 8 whole slices
    (48, 4096, 2048, Q4K, 1),    # 7B QKV at 2048: 88 tiles past two waves (more than half): whole tiles
    (224, 4096, 128, Q4K, 1),    # 7B gate/up at 128: 76 past one wave
    (944, 2048, 64, Q6K, 2),     # lm_head at 64 rows, fp16 operands: 56 past six waves
    (96, 2048, 64, Q2C, 1),      # under one wave: split-K instead
])
def test_tail_split_rule(tiles, K, M, dtype, z):
    assert gemm_tail_slices(tiles, K, M, dtype) == z
    assert gemm_tail_slices(tiles, K, M, dtype, split=True) == 1
    assert gemm_tail_slices(tiles, K, M, dtype, pair=True) == 1
    assert gemm_launches(tiles, K, M, dtype) == 2 + (gemm_splits(tiles, K, M, dtype) > 1) + (z > 1)


def test_tail_slices_fit_the_last_wave():
    """The tail's slices never need more than the SMs left idle by the last
    full wave, each slice is whole block columns, and there are at least two."""
    for tiles in range(148, 2000, 7):
        for K, dtype in ((2048, Q2C), (4096, Q4K), (14336, Q6K), (2048, Q6K)):
            for M in (64, 128, 512):
                bn = 256 if M >= 256 else 128 if M > 64 else 64
                row_tiles = -(-tiles // -(-M // bn))
                z = gemm_tail_slices(row_tiles, K, M, dtype)
                grid = row_tiles * -(-M // bn)
                rem = grid % 148
                nwb = K // {Q2C: 512, Q4K: 256, Q6K: 256}[dtype]
                if z > 1:
                    assert 0 < rem <= 74 and rem * z <= 148 and z <= min(nwb, 16)
                    assert (nwb + z - 1) // z * (z - 1) < nwb  # every slice has a block column


def test_split_grid_stays_within_one_wave():
    for tiles in range(1, 148):
        for K, dtype in ((2048, Q2C), (6144, Q2C), (4096, Q4K), (14336, Q6K)):
            z = gemm_splits(tiles, K, 64, dtype)
            assert 1 <= z <= 16 and tiles * z <= max(148, tiles)


def test_reference_arm_runs_without_the_gpu_library():
    """The reference arm times the CPU port only: one step of it, in a fresh
    process, must not map libhyq.so, and its line carries the GPU arm's
    `config` dict verbatim (decode_config) with the whole lm_head."""
    import json
    import os
    import subprocess
    import sys

    code = (
        "import json, sys, types, bench\n"
        "a = types.SimpleNamespace(steps=1, warmup=0, gpus=1, path='f32', copies=4, no_overlap=False)\n"
        "print(json.dumps(bench.reference_arm(a)))\n"
        "maps = open('/proc/self/maps').read()\n"
        "print(json.dumps({'libhyq': 'libhyq.so' in maps, 'native': 'hy_mt_rs_b200._native' in sys.modules,\n"
        "                  'config': bench.decode_config(a, 1)}))\n")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    res = subprocess.run([sys.executable, "-c", code], cwd=root, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr
    line, probe = [json.loads(x) for x in res.stdout.strip().splitlines()[-2:]]
    assert not probe["libhyq"] and not probe["native"]
    assert line["impl"] == "reference" and line["config"] == probe["config"]
    assert "all 120832 lm_head rows" in line["cpu_baseline"]["sample"]
