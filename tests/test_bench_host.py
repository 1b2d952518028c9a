"""CPU: bench.py's host-side plumbing - the tensor-parallel layout of N ranks
for each workload, the workload shapes, and the algorithmic bytes a
tensor-parallel rank streams per token (the roofline's numerator)."""
import os
import sys

import pytest

import atlas_cuda

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402


def test_tp_layout():
    # the 7B model (4 KV heads): one group up to 4 ranks, then groups of 4
    assert bench.tp_layout(1, 4) == (1, 1)
    assert bench.tp_layout(2, 4) == (2, 1)
    assert bench.tp_layout(4, 4) == (4, 1)
    assert bench.tp_layout(8, 4) == (4, 2)
    # the 14B model (8 KV heads): one group of up to 8
    assert bench.tp_layout(8, 8) == (8, 1)
    with pytest.raises(SystemExit):
        bench.tp_layout(6, 4)


def test_workload_shapes():
    assert set(bench.SHAPES) == {"3b", "7b", "14b"}
    for name, cfg in bench.SHAPES.values():
        assert name in bench.WORKLOAD
        assert cfg["hidden"] % 256 == 0 and cfg["ffn"] % 256 == 0
        assert cfg["q_heads"] % cfg["kv_heads"] == 0
    # the weight bytes the bench lines quote (4.62 GB for the 7B, 9.01 GB for the 14B)
    assert abs(bench.weight_bytes(bench.CFG2) / 1e9 - 4.62) < 0.01
    assert abs(bench.weight_bytes(bench.CFG3) / 1e9 - 9.01) < 0.01
    assert bench.LONG_PROMPT == 8192 and bench.LONG_GEN == 512


@pytest.mark.parametrize("name,size", [("cfg2", 2), ("cfg2", 4), ("cfg3", 2), ("cfg3", 4), ("cfg3", 8)])
def test_rank_bytes_cover_the_model(name, size):
    """The ranks' algorithmic weight bytes add up to the whole model's, plus
    the attn_output block columns that two ranks share where a head split
    falls inside a 256-element block (7B on 4 ranks: 7 heads of 128 each)."""
    cfg = bench.CFG2 if name == "cfg2" else bench.CFG3
    shape = {k: cfg[k] for k in ("hidden", "q_heads", "kv_heads", "ffn", "vocab")}
    slices = [atlas_cuda.tp_slice(shape, r, size).as_dict() for r in range(size)]
    total = sum(bench.weight_bytes(cfg, sl) for sl in slices)
    whole = bench.weight_bytes(cfg)
    shared_blocks = sum(sl["o_blocks"] for sl in slices) - cfg["q_heads"] * 128 // 256
    o_block_bytes = cfg["layers"] * cfg["hidden"] * 256 * bench.Q4K
    # every rank also reads the 4-byte-per-element norm vectors and the final norm
    norms = (size - 1) * (cfg["layers"] * 4 * 2 * cfg["hidden"] + 4 * cfg["hidden"])
    assert total == pytest.approx(whole + shared_blocks * o_block_bytes + norms, rel=1e-9)
