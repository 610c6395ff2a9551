"""CPU checks of bench.py's metric definitions and of its reference arm.

The byte counts are the metric: the chain's algorithmic bytes must be the
BASELINE configs[4] figure, the softmax's touched bytes must average to the
figure the roofline line divides by, and the reference arm (the oracle chain on
the host cores) must print the contract's JSON line. No GPU is used.
"""

import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_chain_bytes_are_the_baseline_figure():
    b = bench.chain_bytes()
    assert sum(b.values()) == 3_170_899_968
    assert b["layernorm"] == b["layernorm2"] == 201_329_664
    assert b["softmax"] == 2 * 64 * 12 * 512 * 512 * 4
    assert b["geglu"] == 3 * 1152 * 32768 * 4


def test_softmax_touched_bytes_of_the_chain():
    c = bench.CHAIN
    local = bench.softmax_touched_bytes(c["batch"], c["heads"], c["seq"], c["window"],
                                        c["seq"] - c["pad"])
    glob = bench.softmax_touched_bytes(c["batch"], c["heads"], c["seq"], -1, c["seq"] - c["pad"])
    assert (local + glob) // 2 == 1_272_127_488
    written = c["batch"] * c["heads"] * c["seq"] ** 2 * 4
    assert written < local < glob <= 2 * written  # every probability written, kept scores read


def test_moved_bytes_are_what_the_kernels_move():
    """value's bytes: the fused add + LayerNorm as one pass and the softmax's
    touched bytes, 2,731,751,424 per step averaged over a window and a global
    step; below the reference-counted 3,170,899,968 by exactly the skipped
    score chunks and the one pass the fusion removes."""
    w, g = bench.chain_moved_bytes(0), bench.chain_moved_bytes(1)
    assert bench.chain_moved_bytes_total(2) == 2 * 2_731_751_424
    assert w["add_layernorm"] == g["add_layernorm"] == 4 * 768 * 32768 * 4 + 768 * 4
    assert w["masked_softmax"] < g["masked_softmax"]  # the window keeps fewer chunks
    ref = bench.chain_bytes()
    fusion_saving = ref["residual_add"] + ref["layernorm2"] - w["add_layernorm"]
    skipped = ref["softmax"] - (w["masked_softmax"] + g["masked_softmax"]) // 2
    assert sum(ref.values()) - 2_731_751_424 == fusion_saving + skipped
    weights = 2 * 768 * 4  # the two LayerNorm gains per step do not scale with batch
    assert (bench.chain_moved_bytes_total(2, batch=8) - 2 * weights) * 8 == \
        bench.chain_moved_bytes_total(2) - 2 * weights


def test_chain_elements():
    T = 64 * 512
    assert bench.chain_elements() == 768 * T * 5 + 64 * 12 * 512 * 512 + 1152 * T


def test_pcie_call_model():
    rates = {"h2d": 50.0, "d2h": 50.0, "both_each": 40.0}
    # equal directions: both at the concurrent rate
    assert bench.pcie_call_seconds(4e9, 4e9, rates) == pytest.approx(0.1)
    # 4 GB in, 2 GB out: 2 GB each way concurrently, then 2 GB in alone
    assert bench.pcie_call_seconds(4e9, 2e9, rates) == pytest.approx(2e9 / 40e9 + 2e9 / 50e9)


def test_percentile_helper():
    assert bench.pct([3, 1, 2], 0.5) == 2
    assert bench.pct(list(range(11)), 0.1) == 1
    assert bench.pct(list(range(11)), 0.9) == 9


def test_reference_arm_prints_the_contract_line():
    res = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                          "--steps", "3", "--warmup", "3"], capture_output=True, text=True,
                         timeout=600, cwd=ROOT)
    assert res.returncode == 0, res.stderr[-2000:]
    line = json.loads(res.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    assert line["metric"] == bench.METRIC and line["unit"] == "GB/s"
    assert line["value"] > 0 and line["higher_is_better"] is True
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["cpu_baseline"]["value"] == line["value"]
    # the same configuration as the GPU arm: batch 64 x seq 512, the same bytes
    assert line["config"]["global_batch"] == 64 and line["config"]["seq_len"] == 512
    assert line["config"]["tokens_per_gpu"] == 32768
    assert line["bytes_moved_per_step"] == bench.chain_moved_bytes_total(3) // 3
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["e2e"]["value"] == line["value"]


def test_warmup_below_three_is_refused():
    res = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                          "--steps", "1", "--warmup", "2"], capture_output=True, text=True,
                         timeout=120, cwd=ROOT)
    assert res.returncode != 0 and "--warmup must be >= 3" in res.stderr
