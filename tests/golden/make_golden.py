"""Writes tests/golden/reference_known_answers.json.

The reference project (AtelierArith/tenferro-decision-rs) holds no per-op golden
tensors; its pins for this path are the known-answer values and explicit inputs
written in its own tests. This script records those values, each with the
reference file and line range it comes from, and -- when the reference source
tree is available (pass its root as argv[1] or set TFX_REFERENCE_ROOT) --
checks that every recorded literal appears verbatim in the cited lines, so the
fixture cannot drift from its source. The JSON follows the reference's fixture
schema (name / metadata / tensors with dtype, order, shape, data).

Run:  python tests/golden/make_golden.py [reference_root]
"""

from __future__ import annotations

import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "reference_known_answers.json")

# Each case: source file, inclusive line range, literals (as written in the
# source) that must appear in that range, and the tensors/values.
CASES = [
    {
        "name": "erf_f32_mlx_known_values",
        "source": "crates/tenferro-ext/tests/erf.rs",
        "lines": [23, 42],
        "literals": ["-3.0f32", "-0.5", "-0.999_977_9f32", "-0.842_700_8", "-0.520_499_9",
                     "0.520_499_9", "0.842_700_8", "0.999_977_9", "1e-6"],
        "tolerance": {"abs": 1e-6},
        "tensors": {
            "x": {"dtype": "f32", "shape": [7], "data": [-3.0, -1.0, -0.5, 0.0, 0.5, 1.0, 3.0]},
            "erf": {"dtype": "f32", "shape": [7],
                    "data": [-0.9999779, -0.8427008, -0.5204999, 0.0, 0.5204999, 0.8427008,
                             0.9999779]},
        },
    },
    {
        "name": "gelu_erf_f32_known_values",
        "source": "crates/tenferro-ext/tests/erf.rs",
        "lines": [45, 54],
        "literals": ["-3.0f32", "2.0", "-0.004_049_7f32", "-0.158_655_3", "0.841_344_8",
                     "1.954_499_7", "1e-6"],
        "tolerance": {"abs": 1e-6},
        "tensors": {
            "x": {"dtype": "f32", "shape": [5], "data": [-3.0, -1.0, 0.0, 1.0, 2.0]},
            "gelu": {"dtype": "f32", "shape": [5],
                     "data": [-0.0040497, -0.1586553, 0.0, 0.8413448, 1.9544997]},
        },
    },
    {
        "name": "erf_f32_branch_boundary_sweep",
        "source": "crates/tenferro-ext/tests/erf.rs",
        "lines": [57, 83],
        "literals": ["-20000..=20000", "0.0003", "0.927_734_4f32", "1e-30", "1e-6"],
        "tolerance": {"abs": 1e-6},
        "sweep": {"start": -20000, "stop": 20000, "step": 0.0003},
        "boundary": 0.9277344,
        "extra": [0.0, -0.0, 1e-30, -1e-30],
    },
    {
        "name": "erf_f32_special_values",
        "source": "crates/tenferro-ext/tests/erf.rs",
        "lines": [86, 103],
        "literals": ["f32::INFINITY", "f32::NEG_INFINITY", "f32::MAX", "-f32::MAX", "f32::NAN",
                     "[1.0, -1.0, 1.0, -1.0]"],
        "tensors": {
            "x": {"dtype": "f32", "shape": [7],
                  "data": [0.0, "-0.0", "inf", "-inf", "f32::MAX", "-f32::MAX", "nan"]},
            "erf": {"dtype": "f32", "shape": [7],
                    "data": [0.0, "-0.0", 1.0, -1.0, 1.0, -1.0, "nan"]},
        },
    },
    {
        "name": "gelu_erf_native_composition_sweep",
        "source": "crates/tenferro-ext/tests/erf.rs",
        "lines": [132, 145],
        "literals": ["-20000..=20000", "0.0005", "2e-6"],
        "tolerance": {"abs": 2e-6},
        "sweep": {"start": -20000, "stop": 20000, "step": 0.0005},
    },
    {
        "name": "erf_gelu_cuda_sweep",
        "source": "crates/tenferro-ext/tests/erf_cuda.rs",
        "lines": [12, 79],
        "literals": ["-2000..=2000", "0.005", "[1.0f32, 0.5, -0.75]", "2e-6", "4e-6"],
        "tolerance": {"erf_abs": 2e-6, "gelu_abs": 4e-6},
        "sweep": {"start": -2000, "stop": 2000, "step": 0.005},
        "scales": [1.0, 0.5, -0.75],
    },
    {
        "name": "erf_f64_native_sweep",
        "source": "crates/tenferro-ext/tests/erf.rs",
        "lines": [106, 129],
        "literals": ["-1000..=1000", "0.006", "5e-16"],
        "tolerance": {"abs": 5e-16},
        "sweep": {"start": -1000, "stop": 1000, "step": 0.006},
    },
    {
        "name": "layernorm_ff_matches_naive",
        "source": "crates/tenferro-ext/src/layernorm.rs",
        "lines": [313, 376],
        "literals": ["6364136223846793005", "(5usize, 3usize, 2usize)", "(1024, 16, 1)",
                     "(1024, 8, 8)", "1e-5f32", "let mut state = 7u64;", "1e-5"],
        "tolerance": {"abs": 1e-5},
        "lcg": {"multiplier": 6364136223846793005, "increment": 1, "shift": 40, "seed": 7},
        "shapes": [[5, 3, 2], [1024, 16, 1], [1024, 8, 8]],
        "eps": 1e-5,
    },
    {
        "name": "geglu_thread_invariance",
        "source": "crates/cpu-kernels/src/lib.rs",
        "lines": [1375, 1402],
        "literals": ["(257, 65)", "(i % 103) as f32 - 51.0) / 7.0", "[1, 3]"],
        "intermediate": 257,
        "cols": 65,
        "threads": [1, 3],
    },
    {
        "name": "masked_attention_empty_rows_and_masked_nonfinite",
        "source": "crates/cpu-kernels/src/lib.rs",
        "lines": [1213, 1250],
        "literals": ["let length = 65;", "keep[query + length * 32] = false;",
                     "[1.0f32, f32::NAN, f32::INFINITY]", "actual.is_nan()", "1e-6"],
        "length": 65,
        "masked_key": 32,
        "empty_queries": [0, 64],
        "excluded_values": [1.0, "nan", "inf"],
    },
    {
        "name": "laya_attention_block_masked_nonfinite_and_empty_rows",
        "source": "crates/cpu-kernels/src/lib.rs",
        "lines": [1212, 1250],
        "literals": ["let length = 65;", "let d = 4;",
                     "qkv[3 * d * key + 2 * d + feature] = (feature + 1) as f32;",
                     "keep[query + length * 32] = false;", "keep[length * key] = false;",
                     "keep[length - 1 + length * key] = false;",
                     "[1.0f32, f32::NAN, f32::INFINITY]",
                     "laya_attention_block_into(&qkv, &keep, d, 1, length, 1, 0.0, &mut output);",
                     "query == 0 || query == length - 1", "<= 1e-6"],
        "length": 65, "hidden": 4, "heads": 1, "batch": 1, "rope_base": 0.0,
        "masked_key": 32, "empty_queries": [0, 64],
        "excluded_values": [1.0, "nan", "inf"],
        "tolerance": {"abs": 1e-6},
    },
    {
        "name": "layer_norm_f64_primitive",
        "source": "crates/tenferro-infer/tests/primitives.rs",
        "lines": [33, 72],
        "literals": ["1.0, 2.0, 3.0, -1.0, 0.0, 1.0, 2.0, 2.0, 2.0, 0.5, -1.5, 4.0",
                     "0.5, 1.0, 2.0", "0.1, -0.2, 0.3", "1e-5", "1e-9"],
        "tolerance": {"abs": 1e-9},
        "rows": 4, "cols": 3, "eps": 1e-5,
        "tensors": {
            "x": {"dtype": "f64", "order": "col-major", "shape": [4, 3],
                  "data": [1.0, 2.0, 3.0, -1.0, 0.0, 1.0, 2.0, 2.0, 2.0, 0.5, -1.5, 4.0]},
            "weight": {"dtype": "f64", "shape": [3], "data": [0.5, 1.0, 2.0]},
            "bias": {"dtype": "f64", "shape": [3], "data": [0.1, -0.2, 0.3]},
        },
    },
    {
        "name": "rms_norm_f64_primitive",
        "source": "crates/tenferro-infer/tests/primitives.rs",
        "lines": [76, 121],
        "literals": ["1.0, -2.0, 0.5, 3.0, 0.0, 1.0, -1.0, 2.0, 4.0, 4.0, 4.0, 4.0",
                     "1.0, 0.5, -0.25, 2.0", "1e-6", "1e-9"],
        "tolerance": {"abs": 1e-9},
        "rows": 3, "cols": 4, "eps": 1e-6,
        "tensors": {
            "x": {"dtype": "f64", "order": "col-major", "shape": [3, 4],
                  "data": [1.0, -2.0, 0.5, 3.0, 0.0, 1.0, -1.0, 2.0, 4.0, 4.0, 4.0, 4.0]},
            "weight": {"dtype": "f64", "shape": [4], "data": [1.0, 0.5, -0.25, 2.0]},
        },
    },
    {
        "name": "softmax_f64_primitive",
        "source": "crates/tenferro-infer/tests/primitives.rs",
        "lines": [125, 162],
        "literals": ["1.0, 2.0, 3.0, 0.0, -1.0, -2.0, 0.5, 0.5, 5.0, -5.0, 0.0, 1.0", "1e-12"],
        "tolerance": {"abs": 1e-12},
        "rows": 3, "cols": 4,
        "tensors": {
            "x": {"dtype": "f64", "order": "col-major", "shape": [3, 4],
                  "data": [1.0, 2.0, 3.0, 0.0, -1.0, -2.0, 0.5, 0.5, 5.0, -5.0, 0.0, 1.0]},
        },
    },
    {
        "name": "rms_norm_rank3_f64_primitive",
        "source": "crates/tenferro-infer/tests/primitives.rs",
        "lines": [164, 195],
        "literals": ["(i as f64) * 0.37 - 2.0", "1.0, 0.5, -0.25, 2.0", "1e-9"],
        "tolerance": {"abs": 1e-9},
        "shape": [2, 3, 4], "eps": 1e-6,
        "weight": [1.0, 0.5, -0.25, 2.0],
    },
    {
        "name": "rope_modernbert_f64_primitive",
        "source": "crates/tenferro-infer/tests/primitives.rs",
        "lines": [299, 335],
        "literals": ["1.0, 0.0, 0.0, 1.0, 2.0, 1.0, 3.0, 0.0, 0.5, -1.0, 2.0, 2.0",
                     "let base = 10000.0;", "1e-12"],
        "tolerance": {"abs": 1e-12},
        "seq": 3, "head": 4, "base": 10000.0,
        "tensors": {
            "x": {"dtype": "f64", "order": "col-major", "shape": [3, 4],
                  "data": [1.0, 0.0, 0.0, 1.0, 2.0, 1.0, 3.0, 0.0, 0.5, -1.0, 2.0, 2.0]},
        },
    },
    {
        "name": "rope_qwen_partial_f64_primitive",
        "source": "crates/tenferro-infer/tests/primitives.rs",
        "lines": [337, 372],
        "literals": ["let rotary = 2;", "(i as f64) * 0.1 - 0.3", "let base = 10000.0;", "1e-12"],
        "tolerance": {"abs": 1e-12},
        "heads": 2, "seq": 3, "head": 4, "rotary": 2, "base": 10000.0,
    },
    {
        "name": "gelu_erf_fused_cuda_parity_bound",
        "source": "crates/tenferro-ext/tests/erf_cuda.rs",
        "lines": [60, 79],
        "literals": ["std::f32::consts::FRAC_1_SQRT_2", "<= 2e-6", "<= 4e-6"],
        "tolerance": {"erf_abs": 2e-6, "gelu_abs": 4e-6},
    },
]


def _check_against_reference(root: str) -> list[str]:
    problems = []
    for case in CASES:
        path = os.path.join(root, case["source"])
        with open(path, encoding="utf-8") as fh:
            lines = fh.read().splitlines()
        lo, hi = case["lines"]
        window = "\n".join(lines[lo - 1:hi])
        for lit in case["literals"]:
            if lit not in window:
                problems.append(f"{case['name']}: {lit!r} not in {case['source']}:{lo}-{hi}")
    return problems


def main(argv: list[str]) -> int:
    root = argv[1] if len(argv) > 1 else os.environ.get("TFX_REFERENCE_ROOT", "")
    if root and os.path.isdir(root):
        problems = _check_against_reference(root)
        if problems:
            print("\n".join(problems))
            return 1
        print(f"all {len(CASES)} cases verified against {root}")
    doc = {
        "name": "reference_known_answers",
        "metadata": {
            "source": "AtelierArith/tenferro-decision-rs test sources (file:line per case)",
            "notes": "known-answer values and explicit inputs of the reference's own tests "
                     "for the non-GEMM extension ops; written by tests/golden/make_golden.py",
        },
        "cases": CASES,
    }
    with open(OUT, "w", encoding="utf-8") as fh:
        json.dump(doc, fh, indent=1)
        fh.write("\n")
    print(f"wrote {OUT}")
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv))
