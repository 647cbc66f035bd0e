"""Write tests/golden/reference_known_answers.json.

The reference (Rust) cannot be built here (no cargo/rustc), so its outputs cannot be generated.
What pins the oracle instead are the reference's own known-answer tests: this script records their
inputs, expected values and tolerances exactly as the Rust test sources state them, each with its
file:line. Run: python tests/golden/make_known_answers.py
"""
import json
from pathlib import Path

S16 = 1 << 16

cases = {
    "f32_linear_known_answer": {
        "source": "crates/v2/sharing/src/secure_linear.rs:416-461 (test_secure_linear_correctness)",
        "in": 4, "out": 2,
        "weight_in_out": [1.0, 0.0, 0.0, 1.0, 1.0, 1.0, 0.5, 0.5],
        "bias": [0.1, 0.2],
        "x": [1.0, 2.0, 3.0, 4.0],
        "share_seed": 42,
        "expected": [6.1, 7.2],
        "tol": 1e-5,
    },
    "f32_linear_shares_not_plaintext": {
        "source": "crates/v2/sharing/src/secure_linear.rs:463-498 (test_shares_are_not_plaintext)",
        "in": 4, "out": 2,
        "weight_in_out": [1.0] * 8,
        "bias": None,
        "x": [1.0, 2.0, 3.0, 4.0],
        "share_seed": 42,
        "expected": [10.0, 10.0],
        "tol": 1e-5,
    },
    "ring_identity": {
        "source": "crates/sharing/src/linear.rs:1264-1287 (test_secure_linear_identity)",
        "in": 4, "out": 4, "scale": 16,
        "weight_in_out": [S16 if i % 5 == 0 else 0 for i in range(16)],
        "bias": None,
        "x_f64": [1.0, 2.0, 3.0, 4.0],
        "expected": [1.0, 2.0, 3.0, 4.0],
        "tol": 0.01,
    },
    "ring_matches_plaintext": {
        "source": "crates/sharing/src/linear.rs:1289-1320 (test_secure_linear_matches_plaintext)",
        "in": 8, "out": 4, "scale": 16,
        "weight_in_out": [((i % 10) - 5) * (1 << 12) for i in range(32)],
        "bias": None,
        "x_f64": [i * 0.1 + 0.5 for i in range(8)],
        "max_lsb_vs_plaintext": 1,
    },
    "ring_bias": {
        "source": "crates/sharing/src/linear.rs:1322-1352 (test_secure_linear_with_bias)",
        "in": 2, "out": 2, "scale": 16,
        "weight_in_out": [S16, 0, 0, S16],
        "bias": [int(0.5 * S16), S16],
        "x_f64": [1.0, 1.0],
        "expected": [1.5, 2.0],
        "tol": 0.01,
    },
    "ring_matrix_multiply": {
        "source": "crates/sharing/tests/e2e_inference_test.rs:57-91 (test_secure_matrix_multiply_matches_plaintext)",
        "in": 2, "out": 3, "scale": 16,
        "weight_f64_in_out": [1.0, 2.0, 3.0, 4.0, 5.0, 6.0],
        "bias": None,
        "x_f64": [1.0, 2.0],
        "expected": [9.0, 12.0, 15.0],
        "tol": 0.01,
    },
    "ring_large_dimension": {
        "source": "crates/sharing/tests/e2e_inference_test.rs:202-241 (test_large_dimension_computation)",
        "in": 256, "out": 64, "scale": 16,
        "weight_f64_in_out": [((i % 100) - 50.0) / 100.0 for i in range(256 * 64)],
        "x_f64": [((i % 20) - 10.0) / 10.0 for i in range(256)],
        "check_indices": [0, 10, 32, 63],
        "tol": 0.5,
    },
    "fixed_roundtrip": {
        "source": "crates/fixed_point/src/fixed.rs:180-199 (test_roundtrip_f64)",
        "values": [0.0, 1.0, -1.0, 0.5, -0.5, 0.123456, -0.123456, 100.0, -100.0],
        "tol": 0.0001,
    },
    "fixed_add": {"source": "crates/fixed_point/src/fixed.rs:201-208", "a": 1.5, "b": 2.5, "expected": 4.0, "tol": 0.0001},
    "fixed_sub": {"source": "crates/fixed_point/src/fixed.rs:210-217", "a": 5.0, "b": 2.0, "expected": 3.0, "tol": 0.0001},
    "fixed_mul": {"source": "crates/fixed_point/src/fixed.rs:219-226", "a": 2.0, "b": 3.0, "expected": 6.0, "tol": 0.0001},
    "fixed_overflow": {"source": "crates/fixed_point/src/fixed.rs:238-243", "value": 100000.0, "scale": 16, "error": "Overflow"},
    "fixed_one": {"source": "crates/fixed_point/src/fixed.rs:252-256", "expected": 1.0, "tol": 0.0001},
    "beaver_triple_correctness": {
        "source": "crates/v2/sharing/src/beaver.rs:239-254 (test_beaver_triple_correctness)",
        "trials": 100, "tol": 1e-5,
    },
    "beaver_multiply_correctness": {
        "source": "crates/v2/sharing/src/beaver.rs:256-290 (test_secure_multiply_correctness)",
        "trials": 100, "x_range": [-10.0, 10.0], "share_range": [-10.0, 10.0], "tol": 1e-4,
    },
    "softmax_sums_to_one": {
        "source": "crates/v2/sharing/src/secure_nonlinear.rs:403-418 (test_secure_softmax)",
        "scores_c": [1.0, 2.0, 3.0], "scores_s": [0.0, 0.0, 0.0], "sum_tol": 0.01,
    },
    "rms_norm_unit_rms": {
        "source": "crates/v2/sharing/src/secure_nonlinear.rs:420-436 (test_secure_rms_norm)",
        "x_c": [1.0, 2.0, 3.0, 4.0], "x_s": [0.0, 0.0, 0.0, 0.0], "gamma": [1.0] * 4, "eps": 1e-6,
        "rms_tol": 0.1,
    },
    "silu_positive": {
        "source": "crates/v2/sharing/src/secure_nonlinear.rs:388-401 (test_secure_silu_approx)",
        "x_c": [0.0, 1.0, -1.0, 2.0, -2.0], "x_s": [0.0] * 5,
    },
}

out = Path(__file__).with_name("reference_known_answers.json")
out.write_text(json.dumps(cases, indent=1) + "\n")
print(f"wrote {out} ({len(cases)} cases)")
