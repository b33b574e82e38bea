"""Writes tests/golden/reference_goldens.json.

The reference (a Rust workspace) keeps its known-answer values as inline
constants in its tests; there are no golden files.  This script transcribes
those constants, each with the reference file:line it comes from, into a
fixture the CPU oracle and the GPU tests are checked against.  It reads
nothing at run time; re-run it only to regenerate the JSON.
"""
import json
from pathlib import Path

TINY_NNUE = {
    "source": "crates/bulletou_lib/src/value/fast_nnue.rs:501-530 (tiny_weights); "
              "crates/cuda_cpp/src/bin/smoke.rs:279-318",
    "shape": [4, 2, 2, 1],
    "weights": {
        "l0w": [0.2, 0.3, 0.4, -0.1, -0.3, 0.5, 0.7, 0.9],
        "l0b": [0.1, 0.2],
        "l1w": [0.5, -0.2, 0.1, 0.3, -0.4, 0.2, 0.6, 0.1],
        "l1b": [0.05, 0.1],
        "l2w": [0.7, -0.2],
        "l2b": [0.2],
        "outw": [1.5],
        "outb": [0.05],
    },
}

TINY_SFNN_FAST = {
    "source": "crates/bulletou_lib/src/value/fast_sfnn.rs:663-705 (tiny_shape / tiny_batch / tiny_weights)",
    "shape": [4, 4, 2, 1, 2, 2],
    "batch": 2, "max_active": 3, "stm": [0, 1, -1, 3, -1, -1], "nstm": [2, -1, -1, 0, 2, -1], "buckets": [0, 1],
    "weights": {
        "l0w": [0.2, 0.1, -0.1, 0.0, -0.1, 0.2, 0.1, 0.2, 0.0, -0.2, 0.2, 0.1, 0.3, 0.0, -0.3, 0.2],
        "l0b": [0.1, 0.2, 0.3, 0.4],
        "l1w": [1.0, 0.0, 0.0, 0.0, 0.0, 1.0, 0.0, 1.0, 0.0, 0.0, 0.0, 0.0,
                0.0, 0.0, 0.0, 1.0, 0.0, 0.0, 0.0, 0.0, 1.0, 0.0, 1.0, 0.0],
        "l1b": [0.0] * 6,
        "l2w": [1.0, 0.0, 0.0, 0.0, 0.0, 1.0, 0.0, 0.0, 1.0, 0.0, 1.0, 0.0, 0.0, 1.0, 0.0, 1.0],
        "l2b": [0.0] * 4,
        "l3w": [2.0, -0.5, -1.0, 0.8],
        "l3b": [0.1, -0.02],
    },
    "trace_source": "crates/bulletou_lib/src/value/fast_sfnn.rs:513-541 (scalar_trace_exposes_intermediate_activations)",
    "stm_l0": [0.2, 0.5, 0.3, 0.6, 0.4, 0.2, 0.0, 0.6],
    "nstm_l0": [0.1, 0.0, 0.5, 0.5, 0.3, 0.1, 0.4, 0.5],
    "combined": [0.05953125, 0.29765625, 0.049609375, 0.0, 0.0, 0.1190625, 0.1190625, 0.049609375],
    "l1": [0.05953125, 0.29765625, 0.0, 0.049609375, 0.0, 0.1190625],
    "l2_input": [0.0035162825, 0.08790706, 0.05953125, 0.29765625, 0.0024418628, 0.0, 0.049609375, 0.0],
    "l2": [0.0035162825, 0.08790706, 0.05205124, 0.0],
    "outputs": [0.06307903, 0.04701126],
    "tolerance": 1e-6,
}

TINY_SFNN_RUNNER = {
    "source": "crates/cuda_cpp/src/lib.rs:14180-14250 (tiny_sfnn_shape / tiny_sfnn_weights, shared L1/L2/L3 factors)",
    "shape": [4, 4, 2, 1, 2, 2],
    "weights": {
        "l0w": [0.2, 0.3, 0.4, 0.5, 0.1, -0.2, 0.3, -0.4, -0.3, 0.2, 0.6, 0.1, 0.7, 0.4, -0.5, 0.2],
        "l0b": [0.05, 0.1, 0.15, 0.2],
        "l1w": [0.4, -0.1, 0.2, 0.3, 0.1, 0.5, -0.2, 0.4, -0.3, 0.2, 0.6, -0.1,
                0.2, 0.3, -0.4, 0.1, -0.2, 0.4, 0.1, 0.5, 0.3, -0.5, 0.2, 0.1],
        "l1b": [0.01, 0.02, 0.03, -0.01, 0.04, -0.02],
        "l1fw": [0.01, -0.02, 0.03, -0.01, 0.02, -0.03, 0.04, 0.01, -0.02, 0.02, -0.04, 0.01],
        "l1fb": [0.005, -0.006, 0.007],
        "l2w": [0.3, -0.1, 0.2, 0.4, -0.2, 0.5, 0.1, -0.3, 0.1, 0.2, -0.4, 0.3, 0.4, -0.2, 0.3, 0.1],
        "l2b": [0.02, -0.03, 0.01, 0.04],
        "l2fw": [0.01, -0.02, 0.03, -0.04, -0.03, 0.02, -0.01, 0.04],
        "l2fb": [0.006, -0.008],
        "l3w": [0.6, -0.4, 0.5, 0.2],
        "l3b": [0.05, -0.02],
        "l3fw": [0.03, -0.02],
        "l3fb": [0.004],
    },
    "train_source": "crates/cuda_cpp/src/lib.rs:13929-13955 (sfnn_tiny_train_step_runner_smoke)",
    "batch": 4, "max_active": 3,
    "stm": [0, 1, -1, 2, -1, -1, 1, 3, -1, 3, 2, -1],
    "nstm": [2, -1, -1, 0, 3, -1, 0, -1, -1, 1, -1, -1],
    "buckets": [0, 1, 0, 1],
    "targets": [0.25, 0.75, 0.6, 0.1],
    "entry_weights": [1.0, 0.5, 0.75, 1.25],
    "ranger": {"step": 1, "learning_rate": 0.01, "beta1": 0.9, "beta2": 0.999, "min_weight": -1.98,
               "max_weight": 1.98, "lookahead_alpha": 0.5, "lookahead_period": 6},
    "tolerance": 1e-6,
}

GOLDENS = {
    "tiny_nnue": TINY_NNUE,
    "tiny_nnue_trace": {
        "source": "crates/bulletou_lib/src/value/fast_nnue.rs:366-390 (scalar_trace_exposes_intermediate_activations)",
        "batch": 1, "max_active": 3, "stm": [0, 1, -1], "nstm": [2, -1, -1],
        "stm_l0": [0.7, 0.4], "nstm_l0": [0.0, 0.7], "combined": [0.7, 0.4, 0.0, 0.7],
        "hidden1": [0.86, 0.15], "hidden2": [0.772], "outputs": [1.208], "tolerance": 1e-6,
    },
    "tiny_nnue_two_samples": {
        "source": "crates/cuda_cpp/src/lib.rs:13242-13256 (nnue_tiny_forward_gpu_smoke); smoke.rs:60-73",
        "batch": 2, "max_active": 3, "stm": [0, 1, -1, 3, -1, -1], "nstm": [2, -1, -1, 1, 2, -1],
        "outputs": [1.208, 1.1195], "tolerance": 1e-5,
    },
    "sigmoid_mse_loss": {
        "source": "crates/bulletou_lib/src/value/fast_loss.rs:98-112; lib.rs:13332-13367",
        "outputs": [-2.0, 0.0, 2.0], "targets": [0.0, 0.5, 1.0], "weights": [1.0, 0.5, 2.0], "pow_exp": 2.0,
        "output_inv_scale": 1.0,
        "per_sample": [0.014209336, 0.0, 0.028418668],
        "mean_output_gradients": [0.008343695, 0.0, -0.01668739],
        "weighted_sum": 0.042628005, "mean": 0.014209335, "tolerance": 1e-6,
    },
    "zero_entry_weight": {
        "source": "crates/bulletou_lib/src/value/fast_loss.rs:114-125",
        "outputs": [10.0, -10.0], "targets": [0.0, 1.0], "weights": [0.0, 1.0],
        "per_sample0": 0.0, "per_sample1_min": 0.999,
    },
    "radam_step_scale": {
        "source": "crates/cuda_cpp/src/lib.rs:12965-12974 (radam_step_scale_matches_reference_points)",
        "step1": {"use_denom": False, "step_size": 10.0, "tolerance": 1e-5},
        "step6": {"finite_positive": True},
    },
    "smoke_backward_batch": {
        "source": "crates/cuda_cpp/src/bin/smoke.rs:123-170 (targets, entry weights of the tiny backward check)",
        "targets": [0.25, 0.75], "entry_weights": [1.0, 0.5], "pow_exp": 2.0, "output_inv_scale": 1.0,
        "tolerance": 1e-6,
    },
    "smoke_ranger": {
        "source": "crates/cuda_cpp/src/bin/smoke.rs:218-273",
        "gradients": [0.25, -0.5, 1.0, -1.5], "weights": [0.1, -0.2, 0.3, -0.4],
        "step": 1, "learning_rate": 0.01, "beta1": 0.9, "beta2": 0.999, "min_weight": -1.98, "max_weight": 1.98,
        "lookahead_alpha": 0.5, "lookahead_period": 6,
    },
    "zero_radam_skip": {
        "source": "crates/cuda_cpp/src/lib.rs:11112-11147 (zero_radam_update_skip_matches_reference)",
        "n": 128, "weights_formula": "0.1 + i*0.002", "weight_overrides": {"4": 2.0, "8": "-0.0", "12": "denorm_min"},
        "grad_overrides": {"16": "-0.0", "20": 0.1}, "momentum_overrides": {"24": 0.2},
        "velocity_overrides": {"28": 0.3}, "steps": [1, 6, 12], "min_weight": -1.0, "max_weight": 1.0,
    },
    "tiny_sfnn_fast": TINY_SFNN_FAST,
    "tiny_sfnn_runner": TINY_SFNN_RUNNER,
}

if __name__ == "__main__":
    out = Path(__file__).with_name("reference_goldens.json")
    out.write_text(json.dumps(GOLDENS, indent=1) + "\n")
    print(f"wrote {out}")
