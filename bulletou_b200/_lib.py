"""ctypes binding of the C ABI (include/bulletou_cuda_cpp.h, include/bulletou_b200.h).

The same binding drives this package's sm_100a library (libbulletou_b200.so,
the product) and, for parity tests and the reference timing arm only, the
reference backend built from its own sources (exported with a ``refx_``
prefix).  There is no fallback: if the library is missing the import fails
loudly.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

P = ctypes.c_void_p
Z = ctypes.c_size_t
I = ctypes.c_int
F = ctypes.c_float
U64 = ctypes.c_uint64

PACKAGE_DIR = Path(__file__).resolve().parent
LIBRARY_PATH = PACKAGE_DIR / "libbulletou_b200.so"


class CudaCppError(RuntimeError):
    """Non-zero status from the C ABI; the message is the library's last error
    (mirrors CudaCppError in crates/cuda_cpp/src/lib.rs:19-37)."""

    def __init__(self, message: str, code: int = -1):
        super().__init__(message)
        self.code = code


class RangerStep(ctypes.Structure):
    """BulletOuB200RangerStep."""

    _fields_ = [
        ("norm_loss_rate", F), ("norm_loss_before", I), ("gradient_factor", F), ("learning_rate", F),
        ("step_size", F), ("use_denom", I), ("decay", F), ("beta1", F), ("beta2", F), ("epsilon", F),
        ("min_weight", F), ("max_weight", F), ("do_lookahead", I), ("lookahead_alpha", F),
        ("clip_after_lookahead", I),
    ]


class SfnnShape(ctypes.Structure):
    """BulletOuB200SfnnShape."""

    _fields_ = [("input_size", Z), ("ft_size", Z), ("l1_hidden", Z), ("l1_skip", I), ("l2_size", Z),
                ("num_stacks", Z), ("ft_factorizer_alpha", F), ("factorizer_shared_alpha", F)]


class QuantRounding(ctypes.Structure):
    """BulletOuB200QuantRounding."""

    _fields_ = [("ft_shift", I), ("ft_round", I), ("crelu_round", I), ("sqr_clipped_relu_round", I),
                ("final_div_round", I), ("fv_scale", I)]


class SfnnQat(ctypes.Structure):
    """BulletOuB200SfnnQat."""

    _fields_ = [("l1", I), ("ft", I), ("l2", I), ("l3", I)]


class ValidationConfig(ctypes.Structure):
    """BulletOuB200ValidationConfig."""

    _fields_ = [("have_results", I), ("score_drop_abs", I), ("loss_kind", I), ("lambda_", F), ("eval_scale", F),
                ("model_output_scale", F), ("pow_exp", F), ("nnue2score", F), ("in_offset", F), ("in_scaling", F)]


class TeacherConfig(ctypes.Structure):
    """BulletOuB200TeacherConfig."""

    _fields_ = [("feature_set", I), ("max_active", I), ("hand_bucket", I), ("king_bucket", I),
                ("result_blend", F), ("score_blend", F), ("rscale", F), ("score_drop_abs", I)]


class RowExchange(ctypes.Structure):
    """BulletOuB200RowExchange."""

    _fields_ = [("world", Z), ("rank", Z), ("recv", U64 * 8), ("table", U64 * 8), ("flags", U64 * 8),
                ("slot_rows", Z), ("epoch", I), ("small_recv", U64 * 8), ("small_len", Z), ("small_flag_base", Z)]


class LossSpec(ctypes.Structure):
    """BulletOuB200LossSpec."""

    _fields_ = [("kind", I), ("output_inv_scale", F), ("loss_pow_exp", F), ("loss_param", F),
                ("finalize_loss", I), ("normalizer", Z)]


_BUF = P  # handle pointers are opaque
# Entries returning void (no status code).
VOID_RETURN = {"bulletou_dense_qat_end", "bulletou_bn_reference_mode"}
SIGNATURES: dict[str, list] = {
    # runtime
    "bulletou_cuda_cpp_last_error": [P, Z],
    "bulletou_cuda_cpp_device_name": [I, P, Z],
    "bulletou_cuda_cpp_context_create": [I, P],
    "bulletou_cuda_cpp_context_destroy": [P],
    "bulletou_cuda_cpp_context_synchronize": [P],
    "bulletou_cuda_cpp_event_create": [P, P],
    "bulletou_cuda_cpp_event_destroy": [P],
    "bulletou_cuda_cpp_event_record": [P, P],
    "bulletou_cuda_cpp_event_wait": [P, P],
    "bulletou_cuda_cpp_event_synchronize": [P],
    "bulletou_cuda_cpp_event_elapsed_ms": [P, P, P],
    "bulletou_cuda_cpp_graph_begin_capture": [P],
    "bulletou_cuda_cpp_graph_end_capture": [P, P],
    "bulletou_cuda_cpp_graph_destroy": [P],
    "bulletou_cuda_cpp_graph_launch": [P, P],
    "bulletou_cuda_cpp_f32_buffer_create": [P, Z, P],
    "bulletou_cuda_cpp_f32_buffer_destroy": [P],
    "bulletou_cuda_cpp_i32_buffer_create": [P, Z, P],
    "bulletou_cuda_cpp_i32_buffer_destroy": [P],
    "bulletou_cuda_cpp_pinned_f32_buffer_create": [P, Z, P],
    "bulletou_cuda_cpp_pinned_f32_buffer_destroy": [P],
    "bulletou_cuda_cpp_pinned_i32_buffer_create": [P, Z, P],
    "bulletou_cuda_cpp_pinned_i32_buffer_destroy": [P],
    "bulletou_cuda_cpp_f32_upload_staged": [P, P, P, P, Z],
    "bulletou_cuda_cpp_i32_upload_staged": [P, P, P, P, Z],
    "bulletou_cuda_cpp_i32_upload": [P, P, P, Z],
    "bulletou_cuda_cpp_i32_download": [P, P, P, Z],
    "bulletou_cuda_cpp_i32_copy_device": [P, P, P, Z],
    "bulletou_cuda_cpp_f32_upload": [P, P, P, Z],
    "bulletou_cuda_cpp_f32_download": [P, P, P, Z],
    "bulletou_cuda_cpp_f32_copy_device": [P, P, P, Z],
    "bulletou_cuda_cpp_f32_fill": [P, P, F, Z],
    "bulletou_cuda_cpp_axpy_device": [P, Z, F, P, P, P],
    "bulletou_cuda_cpp_axpy_host": [I, Z, F, P, P, P],
    # optimizers
    "bulletou_cuda_cpp_ranger_update_device": [P, F, I, Z, F, F, F, I, F, F, F, F, F, F, I, F, I, P, P, P, P, P, P],
    "bulletou_cuda_cpp_ranger_update_host": [I, Z, F, F, F, I, F, F, F, F, F, F, I, F, I, P, P, P, P, P],
    "bulletou_cuda_cpp_sgd_momentum_update_device": [P, Z, F, F, F, F, F, F, P, P, P, P, P],
    # HalfKP
    "bulletou_cuda_cpp_nnue_forward_device": [P, Z, Z, Z, Z, Z, Z] + [P] * 16,
    "bulletou_cuda_cpp_nnue_forward_host": [I, Z, Z, Z, Z, Z, Z] + [P] * 11,
    "bulletou_cuda_cpp_nnue_backward_device": [P, Z, Z, Z, Z, Z, Z] + [P] * 24 + [I],
    "bulletou_cuda_cpp_nnue_train_warmup_device": [P, Z, Z, Z, Z, Z, Z] + [P] * 16,
    # loss
    "bulletou_cuda_cpp_scalar_loss_device_with_finalize": [P, I, F, F, F, Z] + [P] * 7 + [I],
    "bulletou_cuda_cpp_scalar_loss_device": [P, I, F, F, F, Z] + [P] * 7,
    "bulletou_cuda_cpp_scalar_loss_host": [I, I, F, F, F, Z] + [P] * 7,
    # KPPT
    "bulletou_cuda_cpp_kppt_forward_device": [P, Z, Z, Z] + [P] * 9,
    "bulletou_cuda_cpp_kppt_backward_device": [P, Z, Z, Z] + [P] * 10,
    # additive B200 entries
    "bulletou_b200_version": [P, Z],
    "bulletou_b200_context_create_on_stream": [I, P, P],
    "bulletou_b200_context_stream": [P, P],
    "bulletou_b200_f32_buffer_ptr": [P, P],
    "bulletou_b200_i32_buffer_ptr": [P, P],
    "bulletou_b200_i32_upload_pinned": [P, P, P, Z],
    "bulletou_b200_f32_upload_pinned": [P, P, P, Z],
    "bulletou_b200_f32_download_pinned": [P, P, P, Z],
    "bulletou_b200_pinned_f32_ptr": [P, P],
    "bulletou_b200_pinned_i32_ptr": [P, P],
    "bulletou_b200_f32_buffer_view": [P, Z, Z, P],
    "bulletou_b200_profile_begin": [P, Z],
    "bulletou_b200_profile_end": [P, P, Z, P, P],
    "bulletou_b200_l2_read_probe": [P, P, Z, I, P],
    "bulletou_b200_context_scratch_bytes": [P, P],
    "bulletou_b200_context_wait_before_weights": [P, P],
    "bulletou_b200_nnue_forward_device_noalloc": [P, Z, Z, Z, Z, Z, Z] + [P] * 16,
    "bulletou_b200_nnue_train_step_device": [P, Z, Z, Z, Z, Z, Z, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P],
    "bulletou_b200_nnue_dense_gradient_len": [Z, Z, Z, P],
    "bulletou_b200_nnue_local_gradients_device": [P, Z, Z, Z, Z, Z, Z, P, P, P, P, P, P, P, P, P, P, P, P, P],
    "bulletou_b200_kppt_train_step_device": [P, Z, Z, Z, P, P, P, P, P, P, P, P, P, P, P, P, P, P, P],
    # SFNN (cu:11329, cu:12882) and the fused SFNN step
    "bulletou_cuda_cpp_sfnn_forward_device": (
        [P, Z, Z, Z, I] + [Z] * 9 + [P] * 10 + [I] + [P] * 2 + [I] + [P] * 4 + [I] + [P] * 2 + [I] + [P] * 4 + [I]
        + [P] * 2 + [I] + [I] * 6 + [F] * 6 + [P] * 2 + [P] * 7 + [P] * 2 + [I]),
    "bulletou_cuda_cpp_sfnn_backward_train_device": (
        [P, Z, Z, Z, I] + [Z] * 9 + [P] * 12 + [I] + [P] + [I] + [P] * 2 + [I] + [P] + [I] + [P] * 2 + [I] + [P]
        + [I] + [I] * 6 + [F] * 6 + [P] * 2 + [P] + [P] * 8 + [P] * 20 + [I] + [P]),
    "bulletou_b200_sfnn_train_step_device": [P, P, Z, Z] + [P] * 17,
    "bulletou_b200_sfnn_dense_gradient_len": [P, I, I, I, P],
    "bulletou_b200_sfnn_local_gradients_device": [P, P, Z, Z] + [P] * 17 + [Z],
    "bulletou_b200_sfnn_local_gradients_exchange_device": [P, P, Z, Z] + [P] * 20 + [Z],
    "bulletou_b200_sfnn_shard_ranger_exchange_device": [P, P, Z, Z, Z, Z, Z, P, P, P, P, P, P, Z, Z, P],
    "bulletou_b200_exchange_wait_device": [P, P, Z, Z, I, P],
    "bulletou_b200_exchange_reduce_small_device": [P, P, P, P, P],
    "bulletou_b200_context_wait_flags_before_weights": [P, P, Z, Z, I, P],
    "bulletou_b200_f32_buffer_ipc_handle": [P, P],
    "bulletou_b200_i32_buffer_ipc_handle": [P, P],
    "bulletou_b200_ipc_open": [P, P, P],
    "bulletou_b200_ipc_close": [P, U64],
    "bulletou_b200_sfnn_row_launches": [P, P, P, Z],
    # SFNN QAT (reference entries)
    "bulletou_layer_qat": [P, P, P, F, F, F, Z, Z, Z, F],
    "bulletou_layer_qat_nonzero": [P, P, P, P],
    "bulletou_dense_qat_begin": [P, P, P, Z, Z, Z, Z, I],
    "bulletou_dense_qat_end": [P],
    "bulletou_b200_sfnn_quantize_device": [P, P, P, P],
    "bulletou_b200_nnue_quantize_device": [P, Z, Z, Z, Z, P, P, P],
    "bulletou_b200_nnue_integer_forward_device": [P, Z, Z, Z, Z, Z, Z, P, P, P, I, P, P, P],
    "bulletou_b200_sfnn_integer_forward_device": [P, P, Z, Z] + [P] * 9,
    "bulletou_b200_teacher_prepare_device": [P, P, P, Z] + [P] * 7,
    "bulletou_b200_hcpe_to_psv_device": [P, P, Z, P, P, P],
    "bulletou_b200_validation_metrics_device": [P, P, P, P, Z, P, P],
    "bulletou_cuda_cpp_sfnn_validation_stats": [P] * 7 + [Z] * 4,
    "bulletou_cuda_cpp_sfnn_unit_stats": [P] * 7 + [Z] * 5,
    # the rest of the reference ABI (lib.rs mod ffi, batch_norm.rs, bn_qat.rs): implemented or
    # "unsupported on this backend" (include/bulletou_cuda_cpp.h)
    "bulletou_bind_ft_saturation_guard": [P] * 4 + [Z, Z, F, F, I],
    "bulletou_bn_backward": [P] * 9 + [Z] * 4,
    "bulletou_bn_bind": [P, I] + [P] * 6 + [Z] * 4 + [F, F, I],
    "bulletou_bn_forward": [P] * 9 + [Z] * 4 + [F, F, I],
    "bulletou_bn_qat_ft": [P, P, P, Z, Z, Z, F],
    "bulletou_bn_qat_ft_training": [P] * 5 + [Z, Z, Z, F],
    "bulletou_bn_qat_project_l2": [P, P, P, Z, Z],
    "bulletou_bn_qat_pullback": [P] * 9 + [Z, Z, Z, I, Z, F],
    "bulletou_bn_qat_unfold_training": [P] * 7 + [Z, Z, Z, I, Z, F],
    "bulletou_bn_reference_mode": [I],
    "bulletou_center_affine_layout": [P] * 8 + [Z, Z, I, I],
    "bulletou_center_l1_groups": [P] * 14 + [Z, I],
    "bulletou_center_mean_reference": [P, P, P, Z, Z],
    "bulletou_center_scale": [P, P, P, Z, F],
    "bulletou_clip_effective_l1": [P] * 6 + [Z, Z, F],
    "bulletou_clip_effective_l1_axis": [P] * 8 + [Z] * 5 + [I] * 6 + [F] * 5,
    "bulletou_cuda_cpp_context_release_sfnn_ft_fp16_scratch": [P, I, I, I],
    "bulletou_cuda_cpp_context_set_sfnn_ft_fp16": [P, I],
    "bulletou_cuda_cpp_context_set_sfnn_ft_fp16_act": [P, I],
    "bulletou_cuda_cpp_context_set_sfnn_ft_fp16_grad": [P, I],
    "bulletou_cuda_cpp_context_take_ft_half_grad_clipped": [P, P],
    "bulletou_cuda_cpp_ft_half_moments_create": [P, P, P, Z, I, P],
    "bulletou_cuda_cpp_ft_half_moments_decode": [P] * 4,
    "bulletou_cuda_cpp_ft_half_moments_destroy": [P],
    "bulletou_cuda_cpp_ft_half_moments_take_clipped": [P, P, P],
    "bulletou_cuda_cpp_ranger_update_stacked_dirty_device": [P, F, I, Z, Z, Z, F, F, F, I] + [F] * 6 + [I, F, I] + [P] * 6,
    "bulletou_cuda_cpp_rebase_shared_device": [P] * 10 + [Z] * 5 + [F, F],
    "bulletou_cuda_cpp_scale_axis_rows_f32_device": [P, P, Z, P, Z, Z],
    "bulletou_cuda_cpp_sfnn_add_residual_count_decay_gradients_device": [P] * 5 + [Z, Z, Z],
    "bulletou_cuda_cpp_sfnn_add_saturation_penalty_gradients_device": [P, P, P, I, P, I] + [P] * 4 + [Z] * 6 + [I] * 6 + [F] * 6 + [P, P, I, F, F, F],
    "bulletou_cuda_cpp_sfnn_apply_residual_count_gates_to_gradients_device": [P] * 4 + [Z, Z, Z],
    "bulletou_cuda_cpp_sfnn_backward_device": [P, Z, Z, Z, I] + [Z] * 9 + [P] * 12 + [I, P, I, P, P, I, P, I, P, P, I, P] + [I] * 7 + [F] * 6 + [P] * 31,
    "bulletou_cuda_cpp_sfnn_backward_train_profile_device": [P, Z, Z, Z, I] + [Z] * 9 + [P] * 12 + [I, P, I, P, P, I, P, I, P, P, I, P] + [I] * 7 + [F] * 6 + [P] * 31 + [I, P, Z],
    "bulletou_cuda_cpp_sfnn_build_quantized_proxy_device": [P] + [Z] * 5 + [I] + [Z] * 7 + [P] * 6 + [I, P, P, I] + [P] * 4 + [I, P, P, I] + [P] * 4 + [I, P, P] + [I] * 7 + [F] * 6 + [P] * 10 + [I],
    "bulletou_dense_qat_activation_reference": [P] * 7 + [Z],
    "bulletou_dense_qat_integer_reference": [P] * 6 + [Z] * 4,
    "bulletou_dense_qat_l1_backward_reference": [P] * 5 + [Z, Z, I],
    "bulletou_experiment_bucket_centers": [P, P, P, Z, Z],
    "bulletou_experiment_bucket_mean": [P] * 4 + [Z, Z, Z],
    "bulletou_experiment_center_affine": [P] * 8 + [Z, Z, I],
    "bulletou_experiment_center_affine_bucket": [P] * 8 + [Z, Z, Z, I],
    "bulletou_experiment_column_mean": [P, P, P, Z, Z],
    "bulletou_experiment_mean_penalty_test": [P] * 5 + [Z] * 4 + [F],
    "bulletou_factor_axis_update_device": [P] + [Z] * 5 + [F] * 4 + [P] + [F] * 7 + [I, I, F, F, F, I, I, F, I] + [P] * 5,
    "bulletou_ft_saturation_guard": [P] * 10 + [Z] * 4 + [F, F, F, I],
    "bulletou_test_dense_l1_16": [P] * 6 + [Z, Z, Z, I],
    "bulletou_test_dense_qat_exact_ft": [P] * 7 + [Z] * 4,
    "bulletou_test_factorized_ft_half_fold": [P, P, P, Z, Z, F, I],
    "bulletou_test_l1_bucket_fold": [P] * 8 + [I],
    "bulletou_test_l1_gather2": [P] * 9 + [Z] * 4 + [F],
    "bulletou_test_l1_gather2_king_progress": [P] * 12 + [Z] * 5 + [F] * 4,
    "bulletou_test_l1_to_ft_f32_gradient": [P] * 7 + [Z, Z, Z, I],
    "bulletou_test_l1_to_ft_half_gradient": [P] * 7 + [Z, Z, Z, I],
    "bulletou_test_qat_ft_lattice": [P, P, Z, I],
    "bulletou_test_qat_packed_l1": [P] * 7 + [Z] * 4 + [I],
    "bulletou_test_sfnn_ft_fp16_scratch_sizes": [P] * 4,
    "bulletou_test_sfnn_ft_gather": [P] * 5 + [Z, Z, I, I],
    "bulletou_test_sfnn_ft_sort": [P] * 10 + [Z] * 4 + [I],
    "bulletou_test_sfnn_half_grad": [P] * 7 + [Z, Z, I],
    "bulletou_test_sfnn_half_grad_gather": [P] * 5 + [Z] * 4 + [I],
    "bulletou_test_stream_delay": [P],
}


class Library:
    """One loaded backend library.  ``kind`` is "b200" or "reference"."""

    def __init__(self, path: str | os.PathLike, kind: str = "b200"):
        self.path = str(path)
        self.kind = kind
        self.prefix = "refx_" if kind == "reference" else ""
        self._cdll = ctypes.CDLL(self.path, mode=os.RTLD_LOCAL)
        self._fns: dict[str, object] = {}

    def has(self, name: str) -> bool:
        try:
            getattr(self._cdll, self.prefix + name)
            return True
        except AttributeError:
            return False

    def fn(self, name: str):
        f = self._fns.get(name)
        if f is None:
            f = getattr(self._cdll, self.prefix + name)
            f.argtypes = SIGNATURES[name]
            f.restype = None if name in VOID_RETURN else I
            self._fns[name] = f
        return f

    def last_error(self) -> str:
        buf = ctypes.create_string_buffer(1024)
        self.fn("bulletou_cuda_cpp_last_error")(buf, len(buf))
        return buf.value.decode(errors="replace")

    def call(self, name: str, *args) -> None:
        rc = self.fn(name)(*args)
        if name in VOID_RETURN:
            return
        if rc != 0:
            raise CudaCppError(f"{name}: {self.last_error()}", rc)


_default: Library | None = None


def library() -> Library:
    """The product library (loaded once).  Raises if it has not been built."""
    global _default
    if _default is None:
        if not LIBRARY_PATH.exists():
            raise ImportError(
                f"{LIBRARY_PATH} is missing: build it with `make -C bulletou_b200/csrc` "
                "(or __graft_entry__.build()); there is no CPU fallback")
        _default = Library(LIBRARY_PATH, "b200")
    return _default


def reference_library(path: str | os.PathLike | None = None) -> Library:
    """The reference backend built by oracle/build_ref.sh (test/bench only)."""
    p = Path(path) if path else PACKAGE_DIR.parent / "oracle" / "_ref" / "libref_cudacpp.so"
    if not p.exists():
        raise FileNotFoundError(f"reference backend not built: {p} (run oracle/build_ref.sh)")
    return Library(p, "reference")


def exported_names() -> list[str]:
    return list(SIGNATURES)
