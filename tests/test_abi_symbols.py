"""CPU: the product library loads (no GPU needed to dlopen) and exports every
entry declared in include/*.h; the ctypes table matches the headers; every
C-ABI function the reference's Rust host declares (tests/golden/
reference_ffi_symbols.json, from crates/cuda_cpp/src) is exported with the
same parameter count, so the crate links against this library unchanged."""
import ctypes
import json
import re
import subprocess

import pytest

from tests.conftest import ROOT

HEADERS = sorted((ROOT / "include").glob("*.h"))


def declared_functions():
    names = {}
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        text = re.sub(r"//[^\n]*", "", text)
        for m in re.finditer(r"\b(?:int|void)\s+(bulletou_\w+)\s*\(([^;]*?)\)\s*;", text, flags=re.S):
            params = [p for p in m.group(2).split(",") if p.strip()]
            names[m.group(1)] = len(params)
    return names


def test_headers_declare_entries():
    names = declared_functions()
    assert "bulletou_cuda_cpp_nnue_forward_device" in names
    assert "bulletou_b200_nnue_train_step_device" in names
    assert len(names) >= 60


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", lib.path], capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    missing = sorted(n for n in declared_functions() if n not in exported)
    assert not missing, f"declared but not exported: {missing}"


def test_ctypes_table_matches_header_arity(lib):
    from bulletou_b200 import _lib

    decl = declared_functions()
    for name, n in decl.items():
        assert name in _lib.SIGNATURES, f"{name} missing from the ctypes table"
        assert len(_lib.SIGNATURES[name]) == n, f"{name}: header has {n} params, table {len(_lib.SIGNATURES[name])}"
        lib.fn(name)  # resolves


def test_last_error_without_gpu_reports_message(lib):
    import ctypes

    # a validation failure needs no device: null context
    rc = lib.fn("bulletou_cuda_cpp_context_synchronize")(None)
    assert rc == -1
    assert "context must not be null" in lib.last_error()
    buf = ctypes.create_string_buffer(4)
    assert lib.fn("bulletou_cuda_cpp_last_error")(buf, 4) == 0
    assert buf.value == b"con"
    assert lib.fn("bulletou_cuda_cpp_last_error")(None, 0) == -1


def test_destroy_null_handles_is_noop(lib):
    for name in ("context_destroy", "f32_buffer_destroy", "i32_buffer_destroy", "event_destroy", "graph_destroy",
                 "pinned_f32_buffer_destroy", "pinned_i32_buffer_destroy"):
        assert lib.fn(f"bulletou_cuda_cpp_{name}")(None) == 0


@pytest.mark.parametrize("path", ["bulletou_b200/csrc/nnue.cu", "bulletou_b200/csrc/sparse_rows.cu"])
def test_kernel_sources_target_sm100a_build(path):
    mk = (ROOT / "bulletou_b200/csrc/Makefile").read_text()
    assert "compute_100a" in mk and "sm_100a" in mk
    assert (ROOT / path).exists()


REFERENCE_FFI = json.loads((ROOT / "tests" / "golden" / "reference_ffi_symbols.json").read_text())

# Entries of the reference ABI this backend does not implement: each returns -1
# with "unsupported on this backend" whatever its arguments.
UNSUPPORTED = (
    "bulletou_bn_bind", "bulletou_bn_forward", "bulletou_bn_backward", "bulletou_bn_qat_project_l2",
    "bulletou_bn_qat_unfold_training", "bulletou_bn_qat_ft", "bulletou_bn_qat_ft_training",
    "bulletou_bn_qat_pullback", "bulletou_center_l1_groups", "bulletou_center_affine_layout",
    "bulletou_center_mean_reference", "bulletou_experiment_center_affine", "bulletou_experiment_column_mean",
    "bulletou_experiment_bucket_mean", "bulletou_experiment_bucket_centers",
    "bulletou_experiment_center_affine_bucket", "bulletou_experiment_mean_penalty_test",
    "bulletou_bind_ft_saturation_guard", "bulletou_ft_saturation_guard", "bulletou_clip_effective_l1",
    "bulletou_clip_effective_l1_axis", "bulletou_factor_axis_update_device", "bulletou_cuda_cpp_rebase_shared_device",
    "bulletou_cuda_cpp_sfnn_add_saturation_penalty_gradients_device", "bulletou_test_dense_l1_16",
    "bulletou_test_factorized_ft_half_fold", "bulletou_test_sfnn_ft_sort", "bulletou_test_sfnn_ft_gather",
    "bulletou_test_sfnn_half_grad_gather", "bulletou_test_sfnn_half_grad", "bulletou_test_l1_bucket_fold",
    "bulletou_test_qat_ft_lattice", "bulletou_test_qat_packed_l1", "bulletou_test_dense_qat_exact_ft",
    "bulletou_test_l1_to_ft_f32_gradient", "bulletou_test_l1_to_ft_half_gradient", "bulletou_test_l1_gather2",
    "bulletou_test_l1_gather2_king_progress", "bulletou_dense_qat_integer_reference",
    "bulletou_dense_qat_activation_reference", "bulletou_dense_qat_l1_backward_reference",
)


def test_reference_ffi_fixture_covers_the_crate():
    assert len(REFERENCE_FFI) >= 110
    for name in ("bulletou_cuda_cpp_ranger_update_stacked_dirty_device", "bulletou_cuda_cpp_sfnn_backward_device",
                 "bulletou_cuda_cpp_sfnn_backward_train_profile_device", "bulletou_bn_bind", "bulletou_layer_qat"):
        assert name in REFERENCE_FFI


def test_every_reference_ffi_symbol_exported_with_its_arity(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", lib.path], capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    decl = declared_functions()
    from bulletou_b200 import _lib

    missing = sorted(n for n in REFERENCE_FFI if n not in exported)
    assert not missing, f"reference FFI symbols not exported: {missing}"
    for name, info in REFERENCE_FFI.items():
        assert decl.get(name) == info["arity"], f"{name}: header {decl.get(name)} params, lib.rs {info['arity']}"
        assert len(_lib.SIGNATURES[name]) == info["arity"], name
        assert (name in _lib.VOID_RETURN) == (info["returns"] == "void"), name


def test_unsupported_entries_fail_with_a_message(lib):
    from bulletou_b200 import _lib

    for name in UNSUPPORTED:
        sig = _lib.SIGNATURES[name]
        args = [0.0 if t is ctypes.c_float else 0 for t in sig]
        rc = lib.fn(name)(*args)
        assert rc == -1, name
        assert "unsupported on this backend" in lib.last_error(), name


def test_fp16_switches_and_half_moments_without_a_gpu(lib):
    fn = lib.fn
    assert fn("bulletou_cuda_cpp_context_set_sfnn_ft_fp16")(None, 0) == -1
    assert "context must not be null" in lib.last_error()
    out = ctypes.c_void_p(1)
    assert fn("bulletou_cuda_cpp_ft_half_moments_create")(None, None, None, 4, 0, ctypes.byref(out)) == -1
    assert out.value is None
    assert fn("bulletou_cuda_cpp_ft_half_moments_destroy")(None) == 0
    n = ctypes.c_ulonglong(7)
    assert fn("bulletou_cuda_cpp_context_take_ft_half_grad_clipped")(None, ctypes.byref(n)) == -1
    fn("bulletou_bn_reference_mode")(1)  # no BatchNorm: accepted and ignored
