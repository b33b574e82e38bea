"""CPU: the product library loads (no GPU needed to dlopen) and exports every
entry declared in include/*.h; the ctypes table matches the headers."""
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
        for m in re.finditer(r"\bint\s+(bulletou_\w+)\s*\(([^;]*?)\)\s*;", text, flags=re.S):
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
