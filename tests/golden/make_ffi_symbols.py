"""Writes tests/golden/reference_ffi_symbols.json: every C-ABI function the
reference's Rust host declares (name, parameter count, declaring file:line).

Run in a checkout that has the reference tree (default: the path in
BULLETOU_REFERENCE_ROOT):

    BULLETOU_REFERENCE_ROOT=<reference checkout> python tests/golden/make_ffi_symbols.py

Sources scanned: every `extern "C" { ... }` block of crates/cuda_cpp/src --
lib.rs `mod ffi` (lib.rs:9647) and the test-module blocks below it,
batch_norm.rs, bn_qat.rs, layer_qat.rs, ka2_backward_tests.rs and
tests/dense_qat_reference.rs.  A library that exports all of them with these
arities links in place of the reference's static library for both the normal
and the test build of the crate.  Test infrastructure only.
"""
import json
import os
import re
import sys
from pathlib import Path

OUT = Path(__file__).resolve().parent / "reference_ffi_symbols.json"


def extern_blocks(text):
    for m in re.finditer(r'extern "C"\s*\{', text):
        i, depth = m.end(), 1
        while depth:
            depth += (text[i] == "{") - (text[i] == "}")
            i += 1
        yield text[:m.start()].count("\n") + 1, text[m.end():i - 1]


def main():
    root = os.environ.get("BULLETOU_REFERENCE_ROOT")
    if not root:
        sys.exit("set BULLETOU_REFERENCE_ROOT to the reference checkout")
    src = Path(root) / "crates" / "cuda_cpp" / "src"
    symbols = {}
    for rel in sorted(str(p.relative_to(src)) for p in src.rglob("*.rs")):
        text = (src / rel).read_text()
        for line, block in extern_blocks(text):
            block = re.sub(r"//[^\n]*", "", block)
            for m in re.finditer(r"fn\s+(\w+)\s*\((.*?)\)\s*(->\s*[^;]+)?;", block, flags=re.S):
                name = m.group(1)
                if not name.startswith("bulletou_"):
                    continue
                arity = len([a for a in m.group(2).split(",") if a.strip()])
                ret = (m.group(3) or "").replace("->", "").strip() or "void"
                symbols.setdefault(name, {"arity": arity, "returns": ret,
                                          "declared": f"crates/cuda_cpp/src/{rel}:{line}"})
    OUT.write_text(json.dumps(dict(sorted(symbols.items())), indent=1) + "\n")
    print(f"{len(symbols)} symbols -> {OUT}")


if __name__ == "__main__":
    main()
