"""The C-ABI library loads without a GPU and exports every function include/*.h declares."""
import glob
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^\s*[A-Za-z_][\w\s\*]*?\b(ltx_\w+)\s*\(", src, flags=re.M):
            names.add(m.group(1))
    return names


def test_header_declares_entry_points():
    names = declared_functions()
    assert {"ltx_ctx_create", "ltx_dequant_merge", "ltx_last_error"} <= names


def test_library_exports_every_declared_symbol():
    from ltx_b200 import LIB_PATH, lib
    if not os.path.exists(LIB_PATH):
        pytest.fail("libltx_b200.so is not built (run python ltx-rust_b200/build.py)")
    lib()  # loads without a GPU
    out = subprocess.run(["nm", "-D", "--defined-only", LIB_PATH], capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    missing = sorted(declared_functions() - exported)
    assert not missing, f"declared but not exported: {missing}"


def test_rust_binding_in_integration_doc_declares_every_entry_point():
    """The Rust `-sys` declarations of the integration guide bind every function of the header."""
    doc = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    rust = doc[doc.index("```rust"):]
    rust = rust[:rust.index("```", 7)]
    bound = set(re.findall(r"pub fn (ltx_\w+)\(", rust))
    missing = sorted(declared_functions() - bound)
    assert not missing, f"header functions without a Rust declaration: {missing}"


def test_lora_coeff_matches_reference_formula():
    import numpy as np
    from ltx_b200 import lora_coeff
    from oracle.weight_store import lib as olib
    for s, a, r in [(1.0, 64.0, 64), (0.75, 4.0, 2), (0.3, 7.0, 3), (1.7, 1.0, 13)]:
        assert np.float32(lora_coeff(s, a, r)) == np.float32(olib().oracle_lora_coeff(s, a, r))


def test_ctx_create_without_gpu_fails_cleanly():
    import ctypes
    import torch
    from ltx_b200 import lib
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = ctypes.c_void_p()
    assert lib().ltx_ctx_create(0, None, ctypes.byref(h)) != 0
    assert not h.value
