"""CPU tests of the C ABI: the library loads and exports what the header declares.

No compute calls here -- this container has no GPU.
"""
from __future__ import annotations

import ctypes
import os
import re

import pytest

from tests.conftest import ROOT

HEADER = os.path.join(ROOT, "include", "metallm_cuda.h")


def declared_functions() -> list[str]:
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(mlm_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_entry_points():
    names = declared_functions()
    for must in ("mlm_create", "mlm_q4k_dequant_f32", "mlm_q4k_gemv", "mlm_rmsnorm_f16",
                 "mlm_rope_f16", "mlm_attn_decode"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from metallm_b200 import _lib
    lib = _lib.load()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_header():
    from metallm_b200 import exported_symbols
    assert set(declared_functions()) <= set(exported_symbols())


def test_status_strings_and_abi_version():
    from metallm_b200 import _lib
    lib = _lib.load()
    assert lib.mlm_abi_version() == 1
    assert lib.mlm_status_string(0) == b"ok"
    assert lib.mlm_status_string(-2) == b"invalid shape"


def test_null_context_is_rejected_without_a_device():
    from metallm_b200 import _lib
    lib = _lib.load()
    # every op validates its context before touching CUDA
    assert lib.mlm_q4k_gemv(None, None, 0, 0, None, None, None) == -1
    assert lib.mlm_q4k_dequant_f32(None, None, None, 0) == -1
    assert lib.mlm_last_error(None) == b"null context"


def test_create_fails_cleanly_without_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from metallm_b200 import _lib
    lib = _lib.load()
    h = ctypes.c_void_p()
    st = lib.mlm_create(0, ctypes.byref(h))
    assert st in (-5, -1) and not h.value


@pytest.mark.parametrize("lang", ["c", "c++"])
def test_header_compiles_as_plain_c_and_cpp(tmp_path, lang):
    """The header the Swift module map (include/module.modulemap) imports is
    read by the C importer: it must compile as C11 alone, and as C++17."""
    import shutil
    import subprocess
    cc = shutil.which("gcc" if lang == "c" else "g++")
    if cc is None:
        pytest.skip("no host compiler")
    src = tmp_path / ("t.c" if lang == "c" else "t.cpp")
    src.write_text('#include "metallm_cuda.h"\nint main(void) { return MLM_OK; }\n')
    std = "-std=c11" if lang == "c" else "-std=c++17"
    r = subprocess.run([cc, std, "-Wall", "-Werror", "-pedantic", "-fsyntax-only",
                        "-I", os.path.join(ROOT, "include"), str(src)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    mm = open(os.path.join(ROOT, "include", "module.modulemap")).read()
    assert 'header "metallm_cuda.h"' in mm and 'link "metallm_cuda"' in mm
