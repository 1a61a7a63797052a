"""CPU: the C-ABI library loads and exports every entry point that
include/*.h declares; ctypes struct layouts match the C compiler's."""

from __future__ import annotations

import ctypes
import glob
import os
import re
import shutil
import subprocess

import pytest

from imba_chess_b200 import _native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols() -> set[str]:
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        names |= set(re.findall(r"IMBA_API\s+[\w\s\*]+?\b(imba_\w+)\s*\(", text))
    return names


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(_native.LIB_PATH):
        from imba_chess_b200.build import build

        build()
    return _native.load()


def test_header_declares_the_bound_symbols():
    declared = _declared_symbols()
    assert declared, "no IMBA_API declarations found"
    assert declared == set(_native.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol(lib):
    for name in _declared_symbols():
        assert hasattr(lib, name), name
    assert lib.imba_version() >= 1
    assert lib.imba_device_arch() == 1000


def test_struct_layouts_match_c(tmp_path):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("no host C++ compiler")
    src = tmp_path / "sizes.cc"
    src.write_text(
        '#include <cstdio>\n#include <cstddef>\n#include "imba_b200.h"\n'
        "int main(){printf(\"%zu %zu %zu %zu %zu\\n\", sizeof(imba_model_desc), sizeof(imba_step_desc),"
        " sizeof(imba_pool_desc), offsetof(imba_model_desc, policy_w32), offsetof(imba_step_desc, status));}\n"
    )
    exe = tmp_path / "sizes"
    subprocess.run([gxx, "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    got = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    assert got == [
        ctypes.sizeof(_native.ModelDesc),
        ctypes.sizeof(_native.StepDesc),
        ctypes.sizeof(_native.PoolDesc),
        _native.ModelDesc.policy_w32.offset,
        _native.StepDesc.status.offset,
    ]


def test_null_arguments_are_rejected_without_a_device(lib):
    desc = _native.ModelDesc()
    handle = ctypes.c_void_p()
    assert lib.imba_model_create(ctypes.byref(desc), ctypes.byref(handle)) != _native.IMBA_OK
    assert lib.imba_model_create(None, ctypes.byref(handle)) == _native.IMBA_ERR_ARG
    assert lib.imba_step(None, None, None, None, 0, None) == _native.IMBA_ERR_ARG
