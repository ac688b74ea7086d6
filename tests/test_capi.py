"""The C-ABI library without a GPU: it loads, exports every entry that
include/ditch_cuda.h declares, and reports the absence of a device as
Unsupported instead of failing in another way."""
import os
import re
import subprocess

import pytest

import ditch_b200
from ditch_b200 import cuda

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_entries():
    text = open(os.path.join(ROOT, "include", "ditch_cuda.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ditch_cuda_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_entry():
    names = declared_entries()
    assert len(names) >= 40
    out = subprocess.run(["nm", "-D", "--defined-only", cuda.LIB_PATH], capture_output=True, text=True, check=True)
    exported = set(re.findall(r"\bT (ditch_cuda_\w+)", out.stdout))
    missing = [n for n in names if n not in exported]
    assert not missing, f"declared but not exported: {missing}"
    lib = ditch_b200.lib()
    for n in names:
        assert hasattr(lib, n)
    # the ctypes table covers the whole header
    assert set(names) == set(cuda.SIGNATURES)


def test_version_and_error_text():
    lib = ditch_b200.lib()
    assert b"sm_100a" in lib.ditch_cuda_version()
    assert isinstance(lib.ditch_cuda_last_error(), bytes)


def test_no_device_is_unsupported():
    if ditch_b200.lib().ditch_cuda_device_count() > 0:
        pytest.skip("a GPU is present")
    with pytest.raises(ditch_b200.Unsupported):
        ditch_b200.Device(0)


def test_null_arguments_are_invalid():
    lib = ditch_b200.lib()
    assert lib.ditch_cuda_open(0, 0, None) == cuda.INVALID
    assert lib.ditch_cuda_forward(None, None, None, None, 0, None, 0, None, None, 0, None) == cuda.INVALID
