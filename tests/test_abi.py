"""The C-ABI library: it loads, exports what include/b200exec.h declares,
and reports errors without a GPU (no compute calls here)."""

import ctypes
import re
import subprocess

import pytest

from conftest import ROOT, has_gpu
from lbr_b200 import executor as ex_mod

HEADER = ROOT / "include" / "b200exec.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    text = re.sub(r"^#.*$", "", text, flags=re.M)
    return sorted(set(re.findall(r"\b(\w+)\s*\([^;{]*\)\s*;", text)) - {"if", "sizeof"})


def test_header_declares_execute():
    assert "execute" in declared_functions()


def test_library_exports_every_declared_symbol():
    lib_path = ex_mod.LIB_PATH
    if not lib_path.exists():
        from lbr_b200 import build
        build.build()
    out = subprocess.run(["nm", "-D", "--defined-only", str(lib_path)], capture_output=True,
                         text=True, check=True).stdout
    exported = set(l.split()[-1] for l in out.splitlines() if " T " in l)
    missing = [f for f in declared_functions() if f not in exported]
    assert not missing, missing
    lib = ex_mod.load_library()
    for f in declared_functions():
        assert hasattr(lib, f)


def test_calls_before_init_fail_cleanly():
    lib = ex_mod.load_library()
    if has_gpu():
        pytest.skip("checks the uninitialised path only where no device is used")
    lib.rt_clear_error()
    assert lib.rt_alloc(1024) is None
    assert lib.rt_last_error() == 1          # RT_ERR_NOT_INITIALIZED
    assert lib.rt_execute(None, 0, 0) == 1
    assert b"rt_init" in lib.rt_last_error_message()
    assert lib.rt_version().startswith(b"b200exec")


def test_init_without_device_reports_cuda_error():
    if has_gpu():
        pytest.skip("a device is present")
    lib = ex_mod.load_library()
    rc = lib.rt_init(0)
    assert rc == 8   # RT_ERR_CUDA
    assert lib.rt_last_error() == 8


def test_executor_refuses_to_run_without_library(tmp_path):
    with pytest.raises(RuntimeError, match="not found"):
        ex_mod.load_library(tmp_path / "missing.so")
