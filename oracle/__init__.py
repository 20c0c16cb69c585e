"""CPU oracle -- TEST INFRASTRUCTURE ONLY.

Two checkers for the CUDA executor, never part of the product path:

* ``restated``  -- ``_build/liboracle.so`` built from ``oracle_exec.c``, this
  project's plain-C restatement of the reference kernels;
* ``reference`` -- ``_ref/libexecutor.so``, the reference's own C executor
  (csrc/executor.c + csrc/ops/*.c) compiled from its sources by the
  ``Makefile`` here, linked to scipy's OpenBLAS.

Both take the reference ``OpNode`` array bound to host memory.  Only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
import this package.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
RESTATED_SO = HERE / "_build" / "liboracle.so"
REFERENCE_SO = HERE / "_ref" / "libexecutor.so"


def reference_root() -> Path:
    """The reference checkout: $REF_ROOT, else a `reference` directory beside
    this repository (it is absent on machines that only run the tests)."""
    env = os.environ.get("REF_ROOT")
    return Path(env) if env else HERE.parent.parent / "reference"


def build(reference_tree: str | None = None) -> None:
    """Compile the restatement, and the reference when its tree is present."""
    subprocess.run(["make", "-s", "-C", str(HERE), "restate"], check=True)
    ref = reference_tree or os.environ.get("REF_CSRC") or str(reference_root() / "csrc")
    if Path(ref).is_dir():
        subprocess.run(["make", "-s", "-C", str(HERE), "ref", f"REF_CSRC={ref}"], check=True)


_libs: dict[str, ctypes.CDLL] = {}


def load(kind: str = "restated") -> ctypes.CDLL:
    if kind in _libs:
        return _libs[kind]
    path = RESTATED_SO if kind == "restated" else REFERENCE_SO
    if not path.exists():
        raise FileNotFoundError(f"oracle library {path} not built")
    lib = ctypes.CDLL(str(path))
    if kind == "restated":
        lib.oracle_execute.argtypes = [ctypes.c_void_p, ctypes.c_int]
        lib.oracle_execute.restype = ctypes.c_int
    else:
        lib.execute.argtypes = [ctypes.c_void_p, ctypes.c_int]
        lib.execute.restype = None
        lib.oracle_ref_set_threads.argtypes = [ctypes.c_int]
        lib.oracle_ref_get_threads.restype = ctypes.c_int
    _libs[kind] = lib
    return lib


def available(kind: str) -> bool:
    return (RESTATED_SO if kind == "restated" else REFERENCE_SO).exists()


def execute(kind: str, binding) -> None:
    """Run a host-bound node array (``copnode.HostBinding``) on the oracle."""
    lib = load(kind)
    ptr = ctypes.addressof(binding.nodes)
    n = len(binding.program.nodes)
    if kind == "restated":
        rc = lib.oracle_execute(ptr, n)
        if rc:
            raise RuntimeError(f"oracle: unsupported node {rc - 1}")
    else:
        lib.execute(ptr, n)


def set_threads(n: int) -> None:
    if available("reference"):
        load("reference").oracle_ref_set_threads(int(n))


def run_program(kind: str, program, constants, inputs) -> dict:
    from lbr_b200.copnode import HostBinding   # host-binding helper only
    hb = HostBinding(program, constants, inputs)
    execute(kind, hb)
    return hb.outputs()
