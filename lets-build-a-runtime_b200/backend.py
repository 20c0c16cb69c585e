"""Interpreted-executor backend on the B200.

The reference's interpreted executor walks the plan node by node and asks a
chain of backends for a kernel per op (``Backend.get_kernel``,
runtime/executor/interpreted.py:21-32, 118-124); a kernel receives the
node's input arrays, its pre-allocated output array and its attrs and
writes the result in place.  :class:`CudaBackend` serves those calls with
this library's GPU kernels, one op at a time -- the debugging / per-op
profiling path, not the fast one (that is ``CudaCompiledExecutor``):

* each call builds a one-node ``OpNode`` (``extra[]`` from
  :func:`extras.pack_extras`), copies the inputs into device buffers, runs
  it with ``rt_execute(..., RT_FLAG_EAGER)`` and copies the output back;
* device buffers are kept per input slot and grow only, so repeated calls
  with the same shapes reuse the same node array -- and the library's
  cached plan for it (no per-call planning);
* ops without a kernel in the library (PERMUTE, fold-only ops) return None
  from ``get_kernel`` so the chain falls through to the next backend, as the
  reference's C backend does.

Use it with the reference's executor::

    from runtime.executor.interpreted import InterpretedExecutor
    from lbr_b200.backend import CudaBackend
    from runtime.backends.numpy_backend import NumpyBackend
    ex = InterpretedExecutor(backends=[CudaBackend(), NumpyBackend()])
"""

from __future__ import annotations

import ctypes
from typing import Any, Callable

import numpy as np

from .copnode import COpNode
from .executor import RT_FLAG_EAGER, check, load_library
from .extras import pack_extras
from .program import OP, OP_NAME

KernelFn = Callable[[list, np.ndarray, dict], None]

# op codes with a kernel in the library (the reference C dispatch table,
# csrc/executor.c:409-452, less PERMUTE which has no entry there either)
SUPPORTED = frozenset(v for k, v in OP.items() if k != "PERMUTE")


class CudaBackend:
    """``Backend`` protocol (``name``, ``get_kernel``) over the GPU kernels."""

    name = "cuda"

    def __init__(self, device: int = 0, lib_path=None) -> None:
        self._lib = load_library(lib_path)
        check(self._lib, self._lib.rt_init(device), "rt_init")
        self._slots: list[tuple[int, int]] = []     # (device pointer, bytes), per buffer position
        self._node = (COpNode * 1)()
        self.calls = 0

    def get_kernel(self, op) -> KernelFn | None:
        code = int(getattr(op, "value", op))
        if code not in SUPPORTED:
            return None

        def kernel(inputs: list, output: np.ndarray, attrs: dict[str, Any]) -> None:
            self._run(code, inputs, output, attrs or {})

        kernel.__name__ = f"cuda_{OP_NAME[code].lower()}"
        return kernel

    # ------------------------------------------------------------------
    def _slot(self, k: int, nbytes: int) -> int:
        lib = self._lib
        while len(self._slots) <= k:
            self._slots.append((0, 0))
        ptr, cap = self._slots[k]
        if cap < nbytes:
            if ptr:
                lib.rt_free(ptr)
            cap = max(nbytes, 256)
            ptr = lib.rt_alloc(cap)
            if not ptr:
                check(lib, lib.rt_last_error() or 9, f"rt_alloc({cap})")
            self._slots[k] = (ptr, cap)
        return ptr

    def _run(self, code: int, inputs: list, output: np.ndarray, attrs: dict) -> None:
        lib = self._lib
        arrs = [np.ascontiguousarray(a) for a in inputs]
        n_graph = len(arrs)
        if code == OP["ATTENTION"] and arrs and arrs[-1].dtype == np.uint8 and arrs[-1].ndim == 1:
            n_graph -= 1          # the planner's scratch (a slice of the byte arena): not read here
        attrs = dict(attrs, _n_graph_inputs=n_graph)
        if code in (OP["MAX"], OP["SUM"]) and attrs.get("axis", -1) < 0:
            # the reference's dispatch indexes out_shape with the axis as given
            # (csrc/executor.c:172-188), so the graph layer only emits axes >= 0;
            # a kernel called directly may pass -1: count it from the input's rank
            attrs["axis"] = attrs.get("axis", -1) + arrs[0].ndim
        extra = pack_extras(code, [a.shape for a in arrs[:n_graph]], output.shape, attrs)
        if len(arrs) > 12 or output.ndim > 24 or len(extra) > 24:
            raise ValueError(f"{OP_NAME[code]}: node does not fit an OpNode")
        nd = self._node[0]
        ctypes.memset(ctypes.addressof(nd), 0, ctypes.sizeof(COpNode))
        nd.op = code
        nd.n_inputs = len(arrs)
        for k, a in enumerate(arrs):
            ptr = self._slot(k, a.nbytes)
            nd.inputs[k] = ptr
            if k < n_graph and a.nbytes:
                check(lib, lib.rt_upload(ptr, a.ctypes.data, a.nbytes), "upload")
        out_ptr = self._slot(12, output.nbytes)    # output slot past the 12 input positions
        nd.output = out_ptr
        for d, v in enumerate(output.shape):
            nd.out_shape[d] = int(v)
        nd.n_dims = output.ndim
        nd.elem_size = output.dtype.itemsize
        for i, v in enumerate(extra):
            nd.extra[i] = int(v)
        check(lib, lib.rt_execute(self._node, 1, RT_FLAG_EAGER), OP_NAME[code])
        if output.flags["C_CONTIGUOUS"]:
            check(lib, lib.rt_download(output.ctypes.data, out_ptr, output.nbytes), "download")
        else:
            tmp = np.empty(output.shape, output.dtype)
            check(lib, lib.rt_download(tmp.ctypes.data, out_ptr, tmp.nbytes), "download")
            output[...] = tmp
        self.calls += 1

    def close(self) -> None:
        for ptr, _ in self._slots:
            if ptr:
                self._lib.rt_free(ptr)
        self._slots = []
