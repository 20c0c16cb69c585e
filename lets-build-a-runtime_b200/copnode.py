"""The ``OpNode`` / ``COpNode`` struct and pointer binding of programs.

Byte-identical to ``OpNode`` in the reference (csrc/runtime.h:60-69) and
its ctypes mirror ``COpNode`` (runtime/executor/common.py:125-141):
``{int op; int n_inputs; void* inputs[12]; void* output; int out_shape[24];
int n_dims; int elem_size; int extra[24]}``.  The CUDA library's
``execute`` takes the same array; only the pointers are device addresses.
"""

from __future__ import annotations

import ctypes

import numpy as np

from .program import MAX_DIMS, MAX_INPUTS, Program, Ref


class COpNode(ctypes.Structure):
    _fields_ = [
        ("op", ctypes.c_int),
        ("n_inputs", ctypes.c_int),
        ("inputs", ctypes.c_void_p * MAX_INPUTS),
        ("output", ctypes.c_void_p),
        ("out_shape", ctypes.c_int * MAX_DIMS),
        ("n_dims", ctypes.c_int),
        ("elem_size", ctypes.c_int),
        ("extra", ctypes.c_int * MAX_DIMS),
    ]


assert ctypes.sizeof(COpNode) == 8 + 8 * MAX_INPUTS + 8 + 4 * MAX_DIMS + 8 + 4 * MAX_DIMS


def build_node_array(program: Program, resolve) -> "ctypes.Array[COpNode]":
    """Fill a COpNode array; ``resolve(ref) -> int address``."""
    arr = (COpNode * len(program.nodes))()
    for i, n in enumerate(program.nodes):
        c = arr[i]
        c.op = n.op
        c.n_inputs = len(n.inputs)
        if len(n.inputs) > MAX_INPUTS or len(n.out_shape) > MAX_DIMS or len(n.extra) > MAX_DIMS:
            raise ValueError(f"node {i} exceeds OpNode capacity")
        for j, r in enumerate(n.inputs):
            c.inputs[j] = resolve(r)
        c.output = resolve(n.output)
        c.n_dims = len(n.out_shape)
        for d, v in enumerate(n.out_shape):
            c.out_shape[d] = v
        c.elem_size = n.elem_size
        for k, v in enumerate(n.extra):
            c.extra[k] = v
    return arr


class HostBinding:
    """A program bound to host memory: the reference executor's view.

    Holds the arena (``np.uint8``), the constants and the input arrays,
    and the node array whose pointers address them -- what
    ``CompiledExecutor.compile`` + ``run`` hand to ``execute``.
    """

    def __init__(self, program: Program, constants: dict[str, np.ndarray],
                 inputs: dict[str, np.ndarray]):
        self.program = program
        self.arena = np.zeros(max(program.arena_size, 16), dtype=np.uint8)
        self.constants = {k: np.ascontiguousarray(v) for k, v in constants.items()}
        self.inputs = {k: np.ascontiguousarray(v) for k, v in inputs.items()}
        base = self.arena.ctypes.data

        def resolve(r: Ref) -> int:
            if r.kind == "arena":
                return base + r.offset
            if r.kind == "const":
                return self.constants[r.name].ctypes.data + r.offset
            if r.kind == "input":
                return self.inputs[r.name].ctypes.data + r.offset
            raise ValueError(r.kind)

        self.nodes = build_node_array(program, resolve)

    def output(self, name: str) -> np.ndarray:
        spec = self.program.outputs[name]
        r = spec["ref"]
        dt = np.dtype(spec["dtype"])
        count = int(np.prod(spec["shape"]))
        if r.kind == "arena":
            raw = self.arena[r.offset:r.offset + count * dt.itemsize]
        elif r.kind == "input":
            raw = self.inputs[r.name].view(np.uint8).reshape(-1)[r.offset:r.offset + count * dt.itemsize]
        else:
            raw = self.constants[r.name].view(np.uint8).reshape(-1)[r.offset:r.offset + count * dt.itemsize]
        return raw.view(dt).reshape(spec["shape"]).copy()

    def outputs(self) -> dict[str, np.ndarray]:
        return {k: self.output(k) for k in self.program.outputs}
