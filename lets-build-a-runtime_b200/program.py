"""Planned-graph programs: the serialisable form of a compiled node array.

The reference's compiled executor turns a ``MemoryPlan`` into a ``COpNode``
array whose pointers address a host arena, host weight buffers and the
caller's input arrays (runtime/executor/compiled.py:34-70, :108-145).  A
:class:`Program` holds exactly that node array with every pointer replaced
by a symbolic reference:

* ``("arena", None, off)``  -- byte offset into the planned arena
  (runtime/planner.py:500-569 assigns these; aliases are already folded in),
* ``("const", name, off)``  -- byte offset into a graph constant (weights),
* ``("input", name, 0)``    -- a graph input, patched per call in the
  reference (compiled.py:77-82),

plus the arena size, the graph inputs/outputs and a recipe for every
constant.  Binding a program to memory (host arrays for the CPU oracle,
device allocations for the CUDA executor) yields the same ``COpNode`` array
the reference would build, field for field.

Constants are described, not stored, when they are large: ``fill`` (every
element equal: biases, norm gains), ``stored`` (kept verbatim in the
fixture's ``.npz``: rotary tables, small models) or ``randn`` (regenerated
from a seed keyed by the constant's name, with the mean/std recorded from
the exported model).
"""

from __future__ import annotations

import json
import zlib
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

# Op codes: values of enum OpType in the reference (csrc/runtime.h:11-55,
# runtime/ir.py:36-78).  They are part of the ABI and must not change.
OP = {
    "RELU": 100, "EXP": 101, "TANH": 102, "POW": 103, "GELU": 104,
    "RSQRT": 105, "SILU": 106, "NEG": 107, "COS": 108, "SIN": 109,
    "ADD": 200, "SUB": 201, "MUL": 202, "DIV": 203,
    "MAX": 300, "SUM": 301, "SOFTMAX": 302,
    "MATMUL": 400,
    "RESHAPE": 500, "TRANSPOSE": 501, "PERMUTE": 502, "SLICE": 503,
    "EMBEDDING": 504, "CAT": 505,
    "LAYERNORM": 600, "RMSNORM": 601,
    "MATMUL_ADD": 1000, "FUSED_BIAS_RELU": 1001, "ATTENTION": 1002,
    "GATED_ACT": 1003,
}
OP_NAME = {v: k for k, v in OP.items()}

MAX_INPUTS = 12   # csrc/runtime.h:57
MAX_DIMS = 24     # csrc/runtime.h:58


@dataclass
class Ref:
    kind: str            # "arena" | "const" | "input"
    name: str | None
    offset: int = 0

    def to_json(self):
        return [self.kind, self.name, int(self.offset)]

    @staticmethod
    def from_json(v):
        return Ref(v[0], v[1], int(v[2]))


@dataclass
class ProgNode:
    op: int
    inputs: list[Ref]
    output: Ref
    out_shape: list[int]
    elem_size: int
    extra: list[int]

    def to_json(self):
        return {"op": self.op, "inputs": [r.to_json() for r in self.inputs],
                "output": self.output.to_json(), "out_shape": self.out_shape,
                "elem_size": self.elem_size, "extra": self.extra}

    @staticmethod
    def from_json(d):
        return ProgNode(int(d["op"]), [Ref.from_json(r) for r in d["inputs"]],
                        Ref.from_json(d["output"]), list(d["out_shape"]),
                        int(d["elem_size"]), list(d["extra"]))


@dataclass
class ConstSpec:
    name: str
    shape: tuple
    dtype: str
    init: dict

    @property
    def nbytes(self) -> int:
        return int(np.prod(self.shape, dtype=np.int64)) * np.dtype(self.dtype).itemsize


@dataclass
class Program:
    name: str
    meta: dict
    arena_size: int
    inputs: dict           # name -> {"shape", "dtype"}
    outputs: dict          # name -> {"shape", "dtype", "ref"}
    constants: dict        # name -> ConstSpec
    nodes: list[ProgNode]
    stored: dict = field(default_factory=dict)  # name -> np.ndarray ("stored" constants)

    # ---------------------------------------------------------------- io
    def save(self, path: str | Path) -> None:
        path = Path(path)
        doc = {
            "name": self.name, "meta": self.meta, "arena_size": self.arena_size,
            "inputs": self.inputs,
            "outputs": {k: {**v, "ref": v["ref"].to_json()} for k, v in self.outputs.items()},
            "constants": {k: {"shape": list(c.shape), "dtype": c.dtype, "init": c.init}
                          for k, c in self.constants.items()},
            "nodes": [n.to_json() for n in self.nodes],
        }
        path.write_text(json.dumps(doc, separators=(",", ":")))
        if self.stored:
            np.savez_compressed(path.with_suffix(".npz"), **self.stored)

    @staticmethod
    def load(path: str | Path) -> "Program":
        path = Path(path)
        d = json.loads(path.read_text())
        outputs = {k: {**v, "ref": Ref.from_json(v["ref"])} for k, v in d["outputs"].items()}
        consts = {k: ConstSpec(k, tuple(v["shape"]), v["dtype"], v["init"])
                  for k, v in d["constants"].items()}
        stored = {}
        npz = path.with_suffix(".npz")
        if npz.exists():
            with np.load(npz) as z:
                stored = {k: z[k] for k in z.files}
        return Program(d["name"], d["meta"], int(d["arena_size"]), d["inputs"],
                       outputs, consts, [ProgNode.from_json(n) for n in d["nodes"]],
                       stored)

    # ------------------------------------------------------ materialising
    def make_constant(self, name: str, seed: int = 0) -> np.ndarray:
        c = self.constants[name]
        kind = c.init["kind"]
        if kind == "fill":
            return np.full(c.shape, c.init["value"], dtype=c.dtype)
        if kind == "stored":
            arr = self.stored[name]
            assert arr.shape == tuple(c.shape) and arr.dtype == np.dtype(c.dtype), name
            return np.ascontiguousarray(arr)
        if kind == "randn":
            rng = np.random.default_rng([seed, zlib.crc32(name.encode())])
            arr = rng.standard_normal(c.shape, dtype=np.float32)
            arr *= np.float32(c.init["std"])
            if c.init.get("mean", 0.0):
                arr += np.float32(c.init["mean"])
            return arr.astype(c.dtype, copy=False)
        raise ValueError(f"unknown constant init {kind!r} for {name}")

    def make_constants(self, seed: int = 0) -> dict[str, np.ndarray]:
        return {k: self.make_constant(k, seed) for k in self.constants}

    def make_inputs(self, seed: int = 0, batch_offset: int = 0) -> dict[str, np.ndarray]:
        """Seeded N(0,1) graph inputs.  ``batch_offset`` selects rows of a
        larger global batch, so that a batch split across ranks sees the
        same sequences as one unsplit run."""
        out = {}
        for name, spec in self.inputs.items():
            shape = tuple(spec["shape"])
            rows = []
            for b in range(shape[0]):
                rng = np.random.default_rng([seed, zlib.crc32(name.encode()), batch_offset + b])
                rows.append(rng.standard_normal(shape[1:], dtype=np.float32))
            out[name] = np.stack(rows).astype(spec["dtype"], copy=False)
        return out

    # --------------------------------------------------------- statistics
    def constant_bytes(self) -> int:
        return sum(c.nbytes for c in self.constants.values())

    def op_counts(self) -> dict[str, int]:
        counts: dict[str, int] = {}
        for n in self.nodes:
            counts[OP_NAME.get(n.op, str(n.op))] = counts.get(OP_NAME.get(n.op, str(n.op)), 0) + 1
        return counts


def golden_dir() -> Path:
    """Directory that holds the committed program fixtures."""
    return Path(__file__).resolve().parent.parent / "tests" / "golden"
