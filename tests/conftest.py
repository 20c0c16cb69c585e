"""Shared fixtures: package loading, GPU gating, program helpers."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = ROOT / "tests" / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

from __graft_entry__ import load_package  # noqa: E402

load_package()

from lbr_b200.program import ConstSpec, ProgNode, Program, Ref  # noqa: E402


def gemm_scheme() -> str:
    """The GEMM operand scheme the library selects from the environment
    (read once per process, like the library does)."""
    import os
    if os.environ.get("RT_GEMM_3XTF32") == "1" or os.environ.get("RT_GEMM_SCHEME") == "3xtf32":
        return "3xtf32"
    return "cross" if os.environ.get("RT_GEMM_SCHEME") == "cross" else "f16"


# Split-plane hand-offs from an attention epilogue (RT_FUSE_ATTN_SPLIT) exist
# for the tf32 plane schemes only; under the fp16 scheme they are never planned.
PLANE_HANDOFFS = gemm_scheme() != "f16"


def gemm_handoff(env: str | None, K: int) -> bool:
    """Whether a GELU-epilogue GEMM hands its output to the next GEMM as that
    GEMM's split A operand (opt-in, RT_FUSE_HANDOFF=1): under the fp16 scheme
    when K % 128 == 0 (one scale per 128-wide segment), else when K % 4 == 0."""
    return env == "1" and K % (128 if gemm_scheme() == "f16" else 4) == 0


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")
    config.addinivalue_line("markers", "slow: full-size programs")


def has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def gpu_executor_factory():
    if not has_gpu():
        pytest.skip("no CUDA device")
    from lbr_b200.executor import CudaCompiledExecutor

    made = []

    def make(program, constants):
        ex = CudaCompiledExecutor(device=0)
        ex.compile_program(program, constants)
        made.append(ex)
        return ex

    yield make
    for ex in made:
        ex.close()


def mini_programs():
    return sorted(p.name.split(".")[0] for p in GOLDEN.glob("*.golden.npz"))


def load_golden(name):
    prog = Program.load(GOLDEN / f"{name}.json")
    z = np.load(GOLDEN / f"{name}.golden.npz")
    ins = {k[4:]: z[k] for k in z.files if k.startswith("in__")}
    outs = {k[5:]: z[k] for k in z.files if k.startswith("out__")}
    return prog, ins, outs


def single_node_program(op, in_arrays, out_shape, extra, elem_size=4, scratch_bytes=0,
                        out_dtype="float32", name="node"):
    """A one-node program: inputs are stored constants, output in the arena.

    ``in_arrays`` is a list of numpy arrays (one per node input, in order)."""
    consts = {}
    refs = []
    for k, a in enumerate(in_arrays):
        cname = f"in{k}"
        consts[cname] = ConstSpec(cname, tuple(a.shape), str(a.dtype), {"kind": "stored"})
        refs.append(Ref("const", cname, 0))
    out_bytes = int(np.prod(out_shape)) * elem_size
    off = 0
    if scratch_bytes:
        refs.append(Ref("arena", None, out_bytes + 256 - out_bytes % 256))
    arena = out_bytes + 256 - out_bytes % 256 + scratch_bytes
    node = ProgNode(op, refs, Ref("arena", None, off), list(out_shape), elem_size, list(extra))
    prog = Program(name, {}, arena, {}, {"y": {"shape": list(out_shape), "dtype": out_dtype,
                                                "ref": Ref("arena", None, 0)}},
                   consts, [node], {f"in{k}": a for k, a in enumerate(in_arrays)})
    return prog
