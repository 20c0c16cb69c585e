"""Plan-time layout fusion, checked on the host (rt_fusion_report needs no GPU).

The node arrays are the committed programs bound to synthetic addresses
(arena, constants and inputs in disjoint ranges), exactly as the reference
CompiledExecutor would lay them out, so the pointer-overlap analysis sees the
planner's real buffer reuse.
"""

import ctypes

import pytest

from conftest import GOLDEN
from lbr_b200.copnode import build_node_array
from lbr_b200.executor import load_library
from lbr_b200.program import OP, Program

ARENA, INPUTS = 1 << 36, 3 << 36


def bind(prog):
    consts, nxt = {}, [1 << 40]

    def res(r):
        if r.kind == "arena":
            return ARENA + r.offset
        if r.kind == "input":
            return INPUTS + r.offset
        if r.name not in consts:
            consts[r.name] = nxt[0]
            nxt[0] += 1 << 32
        return consts[r.name] + r.offset

    return build_node_array(prog, res), res


def report(prog, arr):
    lib = load_library()
    lib.rt_unprotect_all()
    flags = (ctypes.c_int * len(prog.nodes))()
    n = lib.rt_fusion_report(arr, len(prog.nodes), flags)
    return n, list(flags)


def test_gpt2_head_split_and_merge_copies_fold_into_attention():
    prog = Program.load(GOLDEN / "gpt2_b8.json")
    arr, _ = bind(prog)
    n, flags = report(prog, arr)
    assert n == 14   # per layer: 3 slices + 3 head splits + the head merge
    folded_ops = {prog.nodes[i].op for i, f in enumerate(flags) if f == 1}
    assert folded_ops == {OP["SLICE"], OP["TRANSPOSE"]}
    assert [prog.nodes[i].op for i, f in enumerate(flags) if f == 2] == [OP["ATTENTION"]] * 2


def test_protected_output_blocks_folding():
    """A folded producer must not be the last writer of a graph output.

    The program cut right after the first attention leaves the head-split
    copies' buffers unrecycled; registering one as a graph output (rt_protect)
    keeps its chain."""
    import copy
    prog = copy.copy(Program.load(GOLDEN / "gpt2_mini_s300.json"))
    a = next(i for i, n in enumerate(prog.nodes) if n.op == OP["ATTENTION"])
    prog.nodes = prog.nodes[:a + 1]
    arr, res = bind(prog)
    lib = load_library()
    lib.rt_unprotect_all()
    flags = (ctypes.c_int * len(prog.nodes))()
    assert lib.rt_fusion_report(arr, len(prog.nodes), flags) == 6
    first_t = next(i for i, f in enumerate(flags) if f == 1 and prog.nodes[i].op == OP["TRANSPOSE"])
    out = prog.nodes[first_t].output
    nbytes = 4
    for d in prog.nodes[first_t].out_shape:
        nbytes *= d
    try:
        assert lib.rt_protect(res(out), nbytes) == 0
        assert lib.rt_fusion_report(arr, len(prog.nodes), flags) < 6
        assert flags[first_t] == 0
    finally:
        lib.rt_unprotect_all()


@pytest.mark.parametrize("name", ["qwen3_b8", "7b_b8", "toy"])
def test_no_folding_where_the_chain_does_not_match(name):
    prog = Program.load(GOLDEN / f"{name}.json")
    arr, _ = bind(prog)
    n, _ = report(prog, arr)
    assert n == 0
