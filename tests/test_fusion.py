"""Plan-time layout fusion, checked on the host (rt_fusion_report needs no GPU).

The node arrays are the committed programs bound to synthetic addresses
(arena, constants and inputs in disjoint ranges), exactly as the reference
CompiledExecutor would lay them out, so the pointer-overlap analysis sees the
planner's real buffer reuse.
"""

import ctypes

import pytest

from conftest import GOLDEN, PLANE_HANDOFFS, gemm_handoff
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
    # per layer: 3 slices + 3 head splits + the head merge + the MLP's GELU
    assert n == 16
    folded = [prog.nodes[i].op for i, f in enumerate(flags) if f == 1]
    assert sorted(set(folded)) == sorted({OP["SLICE"], OP["TRANSPOSE"], OP["GELU"]})
    assert folded.count(OP["GELU"]) == 2
    assert [prog.nodes[i].op for i, f in enumerate(flags) if f == 2] == [OP["ATTENTION"]] * 2


def test_gemm_gelu_gemm_chain_hands_over_split_operand(monkeypatch):
    """MLP up-projection -> GELU -> down-projection: the GELU runs in the first
    GEMM's epilogue, which (RT_FUSE_HANDOFF=1) writes the second GEMM's split
    A operand."""
    monkeypatch.setenv("RT_FUSE_HANDOFF", "1")
    prog = Program.load(GOLDEN / "gpt2_b8.json")
    arr, _ = bind(prog)
    _, flags = report(prog, arr)
    gelus = [i for i, nd in enumerate(prog.nodes) if nd.op == OP["GELU"]]
    for u in gelus:
        assert flags[u] == 1
        assert flags[u - 1] == 3 and prog.nodes[u - 1].op == OP["MATMUL_ADD"]
        assert flags[u + 1] == (4 if gemm_handoff("1", 3072) else 0) and prog.nodes[u + 1].op == OP["MATMUL_ADD"]


def test_gelu_fold_hand_off_default(monkeypatch):
    """The hand-off is opt-in."""
    monkeypatch.delenv("RT_FUSE_HANDOFF", raising=False)
    prog = Program.load(GOLDEN / "gpt2_b8.json")
    arr, _ = bind(prog)
    _, flags = report(prog, arr)
    for u in [i for i, nd in enumerate(prog.nodes) if nd.op == OP["GELU"]]:
        assert flags[u - 1:u + 2] == [3, 1, 4 if gemm_handoff(None, 3072) else 0]


def test_gelu_fold_without_hand_off(monkeypatch):
    monkeypatch.setenv("RT_FUSE_HANDOFF", "0")
    prog = Program.load(GOLDEN / "gpt2_b8.json")
    arr, _ = bind(prog)
    _, flags = report(prog, arr)
    for u in [i for i, nd in enumerate(prog.nodes) if nd.op == OP["GELU"]]:
        assert flags[u - 1:u + 2] == [3, 1, 0]


def test_protected_gelu_output_keeps_the_hand_off_out(monkeypatch):
    """If the GELU's output is a graph output it must be written: the GEMM
    still applies the GELU but writes the activation, and the next GEMM
    splits it itself.  (The program is cut after the down-projection so the
    GELU's buffer is never recycled.)"""
    import copy
    monkeypatch.setenv("RT_FUSE_HANDOFF", "1")
    prog = copy.copy(Program.load(GOLDEN / "gpt2_b8.json"))
    u = next(i for i, nd in enumerate(prog.nodes) if nd.op == OP["GELU"])
    prog.nodes = prog.nodes[:u + 2]
    arr, res = bind(prog)
    _, flags = report(prog, arr)
    assert flags[u - 1:u + 2] == [3, 1, 4 if gemm_handoff("1", 3072) else 0]
    nbytes = 4
    for d in prog.nodes[u].out_shape:
        nbytes *= d
    lib = load_library()
    try:
        assert lib.rt_protect(res(prog.nodes[u].output), nbytes) == 0
        flags = (ctypes.c_int * len(prog.nodes))()
        lib.rt_fusion_report(arr, len(prog.nodes), flags)
        assert list(flags)[u - 1:u + 2] == [3, 1, 0]
    finally:
        lib.rt_unprotect_all()


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


def test_qwen3_rotary_chains_fold():
    """Qwen3 q/k paths: SLICE -> RMSNORM -> TRANSPOSE -> rotary (MUL, SLICE, SLICE,
    NEG, CAT, MUL, ADD) run as one fused kernel at the ADD: 9 of 10 nodes per
    chain skipped, 2 chains per layer.  The V path (SLICE -> head-split
    TRANSPOSE) and the head-merge TRANSPOSE fold into the attention although
    the planner put the attention output over the QKV projection V is sliced
    from: the tensor-core path's pre-passes consume V before O is written."""
    prog = Program.load(GOLDEN / "qwen3_b8.json")
    arr, _ = bind(prog)
    n, flags = report(prog, arr)
    assert n == 36 + 2 * 3
    assert [prog.nodes[i].op for i, f in enumerate(flags) if f == 5] == [OP["ADD"]] * 4
    att = [i for i, nd in enumerate(prog.nodes) if nd.op == OP["ATTENTION"]]
    for a in att:
        assert flags[a] == 2
        assert [prog.nodes[a - 2].op, prog.nodes[a - 1].op, prog.nodes[a + 1].op] == \
            [OP["SLICE"], OP["TRANSPOSE"], OP["TRANSPOSE"]]
        assert flags[a - 2] == flags[a - 1] == flags[a + 1] == 1
    folded = sorted({prog.nodes[i].op for i, f in enumerate(flags) if f == 1})
    assert folded == sorted({OP[k] for k in ("SLICE", "RMSNORM", "TRANSPOSE", "MUL", "NEG", "CAT")})


@pytest.mark.parametrize("name,gelus", [("7b_b8", 1), ("toy", 0)])
def test_no_layout_folding_where_the_chain_does_not_match(name, gelus):
    """The custom blocks' bias ADD after the QKV slice folds into
    the merged GEMM only when the bias is a registered constant -- not in this
    host-only report (tests/test_gpu_fusion.py covers it on the device) -- so
    here only the MLP GELU folds into its GEMM (not in the toy block, whose
    GEMMs are below the tensor-core threshold)."""
    prog = Program.load(GOLDEN / f"{name}.json")
    arr, _ = bind(prog)
    n, flags = report(prog, arr)
    assert n == gelus
    assert all(prog.nodes[i].op == OP["GELU"] for i, f in enumerate(flags) if f == 1)


@pytest.mark.parametrize("name,pairs", [("gpt2_b8", 4), ("7b_b8", 2), ("qwen3_b8", 4)])
def test_norms_write_the_split_operand_of_their_gemm(name, pairs):
    """A LAYERNORM / RMSNORM read only as the next GEMM's A operand writes that
    GEMM's split planes (flag 8); the GEMM skips its split pass (flag 4)."""
    prog = Program.load(GOLDEN / f"{name}.json")
    arr, _ = bind(prog)
    _, flags = report(prog, arr)
    producers = [i for i, f in enumerate(flags) if f == 8]
    assert len(producers) == pairs
    assert all(prog.nodes[i].op in (OP["LAYERNORM"], OP["RMSNORM"]) for i in producers)
    # the consumer: 4, or 3 when it also folds an activation into its epilogue
    assert all(flags[i + 1] in (3, 4) and prog.nodes[i + 1].op in (OP["MATMUL"], OP["MATMUL_ADD"])
               for i in producers)


def test_attention_writes_the_projection_split_operand(monkeypatch):
    """GPT-2: each attention (its head merge folded, writing [B, S, H*D]) is
    read only by the output projection's A operand; with RT_FUSE_ATTN_SPLIT=1
    it writes that GEMM's split planes and the GEMM skips its split pass (the
    default keeps the split pass)."""
    prog = Program.load(GOLDEN / "gpt2_b8.json")
    arr, _ = bind(prog)
    ops = [nd.op for nd in prog.nodes]
    proj = [i for i, op in enumerate(ops) if op == OP["MATMUL_ADD"] and OP["ATTENTION"] in ops[max(0, i - 3):i]]
    assert len(proj) == 2
    _, flags = report(prog, arr)
    assert [flags[i] for i in proj] == [0, 0]
    monkeypatch.setenv("RT_FUSE_ATTN_SPLIT", "1")
    _, flags = report(prog, arr)
    assert [flags[i] for i in proj] == ([4, 4] if PLANE_HANDOFFS else [0, 0])


@pytest.mark.parametrize("name,adds", [("gpt2_b8", 4), ("qwen3_b8", 4), ("7b_b8", 2)])
def test_residual_adds_fold_into_their_gemms(name, adds, monkeypatch):
    """Each same-shape residual ADD right after a GEMM is skipped (flag 1) and
    its GEMM (flag 3) adds the residual in the epilogue under
    RT_FUSE_RESIDUAL=1; by default the ADDs run."""
    monkeypatch.setenv("RT_FUSE_RESIDUAL", "1")
    prog = Program.load(GOLDEN / f"{name}.json")
    arr, _ = bind(prog)
    _, flags = report(prog, arr)
    ops = [nd.op for nd in prog.nodes]
    res = [i for i, f in enumerate(flags) if f == 1 and ops[i] == OP["ADD"]]
    assert len(res) == adds
    assert all(prog.nodes[i].extra[0] == 1 and ops[i - 1] in (OP["MATMUL"], OP["MATMUL_ADD"]) and flags[i - 1] == 3
               for i in res)
    monkeypatch.delenv("RT_FUSE_RESIDUAL")
    _, flags = report(prog, arr)
    assert all(flags[i] == 0 for i in res)


def test_plane_hand_offs_under_the_cross_scheme():
    """The split-plane hand-offs above, planned under the tf32 + bf16 cross-term
    scheme (RT_GEMM_SCHEME=cross, read once per process), in a fresh process."""
    import os
    import subprocess
    import sys
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-p", "no:cacheprovider", __file__, "-k",
                        "hands_over or keeps_the_hand_off or projection_split"],
                       env=dict(os.environ, RT_GEMM_SCHEME="cross"), capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and " passed" in r.stdout, r.stdout[-3000:] + r.stderr[-2000:]
