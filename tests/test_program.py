"""Program fixtures, the OpNode ABI and the lowering of reference plans."""

import ctypes
import json
import os
import sys
from pathlib import Path

import numpy as np
import pytest

import oracle
from conftest import GOLDEN, ROOT
from lbr_b200.copnode import COpNode, HostBinding
from lbr_b200.program import OP, Program


def test_opnode_layout_matches_reference_struct():
    # csrc/runtime.h:60-69 on LP64: 4+4 + 12*8 + 8 + 24*4 + 4+4 + 24*4
    assert ctypes.sizeof(COpNode) == 312
    assert COpNode.inputs.offset == 8
    assert COpNode.output.offset == 104
    assert COpNode.out_shape.offset == 112
    assert COpNode.n_dims.offset == 208
    assert COpNode.elem_size.offset == 212
    assert COpNode.extra.offset == 216


def test_op_codes_match_header():
    text = (ROOT / "include" / "b200exec.h").read_text()
    for name, code in OP.items():
        assert f"RT_OP_{name} = {code}" in text, name


@pytest.mark.parametrize("path", sorted(GOLDEN.glob("*.json")), ids=lambda p: p.stem)
def test_program_fixture_is_well_formed(path):
    prog = Program.load(path)
    assert prog.nodes and prog.arena_size > 0
    for n in prog.nodes:
        assert n.op in OP.values() and n.op != OP["PERMUTE"]
        assert len(n.inputs) <= 12 and len(n.extra) <= 24 and 1 <= len(n.out_shape) <= 24
        for r in n.inputs + [n.output]:
            if r.kind == "arena":
                assert 0 <= r.offset < prog.arena_size
            elif r.kind == "const":
                assert r.name in prog.constants
            else:
                assert r.kind == "input" and r.name in prog.inputs
        if n.output.kind == "arena":
            nbytes = int(np.prod(n.out_shape)) * n.elem_size
            assert n.output.offset + nbytes <= prog.arena_size


def test_constant_regeneration_is_deterministic():
    prog = Program.load(GOLDEN / "gpt2_mini_s64.json")
    a = prog.make_constants(0)
    b = prog.make_constants(0)
    for k in a:
        np.testing.assert_array_equal(a[k], b[k])
    w = [v for k, v in a.items() if prog.constants[k].init["kind"] == "randn"][0]
    assert abs(float(w.std()) - 0.02) < 0.002


def test_inputs_split_by_batch_rows():
    prog = Program.load(GOLDEN / "gpt2_b8.json")
    b1 = Program.load(GOLDEN / "gpt2_b1.json")
    full = prog.make_inputs(0)
    name = next(iter(full))
    for r in (0, 5):
        one = b1.make_inputs(0, batch_offset=r)
        np.testing.assert_array_equal(one[name][0], full[name][r])


def test_host_binding_points_into_arena():
    prog = Program.load(GOLDEN / "toy.json")
    hb = HostBinding(prog, prog.make_constants(), prog.make_inputs())
    base = hb.arena.ctypes.data
    for i, n in enumerate(prog.nodes):
        if n.output.kind == "arena":
            assert hb.nodes[i].output == base + n.output.offset


REF = oracle.reference_root()


@pytest.mark.skipif(not (REF / "runtime").is_dir(), reason="reference tree not present")
def test_lowering_matches_reference_compiled_executor():
    """program_from_plan must produce the node array CompiledExecutor.compile builds."""
    import oracle
    if not oracle.available("reference"):
        pytest.skip("oracle/_ref not built")
    sys.path.insert(0, str(REF))
    sys.path.insert(0, str(GOLDEN))
    import make_programs as mp
    for name in ("toy", "qwen3_mini_s272"):
        spec = mp._configs()[name]
        import torch
        torch.manual_seed(0)
        model = spec[0]().eval()
        x = torch.randn(spec[1], spec[2], spec[3])
        graph = mp.export_model(model, (x,))
        mp.run_pipeline(graph)
        ep = mp.ref_plan(graph)
        from lbr_b200.lower import program_from_plan
        prog = program_from_plan(ep, name)
        mp._check_against_reference_compile(prog, ep, graph)
        committed = json.loads((GOLDEN / f"{name}.json").read_text())
        assert [n.to_json() for n in prog.nodes] == committed["nodes"]
