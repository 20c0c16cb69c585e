"""extras.pack_extras (the interpreted backend's extra[] packing) against the
reference's own OP_REGISTRY packers (runtime/ops.py:137-329): on synthetic
nodes covering every mode, and on every node of exported graphs.  Needs the
reference's ``runtime`` package; skipped where it is absent."""

import os
import sys

import numpy as np
import pytest

import oracle

REF_ROOT = str(oracle.reference_root())
if os.path.isdir(REF_ROOT) and REF_ROOT not in sys.path:
    sys.path.insert(0, REF_ROOT)
runtime = pytest.importorskip("runtime")
torch = pytest.importorskip("torch")

from runtime.ir import Graph, OpType  # noqa: E402
from runtime.ops import OP_REGISTRY  # noqa: E402

from lbr_b200.extras import PACKERS, pack_extras  # noqa: E402


def ref_extras(graph, node):
    d = OP_REGISTRY.get(node.op)
    return [] if d is None or d.extras is None else [int(v) for v in d.extras(node, graph)]


def mine(graph, node):
    ins = [graph.tensors[i].shape for i in node.inputs]
    return pack_extras(node.op.value, ins, graph.tensors[node.output].shape, node.attrs)


CASES = [
    # (op, input shapes, output shape, attrs)
    ("MATMUL", [(2, 8, 16), (16, 32)], (2, 8, 32), {}),
    ("MATMUL", [(2, 8, 16), (32, 16)], (2, 8, 32), {"transpose_b": True, "alpha": 0.125}),
    ("MATMUL", [(3, 8, 16), (3, 16, 4)], (3, 8, 4), {}),
    ("MATMUL_ADD", [(8, 16), (32, 16), (32,)], (8, 32), {"transpose_b": True}),
    ("TRANSPOSE", [(5, 7)], (7, 5), {}),
    ("TRANSPOSE", [(2, 3, 4, 5)], (2, 4, 3, 5), {"dim0": 1, "dim1": 2}),
    ("TRANSPOSE", [(2, 3, 4, 5)], (2, 5, 4, 3), {"dim0": 3, "dim1": 1}),
    ("ADD", [(4, 8)], (4, 8), {"scalar": 1.5}),
    ("ADD", [(4, 8), (4, 8)], (4, 8), {}),
    ("ADD", [(4, 8), (8,)], (4, 8), {}),
    ("ADD", [(4, 1, 8), (3, 1)], (4, 3, 8), {}),
    ("SUB", [(4, 8)], (4, 8), {"scalar": 2.0}),
    ("MUL", [(4, 8), (4, 8)], (4, 8), {}),
    ("DIV", [(2, 4, 8), (1, 4, 1)], (2, 4, 8), {}),
    ("MAX", [(4, 8)], (4,), {"axis": -1}),
    ("SUM", [(4, 6, 8)], (4, 8), {"axis": 1}),
    ("LAYERNORM", [(4, 8), (8,), (8,)], (4, 8), {"eps": 1e-6}),
    ("RMSNORM", [(4, 8), (8,)], (4, 8), {}),
    ("ATTENTION", [(1, 4, 32, 16)] * 3, (1, 4, 32, 16), {"causal": True}),
    ("ATTENTION", [(1, 4, 32, 16), (1, 2, 32, 16), (1, 2, 32, 16), (1, 4, 32, 32)], (1, 4, 32, 16),
     {"group_size": 2}),
    ("POW", [(4, 8)], (4, 8), {"scalar": 3.0}),
    ("POW", [(4, 8)], (4, 8), {}),
    ("EMBEDDING", [(2, 5), (100, 16)], (2, 5, 16), {}),
    ("CAT", [(2, 3, 4), (2, 5, 4)], (2, 8, 4), {"dim": 1}),
    ("GATED_ACT", [(4, 8), (8,), (4, 8)], (4, 8), {"has_bias": True, "act": "gelu"}),
    ("GATED_ACT", [(4, 8), (4, 8)], (4, 8), {}),
    ("SLICE", [(2, 6, 10)], (2, 6, 4), {"dim": 2, "start": 3, "end": 7}),
    ("SLICE", [(2, 6, 10)], (2, 2, 10), {"dim": 1, "start": 4, "end": 99}),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c[0]}-{len(c[1])}-{sorted(c[3])}")
def test_synthetic_node(case):
    op, ins, out, attrs = case
    g = Graph()
    names = []
    for k, s in enumerate(ins):
        n = f"i{k}"
        g.add_tensor(n, s, "int64" if op == "EMBEDDING" and k == 0 else "float32")
        names.append(n)
    g.add_tensor("o", out, "float32")
    node = g.add_node(OpType[op], names, "o", dict(attrs))
    assert mine(g, node) == ref_extras(g, node)


def test_every_packer_is_covered():
    assert {OpType[c[0]].value for c in CASES} >= set(PACKERS)


def _graphs():
    from runtime.exporter import export_model
    from runtime.passes import run_pipeline
    sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
    import make_programs as mp          # the fixtures' model definitions
    out = []
    for build, shape in [(lambda: mp.CustomBlock(128, 2, 512, True), (2, 40, 128)),
                         (lambda: mp.GPT2Body(2, 2, 128), (2, 24, 128)),
                         (lambda: mp.Qwen3Body(256, 512, 2, 4, 2, 128), (1, 24, 256))]:
        torch.manual_seed(0)
        g = export_model(build().eval(), (torch.randn(*shape),))
        run_pipeline(g)
        out.append(g)
    return out


def test_exported_graph_nodes():
    n = 0
    for g in _graphs():
        for node in g:
            if node.op.value in PACKERS:
                assert mine(g, node) == ref_extras(g, node), node
                n += 1
    assert n > 20
