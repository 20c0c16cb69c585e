"""Generate the interpreted-executor traces (test infrastructure).

The reference's interpreted executor (runtime/executor/interpreted.py:47-98)
walks ``plan.order`` and, for every node that is not a zero-copy alias of an
intermediate, calls ``kernel(input_buffers, output_buffer, node.attrs)`` on
the first backend that has a kernel, appending the node's planned scratch
region as an extra input.  This script records exactly those calls for a
few small configurations -- op, attrs, input / output tensor names and
shapes, scratch bytes, and the alias nodes it skips -- so that the GPU test
``tests/test_gpu_interp.py`` can replay them through ``CudaBackend`` on a
box where the reference package does not exist.  It also runs the
reference's own ``InterpretedExecutor`` with its numpy backend on the same
weights and inputs and stores that result next to the trace.

Weights and inputs are those of the committed programs (``<name>.json`` /
``<name>.golden.npz``; the traces go to ``interp/<name>.json`` / ``.npz``), so the replay is also checked against the reference
C executor's golden output.

    python tests/golden/make_interp_traces.py
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import make_programs as mp  # noqa: E402  (sets up the reference import path)

from lbr_b200.program import Program                         # noqa: E402
from runtime.exporter import export_model                    # noqa: E402
from runtime.passes import run_pipeline                      # noqa: E402
from runtime.planner import plan as ref_plan                 # noqa: E402
from runtime.ir import FOLD_ONLY_BASE                        # noqa: E402
from runtime.ops import OP_REGISTRY                          # noqa: E402
from runtime.executor.interpreted import InterpretedExecutor  # noqa: E402
from runtime.backends.numpy_backend import NumpyBackend      # noqa: E402

NAMES = ("toy", "gpt2_mini_s64", "qwen3_mini_s272", "block_mini_causal_s300")


def jsonable(v):
    if isinstance(v, (bool, int, float, str)) or v is None:
        return v
    if isinstance(v, (list, tuple)):
        return [jsonable(x) for x in v]
    if isinstance(v, dict):
        return {str(k): jsonable(x) for k, x in v.items()}
    if isinstance(v, (np.integer,)):
        return int(v)
    if isinstance(v, (np.floating,)):
        return float(v)
    raise TypeError(f"attr value {v!r} ({type(v)}) is not JSON-serialisable")


def trace(name):
    builder, B, S, D, _ = mp._configs()[name]
    torch.manual_seed(0)
    model = builder().eval()
    x = torch.randn(B, S, D)
    graph = export_model(model, (x,))
    run_pipeline(graph)
    ep = ref_plan(graph)
    prog = Program.load(HERE / f"{name}.json")
    consts = prog.make_constants(0)
    gold = np.load(HERE / f"{name}.golden.npz")
    inputs = {k[4:]: gold[k] for k in gold.files if k.startswith("in__")}
    # the program's weights, bound to the graph's constant tensors
    for c in graph.constants:
        assert c in consts, c
        graph.tensors[c].buffer = np.ascontiguousarray(consts[c]).reshape(graph.tensors[c].shape)
    external = set(graph.inputs) | set(graph.constants)
    steps = []
    for node in ep.order:
        op_def = OP_REGISTRY.get(node.op)
        out = graph.tensors[node.output]
        entry = {"op": int(node.op.value), "op_name": node.op.name, "inputs": list(node.inputs),
                 "in_shapes": [list(graph.tensors[i].shape) for i in node.inputs],
                 "output": node.output, "out_shape": list(out.shape), "dtype": str(np.dtype(out.dtype)),
                 "attrs": jsonable(dict(node.attrs))}
        if op_def is not None and op_def.is_alias(node) and node.inputs[0] not in external:
            entry["alias"] = True
            entry["alias_offset"] = int(op_def.alias_offset(node)) if op_def.alias_offset else 0
        else:
            assert node.op.value < FOLD_ONLY_BASE
            entry["alias"] = False
            entry["scratch_bytes"] = int(ep.scratch[node.id][1]) if node.id in ep.scratch else 0
        steps.append(entry)
    ex = InterpretedExecutor(backends=[NumpyBackend()])
    ex.compile(ep)
    interp = ex.run(inputs)
    doc = {"name": name, "graph_inputs": list(graph.inputs), "graph_outputs": list(graph.outputs),
           "generator": "tests/golden/make_interp_traces.py", "steps": steps}
    (HERE / "interp" / f"{name}.json").write_text(json.dumps(doc, indent=0))
    np.savez_compressed(HERE / "interp" / f"{name}.npz", **{f"out__{k}": v for k, v in interp.items()})
    ref = {k[5:]: gold[k] for k in gold.files if k.startswith("out__")}
    err = max(float(np.abs(interp[k] - ref[k]).max()) for k in ref)
    print(f"{name}: {len(steps)} steps ({sum(s['alias'] for s in steps)} aliases), "
          f"numpy interpreted vs C executor {err:.2e}", flush=True)


if __name__ == "__main__":
    for n in (sys.argv[1:] or NAMES):
        trace(n)
