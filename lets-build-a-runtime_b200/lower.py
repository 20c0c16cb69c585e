"""Lower a reference ``MemoryPlan`` to a :class:`~program.Program`.

This is the reference compiled executor's compile step
(runtime/executor/compiled.py:34-70 and ``_build_node`` :108-145,
``_fill_extras`` :152-158) with pointers kept symbolic instead of resolved
against a host arena.  It needs the reference's graph layer (``runtime``
package: ``OP_REGISTRY``, ``FOLD_ONLY_BASE``) importable, because the
op-registry hooks -- alias predicates and extras packers -- are consumed
unchanged from there.

Differences from the reference, on purpose:

* none in the node array: same filtering (aliases of internal tensors are
  skipped, aliases of graph inputs/constants are dispatched), same input
  order, scratch appended as the last input, same ``out_shape``,
  ``elem_size`` and ``extra[]``;
* offsets of alias outputs are those the planner already propagated
  (``plan.offsets``), exactly what ``Executor._bind_intermediates``
  (runtime/executor/common.py:96-104) turns into arena views.
"""

from __future__ import annotations

import numpy as np

from .program import ConstSpec, ProgNode, Program, Ref

STORE_MAX_ELEMS = 300_000   # constants up to this size are kept verbatim


def _classify_constant(name: str, arr: np.ndarray, store_all: bool) -> tuple[dict, np.ndarray | None]:
    arr = np.ascontiguousarray(arr)
    if store_all:
        return {"kind": "stored"}, arr
    flat = arr.reshape(-1)
    if flat.size and np.all(flat == flat[0]):
        return {"kind": "fill", "value": float(flat[0])}, None
    # trained parameters ("p_*" from torch.export, "_merged_weight*" from
    # merge_parallel_matmuls) are regenerated; everything else that varies
    # (rotary tables, masks folded from buffers) is kept verbatim
    is_param = name.startswith("p_") or name.startswith("_merged_weight")
    if arr.dtype != np.float32 or (not is_param and flat.size <= STORE_MAX_ELEMS):
        return {"kind": "stored"}, arr
    return {"kind": "randn", "mean": float(flat.mean()), "std": float(flat.std())}, None


def program_from_plan(plan, name: str, meta: dict | None = None,
                      store_all: bool = False) -> Program:
    """Build a Program from a reference MemoryPlan (see module docstring)."""
    from runtime.ir import FOLD_ONLY_BASE          # reference graph layer
    from runtime.ops import OP_REGISTRY

    graph = plan.graph
    inputs = set(graph.inputs)
    consts = set(graph.constants)
    external = inputs | consts

    def ref_of(tname: str) -> Ref:
        if tname in inputs:
            return Ref("input", tname, 0)
        if tname in consts:
            return Ref("const", tname, 0)
        if tname not in plan.offsets:
            raise RuntimeError(f"tensor {tname!r} has no arena offset")
        return Ref("arena", None, int(plan.offsets[tname]))

    # Aliases of external tensors: the reference dispatches them
    # (compiled.py:50-60) -- a RESHAPE of a graph input becomes a copy.
    nodes: list[ProgNode] = []
    for node in plan.order:
        op_def = OP_REGISTRY.get(node.op)
        is_alias = op_def is not None and op_def.is_alias(node)
        if is_alias and node.inputs[0] not in external:
            continue
        if node.op.value >= FOLD_ONLY_BASE:
            raise RuntimeError(f"fold-only op {node.op.name} reached the executor")
        ins = [ref_of(t) for t in node.inputs]
        if node.id in plan.scratch:
            off, _size = plan.scratch[node.id]
            ins.append(Ref("arena", None, int(off)))
        out_t = graph.tensors[node.output]
        extra = []
        if op_def is not None and op_def.extras is not None:
            extra = [int(v) for v in op_def.extras(node, graph)]
        nodes.append(ProgNode(node.op.value, ins, ref_of(node.output),
                              [int(d) for d in out_t.shape],
                              int(np.dtype(out_t.dtype).itemsize), extra))

    const_specs: dict[str, ConstSpec] = {}
    stored: dict[str, np.ndarray] = {}
    used = {r.name for n in nodes for r in n.inputs if r.kind == "const"}
    used |= {n.output.name for n in nodes if n.output.kind == "const"}
    for cname in graph.constants:
        if cname not in used:
            continue
        t = graph.tensors[cname]
        arr = np.asarray(t.buffer)
        init, keep = _classify_constant(cname, arr, store_all)
        const_specs[cname] = ConstSpec(cname, tuple(int(d) for d in arr.shape),
                                       str(arr.dtype), init)
        if keep is not None:
            stored[cname] = keep

    ins_spec = {n: {"shape": [int(d) for d in graph.tensors[n].shape],
                    "dtype": str(np.dtype(graph.tensors[n].dtype))} for n in graph.inputs}
    outs_spec = {n: {"shape": [int(d) for d in graph.tensors[n].shape],
                     "dtype": str(np.dtype(graph.tensors[n].dtype)), "ref": ref_of(n)}
                 for n in graph.outputs}
    return Program(name, dict(meta or {}), int(plan.arena_size), ins_spec, outs_spec,
                   const_specs, nodes, stored)
