"""``OpNode.extra[]`` from input shapes, output shape and node attrs.

The interpreted path hands a backend kernel only ``(inputs, output, attrs)``
(runtime/executor/interpreted.py:21-32); the compiled path packs ``extra[]``
with the per-op hooks of ``OP_REGISTRY`` (runtime/ops.py:137-329), which read
the same information from the graph.  This module restates those packers
over plain shapes so that :class:`~backend.CudaBackend` can build a node
without the reference graph layer.  The encodings must be identical -- the
library decodes them exactly as the reference C executor does -- and
``tests/test_extras.py`` checks them against ``OP_REGISTRY`` on real graphs.
"""

from __future__ import annotations

import struct
from typing import Any, Sequence

from .program import OP


def float_bits(x: float) -> int:
    """fp32 bit pattern as a signed int (runtime/ops.py:34-39)."""
    return struct.unpack("i", struct.pack("f", float(x)))[0]


def _prod(xs) -> int:
    r = 1
    for x in xs:
        r *= int(x)
    return r


def _bcast_strides(shape: Sequence[int], out: Sequence[int]) -> list[int]:
    """Element strides of ``shape`` broadcast against ``out``; 0 on broadcast dims
    (runtime/ops.py:173-190)."""
    nd, off = len(out), len(out) - len(shape)
    return [0 if d < off or shape[d - off] == 1 else _prod(shape[d - off + 1:]) for d in range(nd)]


def _pack_bcast(a, b, out) -> list[int]:
    """[ndim, a_strides..., b_strides..., out_shape...] (runtime/ops.py:193-200)."""
    return [len(out)] + _bcast_strides(a, out) + _bcast_strides(b, out) + [int(x) for x in out]


def _matmul(ins, out, attrs):
    """[K, trans_b, b_is_2d, alpha_bits or 0] (runtime/ops.py:137-146)."""
    a, b = ins[0], ins[1]
    alpha = attrs.get("alpha", 1.0)
    return [int(a[-1]), 1 if attrs.get("transpose_b") else 0, 1 if len(b) == 2 and len(a) > 2 else 0,
            float_bits(alpha) if alpha != 1.0 else 0]


def _transpose(ins, out, attrs):
    """2-D: [rows, cols]; N-D: [outer, A, middle, B, inner] (runtime/ops.py:149-171)."""
    s = ins[0]
    if len(s) == 2:
        return [int(s[0]), int(s[1])]
    d0, d1 = sorted((attrs.get("dim0", 0), attrs.get("dim1", 1)))
    return [_prod(s[:d0]), int(s[d0]), _prod(s[d0 + 1:d1]), int(s[d1]), _prod(s[d1 + 1:])]


def _add(ins, out, attrs):
    """mode 0 bias / 1 same shape / 2 scalar / 3 broadcast (runtime/ops.py:203-219)."""
    if "scalar" in attrs:
        return [2, float_bits(attrs["scalar"])]
    a, b = tuple(ins[0]), tuple(ins[1])
    if a == b:
        return [1]
    if len(b) == 1 and b[-1] == a[-1]:
        return [0]
    o = attrs.get("_out_shape") or out
    return [3] + _pack_bcast(a, b, o)


def _binop(ins, out, attrs):
    """SUB / MUL / DIV: mode 0 same shape / 1 scalar / 2 broadcast (runtime/ops.py:222-235)."""
    if "scalar" in attrs:
        return [1, float_bits(attrs["scalar"])]
    a, b = tuple(ins[0]), tuple(ins[1])
    if a == b:
        return [0]
    return [2] + _pack_bcast(a, b, out)


def _reduce(ins, out, attrs):
    """[axis, axis_size] (runtime/ops.py:238-242)."""
    axis = attrs.get("axis", -1)
    return [axis, int(ins[0][axis])]


def _eps(ins, out, attrs):
    """[eps_bits] (runtime/ops.py:245-254)."""
    return [float_bits(attrs.get("eps", 1e-5))]


def _attention(ins, out, attrs):
    """[seq_len, head_dim, causal, has_mask, group_size] (runtime/ops.py:257-262).
    ``has_mask`` counts graph inputs: a fourth input is the mask (the planner's
    scratch, when present, is appended after them and is not counted)."""
    q = ins[0]
    n_graph_inputs = attrs.get("_n_graph_inputs", len(ins))
    return [int(q[-2]), int(q[-1]), 1 if attrs.get("causal") else 0, 1 if n_graph_inputs > 3 else 0,
            attrs.get("group_size", 1)]


def _pow(ins, out, attrs):
    """[scalar_bits], default exponent 2 (runtime/ops.py:265-267)."""
    return [float_bits(attrs.get("scalar", 2.0))]


def _embedding(ins, out, attrs):
    """[embed_dim] (runtime/ops.py:270-272)."""
    return [int(ins[1][-1])]


def _cat(ins, out, attrs):
    """[dim, size_0, size_1, ...] (runtime/ops.py:275-279)."""
    dim = attrs["dim"]
    return [dim] + [int(s[dim]) for s in ins]


def _gated(ins, out, attrs):
    """[has_bias, act (0 silu, 1 gelu)] (runtime/ops.py:282-286)."""
    return [1 if attrs.get("has_bias") else 0, 0 if attrs.get("act", "silu") == "silu" else 1]


def _slice(ins, out, attrs):
    """[outer, dim_size, start, len, inner] (runtime/ops.py:310-329)."""
    s = ins[0]
    dim, start = attrs["dim"], attrs["start"]
    end = min(attrs["end"], s[dim])
    return [_prod(s[:dim]), int(s[dim]), start, end - start, _prod(s[dim + 1:])]


PACKERS = {
    OP["MATMUL"]: _matmul, OP["MATMUL_ADD"]: _matmul, OP["TRANSPOSE"]: _transpose,
    OP["ADD"]: _add, OP["SUB"]: _binop, OP["MUL"]: _binop, OP["DIV"]: _binop,
    OP["MAX"]: _reduce, OP["SUM"]: _reduce, OP["LAYERNORM"]: _eps, OP["RMSNORM"]: _eps,
    OP["ATTENTION"]: _attention, OP["POW"]: _pow, OP["EMBEDDING"]: _embedding, OP["CAT"]: _cat,
    OP["GATED_ACT"]: _gated, OP["SLICE"]: _slice,
}


def pack_extras(op: int, in_shapes: Sequence[Sequence[int]], out_shape: Sequence[int],
                attrs: dict[str, Any]) -> list[int]:
    """``extra[]`` of a node with op code ``op`` (ops without a packer: none)."""
    fn = PACKERS.get(int(op))
    return [int(v) for v in fn(list(in_shapes), list(out_shape), attrs)] if fn else []
