"""CudaBackend (the interpreted executor's GPU backend): every op through
``get_kernel(op)(inputs, output, attrs)`` against numpy, the reference's own
kernel contract (runtime/executor/interpreted.py:21-32)."""

from types import SimpleNamespace

import numpy as np
import pytest

from lbr_b200.backend import SUPPORTED, CudaBackend
from lbr_b200.program import OP

pytestmark = pytest.mark.gpu
rng = np.random.default_rng(5)


def R(*s):
    return rng.standard_normal(s).astype(np.float32)


@pytest.fixture(scope="module")
def be():
    b = CudaBackend()
    yield b
    b.close()


def run(be, op, ins, out_shape, attrs=None, dtype=np.float32):
    k = be.get_kernel(SimpleNamespace(value=OP[op]))
    out = np.full(out_shape, np.nan, dtype=dtype)
    k(ins, out, attrs or {})
    return out


def gelu(x):
    return 0.5 * x * (1 + np.tanh(0.7978845608 * (x + 0.044715 * x ** 3)))


def silu(x):
    return x / (1 + np.exp(-x))


UNARY = {"RELU": lambda x: np.maximum(x, 0), "EXP": np.exp, "TANH": np.tanh, "GELU": gelu,
         "SILU": silu, "NEG": np.negative, "COS": np.cos, "SIN": np.sin}


@pytest.mark.parametrize("op", sorted(UNARY))
def test_unary(be, op):
    x = R(3, 257)
    np.testing.assert_allclose(run(be, op, [x], x.shape), UNARY[op](x), rtol=2e-6, atol=2e-6)


def test_pow_rsqrt(be):
    x = np.abs(R(1000)) + 0.1
    np.testing.assert_allclose(run(be, "POW", [x], x.shape, {"scalar": 1.5}), x ** 1.5, rtol=1e-5)
    np.testing.assert_allclose(run(be, "RSQRT", [x], x.shape), 1 / np.sqrt(x), rtol=1e-5)


def test_binary_modes(be):
    a, b, bias = R(4, 6, 8), R(4, 6, 8), R(8)
    np.testing.assert_allclose(run(be, "ADD", [a, b], a.shape), a + b, rtol=1e-6)
    np.testing.assert_allclose(run(be, "ADD", [a, bias], a.shape), a + bias, rtol=1e-6)
    np.testing.assert_allclose(run(be, "ADD", [a], a.shape, {"scalar": 2.5}), a + 2.5, rtol=1e-6)
    c = R(6, 1)
    np.testing.assert_allclose(run(be, "ADD", [a, c], a.shape), a + c, rtol=1e-6)
    np.testing.assert_allclose(run(be, "SUB", [a, b], a.shape), a - b, rtol=1e-6)
    np.testing.assert_allclose(run(be, "MUL", [a], a.shape, {"scalar": -3.0}), a * -3.0, rtol=1e-6)
    d = np.abs(R(1, 6, 1)) + 0.5
    np.testing.assert_allclose(run(be, "DIV", [a, d], a.shape), a / d, rtol=1e-6)
    np.testing.assert_allclose(run(be, "FUSED_BIAS_RELU", [a, bias], a.shape), np.maximum(a + bias, 0), rtol=1e-6)


@pytest.mark.parametrize("case", [((5, 64), (64, 48), {}), ((2, 300, 96), (96, 200), {}),
                                  ((2, 300, 96), (200, 96), {"transpose_b": True, "alpha": 0.5}),
                                  ((3, 40, 24), (3, 24, 16), {})], ids=str)
def test_matmul(be, case):
    sa, sb, attrs = case
    a, b = R(*sa), R(*sb) * 0.1
    bb = np.swapaxes(b, -1, -2) if attrs.get("transpose_b") else b
    ref = np.matmul(a, bb) * attrs.get("alpha", 1.0)
    got = run(be, "MATMUL", [a, b], ref.shape, attrs)
    np.testing.assert_allclose(got, ref, atol=1e-4, rtol=1e-3)
    # MATMUL_ADD carries no alpha (the reference's dispatch ignores extra[3] for it)
    bias = R(ref.shape[-1])
    got = run(be, "MATMUL_ADD", [a, b, bias], ref.shape, attrs)
    np.testing.assert_allclose(got, np.matmul(a, bb) + bias, atol=1e-4, rtol=1e-3)


def test_norms_and_reductions(be):
    x, w, b = R(7, 300), R(300), R(300)
    mu, var = x.mean(-1, keepdims=True), x.var(-1, keepdims=True)
    np.testing.assert_allclose(run(be, "LAYERNORM", [x, w, b], x.shape, {"eps": 1e-5}),
                               (x - mu) / np.sqrt(var + 1e-5) * w + b, atol=1e-5, rtol=1e-4)
    np.testing.assert_allclose(run(be, "RMSNORM", [x, w], x.shape, {"eps": 1e-6}),
                               x / np.sqrt((x * x).mean(-1, keepdims=True) + 1e-6) * w, atol=1e-5, rtol=1e-4)
    e = np.exp(x - x.max(-1, keepdims=True))
    np.testing.assert_allclose(run(be, "SOFTMAX", [x], x.shape, {"axis": -1}), e / e.sum(-1, keepdims=True),
                               rtol=1e-5, atol=1e-7)
    y = R(4, 6, 5)
    np.testing.assert_allclose(run(be, "MAX", [y], (4, 5), {"axis": 1}), y.max(1), rtol=1e-6)
    np.testing.assert_allclose(run(be, "SUM", [y], (4, 6), {"axis": -1}), y.sum(-1), rtol=1e-5)


def test_layout(be):
    x = R(2, 3, 4, 5)
    np.testing.assert_array_equal(run(be, "TRANSPOSE", [x], (2, 4, 3, 5), {"dim0": 1, "dim1": 2}),
                                  np.swapaxes(x, 1, 2))
    m = R(7, 9)
    np.testing.assert_array_equal(run(be, "TRANSPOSE", [m], (9, 7)), m.T)
    np.testing.assert_array_equal(run(be, "SLICE", [x], (2, 3, 4, 2), {"dim": 3, "start": 1, "end": 3}),
                                  x[..., 1:3])
    y = R(2, 3, 7, 5)
    np.testing.assert_array_equal(run(be, "CAT", [x, y], (2, 3, 11, 5), {"dim": 2}), np.concatenate([x, y], 2))
    np.testing.assert_array_equal(run(be, "RESHAPE", [x], (6, 20), {"shape": (6, 20)}), x.reshape(6, 20))


def test_embedding_and_gated(be):
    table, ids = R(50, 16), rng.integers(0, 50, (3, 7)).astype(np.int64)
    np.testing.assert_array_equal(run(be, "EMBEDDING", [ids, table], (3, 7, 16)), table[ids])
    g, u, bias = R(5, 64), R(5, 64), R(64)
    np.testing.assert_allclose(run(be, "GATED_ACT", [g, u], g.shape, {"act": "silu"}), silu(g) * u,
                               rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(run(be, "GATED_ACT", [g, bias, u], g.shape, {"has_bias": True, "act": "gelu"}),
                               gelu(g + bias) * u, rtol=1e-5, atol=1e-6)


def attention_ref(q, k, v, causal=False, mask=None):
    g = q.shape[1] // k.shape[1]
    k, v = np.repeat(k, g, 1), np.repeat(v, g, 1)
    s = q @ np.swapaxes(k, -1, -2) / np.sqrt(q.shape[-1])
    if mask is not None:
        s = s + mask
    if causal:
        s = s + np.triu(np.full(s.shape[-2:], -np.inf, np.float32), 1)
    e = np.exp(s - s.max(-1, keepdims=True))
    return (e / e.sum(-1, keepdims=True)) @ v


@pytest.mark.parametrize("S,D,causal,group,mask,scratch", [
    (64, 32, False, 1, False, False), (300, 64, True, 1, False, True),
    (256, 128, True, 2, False, True), (48, 16, False, 1, True, False)])
def test_attention(be, S, D, causal, group, mask, scratch):
    q = R(1, 4, S, D)
    k, v = R(1, 4 // group, S, D), R(1, 4 // group, S, D)
    ins = [q, k, v]
    m = R(1, 4, S, S) if mask else None
    if mask:
        ins.append(m)
    if scratch:                       # the planner's scratch slice, as the interpreted executor appends it
        ins.append(np.zeros(4096, np.uint8))
    got = run(be, "ATTENTION", ins, q.shape, {"causal": causal, "group_size": group})
    np.testing.assert_allclose(got, attention_ref(q, k, v, causal, m), atol=1e-4, rtol=1e-3)


def test_repeated_shapes_reuse_one_plan(be):
    lib = be._lib
    x = R(1000)
    run(be, "EXP", [x], x.shape)
    n = lib.rt_plan_count()
    for _ in range(5):
        run(be, "EXP", [R(1000)], x.shape)
    assert lib.rt_plan_count() == n


def test_unsupported_op_falls_through(be):
    assert be.get_kernel(SimpleNamespace(value=OP["PERMUTE"])) is None
    assert be.get_kernel(SimpleNamespace(value=5000)) is None
    assert OP["MATMUL"] in SUPPORTED
