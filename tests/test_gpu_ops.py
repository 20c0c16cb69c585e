"""Per-op GPU parity: one-node programs against the restated CPU oracle.

Mirrors the reference's per-kernel tests (tests/test_backends.py): every op
code of the dispatch table (csrc/executor.c:409-452), every extras mode,
aligned and ragged sizes.  Tolerances: 1e-5 relative-ish for elementwise
and data movement (bit-exact for pure copies)
(atol 1e-4, rtol 1e-3) for contractions.
"""

import struct

import numpy as np
import pytest

import oracle
from conftest import single_node_program
from lbr_b200.program import OP

pytestmark = pytest.mark.gpu
rng = np.random.default_rng(1234)


def fb(x):
    return struct.unpack("i", struct.pack("f", x))[0]


def rand(*shape, positive=False):
    a = rng.standard_normal(shape).astype(np.float32)
    return np.abs(a) + 0.1 if positive else a


def run_both(factory, prog):
    consts = {k: v for k, v in prog.stored.items()}
    ex = factory(prog, consts)
    got = ex.run({})["y"]
    ref = oracle.run_program("restated", prog, consts, {})["y"]
    ex.close()
    return got, ref


def strides(shape, out):
    nd = len(out)
    off = nd - len(shape)
    s = []
    for d in range(nd):
        if d < off or shape[d - off] == 1:
            s.append(0)
        else:
            s.append(int(np.prod(shape[d - off + 1:])))
    return s


UNARY = ["RELU", "EXP", "TANH", "POW", "GELU", "RSQRT", "SILU", "NEG", "COS", "SIN"]


@pytest.mark.parametrize("n", [4096, 1001])
@pytest.mark.parametrize("op", UNARY)
def test_unary(op, n, gpu_executor_factory):
    x = rand(n, positive=op in ("RSQRT", "POW"))
    extra = [fb(1.5)] if op == "POW" else []
    got, ref = run_both(gpu_executor_factory, single_node_program(OP[op], [x], [n], extra))
    np.testing.assert_allclose(got, ref, rtol=2e-6, atol=1e-6)


@pytest.mark.parametrize("shape", [(4, 33, 64), (3, 7, 5)])
def test_add_modes(shape, gpu_executor_factory):
    a, b = rand(*shape), rand(*shape)
    bias = rand(shape[-1])
    for ins, extra in [([a, bias], [0]), ([a, b], [1]), ([a], [2, fb(0.75)])]:
        got, ref = run_both(gpu_executor_factory, single_node_program(OP["ADD"], ins, shape, extra))
        np.testing.assert_array_equal(got, ref)
    b2 = rand(1, shape[1], 1)
    out = list(shape)
    extra = [3, 3] + strides(shape, out) + strides(b2.shape, out) + out
    got, ref = run_both(gpu_executor_factory, single_node_program(OP["ADD"], [a, b2], out, extra))
    np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("op", ["SUB", "MUL", "DIV"])
def test_binary_modes(op, gpu_executor_factory):
    shape = [2, 4, 16, 8]
    a, b = rand(*shape), rand(*shape, positive=True)
    for ins, extra in [([a, b], [0]), ([a], [1, fb(1.7)])]:
        got, ref = run_both(gpu_executor_factory, single_node_program(OP[op], ins, shape, extra))
        np.testing.assert_allclose(got, ref, rtol=1e-6)
    # RoPE-style broadcast [B,H,S,D] x [1,1,S,D]
    c = rand(1, 1, 16, 8, positive=True)
    extra = [2, 4] + strides(shape, shape) + strides(c.shape, shape) + shape
    got, ref = run_both(gpu_executor_factory, single_node_program(OP[op], [a, c], shape, extra))
    np.testing.assert_allclose(got, ref, rtol=1e-6)


@pytest.mark.parametrize("has_bias,act", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_gated_act(has_bias, act, gpu_executor_factory):
    x, up, bias = rand(6, 48), rand(6, 48), rand(48)
    ins = [x, bias, up] if has_bias else [x, up]
    got, ref = run_both(gpu_executor_factory,
                        single_node_program(OP["GATED_ACT"], ins, [6, 48], [has_bias, act]))
    np.testing.assert_allclose(got, ref, rtol=2e-6, atol=1e-6)


def test_fused_bias_relu(gpu_executor_factory):
    a, b = rand(10, 24), rand(24)
    got, ref = run_both(gpu_executor_factory, single_node_program(OP["FUSED_BIAS_RELU"], [a, b], [10, 24], []))
    np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("C", [16, 64, 100, 128, 768, 1024, 2048, 3000, 4096, 5000])
@pytest.mark.parametrize("op", ["LAYERNORM", "RMSNORM", "SOFTMAX"])
def test_row_ops(op, C, gpu_executor_factory):
    rows = 37
    x = rand(rows, C) * 3 + 1
    g, b = rand(C), rand(C)
    if op == "LAYERNORM":
        ins, extra = [x, g, b], [fb(1e-5)]
    elif op == "RMSNORM":
        ins, extra = [x, g], [fb(1e-6)]
    else:
        ins, extra = [x], []
    got, ref = run_both(gpu_executor_factory, single_node_program(OP[op], ins, [rows, C], extra))
    np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("op", ["MAX", "SUM"])
def test_reductions(op, gpu_executor_factory):
    x = rand(3, 5, 7)
    # reduce axis 1 without keepdim: out [3, 7]
    got, ref = run_both(gpu_executor_factory, single_node_program(OP[op], [x], [3, 7], [1, 5]))
    np.testing.assert_allclose(got, ref, rtol=1e-6)


MM_CASES = [
    # (M, N, K, trans_b, b_is_2d, batches, alpha, bias)
    (32, 64, 64, 1, 1, 1, 1.0, True),
    (300, 200, 136, 1, 1, 1, 1.0, True),
    (257, 130, 96, 0, 1, 1, 1.0, False),
    (128, 256, 512, 1, 1, 1, 0.125, False),
    (1, 96, 64, 1, 1, 1, 1.0, True),
    (64, 48, 40, 1, 0, 3, 1.0, False),
    (50, 70, 33, 0, 0, 2, 1.0, False),
    (1024, 768, 768, 1, 1, 1, 1.0, True),
    (512, 1152, 3072, 1, 1, 1, 1.0, True),
    # CTA-pair tiles (M > 128): ragged M and N, batched, last K block of 4 / 8 / 12
    (300, 520, 200, 0, 0, 3, 1.0, False),
    (640, 1000, 1028, 1, 1, 1, 1.0, True),
    (384, 256, 20, 1, 1, 1, 1.0, False),
    (2000, 300, 1000, 0, 1, 1, 0.5, False),
]


@pytest.mark.parametrize("case", MM_CASES, ids=lambda c: "x".join(map(str, c[:6])))
def test_matmul(case, gpu_executor_factory):
    M, N, K, tb, b2d, batches, alpha, with_bias = case
    if b2d:
        a = rand(2, M // 2, K) if M % 2 == 0 else rand(M, K)
        b = rand(N, K) if tb else rand(K, N)
        out = list(a.shape[:-1]) + [N]
    else:
        a = rand(batches, M, K)
        b = rand(batches, N, K) if tb else rand(batches, K, N)
        out = [batches, M, N]
    b *= 0.05
    if with_bias:
        ins, op, extra = [a, b, rand(N)], OP["MATMUL_ADD"], [K, tb, b2d]
    else:
        ins, op, extra = [a, b], OP["MATMUL"], [K, tb, b2d, fb(alpha) if alpha != 1.0 else 0]
    got, ref = run_both(gpu_executor_factory, single_node_program(op, ins, out, extra))
    np.testing.assert_allclose(got, ref, atol=1e-4, rtol=1e-3)


@pytest.mark.parametrize("M,N,K", [(512, 512, 8192), (100, 256, 4096)])
def test_matmul_accuracy_vs_fp64(M, N, K, gpu_executor_factory):
    """Error of the tensor-core GEMM against an fp64 product, per sqrt(K) of
    unit-variance terms: the split scheme's ~2^-19 per product keeps it
    under 1e-5 (OpenBLAS sgemm sits near 5e-7 here)."""
    rng = np.random.default_rng(7)
    a = rng.standard_normal((M, K), dtype=np.float32)
    b = rng.standard_normal((N, K), dtype=np.float32)
    prog = single_node_program(OP["MATMUL"], [a, b], [M, N], [K, 1, 1, 0])
    got, _ = run_both(gpu_executor_factory, prog)
    exact = a.astype(np.float64) @ b.astype(np.float64).T
    err = np.abs(got.astype(np.float64) - exact).max() / np.sqrt(K)
    assert err < 1e-5, err


ATT_CASES = [
    # (B, Hq, Hkv, S, D, causal, mask)
    (1, 4, 4, 32, 16, 0, False),
    (2, 2, 2, 100, 64, 1, False),
    (1, 4, 2, 300, 128, 1, False),
    (1, 2, 2, 300, 64, 0, False),
    (2, 2, 1, 64, 128, 0, False),
    (1, 2, 2, 48, 80, 0, True),
    (1, 3, 3, 513, 64, 1, False),
    (1, 2, 2, 1024, 128, 1, False),
    (2, 4, 2, 256, 64, 0, False),
    (1, 2, 2, 132, 64, 1, False),
    (1, 4, 1, 640, 128, 0, False),
]


@pytest.mark.parametrize("case", ATT_CASES, ids=lambda c: "-".join(map(str, c)))
def test_attention(case, gpu_executor_factory):
    B, Hq, Hkv, S, D, causal, with_mask = case
    q, k, v = rand(B, Hq, S, D), rand(B, Hkv, S, D), rand(B, Hkv, S, D)
    ins = [q, k, v]
    if with_mask:
        m = np.where(rng.random((B, Hq, S, S)) < 0.2, -np.inf, 0).astype(np.float32)
        m[..., 0] = 0.0
        ins.append(m)
    scratch = B * Hq * (128 * 256 if S > 256 else S * S) * 4
    extra = [S, D, causal, 1 if with_mask else 0, Hq // Hkv]
    prog = single_node_program(OP["ATTENTION"], ins, [B, Hq, S, D], extra, scratch_bytes=scratch)
    got, ref = run_both(gpu_executor_factory, prog)
    np.testing.assert_allclose(got, ref, atol=1e-4, rtol=1e-3)


def test_transpose_nd_and_2d(gpu_executor_factory):
    x = rand(2, 5, 3, 16)   # swap dims 1 and 2 -> [2, 3, 5, 16]
    got, ref = run_both(gpu_executor_factory,
                        single_node_program(OP["TRANSPOSE"], [x], [2, 3, 5, 16], [2, 5, 1, 3, 16]))
    np.testing.assert_array_equal(got, ref)
    np.testing.assert_array_equal(got, np.swapaxes(x, 1, 2))
    y = rand(37, 50)
    got, ref = run_both(gpu_executor_factory, single_node_program(OP["TRANSPOSE"], [y], [50, 37], [37, 50]))
    np.testing.assert_array_equal(got, y.T)


@pytest.mark.parametrize("inner_odd", [False, True])
def test_slice_and_cat(inner_odd, gpu_executor_factory):
    w = 7 if inner_odd else 64
    x = rand(3, 10, 3 * w)
    got, ref = run_both(gpu_executor_factory,
                        single_node_program(OP["SLICE"], [x], [3, 10, w], [30, 3 * w, w, w, 1]))
    np.testing.assert_array_equal(got, x[..., w:2 * w])
    a, b = rand(2, 3, 4, w), rand(2, 3, 4, w + 1)
    got, ref = run_both(gpu_executor_factory,
                        single_node_program(OP["CAT"], [a, b], [2, 3, 4, 2 * w + 1], [3, w, w + 1]))
    np.testing.assert_array_equal(got, np.concatenate([a, b], axis=3))


def test_layout_runs_long_short_and_scalar(gpu_executor_factory):
    """Run-based layout copies: few long runs (cut into pieces across the
    grid), runs shorter than a warp, and 4-byte units with inner == 1."""
    a, b = rand(1, 300001), rand(1, 70000)       # CAT along dim 1: one run per input
    got, ref = run_both(gpu_executor_factory,
                        single_node_program(OP["CAT"], [a, b], [1, 370001], [1, 300001, 70000]))
    np.testing.assert_array_equal(got, np.concatenate([a, b], axis=1))
    x = rand(2, 200003)                           # SLICE: two long rows, odd start
    got, ref = run_both(gpu_executor_factory,
                        single_node_program(OP["SLICE"], [x], [2, 150000], [2, 200003, 17, 150000, 1]))
    np.testing.assert_array_equal(got, x[:, 17:17 + 150000])
    y = rand(3, 7, 5, 11)                         # TRANSPOSE dims 1, 2 with inner 11 (scalar units)
    got, ref = run_both(gpu_executor_factory,
                        single_node_program(OP["TRANSPOSE"], [y], [3, 5, 7, 11], [3, 7, 1, 5, 11]))
    np.testing.assert_array_equal(got, np.swapaxes(y, 1, 2))
    z = rand(4, 64, 8, 128)                       # head split [B, S, H, D] -> [B, H, S, D]
    got, ref = run_both(gpu_executor_factory,
                        single_node_program(OP["TRANSPOSE"], [z], [4, 8, 64, 128], [4, 64, 1, 8, 128]))
    np.testing.assert_array_equal(got, np.swapaxes(z, 1, 2))
    u = rand(6, 9, 4)                             # TRANSPOSE dims 0, 2 with inner 1
    got, ref = run_both(gpu_executor_factory,
                        single_node_program(OP["TRANSPOSE"], [u], [4, 9, 6], [1, 6, 9, 4, 1]))
    np.testing.assert_array_equal(got, np.swapaxes(u, 0, 2))


def test_reshape_copy_and_embedding(gpu_executor_factory):
    x = rand(4, 6)
    got, ref = run_both(gpu_executor_factory, single_node_program(OP["RESHAPE"], [x], [24], []))
    np.testing.assert_array_equal(got, x.reshape(-1))
    ids = np.array([[3, 0, 7, 7]], dtype=np.int64)
    table = rand(10, 12)
    got, ref = run_both(gpu_executor_factory,
                        single_node_program(OP["EMBEDDING"], [ids, table], [1, 4, 12], [12]))
    np.testing.assert_array_equal(got, table[ids[0]][None])


@pytest.mark.gpu
@pytest.mark.parametrize("env", [
    {"RT_GEMM_3XTF32": "1"},                       # three tf32 MMAs (hi.hi + hi.lo + lo.hi)
    {"RT_GEMM_SCHEME": "cross"},                   # tf32 hi.hi + bf16 cross terms
    {"RT_GEMM_SCHEME": "cross", "RT_GEMM_PAIR": "0"},
    {"RT_GEMM_SCHEME": "cross", "RT_GEMM_TMA_STORE": "1"},
    {"RT_GEMM_PAIR": "0"},                         # one-CTA kernel everywhere
    {"RT_GEMM_PAIR": "0", "RT_GEMM_3XTF32": "1"},
    {"RT_GEMM_TMA_STORE": "1"},                    # C through shared memory and TMA stores
    {"RT_GEMM_TMA_STORE": "1", "RT_GEMM_3XTF32": "1"},
], ids=lambda e: ",".join(f"{k}={v}" for k, v in e.items()))
def test_matmul_variants(env):
    """The GEMM variants selected by environment switches (read once per
    process) pass the same matmul cases, each in a fresh process."""
    import os
    import subprocess
    import sys
    full = dict(os.environ, **env)
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-m", "gpu", "-p", "no:cacheprovider",
                        __file__, "-k", "test_matmul and not variants"],
                       env=full, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]


@pytest.mark.gpu
@pytest.mark.parametrize("env", [{"RT_ATTN_3XTF32": "1"}, {"RT_ATTN_SCHEME": "cross"}],
                         ids=lambda e: ",".join(f"{k}={v}" for k, v in e.items()))
def test_attention_scheme_variants(env):
    """The other attention operand forms (three tf32 MMAs; tf32 + bf16 cross
    terms -- read once per process) pass the same attention cases, each in a
    fresh process."""
    import os
    import subprocess
    import sys
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-m", "gpu", "-p", "no:cacheprovider",
                        __file__, "-k", "test_attention and not variant"],
                       env=dict(os.environ, **env), capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]


@pytest.mark.parametrize("M,N,K,splitk", [(1024, 512, 256, False), (512, 256, 2048, True)])
def test_matmul_add_misaligned_output_and_bias(M, N, K, splitk, gpu_executor_factory):
    """The planner's first-fit offsets are raw byte counts (runtime/planner.py:
    470-477): a MATMUL_ADD whose output and bias start 4 bytes past a 16-byte
    boundary must run on the tensor-core kernel's scalar-store path and match
    the oracle (the second shape takes split-K)."""
    from lbr_b200.program import ConstSpec, ProgNode, Program, Ref
    a = rand(M, K)
    w = rand(N, K) * 0.05
    bias_padded = rand(N + 1)
    consts = {"a": ConstSpec("a", a.shape, "float32", {"kind": "stored"}),
              "w": ConstSpec("w", w.shape, "float32", {"kind": "stored"}),
              "bias": ConstSpec("bias", bias_padded.shape, "float32", {"kind": "stored"})}
    node = ProgNode(OP["MATMUL_ADD"], [Ref("const", "a", 0), Ref("const", "w", 0), Ref("const", "bias", 4)],
                    Ref("arena", None, 4), [M, N], 4, [K, 1, 1])
    prog = Program("misaligned", {}, M * N * 4 + 256, {},
                   {"y": {"shape": [M, N], "dtype": "float32", "ref": Ref("arena", None, 4)}},
                   consts, [node], {"a": a, "w": w, "bias": bias_padded})
    got, ref = run_both(gpu_executor_factory, prog)
    np.testing.assert_allclose(got, ref, atol=1e-4, rtol=1e-3)
    exact = a.astype(np.float64) @ w.astype(np.float64).T + bias_padded[1:]
    np.testing.assert_allclose(got, exact, atol=1e-4, rtol=1e-3)
