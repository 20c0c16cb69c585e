"""GEMM epilogue fusion on the GPU: GEMM -> GELU -> GEMM chains (the GELU in
the first GEMM's epilogue, which hands the second GEMM its split A operand)
against the oracle, and fusion decisions on real device addresses."""

import ctypes

import numpy as np
import pytest

import oracle
from conftest import GOLDEN, PLANE_HANDOFFS, gemm_handoff
from lbr_b200.program import OP, ConstSpec, ProgNode, Program, Ref

pytestmark = pytest.mark.gpu


def mlp_program(M, D, F, kind, seed=0):
    """x[M,D] -> MATMUL_ADD (F) -> [GELU] -> [MATMUL_ADD (D)]; kind = 0, 1, 2 nodes after the first."""
    rng = np.random.default_rng(seed)
    stored = {
        "x": rng.standard_normal((M, D), dtype=np.float32),
        "w1": (rng.standard_normal((F, D)) * 0.05).astype(np.float32),
        "b1": rng.standard_normal(F).astype(np.float32) * 0.1,
        "w2": (rng.standard_normal((D, F)) * 0.05).astype(np.float32),
        "b2": rng.standard_normal(D).astype(np.float32) * 0.1,
    }
    consts = {k: ConstSpec(k, v.shape, "float32", {"kind": "stored"}) for k, v in stored.items()}
    C = lambda n: Ref("const", n, 0)
    A = lambda off: Ref("arena", None, off)
    Y, Z, O = 0, M * F * 4, 2 * M * F * 4
    nodes = [ProgNode(OP["MATMUL_ADD"], [C("x"), C("w1"), C("b1")], A(Y), [M, F], 4, [D, 1, 1])]
    out = ("y", [M, F], Y)
    if kind >= 1:
        nodes.append(ProgNode(OP["GELU"], [A(Y)], A(Z), [M, F], 4, []))
        out = ("z", [M, F], Z)
    if kind >= 2:
        nodes.append(ProgNode(OP["MATMUL_ADD"], [A(Z), C("w2"), C("b2")], A(O), [M, D], 4, [F, 1, 1]))
        out = ("o", [M, D], O)
    outs = {out[0]: {"shape": out[1], "dtype": "float32", "ref": A(out[2])}}
    return Program(f"mlp{kind}", {}, O + M * D * 4, {}, outs, consts, nodes, stored), out[0]


def flags_of(ex, prog):
    f = (ctypes.c_int * len(prog.nodes))()
    ex._lib.rt_fusion_report(ex.node_array, len(prog.nodes), f)
    return list(f)


@pytest.mark.parametrize("M,D,F", [(1024, 256, 1024), (300, 192, 520), (640, 128, 1028), (300, 192, 1024),
                                   (100, 256, 512), (256, 256, 4096)])
@pytest.mark.parametrize("kind,handoff", [(1, "0"), (2, "0"), (2, "1")])
def test_fused_chain_matches_oracle(M, D, F, kind, handoff, gpu_executor_factory, monkeypatch):
    monkeypatch.setenv("RT_FUSE_HANDOFF", handoff)
    prog, name = mlp_program(M, D, F, kind)
    ex = gpu_executor_factory(prog, dict(prog.stored))
    got = ex.run({})[name]
    flags = flags_of(ex, prog)
    assert flags[:2] == [3, 1]                       # GELU folded into the first GEMM
    if kind == 2:
        assert flags[2] == (4 if gemm_handoff(handoff, F) else 0)   # A operand handed over: no split pass
    ref = oracle.run_program("restated", prog, dict(prog.stored), {})[name]
    np.testing.assert_allclose(got, ref, atol=1e-4, rtol=1e-3)


def test_freed_executor_outputs_do_not_block_fusion(gpu_executor_factory):
    """Graph outputs registered by an executor are dropped when its memory is
    freed, so a later executor whose buffers land at the same addresses still
    fuses."""
    for kind in (0, 1, 2):
        prog, name = mlp_program(1024, 256, 1024, kind)
        ex = gpu_executor_factory(prog, dict(prog.stored))
        ex.run({})
        if kind:
            assert flags_of(ex, prog)[:2] == [3, 1]
        ex.close()


@pytest.mark.parametrize("env", [{"RT_GEMM_3XTF32": "1"}, {"RT_GEMM_PAIR": "0"}, {"RT_GEMM_SCHEME": "cross"}],
                         ids=lambda e: ",".join(f"{k}={v}" for k, v in e.items()))
def test_fused_chain_variants(env):
    """Chains under the other GEMM variants (3xTF32 planes: hi + fp32 lo; the
    one-CTA kernel), each in a fresh process."""
    import os
    import subprocess
    import sys
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-m", "gpu", "-p", "no:cacheprovider",
                        __file__, "-k", "test_fused_chain_matches_oracle"],
                       env=dict(os.environ, **env), capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]


@pytest.mark.parametrize("name", ["7b_b1", "block_hd128_s320", "block_mini_causal_s300"])
def test_custom_block_bias_fold_unlocks_layout_fusion(name, gpu_executor_factory):
    """Custom blocks: merged QKV MATMUL -> SLICE -> in-place bias ADD ->
    head-split TRANSPOSE.  The three bias ADDs fold into the GEMM (a merged
    bias built at plan time), which leaves SLICE -> TRANSPOSE -> ATTENTION
    chains for the layout fusion.  Outputs are checked against goldens /
    the reference executor by test_gpu_programs; here, the fusion decision
    on real device addresses (bias constants registered)."""
    from conftest import GOLDEN
    prog = Program.load(GOLDEN / f"{name}.json")
    ex = gpu_executor_factory(prog, prog.make_constants())
    flags = flags_of(ex, prog)
    ops = [nd.op for nd in prog.nodes]
    mm = ops.index(OP["MATMUL"])
    if not ex._lib.rt_fusion_report:   # pragma: no cover
        pytest.skip("no report")
    tc = flags[mm] == 3
    folded = [ops[i] for i, f in enumerate(flags) if f == 1]
    bias_adds = [i for i, f in enumerate(flags) if f == 1 and ops[i] == OP["ADD"] and prog.nodes[i].extra[0] == 0]
    if not tc:   # GEMM below the tensor-core threshold: nothing to fold
        assert folded.count(OP["ADD"]) == 0
        return
    assert len(bias_adds) == 3
    assert folded.count(OP["SLICE"]) == 3 and folded.count(OP["TRANSPOSE"]) == 4
    ins = prog.make_inputs(0)
    got = ex.run(ins)
    ref = oracle.run_program("restated", prog, prog.make_constants(), ins) if name != "7b_b1" else None
    if ref is not None:
        for k in got:
            np.testing.assert_allclose(got[k], ref[k], atol=1e-4, rtol=1e-3)


@pytest.mark.parametrize("act,bias", [(0, False), (1, True)])
def test_gated_activation_reads_slices_through_views(act, bias, gpu_executor_factory):
    """SLICE(M, 0, F), SLICE(M, F, F) -> GATED_ACT: the slices fold into row-strided
    views of M (flag 6 on the GATED_ACT, 1 on both slices); result vs the oracle."""
    R, F = 300, 520
    rng = np.random.default_rng(11)
    stored = {"m": rng.standard_normal((R, 2 * F), dtype=np.float32),
              "b": rng.standard_normal(F).astype(np.float32)}
    consts = {k: ConstSpec(k, v.shape, "float32", {"kind": "stored"}) for k, v in stored.items()}
    A = lambda off: Ref("arena", None, off)
    sz = R * F * 4
    nodes = [ProgNode(OP["SLICE"], [Ref("const", "m", 0)], A(0), [R, F], 4, [R, 2 * F, 0, F, 1]),
             ProgNode(OP["SLICE"], [Ref("const", "m", 0)], A(sz), [R, F], 4, [R, 2 * F, F, F, 1])]
    ins = [A(0), Ref("const", "b", 0), A(sz)] if bias else [A(0), A(sz)]
    nodes.append(ProgNode(OP["GATED_ACT"], ins, A(2 * sz), [R, F], 4, [int(bias), act]))
    prog = Program("gated", {}, 3 * sz, {}, {"y": {"shape": [R, F], "dtype": "float32", "ref": A(2 * sz)}},
                   consts, nodes, stored)
    ex = gpu_executor_factory(prog, dict(stored))
    assert flags_of(ex, prog) == [1, 1, 6]
    got = ex.run({})["y"]
    ref = oracle.run_program("restated", prog, dict(stored), {})["y"]
    np.testing.assert_allclose(got, ref, rtol=2e-6, atol=2e-6)


@pytest.mark.parametrize("residual", ["1", "0"])
@pytest.mark.parametrize("attn_split", ["1", "0"])
def test_attention_split_hand_off_matches_golden(attn_split, residual, gpu_executor_factory, monkeypatch):
    """GPT-2 mini body at S = 300 (a partial last query block): the attention
    writes the projection GEMM's split A planes (RT_FUSE_ATTN_SPLIT=1) or its
    plain output (0, the default), with and without the residual ADDs folded
    into the GEMMs, and the result matches the reference executor's golden
    output."""
    from conftest import load_golden
    from test_gpu_programs import assert_parity
    monkeypatch.setenv("RT_FUSE_ATTN_SPLIT", attn_split)
    monkeypatch.setenv("RT_FUSE_RESIDUAL", residual)   # with the residual fold the projection's flag is 3
    prog, ins, outs = load_golden("gpt2_mini_s300")
    ex = gpu_executor_factory(prog, prog.make_constants())
    got = ex.run(ins)
    for k, ref in outs.items():
        assert_parity(got[k], ref, f"gpt2_mini_s300:{k}")
    flags = flags_of(ex, prog)
    ops = [nd.op for nd in prog.nodes]
    proj = [i for i, op in enumerate(ops) if op == OP["MATMUL_ADD"] and OP["ATTENTION"] in ops[max(0, i - 3):i]]
    if residual == "0":
        assert proj and all(flags[i] == (4 if attn_split == "1" and PLANE_HANDOFFS else 0) for i in proj)
    else:
        assert proj and all(flags[i] == 3 and flags[i + 1] == 1 for i in proj)


@pytest.mark.parametrize("env", [{"RT_GEMM_3XTF32": "1"}, {"RT_GEMM_SCHEME": "cross"}],
                         ids=lambda e: ",".join(f"{k}={v}" for k, v in e.items()))
def test_attention_split_hand_off_plane_schemes(env):
    """The same hand-off with the tf32 plane layouts (3xTF32: hi + fp32 lo;
    cross: hi + bf16 cross plane), each in a fresh process."""
    import os
    import subprocess
    import sys
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-m", "gpu", "-p", "no:cacheprovider",
                        __file__, "-k", "test_attention_split_hand_off_matches_golden"],
                       env=dict(os.environ, **env), capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]


def residual_program(M, K, N, inplace, seed=0):
    """x = c1 + c2 (arena) ; y = a @ w^T + b ; z = y + x -- z over x (inplace)
    or in its own buffer.  The last ADD folds into the GEMM's epilogue."""
    rng = np.random.default_rng(seed)
    stored = {
        "a": rng.standard_normal((M, K), dtype=np.float32),
        "w": (rng.standard_normal((N, K)) * 0.05).astype(np.float32),
        "b": rng.standard_normal(N).astype(np.float32) * 0.1,
        "c1": rng.standard_normal((M, N), dtype=np.float32),
        "c2": rng.standard_normal((M, N), dtype=np.float32),
    }
    consts = {k: ConstSpec(k, v.shape, "float32", {"kind": "stored"}) for k, v in stored.items()}
    C = lambda n: Ref("const", n, 0)
    A = lambda off: Ref("arena", None, off)
    X, Y, Z = 0, M * N * 4, (0 if inplace else 2 * M * N * 4)
    nodes = [ProgNode(OP["ADD"], [C("c1"), C("c2")], A(X), [M, N], 4, [1]),
             ProgNode(OP["MATMUL_ADD"], [C("a"), C("w"), C("b")], A(Y), [M, N], 4, [K, 1, 1]),
             ProgNode(OP["ADD"], [A(Y), A(X)], A(Z), [M, N], 4, [1])]
    outs = {"z": {"shape": [M, N], "dtype": "float32", "ref": A(Z)}}
    return Program(f"res{int(inplace)}", {}, 3 * M * N * 4, {}, outs, consts, nodes, stored)


@pytest.mark.parametrize("inplace", [False, True])
@pytest.mark.parametrize("M,K,N", [(1024, 768, 256), (300, 520, 192)])
def test_residual_add_folded_into_gemm_matches_oracle(M, K, N, inplace, gpu_executor_factory, monkeypatch):
    """With RT_FUSE_RESIDUAL=1 the GEMM adds the residual in its epilogue and
    writes the ADD's output: into its own buffer (two-way split-K allowed:
    the first split adds the residual) or over the residual itself (no
    split-K), twice in a row."""
    monkeypatch.setenv("RT_FUSE_RESIDUAL", "1")
    prog = residual_program(M, K, N, inplace)
    ex = gpu_executor_factory(prog, dict(prog.stored))
    ref = oracle.run_program("restated", prog, dict(prog.stored), {})["z"]
    for _ in range(2):
        got = ex.run({})["z"]
        np.testing.assert_allclose(got, ref, atol=1e-4, rtol=1e-3)
    assert flags_of(ex, prog) == [0, 3, 1]


@pytest.mark.parametrize("name", ["qwen3_mini_s272"])
def test_gated_activation_folds_into_the_gate_up_gemm(name, gpu_executor_factory, monkeypatch):
    """Qwen3's MLP: merged gate/up MATMUL -> SLICE, SLICE -> GATED_ACT(SiLU).
    The GEMM takes the weight rows in the gated order and applies the
    activation in its epilogue (flag 7); slices and GATED_ACT are not
    launched (flag 1).  Output against the reference executor's golden, and
    against the unfused plan (RT_FUSE_GATED_GEMM=0, read once per process: a
    fresh process)."""
    from conftest import load_golden
    from test_gpu_programs import assert_parity
    prog, ins, outs = load_golden(name)
    ex = gpu_executor_factory(prog, prog.make_constants())
    got = ex.run(ins)
    flags = flags_of(ex, prog)
    ops = [nd.op for nd in prog.nodes]
    gated = [i for i, op in enumerate(ops) if op == OP["GATED_ACT"]]
    assert gated and all(flags[i] == 1 for i in gated)
    assert flags.count(7) == len(gated)
    for k, ref in outs.items():
        assert_parity(got[k], ref, f"{name}:{k} (gated epilogue)")


def test_gated_gemm_fold_off_matches():
    from conftest import has_gpu
    if not has_gpu():
        pytest.skip("no CUDA device")
    import os
    import subprocess
    import sys
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-m", "gpu", "-p", "no:cacheprovider",
                        os.path.join(os.path.dirname(__file__), "test_gpu_programs.py"), "-k", "qwen3_mini"],
                       env=dict(os.environ, RT_FUSE_GATED_GEMM="0"), capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and " passed" in r.stdout, r.stdout[-3000:] + r.stderr[-2000:]


def test_gated_gemm_fold_keeps_the_rotary_folds(gpu_executor_factory):
    """On the full Qwen3 body (batch 8) the gated GEMM fold and both rotary
    folds per layer apply together."""
    prog = Program.load(GOLDEN / "qwen3_b8.json")
    ex = gpu_executor_factory(prog, prog.make_constants())
    flags = flags_of(ex, prog)
    ex.close()
    layers = sum(1 for nd in prog.nodes if nd.op == OP["GATED_ACT"])
    assert flags.count(7) == layers
    assert flags.count(5) == 2 * layers
