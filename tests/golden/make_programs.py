"""Generate the committed program fixtures (test infrastructure).

Run in a container that has the reference tree (default: `reference` beside the repo,
override with REF_ROOT) and the oracle build of its C executor
(``make -C oracle ref``):

    python tests/golden/make_programs.py [--only NAME ...]

For every configuration it builds the model with seeded weights, runs the
reference's own pipeline -- ``export_model`` -> ``run_pipeline`` -> ``plan``
(runtime/exporter/torch/exporter.py:28, runtime/passes/passes.py:44,
runtime/planner.py:500) -- and writes ``<name>.json`` (+ ``<name>.npz`` for
verbatim constants): the planned node array in symbolic form.  The lowering
is checked field for field against the node array the reference
``CompiledExecutor.compile`` builds (runtime/executor/compiled.py:34-70).

For the small ``mini`` programs and the toy block it also runs the reference
C executor (oracle/_ref/libexecutor.so) on seeded inputs and stores the
outputs in ``<name>.golden.npz``; for the toy block, whose weights are
stored verbatim, the PyTorch model's own output is stored beside it.
"""

from __future__ import annotations

import argparse
import ctypes
import importlib.util
import math
import os
import sys
import time
from pathlib import Path

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
REF_ROOT = Path(os.environ.get("REF_ROOT") or REPO.parent / "reference")
sys.path.insert(0, str(REF_ROOT))

_spec = importlib.util.spec_from_file_location(
    "lbr_b200", REPO / "lets-build-a-runtime_b200" / "__init__.py",
    submodule_search_locations=[str(REPO / "lets-build-a-runtime_b200")])
lbr = importlib.util.module_from_spec(_spec)
sys.modules["lbr_b200"] = lbr
_spec.loader.exec_module(lbr)
from lbr_b200.copnode import COpNode, HostBinding          # noqa: E402
from lbr_b200.lower import program_from_plan                # noqa: E402
from lbr_b200.program import Ref                            # noqa: E402

import runtime.executor.common as ref_common                # noqa: E402
import runtime.executor.compiled as ref_compiled            # noqa: E402
from runtime.exporter import export_model                   # noqa: E402
from runtime.passes import run_pipeline                     # noqa: E402
from runtime.planner import plan as ref_plan                # noqa: E402
from runtime.ops import resolve_graph                       # noqa: E402

REF_LIB = ctypes.CDLL(str(REPO / "oracle" / "_ref" / "libexecutor.so"))
REF_LIB.execute.argtypes = [ctypes.POINTER(ref_common.COpNode), ctypes.c_int]
REF_LIB.execute.restype = None
ref_common._c_executor_lib = REF_LIB
ref_compiled._c_executor_lib = REF_LIB


# ---------------------------------------------------------------- models
class CustomBlock(nn.Module):
    """Pre-LN block with SDPA attention (tests/conftest.py:118-148 of the
    reference) with tanh-GELU in the FFN and an optional causal flag."""

    def __init__(self, d, h, ff, causal):
        super().__init__()
        self.h, self.dk, self.causal = h, d // h, causal
        self.ln1 = nn.LayerNorm(d)
        self.wq, self.wk, self.wv, self.wo = (nn.Linear(d, d) for _ in range(4))
        self.ln2 = nn.LayerNorm(d)
        self.ffn1 = nn.Linear(d, ff)
        self.ffn2 = nn.Linear(ff, d)
        for m in self.modules():
            if isinstance(m, nn.Linear):
                nn.init.normal_(m.weight, 0.0, 0.02)
                nn.init.zeros_(m.bias)

    def forward(self, x):
        B, S, D = x.shape
        h = self.ln1(x)
        q = self.wq(h).reshape(B, S, self.h, self.dk).permute(0, 2, 1, 3)
        k = self.wk(h).reshape(B, S, self.h, self.dk).permute(0, 2, 1, 3)
        v = self.wv(h).reshape(B, S, self.h, self.dk).permute(0, 2, 1, 3)
        a = F.scaled_dot_product_attention(q, k, v, is_causal=self.causal)
        a = a.permute(0, 2, 1, 3).reshape(B, S, D)
        x = x + self.wo(a)
        return x + self.ffn2(F.gelu(self.ffn1(self.ln2(x)), approximate="tanh"))


class GPT2Body(nn.Module):
    """GPT-2 blocks + final LayerNorm (reference tests/test_end_to_end.py:386-397),
    tolerant of blocks that return a tensor instead of a tuple."""

    def __init__(self, n_layer, n_head, n_embd):
        super().__init__()
        from transformers import GPT2Config, GPT2LMHeadModel
        cfg = GPT2Config(n_layer=n_layer, n_head=n_head, n_embd=n_embd,
                         layer_norm_epsilon=1e-5, vocab_size=256)
        full = GPT2LMHeadModel(cfg).eval()
        self.h = full.transformer.h
        self.ln_f = full.transformer.ln_f

    def forward(self, x):
        for blk in self.h:
            o = blk(x)
            x = o[0] if isinstance(o, tuple) else o
        return self.ln_f(x)


class Qwen3Body(nn.Module):
    def __init__(self, hidden, inter, layers, heads, kv_heads, head_dim):
        super().__init__()
        from transformers import Qwen3Config, Qwen3Model
        cfg = Qwen3Config(hidden_size=hidden, intermediate_size=inter,
                          num_hidden_layers=layers, num_attention_heads=heads,
                          num_key_value_heads=kv_heads, head_dim=head_dim,
                          rope_theta=1e6, rms_norm_eps=1e-6, attention_bias=False,
                          vocab_size=256, max_position_embeddings=40960)
        self.m = Qwen3Model(cfg).eval()

    def forward(self, x):
        return self.m(inputs_embeds=x, use_cache=False).last_hidden_state


# name -> (builder, batch, seq, d_model, mini?)
def _configs():
    c = {}
    c["toy"] = (lambda: CustomBlock(64, 4, 256, False), 1, 32, 64, True)
    for b in (1, 2, 4, 8):
        c[f"gpt2_b{b}"] = (lambda: GPT2Body(2, 12, 768), b, 1024, 768, False)
        c[f"qwen3_b{b}"] = (lambda: Qwen3Body(1024, 3072, 2, 16, 8, 128), b, 1024, 1024, False)
        c[f"7b_b{b}"] = (lambda: CustomBlock(4096, 32, 16384, False), b, 1024, 4096, False)
        c[f"1b8k_b{b}"] = (lambda: CustomBlock(2048, 16, 8192, True), b, 8192, 2048, False)
    # small programs with golden outputs (flash path: S > 256, ragged tiles)
    c["gpt2_mini_s300"] = (lambda: GPT2Body(2, 2, 128), 2, 300, 128, True)
    c["gpt2_mini_s64"] = (lambda: GPT2Body(2, 2, 128), 2, 64, 128, True)
    c["gpt2_mini_s64_b1"] = (lambda: GPT2Body(2, 2, 128), 1, 64, 128, False)   # one shard of the batch above
    c["qwen3_mini_s272"] = (lambda: Qwen3Body(256, 512, 2, 4, 2, 128), 1, 272, 256, True)
    c["block_mini_causal_s300"] = (lambda: CustomBlock(128, 2, 512, True), 2, 300, 128, True)
    c["block_mini_s260"] = (lambda: CustomBlock(128, 2, 512, False), 1, 260, 128, True)
    c["block_hd128_s320"] = (lambda: CustomBlock(256, 2, 1024, False), 1, 320, 256, True)
    c["block_hd128_causal_s100"] = (lambda: CustomBlock(256, 2, 1024, True), 1, 100, 256, True)
    return c


def _check_against_reference_compile(prog, ep, graph):
    """Field-by-field comparison with the reference CompiledExecutor's array."""
    ex = ref_compiled.CompiledExecutor()
    ex.compile(ep)
    arena = ex._arena
    a0, a1 = arena.ctypes.data, arena.ctypes.data + arena.nbytes
    consts = [(n, graph.tensors[n].buffer) for n in graph.constants]

    def sym(ptr):
        if ptr is None or ptr == 0:
            return ("input",)
        if a0 <= ptr < a1:
            return ("arena", ptr - a0)
        for n, b in consts:
            if b is not None and b.ctypes.data <= ptr < b.ctypes.data + b.nbytes:
                return ("const", n, ptr - b.ctypes.data)
        raise AssertionError(f"pointer {ptr:#x} not in arena or constants")

    def mine(r: Ref):
        if r.kind == "input":
            return ("input",)
        if r.kind == "arena":
            return ("arena", r.offset)
        # constants may share one buffer (e.g. a rotary table used by two
        # layers): compare the addresses they resolve to
        return sym(graph.tensors[r.name].buffer.ctypes.data + r.offset)

    assert ex._n_nodes == len(prog.nodes), (ex._n_nodes, len(prog.nodes))
    for i, pn in enumerate(prog.nodes):
        cn = ex._nodes[i]
        assert cn.op == pn.op and cn.n_inputs == len(pn.inputs), i
        for j, r in enumerate(pn.inputs):
            assert sym(cn.inputs[j]) == mine(r), (i, j, sym(cn.inputs[j]), r)
        assert sym(cn.output) == mine(pn.output), i
        assert list(cn.out_shape[:cn.n_dims]) == pn.out_shape, i
        assert cn.elem_size == pn.elem_size, i
        assert list(cn.extra[:len(pn.extra)]) == pn.extra, i
        assert all(v == 0 for v in cn.extra[len(pn.extra):]), i
    return ex


def _run_ref(prog, seed=0):
    consts = prog.make_constants(seed)
    ins = prog.make_inputs(seed)
    hb = HostBinding(prog, consts, ins)
    REF_LIB.execute(ctypes.cast(hb.nodes, ctypes.POINTER(ref_common.COpNode)), len(prog.nodes))
    return ins, hb.outputs()


def build(name, spec):
    builder, B, S, D, mini = spec
    torch.manual_seed(0)
    model = builder().eval()
    x = torch.randn(B, S, D)
    t0 = time.time()
    graph = export_model(model, (x,))
    run_pipeline(graph)
    ep = ref_plan(graph)
    meta = {"config": name, "batch": B, "seq_len": S, "d_model": D,
            "generator": "tests/golden/make_programs.py"}
    prog = program_from_plan(ep, name, meta, store_all=(name == "toy"))
    ex = _check_against_reference_compile(prog, ep, graph)
    prog.save(HERE / f"{name}.json")
    msg = f"{name}: {len(prog.nodes)} nodes, arena {prog.arena_size/2**20:.1f} MiB, " \
          f"consts {prog.constant_bytes()/2**20:.1f} MiB, {time.time()-t0:.1f}s"
    if mini:
        # regenerated weights: reference C executor on seeded inputs
        ins, outs = _run_ref(prog)
        gold = {f"in__{k}": v for k, v in ins.items()}
        gold.update({f"out__{k}": v for k, v in outs.items()})
        if name == "toy":
            # verbatim weights: the PyTorch model itself is a second witness
            with torch.no_grad():
                tout = model(torch.from_numpy(ins[graph.inputs[0]])).numpy()
            gold[f"torch__{graph.outputs[0]}"] = tout
            msg += f", ref-vs-torch {np.abs(tout - outs[graph.outputs[0]]).max():.2e}"
        np.savez_compressed(HERE / f"{name}.golden.npz", **gold)
    print(msg, flush=True)
    del ex, graph, model


DYN_SEQ = (64, 128, 200, 384)


def build_dynamic():
    """One causal block exported ONCE with a symbolic sequence length S
    (the reference's dynamic-shape path, tests/test_dynamic_shapes.py), then
    ``resolve_graph`` + ``plan`` per binding: dyn_s<S>.json share constant
    names and shapes, as the reference's rebind shares weight arrays."""
    torch.manual_seed(0)
    model = CustomBlock(256, 4, 1024, True).eval()
    x = torch.randn(1, 32, 256)
    graph = export_model(model, (x,), dynamic_dims={"S": [("x", 1)]})
    run_pipeline(graph)
    shapes = None
    for S in DYN_SEQ:
        t0 = time.time()
        resolved = resolve_graph(graph, {"S": S})
        ep = ref_plan(resolved)
        name = f"dyn_s{S}"
        meta = {"config": name, "batch": 1, "seq_len": S, "d_model": 256, "bindings": {"S": S},
                "generator": "tests/golden/make_programs.py"}
        prog = program_from_plan(ep, name, meta)
        ex = _check_against_reference_compile(prog, ep, resolved)
        cs = {n: (c.shape, c.dtype) for n, c in prog.constants.items()}
        assert shapes is None or cs == shapes, "constants differ between bindings"
        shapes = cs
        prog.save(HERE / f"{name}.json")
        print(f"{name}: {len(prog.nodes)} nodes, arena {prog.arena_size/2**20:.1f} MiB, "
              f"{time.time()-t0:.1f}s", flush=True)
        del ex


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", nargs="*")
    args = ap.parse_args()
    for name, spec in _configs().items():
        if args.only and not any(name.startswith(o) for o in args.only):
            continue
        build(name, spec)
    if not args.only or any(o.startswith("dyn") for o in args.only):
        build_dynamic()


if __name__ == "__main__":
    main()
