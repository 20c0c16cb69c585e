"""Dynamic-shape rebind (session.py), host logic: the reference Session
pipeline (export -> passes -> resolve_graph -> plan) with the GPU executor
replaced by a recorder.  Needs the reference's ``runtime`` package (present
where the fixtures are generated); skipped elsewhere.  The GPU side --
weights shared, one captured graph per binding, results per binding -- is
tests/test_gpu_rebind.py."""

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

import lbr_b200.session as sess  # noqa: E402


class FakeExecutor:
    compiled = []

    def __init__(self, profile=False, device=0, lib_path=None, constants=None):
        self.constants = constants
        self.plan = None
        self.closed = False
        self._last_profile = None

    def compile(self, plan):
        self.plan = plan
        FakeExecutor.compiled.append(plan)

    def run(self, inputs):
        (name, x), = inputs.items()
        return {"shape": np.array(x.shape)}

    def close(self):
        self.closed = True


class FakePool:
    def __init__(self, device=0, lib_path=None):
        self.cleared = False

    def clear(self):
        self.cleared = True


@pytest.fixture
def session_cls(monkeypatch):
    monkeypatch.setattr(sess, "CudaCompiledExecutor", FakeExecutor)
    monkeypatch.setattr(sess, "ConstantPool", FakePool)
    FakeExecutor.compiled = []
    return sess.b200_session_class()


class Block(torch.nn.Module):
    """LayerNorm -> QKV -> SDPA -> projection, residual: enough for symbolic S."""

    def __init__(self, d=64, h=4):
        super().__init__()
        self.h = h
        self.ln = torch.nn.LayerNorm(d)
        self.q, self.k, self.v = (torch.nn.Linear(d, d) for _ in range(3))
        self.proj = torch.nn.Linear(d, d)

    def forward(self, x):
        B, S, D = x.shape
        h = self.ln(x)
        q, k, v = (m(h).reshape(B, S, self.h, D // self.h).transpose(1, 2) for m in (self.q, self.k, self.v))
        o = torch.nn.functional.scaled_dot_product_attention(q, k, v)
        return x + self.proj(o.transpose(1, 2).reshape(B, S, D))


@pytest.fixture
def dynamic_graph():
    from runtime.exporter import export_pytorch
    from runtime.passes import run_pipeline
    torch.manual_seed(0)
    model = Block().eval()
    graph = export_pytorch(model, (torch.randn(1, 8, 64),), dynamic_dims={"S": [("x", 1)]})
    run_pipeline(graph)
    return graph


def input_shape(plan):
    g = plan.graph
    return g.tensors[g.inputs[0]].shape


def test_rebind_compiles_each_binding_once(session_cls, dynamic_graph):
    s = session_cls(dynamic_graph, max_bindings=4)
    s.create(execution_mode="cuda", bindings={"S": 8})
    first = s._executor
    assert len(FakeExecutor.compiled) == 1 and input_shape(first.plan) == (1, 8, 64)
    s.rebind({"S": 16})
    assert len(FakeExecutor.compiled) == 2 and input_shape(s._executor.plan) == (1, 16, 64)
    s.rebind({"S": 8})
    assert len(FakeExecutor.compiled) == 2 and s._executor is first     # cached: no re-plan
    assert s.binding_cache.hits == 1 and s.binding_cache.compiles == 2
    out = s.run({dynamic_graph.inputs[0]: np.zeros((1, 8, 64), np.float32)})
    assert list(out["shape"]) == [1, 8, 64]


def test_least_recently_used_binding_is_closed(session_cls, dynamic_graph):
    s = session_cls(dynamic_graph, max_bindings=2)
    s.create(execution_mode="cuda", bindings={"S": 4})
    ex4 = s._executor
    s.rebind({"S": 8})
    s.rebind({"S": 4})          # 4 most recent
    s.rebind({"S": 12})         # evicts 8
    cache = s.binding_cache
    assert ("S", 8) not in {k[0] for k in cache._execs} and len(cache) == 2
    assert not ex4.closed
    s.rebind({"S": 8})          # re-planned
    assert len(FakeExecutor.compiled) == 4
    s.close()
    assert cache.pool.cleared and len(cache) == 0


def test_other_modes_stay_the_reference(session_cls, dynamic_graph):
    """execution_mode="compiled" / "interpreted" keep the reference's executors."""
    s = session_cls(dynamic_graph)
    s.create(execution_mode="interpreted", backend="numpy", bindings={"S": 8})
    from runtime.executor.interpreted import InterpretedExecutor
    assert isinstance(s._executor, InterpretedExecutor)
    assert FakeExecutor.compiled == []
