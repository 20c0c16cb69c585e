"""CudaBackend driven the way the reference's interpreted executor drives a
backend (runtime/executor/interpreted.py:47-98): every node of ``plan.order``
that is not a zero-copy alias becomes one ``kernel(input_buffers,
output_buffer, node.attrs)`` call, with the planned scratch region appended.

The calls were recorded from the reference's own plan by
tests/golden/make_interp_traces.py (the reference package is not present on
the GPU box).  Replaying them through CudaBackend must reproduce both the
reference C executor's golden output and the reference interpreted
executor's numpy-backend output, within the parity bar."""

import json
from types import SimpleNamespace

import numpy as np
import pytest

from conftest import GOLDEN
from lbr_b200.program import Program

pytestmark = pytest.mark.gpu
ATOL, RTOL = 1e-4, 1e-3
NAMES = ["toy", "gpt2_mini_s64", "qwen3_mini_s272", "block_mini_causal_s300"]


@pytest.fixture(scope="module")
def backend():
    from conftest import has_gpu
    if not has_gpu():
        pytest.skip("no CUDA device")
    from lbr_b200.backend import CudaBackend
    b = CudaBackend()
    yield b
    b.close()


def replay(backend, doc, consts, inputs):
    env = {k: np.ascontiguousarray(v) for k, v in inputs.items()}
    calls = 0
    for st in doc["steps"]:
        for name, shape in zip(st["inputs"], st["in_shapes"]):
            if name not in env:
                env[name] = np.ascontiguousarray(consts[name]).reshape(shape)
        if st["alias"]:
            assert st["op_name"] == "RESHAPE" and st["alias_offset"] == 0, st
            env[st["output"]] = env[st["inputs"][0]].reshape(st["out_shape"])
            continue
        kernel = backend.get_kernel(SimpleNamespace(value=st["op"], name=st["op_name"]))
        assert kernel is not None, st["op_name"]
        bufs = [env[n] for n in st["inputs"]]
        if st["scratch_bytes"]:
            bufs.append(np.zeros(st["scratch_bytes"], np.uint8))
        out = np.full(st["out_shape"], np.nan, dtype=st["dtype"])
        kernel(bufs, out, st["attrs"])
        env[st["output"]] = out
        calls += 1
    return {k: env[k] for k in doc["graph_outputs"]}, calls


@pytest.mark.parametrize("name", NAMES)
def test_interpreted_replay_matches_reference(name, backend):
    doc = json.loads((GOLDEN / "interp" / f"{name}.json").read_text())
    gold = np.load(GOLDEN / f"{name}.golden.npz")
    interp = np.load(GOLDEN / "interp" / f"{name}.npz")
    consts = Program.load(GOLDEN / f"{name}.json").make_constants(0)
    inputs = {k[4:]: gold[k] for k in gold.files if k.startswith("in__")}
    got, calls = replay(backend, doc, consts, inputs)
    assert calls == sum(not s["alias"] for s in doc["steps"])
    for k, v in got.items():
        ref = gold["out__" + k]
        err = float(np.abs(v - ref).max())
        print(f"{name}:{k} CudaBackend vs reference C executor: max abs {err:.3e}")
        np.testing.assert_allclose(v, ref, atol=ATOL, rtol=RTOL, err_msg=f"{name}:{k} vs C executor")
        np.testing.assert_allclose(v, interp["out__" + k], atol=ATOL, rtol=RTOL,
                                   err_msg=f"{name}:{k} vs reference interpreted (numpy backend)")
