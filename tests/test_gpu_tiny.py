"""The small-graph path (k_tiny.cu): a plan whose nodes are all tiny runs as
one cluster launch that walks the node array on the device.

* the toy block takes it: one launch per forward, the
  reference C executor's golden output, and the same result as the
  one-kernel-per-node path (RT_TINY=0);
* every per-op case of test_gpu_ops.py that fits the path runs on it in a
  fresh process (RT_TINY=force also takes one-node plans) against the oracle.
"""

import os
import subprocess
import sys

import numpy as np
import pytest

from conftest import load_golden

pytestmark = pytest.mark.gpu
ATOL, RTOL = 1e-4, 1e-3


def test_toy_runs_as_one_launch(gpu_executor_factory, monkeypatch):
    prog, ins, outs = load_golden("toy")
    monkeypatch.delenv("RT_TINY", raising=False)
    ex = gpu_executor_factory(prog, prog.make_constants())
    got = ex.run(ins)
    assert ex.kernel_launches == 1
    for k, ref in outs.items():
        np.testing.assert_allclose(got[k], ref, atol=ATOL, rtol=RTOL)
    monkeypatch.setenv("RT_TINY", "0")
    ex2 = gpu_executor_factory(prog, prog.make_constants())
    per_node = ex2.run(ins)
    assert ex2.kernel_launches > 10
    for k in got:
        np.testing.assert_allclose(got[k], per_node[k], atol=ATOL, rtol=RTOL)
    # eager launch (no graph) and graph replay agree bit for bit
    ex.upload_inputs(ins)
    ex.execute_eager()
    eager = ex.download_outputs()
    for k in got:
        np.testing.assert_array_equal(got[k], eager[k])


def test_per_op_cases_on_the_small_graph_kernel():
    here = os.path.dirname(__file__)
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-m", "gpu", "-p", "no:cacheprovider",
                        os.path.join(here, "test_gpu_ops.py"), "-k", "not variant and not variants"],
                       env=dict(os.environ, RT_TINY="force"), capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
