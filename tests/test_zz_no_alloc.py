"""rt_matmul_noalloc: the tensor-core GEMM for callers that may not allocate.

Some callers of this library cannot call cudaMalloc at all -- a plugin whose
host application owns every device allocation through its own pool, or a
process whose device footprint is fixed once it has started.  For them
rt_matmul_noalloc runs the same split-operand tensor-core GEMM as a
MATMUL / MATMUL_ADD node, with its scratch in a fixed 32 MiB device array
inside the library instead of a workspace the runtime allocates.

The first test calls it through the C ABI twice in a row (different
operands, so stale scratch from the first call would show) and compares each
result with the existing entry point, `rt_execute` on a one-node array,
within the tolerance the other GEMM tests use.  Another runs it in a fresh
child process that never calls rt_init, on a stream and device memory that
PyTorch owns, with alpha != 1 and no bias, against an fp64 product.  The file
is named to be collected last, and works alone as well as after the others.
"""

import ctypes

import numpy as np
import pytest

from conftest import has_gpu
from lbr_b200.copnode import COpNode
from lbr_b200.executor import load_library

pytestmark = pytest.mark.gpu
ATOL, RTOL = 1e-4, 1e-3
RT_ERR_OUT_OF_RANGE, RT_ERR_UNSUPPORTED = 6, 7


@pytest.fixture()
def lib():
    if not has_gpu():
        pytest.skip("no CUDA device")
    lib = load_library()
    assert lib.rt_init(0) == 0
    f = lib.rt_matmul_noalloc
    f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                  ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_void_p]
    f.restype = ctypes.c_int
    return lib


def device_array(lib, host):
    p = lib.rt_alloc(host.nbytes)
    assert p
    assert lib.rt_upload(p, host.ctypes.data, host.nbytes) == 0
    return p


def download(lib, p, shape):
    out = np.empty(shape, np.float32)
    assert lib.rt_download(out.ctypes.data, p, out.nbytes) == 0
    return out


def via_execute(lib, a, b, bias, c, M, N, K, trans_b):
    """The existing path: a MATMUL_ADD node through rt_execute."""
    arr = (COpNode * 1)()
    n = arr[0]
    n.op = 1000
    n.n_inputs = 3
    n.inputs[0], n.inputs[1], n.inputs[2] = a, b, bias
    n.output = c
    n.n_dims = 2
    n.out_shape[0], n.out_shape[1] = M, N
    n.elem_size = 4
    n.extra[0], n.extra[1], n.extra[2] = K, trans_b, 1
    rc = lib.rt_execute(arr, 1, 0)
    assert rc == 0, lib.rt_last_error_message()


@pytest.mark.parametrize("M,N,K,trans_b", [(1000, 768, 768, 1), (300, 520, 1024, 0)])
def test_noalloc_matches_execute_on_two_calls(lib, M, N, K, trans_b):
    rng = np.random.default_rng(7)
    for call in range(2):
        a = rng.standard_normal((M, K)).astype(np.float32)
        b = (rng.standard_normal((N, K) if trans_b else (K, N)) * 0.02).astype(np.float32)
        bias = rng.standard_normal(N).astype(np.float32)
        da, db, dbias = device_array(lib, a), device_array(lib, b), device_array(lib, bias)
        c_ref, c_new = lib.rt_alloc(M * N * 4), lib.rt_alloc(M * N * 4)
        via_execute(lib, da, db, dbias, c_ref, M, N, K, trans_b)
        rc = lib.rt_matmul_noalloc(da, db, dbias, c_new, M, N, K, trans_b, 1.0, lib.rt_stream())
        assert rc == 0, f"call {call}: status {rc}"
        ref = download(lib, c_ref, (M, N))
        got = download(lib, c_new, (M, N))
        np.testing.assert_allclose(got, ref, atol=ATOL, rtol=RTOL, err_msg=f"call {call}")
        truth = a.astype(np.float64) @ (b.T if trans_b else b).astype(np.float64) + bias
        np.testing.assert_allclose(got, truth, atol=ATOL, rtol=RTOL, err_msg=f"call {call} vs fp64")
        for p in (da, db, dbias, c_ref, c_new):
            lib.rt_free(p)


def test_noalloc_rejects_oversize_and_ragged_k(lib):
    dummy = lib.rt_alloc(1024)
    # 8*(M*K + N*K) bytes of scratch > 32 MiB
    assert lib.rt_matmul_noalloc(dummy, dummy, None, dummy, 4096, 4096, 1024, 1, 1.0, None) == \
        RT_ERR_OUT_OF_RANGE
    assert lib.rt_matmul_noalloc(dummy, dummy, None, dummy, 64, 64, 66, 1, 1.0, None) == \
        RT_ERR_UNSUPPORTED
    lib.rt_free(dummy)


CHILD = r"""
import ctypes, sys
import numpy as np
import torch
sys.path.insert(0, sys.argv[1])
from __graft_entry__ import load_package
load_package()
from lbr_b200.executor import load_library

lib = load_library()          # no rt_init: the entry point must not need it
f = lib.rt_matmul_noalloc
f.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 4 + [ctypes.c_float, ctypes.c_void_p]
f.restype = ctypes.c_int
torch.cuda.set_device(0)
st = torch.cuda.Stream()
g = torch.Generator().manual_seed(3)
M, N, K, alpha = 520, 384, 640, 0.37
for call in range(2):
    a = torch.randn(M, K, generator=g)
    b = torch.randn(K, N, generator=g) * 0.05
    da, db = a.cuda(), b.cuda()          # torch's caching allocator owns these
    dc = torch.full((M, N), float("nan"), device="cuda")
    torch.cuda.synchronize()
    rc = f(da.data_ptr(), db.data_ptr(), None, dc.data_ptr(), M, N, K, 0, alpha, st.cuda_stream)
    assert rc == 0, f"status {rc}"
    got = dc.cpu().numpy()
    truth = alpha * (a.double().numpy() @ b.double().numpy())
    err = float(np.abs(got - truth).max())
    assert np.allclose(got, truth, atol=1e-4, rtol=1e-3), f"call {call}: max abs {err:.3e}"
    print(f"call {call}: max abs vs fp64 {err:.3e}")
print("ok")
"""


def test_noalloc_fresh_process_without_rt_init():
    """A caller that never touched rt_init: current device, its own stream and
    PyTorch-owned buffers; alpha != 1 and bias NULL, checked against fp64."""
    if not has_gpu():
        pytest.skip("no CUDA device")
    import subprocess
    import sys
    from conftest import ROOT
    r = subprocess.run([sys.executable, "-c", CHILD, str(ROOT)], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout + r.stderr
