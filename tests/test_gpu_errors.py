"""Failure handling of the C ABI on a device: bad node arrays are rejected on
the host, before any launch, with a status instead of the reference's
abort() (csrc/executor.c:461-464); the library stays usable afterwards."""

import ctypes

import numpy as np
import pytest

from conftest import GOLDEN, has_gpu
from lbr_b200.copnode import COpNode
from lbr_b200.executor import load_library
from lbr_b200.program import Program

pytestmark = pytest.mark.gpu


@pytest.fixture()
def lib():
    if not has_gpu():
        pytest.skip("no CUDA device")
    lib = load_library()
    assert lib.rt_init(0) == 0
    lib.rt_clear_error()
    return lib


def one_node(lib, op=104, n=256, out=None, inp=None):
    arr = (COpNode * 1)()
    arr[0].op = op
    arr[0].n_inputs = 1
    arr[0].inputs[0] = inp if inp is not None else lib.rt_alloc(n * 4)
    arr[0].output = out if out is not None else lib.rt_alloc(n * 4)
    arr[0].n_dims = 1
    arr[0].out_shape[0] = n
    arr[0].elem_size = 4
    return arr


def test_unknown_op_returns_status(lib):
    arr = one_node(lib, op=999)
    assert lib.rt_execute(arr, 1, 0) == 2
    assert b"unknown op" in lib.rt_last_error_message()
    lib.execute(arr, 1)                   # void entry point: records, never aborts
    assert lib.rt_last_error() == 2


def test_permute_has_no_dispatch_entry(lib):
    assert lib.rt_execute(one_node(lib, op=502), 1, 0) == 2


def test_host_pointer_rejected(lib):
    host = np.zeros(256, np.float32)
    assert lib.rt_execute(one_node(lib, inp=host.ctypes.data), 1, 0) == 5


def test_pinned_host_pointer_rejected(lib):
    pinned = lib.rt_host_alloc(1024)
    assert lib.rt_execute(one_node(lib, inp=pinned), 1, 0) == 5


def test_out_of_range_rejected(lib):
    small = lib.rt_alloc(64)
    assert lib.rt_execute(one_node(lib, n=256, out=small), 1, 0) == 6


def test_null_pointer_rejected(lib):
    arr = one_node(lib)
    arr[0].inputs[0] = None
    assert lib.rt_execute(arr, 1, 0) == 4


def test_too_few_inputs_rejected(lib):
    arr = one_node(lib, op=1000)          # MATMUL_ADD needs 3
    assert lib.rt_execute(arr, 1, 0) == 3


def test_library_usable_after_errors(lib):
    lib.rt_execute(one_node(lib, op=999), 1, 0)
    x = lib.rt_alloc(1024 * 4)
    y = lib.rt_alloc(1024 * 4)
    host = np.linspace(-3, 3, 1024, dtype=np.float32)
    assert lib.rt_upload(x, host.ctypes.data, host.nbytes) == 0
    arr = one_node(lib, op=107, n=1024, inp=x, out=y)   # NEG
    assert lib.rt_execute(arr, 1, 0) == 0
    out = np.empty_like(host)
    assert lib.rt_download(out.ctypes.data, y, out.nbytes) == 0
    np.testing.assert_array_equal(out, -host)


def test_bounded_wait_times_out_and_library_stays_usable(lib):
    """A kernel waits on an mbarrier nothing arrives on; its bounded wait gives
    up after 50 ms, records a code and returns -- no fault, no hang."""
    assert lib.rt_check_wait_timeout(50_000_000) == 11          # RT_ERR_KERNEL_TIMEOUT
    assert b"bounded wait" in lib.rt_last_error_message()
    assert lib.rt_check_wait_timeout(0) == 10                   # RT_ERR_ARGUMENT
    test_library_usable_after_errors(lib)


def _matmul_node(lib, a, b, bias, out, M, N, K, trans_b=1):
    arr = (COpNode * 1)()
    n = arr[0]
    n.op = 1000 if bias is not None else 400
    n.n_inputs = 3 if bias is not None else 2
    n.inputs[0], n.inputs[1] = a, b
    if bias is not None:
        n.inputs[2] = bias
    n.output = out
    n.n_dims = 2
    n.out_shape[0], n.out_shape[1] = M, N
    n.elem_size = 4
    n.extra[0], n.extra[1], n.extra[2] = K, trans_b, 1
    return arr


def test_undersized_gemm_operands_rejected(lib):
    M, N, K = 512, 256, 128
    a, b = lib.rt_alloc(M * K * 4), lib.rt_alloc(N * K * 4)
    bias, out = lib.rt_alloc(N * 4), lib.rt_alloc(M * N * 4)
    assert lib.rt_execute(_matmul_node(lib, a, b, bias, out, M, N, K), 1, 0) == 0
    short_b = lib.rt_alloc(N * K * 4 - 64)
    assert lib.rt_execute(_matmul_node(lib, a, short_b, bias, out, M, N, K), 1, 0) == 6
    assert b"input 1" in lib.rt_last_error_message()
    short_a = lib.rt_alloc(M * K * 4 - 4)
    assert lib.rt_execute(_matmul_node(lib, short_a, b, bias, out, M, N, K), 1, 0) == 6
    short_bias = lib.rt_alloc(N * 4 - 4)
    assert lib.rt_execute(_matmul_node(lib, a, b, short_bias, out, M, N, K), 1, 0) == 6


def test_undersized_attention_kv_rejected(lib):
    BH, S, D, group = 8, 256, 64, 2
    arr = (COpNode * 1)()
    n = arr[0]
    n.op = 1002
    n.n_inputs = 4
    q, o = lib.rt_alloc(BH * S * D * 4), lib.rt_alloc(BH * S * D * 4)
    kv = BH // group * S * D * 4
    k, v, scratch = lib.rt_alloc(kv), lib.rt_alloc(kv - 256), lib.rt_alloc(1 << 20)
    n.inputs[0], n.inputs[1], n.inputs[2], n.inputs[3] = q, k, v, scratch
    n.output = o
    n.n_dims = 3
    n.out_shape[0], n.out_shape[1], n.out_shape[2] = BH, S, D
    n.elem_size = 4
    for j, x in enumerate([S, D, 1, 0, group]):
        n.extra[j] = x
    assert lib.rt_execute(arr, 1, 0) == 6
    assert b"input 2" in lib.rt_last_error_message()
    n.inputs[2] = lib.rt_alloc(kv)
    assert lib.rt_execute(arr, 1, 0) == 0
