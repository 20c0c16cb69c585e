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
