"""DataParallelExecutor: the batch scattered by rows over worker processes,
outputs gathered into one batch behind one run() (SURVEY row e's host
scatter / gather behind the reference's run() contract,
runtime/executor/compiled.py:72-97).

On the CPU the workers run the oracle (test infrastructure) instead of a
GPU: two workers each run gpt2_mini_s64_b1, one shard of gpt2_mini_s64, and
together they must reproduce the reference C executor's golden output for
the full batch.  The GPU test runs the CUDA executor in the workers."""

import numpy as np
import pytest

from conftest import GOLDEN, has_gpu, load_golden
from lbr_b200.parallel import DataParallelExecutor
from lbr_b200.program import Program

ATOL, RTOL = 1e-4, 1e-3


class OracleExecutor:
    """A worker executor on the host: the restated oracle."""

    def __init__(self, device):
        self.device = device

    def compile_program(self, program, constants):
        self.program, self.constants = program, constants

    def run(self, inputs):
        import oracle
        return oracle.run_program("restated", self.program, self.constants, inputs)


class FailingExecutor(OracleExecutor):
    def run(self, inputs):
        if self.device == 1:
            raise RuntimeError("injected failure on device 1")
        return super().run(inputs)


def oracle_factory(device):
    return OracleExecutor(device)


def failing_factory(device):
    return FailingExecutor(device)


def _shard_and_golden():
    shard = Program.load(GOLDEN / "gpt2_mini_s64_b1.json")
    _, ins, outs = load_golden("gpt2_mini_s64")
    return shard, shard.make_constants(), ins, outs


def test_two_workers_reproduce_the_full_batch():
    shard, consts, ins, outs = _shard_and_golden()
    with DataParallelExecutor(shard, [0, 1], consts, executor_factory=oracle_factory) as dp:
        assert dp.batch == 2
        for _ in range(2):   # the workers keep their compiled state between calls
            got = dp.run(ins)
            for k, ref in outs.items():
                np.testing.assert_allclose(got[k], ref, atol=ATOL, rtol=RTOL)


def test_worker_failure_is_reported_and_the_others_stay_usable():
    shard, consts, ins, outs = _shard_and_golden()
    dp = DataParallelExecutor(shard, [0, 1], consts, executor_factory=failing_factory)
    try:
        with pytest.raises(RuntimeError, match="rank 1 .*injected failure"):
            dp.run(ins)
        with pytest.raises(RuntimeError, match="injected failure"):   # still answering
            dp.run(ins)
    finally:
        dp.close()


@pytest.mark.gpu
def test_cuda_workers_reproduce_the_full_batch():
    if not has_gpu():
        pytest.skip("no CUDA device")
    import torch
    n = torch.cuda.device_count()
    devices = [0, 1] if n < 2 else [0, 1]   # one GPU: both workers share it
    devices = devices if n >= 2 else [0, 0]
    shard, consts, ins, outs = _shard_and_golden()
    with DataParallelExecutor(shard, devices, consts) as dp:
        got = dp.run(ins)
        for k, ref in outs.items():
            np.testing.assert_allclose(got[k], ref, atol=ATOL, rtol=RTOL)
