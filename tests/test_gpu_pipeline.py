"""PipelinedExecutor: the batch as row chunks (graphs planned for fewer rows)
whose host copies overlap each other's kernels (rt_execute_chunks).  Same
results as the whole-batch graph / the reference golden."""

import numpy as np
import pytest

from conftest import GOLDEN, load_golden
from lbr_b200.executor import CudaCompiledExecutor
from lbr_b200.pipeline import PipelinedExecutor
from lbr_b200.program import Program

pytestmark = pytest.mark.gpu


def test_two_chunks_match_reference_golden():
    """gpt2_mini_s64 (batch 2) as two batch-1 chunks vs the reference C
    executor's golden output for the whole batch."""
    prog2, ins, outs = load_golden("gpt2_mini_s64")
    chunk = Program.load(GOLDEN / "gpt2_mini_s64_b1.json")
    consts = prog2.make_constants()
    pipe = PipelinedExecutor(chunk, 2, consts)
    try:
        for _ in range(2):   # second call: replayed graphs, same buffers
            got = pipe.run(ins)
            for k, ref in outs.items():
                np.testing.assert_allclose(got[k], ref, atol=1e-4, rtol=1e-3)
    finally:
        pipe.close()


@pytest.mark.slow
def test_chunked_gpt2_equals_whole_batch():
    p8 = Program.load(GOLDEN / "gpt2_b8.json")
    p4 = Program.load(GOLDEN / "gpt2_b4.json")
    consts = p8.make_constants()
    ins = p8.make_inputs(3)
    ex = CudaCompiledExecutor()
    ex.compile_program(p8, consts)
    whole = ex.run(ins)
    ex.close()
    pipe = PipelinedExecutor(p4, 2, consts)
    try:
        got = pipe.run(ins)
    finally:
        pipe.close()
    for k in whole:
        np.testing.assert_allclose(got[k], whole[k], atol=2e-5, rtol=1e-4)
