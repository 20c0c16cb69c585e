"""The CPU oracle pinned against the reference's own outputs.

Goldens (tests/golden/*.golden.npz) were produced by the reference C
executor (csrc/executor.c, built from its sources by oracle/Makefile) on the
programs the reference pipeline planned; the toy block's golden also holds
the PyTorch model's output.  The restated oracle must agree with them to
fp32 summation-order rounding, and the reference build (when present) must
reproduce them bit for bit.
"""

import numpy as np
import pytest

import oracle
from conftest import load_golden, mini_programs


@pytest.mark.parametrize("name", mini_programs())
def test_restated_oracle_matches_reference_golden(name):
    prog, ins, outs = load_golden(name)
    got = oracle.run_program("restated", prog, prog.make_constants(), ins)
    for k, ref in outs.items():
        np.testing.assert_allclose(got[k], ref, atol=2e-6, rtol=1e-5)


@pytest.mark.parametrize("name", mini_programs())
def test_reference_build_reproduces_golden(name):
    if not oracle.available("reference"):
        pytest.skip("reference build (oracle/_ref) not present")
    prog, ins, outs = load_golden(name)
    got = oracle.run_program("reference", prog, prog.make_constants(), ins)
    for k, ref in outs.items():
        np.testing.assert_array_equal(got[k], ref)


def test_toy_golden_matches_pytorch():
    prog, ins, outs = load_golden("toy")
    import numpy as np  # noqa
    z = np.load(oracle.HERE.parent / "tests" / "golden" / "toy.golden.npz")
    for k, ref in outs.items():
        np.testing.assert_allclose(ref, z["torch__" + k], atol=1e-5)
