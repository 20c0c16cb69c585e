"""Dynamic-shape bindings on the GPU (session.BindingCache): one block
exported once with a symbolic sequence length, planned per binding
(tests/golden/dyn_s*.json).  Weights are uploaded once for all bindings,
each binding compiles (and captures its CUDA graph) once, revisits replay,
eviction releases only the evicted binding's plan, and every binding's
result matches the oracle."""

import numpy as np
import pytest

import oracle
from conftest import GOLDEN
from lbr_b200.program import Program
from lbr_b200.session import BindingCache

pytestmark = pytest.mark.gpu

SEQ = (64, 128, 200, 384)


@pytest.fixture(scope="module")
def progs():
    ps = {s: Program.load(GOLDEN / f"dyn_s{s}.json") for s in SEQ}
    # one set of weight arrays for every binding, as resolve_graph shares them
    consts = ps[SEQ[0]].make_constants(0)
    for p in ps.values():
        assert set(p.constants) == set(consts)
    return ps, consts


def test_bindings_share_weights_and_graphs(progs):
    ps, consts = progs
    cache = BindingCache(max_bindings=3)
    lib = cache.pool._lib
    try:
        order = [128, 64, 128, 384, 64, 200, 128]
        for s in order:
            hit = s in cache
            before = lib.rt_plan_count()
            ex = cache.get(s, lambda e, s=s: e.compile_program(ps[s], consts))
            # a new binding is planned and captured at compile (evicting at most
            # one other binding's plan); a revisit neither plans nor captures
            plans = lib.rt_plan_count()
            assert plans == before if hit else plans in (before, before + 1)
            ins = ps[s].make_inputs(s)
            got = ex.run(ins)
            assert lib.rt_plan_count() == plans
            ref = oracle.run_program("restated", ps[s], consts, ins)
            for k in got:
                np.testing.assert_allclose(got[k], ref[k], atol=1e-4, rtol=1e-3, err_msg=f"S={s}")
        # 128 64 [128] 384 [64] 200(evicts 128) 128(evicts 384)
        assert cache.compiles == 5 and cache.hits == 2
        assert cache.pool.uploads == len(consts)           # weights uploaded once
        assert len(cache) == 3
    finally:
        cache.close()


def test_evicted_binding_releases_only_its_plan(progs):
    ps, consts = progs
    cache = BindingCache(max_bindings=2)
    lib = cache.pool._lib
    try:
        base = lib.rt_plan_count()
        for s in (64, 128):
            cache.get(s, lambda e, s=s: e.compile_program(ps[s], consts)).run(ps[s].make_inputs(0))
        assert lib.rt_plan_count() == base + 2
        cache.get(200, lambda e: e.compile_program(ps[200], consts))
        assert lib.rt_plan_count() == base + 2              # 64's plan released, 200's made, 128's kept
        ex128 = cache.get(128, lambda e: pytest.fail("128 should be cached"))
        got = ex128.run(ps[128].make_inputs(1))
        ref = oracle.run_program("restated", ps[128], consts, ps[128].make_inputs(1))
        for k in got:
            np.testing.assert_allclose(got[k], ref[k], atol=1e-4, rtol=1e-3)
    finally:
        cache.close()
