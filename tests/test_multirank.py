"""Data-parallel sharding on CPU ranks (gloo, world size 2).

The multi-GPU path splits the batch across ranks with no collective on the
data path (bench.py: rank r runs the batch-B/N program on sequences
[r*B/N, (r+1)*B/N)).  Here two gloo ranks each run the batch-1 program of
the GPT-2-style mini body on their own sequence with the CPU oracle, gather
the outputs, and compare with the batch-2 program run whole; a rank that
raises is reported to the other as a failed collective, not a hang.
"""

import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q, fail_rank):
    try:
        sys.path.insert(0, str(ROOT))
        from __graft_entry__ import load_package
        load_package()
        import torch
        import torch.distributed as dist
        import oracle
        from lbr_b200.program import Program
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=30))
        if rank == fail_rank:
            raise RuntimeError("injected rank failure")
        prog = Program.load(ROOT / "tests" / "golden" / "gpt2_mini_s64_b1.json")
        consts = prog.make_constants(0)
        ins = prog.make_inputs(0, batch_offset=rank)
        out = oracle.run_program("restated", prog, consts, ins)
        name = next(iter(out))
        t = torch.from_numpy(out[name])
        gathered = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(gathered, t)
        if rank == 0:
            q.put(("ok", torch.cat(gathered).numpy()))
        dist.destroy_process_group()
    except Exception as e:   # reported to the parent, which decides
        q.put(("error", f"rank {rank}: {e}"))


def _run(world, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, fail_rank)) for r in range(world)]
    for p in procs:
        p.start()
    # drain the queue before joining: a child cannot exit while its queued
    # message is still unread
    import queue as _queue
    msgs = []
    expected = 1 if fail_rank < 0 else world
    for _ in range(expected):
        try:
            msgs.append(q.get(timeout=150))
        except _queue.Empty:
            break
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return msgs


def test_batch_split_across_two_ranks_matches_whole_batch():
    import oracle
    from lbr_b200.program import Program
    msgs = _run(2)
    oks = [m for m in msgs if m[0] == "ok"]
    assert oks, msgs
    got = oks[0][1]
    whole = Program.load(ROOT / "tests" / "golden" / "gpt2_mini_s64.json")
    ref = oracle.run_program("restated", whole, whole.make_constants(0), whole.make_inputs(0))
    ref = next(iter(ref.values()))
    np.testing.assert_allclose(got, ref, atol=1e-5, rtol=1e-5)


def test_failed_rank_is_reported_not_hung():
    msgs = _run(2, fail_rank=1)
    errors = [m for m in msgs if m[0] == "error"]
    assert any("injected" in m[1] for m in errors), msgs
    # the surviving rank's collective fails (peer gone) instead of blocking forever
    assert not any(m[0] == "ok" for m in msgs)
