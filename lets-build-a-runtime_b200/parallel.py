"""Data-parallel execution over several GPUs behind one ``run()``.

The graphs this backend runs treat the rows of a batch independently (every
node of the transformer bodies is per row: norms, GEMMs, per-(batch, head)
attention -- csrc/ops/attn.c:246-252), so a batch shards across GPUs with no
exchange at all: each GPU holds a replica of the weights, a graph planned for
its share of the rows (its own arena and captured CUDA graph) and runs it
independently.  :class:`DataParallelExecutor` is the host side of that: one
worker process per GPU (the library keeps one device per process), a
full-batch host array per graph input and output in shared memory, and
``run(inputs) -> dict`` with the reference executor's contract
(runtime/executor/compiled.py:72-97): inputs scattered by rows to the
workers, each worker's output rows written straight into the shared output
arrays (no host-side concatenation), outputs returned as one batch.

No collective is involved; a worker that fails reports its exception and
``run`` raises it (the other workers keep their state and stay usable).
"""

from __future__ import annotations

import multiprocessing as mp
import pickle
from multiprocessing import shared_memory
from pathlib import Path
from typing import Any, Callable

import numpy as np

from .program import Program


def _shared_array(shape, dtype) -> tuple[shared_memory.SharedMemory, np.ndarray]:
    nbytes = max(1, int(np.prod(shape)) * np.dtype(dtype).itemsize)
    shm = shared_memory.SharedMemory(create=True, size=nbytes)
    return shm, np.ndarray(shape, dtype=dtype, buffer=shm.buf)


def _attach(spec) -> tuple[shared_memory.SharedMemory, np.ndarray]:
    name, shape, dtype = spec
    shm = shared_memory.SharedMemory(name=name)
    return shm, np.ndarray(shape, dtype=dtype, buffer=shm.buf)


def _cuda_executor(device: int):
    from .executor import CudaCompiledExecutor
    return CudaCompiledExecutor(device=device)


# A spawned worker starts in a fresh interpreter where this package (whose
# directory name is not a Python identifier) is not importable by name: it
# runs this bootstrap through the builtin ``exec``, which registers the
# package as ``lbr_b200`` and then unpickles its arguments.
_BOOTSTRAP = """
import importlib.util, pickle, sys
if "lbr_b200" not in sys.modules:
    _s = importlib.util.spec_from_file_location("lbr_b200", pkg_dir + "/__init__.py",
                                                submodule_search_locations=[pkg_dir])
    _m = importlib.util.module_from_spec(_s)
    sys.modules["lbr_b200"] = _m
    _s.loader.exec_module(_m)
from lbr_b200.parallel import _worker
_worker(*pickle.loads(payload), conn)
"""


def _worker(rank, device, program, const_specs, in_specs, out_specs, rows, factory, conn):
    """One shard: rows [rank*rows, (rank+1)*rows) of every input and output."""
    held = []
    try:
        consts = {}
        for k, spec in const_specs.items():
            shm, arr = _attach(spec)
            held.append(shm)
            consts[k] = arr
        ins, outs = {}, {}
        for k, spec in in_specs.items():
            shm, arr = _attach(spec)
            held.append(shm)
            ins[k] = arr[rank * rows:(rank + 1) * rows]
        for k, spec in out_specs.items():
            shm, arr = _attach(spec)
            held.append(shm)
            outs[k] = arr[rank * rows:(rank + 1) * rows]
        ex = (factory or _cuda_executor)(device)
        ex.compile_program(program, consts)
        conn.send(("ready", None))
    except Exception as e:  # noqa: BLE001 -- reported to the parent
        conn.send(("error", f"{type(e).__name__}: {e}"))
        return
    while True:
        msg = conn.recv()
        if msg == "stop":
            break
        try:
            got = ex.run({k: v for k, v in ins.items()})
            for k, v in got.items():
                outs[k][...] = v
            conn.send(("done", None))
        except Exception as e:  # noqa: BLE001
            conn.send(("error", f"{type(e).__name__}: {e}"))
    close = getattr(ex, "close", None)
    if close:
        close()
    del ins, outs, consts
    for shm in held:
        try:
            shm.close()
        except BufferError:   # a view still referenced by the executor: freed at exit
            pass


class DataParallelExecutor:
    """``run()`` over ``len(devices)`` GPUs, each running ``shard_program``
    (the graph planned for the rows one GPU takes) on its row slice.

    ``constants``: the weights by name (shared once in host memory; each
    worker uploads its replica).  ``executor_factory(device)`` builds a
    worker's executor (default: :class:`~executor.CudaCompiledExecutor` on that
    device); it must offer ``compile_program(program, constants)`` and
    ``run(inputs) -> dict``.  Every graph input and output must have the
    batch as its leading dimension."""

    def __init__(self, shard_program: Program, devices: list[int], constants: dict[str, np.ndarray],
                 executor_factory: Callable[[int], Any] | None = None, start_method: str = "spawn") -> None:
        if not devices:
            raise ValueError("at least one device")
        self.program = shard_program
        self.devices = list(devices)
        self._shms: list[shared_memory.SharedMemory] = []
        const_specs = {}
        for k, v in constants.items():
            v = np.ascontiguousarray(v)
            shm, arr = _shared_array(v.shape, v.dtype)
            arr[...] = v
            self._shms.append(shm)
            const_specs[k] = (shm.name, v.shape, v.dtype.str)
        n = len(self.devices)
        self.rows = None
        self.inputs: dict[str, np.ndarray] = {}
        self.outputs: dict[str, np.ndarray] = {}
        in_specs, out_specs = {}, {}
        for group, specs, store in (("inputs", in_specs, self.inputs), ("outputs", out_specs, self.outputs)):
            for k, s in getattr(shard_program, group).items():
                shape = list(s["shape"])
                if self.rows is None:
                    self.rows = shape[0]
                if shape[0] != self.rows:
                    raise ValueError(f"{k}: every graph input and output needs the batch as its leading dim")
                shape[0] *= n
                shm, arr = _shared_array(tuple(shape), s["dtype"])
                self._shms.append(shm)
                store[k] = arr
                specs[k] = (shm.name, tuple(shape), np.dtype(s["dtype"]).str)
        ctx = mp.get_context(start_method)
        self._conns, self._procs = [], []
        for rank, dev in enumerate(self.devices):
            parent, child = ctx.Pipe()
            payload = pickle.dumps((rank, dev, shard_program, const_specs, in_specs, out_specs, self.rows,
                                    executor_factory))
            env = {"pkg_dir": str(Path(__file__).resolve().parent), "payload": payload, "conn": child}
            p = ctx.Process(target=exec, args=(_BOOTSTRAP, env), daemon=True)
            p.start()
            self._conns.append(parent)
            self._procs.append(p)
        self._gather("ready")

    @property
    def batch(self) -> int:
        return self.rows * len(self.devices)

    def input_buffer(self, name: str) -> np.ndarray:
        """The full-batch shared host array of a graph input (fill it in place
        to skip the copy in ``run``)."""
        return self.inputs[name]

    def _gather(self, what: str) -> None:
        errors = []
        for rank, c in enumerate(self._conns):
            kind, msg = c.recv()
            if kind == "error":
                errors.append(f"rank {rank} (device {self.devices[rank]}): {msg}")
        if errors:
            raise RuntimeError(f"data-parallel {what} failed: " + "; ".join(errors))

    def run(self, inputs: dict[str, np.ndarray] | None = None, copy_outputs: bool = True) -> dict[str, np.ndarray]:
        for k, v in (inputs or {}).items():
            if v is not self.inputs[k]:
                self.inputs[k][...] = v
        for c in self._conns:
            c.send("run")
        self._gather("run")
        return {k: (v.copy() if copy_outputs else v) for k, v in self.outputs.items()}

    def close(self) -> None:
        for c, p in zip(self._conns, self._procs):
            if p.is_alive():
                try:
                    c.send("stop")
                except (BrokenPipeError, OSError):
                    pass
        for p in self._procs:
            p.join(timeout=60)
            if p.is_alive():
                p.terminate()
        self._procs = []
        self.inputs, self.outputs = {}, {}
        for shm in self._shms:
            try:
                shm.close()
            except BufferError:   # an output view the caller still holds (run(copy_outputs=False))
                pass
            shm.unlink()
        self._shms = []

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()
