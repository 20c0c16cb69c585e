"""CudaCompiledExecutor -- drop-in for the reference ``CompiledExecutor``.

Same two-call interface as runtime/executor/compiled.py:20-158:
``compile(plan)`` once per plan, ``run(inputs) -> {output name: array}`` per
inference, ``profile`` flag and ``last_profile``.  Differences, all about
where memory lives:

* the arena (runtime/executor/common.py:83-87) is ONE device allocation of
  ``plan.arena_size`` bytes; planner offsets become device addresses and
  RESHAPE/contiguous-SLICE aliases stay zero-copy views into it;
* constants (weights) are uploaded once and stay resident in HBM, marked
  immutable so derived operand forms can be cached;
* each graph input gets a fixed device staging buffer (plus a pinned host
  mirror), so the node array never changes between calls -- the reference
  instead patches input pointers per call (compiled.py:77-82) -- and the
  launch sequence is captured once into a CUDA graph by the library.

``run`` copies inputs host->device, replays the graph and copies outputs
device->host in one library call (``rt_execute_io``).
"""

from __future__ import annotations

import ctypes
import time
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

from .copnode import COpNode, build_node_array
from .program import OP_NAME, Program, Ref

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libb200exec.so"

RT_FLAG_EAGER = 1
RT_FLAG_ASYNC = 2


class RtCopy(ctypes.Structure):
    _fields_ = [("dst", ctypes.c_void_p), ("src", ctypes.c_void_p), ("bytes", ctypes.c_size_t)]


_lib: ctypes.CDLL | None = None


def load_library(path: str | Path | None = None) -> ctypes.CDLL:
    """Load libb200exec.so (raises if it has not been built: no fallback)."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise RuntimeError(f"CUDA executor library not found at {p} -- run build() first")
    lib = ctypes.CDLL(str(p))
    vp, sz, i = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int
    sig = {
        "rt_init": ([i], i), "rt_destroy": ([], i), "rt_version": ([], ctypes.c_char_p),
        "rt_alloc": ([sz], vp), "rt_free": ([vp], i),
        "rt_host_alloc": ([sz], vp), "rt_host_free": ([vp], i),
        "rt_upload": ([vp, vp, sz], i), "rt_download": ([vp, vp, sz], i),
        "rt_mark_constant": ([vp, sz], i),
        "execute": ([ctypes.POINTER(COpNode), i], None),
        "rt_execute": ([ctypes.POINTER(COpNode), i, i], i),
        "rt_execute_io": ([ctypes.POINTER(COpNode), i, ctypes.POINTER(RtCopy), i,
                           ctypes.POINTER(RtCopy), i], i),
        "rt_prepare": ([ctypes.POINTER(COpNode), i], i),
        "rt_kernel_launches": ([ctypes.POINTER(COpNode), i], i),
        "rt_profile": ([ctypes.POINTER(COpNode), i, i, ctypes.POINTER(ctypes.c_float)], i),
        "rt_reset_plans": ([], i), "rt_synchronize": ([], i), "rt_stream": ([], vp),
        "rt_fusion_report": ([ctypes.POINTER(COpNode), i, ctypes.POINTER(ctypes.c_int)], i),
        "rt_protect": ([vp, sz], i), "rt_unprotect_all": ([], i),
        "rt_release": ([ctypes.POINTER(COpNode), i], i), "rt_plan_count": ([], i),
        "rt_last_error": ([], i), "rt_last_error_message": ([], ctypes.c_char_p),
        "rt_clear_error": ([], None), "rt_check_wait_timeout": ([ctypes.c_ulonglong], i),
    }
    for name, (args, res) in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    if path is None:
        _lib = lib
    return lib


class CudaRuntimeError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[rt status {code}] {msg}")
        self.code = code


def check(lib: ctypes.CDLL, rc: int, what: str = "") -> None:
    if rc != 0:
        msg = (lib.rt_last_error_message() or b"").decode(errors="replace")
        raise CudaRuntimeError(rc, f"{what}: {msg}" if what else msg)


# Profiling records with the reference's field names (common.py:24-63).
@dataclass
class OpTiming:
    node_id: int
    op: str
    time_ns: int
    output_name: str
    output_shape: tuple


@dataclass
class RunProfile:
    op_timings: list = field(default_factory=list)
    total_ns: int = 0

    def __str__(self) -> str:
        lines = [f"Execution Profile (device):", f"  Total: {self.total_ns / 1e6:.3f} ms"]
        by: dict[str, list[int]] = {}
        for t in self.op_timings:
            by.setdefault(t.op, []).append(t.time_ns)
        for op, ts in sorted(by.items(), key=lambda kv: -sum(kv[1])):
            pct = 100.0 * sum(ts) / self.total_ns if self.total_ns else 0.0
            lines.append(f"  {op:<20} {sum(ts) / 1e6:8.3f} ms ({pct:5.1f}%)  {len(ts)} ops")
        return "\n".join(lines)


class ConstantPool:
    """Device-resident constants shared by several executors.

    The reference re-plans and re-compiles for every new dynamic-shape binding
    (``Session.rebind``, runtime/session.py:187-207) while the weight buffers
    stay the same numpy arrays (``resolve_graph`` shares them,
    runtime/ops.py:589-613).  Executors compiled against one pool upload each
    such array once: entries are keyed by the host array (data address, size,
    dtype) and hold a reference to it, so the address cannot be reused while
    the entry lives.  Like ``rt_mark_constant``, it assumes constants are not
    modified in place afterwards; ``clear()`` drops every entry.
    """

    def __init__(self, device: int = 0, lib_path=None) -> None:
        self._lib = load_library(lib_path)
        check(self._lib, self._lib.rt_init(device), "rt_init")
        self._entries: dict[tuple, tuple[int, np.ndarray]] = {}
        self.uploads = 0

    def get(self, arr: np.ndarray) -> int:
        arr = np.ascontiguousarray(arr)
        key = (arr.__array_interface__["data"][0], arr.nbytes, arr.dtype.str)
        hit = self._entries.get(key)
        if hit is not None:
            return hit[0]
        lib = self._lib
        ptr = lib.rt_alloc(max(arr.nbytes, 1))
        if not ptr:
            check(lib, lib.rt_last_error() or 9, f"rt_alloc({arr.nbytes})")
        check(lib, lib.rt_upload(ptr, arr.ctypes.data, arr.nbytes), "upload constant")
        check(lib, lib.rt_mark_constant(ptr, arr.nbytes), "mark constant")
        self._entries[key] = (ptr, arr)
        self.uploads += 1
        return ptr

    def __len__(self) -> int:
        return len(self._entries)

    def clear(self) -> None:
        if self._entries:
            self._lib.rt_synchronize()
        for ptr, _ in self._entries.values():
            self._lib.rt_free(ptr)
        self._entries.clear()


class CudaCompiledExecutor:
    """Compiled executor whose one C-ABI call runs the graph on a B200.

    ``constants``: an optional :class:`ConstantPool` shared with other
    executors (dynamic-shape bindings of one model); without one, the
    executor owns its constants."""

    def __init__(self, profile: bool = False, device: int = 0, lib_path=None,
                 constants: ConstantPool | None = None) -> None:
        self._lib = load_library(lib_path)
        check(self._lib, self._lib.rt_init(device), "rt_init")
        self._pool = constants
        self._profile = profile
        self._last_profile: RunProfile | None = None
        self._device_allocs: list[int] = []
        self._host_allocs: list[int] = []
        self.program: Program | None = None
        self._nodes = None
        self._n_nodes = 0

    # ------------------------------------------------------------ compile
    def compile(self, plan) -> None:
        """Compile a reference ``MemoryPlan`` (needs the reference graph layer)."""
        from .lower import program_from_plan
        graph = plan.graph
        program = program_from_plan(plan, "plan", store_all=False)
        constants = {n: np.ascontiguousarray(graph.tensors[n].buffer) for n in program.constants}
        self.compile_program(program, constants)

    def compile_program(self, program: Program, constants: dict[str, np.ndarray]) -> None:
        self.close()
        lib = self._lib
        self.program = program
        self._arena = self._alloc(max(program.arena_size, 16))
        self._const_ptr: dict[str, int] = {}
        for name, spec in program.constants.items():
            arr = np.ascontiguousarray(constants[name], dtype=spec.dtype)
            if arr.nbytes != spec.nbytes:
                raise ValueError(f"constant {name}: {arr.nbytes} bytes, plan expects {spec.nbytes}")
            if self._pool is not None:
                self._const_ptr[name] = self._pool.get(arr)
                continue
            ptr = self._alloc(arr.nbytes)
            check(lib, lib.rt_upload(ptr, arr.ctypes.data, arr.nbytes), f"upload {name}")
            check(lib, lib.rt_mark_constant(ptr, arr.nbytes), f"mark {name}")
            self._const_ptr[name] = ptr
        # graph inputs: device staging + pinned host mirror
        self._in_dev: dict[str, int] = {}
        self._in_host: dict[str, np.ndarray] = {}
        for name, spec in program.inputs.items():
            dt = np.dtype(spec["dtype"])
            nbytes = int(np.prod(spec["shape"])) * dt.itemsize
            self._in_dev[name] = self._alloc(nbytes)
            self._in_host[name] = self._host_array(spec["shape"], dt)
        self._out_host: dict[str, np.ndarray] = {}
        for name, spec in program.outputs.items():
            self._out_host[name] = self._host_array(spec["shape"], np.dtype(spec["dtype"]))

        def resolve(r: Ref) -> int:
            if r.kind == "arena":
                return self._arena + r.offset
            if r.kind == "const":
                return self._const_ptr[r.name] + r.offset
            return self._in_dev[r.name] + r.offset

        self._resolve = resolve
        self._nodes = build_node_array(program, resolve)
        self._n_nodes = len(program.nodes)
        self._h2d = (RtCopy * max(1, len(self._in_dev)))()
        for k, name in enumerate(program.inputs):
            self._h2d[k] = RtCopy(self._in_dev[name], self._in_host[name].ctypes.data,
                                  self._in_host[name].nbytes)
        self._d2h = (RtCopy * max(1, len(self._out_host)))()
        # graph outputs must be materialised: keep layout fusion away from them
        for name, spec in program.outputs.items():
            check(lib, lib.rt_protect(resolve(spec["ref"]), self._out_host[name].nbytes), "protect")
        for k, (name, spec) in enumerate(program.outputs.items()):
            self._d2h[k] = RtCopy(self._out_host[name].ctypes.data, resolve(spec["ref"]),
                                  self._out_host[name].nbytes)
        check(lib, lib.rt_prepare(self._nodes, self._n_nodes), "prepare")

    # ---------------------------------------------------------------- run
    def run(self, inputs: dict[str, np.ndarray], copy_outputs: bool = True) -> dict[str, np.ndarray]:
        """Host in, host out: the reference ``CompiledExecutor.run`` contract."""
        for name, buf in self._in_host.items():
            if name not in inputs:
                raise ValueError(f"Missing input tensor: '{name}'")
            src = inputs[name]
            if not (isinstance(src, np.ndarray) and src.ctypes.data == buf.ctypes.data):
                np.copyto(buf, np.asarray(src, dtype=buf.dtype).reshape(buf.shape))
        t0 = time.perf_counter_ns() if self._profile else 0
        lib = self._lib
        check(lib, lib.rt_execute_io(self._nodes, self._n_nodes, self._h2d, len(self._in_host),
                                     self._d2h, len(self._out_host)), "execute")
        if self._profile:
            self._last_profile = RunProfile(total_ns=time.perf_counter_ns() - t0)
        if copy_outputs:
            return {k: v.copy() for k, v in self._out_host.items()}
        return dict(self._out_host)

    def execute_resident(self, sync: bool = True) -> None:
        """Replay the graph on inputs already in device staging (no copies)."""
        flags = 0 if sync else RT_FLAG_ASYNC
        check(self._lib, self._lib.rt_execute(self._nodes, self._n_nodes, flags), "execute")

    def execute_eager(self) -> None:
        check(self._lib, self._lib.rt_execute(self._nodes, self._n_nodes, RT_FLAG_EAGER), "execute")

    def upload_inputs(self, inputs: dict[str, np.ndarray]) -> None:
        for name, dev in self._in_dev.items():
            arr = np.ascontiguousarray(inputs[name], dtype=self._in_host[name].dtype)
            check(self._lib, self._lib.rt_upload(dev, arr.ctypes.data, arr.nbytes), "upload")

    def download_outputs(self) -> dict[str, np.ndarray]:
        out = {}
        for name, spec in self.program.outputs.items():
            arr = np.empty(spec["shape"], dtype=spec["dtype"])
            check(self._lib, self._lib.rt_download(arr.ctypes.data, self._resolve(spec["ref"]),
                                                   arr.nbytes), "download")
            out[name] = arr
        return out

    def input_buffer(self, name: str) -> np.ndarray:
        """Pinned host staging array of a graph input (write here: no host copy)."""
        return self._in_host[name]

    # ------------------------------------------------------ introspection
    @property
    def kernel_launches(self) -> int:
        n = self._lib.rt_kernel_launches(self._nodes, self._n_nodes)
        if n < 0:
            check(self._lib, -n, "kernel_launches")
        return n

    def profile_nodes(self, reps: int = 5) -> RunProfile:
        ms = (ctypes.c_float * self._n_nodes)()
        check(self._lib, self._lib.rt_profile(self._nodes, self._n_nodes, reps, ms), "profile")
        timings = [OpTiming(i, OP_NAME.get(n.op, str(n.op)), int(ms[i] * 1e6), f"node{i}",
                            tuple(n.out_shape)) for i, n in enumerate(self.program.nodes)]
        prof = RunProfile(timings, sum(t.time_ns for t in timings))
        self._last_profile = prof
        return prof

    @property
    def last_profile(self) -> RunProfile | None:
        return self._last_profile

    @property
    def node_array(self):
        return self._nodes

    @property
    def stream(self) -> int:
        return self._lib.rt_stream()

    # ------------------------------------------------------------ memory
    def _alloc(self, nbytes: int) -> int:
        p = self._lib.rt_alloc(nbytes)
        if not p:
            check(self._lib, self._lib.rt_last_error() or 9, f"rt_alloc({nbytes})")
        self._device_allocs.append(p)
        return p

    def _host_array(self, shape, dtype) -> np.ndarray:
        nbytes = int(np.prod(shape)) * np.dtype(dtype).itemsize
        p = self._lib.rt_host_alloc(max(nbytes, 1))
        if not p:
            check(self._lib, self._lib.rt_last_error() or 9, "rt_host_alloc")
        self._host_allocs.append(p)
        buf = (ctypes.c_char * max(nbytes, 1)).from_address(p)
        return np.frombuffer(buf, dtype=dtype, count=int(np.prod(shape))).reshape(shape)

    def close(self) -> None:
        lib = self._lib
        if self._device_allocs or self._host_allocs:
            lib.rt_synchronize()
            if self._nodes is not None:   # this graph's plan only; other executors keep theirs
                lib.rt_release(self._nodes, self._n_nodes)
        for p in self._device_allocs:
            lib.rt_free(p)
        for p in self._host_allocs:
            lib.rt_host_free(p)
        self._device_allocs, self._host_allocs = [], []
        self._nodes = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
