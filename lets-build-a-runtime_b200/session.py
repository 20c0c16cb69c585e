"""Dynamic-shape bindings on the B200: one compiled graph per binding.

The reference re-plans and re-compiles on every ``Session.rebind``
(runtime/session.py:187-207): autoregressive decode re-plans each token
(run_gpt2.py:92-113).  On the GPU a compile means uploading the weights,
allocating an arena and capturing a CUDA graph, so this module keeps them:

* :class:`~executor.ConstantPool` -- weights uploaded once for all bindings
  (``resolve_graph`` shares the weight arrays between bindings,
  runtime/ops.py:589-613);
* :class:`BindingCache` -- per binding, the compiled executor (arena, node
  array, and through the library's plan cache its captured CUDA graph),
  least-recently-used first out beyond ``max_bindings``;
* :func:`b200_session_class` -- the reference ``Session`` with
  ``execution_mode="cuda"`` served by :class:`~executor.CudaCompiledExecutor`
  and ``rebind`` served from the cache (needs the reference's ``runtime``
  package, like ``CudaCompiledExecutor.compile``).
"""

from __future__ import annotations

from collections import OrderedDict
from typing import Callable, Hashable

from .executor import ConstantPool, CudaCompiledExecutor


def binding_key(bindings: dict[str, int] | None) -> tuple:
    return tuple(sorted((bindings or {}).items()))


class BindingCache:
    """Compiled executors keyed by binding, sharing one constant pool."""

    def __init__(self, device: int = 0, max_bindings: int = 16, lib_path=None) -> None:
        if max_bindings < 1:
            raise ValueError("max_bindings must be >= 1")
        self.device = device
        self.max_bindings = max_bindings
        self._lib_path = lib_path
        self.pool = ConstantPool(device, lib_path)
        self._execs: OrderedDict[Hashable, CudaCompiledExecutor] = OrderedDict()
        self.compiles = 0
        self.hits = 0

    def get(self, key: Hashable, compile_fn: Callable[[CudaCompiledExecutor], None],
            profile: bool = False) -> CudaCompiledExecutor:
        """The executor for ``key``; on a miss ``compile_fn(executor)`` compiles a
        fresh executor bound to the shared pool (e.g. ``ex.compile(plan)``)."""
        ex = self._execs.get(key)
        if ex is not None:
            self._execs.move_to_end(key)
            self.hits += 1
            return ex
        ex = CudaCompiledExecutor(profile=profile, device=self.device, lib_path=self._lib_path,
                                  constants=self.pool)
        compile_fn(ex)
        self.compiles += 1
        self._execs[key] = ex
        while len(self._execs) > self.max_bindings:
            _, old = self._execs.popitem(last=False)
            old.close()
        return ex

    def __contains__(self, key: Hashable) -> bool:
        return key in self._execs

    def __len__(self) -> int:
        return len(self._execs)

    def close(self) -> None:
        for ex in self._execs.values():
            ex.close()
        self._execs.clear()
        self.pool.clear()


def b200_session_class():
    """The reference ``Session`` with a ``"cuda"`` execution mode.

    ``create(execution_mode="cuda", bindings=...)`` optimizes, resolves and
    plans exactly like the reference, then compiles on the GPU;
    ``rebind(bindings)`` re-plans only bindings not seen before and otherwise
    switches to the cached executor (graph replay, no upload, no capture).
    Other execution modes behave as in the reference.
    """
    from runtime.ops import resolve_graph      # reference graph layer
    from runtime.planner import plan as plan_memory
    from runtime.session import Session

    class B200Session(Session):
        def __init__(self, graph, device: int = 0, max_bindings: int = 16) -> None:
            super().__init__(graph)
            self._bindings = BindingCache(device, max_bindings)
            self._binding = None

        def _make_executor(self, execution_mode, backend, profile=False):
            if execution_mode == "cuda":
                raise AssertionError("cuda executors come from the binding cache")
            return Session._make_executor(execution_mode, backend, profile)

        def create(self, execution_mode: str = "cuda", backend: str = "c", bindings=None, **kw) -> None:
            if execution_mode != "cuda":
                return super().create(execution_mode=execution_mode, backend=backend, bindings=bindings, **kw)
            # the reference pipeline up to the memory plan, then our compile
            holder = {}

            def capture(mode, be, profile=False):
                holder["profile"] = profile
                return _Deferred(holder)

            self._make_executor = capture          # intercept the reference's compile step
            try:
                super().create(execution_mode="compiled", backend=backend, bindings=bindings, **kw)
            finally:
                del self._make_executor
            self._execution_mode = "cuda"
            key = binding_key(bindings)
            self._binding = key
            self._executor = self._bindings.get(key, lambda ex: ex.compile(holder["plan"]),
                                                profile=holder.get("profile", False))

        def rebind(self, bindings: dict[str, int]) -> None:
            if self._execution_mode != "cuda":
                return super().rebind(bindings)
            key = binding_key(bindings)

            def compile_fn(ex):
                self._resolved = resolve_graph(self._graph, bindings)
                mp = plan_memory(self._resolved)
                self._plan_stats = mp.stats
                ex.compile(mp)

            self._executor = self._bindings.get(key, compile_fn, profile=self._profile)
            self._binding = key

        @property
        def binding_cache(self) -> BindingCache:
            return self._bindings

        def close(self) -> None:
            self._executor = None
            self._bindings.close()

    return B200Session


class _Deferred:
    """Stand-in executor for the reference ``create``: records the plan its
    compile step receives, so the session compiles it through the cache."""

    def __init__(self, holder: dict) -> None:
        self._holder = holder
        self._last_profile = None

    def compile(self, plan) -> None:
        self._holder["plan"] = plan
