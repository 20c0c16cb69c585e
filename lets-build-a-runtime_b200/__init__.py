"""B200-native backend for the compiled executor of lets-build-a-runtime.

The reference's Python graph layer (export -> IR -> passes -> planner)
produces a planned graph; this package runs it on one B200 through one
C-ABI library, ``libb200exec.so`` (sources in ``csrc/``), whose entry point
``execute(OpNode*, int)`` is the reference's (csrc/executor.c:458).
"""
