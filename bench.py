"""Forward-pass benchmark of the CUDA compiled executor (and the reference arm).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config gpt2] [--impl b200|reference]

One step = one forward of the planned graph (by default the largest
single-GPU BASELINE configuration, configs[4]: the 1B-8K long-context block,
batch 8 x 8192 tokens, causal, fp32) through one `execute` of the node
array; `--config` selects the others (gpt2, qwen3, 7b, toy).  With N GPUs (torchrun, one process per
GPU) the batch of 8 is split into 8/N sequences per rank: each rank holds a
full weight replica, its own arena and CUDA graph; no collective is on the
data path (the only collectives are the timing barrier and max-reduction).

`value` = sequences/s of the whole job with inputs already resident in HBM;
`e2e` = the same through the public run() with pinned host inputs: PipelinedExecutor
(row chunks, copies overlapped with kernels) where a chunk program exists,
else CudaCompiledExecutor; the single-graph figure is reported beside it
and outputs (host->device and device->host copies inside the timed region).
The reference arm (--impl reference) times the reference's own C executor
(oracle/_ref, built from its sources) on the host cores for the same config.
For 7b and 1b8k (tens of seconds per batch-8 forward on the host) each step
is a bounded sample: one forward of the batch-1 program of the same graph
(every node treats batch rows independently, so a batch-8 forward is eight
such rows of work), reported as sequences/s.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
from __graft_entry__ import load_package  # noqa: E402

load_package()
from lbr_b200.program import OP, Program  # noqa: E402

GOLDEN = ROOT / "tests" / "golden"
CONFIGS = {
    "gpt2": "GPT-2-style 2-layer decoder body, d768 h12, causal, B8 S1024, fp32",
    "qwen3": "Qwen3-0.6B-shaped 2-layer body, d1024 GQA 16/8 hd128, RoPE, B8 S1024, fp32",
    "7b": "7B-shaped block d4096 h32 ff16384, non-causal, B8 S1024, fp32",
    "1b8k": "1B-8K block d2048 h16 ff8192, causal, B8 S8192, fp32",
    "toy": "toy block d64 h4 ff256, B1 S32, fp32",
}
GLOBAL_BATCH = {"gpt2": 8, "qwen3": 8, "7b": 8, "1b8k": 8, "toy": 1}
# Row chunks of the pipelined e2e run: the long 1b8k forward hides more of its
# PCIe copies behind kernels with smaller chunks.
E2E_CHUNKS = {"gpt2": 2, "qwen3": 2, "7b": 2, "1b8k": 8}
# Batch of the host-side sample timed for the CPU baseline / reference arm.
CPU_SAMPLE_BATCH = {"gpt2": 8, "qwen3": 8, "7b": 1, "1b8k": 1, "toy": 1}


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained"), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def program_name(cfg, b_local):
    return "toy" if cfg == "toy" else f"{cfg}_b{b_local}"


def node_flops(n):
    """Algorithmic flops of a contraction node (2*M*N*K; attention 4*BH*D*P)."""
    if n.op in (OP["MATMUL"], OP["MATMUL_ADD"]):
        N, K = n.out_shape[-1], n.extra[0]
        M = int(np.prod(n.out_shape[:-1]))
        return 2.0 * M * N * K
    if n.op == OP["ATTENTION"]:
        S, D, causal = n.extra[0], n.extra[1], n.extra[2]
        BH = int(np.prod(n.out_shape[:-2]))
        pairs = S * (S + 1) / 2 if causal else S * S
        return 4.0 * BH * D * pairs
    return 0.0


class ClockSampler:
    """SM clock and throttle reasons sampled during the timed region.

    NVML (nvidia_ml_py) polled every 10 ms from a thread; the nvidia-smi CLI
    (`-lms 100`) is the fallback when NVML is unavailable."""

    REASONS = {  # NVML clock-event reason bits
        "sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.samples = []       # (sm_mhz, reasons_mask)
        self.sm_max = None
        self._stop = threading.Event()
        self._thread = None

    def _poll_nvml(self):
        import pynvml
        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByIndex(self.gpu)
        self.sm_max = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
        get_reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
        while not self._stop.is_set():
            self.samples.append((pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM), get_reasons(h)))
            time.sleep(0.01)

    def _poll_smi(self):
        proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}",
                                 "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.active",
                                 "--format=csv,noheader,nounits", "-lms", "100"],
                                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        while not self._stop.is_set():
            line = proc.stdout.readline()
            if not line:
                break
            f = [x.strip() for x in line.split(",")]
            try:
                self.sm_max = float(f[1])
                self.samples.append((float(f[0]), int(f[2], 16)))
            except (ValueError, IndexError):
                pass
        proc.terminate()

    def __enter__(self):
        def run():
            try:
                self._poll_nvml()
            except Exception:
                try:
                    self._poll_smi()
                except Exception:
                    pass
        self._thread = threading.Thread(target=run, daemon=True)
        self._thread.start()
        time.sleep(0.05)
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._thread:
            self._thread.join(timeout=5)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.sm_max, "reasons": [], "samples": 0}
        mask = 0
        for _, m in self.samples:
            mask |= m
        reasons = sorted(k for k, bit in self.REASONS.items() if mask & bit)
        return {"sm_mhz": statistics.median(s for s, _ in self.samples), "sm_max_mhz": self.sm_max,
                "reasons": reasons, "samples": len(self.samples)}


def cpu_reference_run(prog, consts, inputs, budget_s, threads):
    """Time the reference C executor (oracle/_ref) or the restated oracle on the host."""
    import oracle
    kind = "reference" if oracle.available("reference") else "restated"
    if kind == "reference":
        oracle.set_threads(threads)
    from lbr_b200.copnode import HostBinding
    hb = HostBinding(prog, consts, inputs)
    oracle.execute(kind, hb)        # warm-up (page-in, BLAS thread start)
    times = []
    t_start = time.perf_counter()
    while True:
        t0 = time.perf_counter()
        oracle.execute(kind, hb)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_start > budget_s or len(times) >= 50:
            break
    return kind, statistics.median(times), len(times)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--config", default="1b8k", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--cpu-budget", type=float, default=15.0,
                    help="seconds of host time for the CPU baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-chunks", type=int, default=0,
                    help="row chunks of the pipelined e2e run (0: the per-config default)")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    n_gpus = max(args.gpus, world)
    gb = GLOBAL_BATCH[args.config]
    b_local = max(1, gb // n_gpus)
    metric = "forward throughput (sequences/s) and latency (ms)"
    unit = "sequences/s"

    if args.impl == "reference":
        return reference_arm(args, rank, world, n_gpus, gb, metric, unit)

    import torch
    import torch.distributed as dist
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    torch.cuda.set_device(local_rank)
    from lbr_b200.executor import CudaCompiledExecutor

    prog = Program.load(GOLDEN / f"{program_name(args.config, b_local)}.json")
    consts = prog.make_constants(0)
    inputs = prog.make_inputs(0, batch_offset=rank * b_local)
    ex = CudaCompiledExecutor(device=local_rank)
    ex.compile_program(prog, consts)
    ex.upload_inputs(inputs)
    ext = torch.cuda.ExternalStream(ex.stream, device=torch.device("cuda", local_rank))
    # L2 flush buffer (> 126 MB L2), written between timed steps on the same stream
    flush = torch.empty(256 * 2**20 // 4, dtype=torch.float32, device=f"cuda:{local_rank}")

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(max(args.warmup, 3)):
        ex.execute_resident(sync=False)
    ex._lib.rt_synchronize()

    # ---- device-resident timing: per-step CUDA events on the library stream
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clocks:
        for i in range(args.steps):
            with torch.cuda.stream(ext):
                flush.fill_(float(i))
                starts[i].record(ext)
            ex.execute_resident(sync=False)
            with torch.cuda.stream(ext):
                ends[i].record(ext)
        ex._lib.rt_synchronize()
        torch.cuda.synchronize()
        barrier()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    ms = sum(step_ms) / len(step_ms)

    # ---- end to end through the public API: pinned host in/out, copies inside
    host_in = {k: ex.input_buffer(k) for k in prog.inputs}
    for k, v in inputs.items():
        host_in[k][...] = v
    h2d = sum(v.nbytes for v in host_in.values())
    d2h = sum(int(np.prod(s["shape"])) * np.dtype(s["dtype"]).itemsize for s in prog.outputs.values())
    for _ in range(2):
        ex.run(host_in, copy_outputs=False)
    barrier()
    e2e_times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        ex.run(host_in, copy_outputs=False)
        e2e_times.append(time.perf_counter() - t0)
    barrier()
    e2e_ms = 1e3 * sum(e2e_times) / len(e2e_times)
    e2e_single_ms = e2e_ms
    # The same through PipelinedExecutor: the batch as row chunks (graphs
    # planned for b_local / chunks rows) whose host copies overlap each other's kernels.
    pipe = None
    chunks = args.e2e_chunks or E2E_CHUNKS.get(args.config, 2)
    while chunks > 1 and (b_local % chunks or
                          not (GOLDEN / f"{program_name(args.config, b_local // chunks)}.json").exists()):
        chunks //= 2
    if chunks > 1:
        from lbr_b200.pipeline import PipelinedExecutor
        cprog = Program.load(GOLDEN / f"{program_name(args.config, b_local // chunks)}.json")
        pipe = PipelinedExecutor(cprog, chunks, consts, device=local_rank)
        p_in = {k: pipe.input_buffer(k) for k in prog.inputs}
        for k, v in inputs.items():
            p_in[k][...] = v
        for _ in range(2):
            pipe.run(p_in, copy_outputs=False)
        barrier()
        p_times = []
        for _ in range(args.steps):
            t0 = time.perf_counter()
            pipe.run(p_in, copy_outputs=False)
            p_times.append(time.perf_counter() - t0)
        barrier()
        e2e_ms = 1e3 * sum(p_times) / len(p_times)
        pipe.close()

    # ---- per-node device times (eager launches bracketed by CUDA events)
    prof = ex.profile_nodes(reps=3)
    per_node_ms = [t.time_ns / 1e6 for t in prof.op_timings]

    if world > 1:
        t = torch.tensor([ms, e2e_ms, e2e_single_ms], device=f"cuda:{local_rank}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms, e2e_single_ms = t.tolist()

    launches = ex.kernel_launches
    if rank == 0:
        hbm, bf16, bf16_sus, basis = load_peaks()
        peak, peak_kind = (bf16_sus, "sustained") if bf16_sus else (bf16, "burst")
        gemm_ids = [i for i, n in enumerate(prog.nodes) if n.op in (OP["MATMUL"], OP["MATMUL_ADD"])]
        gemm_flops = sum(node_flops(prog.nodes[i]) for i in gemm_ids)
        gemm_ms = sum(per_node_ms[i] for i in gemm_ids)
        achieved = gemm_flops / (gemm_ms / 1e3) / 1e12 if gemm_ms else 0.0
        line = {
            "metric": metric, "value": round(gb / (ms / 1e3), 3), "unit": unit,
            "n_gpus": n_gpus, "steps": args.steps, "warmup": max(args.warmup, 3),
            "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None,
            "dtype": "f32 (contractions: fp32 operands as scaled fp16 hi / lo, three tensor-core MMAs per product)",
            "data": "synthetic: seeded N(0,0.02) weights, N(0,1) hidden states",
            "config": {"workload": CONFIGS[args.config], "program": program_name(args.config, b_local),
                       "global_batch": gb, "batch_per_gpu": b_local, "parallelism": f"dp{n_gpus}",
                       "l2": "256 MiB buffer written between timed steps (outside the step events)"},
            "latency_ms": round(ms, 4),
            "e2e": {"value": round(gb / (e2e_ms / 1e3), 3), "unit": unit, "latency_ms": round(e2e_ms, 4),
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                    "api": (f"PipelinedExecutor.run ({chunks} row chunks, copies overlapped with kernels)"
                            if pipe is not None else "CudaCompiledExecutor.run"),
                    "single_graph_value": round(gb / (e2e_single_ms / 1e3), 3)},
            "gpu_launches": launches * args.steps,
            "roofline": {"bound": "tensor", "kernel": "MATMUL/MATMUL_ADD nodes (sum, incl. their A split)",
                         "achieved": round(achieved, 3), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(achieved / peak, 4),
                         "traffic": GEMM_TRAFFIC.get(args.config),
                         "traffic_source": GEMM_TRAFFIC_SOURCE.get(args.config),
                         "peak_basis": f"{basis} bf16 dense, {peak_kind} (the GEMMs run inside a "
                                       f"seconds-long step)",
                         "frac_burst": round(achieved / bf16, 4),
                         # fp32 products from `slots` bf16-rate MMA slots each (fp16 hi / lo: 3)
                         "peak_split_effective": round(peak / GEMM_SLOTS[gemm_scheme()], 1),
                         "frac_split": round(achieved / (peak / GEMM_SLOTS[gemm_scheme()]), 4)},
            "roofline_attention": attention_roofline(prog, per_node_ms, peak),
            "clocks": clocks.summary(),
            "per_op_ms": summarize_ops(prog, per_node_ms),
        }
        if n_gpus == 1 and not args.no_cpu_baseline:
            threads = os.cpu_count() or 1
            sb = CPU_SAMPLE_BATCH[args.config]
            if sb == b_local:
                cprog, cconsts, cins = prog, consts, inputs
            else:
                cprog = Program.load(GOLDEN / f"{program_name(args.config, sb)}.json")
                cconsts, cins = cprog.make_constants(0), cprog.make_inputs(0)
            kind, t_cpu, runs = cpu_reference_run(cprog, cconsts, cins, args.cpu_budget, threads)
            line["cpu_baseline"] = {
                "value": round(sb / t_cpu, 4), "unit": unit, "cores": threads,
                "kind": "reference" if kind == "reference" else "port",
                "sample": f"{runs} forward(s) of program {program_name(args.config, sb)} ({sb} sequence(s)) "
                          f"on the host, median {t_cpu * 1e3:.1f} ms"}
        print(json.dumps(line), flush=True)
    ex.close()
    if world > 1:
        dist.destroy_process_group()


# DRAM bytes per GEMM launch from the committed ncu capture of this workload
# (mean of the two captured FFN launches), used as the roofline "traffic".
GEMM_TRAFFIC = {"gpt2": round((70.72 + 56.72 + 293.58 + 23.13) / 2 * 1e6),
                # 1b8k: mean over the four GEMMs of profiles/tc_gemm_pair_kernel_1b8k_b1.md (B1
                # capture, 574 MB per launch) scaled by the rows of a B8 launch (x8)
                "1b8k": round((303.24 + 174.15 + 85.55 + 27.80 + 839.96 + 242.60 + 561.09 + 61.64) / 4 * 8 * 1e6)}
GEMM_TRAFFIC_SOURCE = {"gpt2": "profiles/tc_gemm_pair_kernel_gpt2_b8.md (ncu dram__bytes_read+write, mean per "
                               "launch of the captured FFN GEMMs; tf32 + bf16 cross-term form)",
                       "1b8k": "profiles/tc_gemm_pair_kernel_1b8k_b1.md (ncu dram__bytes_read+write, mean per "
                               "launch of the four GEMMs at B1, scaled x8 to the B8 launch's rows)"}


# bf16-rate MMA slots per fp32 product of each operand scheme (the library's
# defaults and switches: RT_GEMM_SCHEME / RT_GEMM_3XTF32, RT_ATTN_SCHEME / RT_ATTN_3XTF32)
GEMM_SLOTS = {"f16": 3, "cross": 4, "3xtf32": 6}


def gemm_scheme():
    if os.environ.get("RT_GEMM_3XTF32") == "1" or os.environ.get("RT_GEMM_SCHEME") == "3xtf32":
        return "3xtf32"
    return "cross" if os.environ.get("RT_GEMM_SCHEME") == "cross" else "f16"


def attn_scheme():
    if os.environ.get("RT_ATTN_3XTF32") == "1" or os.environ.get("RT_ATTN_SCHEME") == "3xtf32":
        return "3xtf32"
    return "cross" if os.environ.get("RT_ATTN_SCHEME") == "cross" else "f16"


def attention_roofline(prog, per_node_ms, bf16):
    ids = [i for i, n in enumerate(prog.nodes) if n.op == OP["ATTENTION"]]
    if not ids:
        return None
    fl = sum(node_flops(prog.nodes[i]) for i in ids)
    ms = sum(per_node_ms[i] for i in ids)
    ach = fl / (ms / 1e3) / 1e12 if ms else 0.0
    return {"bound": "tensor", "kernel": "ATTENTION nodes (pack + attn_tc_kernel)", "achieved": round(ach, 3),
            "peak": bf16, "unit": "TFLOP/s", "frac": round(ach / bf16, 4),
            "frac_split": round(ach / (bf16 / GEMM_SLOTS[attn_scheme()]), 4)}


def summarize_ops(prog, per_node_ms):
    from lbr_b200.program import OP_NAME
    agg = {}
    for n, t in zip(prog.nodes, per_node_ms):
        k = OP_NAME.get(n.op, str(n.op))
        agg[k] = agg.get(k, 0.0) + t
    return {k: round(v, 4) for k, v in sorted(agg.items(), key=lambda kv: -kv[1])}


def reference_arm(args, rank, world, n_gpus, gb, metric, unit):
    """The reference's own C executor on the host cores, same config and metric."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    sb = CPU_SAMPLE_BATCH[args.config]
    prog = Program.load(GOLDEN / f"{program_name(args.config, sb)}.json")
    consts = prog.make_constants(0)
    inputs = prog.make_inputs(0)
    import oracle
    kind = "reference" if oracle.available("reference") else "restated"
    if kind == "reference":
        oracle.set_threads(threads)
    from lbr_b200.copnode import HostBinding
    hb = HostBinding(prog, consts, inputs)
    warm = 1 if sb < gb else max(1, min(args.warmup, 3))
    for _ in range(warm):
        oracle.execute(kind, hb)
    times = []
    steps = max(1, min(args.steps, 3 if sb < gb else 5))
    for _ in range(steps):
        t0 = time.perf_counter()
        oracle.execute(kind, hb)
        times.append(time.perf_counter() - t0)
    ms = 1e3 * statistics.median(times)
    value = sb / (ms / 1e3)
    line = {
        "impl": "reference", "metric": metric, "value": round(value, 4), "unit": unit,
        "n_gpus": n_gpus, "steps": steps, "warmup": warm,
        "ms_per_step": round(ms * gb / sb, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic: seeded N(0,0.02) weights, N(0,1) hidden states",
        "config": {"workload": CONFIGS[args.config], "program": program_name(args.config, sb),
                   "global_batch": gb, "parallelism": "host CPU"},
        "cpu_baseline": {"value": round(value, 4), "unit": unit, "cores": threads,
                         "kind": "reference" if kind == "reference" else "port",
                         "sample": f"{steps} forwards (median {ms:.1f} ms) of program "
                                   f"{program_name(args.config, sb)} ({sb} of the {gb} sequences; "
                                   f"ms_per_step scaled to the full batch) by the reference C executor "
                                   f"(csrc/executor.c + csrc/ops, OpenBLAS sgemm)"},
        "e2e": {"value": round(value, 4), "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
