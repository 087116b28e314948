"""Benchmark of the fused GEMM + bias + activation hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload NAME] [--no-extra]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N
    python bench.py --profile --workload NAME --steps 1 --warmup 2   (for ncu)

Headline workload: ``ffn_up_silu_8192x4096x14336_bf16`` —
Y = SiLU(X[8192,4096] @ W[4096,14336] + b), bf16 in/out, fp32 accumulate,
seeded synthetic inputs.  With N ranks, W and b are column-sharded
(N-slices of 14336/N), X is replicated, and each rank computes its slice of Y
with no collective: total work is fixed (strong scaling).

A step is one fused launch per rank.  `value` = 2*M*N*K / step time in
TFLOP/s (whole job), where the step time is the CUDA-event time of the
launch on the launching stream, summed over K steps, max over ranks.  L2 is
flushed (256 MiB write) before every timed launch, outside the events.
`e2e` is the same metric through the public host-buffer API
(`fused_linear_host`) with the step's inputs copied from pinned host memory
and Y copied back inside the timed region (copies overlapped with the
compute block by block).  `--impl reference` times the CPU reference arm: the
reference expression act(a @ b + bias) (kernel.py:64-66, ACTIVATION_PT of
fusion.py:87-92) in fp32 torch on all the host cores, on a bounded row sample
of the same workload.  At N=1 the line's `extra.reference_gpu_engines` also
times the reference's own GPU engines (its Triton and TileLang kernels, from
the reference package installed under baseline/_ref) beside this engine on
the same inputs.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "fused GEMM+bias+act TFLOP/s & % bf16 peak at 1/2/4/8 B200; decode HBM GB/s"
DEFAULT_WORKLOAD = "ffn_up_silu_8192x4096x14336_bf16"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
L2_FLUSH_BYTES = 256 << 20
L2_BYTES = 128 << 20  # B200 L2 (126 MB), rounded up
DATA = "synthetic: seeded X~N(0,1), W~N(0,1/K), bias~U(-0.1,0.1)"


def _peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text()), "measured"
        except ValueError:
            pass
    return dict(FALLBACK_PEAKS), "fallback"


def _dist_env() -> tuple[int, int, int]:
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def _traffic(workload: str, world: int):
    """DRAM bytes per launch from a committed ncu capture, if one exists."""
    p = ROOT / "profiles" / "dram_traffic.json"
    if not p.exists():
        return None
    try:
        data = json.loads(p.read_text())
    except ValueError:
        return None
    entry = data.get(f"{workload}@{world}") or (data.get(workload) if world == 1 else None)
    return entry.get("bytes_per_launch") if isinstance(entry, dict) else None


# --------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock, power and clock-event reasons of one GPU via NVML
    (what nvidia-smi reads) every `period` seconds in a background thread."""

    REASONS = {
        "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
        "hw_power_brake_slowdown": 0x80, "sw_power_cap": 0x4,
    }

    def __init__(self, uuid: str | None, period: float = 0.002):
        self.samples: list[tuple[float, int, float, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self._handle = None
        self._nvml = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nvml = pynvml
            self._handle = (pynvml.nvmlDeviceGetHandleByUUID(uuid) if uuid
                            else pynvml.nvmlDeviceGetHandleByIndex(0))
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._handle, pynvml.NVML_CLOCK_SM)
        except Exception:  # NVML unavailable: report no clocks
            self._handle = None
        self.period = period

    def _run(self):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self._handle, nv.NVML_CLOCK_SM)
                pw = nv.nvmlDeviceGetPowerUsage(self._handle) / 1000.0
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self._handle)
                self.samples.append((time.time(), sm, pw, rs))
            except Exception:
                pass
            self._stop.wait(self.period)

    def start(self):
        if self._handle is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def stop(self) -> dict | None:
        if self._thread is None:
            return None
        self._stop.set()
        self._thread.join()
        if not self.samples:
            return None
        loaded = [s for s in self.samples if s[2] > 200.0] or self.samples
        reasons = sorted({name for s in loaded for name, bit in self.REASONS.items() if s[3] & bit})
        return {"sm_mhz": statistics.median(s[1] for s in loaded), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(loaded),
                "power_w_max": round(max(s[2] for s in loaded), 1)}


# ------------------------------------------------------------ CPU arm
def _cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def cpu_reference_step(X, W, b, act: str) -> float:
    """One step of the CPU reference arm: the reference's own expression
    act(a @ b + bias) (kernel.py:64-66, fusion.py:87-92) in torch fp32 on
    the host cores, from the oracle's restatement; returns seconds."""
    import oracle
    t0 = time.perf_counter()
    oracle.torch_cpu.fused_linear(X, W, b, act)
    return time.perf_counter() - t0


def _cpu_sample(w, rows: int, W_host=None):
    """fp32 host copies of a bounded row sample of the workload's inputs."""
    from deepx_op_gpukernelcompiler_b200.workloads import make_inputs
    inp = make_inputs(w, device="cpu", M=rows)
    W = (W_host if W_host is not None else inp["W"]).float().contiguous()
    return inp["X"].float().contiguous(), W, inp["bias"].float().contiguous()


def cpu_baseline(w, W_host=None, target_s: float = 8.0) -> dict:
    """The reference's CPU expression (torch fp32, all host cores) timed on a
    bounded row sample of the workload; value in TFLOP/s."""
    import oracle
    threads = oracle.torch_cpu.use_threads()
    rows0 = min(w.M, 64)
    X, W, b = _cpu_sample(w, rows0, W_host)
    cpu_reference_step(X, W, b, w.act)  # warm the thread pool
    t = cpu_reference_step(X, W, b, w.act)
    rows = int(min(w.M, max(rows0, rows0 * target_s / max(t, 1e-6) / 2)))
    X, _, _ = _cpu_sample(w, rows, W_host)
    reps, elapsed = 0, 0.0
    while reps < 2 or elapsed < target_s * 0.5:
        elapsed += cpu_reference_step(X, W, b, w.act)
        reps += 1
        if elapsed > target_s * 1.5:
            break
    flops = 2.0 * rows * w.K * W.shape[1] * reps
    return {"value": round(flops / elapsed / 1e12, 4), "unit": "TFLOP/s",
            "cores": threads, "kind": "port",
            "sample": f"{reps} x act(X[{rows},{w.K}] @ W[{w.K},{W.shape[1]}] + b) in fp32, torch "
                      f"CPU on {threads} threads (kernel.py:64-66 restated), {elapsed:.1f} s"}


def cpu_baseline_config(w, target_s: float = 2.0) -> dict:
    """The reference's CPU expression on a bounded row sample of any
    configuration (single linear or the MLP chain), torch fp32 on all host
    cores; value in the configuration's unit (TFLOP/s, GB/s for decode)."""
    import oracle
    from deepx_op_gpukernelcompiler_b200.workloads import make_inputs
    threads = oracle.torch_cpu.use_threads()
    rows = min(w.M, 256)
    inp = {k: v.float() for k, v in make_inputs(w, device="cpu", M=rows).items()}
    if w.mlp:
        fn = lambda: oracle.torch_cpu.mlp_residual(inp["X"], inp["W1"], inp["b1"],  # noqa: E731
                                                   inp["W2"], inp["b2"], w.act)
    else:
        fn = lambda: oracle.torch_cpu.fused_linear(inp["X"], inp["W"], inp["bias"], w.act)  # noqa
    fn()
    reps, elapsed = 0, 0.0
    while reps < 2 or elapsed < target_s:
        t0 = time.perf_counter()
        fn()
        elapsed += time.perf_counter() - t0
        reps += 1
    per = elapsed / reps
    flops = (4 if w.mlp else 2) * rows * w.K * w.N
    line = {"value": round(flops / per / 1e12, 4), "unit": "TFLOP/s", "cores": threads,
            "kind": "port", "ms_per_sample": round(per * 1e3, 3),
            "sample": f"{reps} x the configuration on X[{rows},{w.K}] (of {w.M} rows), fp32 torch "
                      f"CPU on {threads} threads"}
    if w.name.startswith("decode"):
        line.update(value=round(w.min_bytes * rows / w.M / per / 1e9, 2), unit="GB/s")
    return line


def run_reference(args) -> None:
    rank, world, _ = _dist_env()
    if rank != 0:
        return
    import oracle
    from deepx_op_gpukernelcompiler_b200.workloads import WORKLOADS

    threads = oracle.torch_cpu.use_threads()
    w = WORKLOADS[args.workload]
    rows = 512 if w.M >= 512 else w.M
    X, W, b = _cpu_sample(w, rows)
    for _ in range(args.warmup):
        cpu_reference_step(X, W, b, w.act)
    times = [cpu_reference_step(X, W, b, w.act) for _ in range(args.steps)]
    total = sum(times)
    flops_step = 2.0 * rows * w.K * w.N
    value = flops_step * len(times) / total / 1e12
    line = {
        "metric": METRIC, "impl": "reference", "value": round(value, 4), "unit": "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total / len(times) * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": DATA,
        "config": {"workload": w.name, "M": w.M, "K": w.K, "N": w.N, "act": w.act,
                   "sample_rows_per_step": rows, "parallelism": "host cores (rank 0)"},
        "cpu_baseline": {"value": round(value, 4), "unit": "TFLOP/s", "cores": threads,
                         "kind": "port",
                         "sample": f"per step act(X[{rows},{w.K}] @ W[{w.K},{w.N}] + b), fp32 "
                                   f"torch CPU on {threads} threads: the reference expression "
                                   "kernel.py:64-66 with fusion.py:87-92 activations, restated"},
        "e2e": {"value": round(value, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------ parity
def _sample_rows(M: int, rows: int = 16) -> list[tuple[int, int]]:
    """First, middle and last row blocks of an M-row output."""
    mid = max(0, M // 2 - rows // 2)
    return sorted({(0, min(rows, M)), (mid, min(M, mid + rows)), (max(0, M - rows), M)})


def _row_index(M: int):
    import numpy as np
    return np.concatenate([np.arange(a, b) for a, b in _sample_rows(M)])


def _parity(got_rows, want, rtol: float, atol: float) -> dict:
    """Row sample of the engine's output against the fp64 oracle's rows."""
    import numpy as np
    g = got_rows.float().cpu().numpy()
    err = np.abs(g - want)
    ok = bool((err <= atol + rtol * np.abs(want)).all())
    return {"ok": ok, "max_abs_err": float(err.max()) if err.size else 0.0,
            "rows": int(g.shape[0]), "tol": [rtol, atol]}


def _linear_parity(X, W, b, act, Y, rtol=2e-2, atol=2e-2) -> dict:
    """act(X W + b) on sampled rows of X, fp64 oracle, against Y's rows."""
    import oracle
    idx = _row_index(X.shape[0])
    want = oracle.fused_linear_f64(X[idx].float().cpu().numpy(), W.float().cpu().numpy(),
                                   b.float().cpu().numpy() if b is not None else None, act)
    return _parity(Y[idx], want, rtol, atol)


def _row_parallel_parity(X, first_fn, W2, b2, residual: bool, out, world, dev) -> dict:
    """Sampled rows of Y = sum_r first_r(X) W2_r + b2 (+ X), each rank adding
    its own term in fp64 (oracle) and the terms summed over ranks, against
    this rank's output rows."""
    import oracle
    import torch
    import torch.distributed as dist
    idx = _row_index(X.shape[0])
    Xr = X[idx].float().cpu().numpy()
    H = first_fn(Xr)
    part = torch.from_numpy(oracle.fused_linear_f64(H, W2.float().cpu().numpy(), None, None))
    part = part.to(dev)
    if world > 1:
        dist.all_reduce(part)
    want = part.cpu().numpy() + b2.float().cpu().numpy()
    if residual:
        want = want + Xr
    return _parity(out[idx], want, 2e-2, 2e-2)


# ------------------------------------------------------------ GPU arm
def _time_launches(fn, steps, flush, stream, host_us_per_step: float = 80.0):
    """CUDA-event time of each launch (flush outside the events), ms list.

    A device-side sleep is queued first, long enough for the host to enqueue
    every step behind it, so no event pair brackets host enqueue time."""
    import torch
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(steps)]
    torch.cuda._sleep(int(steps * host_us_per_step * 1e-6 * 2.0e9))
    for s, e in evs:
        flush()
        s.record(stream)
        fn()
        e.record(stream)
    torch.cuda.synchronize()
    return [s.elapsed_time(e) for s, e in evs]


def _time_back_to_back(fn, steps, stream, host_us_per_step: float = 80.0) -> float:
    """CUDA-event time of `steps` consecutive launches (one event pair around
    all of them, a device-side sleep first so the host has enqueued them all
    before they start), in ms per launch.  For kernels whose inputs already
    defeat L2 (rotated weight copies), this is the launch-to-launch
    throughput; per-launch event pairs would add their own latency to every
    launch of a ~10 us kernel."""
    import torch
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda._sleep(int(steps * host_us_per_step * 1e-6 * 2.0e9))
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def _max_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def run_gpu(args) -> None:
    import torch
    import torch.distributed as dist

    from deepx_op_gpukernelcompiler_b200 import _native, fused_linear
    from deepx_op_gpukernelcompiler_b200.shard import shard_bounds
    from deepx_op_gpukernelcompiler_b200.workloads import WORKLOADS

    rank, world, local = _dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    peaks, peak_kind = _peaks()
    w = WORKLOADS[args.workload]
    n0, n1 = shard_bounds(w.N, world, rank, 64)
    if args.shard_of > 1:
        # One GPU running rank 0's share of an N-way column split.
        n0, n1 = shard_bounds(w.N, args.shard_of, 0, 64)
    n_loc = n1 - n0

    # Inputs: X replicated, this rank's W/bias column shard; seeded on device.
    gen = torch.Generator(device=dev)
    gen.manual_seed(w.seed * 1000 + rank)
    dt = w.torch_dtype
    X = torch.randn(w.M, w.K, generator=gen, device=dev).to(dt)
    Wt = (torch.randn(w.K, n_loc, generator=gen, device=dev) / math.sqrt(w.K)).to(dt)
    b = (torch.rand(n_loc, generator=gen, device=dev) * 0.2 - 0.1).to(dt)
    Y = torch.empty(w.M, n_loc, dtype=dt, device=dev)
    flush_buf = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    if w.gated:
        if not args.profile:
            raise SystemExit(f"{w.name} runs in --profile mode (its bench line is an extra)")
        from deepx_op_gpukernelcompiler_b200 import fused_gated_linear
        Wu = (torch.randn(w.K, n_loc, generator=gen, device=dev) / math.sqrt(w.K)).to(dt)
        bu = (torch.rand(n_loc, generator=gen, device=dev) * 0.2 - 0.1).to(dt)

    def step():
        if w.gated:
            fused_gated_linear(X, Wt, Wu, b, bu, w.act, out=Y)
        else:
            fused_linear(X, Wt, b, w.act, out=Y)

    def flush():
        flush_buf.zero_()

    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        pass
    sampler = ClockSampler(uuid).start()

    # Warm-up: at least W steps and ~1 s of work so clocks settle.
    for _ in range(max(1, args.warmup)):
        step()
    torch.cuda.synchronize()
    plan = _native.last_launch_plan()
    if args.profile:
        # Profiling mode: exactly W warm-up + K timed launches, nothing else.
        times = _time_launches(step, args.steps, flush, stream)
        sampler.stop()
        print(json.dumps({"profile": w.name, "rank": rank, "launch_ms": times, "plan": plan}),
              flush=True)
        if world > 1:
            dist.destroy_process_group()
        return
    _barrier(world)
    torch.cuda.synchronize()
    times = _time_launches(step, args.steps, flush, stream)
    torch.cuda.synchronize()
    _barrier(world)
    clocks = sampler.stop()
    status = _native.device_status(stream.cuda_stream)
    if status:
        raise RuntimeError(f"device status {status}: a kernel wait timed out")

    parity = {"headline_shard": _linear_parity(X, Wt, b, w.act, Y)}

    local_ms = sum(times)
    total_ms = _max_over_ranks(local_ms, world, dev)
    ms_step = total_ms / args.steps
    flops_total = 2.0 * w.M * w.N * w.K
    value = flops_total / (ms_step * 1e-3) / 1e12
    flops_rank = 2.0 * w.M * n_loc * w.K
    achieved = flops_rank / (local_ms / args.steps * 1e-3) / 1e12
    peak = peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])

    # End to end through the public API: pinned host inputs in, Y out.
    Xh = X.cpu().pin_memory()
    Wh = Wt.cpu().pin_memory()
    bh = b.cpu().pin_memory()
    Yh = torch.empty(w.M, n_loc, dtype=dt).pin_memory()

    from deepx_op_gpukernelcompiler_b200 import fused_linear_host

    def e2e_step():
        # X, W, b copied in and Y copied out every step, block by block, the
        # copies overlapping the fused launches (fused_linear_host).
        fused_linear_host(Xh, Wh, bh, w.act, out=Yh, device=dev)

    e2e_steps = max(3, min(args.steps, 10))
    e2e_step()
    torch.cuda.synchronize()
    _barrier(world)
    e2e_times = _time_launches(e2e_step, e2e_steps, lambda: None, stream)
    _barrier(world)
    e2e_ms = _max_over_ranks(sum(e2e_times), world, dev) / e2e_steps
    esz = torch.finfo(dt).bits // 8
    h2d = (w.M * w.K + w.K * n_loc + n_loc) * esz
    d2h = w.M * n_loc * esz

    # Sustained: back-to-back launches (no flush) for ~1.5 s under the power
    # cap, against the sustained bf16 peak.
    sus_n = max(20, int(1.5 / max(ms_step * 1e-3, 1e-6)))
    _barrier(world)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sus_sampler = ClockSampler(uuid).start()
    ev0.record(stream)
    for _ in range(sus_n):
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    sus_clocks = sus_sampler.stop()
    sus_ms = _max_over_ranks(ev0.elapsed_time(ev1), world, dev) / sus_n
    sus_tf = flops_total / (sus_ms * 1e-3) / 1e12
    peak_sus = peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"])
    sustained = {"value": round(sus_tf, 2), "unit": "TFLOP/s", "ms": round(sus_ms, 4),
                 "launches": sus_n, "peak": peak_sus,
                 "frac": round(sus_tf / world / peak_sus, 4),
                 "peak_source": f"bf16_tflops_sustained, {peak_kind}", "clocks": sus_clocks}

    # The reference's own GPU comparator (kernel.py:84-91): torch `a @ b + bias`
    # then the activation, as separate kernels (cuBLAS + elementwise).
    act_fn = {"silu": torch.nn.functional.silu, "relu": torch.relu,
              "gelu_tanh": lambda t: torch.nn.functional.gelu(t, approximate="tanh"),
              "gelu_erf": torch.nn.functional.gelu}.get(w.act, lambda t: t)

    def torch_step():
        act_fn(X @ Wt + b)

    for _ in range(3):
        torch_step()
    torch.cuda.synchronize()
    _barrier(world)
    pt_times = _time_launches(torch_step, min(args.steps, 20), flush, stream)
    pt_ms = _max_over_ranks(sum(pt_times), world, dev) / len(pt_times)
    pytorch_gpu = {"value": round(flops_total / (pt_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                   "ms": round(pt_ms, 4),
                   "what": "torch act(X @ W + b) on the GPU (cuBLAS + elementwise), kernel.py:84-91"}

    extra = {"sustained": sustained, "pytorch_gpu": pytorch_gpu}
    if not args.no_extra:
        extra.update(run_extras(args, world, rank, dev, peaks, flush, parity))
        if world == 1 and not args.no_ref_engines:
            extra["reference_gpu_engines"] = run_reference_engines(args, dev, peaks, flush)
    # Parity of every rank's outputs: the line says ok only if all ranks agree.
    ok_all = all(v["ok"] for v in parity.values())
    if world > 1:
        flag = torch.tensor([1 if ok_all else 0], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        ok_all = bool(flag.item())
    if clocks and clocks.get("sm_mhz"):
        # Clock-normalised step time: thousands of SM cycles per step.
        clocks["kcycles_per_step"] = round(ms_step * clocks["sm_mhz"], 1)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(w, W_host=Wt.cpu())
        # The other configurations of the metric, same CPU expression.
        extra["cpu_baselines"] = {name: cpu_baseline_config(WORKLOADS[name]) for name in (
            "linear_relu_256x512x512_f32", "linear_gelu_tanh_4096x4096x4096_bf16",
            "decode_gelu_erf_16x8192x28672_f16", "mlp_residual_16384x4096x16384_bf16")}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16" if dt == torch.bfloat16 else str(dt).replace("torch.", ""),
            "data": DATA,
            "config": {"workload": w.name, "M": w.M, "K": w.K, "N": w.N, "act": w.act,
                       "parallelism": f"column-parallel N-shard x{world} (no collective)",
                       "n_per_rank": n_loc, "l2": "flushed before each timed launch (256 MiB write)",
                       "kernel": plan},
            "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak,
                         "unit": "TFLOP/s", "frac": round(achieved / peak, 4),
                         "peak_source": f"bf16_tflops burst, {peak_kind}",
                         "traffic": _traffic(w.name, world)},
            "e2e": {"value": round(flops_total / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                    "ms_per_step": round(e2e_ms, 3), "h2d_bytes_per_step": h2d * world,
                    "d2h_bytes_per_step": d2h * world,
                    "api": "deepx_op_gpukernelcompiler_b200.fused_linear_host (C ABI dx_fused_linear "
                           "per output block, dx_copy_2d_async for the copies)"},
            "gpu_launches": args.steps,
            "clocks": clocks,
            "parity": {"ok": ok_all, "all_ranks": world, "oracle": "fp64 C restatement of "
                       "act(a @ b + bias) (kernel.py:64-66) on sampled rows",
                       "items": parity},
            "extra": extra,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.cuda.synchronize()  # nothing of ours in flight before any rank leaves
        dist.barrier()
        dist.destroy_process_group()


def run_extras(args, world, rank, dev, peaks, flush, parity) -> dict:
    """The other workloads of the metric: decode HBM GB/s, the square GEMM,
    the fp32 configuration, the gated dual GEMM and the two row-parallel
    chains (all ranks take part; timings are max over ranks).  Each adds its
    oracle check of sampled output rows to `parity`."""
    import torch
    from deepx_op_gpukernelcompiler_b200 import _native, fused_linear
    from deepx_op_gpukernelcompiler_b200.shard import shard_bounds
    from deepx_op_gpukernelcompiler_b200.workloads import WORKLOADS

    out = {}
    stream = torch.cuda.current_stream(dev)
    steps = max(5, min(args.steps, 20))
    hbm = peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
    tflops_peak = peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])

    # Decode: GELU-erf(X[16,8192] W[8192,28672] + b), fp16, N-sharded.
    w = WORKLOADS["decode_gelu_erf_16x8192x28672_f16"]
    n0, n1 = shard_bounds(w.N, world, rank, 64)
    n_loc = n1 - n0
    g = torch.Generator(device=dev)
    g.manual_seed(w.seed * 1000 + rank)
    X = torch.randn(w.M, w.K, generator=g, device=dev).to(w.torch_dtype)
    # Rotated weight copies, together at least 3x the L2 size: every step
    # streams W from HBM without an L2 flush (whose dirty lines would be
    # written back during the timed launch).
    copies = max(2, math.ceil(3 * L2_BYTES / (w.K * n_loc * 2)))
    Ws = [(torch.randn(w.K, n_loc, generator=g, device=dev) / math.sqrt(w.K)).to(w.torch_dtype)
          for _ in range(copies)]
    b = (torch.rand(n_loc, generator=g, device=dev) * 0.2 - 0.1).to(w.torch_dtype)
    Y = torch.empty(w.M, n_loc, dtype=w.torch_dtype, device=dev)
    it = [0]

    def dec():
        fused_linear(X, Ws[it[0] % copies], b, w.act, out=Y)
        it[0] += 1

    for _ in range(5):
        dec()
    torch.cuda.synchronize()
    dec_plan = _native.last_launch_plan()
    _barrier(world)
    t = _time_launches(dec, steps, lambda: None, stream)
    ms_each = _max_over_ranks(sum(t), world, dev) / steps
    _barrier(world)
    local_b2b = _time_back_to_back(dec, 4 * steps, stream)
    ms = _max_over_ranks(local_b2b, world, dev)
    fused_linear(X, Ws[0], b, w.act, out=Y)
    parity["decode_shard"] = _linear_parity(X, Ws[0], b, w.act, Y)
    bytes_rank = 2 * (w.M * w.K + w.K * n_loc + n_loc + w.M * n_loc)
    bytes_total = w.min_bytes
    out[w.name] = {"value": round(bytes_total / (ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                   "ms": round(ms, 4), "kernel": dec_plan,
                   "timing": f"{4 * steps} back-to-back launches between one event pair",
                   "ms_with_event_pair_per_launch": round(ms_each, 4),
                   "roofline": {"bound": "hbm", "achieved": round(bytes_rank / (local_b2b * 1e-3) / 1e9, 1),
                                "peak": hbm, "unit": "GB/s",
                                "frac": round(bytes_rank / (local_b2b * 1e-3) / 1e9 / hbm, 4)},
                   "l2": f"{copies} rotated weight copies (>= 3x L2), no flush"}
    del Ws, X, Y

    # Square GEMM: GELU-tanh(X[4096,4096] W[4096,4096] + b), bf16 (per rank
    # an N-slice, no collective).
    w = WORKLOADS["linear_gelu_tanh_4096x4096x4096_bf16"]
    n0, n1 = shard_bounds(w.N, world, rank, 64)
    n_loc = n1 - n0
    X = torch.randn(w.M, w.K, generator=g, device=dev).to(w.torch_dtype)
    Wt = (torch.randn(w.K, n_loc, generator=g, device=dev) / math.sqrt(w.K)).to(w.torch_dtype)
    b = (torch.rand(n_loc, generator=g, device=dev) * 0.2 - 0.1).to(w.torch_dtype)
    Y = torch.empty(w.M, n_loc, dtype=w.torch_dtype, device=dev)

    def sq():
        fused_linear(X, Wt, b, w.act, out=Y)

    for _ in range(5):
        sq()
    torch.cuda.synchronize()
    sq_plan = _native.last_launch_plan()
    _barrier(world)
    t = _time_launches(sq, steps, flush, stream)
    ms = _max_over_ranks(sum(t), world, dev) / steps
    parity["square_shard"] = _linear_parity(X, Wt, b, w.act, Y)
    tf = w.flops / (ms * 1e-3) / 1e12
    out[w.name] = {"value": round(tf, 2), "unit": "TFLOP/s", "ms": round(ms, 4),
                   "frac_of_peak": round(tf / world / tflops_peak, 4), "kernel": sq_plan}
    del X, Wt, b, Y

    # The reference's CPU-runnable configuration on the GPU: ReLU(X[256,512]
    # W[512,512] + b) in exact fp32 (every rank runs the whole problem).
    w = WORKLOADS["linear_relu_256x512x512_f32"]
    from deepx_op_gpukernelcompiler_b200.workloads import make_inputs
    inp = make_inputs(w, device="cpu")
    X, Wt, b = (inp[k].to(dev) for k in ("X", "W", "bias"))
    Y = torch.empty(w.M, w.N, dtype=torch.float32, device=dev)

    def f32():
        fused_linear(X, Wt, b, w.act, out=Y)

    for _ in range(5):
        f32()
    torch.cuda.synchronize()
    f32_plan = _native.last_launch_plan()
    _barrier(world)
    t = _time_launches(f32, steps, flush, stream)
    ms = _max_over_ranks(sum(t), world, dev) / steps
    parity["fp32_relu_256x512x512"] = _linear_parity(X, Wt, b, w.act, Y, 1e-4, 1e-4)
    out[w.name] = {"value": round(ms * 1e3, 2), "unit": "us per launch (lower is better)",
                   "tflops": round(w.flops / (ms * 1e-3) / 1e12, 3), "kernel": f32_plan,
                   "bound": "latency (0.134 GFLOP, exact fp32 FFMA)"}
    del X, Wt, b, Y

    # Gated FFN's gate/up projections in one dual-GEMM launch:
    # H = silu(X Wg + bg) * (X Wu + bu), X[8192,4096], Wg/Wu[4096,14336] (per
    # rank an N-slice of both, no collective).
    M_g, K_g, N_g = 8192, 4096, 14336
    n0, n1 = shard_bounds(N_g, world, rank, 64)
    n_loc = n1 - n0
    X = torch.randn(M_g, K_g, generator=g, device=dev).to(torch.bfloat16)
    Wg = (torch.randn(K_g, n_loc, generator=g, device=dev) / math.sqrt(K_g)).to(torch.bfloat16)
    Wu = (torch.randn(K_g, n_loc, generator=g, device=dev) / math.sqrt(K_g)).to(torch.bfloat16)
    bg = (torch.rand(n_loc, generator=g, device=dev) * 0.2 - 0.1).to(torch.bfloat16)
    bu = (torch.rand(n_loc, generator=g, device=dev) * 0.2 - 0.1).to(torch.bfloat16)
    Y = torch.empty(M_g, n_loc, dtype=torch.bfloat16, device=dev)
    from deepx_op_gpukernelcompiler_b200 import fused_gated_linear

    def gated():
        fused_gated_linear(X, Wg, Wu, bg, bu, "silu", out=Y)

    for _ in range(3):
        gated()
    torch.cuda.synchronize()
    _barrier(world)
    t = _time_launches(gated, steps, flush, stream)
    ms = _max_over_ranks(sum(t), world, dev) / steps
    idx = _row_index(M_g)
    import oracle
    parity["gated_dual_gemm_shard"] = _parity(Y[idx], oracle.gated_linear_f64(
        X[idx].float().cpu().numpy(), Wg.float().cpu().numpy(), bg.float().cpu().numpy(),
        Wu.float().cpu().numpy(), bu.float().cpu().numpy(), "silu"), 2e-2, 2e-2)
    tf = 2 * 2 * M_g * N_g * K_g / (ms * 1e-3) / 1e12
    out[f"ffn_gated_gate_up_{M_g}x{K_g}x{N_g}_bf16"] = {
        "value": round(tf, 2), "unit": "TFLOP/s", "ms": round(ms, 4),
        "frac_of_peak": round(tf / world / tflops_peak, 4), "kernel": "umma gated (dual GEMM)"}
    del X, Wg, Wu, bg, bu, Y

    out.update(run_mlp_extras(args, world, rank, dev, peaks, flush, parity, g))
    return out


REF_PKG = ROOT / "baseline" / "_ref" / "deepx_op_gpukernelcompiler"


def _reference_module(name: str):
    """One module of the reference package installed under baseline/_ref,
    imported by file path and unmodified (the package's __init__ imports the
    kvspace client, which its engine modules do not need)."""
    import importlib.util
    path = REF_PKG / f"{name}.py"
    if not path.exists():
        raise FileNotFoundError(f"{path} (install the reference into baseline/_ref)")
    spec = importlib.util.spec_from_file_location(f"_deepx_reference_{name}", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def run_reference_engines(args, dev, peaks, flush) -> dict:
    """The reference's own GPU engines on this B200, beside this engine, on the
    same fp16 inputs: its Triton kernel (kernel_triton.py:24-89, autotuned
    over its own config list on first call) and its TileLang kernel
    (kernel_tilelang.py:23-55, with the harness's default block
    BM=BN=128, BK=32, kernel.py:10).  Both compute the GELU of the
    `"gelu"` key with erf, so this engine runs "gelu_erf" there.  Same
    timing as the other GEMM lines: one event pair per launch, L2 flushed
    before each.  Speed only (the reference engines store fp16); each line
    carries the max |diff| of its output from this engine's.  An engine that
    fails to build or run is recorded with its error, not retried."""
    import torch
    from deepx_op_gpukernelcompiler_b200 import fused_linear

    stream = torch.cuda.current_stream(dev)
    steps = max(5, min(args.steps, 10))
    tflops_peak = peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])
    mods, out = {}, {"source": "unmodified reference package, baseline/_ref",
                     "timing": "one event pair per launch, L2 flushed before each"}
    for name in ("kernel_triton", "kernel_tilelang"):
        try:
            mods[name] = _reference_module(name)
        except Exception as e:  # noqa: BLE001 - recorded in the line
            out[name] = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
    g = torch.Generator(device=dev)
    g.manual_seed(4242)
    for M, K, N, act in ((4096, 4096, 4096, "gelu"), (8192, 4096, 14336, "silu")):
        flops = 2.0 * M * N * K
        X = torch.randn(M, K, generator=g, device=dev).half()
        W = (torch.randn(K, N, generator=g, device=dev) / math.sqrt(K)).half()
        b = (torch.rand(N, generator=g, device=dev) * 0.2 - 0.1).half()
        Y = torch.empty(M, N, dtype=torch.float16, device=dev)
        ours_act = "gelu_erf" if act == "gelu" else act
        fns = {"b200": lambda: fused_linear(X, W, b, ours_act, out=Y)}
        if "kernel_triton" in mods:
            fns["triton"] = (lambda f: (lambda: f(X, W, b)))(
                mods["kernel_triton"].make_linear_kernel(act))
        row = {}
        t0 = time.time()
        if "kernel_tilelang" in mods:
            try:
                tl = mods["kernel_tilelang"].make_linear_kernel(act)(
                    M, N, K, 128, 128, 32, "float16", "float32")
                fns["tilelang"] = (lambda f: (lambda: f(X, W, b)))(tl)
            except Exception as e:  # noqa: BLE001
                row["tilelang"] = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
        ref_y = None
        for eng, fn in fns.items():
            try:
                t1 = time.time()
                r = fn()
                torch.cuda.synchronize()
                first_s = time.time() - t1
                got = Y if eng == "b200" else r
                if eng == "b200":
                    ref_y = Y.float()
                diff = None if ref_y is None else float((got.float() - ref_y).abs().max())
                for _ in range(3):
                    fn()
                torch.cuda.synchronize()
                t = _time_launches(fn, steps, flush, stream)
                ms = sum(t) / len(t)
                tf = flops / (ms * 1e-3) / 1e12
                row[eng] = {"ms": round(ms, 4), "tflops": round(tf, 2),
                            "frac_of_peak": round(tf / tflops_peak, 4),
                            "max_abs_diff_vs_b200": None if eng == "b200" else round(diff, 4),
                            "first_call_s": round(first_s, 2)}
            except Exception as e:  # noqa: BLE001
                row[eng] = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
        if "tflops" in row.get("b200", {}):
            for eng in ("triton", "tilelang"):
                if "tflops" in row.get(eng, {}):
                    row[eng]["b200_speedup"] = round(row["b200"]["tflops"] / row[eng]["tflops"], 2)
        row["setup_s"] = round(time.time() - t0, 1)
        out[f"linear_{act}_{M}x{K}x{N}_f16"] = row
        del X, W, b, Y, fns
    return out


def run_mlp_extras(args, world, rank, dev, peaks, flush, parity, g) -> dict:
    """The two-layer MLP chain Y = GELU(X W1 + b1) W2 + b2 + X at
    X[16384,4096], hidden 16384: one GPU runs the two fused launches; N GPUs
    run column -> row parallel with the overlapped NVLink reduction (several
    chunkings, the fastest reported as the value) and with NCCL.  X and b2
    are the same on every rank (seeded alike), the weight shards differ."""
    import torch

    import oracle
    from deepx_op_gpukernelcompiler_b200.shard import (ParallelGatedFFN, ParallelMLP,
                                                       first_groups, row_chunks, row_schedule,
                                                       shard_bounds)
    from deepx_op_gpukernelcompiler_b200.workloads import WORKLOADS

    out = {}
    stream = torch.cuda.current_stream(dev)
    tflops_peak = peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])
    w = WORKLOADS["mlp_residual_16384x4096x16384_bf16"]
    h0, h1 = shard_bounds(w.N, world, rank, 64)
    h_loc = h1 - h0
    dt = w.torch_dtype
    g_shared = torch.Generator(device=dev)
    g_shared.manual_seed(w.seed)
    X = torch.randn(w.M, w.K, generator=g_shared, device=dev).to(dt)
    b2 = (torch.rand(w.K, generator=g_shared, device=dev) * 0.2 - 0.1).to(dt)
    W1 = (torch.randn(w.K, h_loc, generator=g, device=dev) / math.sqrt(w.K)).to(dt)
    b1 = (torch.rand(h_loc, generator=g, device=dev) * 0.2 - 0.1).to(dt)
    W2 = (torch.randn(h_loc, w.K, generator=g, device=dev) / math.sqrt(w.N)).to(dt)
    H = torch.empty(w.M, h_loc, dtype=dt, device=dev)
    Yo = torch.empty(w.M, w.K, dtype=dt, device=dev)
    W1c, b1c = W1.float().cpu().numpy(), b1.float().cpu().numpy()

    def first_ref(Xr):
        return oracle.fused_linear_f64(Xr, W1c, b1c, w.act)

    msteps = max(3, min(args.steps, 20) // 2)

    def time_run(run, host_us):
        for _ in range(3):
            run()
        torch.cuda.synchronize()
        _barrier(world)
        t = _time_launches(run, msteps, flush, stream, host_us)
        return _max_over_ranks(sum(t), world, dev) / msteps

    if world == 1:
        from deepx_op_gpukernelcompiler_b200 import mlp_residual
        ms = time_run(lambda: mlp_residual(X, W1, b1, W2, b2, w.act, hidden=H, out=Yo), 200.0)
        parity["mlp_chain"] = _row_parallel_parity(X, first_ref, W2, b2, True, Yo, world, dev)
        tf = w.flops / (ms * 1e-3) / 1e12
        out[w.name] = {"value": round(tf, 2), "unit": "TFLOP/s", "ms": round(ms, 4),
                       "frac_of_peak": round(tf / tflops_peak, 4),
                       "parallelism": "one GPU, two fused launches", "gpu_launches_per_step": 2}
    else:
        # Every schedule of the engine's reduction, in both NVLink forms: the
        # reduction carried by the GEMM launches at several chunkings, and
        # one chunk (the two whole GEMMs, then one reduction launch of its
        # own).  The fastest is the value; all are listed.
        sweep, modules = {}, {}
        for nvls in (True, False):
            mlp = ParallelMLP.from_shards(W1, b1, W2, b2, w.act, mode="fused", nvls=nvls)
            modules[nvls] = mlp
            for chunks, first in ((4, 4), (4, 2), (4, 1), (8, 4), (2, 2), (2, 1), (1, 1)):
                mlp.chunks, mlp.first_chunks = chunks, first
                ms = time_run(lambda: mlp(X, hidden=H, out=Yo), 1500.0)
                form = "multicast" if mlp.last_multicast else "peer"
                sweep[f"{form},chunks={chunks},first={first}"] = round(ms, 4)
        best = min(sweep, key=sweep.get)
        form, chunks, first = best.split(",")
        chunks, first = int(chunks.split("=")[1]), int(first.split("=")[1])
        mlp = modules[True] if form == "multicast" else modules[False]
        mlp.chunks, mlp.first_chunks = chunks, first
        ms = time_run(lambda: mlp(X, hidden=H, out=Yo), 1500.0)
        assert mlp.last_path == "fused"
        multicast = mlp.last_multicast
        parity["mlp_fused"] = _row_parallel_parity(X, first_ref, W2, b2, True, Yo, world, dev)
        tf = w.flops / (ms * 1e-3) / 1e12
        n_ch = len(row_chunks(w.M, world, chunks))
        plan = row_schedule(n_ch, first_groups(n_ch, first))
        out[w.name] = {"value": round(tf, 2), "unit": "TFLOP/s", "ms": round(ms, 4),
                       "frac_of_peak": round(tf / world / tflops_peak, 4),
                       "parallelism": f"column->row x{world}, reduction carried by the GEMM "
                                      f"launches ({chunks} row chunks, first GEMM in {first} "
                                      "launches; dx_row_reduce_job over NVLink "
                                      + ("multicast: multimem.ld_reduce / multimem.st)"
                                         if multicast else "peer loads)"),
                       "chunking_ms": sweep,
                       "gpu_launches_per_step": len(plan)}
        # The same chain with an NCCL all-reduce of Y in 4 asynchronous chunks.
        mlp_n = ParallelMLP.from_shards(W1, b1, W2, b2, w.act, chunks=4, mode="nccl")
        Yn = torch.empty_like(Yo)
        ms = time_run(lambda: mlp_n(X, hidden=H, out=Yn), 1500.0)
        parity["mlp_nccl"] = _row_parallel_parity(X, first_ref, W2, b2, True, Yn, world, dev)
        tf = w.flops / (ms * 1e-3) / 1e12
        out[w.name + "_nccl"] = {"value": round(tf, 2), "unit": "TFLOP/s", "ms": round(ms, 4),
                                 "frac_of_peak": round(tf / world / tflops_peak, 4),
                                 "parallelism": f"column->row x{world} + NCCL all-reduce "
                                                "(4 chunks)"}
        for m in modules.values():
            m.release()
        del mlp, mlp_n, Yn, modules
    del X, W1, b1, W2, b2, H, Yo

    # The gated FFN chain (ffn_gated, fusion.py:44-46): Y = (silu(X Wg + bg) *
    # (X Wu + bu)) Wo + bo, X[8192,4096], hidden 14336; one GPU runs the
    # engine chain, N GPUs the column -> row sharding with the overlapped
    # reduction.
    M_g, K_g, N_g = 8192, 4096, 14336
    h0, h1 = shard_bounds(N_g, world, rank, 64)
    h_loc = h1 - h0
    g_shared.manual_seed(5)
    X = torch.randn(M_g, K_g, generator=g_shared, device=dev).to(torch.bfloat16)
    bo = (torch.rand(K_g, generator=g_shared, device=dev) * 0.2 - 0.1).to(torch.bfloat16)
    Wg = (torch.randn(K_g, h_loc, generator=g, device=dev) / math.sqrt(K_g)).to(torch.bfloat16)
    Wu = (torch.randn(K_g, h_loc, generator=g, device=dev) / math.sqrt(K_g)).to(torch.bfloat16)
    bg = (torch.rand(h_loc, generator=g, device=dev) * 0.2 - 0.1).to(torch.bfloat16)
    bu = (torch.rand(h_loc, generator=g, device=dev) * 0.2 - 0.1).to(torch.bfloat16)
    Wo = (torch.randn(h_loc, K_g, generator=g, device=dev) / math.sqrt(N_g)).to(torch.bfloat16)
    Hg = torch.empty(M_g, h_loc, dtype=torch.bfloat16, device=dev)
    Yg = torch.empty(M_g, K_g, dtype=torch.bfloat16, device=dev)
    if world == 1:
        from deepx_op_gpukernelcompiler_b200 import gated_ffn
        run = lambda: gated_ffn(X, Wg, bg, Wu, bu, Wo, bo, "silu", hidden=Hg, out=Yg)  # noqa
        launches = 2
    else:
        ffn = ParallelGatedFFN.from_shards(Wg, bg, Wu, bu, Wo, bo, "silu", mode="fused",
                                           chunks=chunks, first_chunks=first)
        run = lambda: ffn(X, hidden=Hg, out=Yg)  # noqa: E731
        n_ch = len(row_chunks(M_g, world, chunks))
        launches = len(row_schedule(n_ch, first_groups(n_ch, first)))
    ms = time_run(run, 1500.0)
    Wgc, Wuc = Wg.float().cpu().numpy(), Wu.float().cpu().numpy()
    bgc, buc = bg.float().cpu().numpy(), bu.float().cpu().numpy()
    parity["gated_ffn_chain"] = _row_parallel_parity(
        X, lambda Xr: oracle.gated_linear_f64(Xr, Wgc, bgc, Wuc, buc, "silu"), Wo, bo, False, Yg,
        world, dev)
    tf = 2 * M_g * K_g * N_g * 3 / (ms * 1e-3) / 1e12
    out[f"ffn_gated_chain_{M_g}x{K_g}x{N_g}_bf16"] = {
        "value": round(tf, 2), "unit": "TFLOP/s", "ms": round(ms, 4),
        "frac_of_peak": round(tf / world / tflops_peak, 4),
        "parallelism": "one GPU" if world == 1 else
        f"column->row x{world}, reduction carried by the GEMM launches ({chunks} row chunks)",
        "gpu_launches_per_step": launches}
    if world > 1:
        ffn.release()
    return out


def run_skinny(args) -> None:
    """The evidence for the skinny-M kernel choice: the decode kernel against
    the single-CTA tensor-core kernel on decode-shaped problems (fp16, W
    rotated over copies larger than 3x L2, no flush), plain and gated, one
    JSON line per (M, K, N) with both times and the variant AUTO picks."""
    import numpy as np
    import torch

    from deepx_op_gpukernelcompiler_b200 import _native, fused_gated_linear, fused_linear

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)

    def timed(fn, n):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        return float(np.median(_time_launches(fn, n, lambda: None, stream, 150.0))) * 1e3

    g = torch.Generator(device=dev)
    g.manual_seed(11)
    for gated in (False, True):
        for K in (4096, 8192):
            for N in (1792, 3584, 7168, 14336, 28672):
                nw = 2 if gated else 1
                copies = max(2, math.ceil(3 * L2_BYTES / (nw * K * N * 2)))
                Ws = [(torch.randn(K, N, generator=g, device=dev) / math.sqrt(K)).half()
                      for _ in range(copies * nw)]
                b = torch.zeros(N, dtype=torch.float16, device=dev)
                for M in (1, 4, 8, 12, 16, 32, 64):
                    X = torch.randn(M, K, generator=g, device=dev).half()
                    Y = torch.empty(M, N, dtype=torch.float16, device=dev)
                    res = {}
                    for kern in ("decode", "umma_1cta", "auto"):
                        it = [0]

                        def fn(kern=kern):
                            i = it[0] % copies
                            it[0] += 1
                            if gated:
                                fused_gated_linear(X, Ws[2 * i], Ws[2 * i + 1], b, b, "silu",
                                                   out=Y, kernel=kern)
                            else:
                                fused_linear(X, Ws[i], b, "gelu_erf", out=Y, kernel=kern)
                        res[kern] = round(timed(fn, max(5, min(args.steps, 12))), 1)
                        if kern == "auto":
                            res["auto_kernel"] = _native.last_launch_plan().split()[0]
                    byts = 2 * (M * K + nw * K * N + nw * N + M * N)
                    print(json.dumps({"skinny": "gated" if gated else "plain", "M": M, "K": K,
                                      "N": N, "us": res,
                                      "auto_GBps": round(byts / res["auto"] / 1e3, 1)}),
                          flush=True)
                del Ws
                torch.cuda.empty_cache()


def run_timeline(args) -> None:
    """Per-launch CTA timeline of one overlapped MLP step (the 16384 x 4096 x
    16384 chain, column -> row over the torchrun ranks): each launch of the
    step records %globaltimer stamps into its own trace buffer
    (dx_set_trace_buffer switched between launches), and rank 0 prints, per
    launch, its start, the end of its last tile's epilogue, the end of its
    carried reduction job and its exit, in microseconds from the first
    launch's start, plus the step time and that of the same two GEMMs
    unchunked.  --chunks / --first set the schedule, --nvls 0 forces peer
    loads."""
    import torch
    import torch.distributed as dist

    from deepx_op_gpukernelcompiler_b200 import _native, fused_linear
    from deepx_op_gpukernelcompiler_b200.shard import ParallelMLP, shard_bounds
    from deepx_op_gpukernelcompiler_b200.workloads import WORKLOADS

    rank, world, local = _dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    w = WORKLOADS["mlp_residual_16384x4096x16384_bf16"]
    h0, h1 = shard_bounds(w.N, world, rank, 64)
    g = torch.Generator(device=dev)
    g.manual_seed(w.seed)
    X = torch.randn(w.M, w.K, generator=g, device=dev).bfloat16()
    b2 = (torch.rand(w.K, generator=g, device=dev) * 0.2 - 0.1).bfloat16()
    g.manual_seed(w.seed * 1000 + rank)
    W1 = (torch.randn(w.K, h1 - h0, generator=g, device=dev) / math.sqrt(w.K)).bfloat16()
    b1 = (torch.rand(h1 - h0, generator=g, device=dev) * 0.2 - 0.1).bfloat16()
    W2 = (torch.randn(h1 - h0, w.K, generator=g, device=dev) / math.sqrt(w.N)).bfloat16()
    H = torch.empty(w.M, h1 - h0, dtype=torch.bfloat16, device=dev)
    Y = torch.empty(w.M, w.K, dtype=torch.bfloat16, device=dev)
    mlp = ParallelMLP.from_shards(W1, b1, W2, b2, w.act, mode="fused" if world > 1 else "nccl",
                                  chunks=args.chunks, first_chunks=args.first,
                                  nvls=None if args.nvls else False)
    stream = torch.cuda.current_stream(dev)

    def timed(fn, n=10):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        _barrier(world)
        return _max_over_ranks(_time_back_to_back(fn, n, stream, 2000.0), world, dev)

    step_ms = timed(lambda: mlp(X, hidden=H, out=Y))
    unchunked_ms = timed(lambda: (fused_linear(X, W1, b1, w.act, out=H),
                                  fused_linear(H, W2, None, None, out=Y)))
    slots = 148 * 16
    traces, kinds = [], []

    def hook(i, launch):
        while len(traces) <= i:
            traces.append(torch.zeros(slots, dtype=torch.int64, device=dev))
        kinds.append((launch[0], str(launch[-1])))
        _native.load().dx_set_trace_buffer(traces[i].data_ptr(), slots * 8)

    torch.cuda.synchronize()
    _barrier(world)
    mlp.launch_hook = hook
    mlp(X, hidden=H, out=Y)
    mlp.launch_hook = None
    _native.load().dx_set_trace_buffer(None, 0)
    torch.cuda.synchronize()
    t0, rows = None, []
    for i, (kind, job) in enumerate(kinds):
        t = traces[i].view(148, 16).cpu()
        used = t[:, 15] > 0
        if not bool(used.any()):
            rows.append({"launch": i, "kind": kind, "job": job, "traced": False})
            continue
        t = t[used]
        if t0 is None:
            t0 = int(t[:, 0].min())
        items = t[:, 1:14]
        rel = lambda v: round((int(v) - t0) / 1e3, 1)  # noqa: E731
        rows.append({"launch": i, "kind": kind, "job": job, "start": rel(t[:, 0].min()),
                     "last_tile": rel(items[items > 0].max()) if bool((items > 0).any()) else None,
                     "job_end": rel(t[:, 14][t[:, 14] > 0].max()) if bool((t[:, 14] > 0).any())
                     else None, "exit": rel(t[:, 15].max())})
    if rank == 0:
        print(json.dumps({"timeline": w.name, "world": world, "chunks": args.chunks,
                          "first": args.first, "multicast": bool(mlp.last_multicast),
                          "step_ms": round(step_ms, 4), "unchunked_gemms_ms": round(unchunked_ms, 4),
                          "launches": rows}), flush=True)
    torch.cuda.synchronize()
    mlp.release()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_decode_shards(args) -> None:
    """The decode configuration's column shards for 1/2/4/8-way splits, each
    timed on one GPU (what every rank of a column-parallel run executes; the
    shards need no collective): back-to-back launches over rotated weight
    copies together >= 3x L2, one JSON line per split with GB/s, the fraction
    of the HBM peak and the launch plan."""
    import torch

    from deepx_op_gpukernelcompiler_b200 import _native, fused_linear
    from deepx_op_gpukernelcompiler_b200.shard import shard_bounds
    from deepx_op_gpukernelcompiler_b200.workloads import WORKLOADS

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    peaks, peak_kind = _peaks()
    hbm = peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
    w = WORKLOADS["decode_gelu_erf_16x8192x28672_f16"]
    g = torch.Generator(device=dev)
    g.manual_seed(w.seed)
    X = torch.randn(w.M, w.K, generator=g, device=dev).to(w.torch_dtype)
    for ways in (1, 2, 4, 8):
        n0, n1 = shard_bounds(w.N, ways, 0, 64)
        n = n1 - n0
        copies = max(2, math.ceil(3 * L2_BYTES / (w.K * n * 2)))
        Ws = [(torch.randn(w.K, n, generator=g, device=dev) / math.sqrt(w.K)).to(w.torch_dtype)
              for _ in range(copies)]
        b = (torch.rand(n, generator=g, device=dev) * 0.2 - 0.1).to(w.torch_dtype)
        Y = torch.empty(w.M, n, dtype=w.torch_dtype, device=dev)
        it = [0]

        def dec():
            fused_linear(X, Ws[it[0] % copies], b, w.act, out=Y)
            it[0] += 1

        for _ in range(5):
            dec()
        torch.cuda.synchronize()
        ms = _time_back_to_back(dec, max(40, args.steps), stream)
        byts = 2 * (w.M * w.K + w.K * n + n + w.M * n)
        print(json.dumps({"decode_shard": f"1/{ways}", "M": w.M, "K": w.K, "N": n,
                          "us": round(ms * 1e3, 2), "GBps": round(byts / (ms * 1e-3) / 1e9, 1),
                          "frac_of_hbm": round(byts / (ms * 1e-3) / 1e9 / hbm, 4),
                          "peak": f"{hbm} GB/s, {peak_kind}",
                          "plan": _native.last_launch_plan()}), flush=True)
        del Ws, b, Y


DECODE_TRACE_SLOTS = {12: "entry", 0: "setup", 1: "first_load", 2: "last_load",
                      3: "last_mma", 4: "acc_ready", 5: "acc_read", 7: "slices_sent",
                      8: "last_cluster_barrier", 9: "finished", 15: "exit"}


def run_decode_timeline(args) -> None:
    """Per-CTA timeline of one decode launch on the 1/`--ways` column shard of
    the decode configuration (dx_set_trace_buffer: global-timer stamps per CTA
    at fixed points of the kernel), after back-to-back launches over rotated
    weights; one JSON line with, per point, the min / median / max over CTAs
    in us from the first CTA's entry.  A traced launch has no early start, so
    the shard is also timed untraced."""
    import numpy as np
    import torch

    from deepx_op_gpukernelcompiler_b200 import _native, fused_linear
    from deepx_op_gpukernelcompiler_b200.shard import shard_bounds
    from deepx_op_gpukernelcompiler_b200.workloads import WORKLOADS

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    lib = _native.load()
    w = WORKLOADS["decode_gelu_erf_16x8192x28672_f16"]
    n0, n1 = shard_bounds(w.N, args.ways, 0, 64)
    n = n1 - n0
    g = torch.Generator(device=dev)
    g.manual_seed(w.seed)
    X = torch.randn(w.M, w.K, generator=g, device=dev).to(w.torch_dtype)
    copies = max(2, math.ceil(3 * L2_BYTES / (w.K * n * 2)))
    Ws = [(torch.randn(w.K, n, generator=g, device=dev) / math.sqrt(w.K)).to(w.torch_dtype)
          for _ in range(copies)]
    b = (torch.rand(n, generator=g, device=dev) * 0.2 - 0.1).to(w.torch_dtype)
    Y = torch.empty(w.M, n, dtype=w.torch_dtype, device=dev)
    slots = 16
    tr = torch.zeros(4096 * slots, dtype=torch.int64, device=dev)
    it = [0]

    def dec():
        fused_linear(X, Ws[it[0] % copies], b, w.act, out=Y)
        it[0] += 1

    line = {"decode_shard": f"1/{args.ways}", "M": w.M, "K": w.K, "N": n, "act": w.act}
    for traced in (False, True):
        if traced:
            _native.check("dx_set_trace_buffer", lib.dx_set_trace_buffer(tr.data_ptr(),
                                                                         tr.numel() * 8))
        for _ in range(5):
            dec()
        torch.cuda.synchronize()
        ms = _time_back_to_back(dec, max(40, args.steps), stream)
        line["us_traced" if traced else "us"] = round(ms * 1e3, 2)
        if traced:
            plan = _native.last_launch_plan()
            grid = int(plan.split("grid=")[1].split()[0])
            t = tr.view(-1, slots)[:grid].cpu().numpy().astype(np.int64)
            base = t[:, 12].min()
            points = {}
            for slot, name in DECODE_TRACE_SLOTS.items():
                col = t[:, slot]
                col = col[col > 0]
                if col.size:
                    rel = (col - base) / 1e3
                    points[name] = [round(float(np.percentile(rel, q)), 2) for q in (0, 50, 100)]
            line["plan"] = plan
            line["timeline_us_min_median_max"] = points
            _native.check("dx_set_trace_buffer", lib.dx_set_trace_buffer(None, 0))
    print(json.dumps(line), flush=True)


def run_fabric(args) -> None:
    """All-to-all NVLink throughput between the ranks of one box (the bound of
    the row-parallel reduction): every rank moves one slab of 16384 x 4096
    bf16 / world to or from every peer at once over symmetric (peer-mapped)
    memory, by copy engine (cudaMemcpyAsync via tensor copies, one stream per
    peer) and by SM kernels (elementwise kernels reading or writing peer
    memory).  One JSON line per method: GB/s per GPU per direction."""
    import torch
    import torch.distributed as dist
    import torch.distributed._symmetric_memory as symm_mem

    rank, world, local = _dist_env()
    if world < 2:
        raise SystemExit("--fabric needs torchrun with at least 2 ranks")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    N, slab = 4096, 16384 // world
    rows = slab * world
    src = symm_mem.empty(rows, N, dtype=torch.bfloat16, device=dev)
    dst_sym = symm_mem.empty(rows, N, dtype=torch.bfloat16, device=dev)
    src.normal_()
    torch.cuda.synchronize()
    hs = symm_mem.rendezvous(src, dist.group.WORLD)
    hd = symm_mem.rendezvous(dst_sym, dist.group.WORLD)
    dist.barrier()
    peer_src = [hs.get_buffer(s, (rows, N), torch.bfloat16) for s in range(world)]
    peer_dst = [hd.get_buffer(s, (rows, N), torch.bfloat16) for s in range(world)]
    out = torch.empty(rows, N, dtype=torch.bfloat16, device=dev)
    peers = [s for s in range(world) if s != rank]
    streams = [torch.cuda.Stream(dev) for _ in peers]
    main = torch.cuda.current_stream(dev)
    moved = len(peers) * slab * N * 2  # bytes in (and out) per rank

    def on_streams(copy):
        for st, s in zip(streams, peers):
            st.wait_stream(main)
            with torch.cuda.stream(st):
                copy(s)
        for st in streams:
            main.wait_stream(st)

    def sl(t, i):
        return t[i * slab:(i + 1) * slab]

    methods = {
        "copy_engine_pull": lambda: on_streams(lambda s: sl(out, s).copy_(sl(peer_src[s], rank))),
        "copy_engine_push": lambda: on_streams(lambda s: sl(peer_dst[s], rank).copy_(sl(src, s))),
        "sm_pull": lambda: [torch.mul(sl(peer_src[s], rank), 1, out=sl(out, s)) for s in peers],
        "sm_push": lambda: [torch.mul(sl(src, s), 1, out=sl(peer_dst[s], rank)) for s in peers],
    }
    for name, fn in methods.items():
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        ms = _max_over_ranks(_time_back_to_back(fn, max(5, args.steps), main, 200.0), world, dev)
        if rank == 0:
            print(json.dumps({"fabric": name, "world": world, "MiB_per_rank_each_way":
                              moved / 2 ** 20, "us": round(ms * 1e3, 1),
                              "GBps_per_gpu_per_direction": round(moved / (ms * 1e-3) / 1e9, 1)}),
                  flush=True)
    torch.cuda.synchronize()
    dist.barrier()
    del peer_src, peer_dst, hs, hd
    dist.barrier()
    dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD)
    ap.add_argument("--no-extra", action="store_true", help="skip the decode/square/MLP lines")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--no-ref-engines", action="store_true",
                    help="skip timing the reference's Triton/TileLang engines (N=1)")
    ap.add_argument("--profile", action="store_true",
                    help="run only W warm-up and K timed launches of the workload (for ncu)")
    ap.add_argument("--shard-of", type=int, default=1,
                    help="with --profile: run rank 0's column shard of an N-way split on one GPU")
    ap.add_argument("--timeline", action="store_true",
                    help="per-launch timeline of one overlapped MLP step (torchrun)")
    ap.add_argument("--chunks", type=int, default=4, help="--timeline: row chunks")
    ap.add_argument("--first", type=int, default=4, help="--timeline: first-GEMM launches")
    ap.add_argument("--nvls", type=int, default=1, help="--timeline: 0 forces peer loads")
    ap.add_argument("--decode-shards", action="store_true",
                    help="time the decode configuration's 1/2/4/8-way column shards on one GPU")
    ap.add_argument("--decode-timeline", action="store_true",
                    help="per-CTA timeline of a decode launch on the 1/--ways column shard")
    ap.add_argument("--ways", type=int, default=8, help="column shard for --decode-timeline")
    ap.add_argument("--fabric", action="store_true",
                    help="all-to-all NVLink throughput between the ranks (torchrun, >= 2 GPUs)")
    ap.add_argument("--skinny", action="store_true",
                    help="time the decode and single-CTA tensor-core kernels on decode shapes "
                         "(the evidence for AUTO's skinny-M choice), one JSON line per shape")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    _, world, _ = _dist_env()
    if world != args.gpus and args.impl == "b200":
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE={world}; using WORLD_SIZE",
              file=sys.stderr)
    if args.impl == "reference":
        run_reference(args)
    elif args.fabric:
        run_fabric(args)
    elif args.decode_shards:
        run_decode_shards(args)
    elif args.decode_timeline:
        run_decode_timeline(args)
    elif args.timeline:
        run_timeline(args)
    elif args.skinny:
        run_skinny(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
