"""Benchmark: Evoformer pair-GEMM throughput at N=1024 on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step is one Evoformer pair-stack block's triangle multiplications at
N=1024, c_z = c_hidden = 128: the outgoing update then the incoming update,
each added in place into a bf16 pair (the in-model encoder's residual form,
src/evoformer/block.ts:1720-1725 of the reference).  value = algorithmic
TFLOP/s over the whole job (FLOP formulas of src/runtime/kernel-cost.ts:158-162,
481.0 GFLOP per direction), with every input resident in HBM before the timed
region; the pair (268 MB) is larger than L2, so no flush is needed.

e2e times the same step through the reference-facing host form
(af2_triangle_multiplication_host: f32 host arrays in, f32 host array out,
like TriangleMultiplication*Gpu.run) from pinned host memory.

--impl reference times the CPU restatement of the reference's own CPU path
(the reference is TypeScript and no JavaScript runtime exists on this box) on
a bounded sample of the same workload, with every host thread.

Multi-GPU (torchrun): every rank runs its own independent pair (replicas,
weak scaling); value sums the work of all ranks over the max-over-ranks time.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "alphafold2-webgpu_b200"))

N = 1024
CZ = CH = 128
METRIC = "Evoformer pair-GEMM TFLOP/s & ms/block at N=1024; % of B200 bf16 TC peak"
# dram__bytes_read.sum + dram__bytes_write.sum of one contract_kernel launch, from one ncu
# capture of this script (profiles/triangle_contract_n1024_dram.md).
CONTRACT_DRAM_BYTES = {1024: 771_527_680}


def triangle_flops(n: int, cz: int = CZ, ch: int = CH) -> float:
    """kernel-cost.ts:158-162: gate, block + whole projections, contraction, output."""
    return 2.0 * n * n * (cz * cz + 4 * cz * ch + n * ch + ch * cz)


def contraction_flops(n: int, ch: int = CH) -> float:
    return 2.0 * n * n * n * ch


def measured_peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return {"bf16_tflops": d["bf16_tflops"], "bf16_tflops_sustained": d["bf16_tflops_sustained"],
                "hbm_gbs": d["hbm_gbs"], "source": "measured"}
    return {"bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6650.0, "source": "fallback"}


def synthetic_weights(rng, cz=CZ, ch=CH):
    """Projection weights ~N(0, 1/fan_in) in the reference's [out, in] layouts, LN gamma 1 / beta 0, biases 0."""
    import numpy as np

    def normal(rows, cols):
        return (rng.standard_normal((rows, cols)) / np.sqrt(cols)).astype(np.float32).ravel()

    parts = [np.ones(cz), np.zeros(cz)]
    for _ in range(4):
        parts += [normal(ch, cz), np.zeros(ch)]
    parts += [np.ones(ch), np.zeros(ch), normal(cz, ch), np.zeros(cz), normal(cz, cz), np.zeros(cz)]
    return np.concatenate([np.asarray(p, np.float32) for p in parts])


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while the timed region runs."""

    def __init__(self, index: int):
        self.samples, self.reasons = [], set()
        self.max_mhz = None
        self._stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            self.handle = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
        except Exception:  # no NVML: no clock record
            self.nvml = None

    def _run(self):
        nv = self.nvml
        flags = {
            "hw_slowdown": getattr(nv, "nvmlClocksEventReasonHwSlowdown", 0x8),
            "hw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
            "sw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
            "sw_power_cap": getattr(nv, "nvmlClocksEventReasonSwPowerCap", 0x4),
            "hw_power_brake_slowdown": getattr(nv, "nvmlClocksEventReasonHwPowerBrakeSlowdown", 0x80),
        }
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM))
                mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                for k, bit in flags.items():
                    if mask & bit:
                        self.reasons.add(k)
            except Exception:
                pass
            time.sleep(0.02)

    def __enter__(self):
        if self.nvml:
            self.thread = threading.Thread(target=self._run, daemon=True)
            self.thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self.nvml:
            self.thread.join()

    def record(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def cpu_reference_rate(sample_n: int, repeats: int, threads: int) -> tuple[float, float, str]:
    """Times the oracle (CPU restatement of the reference's CPU path) on a bounded
    sample: `repeats` x (outgoing + incoming) at N=sample_n.  Returns (TFLOP/s, seconds, description)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import numpy as np

    import oracle
    rng = np.random.default_rng(0)
    z = rng.standard_normal((sample_n, sample_n, CZ)).astype(np.float32)
    mask = np.ones((sample_n, sample_n), np.float32)
    w = synthetic_weights(rng)
    t0 = time.perf_counter()
    for _ in range(repeats):
        for d in (0, 1):
            oracle.triangle(d, z, mask, w, 1e-5, threads=threads)
    dt = time.perf_counter() - t0
    flops = repeats * 2 * triangle_flops(sample_n)
    return flops / dt / 1e12, dt, f"{repeats} x (outgoing + incoming) at N={sample_n}, c=128, f64-accumulating CPU port"


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    # Size each step's sample so that warm-up plus timed steps take about a minute.
    rate, _, _ = cpu_reference_rate(96, 1, threads)
    budget_flops = rate * 1e12 * 60.0 / max(1, args.steps + args.warmup)
    sample_n = 32
    while sample_n < N and 2 * triangle_flops(sample_n + 16) <= budget_flops:
        sample_n += 16
    for _ in range(args.warmup):
        cpu_reference_rate(sample_n, 1, threads)
    rates, secs = [], []
    for _ in range(args.steps):
        r, s, desc = cpu_reference_rate(sample_n, 1, threads)
        rates.append(r)
        secs.append(s)
    value = statistics.median(rates)
    ms_per_step = triangle_flops(N) * 2 / (value * 1e12) * 1e3
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": "triangle multiplication outgoing+incoming, N=1024, c_z=c_hidden=128 "
                               f"(each step timed on a bounded N={sample_n} sample; ms_per_step extrapolated "
                               "to N=1024 by FLOPs)",
                   "N": N, "parallelism": "host threads"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": f"per step: outgoing + incoming at N={sample_n} (median {statistics.median(secs):.2f} s)"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args) -> None:
    import numpy as np
    import torch

    import af2cuda
    from af2cuda import _lib

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as td
        td.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
        dist = td

    dev = af2cuda.Device(local)
    L = _lib.lib()
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    sh = stream.cuda_stream
    rng = np.random.default_rng(1234 + rank)
    gen = torch.Generator(device="cuda").manual_seed(1234 + rank)
    pair = torch.randn(N, N, CZ, device="cuda", generator=gen).to(torch.bfloat16)
    mask = torch.ones(N, N, device="cuda")
    w_out = torch.from_numpy(synthetic_weights(rng)).cuda()
    w_in = torch.from_numpy(synthetic_weights(rng)).cuda()
    torch.cuda.synchronize()

    def step():
        af2cuda.encode_triangle_multiplication_tensors(dev, 0, pair, mask, w_out, residual=True, stream=sh)
        af2cuda.encode_triangle_multiplication_tensors(dev, 1, pair, mask, w_in, residual=True, stream=sh)

    for _ in range(max(args.warmup, 3)):
        step()
    dev.sync(sh)

    def barrier():
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    # ---- timed region: K steps, device events, profiler on for the per-kernel roofline ----
    L.af2_profile_enable(dev.handle, 1)
    L.af2_profile_reset(dev.handle)
    launches0 = dev.launch_count
    barrier()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record(stream)
        for _ in range(args.steps):
            step()
        stop.record(stream)
        stop.synchronize()
    dev.sync(sh)
    barrier()
    launches = dev.launch_count - launches0
    ms = start.elapsed_time(stop)
    kernel = {}
    for name in ("triangle.prepare", "triangle.relayout", "triangle.project", "triangle.contract", "triangle.output"):
        c, t = ctypes.c_uint64(), ctypes.c_double()
        L.af2_profile_read(dev.handle, name.encode(), ctypes.byref(c), ctypes.byref(t))
        if c.value:
            kernel[name] = {"launches": int(c.value), "avg_us": t.value / c.value * 1e3,
                            "share": 0.0, "total_ms": t.value}
    L.af2_profile_enable(dev.handle, 0)
    total_kernel_ms = sum(k["total_ms"] for k in kernel.values()) or 1.0
    for k in kernel.values():
        k["share"] = k["total_ms"] / total_kernel_ms
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    flops_step = 2 * triangle_flops(N)
    value = world * flops_step * args.steps / (ms * 1e-3) / 1e12
    peaks = measured_peaks()

    # ---- roofline of the dominant kernel (the per-channel contraction) ----
    con = kernel["triangle.contract"]
    achieved = contraction_flops(N) / (con["avg_us"] * 1e-6) / 1e12
    traffic = CONTRACT_DRAM_BYTES.get(N)
    roofline = {"kernel": "triangle.contract", "bound": "tensor", "achieved": achieved,
                "peak": peaks["bf16_tflops"], "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops"],
                "traffic": traffic, "peak_source": f"{peaks['source']} burst bf16",
                "flops_per_launch": contraction_flops(N), "avg_launch_us": con["avg_us"]}

    # ---- e2e: the reference-facing host form, f32 host arrays in and out ----
    e2e = None
    if True:  # every rank: the e2e time is also a max over ranks
        host_z = torch.empty(N, N, CZ, dtype=torch.float32, pin_memory=True)
        host_z.copy_(pair.float().cpu())
        host_out = torch.empty_like(host_z, pin_memory=True)
        host_mask = torch.ones(N, N, dtype=torch.float32, pin_memory=True)
        hw = [torch.from_numpy(synthetic_weights(rng)).pin_memory() for _ in range(2)]
        shape = _lib.TriangleShape(N, CZ, CH)
        opts = _lib.TriangleOptions(0, 1)
        stats = _lib.OpStats()

        def host_step():
            src = host_z
            for d in (0, 1):
                st = L.af2_triangle_multiplication_host(
                    dev.handle, d, ctypes.byref(shape), src.data_ptr(), host_mask.data_ptr(), hw[d].data_ptr(),
                    hw[d].numel(), 1e-5, ctypes.byref(opts), _lib.AF2_F32, host_out.data_ptr(), ctypes.byref(stats))
                _lib.check(st, dev.handle)
                src = host_out

        host_step()
        e2e_steps = max(3, min(args.steps, 10))
        barrier()
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            host_step()
        e2e_s = time.perf_counter() - t0
        if dist:
            t = torch.tensor([e2e_s], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e_s = float(t.item())
        per_dir_in = N * N * CZ * 4 + N * N * 4 + hw[0].numel() * 4
        e2e = {"value": world * flops_step * e2e_steps / e2e_s / 1e12, "unit": "TFLOP/s",
               "h2d_bytes_per_step": 2 * per_dir_in, "d2h_bytes_per_step": 2 * N * N * CZ * 4,
               "ms_per_step": e2e_s / e2e_steps * 1e3,
               "path": "af2_triangle_multiplication_host (f32 host arrays, pinned), outgoing then incoming"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        rate, secs, desc = cpu_reference_rate(256, 1, threads)
        cpu = {"value": rate, "unit": "TFLOP/s", "cores": threads, "kind": "port",
               "sample": f"{desc} ({secs:.1f} s)"}

    if dist:
        dist.barrier()
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": "triangle multiplication outgoing+incoming (one Evoformer block's pair "
                                   "triangle updates), N=1024, c_z=c_hidden=128, bf16 pair updated in place, "
                                   "f16 tensor-core operands with f32 accumulation",
                       "N": N, "c_z": CZ, "c_hidden": CH, "flops_per_step": flops_step,
                       "l2": "inputs larger than L2 (pair 268 MB bf16; scratch 805 MB), no flush",
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU"},
            "pct_of_peak": value / world / peaks["bf16_tflops"],
            "roofline": roofline, "kernels": kernel, "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": int(launches), "clocks": clocks.record(),
        }
        print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()
    dev.close()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
