"""Benchmark: Evoformer pair-GEMM throughput at N=1024 on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step is one Evoformer block's pair GEMM set at N=1024 (the metric's
workload): the outer-product mean of an S=512, c_m=256 MSA added into the
pair, the triangle multiplications outgoing then incoming (c_z = c_hidden =
128), and the pair transition (128 -> 512 -> 128, mixed-q8 weights with f32
per-output-channel scales), each updating one bf16 pair [1024, 1024, 128] in
place -- the in-model order and residual form of the reference
(src/evoformer/block.ts:1673-1751).  value = algorithmic TFLOP/s over the
whole job (FLOP formulas of src/runtime/kernel-cost.ts: 962.1 triangle +
1391.6 OPM + 274.9 transition = 2628.6 GFLOP per block), with every input
resident in HBM before the timed region; the pair and the MSA (268 MB each)
are larger than L2, so no flush is needed.

e2e times the same step through the public device-form API with the step's
inputs copied in from pinned host memory (pair and MSA, bf16) and the pair
read back, every step.

--impl reference times the CPU restatement of the reference's own CPU path
(the reference is TypeScript and no JavaScript runtime exists on this box) on
a bounded sample of the same block, with every host thread.

Multi-GPU (torchrun, one process per GPU): the same N=1024 block with the
pair sharded by rows across the ranks (strong scaling).  Each triangle
direction projects the rank's own rows, exchanges hidden-channel groups so
that every rank contracts its 128/R channels over the whole N x N, and
returns the contracted channels of each rank's rows for the output
projection (two all-to-alls: copy-engine copies into the peers' IPC-mapped
scratch between NCCL barriers, NCCL send/recv where the mapping is refused);
the OPM projects each rank's residues and all-gathers the right operand; the
transition is row-local.  value = the block's FLOPs over the max-over-ranks
time.
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
S_MSA, CM, C_OUTER = 512, 256, 32
HIDDEN = 4 * CZ
METRIC = "Evoformer pair-GEMM TFLOP/s & ms/block at N=1024; % of B200 bf16 TC peak"
# dram__bytes_read.sum + dram__bytes_write.sum per launch of the default block at N=1024, from
# one single-pass ncu capture of this workload (profiles/block_n1024_launches.md, the mean over
# 14 block steps); kernels without a capture report null.
KERNEL_DRAM_BYTES = {"opm.fused": 606_830_208, "triangle.contract": 777_577_673, "triangle.project": 747_430_601,
                     "triangle.output": 750_551_470, "transition.fused": 473_526_985, "opm.project": 314_026_478,
                     "opm.count": 2_116_352}
KERNELS = ("weights.prepare", "triangle.prepare", "triangle.relayout", "triangle.project", "triangle.contract",
           "triangle.output", "opm.normalize", "opm.project", "opm.count", "opm.outer", "opm.output",
           "opm.fused", "transition.prepare", "transition.normalize", "transition.fused", "transition.linear",
           "linear", "activations.convert", "attention.normalize", "attention.project", "attention.flash",
           "attention.output")
PAIR_HEADS = 4


def triangle_flops(n: int, cz: int = CZ, ch: int = CH) -> float:
    """kernel-cost.ts:158-162: gate, block + whole projections, contraction, output."""
    return 2.0 * n * n * (cz * cz + 4 * cz * ch + n * ch + ch * cz)


def contraction_flops(n: int, ch: int = CH) -> float:
    return 2.0 * n * n * n * ch


def opm_flops(n: int, s: int = S_MSA, cm: int = CM, c: int = C_OUTER, cz: int = CZ) -> float:
    """kernel-cost.ts: projection 2 S N c_m 2c, contraction 2 (N c)^2 S, output 2 N^2 c^2 c_z."""
    return 2.0 * s * n * cm * 2 * c + 2.0 * (n * c) ** 2 * s + 2.0 * n * n * c * c * cz


def transition_flops(n: int, c: int = CZ, h: int = HIDDEN) -> float:
    return 4.0 * n * n * c * h


def attention_flops(n: int, c: int = CZ, heads: int = PAIR_HEADS) -> float:
    """kernel-cost.ts:79-92, one triangle attention direction: project gemm(N^2, C, 4C), flash
    2 gemm(N H N, 32, N), output gemm(N^2, C, C), pair bias gemm(N^2, C, H)."""
    return 2.0 * n * n * c * 4 * c + 4.0 * n ** 3 * heads * 32 + 2.0 * n * n * c * c + 2.0 * n * n * c * heads


def block_flops(n: int = N, s: int = S_MSA) -> float:
    return 2 * triangle_flops(n) + opm_flops(n, s) + transition_flops(n)


def kernel_step_flops(name: str, world: int = 1, n: int = N, s: int = S_MSA) -> float | None:
    """Algorithmic FLOPs one rank's launches of a tensor-core kernel do per block
    (each rank does 1/world of every operator on a row-sharded pair)."""
    per_block = {"triangle.contract": 2 * contraction_flops(n),
                 "triangle.project": 2 * 2.0 * n * n * CZ * 4 * CH,
                 "triangle.output": 2 * 2.0 * n * n * (CH * CZ + CZ * CZ),
                 "opm.outer": 2.0 * (n * C_OUTER) ** 2 * s,
                 "opm.output": 2.0 * n * n * C_OUTER * C_OUTER * CZ,
                 "opm.fused": 2.0 * (n * C_OUTER) ** 2 * s + 2.0 * n * n * C_OUTER * C_OUTER * CZ,
                 "opm.project": 2.0 * s * n * CM * 2 * C_OUTER,
                 "transition.fused": transition_flops(n),
                 # triangle attention, both directions (pair-block workloads only)
                 "attention.flash": 2 * 4.0 * n ** 3 * PAIR_HEADS * 32,
                 "attention.project": 2 * 2.0 * n * n * CZ * (4 * CZ + PAIR_HEADS),
                 "attention.output": 2 * 2.0 * n * n * CZ * CZ}.get(name)
    return None if per_block is None else per_block / world


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


def opm_weights(rng, cm=CM, c=C_OUTER, cz=CZ):
    """The benchmark configs' OPM law: LN gamma 1 / beta 0, W ~ N(0, 1/fan_in) in [in, out], biases 0."""
    import numpy as np
    return np.concatenate([np.ones(cm), np.zeros(cm),
                           rng.standard_normal(cm * c) / np.sqrt(cm), np.zeros(c),
                           rng.standard_normal(cm * c) / np.sqrt(cm), np.zeros(c),
                           rng.standard_normal(c * c * cz) / np.sqrt(c * c), np.zeros(cz)]).astype(np.float32)


def attention_weights(rng, c=CZ, heads=PAIR_HEADS):
    """Triangle attention weights in packAttentionWeights order (src/evoformer/attention.ts:179-201):
    LN gamma 1 / beta 0, q/k/v/gate/output weights ~N(0, 1/fan_in) [in, out], biases 0, the
    normalized-input pair projection [C, heads] last."""
    import numpy as np

    def mat(i, o):
        return (rng.standard_normal((i, o)) / np.sqrt(i)).astype(np.float32).ravel()

    return np.concatenate([np.ones(c), np.zeros(c), mat(c, c), mat(c, c), mat(c, c), mat(c, c), np.zeros(c),
                           mat(c, c), np.zeros(c), mat(c, heads)]).astype(np.float32)


def transition_weights(rng, c=CZ, h=HIDDEN):
    """Pair transition weights ~N(0, 1/fan_in), [in, out]; the matrices as symmetric int8
    with one f32 scale per output column (the mixed-q8 format of the benchmark configs)."""
    import numpy as np

    def q8(w):
        scale = np.abs(w).max(axis=0) / 127.0
        scale[scale == 0] = 1.0
        codes = np.clip(np.floor(w / scale + 0.5), -127, 127).astype(np.int8)
        return codes, scale.astype(np.float32)

    w1 = (rng.standard_normal((c, h)) / np.sqrt(c)).astype(np.float32)
    w2 = (rng.standard_normal((h, c)) / np.sqrt(h)).astype(np.float32)
    return {"ln": (np.ones(c, np.float32), np.zeros(c, np.float32)), "w1": q8(w1), "b1": np.zeros(h, np.float32),
            "w2": q8(w2), "b2": np.zeros(c, np.float32)}


def multimer_block(dev, torch, af2cuda, rng, world: int, rank: int, sh: int, stream, dist, steps: int = 10) -> dict:
    """BASELINE config 5 on the job's GPUs: triangle multiplication out + in and the pair transition on a
    bf16 pair [2048, 2048, 128] (rows sharded over the ranks), mask 1 inside the four 512-residue chain
    blocks; `steps` timed on CUDA events after 3 warm-up steps, max over ranks."""
    n = 2048
    rows = n // world
    r0 = rank * rows
    gen = torch.Generator(device="cuda").manual_seed(2048 + rank)
    pair = torch.randn(rows, n, CZ, device="cuda", generator=gen).to(torch.bfloat16)
    chain = torch.arange(n, device="cuda") // 512
    mask = (chain[r0:r0 + rows, None] == chain[None, :]).float().contiguous()
    w_tri = [torch.from_numpy(synthetic_weights(rng)).cuda() for _ in range(2)]
    tw = transition_weights(rng)
    tws = {"layerNormScale": torch.from_numpy(tw["ln"][0]).cuda(), "layerNormOffset": torch.from_numpy(tw["ln"][1]).cuda(),
           "firstWeight": af2cuda.Q8Matrix(torch.from_numpy(tw["w1"][0]).cuda(), torch.from_numpy(tw["w1"][1]).cuda()),
           "firstBias": torch.from_numpy(tw["b1"]).cuda(),
           "secondWeight": af2cuda.Q8Matrix(torch.from_numpy(tw["w2"][0]).cuda(), torch.from_numpy(tw["w2"][1]).cuda()),
           "secondBias": torch.from_numpy(tw["b2"]).cuda()}
    torch.cuda.synchronize()

    def step():
        for d in (0, 1):
            if world > 1:
                af2cuda.encode_triangle_multiplication_sharded_tensors(dev, d, pair, mask, w_tri[d], n, residual=True,
                                                                       stream=sh)
            else:
                af2cuda.encode_triangle_multiplication_tensors(dev, d, pair, mask, w_tri[d], residual=True, stream=sh)
        af2cuda.encode_transition_tensors(dev, pair.view(rows * n, CZ), tws, residual=True, stream=sh)

    for _ in range(3):
        step()
    dev.sync(sh)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(steps):
        step()
    t1.record(stream)
    t1.synchronize()
    dev.sync(sh)
    ms = t0.elapsed_time(t1) / steps
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    flops = 2 * triangle_flops(n) + transition_flops(n)
    del pair
    torch.cuda.empty_cache()
    return {"workload": "BASELINE config 5: N=2048 (4 chains x 512, mask 1 inside the chain blocks), triangle "
                        "multiplication out + in and the pair transition on a bf16 pair updated in place, rows "
                        "sharded over the job's GPUs",
            "ms_per_block": ms, "tflops": flops / (ms * 1e-3) / 1e12,
            "per_gpu_tflops": flops / (ms * 1e-3) / 1e12 / world, "flops_per_block": flops, "steps": steps,
            "warmup": 3, "n_gpus": world}


def cpu_block_rate(n: int, s: int, threads: int) -> tuple[float, float, str]:
    """Times the oracle (CPU restatement of the reference's CPU path) on one block
    at pair length n and s MSA rows: triangle out + in, OPM, pair transition.
    Returns (TFLOP/s, seconds, description)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import numpy as np

    import oracle
    rng = np.random.default_rng(0)
    z = rng.standard_normal((n, n, CZ)).astype(np.float32)
    mask = np.ones((n, n), np.float32)
    msa = rng.standard_normal((s, n, CM)).astype(np.float32)
    msa_mask = np.ones((s, n), np.float32)
    wt = [synthetic_weights(rng) for _ in range(2)]
    wo = opm_weights(rng)
    tw = transition_weights(rng)
    dense = np.concatenate([tw["ln"][0], tw["ln"][1], oracle.dequant_q8_columns(*tw["w1"]).ravel(), tw["b1"],
                            oracle.dequant_q8_columns(*tw["w2"]).ravel(), tw["b2"]])
    t0 = time.perf_counter()
    z = z + oracle.outer_product_mean(msa, msa_mask, wo, C_OUTER, CZ, threads=threads)
    for d in (0, 1):
        z = z + oracle.triangle(d, z, mask, wt[d], 1e-5, threads=threads)
    z = oracle.transition(z.reshape(-1, CZ), dense, HIDDEN, residual=True, threads=threads)
    dt = time.perf_counter() - t0
    return block_flops(n, s) / dt / 1e12, dt, (f"one block at N={n}, S={s} (OPM, triangle out + in, pair "
                                               "transition), f64-accumulating CPU port")


def cpu_sample_size(threads: int, seconds: float, smallest: int = 64) -> tuple[int, int]:
    """Pair length and MSA depth (S = N/2) of a CPU block sample that takes about
    `seconds`, from a calibration run at N=64, S=32 (block FLOPs grow as N^3)."""
    rate, _, _ = cpu_block_rate(64, 32, threads)
    budget = rate * 1e12 * seconds
    n = smallest
    while n < N and block_flops(n + 16, (n + 16) // 2) <= budget:
        n += 16
    return n, n // 2


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    # Size each step's sample so that warm-up plus timed steps take about a minute.
    sample_n, sample_s = cpu_sample_size(threads, 60.0 / max(1, args.steps + args.warmup), smallest=48)
    for _ in range(args.warmup):
        cpu_block_rate(sample_n, sample_s, threads)
    rates, secs = [], []
    for _ in range(args.steps):
        r, sec, desc = cpu_block_rate(sample_n, sample_s, threads)
        rates.append(r)
        secs.append(sec)
    value = statistics.median(rates)
    ms_per_step = block_flops() / (value * 1e12) * 1e3
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": "one Evoformer block's pair GEMM set at N=1024, S=512 (OPM, triangle "
                               f"out + in, pair transition); each step timed on a bounded N={sample_n}, "
                               f"S={sample_s} sample, ms_per_step extrapolated to N=1024 by FLOPs",
                   "N": N, "S": S_MSA, "parallelism": "host threads"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": f"per step: one block at N={sample_n}, S={sample_s} "
                                   f"(median {statistics.median(secs):.2f} s)"},
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
    # prepared weights kept per weights object, as the reference's in-model path keeps its packings
    # (src/evoformer/block.ts:1310-1333): the step launches no preparation kernels after the first
    dev.set_weight_cache(True)
    L = _lib.lib()
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    sh = stream.cuda_stream
    sharded = world > 1
    rows = N // world
    if sharded:
        uid = [af2cuda.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        af2cuda.comm_init(dev, uid[0], world, rank)
    rng = np.random.default_rng(1234)
    gen = torch.Generator(device="cuda").manual_seed(1234 + rank)
    pair = torch.randn(rows, N, CZ, device="cuda", generator=gen).to(torch.bfloat16)
    pair_init = pair.clone()  # the step's input before any step ran (the sharded bit-identity check)
    mask = torch.ones(rows, N, device="cuda")
    # one MSA for the whole job (the same on every rank); a rank holds its own residue columns
    gen_msa = torch.Generator(device="cuda").manual_seed(4321)
    msa_full = torch.randn(S_MSA, N, CM, device="cuda", generator=gen_msa).to(torch.bfloat16)
    msa_mask = (torch.rand(S_MSA, N, device="cuda", generator=gen_msa) < 0.9).float()
    msa_mask[0] = 1
    msa = msa_full[:, rank * rows:(rank + 1) * rows].contiguous() if sharded else msa_full
    w_out = torch.from_numpy(synthetic_weights(rng)).cuda()
    w_in = torch.from_numpy(synthetic_weights(rng)).cuda()
    w_opm = torch.from_numpy(opm_weights(rng)).cuda()
    tw = transition_weights(rng)
    tws = {"layerNormScale": torch.from_numpy(tw["ln"][0]).cuda(), "layerNormOffset": torch.from_numpy(tw["ln"][1]).cuda(),
           "firstWeight": af2cuda.Q8Matrix(torch.from_numpy(tw["w1"][0]).cuda(), torch.from_numpy(tw["w1"][1]).cuda()),
           "firstBias": torch.from_numpy(tw["b1"]).cuda(),
           "secondWeight": af2cuda.Q8Matrix(torch.from_numpy(tw["w2"][0]).cuda(), torch.from_numpy(tw["w2"][1]).cuda()),
           "secondBias": torch.from_numpy(tw["b2"]).cuda()}
    torch.cuda.synchronize()

    def step(pair=pair, msa=msa):
        if sharded:
            af2cuda.encode_outer_product_mean_sharded_tensors(dev, msa, msa_mask, w_opm, C_OUTER, CZ, pair,
                                                              residual=True, stream=sh)
            for d, w in ((0, w_out), (1, w_in)):
                af2cuda.encode_triangle_multiplication_sharded_tensors(dev, d, pair, mask, w, N, residual=True,
                                                                       stream=sh)
        else:
            af2cuda.encode_outer_product_mean_tensors(dev, msa, msa_mask, w_opm, C_OUTER, CZ, pair=pair,
                                                      residual=True, stream=sh)
            af2cuda.encode_triangle_multiplication_tensors(dev, 0, pair, mask, w_out, residual=True, stream=sh)
            af2cuda.encode_triangle_multiplication_tensors(dev, 1, pair, mask, w_in, residual=True, stream=sh)
        af2cuda.encode_transition_tensors(dev, pair.view(rows * N, CZ), tws, residual=True, stream=sh)

    for _ in range(max(args.warmup, 3)):
        step()
    dev.sync(sh)

    def barrier():
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    # ---- timed region: K steps on the device, nothing else running ----
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
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    flops_step = block_flops()
    value = flops_step * args.steps / (ms * 1e-3) / 1e12  # the block's work, shared by the ranks
    peaks = measured_peaks()

    # ---- per-kernel device times (CUDA events around each launch, a separate profiled pass) ----
    L.af2_profile_enable(dev.handle, 1)
    L.af2_profile_reset(dev.handle)
    prof_steps = 3
    for _ in range(prof_steps):
        step()
    dev.sync(sh)
    kernel = {}
    for name in KERNELS:
        c, t = ctypes.c_uint64(), ctypes.c_double()
        L.af2_profile_read(dev.handle, name.encode(), ctypes.byref(c), ctypes.byref(t))
        if c.value:
            kernel[name] = {"launches_per_step": c.value / prof_steps, "avg_us": t.value / c.value * 1e3,
                            "ms_per_step": t.value / prof_steps, "share": 0.0}
    L.af2_profile_enable(dev.handle, 0)
    total_kernel_ms = sum(k["ms_per_step"] for k in kernel.values()) or 1.0
    for k in kernel.values():
        k["share"] = k["ms_per_step"] / total_kernel_ms

    # ---- roofline of the dominant kernel ----
    tensor = {k: v for k, v in kernel.items() if kernel_step_flops(k, world) is not None}
    dom = max(tensor, key=lambda k: tensor[k]["ms_per_step"])
    step_fl = kernel_step_flops(dom, world)
    achieved = step_fl / (tensor[dom]["ms_per_step"] * 1e-3) / 1e12
    per_launch = step_fl / tensor[dom]["launches_per_step"]
    traffic = KERNEL_DRAM_BYTES.get(dom) if world == 1 else None
    roofline = {"kernel": dom, "bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"],
                "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops"], "traffic": traffic,
                "peak_source": f"{peaks['source']} burst bf16", "flops_per_launch": per_launch,
                "avg_launch_us": tensor[dom]["avg_us"]}

    # ---- e2e: the public device-form API, inputs copied in from pinned host memory every step ----
    # Every step copies its pair rows and MSA in from pinned host memory and reads its pair rows
    # back.  With two device copies of the inputs, step k+1's host->device copies (one copy
    # stream) and step k-1's device->host read (another) run while step k's block computes, and
    # the two directions share PCIe full duplex; the timed region spans all copies of all steps.
    host_pair = torch.empty(rows, N, CZ, dtype=torch.bfloat16, pin_memory=True)
    host_pair.copy_(pair.cpu())
    host_msa = torch.empty(msa.shape, dtype=torch.bfloat16, pin_memory=True)
    host_msa.copy_(msa.cpu())
    host_out = torch.empty_like(host_pair, pin_memory=True)
    pairs2, msas2 = [pair, torch.empty_like(pair)], [msa, torch.empty_like(msa)]
    h2d_s, d2h_s = torch.cuda.Stream(), torch.cuda.Stream()

    def e2e_run(steps):
        free = [None, None]  # buffer b has been read back (so its last block is done too)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(h2d_s)
        for k in range(steps):
            b = k % 2
            with torch.cuda.stream(h2d_s):
                if free[b] is not None:
                    h2d_s.wait_event(free[b])
                pairs2[b].copy_(host_pair, non_blocking=True)
                msas2[b].copy_(host_msa, non_blocking=True)
                ready = torch.cuda.Event()
                ready.record(h2d_s)
            stream.wait_event(ready)
            step(pairs2[b], msas2[b])
            done = torch.cuda.Event()
            done.record(stream)
            with torch.cuda.stream(d2h_s):
                d2h_s.wait_event(done)
                host_out.copy_(pairs2[b], non_blocking=True)
                free[b] = torch.cuda.Event()
                free[b].record(d2h_s)
        for f in free:
            if f is not None:
                stream.wait_event(f)
        t1.record(stream)
        t1.synchronize()
        return t0.elapsed_time(t1)

    e2e_run(2)
    torch.cuda.synchronize()
    e2e_steps = max(3, min(args.steps, 10))
    barrier()
    e2e_ms = e2e_run(e2e_steps)
    if dist:
        t = torch.tensor([e2e_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e = {"value": flops_step * e2e_steps / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
           "h2d_bytes_per_step": host_pair.numel() * 2 + host_msa.numel() * 2,
           "d2h_bytes_per_step": host_out.numel() * 2, "ms_per_step": e2e_ms / e2e_steps,
           "path": "pair (this rank's rows) and MSA (this rank's residue columns) copied in from pinned host "
                   "memory, the block through the af2cuda device-form API (outer product mean, triangle "
                   "multiplication x2, transition; the row-sharded forms on several GPUs), pair rows read back; "
                   "copies of neighbouring steps overlap the block (two device input buffers, separate copy "
                   "streams)"}

    # ---- sharded: one step checked bit for bit against the single-GPU block on rank 0 ----
    identical = None
    if sharded:
        got = pair_init.clone()
        step(got, msa)
        dev.sync(sh)
        torch.cuda.synchronize()
        inits = [torch.empty_like(pair_init) for _ in range(world)]
        outs = [torch.empty_like(got) for _ in range(world)]
        dist.all_gather(inits, pair_init)
        dist.all_gather(outs, got)
        flag = torch.zeros(1, device="cuda")
        if rank == 0:
            whole = torch.cat(inits).contiguous()
            mask_whole = torch.ones(N, N, device="cuda")
            af2cuda.encode_outer_product_mean_tensors(dev, msa_full, msa_mask, w_opm, C_OUTER, CZ, pair=whole,
                                                      residual=True, stream=sh)
            af2cuda.encode_triangle_multiplication_tensors(dev, 0, whole, mask_whole, w_out, residual=True, stream=sh)
            af2cuda.encode_triangle_multiplication_tensors(dev, 1, whole, mask_whole, w_in, residual=True, stream=sh)
            af2cuda.encode_transition_tensors(dev, whole.view(N * N, CZ), tws, residual=True, stream=sh)
            dev.sync(sh)
            flag[0] = 1.0 if torch.equal(whole, torch.cat(outs)) else 0.0
        dist.broadcast(flag, src=0)
        identical = bool(flag.item() == 1.0)

    # ---- the multimer config: N=2048, chain-block mask, triangle out + in and the
    # pair transition, rows sharded over the same ranks ----
    multimer = multimer_block(dev, torch, af2cuda, rng, world, rank, sh, stream, dist)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        rate, secs, desc = cpu_block_rate(*cpu_sample_size(threads, 15.0), threads)
        cpu = {"value": rate, "unit": "TFLOP/s", "cores": threads, "kind": "port",
               "sample": f"{desc} ({secs:.1f} s)"}

    if dist:
        dist.barrier()
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong" if world > 1 else "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": "one Evoformer block's pair GEMM set at N=1024 (OPM of an S=512, c_m=256 MSA "
                                   "into the pair, triangle multiplication outgoing + incoming with c_z=c_hidden="
                                   "128, pair transition 128->512->128 with mixed-q8 weights), bf16 pair updated "
                                   "in place, f16 tensor-core operands with f32 accumulation",
                       "N": N, "S": S_MSA, "c_m": CM, "c_outer": C_OUTER, "c_z": CZ, "c_hidden": CH,
                       "flops_per_step": flops_step,
                       "gflop_per_block": {"triangle": 2 * triangle_flops(N) / 1e9, "opm": opm_flops(N) / 1e9,
                                           "transition": transition_flops(N) / 1e9},
                       "l2": "inputs larger than L2 (pair 268 MB, MSA 268 MB, bf16), no flush",
                       "parallelism": (f"pair rows sharded x{world}: triangle contraction sharded by hidden "
                                       "channel between two all-to-alls (copy-engine copies into the peers' "
                                       "IPC-mapped scratch, NCCL barriers), OPM right operand all-gathered")
                       if world > 1
                       else "single GPU"},
            "ms_per_block": ms / args.steps,
            "pct_of_peak": value / world / peaks["bf16_tflops"],
            "per_gpu_tflops": value / world,
            "roofline": roofline, "kernels": kernel, "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": int(launches), "clocks": clocks.record(),
            "multimer_n2048": multimer,
        }
        if identical is not None:
            line["sharded_bit_identical"] = identical
        print(json.dumps(line), flush=True)
    if sharded:
        af2cuda.comm_destroy(dev)
    if dist:
        dist.destroy_process_group()
    dev.close()


WORKLOADS = {
    "tri128": "config 1: triangle multiplication outgoing, z [128,128,128] f32 ~N(0,1), mask 1, f32 output",
    "transition": "config 2: pair transition, X [65536,128] f16 ~N(0,1), LayerNorm in, 128->512 ReLU ->128 with "
                  "symmetric int8 weights and f32 per-output-channel scales, f16 output",
    "opm": "config 3: outer product mean, MSA [512,256,256] f32 ~N(0,1), mask Bernoulli(0.9) with row 0 ones, "
           "c=32, output [256,256,128] f32",
    "block768": "config 4: one block's pair GEMM set at N=768 (OPM with S=512, c_m=256; triangle out + in; pair "
                "transition with mixed-q8 weights), bf16 pair updated in place",
    "multimer": "config 5: N=2048 (4 chains x 512, mask 1 inside the four diagonal chain blocks): triangle out + "
                "in and pair transition on a bf16 pair [2048,2048,128] updated in place, rows sharded over the ranks",
    "triangle_attention": "next-row widening: triangle attention around the starting and the ending node at "
                          "N=1024 (c_z=128, 4 heads of 32, pair bias from the normalised pair, mask 1), bf16 pair "
                          "updated in place",
    "pair_block": "next-row widening: the whole Evoformer pair block at N=1024 through one af2_evoformer_pair_block "
                  "call (OPM of an S=512, c_m=256 MSA, triangle multiplication out + in, triangle attention "
                  "starting + ending, pair transition with mixed-q8 weights), bf16 pair updated in place",
    "msa_transition": "next-row widening: the MSA transition of the N=1024 block, bf16 MSA rows [512*1024, 256] "
                      "updated in place, 256->1024 ReLU ->256 with symmetric int8 weights and f32 per-output-"
                      "channel scales",
}


def run_workload(args) -> None:
    """The other BASELINE configs: one step is one call of the named op (or block) on
    resident device inputs; value = its algorithmic TFLOP/s (kernel-cost.ts formulas)."""
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
        if args.workload != "multimer":
            raise SystemExit(f"--workload {args.workload} runs on one GPU; only 'multimer' is sharded")
        import datetime

        import torch.distributed as td
        td.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
        dist = td
    dev = af2cuda.Device(local)
    dev.set_weight_cache(True)  # as in the default block: weights prepared once
    L = _lib.lib()
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    sh = stream.cuda_stream
    if world > 1:
        uid = [af2cuda.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        af2cuda.comm_init(dev, uid[0], world, rank)
    rng = np.random.default_rng(0)
    gen = torch.Generator(device="cuda").manual_seed(rank)
    tw = transition_weights(rng)

    def transition_tensors(tw=tw):
        return {"layerNormScale": torch.from_numpy(tw["ln"][0]).cuda(),
                "layerNormOffset": torch.from_numpy(tw["ln"][1]).cuda(),
                "firstWeight": af2cuda.Q8Matrix(torch.from_numpy(tw["w1"][0]).cuda(),
                                                torch.from_numpy(tw["w1"][1]).cuda()),
                "firstBias": torch.from_numpy(tw["b1"]).cuda(),
                "secondWeight": af2cuda.Q8Matrix(torch.from_numpy(tw["w2"][0]).cuda(),
                                                 torch.from_numpy(tw["w2"][1]).cuda()),
                "secondBias": torch.from_numpy(tw["b2"]).cuda()}

    wl = args.workload
    if wl == "tri128":
        n = 128
        z = torch.randn(n, n, CZ, device="cuda", generator=gen)
        mask = torch.ones(n, n, device="cuda")
        w = torch.from_numpy(synthetic_weights(rng)).cuda()
        out = torch.empty_like(z)
        flops = triangle_flops(n)

        def step():
            af2cuda.encode_triangle_multiplication_tensors(dev, 0, z, mask, w, out=out, residual=False, stream=sh)
    elif wl == "transition":
        rows = 65536
        x = torch.randn(rows, CZ, device="cuda", generator=gen).half()
        out = torch.empty_like(x)
        tws = transition_tensors()
        flops = 4.0 * rows * CZ * HIDDEN

        def step():
            af2cuda.encode_transition_tensors(dev, x, tws, out=out, residual=False, stream=sh)
    elif wl == "msa_transition":
        rows, c, h = S_MSA * N, CM, 4 * CM
        x = torch.randn(rows, c, device="cuda", generator=gen).to(torch.bfloat16)
        tws = transition_tensors(transition_weights(rng, c, h))
        flops = 4.0 * rows * c * h

        def step():
            af2cuda.encode_transition_tensors(dev, x, tws, residual=True, stream=sh)
    elif wl in ("triangle_attention", "pair_block"):
        n = args.length or N
        pair = torch.randn(n, n, CZ, device="cuda", generator=gen).to(torch.bfloat16)
        mask = torch.ones(n, n, device="cuda")
        w_att = [torch.from_numpy(attention_weights(rng)).cuda() for _ in range(2)]
        flops = 2 * attention_flops(n)
        if n != N and wl == "pair_block":
            raise SystemExit("--length applies to triangle_attention only")
        if wl == "pair_block":
            msa = torch.randn(S_MSA, n, CM, device="cuda", generator=gen).to(torch.bfloat16)
            msa_mask = (torch.rand(S_MSA, n, device="cuda", generator=gen) < 0.9).float()
            msa_mask[0] = 1
            block_w = {"outerProductMean": torch.from_numpy(opm_weights(rng)).cuda(),
                       "triangleMultiplicationOutgoing": torch.from_numpy(synthetic_weights(rng)).cuda(),
                       "triangleMultiplicationIncoming": torch.from_numpy(synthetic_weights(rng)).cuda(),
                       "triangleAttentionStarting": w_att[0], "triangleAttentionEnding": w_att[1],
                       "pairTransition": transition_tensors()}
            flops += block_flops(n)

        def step():
            if wl == "pair_block":
                af2cuda.encode_evoformer_pair_block_tensors(dev, pair, mask, block_w, msa=msa, msa_mask=msa_mask,
                                                            c_outer=C_OUTER, c_hidden=CH, pair_heads=PAIR_HEADS,
                                                            stream=sh)
            else:
                af2cuda.encode_triangle_attention_tensors(dev, "starting", pair, mask, w_att[0], PAIR_HEADS, stream=sh)
                af2cuda.encode_triangle_attention_tensors(dev, "ending", pair, mask, w_att[1], PAIR_HEADS, stream=sh)
    elif wl == "opm":
        n, s = 256, 512
        msa = torch.randn(s, n, CM, device="cuda", generator=gen)
        msa_mask = (torch.rand(s, n, device="cuda", generator=gen) < 0.9).float()
        msa_mask[0] = 1
        w = torch.from_numpy(opm_weights(rng)).cuda()
        out = torch.empty(n, n, CZ, device="cuda")
        flops = opm_flops(n, s)

        def step():
            af2cuda.encode_outer_product_mean_tensors(dev, msa, msa_mask, w, C_OUTER, CZ, out=out, residual=False,
                                                      stream=sh)
    else:
        n = 768 if wl == "block768" else 2048
        s = S_MSA
        rows = n // world
        r0 = rank * rows
        pair = torch.randn(rows, n, CZ, device="cuda", generator=gen).to(torch.bfloat16)
        if wl == "multimer":
            chain = torch.arange(n, device="cuda") // 512
            mask = (chain[r0:r0 + rows, None] == chain[None, :]).float().contiguous()
        else:
            mask = torch.ones(rows, n, device="cuda")
            msa = torch.randn(s, n, CM, device="cuda", generator=gen).to(torch.bfloat16)
            msa_mask = (torch.rand(s, n, device="cuda", generator=gen) < 0.9).float()
            msa_mask[0] = 1
            w_opm = torch.from_numpy(opm_weights(rng)).cuda()
        w_tri = [torch.from_numpy(synthetic_weights(rng)).cuda() for _ in range(2)]
        tws = transition_tensors()
        flops = 2 * triangle_flops(n) + transition_flops(n) + (opm_flops(n, s) if wl == "block768" else 0.0)

        def step():
            if wl == "block768":
                af2cuda.encode_outer_product_mean_tensors(dev, msa, msa_mask, w_opm, C_OUTER, CZ, pair=pair,
                                                          residual=True, stream=sh)
            for d in (0, 1):
                if world > 1:
                    af2cuda.encode_triangle_multiplication_sharded_tensors(dev, d, pair, mask, w_tri[d], n,
                                                                           residual=True, stream=sh)
                else:
                    af2cuda.encode_triangle_multiplication_tensors(dev, d, pair, mask, w_tri[d], residual=True,
                                                                   stream=sh)
            af2cuda.encode_transition_tensors(dev, pair.view(rows * n, CZ), tws, residual=True, stream=sh)
    torch.cuda.synchronize()
    for _ in range(max(args.warmup, 3)):
        step()
    dev.sync(sh)

    def barrier():
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

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
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = flops * args.steps / (ms * 1e-3) / 1e12
    peaks = measured_peaks()
    L.af2_profile_enable(dev.handle, 1)
    L.af2_profile_reset(dev.handle)
    for _ in range(3):
        step()
    dev.sync(sh)
    kernel = {}
    for name in KERNELS:
        c, t = ctypes.c_uint64(), ctypes.c_double()
        L.af2_profile_read(dev.handle, name.encode(), ctypes.byref(c), ctypes.byref(t))
        if c.value:
            kernel[name] = {"launches_per_step": c.value / 3, "avg_us": t.value / c.value * 1e3,
                            "ms_per_step": t.value / 3}
    L.af2_profile_enable(dev.handle, 0)
    total = sum(k["ms_per_step"] for k in kernel.values()) or 1.0
    for k in kernel.values():
        k["share"] = k["ms_per_step"] / total
    roofline = None
    if wl in ("triangle_attention", "pair_block") and not args.length:
        # the dominant tensor kernel of the N=1024 workload, as in the default line
        tensor = {k: v for k, v in kernel.items() if kernel_step_flops(k) is not None}
        dom = max(tensor, key=lambda k: tensor[k]["ms_per_step"])
        achieved = kernel_step_flops(dom) / (tensor[dom]["ms_per_step"] * 1e-3) / 1e12
        roofline = {"kernel": dom, "bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"],
                    "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops"], "traffic": None,
                    "peak_source": f"{peaks['source']} burst bf16", "avg_launch_us": tensor[dom]["avg_us"]}
    if dist:
        dist.barrier()
    if rank == 0:
        print(json.dumps({
            "metric": f"{wl} TFLOP/s", "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": WORKLOADS[wl], "flops_per_step": flops},
            "pct_of_peak": value / world / peaks["bf16_tflops"], "peak_source": f"{peaks['source']} burst bf16",
            "kernels": kernel, "roofline": roofline, "gpu_launches": int(launches),
            "clocks": clocks.record()}), flush=True)
    if world > 1:
        af2cuda.comm_destroy(dev)
    if dist:
        dist.destroy_process_group()
    dev.close()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["block", *WORKLOADS], default="block",
                    help="block (default): the metric's N=1024 block; the others: the remaining BASELINE configs")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--length", type=int, default=0,
                    help="triangle_attention / pair_block: residues N (default 1024; smaller for profiling)")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.workload != "block":
        run_workload(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
