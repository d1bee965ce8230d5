"""Benchmark of the rouge-numerics-b200 hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One GPU (the configuration the headline metric is quoted
on): the W8A8 linear step. X[4096][4096] f32 ~ N(0,1) with 1% of entries
x20, W[4096][4096] f32 ~ N(0, 0.02) quantized once per output channel. One
step = per-token int8 quantization of X + int8 x int8 -> int32 tcgen05 GEMM
with the dequant ((float)acc * sx) * sw fused into the epilogue, f32 output,
all in one launch. `value` = 2*M*N*K / step time (TOP/s), inputs resident in
HBM and larger than L2 (four rotating device copies of the step's data), K
steps launched back to back between one pair of CUDA events. `e2e` = the
same metric through the drop-in host-pointer C ABI (rouge_quantize_i8_channel
+ rouge_gemm_i8) from pinned host buffers, copies included. The config-5 GEMM
on one GPU is reported beside it (`config5_g1`).

N GPUs (torchrun, one rank per GPU; BASELINE config 5, the sharded GEMM):
M=16384, K=8192, N=28672 int8 W8A8 with W split N-wise over the N GPUs,
bf16 output, the whole C[M][N] on every rank at the end of each step (the
all-gather is fused into the GEMM epilogue). `value` = 2*M*N*K / step time
of the whole job (strong scaling), max over ranks. `e2e` adds, every step,
the copy of the int8 activations from pinned host memory and of a 1/N band
of C's rows back to the host on every rank. N independent config-2 replicas
are reported beside it (`config2_replicas`).

--impl reference times the reference rouge-numerics CPU implementation
(oracle/_ref, compiled from the reference sources) on this host's cores for
the same workload, metric and config, on a bounded row sample per step; its
process loads only the checker libraries under oracle/.
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

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "rouge-v_b200"))

PEAKS_PATH = os.path.join(ROOT, "MEASURED_PEAKS.json")
FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks():
    try:
        with open(PEAKS_PATH) as f:
            p = json.load(f)
        return p, "measured"
    except OSError:
        return FALLBACK, "fallback"


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ workload

M = N = K = 4096
SETS = 4   # rotating device copies of the step's data (inputs larger than L2)
# DRAM bytes (read + write) of one fused launch: dram__bytes_read.sum +
# dram__bytes_write.sum of an ncu --set full capture of this workload
FUSED_TRAFFIC = 116.4e6


M5, N5, K5 = 16384, 28672, 8192
METRIC = "W8A8 int8 GEMM TOP/s (int8 x int8 -> int32 tcgen05 GEMM, fused dequant)"


def workload_config(world):
    """The `config` of the JSON line, shared by both arms (same dict)."""
    if world == 1:
        return {"workload": "w8a8_linear_4096 (BASELINE config 2): per-token int8 quantization "
                            "of X + int8 GEMM + fused dequant, f32 out",
                "M": M, "N": N, "K": K, "out": "f32",
                "weights": "pre-quantized per output channel (setup)",
                "l2": f"inputs larger than L2: {SETS} rotating device copies of X, codes, "
                      "quantized W and C (160 MB per step, 640 MB in all); K steps launched "
                      "back to back between one pair of CUDA events",
                "parallelism": "single GPU"}
    return {"workload": f"sharded_w8a8 (BASELINE config 5): M={M5} K={K5} N={N5} int8 "
                        f"activations and weights, W split N-wise over {world} GPUs, int32 "
                        "accumulation, bf16 out, C[M][N] complete on every rank",
            "M": M5, "N": N5, "K": K5, "out": "bf16",
            "weights": "pre-quantized per output channel (setup), each rank its column block",
            "l2": "inputs larger than L2 (every step writes the 939.5 MB C on every rank); K "
                  "steps launched back to back between one pair of CUDA events",
            "parallelism": f"N-sharded x{world} over output columns, all-gather fused into the "
                           "GEMM epilogue (NVLink)"}


def make_inputs(gen):
    """Config-2 inputs from `gen` (the product library's generator, or the
    checker library's bit-identical copy in the reference arm)."""
    X = gen.synth_normal(1, (M, K), 0.0, 1.0)
    gen.synth_outliers(1, X, 0.01, 20.0)
    W = gen.synth_normal(2, (N, K), 0.0, 0.02)
    return X, W


def l2_flush(buf):
    """Evict the 126 MB L2 before a timed step: write the first 256 MiB half
    of `buf`, then read the second half, so the write-backs of the dirty lines
    happen here and not inside the next timed kernel."""
    half = buf.numel() // 2
    buf[:half].zero_()
    buf[half:].view(torch_int32()).sum()


def torch_int32():
    import torch
    return torch.int32


def run_config2(args, rank, world, local_rank):
    """BASELINE config 2 on this rank's GPU (one replica per rank): the
    W8A8 step timed as one fused launch and as two launches, its parity on
    sampled rows and, on request, its drop-in end-to-end number."""
    import torch
    import rouge_b200 as rb

    dev = torch.device("cuda", local_rank)
    peaks, peak_src = load_peaks()
    X, W = make_inputs(rb)
    Xh = torch.from_numpy(X).pin_memory()
    Wh = torch.from_numpy(W).pin_memory()
    # SETS independent copies of the step's device data (X, its codes and
    # scales, the quantized weights, C): 160 MB per set, so a step's inputs
    # were last touched SETS-1 steps (480 MB of traffic) earlier and come
    # from HBM, not from the 126 MB L2.
    wd = Wh.to(dev)
    qw0 = torch.empty((N, K), dtype=torch.int8, device=dev)
    sw = torch.empty(N, dtype=torch.float32, device=dev)
    rb.quantize_i8_rows(wd, sw, qw0)          # weights: quantized once per output channel
    del wd
    sets = []
    for j in range(SETS):
        sets.append({"x": Xh.to(dev), "qx": torch.empty((M, K), dtype=torch.int8, device=dev),
                     "sx": torch.empty(M, dtype=torch.float32, device=dev),
                     "qw": qw0.clone(), "c": torch.empty((M, N), dtype=torch.float32, device=dev),
                     "ws": rb.w8a8_workspace(M, dev)})
    del qw0
    busy = torch.zeros(512 << 20, dtype=torch.uint8, device=dev)

    def step(s):
        # one launch: the per-row quantizer fused into the CTA-pair GEMM
        rb.w8a8_linear(s["x"], s["qw"], sw, s["qx"], s["sx"], s["c"], rb.OUT_F32, s["ws"])

    def quant(s):
        rb.quantize_i8_rows(s["x"], s["sx"], s["qx"])

    def gemm(s):
        rb.gemm_i8(s["qx"], s["qw"], rb.B_NK, s["c"], rb.OUT_F32, s["sx"], 1, sw, 1)

    def keep_busy():
        # ~80 us read of 512 MiB (clean L2 lines): the device is still busy
        # when the timed region's first event is recorded, so host launch
        # latency does not land inside it.
        busy.view(torch.int32).sum()

    # The clock sampler starts before the warm-up: an idle pause right
    # before the timed region would let the GPU settle into a slower state
    # for the first milliseconds of it.
    clocks = ClockSampler(local_rank) if world == 1 else None
    if clocks:
        clocks.start()
        time.sleep(0.3)
    dist = None
    if world > 1:
        import torch.distributed as dist
    # The device read that precedes the timed region is launched once here:
    # its first launch in a process loads its kernel, which left the GPU idle
    # for ~30 us inside the timed region when it happened there.
    keep_busy()
    torch.cuda.synchronize()
    for i in range(args.warmup):
        step(sets[i % SETS])
    rb.sync_status()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    # Timed region: K steps launched back to back, one event pair around all.
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    keep_busy()
    e0.record()
    for i in range(args.steps):
        step(sets[i % SETS])
    e1.record()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clk = clocks.stop() if clocks else None
    rb.sync_status()
    t_step = e0.elapsed_time(e1) / args.steps

    # The same step as two launches (quantizer, then GEMM; a second run of K
    # steps with an event between every two kernels): each kernel's own
    # device time, and the GEMM's roofline on its own.
    for i in range(3):
        quant(sets[i % SETS])
        gemm(sets[i % SETS])
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(2 * args.steps + 1)]
    keep_busy()
    evs[0].record()
    for i in range(args.steps):
        quant(sets[i % SETS])
        evs[2 * i + 1].record()
        gemm(sets[i % SETS])
        evs[2 * i + 2].record()
    torch.cuda.synchronize()
    rb.sync_status()
    t_quant = sum(evs[2 * i].elapsed_time(evs[2 * i + 1]) for i in range(args.steps)) / args.steps
    t_gemm = sum(evs[2 * i + 1].elapsed_time(evs[2 * i + 2]) for i in range(args.steps)) / args.steps
    # the quantizer alone: K launches back to back over the rotating sets
    # (inputs larger than L2), one event pair around them
    for i in range(3):
        quant(sets[i % SETS])
    keep_busy()
    q0 = torch.cuda.Event(enable_timing=True)
    q1 = torch.cuda.Event(enable_timing=True)
    q0.record()
    for i in range(args.steps):
        quant(sets[i % SETS])
    q1.record()
    torch.cuda.synchronize()
    rb.sync_status()
    t_quant_alone = q0.elapsed_time(q1) / args.steps
    # the plain GEMM alone: K launches back to back over the rotating sets
    # (the two-launch timing above puts an event between every two kernels,
    # which keeps each GEMM's set-up from overlapping the kernel before it)
    keep_busy()
    g0 = torch.cuda.Event(enable_timing=True)
    g1 = torch.cuda.Event(enable_timing=True)
    g0.record()
    for i in range(args.steps):
        gemm(sets[i % SETS])
    g1.record()
    torch.cuda.synchronize()
    rb.sync_status()
    t_gemm_alone = g0.elapsed_time(g1) / args.steps
    if dist:
        t = torch.tensor([t_step, t_gemm, t_quant, t_quant_alone, t_gemm_alone], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        t_step, t_gemm, t_quant, t_quant_alone, t_gemm_alone = t.tolist()
    # The SM clock the fused launch itself runs at, from its CTAs' own
    # %clock64 / %globaltimer stamps (rouge_b200_set_clock_probe), on an
    # untimed repeat of the timed loop: nvidia-smi samples the clock every
    # 200 ms and so mostly between launches. Same collective steps on every
    # rank (none inside).
    with rb.clock_probe(2 * torch.cuda.get_device_properties(dev).multi_processor_count,
                        dev) as probe:
        keep_busy()
        for i in range(args.steps):
            step(sets[i % SETS])
        torch.cuda.synchronize()
        mhz = probe.sm_mhz()
    rb.sync_status()
    kernel_clock = {"sm_mhz_median": round(float(np.median(mhz)), 1) if len(mhz) else None,
                    "sm_mhz_min": round(float(np.min(mhz)), 1) if len(mhz) else None,
                    "ctas": int(len(mhz)),
                    "how": "per-CTA %clock64 / %globaltimer stamps of the last fused launch of an "
                           "untimed repeat of the timed loop (rouge_b200_set_clock_probe)"}
    # parity on the fused launch's own outputs
    last = sets[0]
    step(last)
    rb.sync_status()
    qx, sx, qw, C = last["qx"], last["sx"], last["qw"], last["c"]

    ops = 2.0 * M * N * K
    value = world * ops / (t_step * 1e-3) / 1e12
    gemm_tops = ops / (t_gemm * 1e-3) / 1e12
    quant_bytes = M * K * 5 + M * 4
    quant_gbs = quant_bytes / (t_quant * 1e-3) / 1e9
    quant_alone_gbs = quant_bytes / (t_quant_alone * 1e-3) / 1e9
    int8_peak = 2.0 * peaks["bf16_tflops"]

    res = {
        "value": round(value, 2), "ms_per_step": round(t_step, 5),
        # the step is one launch: its average duration is ms_per_step
        "roofline": {"bound": "tensor",
                     "kernel": "gemm_tc2_kernel<I8, fused row quantizer> (2-CTA pairs, 256x256 "
                               "tiles; one launch per step)",
                     "achieved": round(value / world, 2), "peak": round(int8_peak, 1),
                     "unit": "TOP/s", "frac": round(value / world / int8_peak, 4),
                     # dram__bytes_read.sum + dram__bytes_write.sum of one launch,
                     # ncu capture summarised in profiles/
                     "traffic": FUSED_TRAFFIC, "traffic_unit": "bytes per launch (ncu)",
                     "peak_source": f"2 x {peak_src} dense bf16 ({peaks['bf16_tflops']} TF/s); "
                                    "int8 dense rate is twice bf16 on B200",
                     "frac_of_datasheet_4500": round(value / world / 4500.0, 4)},
        # the same step as two launches (rouge_b200_quantize_i8_rows, then
        # rouge_b200_gemm_i8): each kernel's own time and roofline
        "kernels": {"two_launch_ms": round(t_gemm + t_quant, 5),
                    "gemm_ms": round(t_gemm, 5), "gemm_tops": round(gemm_tops, 2),
                    "gemm_frac": round(gemm_tops / int8_peak, 4),
                    "gemm_traffic": 56.28e6,
                    "gemm_alone_ms": round(t_gemm_alone, 5),
                    "gemm_alone_frac": round(ops / (t_gemm_alone * 1e-3) / 1e12 / int8_peak, 4),
                    "quant_ms": round(t_quant, 5), "quant_gbs": round(quant_gbs, 1),
                    "quant_hbm_frac": round(quant_gbs / peaks["hbm_gbs"], 4),
                    "quant_alone_ms": round(t_quant_alone, 5),
                    "quant_alone_hbm_frac": round(quant_alone_gbs / peaks["hbm_gbs"], 4),
                    "quant_note": "quant_ms: inside the two-launch step (absorbs the previous "
                                  "GEMM's 64 MB f32 write-back); quant_alone / gemm_alone: K "
                                  "launches back to back over the rotating input sets"},
        "clocks": clk,
        "sm_clock_in_kernel": kernel_clock,
    }
    if not args.profile:
        # parity of this run's output against the oracle on sampled rows
        res["parity"] = check_parity(rb, X, qx, sx, qw, sw, C)
        if args.e2e:
            # e2e through the drop-in C ABI from pinned host buffers
            res["e2e"] = run_e2e(args, rb, torch, Xh, qw, sw, dev, dist)
    del Xh, Wh, qx, qw, C, sets, last, busy
    return res, X, W


def run_ours(args, rank, world, local_rank):
    import torch
    import rouge_b200 as rb

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    peaks, peak_src = load_peaks()
    if world > 1:
        return run_sharded_headline(args, rank, world, local_rank, peaks, peak_src)

    args.e2e = not args.profile
    c2, X, W = run_config2(args, rank, world, local_rank)
    line = {
        "metric": METRIC,
        "value": c2["value"],
        "unit": "TOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": c2["ms_per_step"],
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "int8",
        "data": "synthetic (seeded splitmix64/Box-Muller, BASELINE config 2 distributions)",
        "config": workload_config(world),
        "roofline": c2["roofline"],
        "kernels": c2["kernels"],
        "parity": c2.get("parity"),
        "e2e": c2.get("e2e"),
        "clocks": c2["clocks"],
        "sm_clock_in_kernel": c2["sm_clock_in_kernel"],
        "gpu_launches": args.steps,
    }
    if args.profile:
        return line
    line["cpu_baseline"] = cpu_baseline(X, W)
    del X, W
    flush = torch.zeros(512 << 20, dtype=torch.uint8, device=dev)
    # the config-5 GEMM on this one GPU (g = 1), before the long tail of
    # other configurations
    line["config5_g1"] = run_config5(args, rank, world, local_rank, peaks, flush, compact=True)
    line["other_configs"] = other_configs(rb, torch, dev, peaks, peak_src, flush)
    return line


def run_sharded_headline(args, rank, world, local_rank, peaks, peak_src):
    """N > 1: the headline is BASELINE config 5 sharded over the N ranks
    (strong scaling, whole-job TOP/s); N config-2 replicas beside it."""
    import torch
    dev = torch.device("cuda", local_rank)
    flush = torch.zeros(512 << 20, dtype=torch.uint8, device=dev)
    c5 = run_config5(args, rank, world, local_rank, peaks, flush, compact=False)
    args.e2e = False
    c2, X, W = run_config2(args, rank, world, local_rank)
    del X, W
    line = {
        "metric": METRIC,
        "value": c5["value"],
        "unit": "TOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": c5["ms_per_step"],
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "int8",
        "data": "synthetic (seeded splitmix64/Box-Muller, BASELINE config 5 distributions)",
        "config": workload_config(world),
        "roofline": c5["roofline"],
        "parity": c5["parity"],
        "e2e": c5["e2e"],
        "clocks": c5["clocks"],
        "gpu_launches": args.steps,
        "config5": c5["detail"],
        "config2_replicas": {"value": c2["value"], "ms_per_step": c2["ms_per_step"],
                             "scaling": "weak", "note": f"{world} independent config-2 steps, "
                             "one per GPU, no collective (sum over ranks)",
                             "frac_per_gpu": c2["roofline"]["frac"], "parity": c2.get("parity")},
    }
    return line


# ------------------------------------------------------------------ config 5 (sharded)


def run_config5(args, rank, world, local_rank, peaks, flush, compact):
    """W8A8 GEMM M=16384, K=8192, N=28672 with W split
    N-wise over the `world` GPUs, int32 accumulation, dequant to bf16, the
    output assembled row-major C[M][N] on every rank. Strong scaling.

    The product form (fused: each epilogue tile is written into every
    rank's C, through NVLink multicast stores or TMA stores to each peer,
    then a device-side barrier) is timed over K back-to-back steps between
    one event pair, max over ranks; its e2e adds the host copies. With
    compact=False the other fused form and the NCCL form (the GEMM in row
    bands, each band all-gathered by NCCL on a communication stream, then a
    layout kernel) are timed too, as baselines."""
    import torch
    import rouge_b200 as rb
    from rouge_b200.sharded import FusedShardedW8A8, ShardedW8A8, shard_columns
    dist = None
    if world > 1:
        import torch.distributed as dist
    dev = torch.device("cuda", local_rank)
    ns, ranges = shard_columns(N5, world)
    n0, n1 = ranges[rank]
    ncols = n1 - n0
    # activations: full X on every rank, quantized per token (setup: the
    # config's inputs are int8)
    x = torch.from_numpy(rb.synth_normal(8, (M5, K5), 0.0, 1.0))
    rb.synth_outliers(8, x.numpy(), 0.01, 20.0)
    xd = x.to(dev)
    del x
    qx = torch.empty((M5, K5), dtype=torch.int8, device=dev)
    sx = torch.empty(M5, dtype=torch.float32, device=dev)
    rb.quantize_i8_rows(xd, sx, qx)
    del xd
    # this rank's weight rows [n0, n1), quantized per output channel (setup)
    w = torch.zeros((ns, K5), dtype=torch.float32)
    if ncols > 0:
        w[:ncols] = torch.from_numpy(rb.synth_normal_at(9, n0 * K5, (ncols, K5), 0.0, 0.02))
    wd = w.to(dev)
    del w
    qw = torch.empty((ns, K5), dtype=torch.int8, device=dev)
    sw = torch.empty(ns, dtype=torch.float32, device=dev)
    rb.quantize_i8_rows(wd, sw, qw)
    del wd
    torch.cuda.synchronize()

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    orc = O.Oracle()
    # rows at the first, middle and last row bands of C and at NCCL band
    # edges; every rank checks its own columns (both shard edges included)
    rows = np.array([0, 1, 127, 128, 2047, 2048, 8191, 16383], np.int32)
    want = None
    if ncols > 0:
        _, c = orc.gemm_i8(qx[rows.tolist()].cpu().numpy(), qw[:ncols].cpu().numpy(), True,
                           sx[rows.tolist()].cpu().numpy(), 1, sw[:ncols].cpu().numpy(), 1)
        want = orc.bf16_encode(c)
    ops = 2.0 * M5 * N5 * K5
    tc8 = 2.0 * peaks["bf16_tflops"]
    sms = torch.cuda.get_device_properties(dev).multi_processor_count

    def check(out):
        """Bit-exact columns of this rank on sampled rows; placement of every
        rank's block in this rank's output (per-row checksums over NCCL)."""
        ok = True
        if ncols > 0:
            got = out[rows.tolist(), n0:n1].view(torch.int16).cpu().numpy().view(np.uint16)
            ok = bool((got == want).all())
        placed = True
        if dist:
            mine = torch.zeros((M5, ns), dtype=torch.float32, device=dev)
            mine[:, :ncols] = out[:, n0:n1].float()
            mine = mine.sum(dim=1)
            allsums = [torch.empty_like(mine) for _ in range(world)]
            dist.all_gather(allsums, mine)
            for q, (q0, q1) in enumerate(ranges):
                blk = torch.zeros((M5, ns), dtype=torch.float32, device=dev)
                blk[:, : q1 - q0] = out[:, q0:q1].float()
                placed &= bool(torch.equal(blk.sum(dim=1), allsums[q]))
            flags = torch.tensor([int(ok), int(placed)], device=dev)
            dist.all_reduce(flags, op=dist.ReduceOp.MIN)
            ok, placed = bool(flags[0].item()), bool(flags[1].item())
        return {"rows_checked": int(rows.size), "columns_per_rank": ncols,
                "bf16_bit_exact_sampled_rows": ok, "placement_checksum_ok": placed}

    def max_ranks(vals):
        if not dist:
            return vals
        t = torch.tensor(vals, device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.tolist()

    def timed_steps(sh, steps, clocks=None):
        """`steps` calls back to back between one event pair (inputs larger
        than L2), an event after every call and one after every GEMM: total
        and GEMM-part milliseconds per step, max over ranks."""
        if clocks:  # before the warm-up (no idle pause before the timed loop)
            clocks.start()
            time.sleep(0.3)
        if dist:
            dist.barrier()
        for _ in range(max(3, args.warmup)):
            sh(qx, sx, qw, sw)
        rb.sync_status()
        if dist:  # every rank enters the timed loop together
            dist.barrier()
        torch.cuda.synchronize()
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
        gd = [dict() for _ in range(steps)]
        evs[0].record()
        for i in range(steps):
            sh(qx, sx, qw, sw, events=gd[i])
            evs[i + 1].record()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        clk = clocks.stop() if clocks else None
        rb.sync_status()
        total = evs[0].elapsed_time(evs[steps]) / steps
        gemm = sum(evs[i].elapsed_time(gd[i]["gemm_done"]) for i in range(steps)) / steps
        total, gemm = max_ranks([total, gemm])
        return total, gemm, clk

    def summary(total, gemm):
        return {"total_ms": round(total, 4), "gemm_ms": round(gemm, 4),
                "tops": round(ops / (total * 1e-3) / 1e12, 1),
                "gemm_tops_per_gpu": round(2.0 * M5 * ns * K5 / (gemm * 1e-3) / 1e12, 1),
                "gemm_frac_per_gpu": round(2.0 * M5 * ns * K5 / (gemm * 1e-3) / 1e12 / tc8, 4)}

    # Roofline of the compute + collective step: the slower of the GEMM at
    # the measured tensor peak and the NVLink ingress every GPU must receive
    # ((g-1)/g of C) at the pool's measured 770 GB/s peer bandwidth.
    ingress = M5 * N5 * 2 * (world - 1) / world
    t_tensor = ops / world / (tc8 * 1e12)
    t_link = ingress / 770e9
    bound_ms = max(t_tensor, t_link) * 1e3

    # the product form: the library's choice of fused broadcast for `world`
    fused = FusedShardedW8A8(M5, N5, K5, rank, world, dev)
    steps = args.steps if not compact else max(3, min(args.steps, 10))
    clocks = ClockSampler(local_rank) if not compact and rank == 0 else None
    total, gemm, clk = timed_steps(fused, steps, clocks)
    out = fused(qx, sx, qw, sw)
    parity = check(out)
    value = ops / (total * 1e-3) / 1e12
    res = {"value": round(value, 2), "ms_per_step": round(total, 5), "parity": parity,
           "clocks": clk}
    prim = summary(total, gemm)
    prim["mode"] = fused.mode
    res["roofline"] = {
        "bound": "nvlink ingress" if t_link > t_tensor else "tensor",
        "kernel": "gemm_tc2_kernel<I8> with the all-gather fused into its epilogue "
                  f"({fused.mode}); one launch per step plus a device barrier",
        "achieved": round(value / world, 2), "peak": round(ops / world / (bound_ms * 1e-3) / 1e12, 2),
        "unit": "TOP/s per GPU", "frac": round(bound_ms / total, 4),
        "bound_ms": round(bound_ms, 4), "ingress_bytes_per_gpu": int(ingress),
        "traffic": None,
        "peak_source": "the slower of the GEMM at 2 x measured dense bf16 and the NVLink "
                       "ingress at the pool's measured 770 GB/s peer bandwidth"}
    if compact:
        res.update(prim)
        res["frac_of_int8_peak"] = round(value / tc8, 4)
        fused.close()
        del fused, qx, qw, out
        torch.cuda.synchronize()
        return res

    # e2e: every step copies the int8 activations (and scales) in from pinned
    # host memory and a band of 1/world of C's rows (all N columns, so every
    # rank's block is read on some rank) back to the host.
    r0, r1 = rank * M5 // world, (rank + 1) * M5 // world
    qx_h = qx.cpu().pin_memory()
    sx_h = sx.cpu().pin_memory()
    c_h = torch.empty((r1 - r0, N5), dtype=torch.bfloat16).pin_memory()
    cur = torch.cuda.current_stream(dev)

    def e2e_once():
        qx.copy_(qx_h, non_blocking=True)
        sx.copy_(sx_h, non_blocking=True)
        o = fused(qx, sx, qw, sw)
        c_h.copy_(o[r0:r1], non_blocking=True)
        cur.synchronize()

    for _ in range(2):
        e2e_once()
    if dist:
        dist.barrier()
    reps = max(3, min(args.steps, 10))
    t0 = time.perf_counter()
    for _ in range(reps):
        e2e_once()
    dt = max_ranks([(time.perf_counter() - t0) / reps])[0]
    e2e_ok = bool(torch.equal(c_h.to(dev), out[r0:r1]))
    if dist:
        f = torch.tensor([int(e2e_ok)], device=dev)
        dist.all_reduce(f, op=dist.ReduceOp.MIN)
        e2e_ok = bool(f.item())
    res["e2e"] = {"value": round(ops / dt / 1e12, 3), "unit": "TOP/s",
                  "h2d_bytes_per_step": M5 * K5 + M5 * 4,
                  "d2h_bytes_per_step": (r1 - r0) * N5 * 2,
                  "ms_per_step": round(dt * 1e3, 3), "copied_band_matches_device": e2e_ok,
                  "path": "FusedShardedW8A8 (rouge_b200_gemm_i8_bcast + device barrier); "
                          "pinned host int8 activations in, a 1/N row band of C out, per rank"}
    fused.close()
    del fused, out
    torch.cuda.synchronize()
    if dist:
        dist.barrier()

    detail = {"fused": prim, "roofline_note": "frac = bound_ms / total_ms"}
    # the other fused form (TMA stores to every peer vs multicast stores)
    alt = FusedShardedW8A8(M5, N5, K5, rank, world, dev,
                           use_multicast=not FusedShardedW8A8.default_multicast(world))
    if alt.mode != prim["mode"]:
        t_a, g_a, _ = timed_steps(alt, max(3, min(args.steps, 10)))
        r = summary(t_a, g_a)
        r["mode"] = alt.mode
        r["parity"] = check(alt(qx, sx, qw, sw))
        detail["fused_alt"] = r
    alt.close()
    del alt
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    # the NCCL baseline: bands of 2048 rows, each all-gathered on a
    # communication stream while the next band computes (GEMM on SMs - 8)
    prev = rb.lib().rouge_b200_set_sm_budget(max(0, sms - 8))
    try:
        sh = ShardedW8A8(M5, N5, K5, rank, world, dev, R=2048)
        t_n, g_n, _ = timed_steps(sh, max(3, min(args.steps, 10)))
        r = summary(t_n, g_n)
        r["mode"] = "nccl all-gather per 2048-row band + unshard"
        r["nvlink_gbs_per_gpu"] = round(ingress / max(t_n - g_n, 1e-6) / 1e6, 1)
        r["parity"] = check(sh(qx, sx, qw, sw))
        detail["nccl"] = r
        del sh
    finally:
        rb.lib().rouge_b200_set_sm_budget(prev)
    res["detail"] = detail
    return res


# ------------------------------------------------------------------ configs 1, 3, 4

def time_launch(torch, fn, flush, reps=20):
    """Mean device time (ms) of one launch of fn, L2 flushed before each
    launch, CUDA events on the launching stream. fn is launched directly
    (not from a graph) right after the ~80 us flush, so the host-side launch
    path overlaps the flush and no graph-launch latency enters the interval;
    the mean over `reps` launches smooths the event timer's microsecond
    granularity."""
    for _ in range(3):
        l2_flush(flush)
        fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        l2_flush(flush)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1))
    return sum(ts) / len(ts)


def other_configs(rb, torch, dev, peaks, peak_src, flush):
    """Kernel-level numbers for BASELINE configs 1, 3 and 4 (one GPU), each
    checked against the oracle on a sample so a wrong kernel cannot report."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    orc = O.Oracle()
    out = {}
    tc16 = peaks["bf16_tflops"]
    tc8 = 2.0 * peaks["bf16_tflops"]
    hbm = peaks["hbm_gbs"]

    # config 1: fp16 GEMM 512^3, A row-major, B column-major, f32 out
    n1 = 512
    a = orc.f16_encode(rb.synth_uniform(0, (n1, n1), -1.0, 1.0))
    b = orc.f16_encode(rb.synth_uniform(10, (n1, n1), -1.0, 1.0))   # B[N][K] (column-major B)
    ad = torch.from_numpy(a.view(np.int16)).to(dev)
    bd = torch.from_numpy(b.view(np.int16)).to(dev)
    c1 = torch.empty((n1, n1), dtype=torch.float32, device=dev)
    t = time_launch(torch, lambda: rb.gemm_f16(ad, bd, rb.B_NK, c1, rb.OUT_F32), flush)
    want = orc.gemm_f32(orc.f16_decode(a), orc.f16_decode(b), True)
    err = float(np.linalg.norm(c1.cpu().numpy() - want) / np.linalg.norm(want))
    fl = 2.0 * n1 ** 3
    # torch's cuBLAS on the same operands, timed the same way (context only)
    ah16, bh16 = ad.view(torch.float16), bd.view(torch.float16)
    t_torch = time_launch(torch, lambda: torch.matmul(ah16, bh16.t()), flush)
    out["config1_f16_gemm_512"] = {
        "ms": round(t, 5), "tflops": round(fl / (t * 1e-3) / 1e12, 2),
        "frac_of_bf16_peak": round(fl / (t * 1e-3) / 1e12 / tc16, 4), "rel_l2_vs_oracle": err,
        "torch_matmul_ms": round(t_torch, 5),
        "note": "64 output tiles of 128 x 32 for 148 SMs: latency-bound by construction"}

    # config 3: fp8 e4m3 path, A, B [8192][8192] f32 ~ N(0,1); B in the
    # reference layout [K][N]; per-tensor absmax scale; GEMM -> bf16
    n3 = 8192
    A = torch.from_numpy(rb.synth_normal(3, (n3, n3), 0.0, 1.0)).to(dev)
    B = torch.from_numpy(rb.synth_normal(4, (n3, n3), 0.0, 1.0)).to(dev)
    qa = torch.empty((n3, n3), dtype=torch.uint8, device=dev)
    qb = torch.empty((n3, n3), dtype=torch.uint8, device=dev)
    sc = torch.zeros(4, dtype=torch.float32, device=dev)  # amaxA, sA, amaxB, sB
    c3 = torch.empty((n3, n3), dtype=torch.int16, device=dev)
    t_cvt = time_launch(torch, lambda: rb.quantize_e4m3_tensor(A, sc[0:1], sc[1:2], qa), flush)
    rb.quantize_e4m3_tensor(B, sc[2:3], sc[3:4], qb)
    t_g = time_launch(torch, lambda: rb.gemm_e4m3(qa, qb, rb.B_KN, c3, rb.OUT_BF16, sc[1:2], sc[3:4]),
                     flush)
    rb.sync_status()
    rows = np.array([0, 1, 4095, 8191], np.int32)
    a_rows = A[rows.tolist()].cpu().numpy()
    amax_a = float(sc[0].item())
    codes_ok = bool((qa[rows.tolist()].cpu().numpy() ==
                     orc.e4m3_encode(a_rows / np.float32(sc[1].item()))).all()
                    and amax_a == float(A.abs().max().item()))
    qb_h = qb.cpu().numpy()
    want = orc.gemm_f32(orc.e4m3_decode(qa[rows.tolist()].cpu().numpy()), orc.e4m3_decode(qb_h),
                        False) * np.float32(np.float32(sc[1].item()) * np.float32(sc[3].item()))
    got = orc.bf16_decode(c3[rows.tolist()].cpu().numpy().view(np.uint16))
    err = float(np.linalg.norm(got - want) / np.linalg.norm(want))
    fl = 2.0 * n3 ** 3
    cvt_bytes = n3 * n3 * 9 + 4
    out["config3_fp8_8192"] = {
        "gemm_ms": round(t_g, 4), "gemm_tflops": round(fl / (t_g * 1e-3) / 1e12, 1),
        "gemm_frac": round(fl / (t_g * 1e-3) / 1e12 / tc8, 4),
        "convert_ms": round(t_cvt, 4),
        "convert_gbs": round(cvt_bytes / (t_cvt * 1e-3) / 1e9, 1),
        "convert_hbm_frac": round(cvt_bytes / (t_cvt * 1e-3) / 1e9 / hbm, 4),
        "b_layout": "[K][N] (reference layout, MN-major operand)",
        "codes_bit_exact_sampled_rows": codes_ok, "rel_l2_sampled_rows": err,
        "peak": f"gemm vs 2 x {peak_src} bf16; convert vs {peak_src} HBM {hbm} GB/s "
                "(9 B/element: absmax read, encode read, code write)"}
    del A, B, qa, qb, c3

    # config 4: conv NHWC f16, N=32, 56x56, 256 -> 256, 3x3 s1 p1, + bias
    Nn, H, W_, Ci, Co = 32, 56, 56, 256, 256
    x = orc.f16_encode(rb.synth_uniform(5, (Nn, H, W_, Ci), -1.0, 1.0))
    w = orc.f16_encode(rb.synth_normal(6, (Co, 3, 3, Ci), 0.0, float(np.sqrt(2.0 / 2304.0))))
    bias = rb.synth_normal(7, (Co,), 0.0, 1.0)
    xd = torch.from_numpy(x.view(np.int16)).to(dev)
    wd = torch.from_numpy(w.view(np.int16)).to(dev)
    bd2 = torch.from_numpy(bias).to(dev)
    y = torch.empty((Nn, H, W_, Co), dtype=torch.float32, device=dev)
    t = time_launch(torch, lambda: rb.conv2d_nhwc_f16(xd, wd, bd2, y, 1, 1), flush)
    rb.sync_status()
    want = orc.conv2d_nhwc(orc.f16_decode(x), orc.f16_decode(w), bias, 1, 1, 0, 256)
    err = float(np.linalg.norm(y.cpu().numpy().reshape(-1, Co)[:256] - want) / np.linalg.norm(want))
    fl = 2.0 * Nn * H * W_ * Co * 9 * Ci
    out["config4_conv_nhwc_f16"] = {
        "ms": round(t, 4), "tflops": round(fl / (t * 1e-3) / 1e12, 1),
        "frac_of_bf16_peak": round(fl / (t * 1e-3) / 1e12 / tc16, 4),
        "rel_l2_first_256_pixels": err,
        "kernel": "gemm_tc2_kernel<F16, conv> (2-CTA pairs, im2col TMA A, fused bias)"}
    del xd, wd, y

    # cuBLAS-API shim: cublasSgemm_v2 (f32, 3xTF32 on tcgen05) at 8192^3,
    # against torch's own f32 matmul (cuBLAS SGEMM, TF32 off) on the same data
    import ctypes as C_
    shim = C_.CDLL(os.path.join(ROOT, "rouge-v_b200", "lib", "librouge_b200_cublas.so"))
    h = C_.c_void_p()
    if shim.cublasCreate_v2(C_.byref(h)) == 0:
        shim.cublasSetStream_v2(h, C_.c_void_p(torch.cuda.current_stream().cuda_stream))
        ns = 8192
        As = torch.randn((ns, ns), device=dev)
        Bs = torch.randn((ns, ns), device=dev)
        Cs = torch.empty((ns, ns), device=dev)
        one, zero = C_.c_float(1.0), C_.c_float(0.0)

        def sgemm():
            st = shim.cublasSgemm_v2(h, 0, 0, ns, ns, ns, C_.byref(one), C_.c_void_p(As.data_ptr()),
                                     ns, C_.c_void_p(Bs.data_ptr()), ns, C_.byref(zero),
                                     C_.c_void_p(Cs.data_ptr()), ns)
            assert st == 0, st
        t_s = time_launch(torch, sgemm, flush)
        prev_tf32 = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = False
        Ct = torch.empty_like(Cs)
        t_t = time_launch(torch, lambda: torch.matmul(Bs, As, out=Ct), flush)  # same column-major product
        torch.backends.cuda.matmul.allow_tf32 = prev_tf32
        rows = torch.arange(0, ns, 1024, device=dev)
        ref = (Bs[rows].double() @ As.double())          # rows of the row-major view = columns of C
        err = float((Cs[rows].double() - ref).norm() / ref.norm())
        fl = 2.0 * ns ** 3
        out["cublas_shim_sgemm_8192"] = {
            "ms": round(t_s, 4), "tflops": round(fl / (t_s * 1e-3) / 1e12, 1),
            "torch_f32_matmul_ms": round(t_t, 4),
            "torch_f32_matmul_tflops": round(fl / (t_t * 1e-3) / 1e12, 1),
            "rel_l2_sampled_columns_vs_f64": err,
            "kernel": "pack (hi/lo split) + gemm_tc2_kernel<TF32> over 3K (3xTF32)"}
        del As, Bs, Cs, Ct
        shim.cublasDestroy_v2(h)

    # MX formats: MXFP8 block quantization of 8192^2
    # f32 (e4m3 codes + E8M0 scale per 32) and the block-scaled tcgen05 GEMM
    # 8192^3 on those codes, checked against the oracle (exact decode, f64
    # sums) on sampled rows.
    nm = 8192
    xa = torch.from_numpy(rb.synth_normal(11, (nm, nm), 0.0, 1.0)).to(dev)
    xb = torch.from_numpy(rb.synth_normal(12, (nm, nm), 0.0, 1.0)).to(dev)
    qa = torch.empty((nm, nm), dtype=torch.uint8, device=dev)
    qb = torch.empty((nm, nm), dtype=torch.uint8, device=dev)
    sa = torch.empty((nm, nm // 32), dtype=torch.uint8, device=dev)
    sb = torch.empty((nm, nm // 32), dtype=torch.uint8, device=dev)
    t_q = time_launch(torch, lambda: rb.mx_quantize(xa, rb.FMT_E4M3, qa, sa), flush)
    rb.mx_quantize(xb, rb.FMT_E4M3, qb, sb)
    ta = torch.empty(rb.mx_scale_atoms_bytes(nm, nm), dtype=torch.uint8, device=dev)
    tb = torch.empty_like(ta)
    t_atoms = time_launch(torch, lambda: rb.mx_scale_atoms(sa, nm, nm, ta), flush)
    rb.mx_scale_atoms(sb, nm, nm, tb)
    cm = torch.empty((nm, nm), dtype=torch.bfloat16, device=dev)
    t_g = time_launch(torch, lambda: rb.gemm_mx(qa, rb.FMT_E4M3, ta, qb, rb.FMT_E4M3, tb, cm,
                                                rb.OUT_BF16), flush)
    rb.sync_status()
    rows = [0, 1, 4095, 8191]
    xs = xa[rows].cpu().numpy()
    wq, ws = orc.mx_quantize(xs, "e4m3")
    codes_ok = bool((qa[rows].cpu().numpy().ravel() == wq).all()
                    and (sa[rows].cpu().numpy().ravel() == ws).all())
    A = orc.mx_dequantize(qa[rows].cpu().numpy(), sa[rows].cpu().numpy(), "e4m3").reshape(4, nm)
    B = orc.mx_dequantize(qb.cpu().numpy(), sb.cpu().numpy(), "e4m3").reshape(nm, nm)
    want = A.astype(np.float64) @ B.T.astype(np.float64)
    got = cm[rows].float().cpu().numpy()
    err = float(np.linalg.norm(got - want) / np.linalg.norm(want))
    fl = 2.0 * nm ** 3
    qbytes = nm * nm * (4 + 1) + nm * nm // 32
    out["mxfp8_8192"] = {
        "quantize_ms": round(t_q, 4), "quantize_gbs": round(qbytes / (t_q * 1e-3) / 1e9, 1),
        "quantize_hbm_frac": round(qbytes / (t_q * 1e-3) / 1e9 / hbm, 4),
        "scale_atoms_ms": round(t_atoms, 4),
        "gemm_ms": round(t_g, 4), "gemm_tflops": round(fl / (t_g * 1e-3) / 1e12, 1),
        "gemm_frac": round(fl / (t_g * 1e-3) / 1e12 / tc8, 4),
        "codes_and_scales_bit_exact_sampled_rows": codes_ok, "rel_l2_sampled_rows": err,
        "kernels": "mx_quant_kernel<e4m3>; gemm_tc2_kernel<MXF8> (kind::mxf8f6f4.block_scale, "
                   "256x256 CTA-pair tiles, overlapping TMEM accumulators)",
        "peak": f"gemm vs 2 x {peak_src} bf16; quantize vs {peak_src} HBM "
                "(5 B/element + 1/32 B scale)"}
    del qa, qb, sa, sb, ta, tb

    # NVFP4: block quantization (e2m1 + UE4M3 scale per 16, global scale 1),
    # packing two codes per byte, and the block-scaled fp4 GEMM 8192^3
    qa = torch.empty((nm, nm), dtype=torch.uint8, device=dev)
    qb = torch.empty((nm, nm), dtype=torch.uint8, device=dev)
    sa = torch.empty((nm, nm // 16), dtype=torch.uint8, device=dev)
    sb = torch.empty((nm, nm // 16), dtype=torch.uint8, device=dev)
    t_q = time_launch(torch, lambda: rb.nvfp4_quantize(xa, 1.0, qa, sa), flush)
    rb.nvfp4_quantize(xb, 1.0, qb, sb)
    pa = torch.empty((nm, nm // 2), dtype=torch.uint8, device=dev)
    pb = torch.empty((nm, nm // 2), dtype=torch.uint8, device=dev)
    rb.fp4_pack(qa, pa)
    rb.fp4_pack(qb, pb)
    ta = torch.empty(rb.nvfp4_scale_atoms_bytes(nm, nm), dtype=torch.uint8, device=dev)
    tb = torch.empty_like(ta)
    rb.nvfp4_scale_atoms(sa, nm, nm, ta)
    rb.nvfp4_scale_atoms(sb, nm, nm, tb)
    g1 = torch.ones(1, device=dev)
    t_g = time_launch(torch, lambda: rb.gemm_nvfp4(pa, ta, g1, pb, tb, g1, cm, rb.OUT_BF16), flush)
    rb.sync_status()
    wq, ws = orc.nvfp4_quantize(xs, 1.0)
    codes_ok = bool((qa[rows].cpu().numpy().ravel() == wq).all()
                    and (sa[rows].cpu().numpy().ravel() == ws).all())

    def dec(q, s_, r):
        v = orc.narrow_decode(q.ravel(), "e2m1").astype(np.float64).reshape(r, nm // 16, 16)
        return (v * orc.narrow_decode(s_.ravel(), "e4m3").astype(np.float64).reshape(r, -1, 1)).reshape(r, nm)
    A = dec(qa[rows].cpu().numpy(), sa[rows].cpu().numpy(), 4)
    B = dec(qb.cpu().numpy(), sb.cpu().numpy(), nm)
    want = A @ B.T
    got = cm[rows].float().cpu().numpy()
    err = float(np.linalg.norm(got - want) / np.linalg.norm(want))
    qbytes = nm * nm * (4 + 1) + nm * nm // 16
    tc4 = 4.0 * peaks["bf16_tflops"]
    out["nvfp4_8192"] = {
        "quantize_ms": round(t_q, 4), "quantize_gbs": round(qbytes / (t_q * 1e-3) / 1e9, 1),
        "quantize_hbm_frac": round(qbytes / (t_q * 1e-3) / 1e9 / hbm, 4),
        "gemm_ms": round(t_g, 4), "gemm_tflops": round(fl / (t_g * 1e-3) / 1e12, 1),
        "gemm_frac": round(fl / (t_g * 1e-3) / 1e12 / tc4, 4),
        "codes_and_scales_bit_exact_sampled_rows": codes_ok, "rel_l2_sampled_rows": err,
        "kernels": "nvfp4_quant_kernel; gemm_tc2_kernel<NVF4> (kind::mxf4nvf4.block_scale."
                   "scale_vec::4X, 256x256 CTA-pair tiles, packed e2m1)",
        "peak": f"gemm vs 4 x {peak_src} bf16 (dense fp4 is four times bf16); quantize vs "
                f"{peak_src} HBM (5 B/element + 1/16 B scale)"}
    del qa, qb, sa, sb, pa, pb, ta, tb

    # MXFP4: MX block quantization to e2m1 (E8M0 scale per 32), packing, and
    # the block-scaled fp4 GEMM 8192^3 (kind::mxf4.block_scale)
    qa = torch.empty((nm, nm), dtype=torch.uint8, device=dev)
    qb = torch.empty((nm, nm), dtype=torch.uint8, device=dev)
    sa = torch.empty((nm, nm // 32), dtype=torch.uint8, device=dev)
    sb = torch.empty((nm, nm // 32), dtype=torch.uint8, device=dev)
    t_q = time_launch(torch, lambda: rb.mx_quantize(xa, rb.FMT_E2M1, qa, sa), flush)
    rb.mx_quantize(xb, rb.FMT_E2M1, qb, sb)
    pa = torch.empty((nm, nm // 2), dtype=torch.uint8, device=dev)
    pb = torch.empty((nm, nm // 2), dtype=torch.uint8, device=dev)
    rb.fp4_pack(qa, pa)
    rb.fp4_pack(qb, pb)
    ta = torch.empty(rb.mxfp4_scale_atoms_bytes(nm, nm), dtype=torch.uint8, device=dev)
    tb = torch.empty_like(ta)
    rb.mxfp4_scale_atoms(sa, nm, nm, ta)
    rb.mxfp4_scale_atoms(sb, nm, nm, tb)
    t_g = time_launch(torch, lambda: rb.gemm_mxfp4(pa, ta, pb, tb, cm, rb.OUT_BF16), flush)
    rb.sync_status()
    wq, ws = orc.mx_quantize(xs, "e2m1")
    codes_ok = bool((qa[rows].cpu().numpy().ravel() == wq).all()
                    and (sa[rows].cpu().numpy().ravel() == ws).all())
    A = orc.mx_dequantize(qa[rows].cpu().numpy(), sa[rows].cpu().numpy(), "e2m1").reshape(
        4, nm).astype(np.float64)
    B = orc.mx_dequantize(qb.cpu().numpy(), sb.cpu().numpy(), "e2m1").reshape(nm, nm).astype(np.float64)
    want = A @ B.T
    got = cm[rows].float().cpu().numpy()
    err = float(np.linalg.norm(got - want) / np.linalg.norm(want))
    qbytes = nm * nm * (4 + 1) + nm * nm // 32
    out["mxfp4_8192"] = {
        "quantize_ms": round(t_q, 4), "quantize_gbs": round(qbytes / (t_q * 1e-3) / 1e9, 1),
        "quantize_hbm_frac": round(qbytes / (t_q * 1e-3) / 1e9 / hbm, 4),
        "gemm_ms": round(t_g, 4), "gemm_tflops": round(fl / (t_g * 1e-3) / 1e12, 1),
        "gemm_frac": round(fl / (t_g * 1e-3) / 1e12 / tc4, 4),
        "codes_and_scales_bit_exact_sampled_rows": codes_ok, "rel_l2_sampled_rows": err,
        "kernels": "mx_quant_blocks_kernel<e2m1>; gemm_tc2_kernel<MXF4> (kind::mxf4.block_scale."
                   "scale_vec::2X, 256x256 CTA-pair tiles, packed e2m1)",
        "peak": f"gemm vs 4 x {peak_src} bf16 (dense fp4 is four times bf16); quantize vs "
                f"{peak_src} HBM (5 B/element + 1/32 B scale)"}
    del xa, xb, qa, qb, sa, sb, pa, pb, ta, tb, cm

    # Rank-4 consumers at the reference benchmark's shapes (bench_ai.cpp:73-126):
    # causal GQA attention S=512, Dh=64, Hq=8, Hkv=2, and the transformer block
    # S=256, D=512, Hq=8, Hkv=2, Dq=64, Dff=1376; device time of the device
    # entries (inputs resident) beside one call of the reference's CPU code.
    S_, Dh_, Hq_, Hkv_ = 512, 64, 8, 2
    Qa = torch.randn((Hq_, S_, Dh_), device=dev)
    Ka = torch.randn((Hkv_, S_, Dh_), device=dev)
    Va = torch.randn((Hkv_, S_, Dh_), device=dev)
    Oa = torch.empty_like(Qa)
    wsa = torch.empty(rb.attention_workspace(S_, S_, Dh_, Hq_, Hkv_), dtype=torch.uint8, device=dev)
    t_att = time_launch(torch, lambda: rb.attention_gqa(Qa, Ka, Va, Oa, workspace=wsa), flush)
    Sx, Dx, Dqx, Dffx = 256, 512, 64, 1376
    g_ = torch.Generator(device=dev).manual_seed(9)
    mk = lambda *sh: torch.randn(sh, device=dev, generator=g_) * 0.05  # noqa: E731
    xb_ = torch.randn((Sx, Dx), device=dev, generator=g_)
    w1_ = torch.ones(Dx, device=dev)
    wts = [mk(Dx, Hq_ * Dqx), mk(Dx, Hkv_ * Dqx), mk(Dx, Hkv_ * Dqx), mk(Hq_ * Dqx, Dx)]
    mlp = [mk(Dx, Dffx), mk(Dx, Dffx), mk(Dffx, Dx)]
    ob_ = torch.empty_like(xb_)
    wsb = torch.empty(rb.transformer_block_workspace(Sx, Dx, Hq_, Hkv_, Dqx, Dffx), dtype=torch.uint8,
                      device=dev)
    t_blk = time_launch(torch, lambda: rb.transformer_block(xb_, w1_, *wts, w1_, *mlp, Hq_, Hkv_, Dqx,
                                                            ob_, workspace=wsb), flush)
    rb.sync_status()
    ops_att = 2.0 * S_ * S_ * Dh_ * Hq_
    ops_blk = (2.0 * Sx * Dx * (Hq_ * Dqx + 2 * Hkv_ * Dqx + Dx) + 2.0 * Sx * Dx * 3 * Dffx
               + 2.0 * Sx * Sx * Dqx * Hq_)
    cons = {"attention_gqa_ms": round(t_att, 4),
            "attention_gqa_gflops": round(ops_att / (t_att * 1e-3) / 1e9, 1),
            "transformer_block_ms": round(t_blk, 4),
            "transformer_block_gflops": round(ops_blk / (t_blk * 1e-3) / 1e9, 1),
            "flops_counted_as": "bench_ai.cpp:88,118-120 (the reference benchmark's own counts)"}
    refp = os.path.join(ROOT, "oracle", "_ref", "librouge_ref_shims.so")
    if os.path.exists(refp):
        import ctypes as C_
        R = C_.CDLL(refp)
        P_ = C_.c_void_p
        R.rouge_attention_gqa.argtypes = [C_.c_int] * 5 + [P_] * 4 + [C_.c_float] + [C_.c_int] * 3
        q_, k_, v_ = (t.cpu().numpy() for t in (Qa, Ka, Va))
        o_ = np.empty_like(q_)
        t0 = time.perf_counter()
        R.rouge_attention_gqa(S_, S_, Dh_, Hq_, Hkv_, *(P_(a.ctypes.data) for a in (q_, k_, v_, o_)),
                              0.0, 1, 0, 0)
        cons["reference_cpu_attention_gqa_ms"] = round((time.perf_counter() - t0) * 1e3, 2)
        cons["attention_max_abs_diff_vs_reference"] = float(np.abs(o_ - Oa.cpu().numpy()).max())
        R.rouge_transformer_block.argtypes = [C_.c_int] * 6 + [P_] * 10 + [C_.c_int, C_.c_float,
                                                                          C_.c_float, P_]
        host = [t.cpu().numpy() for t in [xb_, w1_] + wts + [w1_] + mlp]
        ro = np.empty((Sx, Dx), np.float32)
        t0 = time.perf_counter()
        R.rouge_transformer_block(Sx, Dx, Hq_, Hkv_, Dqx, Dqx, *(P_(a.ctypes.data) for a in host),
                                  Dffx, 10000.0, 1e-5, P_(ro.ctypes.data))
        cons["reference_cpu_transformer_block_ms"] = round((time.perf_counter() - t0) * 1e3, 2)
        cons["block_max_abs_diff_vs_reference"] = float(np.abs(ro - ob_.cpu().numpy()).max())
    out["consumers"] = cons
    del Qa, Ka, Va, Oa, wsa, xb_, wts, mlp, ob_, wsb

    # The reference's own CPU code for the rows past the hot path, timed on
    # bounded samples on this host (one call each), beside the numbers above
    out["reference_cpu_samples"] = reference_cpu_samples()

    # cuDNN-API library: cudnnConvolutionForward at the config-4 shape
    # (N=32, 56x56, 256 -> 256, 3x3 s1 p1), HALF + NHWC (direct: no
    # workspace, alpha / beta in the epilogue, f16 out) and FLOAT + NCHW
    # (3xTF32), each against torch's conv2d (cuDNN) on the same tensors:
    # channels-last f16, and f32 with TF32 off.
    dnn = C_.CDLL(os.path.join(ROOT, "rouge-v_b200", "lib", "librouge_b200_cudnn.so"))
    hd = C_.c_void_p()
    if dnn.cudnnCreate(C_.byref(hd)) == 0:
        dnn.cudnnSetStream(hd, C_.c_void_p(torch.cuda.current_stream().cuda_stream))
        F = torch.nn.functional

        def desc(kind, *vals):
            d = C_.c_void_p()
            assert getattr(dnn, f"cudnnCreate{kind}Descriptor")(C_.byref(d)) == 0
            setter = {"Tensor": dnn.cudnnSetTensor4dDescriptor, "Filter": dnn.cudnnSetFilter4dDescriptor,
                      "Convolution": dnn.cudnnSetConvolution2dDescriptor}[kind]
            assert setter(d, *[C_.c_int(v) for v in vals]) == 0
            return d

        cdsc = desc("Convolution", 1, 1, 1, 1, 1, 1, 0, 0)
        fl = 2.0 * Nn * H * W_ * Co * 9 * Ci
        for name, dtype, fmt in (("cudnn_shim_conv_nhwc_f16", 2, 1), ("cudnn_shim_conv_nchw_f32", 0, 0)):
            tdt = torch.float16 if dtype == 2 else torch.float32
            xt = torch.randn((Nn, Ci, H, W_), device=dev).to(tdt)
            wt = (torch.randn((Co, Ci, 3, 3), device=dev) * 0.03).to(tdt)
            if fmt == 1:
                xt = xt.contiguous(memory_format=torch.channels_last)
                wt = wt.contiguous(memory_format=torch.channels_last)
            yt = torch.zeros((Nn, Co, H, W_), device=dev, dtype=tdt)
            if fmt == 1:
                yt = yt.contiguous(memory_format=torch.channels_last)
            xdsc = desc("Tensor", fmt, dtype, Nn, Ci, H, W_)
            ydsc = desc("Tensor", fmt, dtype, Nn, Co, H, W_)
            wdsc = desc("Filter", dtype, fmt, Co, Ci, 3, 3)
            ws_n = C_.c_size_t(0)
            assert dnn.cudnnGetConvolutionForwardWorkspaceSize(hd, xdsc, wdsc, cdsc, ydsc, 0,
                                                               C_.byref(ws_n)) == 0
            wsb = torch.empty(max(ws_n.value, 256), dtype=torch.uint8, device=dev)
            al, be = C_.c_float(1.0), C_.c_float(0.0)

            def fwd():
                st = dnn.cudnnConvolutionForward(
                    hd, C_.byref(al), xdsc, C_.c_void_p(xt.data_ptr()), wdsc,
                    C_.c_void_p(wt.data_ptr()), cdsc, 0, C_.c_void_p(wsb.data_ptr()),
                    C_.c_size_t(ws_n.value), C_.byref(be), ydsc, C_.c_void_p(yt.data_ptr()))
                assert st == 0, st
            t_d = time_launch(torch, fwd, flush)
            prev = torch.backends.cudnn.allow_tf32
            torch.backends.cudnn.allow_tf32 = False
            torch.backends.cudnn.benchmark = True
            F.conv2d(xt, wt, padding=1)
            t_t = time_launch(torch, lambda: F.conv2d(xt, wt, padding=1), flush)
            want = F.conv2d(xt[:2].double(), wt.double(), padding=1)   # first two images
            torch.backends.cudnn.allow_tf32 = prev
            torch.backends.cudnn.benchmark = False
            err = float((yt[:2].double() - want).norm() / want.norm())
            out[name] = {
                "ms": round(t_d, 4), "tflops": round(fl / (t_d * 1e-3) / 1e12, 1),
                "workspace_bytes": ws_n.value,
                "torch_cudnn_conv2d_ms": round(t_t, 4),
                "torch_cudnn_conv2d_tflops": round(fl / (t_t * 1e-3) / 1e12, 1),
                "rel_l2_vs_f64_first_2_images": err,
                "kernel": ("gemm_tc2_kernel<F16, conv, f16 out> (direct, alpha/beta epilogue)"
                           if dtype == 2 else
                           "pack (NCHW -> NHWC hi/lo split) + gemm_tc2_kernel<TF32, conv> + NCHW finish")}
            del xt, wt, yt, wsb, want
        dnn.cudnnDestroy(hd)
    return out


def reference_cpu_samples():
    """One call of the reference library's cuBLAS shim SGEMM, cuDNN shim
    convolution, MX / NVFP4 quantizers and dequantize-then-GEMM on bounded
    samples (oracle/_ref, compiled from the reference's sources)."""
    import ctypes as C_
    refp = os.path.join(ROOT, "oracle", "_ref", "librouge_ref_shims.so")
    if not os.path.exists(refp):
        return {"unavailable": "oracle/_ref/librouge_ref_shims.so not built"}
    R = C_.CDLL(refp)
    P_, I_, F_ = C_.c_void_p, C_.c_int, C_.c_float
    ptr = lambda a: P_(a.ctypes.data)  # noqa: E731
    res = {"cores": os.cpu_count()}
    rng = np.random.default_rng(0)

    def timed(fn):
        t0 = time.perf_counter()
        fn()
        return time.perf_counter() - t0

    # cublasSgemm_v2 (cublas_shim.cpp:199-211) at 1024^3
    n = 1024
    a = rng.standard_normal((n, n)).astype(np.float32)
    b = rng.standard_normal((n, n)).astype(np.float32)
    c = np.zeros((n, n), np.float32)
    h = P_()
    R.cublasCreate_v2(C_.byref(h))
    one, zero = F_(1.0), F_(0.0)
    R.cublasSgemm_v2.argtypes = [P_, I_, I_, I_, I_, I_, P_, P_, I_, P_, I_, P_, P_, I_]
    t = timed(lambda: R.cublasSgemm_v2(h, 0, 0, n, n, n, C_.byref(one), ptr(a), n, ptr(b), n,
                                       C_.byref(zero), ptr(c), n))
    R.cublasDestroy_v2(h)
    res["cublas_sgemm_1024_gflops"] = round(2.0 * n ** 3 / t / 1e9, 2)
    # cudnnConvolutionForward FLOAT NCHW (cudnn_shim.cpp:188-232): the
    # config-4 convolution on 2 of its 32 images
    N, Ci, H, W, Co = 2, 256, 56, 56, 256
    x = rng.uniform(-1, 1, (N, Ci, H, W)).astype(np.float32)
    w = rng.uniform(-1, 1, (Co, Ci, 3, 3)).astype(np.float32) * 0.03
    y = np.zeros((N, Co, H, W), np.float32)
    R.rouge_conv2d_f32.argtypes = [I_] * 9 + [P_] * 5
    t = timed(lambda: R.rouge_conv2d_f32(N, Ci, H, W, Co, 3, 3, 1, 1, ptr(x), ptr(w), None, ptr(y),
                                         None))
    res["conv2d_f32_2x256x56x56_gflops"] = round(2.0 * N * H * W * Co * 9 * Ci / t / 1e9, 2)
    # MX / NVFP4 quantizers (narrow.cpp:200-300) on 16 M elements
    m = 16 << 20
    xs = rng.standard_normal(m).astype(np.float32)
    q = np.empty(m, np.uint8)
    sc = np.empty(m // 16, np.uint8)
    R.rouge_mx_quantize_f32.argtypes = [P_, I_, I_, P_, P_]
    R.rouge_nvfp4_quantize_f32.argtypes = [P_, I_, F_, P_, P_]
    t = timed(lambda: R.rouge_mx_quantize_f32(ptr(xs), m, 1, ptr(q), ptr(sc)))
    res["mxfp8_quantize_16M_gbs"] = round(m * 5 / t / 1e9, 3)
    t = timed(lambda: R.rouge_nvfp4_quantize_f32(ptr(xs), m, F_(1.0), ptr(q), ptr(sc)))
    res["nvfp4_quantize_16M_gbs"] = round(m * 5 / t / 1e9, 3)
    # the reference's route to a GEMM on MX data: dequantize, then its f32
    # GEMM (rouge_mx_dequantize_f32 + rouge_gemm_f32) at 1024^3
    R.rouge_mx_quantize_f32(ptr(a), n * n, 1, ptr(q), ptr(sc))
    R.rouge_mx_dequantize_f32.argtypes = [P_, P_, I_, I_, P_]
    R.rouge_gemm_f32.argtypes = [I_, I_, I_, P_, P_, P_, P_]
    deq = np.empty(n * n, np.float32)
    t = timed(lambda: (R.rouge_mx_dequantize_f32(ptr(q), ptr(sc), n * n, 1, ptr(deq)),
                       R.rouge_gemm_f32(n, n, n, ptr(deq), ptr(b), ptr(c), None)))
    res["mx_dequantize_plus_gemm_f32_1024_gflops"] = round(2.0 * n ** 3 / t / 1e9, 2)
    return res


def check_parity(rb, X, qx, sx, qw, sw, C):
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    orc = O.Oracle()
    rows = np.unique(np.concatenate([np.arange(0, M, M // 16), [M - 1, 127, 128]])).astype(np.int32)
    oq, os_ = orc.quantize_i8_rows(X[rows])
    gq = qx.cpu().numpy()
    gs = sx.cpu().numpy()
    codes_ok = bool((gq[rows] == oq).all() and (gs[rows] == os_).all())
    _, oc = orc.gemm_i8(gq, qw.cpu().numpy(), True, gs, 1, sw.cpu().numpy(), 1, rows=rows)
    out_ok = bool((C.cpu().numpy()[rows].view(np.uint32) == oc.view(np.uint32)).all())
    return {"rows_checked": int(rows.size), "codes_bit_exact": codes_ok, "f32_bit_exact": out_ok}


def run_e2e(args, rb, torch, Xh, qw, sw, dev, dist):
    """rouge_quantize_i8_channel(X) -> rouge_gemm_i8(Xq, Wq^T) on host buffers."""
    import ctypes as C_
    L = rb.lib()
    Wt = torch.from_numpy(np.ascontiguousarray(qw.cpu().numpy().T)).pin_memory()  # B[K][N]
    swh = sw.cpu().pin_memory()
    qxh = torch.empty((M, K), dtype=torch.int8).pin_memory()
    sxh = torch.empty(M, dtype=torch.float32).pin_memory()
    Ch = torch.empty((M, N), dtype=torch.float32).pin_memory()
    p = lambda t: C_.c_void_p(t.data_ptr())  # noqa: E731

    def once():
        ok = L.rouge_quantize_i8_channel(p(Xh), M, K, p(sxh), p(qxh))
        L.rouge_gemm_i8(M, N, K, p(qxh), p(Wt), p(sxh), 1, p(swh), 1, p(Ch))
        return ok == 1 and L.rouge_b200_last_error() == 0

    for _ in range(max(1, args.warmup)):
        assert once(), "drop-in path failed"
    if dist:
        dist.barrier()
    reps = max(3, min(args.steps, 10))
    t0 = time.perf_counter()
    for _ in range(reps):
        once()
    dt = (time.perf_counter() - t0) / reps
    if dist:
        t = torch.tensor([dt], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt = t.item()
    world = dist.get_world_size() if dist else 1
    h2d = M * K * 4 + M * K + K * N + M * 4 + N * 4
    d2h = M * K + M * 4 + M * N * 4
    return {"value": round(world * 2.0 * M * N * K / dt / 1e12, 3), "unit": "TOP/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": round(dt * 1e3, 3),
            "path": "rouge_quantize_i8_channel + rouge_gemm_i8 (host pointers, pinned)"}


# ------------------------------------------------------------------ CPU reference

def ref_lib():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    if not O.Reference.available():
        return None, "oracle/_ref/librouge_ref.so not built (reference sources absent at build)"
    return O.Reference(), None


def ref_rows(world, threads):
    """Rows of A per sampled step of the reference CPU path: the same sample
    for `cpu_baseline` and for the reference arm (about a second of work)."""
    return min(M, 64 * threads) if world == 1 else min(M5, 32 * threads)


def ref_inputs(R, world, threads):
    """The reference arm's inputs, made by the checker library's copy of the
    benchmark generator (bit-identical; the product library is not loaded):
    the sampled rows of A and the whole quantized weight matrix in the
    reference's B[K][N] layout."""
    rows = ref_rows(world, threads)
    if world == 1:
        X, W = make_inputs(R)
        qw, sw = R.quantize_i8_channel(W, threads=threads)
        return {"x": X[:rows], "wq_kn": np.ascontiguousarray(qw.T), "sw": sw, "rows": rows,
                "N": N, "K": K, "M": M}
    # config 5: the first rows of the activation stream (counter-based, so
    # they equal the first rows of the full matrix), quantized per token at
    # setup as on the GPU side, and all of W quantized per output channel
    x = R.synth_normal(8, (rows, K5), 0.0, 1.0)
    R.synth_outliers(8, x, 0.01, 20.0)
    qx, sx = R.quantize_i8_channel(x, threads=threads)
    W = R.synth_normal(9, (N5, K5), 0.0, 0.02)
    qw, sw = R.quantize_i8_channel(W, threads=threads)
    del W
    return {"qx": qx, "sx": sx, "wq_kn": np.ascontiguousarray(qw.T), "sw": sw, "rows": rows,
            "N": N5, "K": K5, "M": M5}


def ref_step(R, inp, threads):
    """One sampled step of the reference CPU path; returns seconds.
    Config 2: rouge_quantize_i8_channel of the rows + rouge_gemm_i8.
    Config 5: rouge_gemm_i8 of the int8 rows + rouge_quantize_bf16 of C."""
    t0 = time.perf_counter()
    if "x" in inp:
        q, s = R.quantize_i8_channel(inp["x"], threads=threads)
        R.gemm_i8(q, inp["wq_kn"], s, 1, inp["sw"], 1, threads=threads)
    else:
        c = R.gemm_i8(inp["qx"], inp["wq_kn"], inp["sx"], 1, inp["sw"], 1, threads=threads)
        R.bf16_encode(c, threads=threads)
    return time.perf_counter() - t0


def ref_sample_text(inp, threads):
    what = ("rouge_quantize_i8_channel + rouge_gemm_i8" if "x" in inp
            else "rouge_gemm_i8 + rouge_quantize_bf16")
    return (f"{inp['rows']} of {inp['M']} rows of A per step: {what} (row-sliced std::thread over "
            f"{threads} threads; N={inp['N']}, K={inp['K']})")


def cpu_baseline(X, W):
    """The reference library on this host's cores, on the same row sample as
    the reference arm (mean of three samples)."""
    R, why = ref_lib()
    if R is None:
        return {"value": None, "unavailable": why}
    threads = R.lib.ref_hw_threads()
    qw, sw = R.quantize_i8_channel(W, threads=threads)
    rows = ref_rows(1, threads)
    inp = {"x": X[:rows], "wq_kn": np.ascontiguousarray(qw.T), "sw": sw, "rows": rows,
           "N": N, "K": K, "M": M}
    ref_step(R, inp, threads)
    dt = sum(ref_step(R, inp, threads) for _ in range(3)) / 3
    return {"value": round(2.0 * rows * N * K / dt / 1e12, 5), "unit": "TOP/s", "cores": threads,
            "kind": "reference", "sample": ref_sample_text(inp, threads) + f", {dt:.3f} s"}


def run_reference(args, rank, world):
    """The reference CPU implementation (oracle/_ref, built from the
    reference sources) on this host's cores, rank 0 only. Its process loads
    only the checker libraries under oracle/."""
    if rank != 0:
        return None
    R, why = ref_lib()
    if R is None:
        return {"impl": "reference", "unavailable": why}
    threads = R.lib.ref_hw_threads()
    inp = ref_inputs(R, world, threads)
    for _ in range(max(1, min(args.warmup, 1))):
        ref_step(R, inp, threads)
    times = [ref_step(R, inp, threads) for _ in range(args.steps)]
    dt = sum(times) / len(times)
    rows, n_, k_, m_ = inp["rows"], inp["N"], inp["K"], inp["M"]
    value = 2.0 * rows * n_ * k_ / dt / 1e12
    return {
        "impl": "reference",
        "metric": METRIC,
        "value": round(value, 5), "unit": "TOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(dt * 1e3 * m_ / rows, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic (seeded splitmix64/Box-Muller, BASELINE config "
                f"{2 if world == 1 else 5} distributions)",
        "config": workload_config(world),
        "cpu_baseline": {"value": round(value, 5), "unit": "TOP/s", "cores": threads,
                         "kind": "reference",
                         "sample": ref_sample_text(inp, threads) +
                         " (ms_per_step extrapolated to all rows)"},
        "e2e": {"value": round(value, 5), "unit": "TOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


# ------------------------------------------------------------------ ncu drivers

def profile_kernel(name):
    """Runs one kernel of another configuration three times on cuda:0 and
    exits (the short command lines the ncu captures of those kernels use):
      conv4  rouge_b200_conv2d_nhwc_f16 on the config-4 shape
      mxfp8  MXFP8 quantization of a 4096^2 operand and gemm_mx 4096^3."""
    import torch
    import rouge_b200 as rb
    dev = torch.device("cuda", 0)
    if name == "conv4":
        n, h, w, ci, co = 32, 56, 56, 256, 256
        x = torch.randn((n, h, w, ci), device=dev).half()
        wt = (torch.randn((co, 3, 3, ci), device=dev) * 0.03).half()
        b = torch.zeros(co, device=dev)
        y = torch.empty((n, h, w, co), dtype=torch.float32, device=dev)
        for _ in range(3):
            rb.conv2d_nhwc_f16(x.view(torch.int16), wt.view(torch.int16), b, y, 1, 1)
    else:
        n = 4096
        x = torch.randn((n, n), device=dev)
        q = torch.empty((n, n), dtype=torch.uint8, device=dev)
        sc = torch.empty((n, n // 32), dtype=torch.uint8, device=dev)
        for _ in range(3):
            rb.mx_quantize(x, rb.FMT_E4M3, q, sc)
        at = torch.empty(rb.mx_scale_atoms_bytes(n, n), dtype=torch.uint8, device=dev)
        rb.mx_scale_atoms(sc, n, n, at)
        c = torch.empty((n, n), dtype=torch.float32, device=dev)
        for _ in range(3):
            rb.gemm_mx(q, rb.FMT_E4M3, at, q, rb.FMT_E4M3, at, c, rb.OUT_F32)
    torch.cuda.synchronize()
    rb.sync_status()
    print(json.dumps({"profile_kernel": name, "status": "ok"}), flush=True)


# ------------------------------------------------------------------ main

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--profile", action="store_true",
                    help="time the kernels only (no e2e / parity / CPU baseline), for ncu")
    ap.add_argument("--profile-kernel", default=None, choices=["conv4", "mxfp8"],
                    help="run only this kernel three times and exit (ncu captures)")
    args = ap.parse_args()
    if args.profile_kernel:
        profile_kernel(args.profile_kernel)
        return
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        line = run_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return

    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    line = run_ours(args, rank, world, local_rank)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
