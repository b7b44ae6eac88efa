#!/usr/bin/env python3
"""Benchmark of the H24 hot path on B200 (one JSON line on rank 0).

Workload (config 3 of the benchmark plan): a synthetic Pollux-1920 backbone,
18 layers x {QKV [5760,1920], O [1920,1920], up [7680,1920], down [1920,7680]}
bf16 N(0, 0.02^2) from seed 2: 72 matrices, 33,177,600 atoms of 24 values.
One step = whole-backbone pack-rule quantisation: per-row fp16 sigma, nearest
codeword (tcgen05 screening + rescore) and 18-bit pack of every matrix
(pack._quantize_h24_layer, pack.py:139-180, over pack_checkpoint's loop,
pack.py:268-283), in one shared pipeline, reading the bf16 weights as they are.
With N ranks (torchrun), rank r quantises rows shard_rows(rows, in, N, r) of
every matrix (strong scaling: the backbone is fixed, no collective on the
path); the optional NCCL all-gather of the packed shards is timed on its own.
value = backbone atoms quantised per second, whole job.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

--impl reference times the reference's algorithm on the host cores: the CPU
port in oracle/ of pack._quantize_h24_layer's fp32 matmul + argmax search, row
scale and 18-bit pack, each step a bounded sample of the same atoms.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

# Screening GEMM per atom: 4 rows (two position slices, x, |x|) against the
# 2048 Golay sign columns that stand for all 4096 (column c + 2048 is the
# complement of column c, and every row gives r(~c) = -r(c)), K = 24 (the
# tensor core runs K padded to 32).
SCREEN_FLOP_PER_ATOM = 4 * 2048 * 2 * 24
# An exhaustive search (x . kp_j for all 196,560 kissing points), for context.
EXHAUSTIVE_FLOP_PER_ATOM = 2 * 24 * 196_560
# Bytes the rescore must read per atom: its 24 coordinates (bf16), four 64-bit
# chunk masks, the 48-byte per-atom constants; and write: one int32 index.
RESCORE_BYTES_PER_ATOM_BF16 = 48 + 32 + 48 + 4
# The rescore is bound by instruction issue (ncu: 72 % issue active, warps
# mostly ready, DRAM at its floor), so its roofline is the SM issue rate:
# 4 warp instructions per cycle per SM.  Its count per atom is ncu's
# smsp__inst_executed.sum over one launch of 262,144 bf16 atoms (149.6 M,
# profiles/rescore_kernel_262k.md).
RESCORE_WARP_INST_PER_ATOM = 149.6e6 / 262_144
ISSUE_SLOTS_PER_SM = 4
# DRAM traffic per atom (dram__bytes_read.sum + dram__bytes_write.sum) of one
# captured launch of each kernel on 262,144 bf16 atoms, scaled to a launch of
# the bench's size by its atom count (the traffic of both kernels grows in
# proportion to the atoms): screen 79.9 + 3.2 MB, rescore 33.9 + 3.8 MB.
SCREEN_TRAFFIC_PER_ATOM = (79.9e6 + 3.2e6) / 262_144
RESCORE_TRAFFIC_PER_ATOM = (33.9e6 + 3.8e6) / 262_144
CONFIG = 3
METRIC = ("G atoms/s quantized (config-3 bf16 Pollux-1920 backbone: whole-backbone sigma16 + "
          "nearest codeword + 18-bit pack)")
WORKLOAD = ("config3: synthetic Pollux-1920 backbone, 18 layers x [5760x1920, 1920x1920, "
            "7680x1920, 1920x7680] bf16 N(0,0.02^2) seed 2 (33,177,600 atoms); rank r of N "
            "quantises rows shard_rows(rows, in, N, r) of every matrix; step = pack-rule sigma16 "
            "+ nearest codeword + 18-bit pack of those rows of all 72 matrices")


def _env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def _peaks() -> dict:
    try:
        with open(os.path.join(HERE, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except (OSError, ValueError):
        return {}


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    """SM clock, power and clock-event reasons of one GPU during the timed
    region, read-only: NVML polled every 5 ms from a thread (so that even a
    timed region of a few tens of ms has samples), else `nvidia-smi -lms 200`.
    The GPU is found by the UUID torch reports for the CUDA device."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.nvml = None
        self.samples = []  # (sm MHz, power W, reason bits)
        self.max_mhz = None

    def _nvml_handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        uuid = str(torch.cuda.get_device_properties(self.gpu).uuid)
        for cand in (uuid, "GPU-" + uuid):
            try:
                return pynvml, pynvml.nvmlDeviceGetHandleByUUID(cand)
            except pynvml.NVMLError:
                continue
        return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.gpu)

    def start(self):
        try:
            nv, h = self._nvml_handle()
            self.nvml = (nv, h)
            self.max_mhz = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            self.stop_flag = threading.Event()

            def poll():
                while not self.stop_flag.is_set():
                    try:
                        self.samples.append((nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM),
                                             nv.nvmlDeviceGetPowerUsage(h) / 1000.0,
                                             nv.nvmlDeviceGetCurrentClocksEventReasons(h)))
                    except nv.NVMLError:
                        pass
                    time.sleep(0.005)
            self.thread = threading.Thread(target=poll, daemon=True)
            self.thread.start()
            return
        except Exception:  # no NVML bindings or device: nvidia-smi instead
            self.nvml = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (OSError, ValueError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.nvml is not None:
            nv, _ = self.nvml
            self.stop_flag.set()
            self.thread.join(timeout=2)
            reasons = set()
            for _, _, bits in self.samples:
                for name, const in self.REASONS:
                    if bits & getattr(nv, const, 0):
                        reasons.add(name)
            sm = [m for m, _, _ in self.samples]
            return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz,
                    "reasons": sorted(reasons), "samples": len(sm),
                    "power_w_max": max(p for _, p, _ in self.samples) if self.samples else None,
                    "source": "NVML every 5 ms"}
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, mx, reasons, power = [], None, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
                power.append(float(parts[3]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm),
                "power_w_max": max(power) if power else None, "source": "nvidia-smi -lms 200"}


# ---------------------------------------------------------------------------
# CPU baseline: the reference's pack-rule algorithm restated in oracle/
# ---------------------------------------------------------------------------
def _cpu_threads():
    import torch
    from threadpoolctl import threadpool_limits
    n = os.cpu_count() or 1
    torch.set_num_threads(n)  # also under torchrun, which sets OMP_NUM_THREADS=1
    return n, threadpool_limits(limits=n)


def cpu_sample(seconds: float, chunk: int = 2048) -> dict:
    """The reference's pack-rule path (pack.py:139-180 on CPU tensors) on the
    first rows of config-3 matrix 0, restated in oracle/: fp32 matmul + argmax
    over the codebook (numpy/BLAS), the row scales of the reference's torch
    expression on CPU, and the 18-bit pack; whole rows, as many as fit in
    about ``seconds``."""
    import torch
    from oracle import oracle as O
    from pollux_b200 import synth
    nthreads, limit = _cpu_threads()
    w = synth.backbone_weights(CONFIG, device="cpu", shapes=[synth.CONFIG3_LAYER_SHAPES[0]])[0]
    wf = w.float().numpy()
    apr = wf.shape[1] // 24
    rows_per_chunk = max(1, chunk // apr)
    with limit:
        done_rows, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < seconds and done_rows + rows_per_chunk <= wf.shape[0]:
            blk = wf[done_rows:done_rows + rows_per_chunk]
            idx = O.nearest_fp32_pack_rule(blk.reshape(-1, 24))
            O.sigma16_pack_rule_cpu_torch(blk)
            O.pack_indices(idx)
            done_rows += rows_per_chunk
        dt = time.perf_counter() - t0
    atoms = done_rows * apr
    return {"value": atoms / dt / 1e9, "unit": "G atoms/s", "cores": nthreads, "kind": "port",
            "seconds": dt, "atoms": atoms,
            "sample": f"{atoms} atoms ({done_rows} rows) of config-3 matrix 0 (QKV [5760,1920], bf16 "
                      f"widened to fp32): fp32 matmul + argmax over the codebook, sigma16, 18-bit pack "
                      f"(oracle port of pack._quantize_h24_layer) with numpy/BLAS on {nthreads} host "
                      f"threads in {dt:.1f} s; torch threads {torch.get_num_threads()}"}


def cpu_stress_agreement(x_sample: np.ndarray, cat_sample: np.ndarray, ours: np.ndarray) -> dict:
    """Config 4 on the host: the exact fp64 oracle and the reference's
    training-rule semantics (bf16-rounded scores, castor.py:549-557) on a
    stratified sample of the stress atoms, timed, and the GPU's indices
    checked against them: index agreement per category, and the largest
    squared-distance excess of the GPU's codeword over the reference's choice
    (negative: the GPU's is nearer)."""
    from oracle import oracle as O
    from pollux_b200 import synth
    nthreads, limit = _cpu_threads()
    with limit:
        t0 = time.perf_counter()
        exact = O.nearest_exact(x_sample, O.RULE_TRAIN)
        t_exact = time.perf_counter() - t0
        t0 = time.perf_counter()
        ref = O.nearest_bf16_train_rule(x_sample)
        t_ref = time.perf_counter() - t0
    out = {"sample_atoms": int(x_sample.shape[0]), "cores": nthreads,
           "oracle_exact_atoms_per_s": x_sample.shape[0] / t_exact,
           "reference_bf16_port_atoms_per_s": x_sample.shape[0] / t_ref,
           "agreement_vs_exact_fp64": float(np.mean(ours == exact)),
           "agreement_vs_reference_bf16": float(np.mean(ours == ref)), "per_category": {}}
    diff = ours != ref
    if diff.any():
        d_o = O.dist2_fp64(x_sample[diff], ours[diff])
        d_r = O.dist2_fp64(x_sample[diff], ref[diff])
        out["max_rel_excess_vs_reference_bf16"] = float(np.max((d_o - d_r) / np.maximum(d_r, 1e-30)))
    else:
        out["max_rel_excess_vs_reference_bf16"] = 0.0
    for k, name in enumerate(synth.STRESS_CATEGORIES):
        m = cat_sample == k
        out["per_category"][name] = {"atoms": int(m.sum()),
                                     "agreement_vs_exact_fp64": float(np.mean(ours[m] == exact[m])),
                                     "agreement_vs_reference_bf16": float(np.mean(ours[m] == ref[m]))}
    return out


def run_reference(args) -> None:
    """The reference arm: each step one bounded sample of the workload through
    the CPU port of the reference's path, on all host threads; rank 0 only."""
    rank = _env_int("RANK", 0)
    if rank != 0:
        return
    from oracle import oracle as O
    O.build()
    per_step = []
    seconds = max(1.0, min(4.0, 90.0 / max(1, args.steps + args.warmup)))
    for i in range(args.warmup + args.steps):
        r = cpu_sample(seconds)
        if i >= args.warmup:
            per_step.append(r)
    secs = sum(r["seconds"] for r in per_step)
    atoms = sum(r["atoms"] for r in per_step)
    value = atoms / secs / 1e9
    out = {"metric": METRIC, "value": value, "unit": "G atoms/s", "n_gpus": args.gpus,
           "steps": args.steps, "warmup": args.warmup,
           "ms_per_step": secs / len(per_step) * 1e3, "higher_is_better": True,
           "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
           "impl": "reference",
           "config": {"workload": WORKLOAD, "atoms_per_step": atoms // len(per_step),
                      "step": "one bounded sample of whole rows of config-3 matrix 0 per step "
                              "(the full backbone would take hours on the host)"},
           "cpu_baseline": {**per_step[-1], "value": value},
           "e2e": {"value": value, "unit": "G atoms/s", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def _kernel_times(N) -> dict:
    """Summed event-timed ms and launch count of each instrumented kernel."""
    out = {}
    for name, k in (("screen_kernel", N.KERNEL_SCREEN), ("rescore_kernel", N.KERNEL_RESCORE),
                    ("prep_kernel", N.KERNEL_PREP)):
        ms, n = ctypes.c_double(0), ctypes.c_int64(0)
        N.check(N.load().h24_timing_read_kernel(k, ctypes.byref(ms), ctypes.byref(n)), "timing")
        out[name] = (ms.value, int(n.value))
    return out


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    world = _env_int("WORLD_SIZE", 1)
    rank = _env_int("RANK", 0)
    local = _env_int("LOCAL_RANK", 0)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    from pollux_b200 import castor, pack, shard, synth
    from pollux_b200 import _native as N

    shapes = synth.backbone_shapes(CONFIG)
    weights = synth.backbone_weights(CONFIG, device=dev)  # identical on every rank (seeded)
    atoms_total = sum(o * i // 24 for o, i in shapes)
    ranges = [shard.shard_rows(o, i, world, rank) for o, i in shapes]
    parts = [(w, r0, r1) for w, (r0, r1) in zip(weights, ranges)]
    atoms_rank = sum((r1 - r0) * i // 24 for (r0, r1), (o, i) in zip(ranges, shapes))
    # This rank's packed bytes and scales of all 72 matrices in one buffer each,
    # padded to the largest rank's size (the all-gather's equal-size blocks).
    def sizes(r):
        pb = sb = 0
        for o, i in shapes:
            s0, s1 = shard.shard_rows(o, i, world, r)
            b0, b1 = shard.packed_range(s0, s1, i)
            pb += b1 - b0
            sb += s1 - s0
        return pb, sb
    all_sizes = [sizes(r) for r in range(world)]
    max_pb = max(p for p, _ in all_sizes)
    max_sb = max(s for _, s in all_sizes)
    pbuf = torch.zeros(max_pb, dtype=torch.uint8, device=dev)
    sbuf = torch.zeros(max_sb, dtype=torch.float16, device=dev)
    outs, po, so = [], 0, 0
    for (o, i), (r0, r1) in zip(shapes, ranges):
        b0, b1 = shard.packed_range(r0, r1, i)
        outs.append((pbuf[po:po + b1 - b0], sbuf[so:so + r1 - r0]))
        po += b1 - b0
        so += r1 - r0
    stream = torch.cuda.current_stream(dev)

    def step():
        pack.quantize_layer_rows(parts, outs)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    castor.device_check(dev)
    # Checks outside the timed region: every index in range and unpack(pack)
    # the identity on matrix 0's shard.
    p0, _ = outs[0]
    n0 = (ranges[0][1] - ranges[0][0]) * shapes[0][1] // 24
    idx0 = castor.unpack_indices(p0, n0)
    assert int(idx0.max()) <= 196560 and int(idx0.min()) >= 0
    assert torch.equal(castor.pack_indices(idx0), p0), "pack/unpack round trip failed"

    N.load().h24_timing_enable(1)
    _kernel_times(N)
    castor.quantize_stats(dev)
    launches0 = castor.launch_count()
    clocks = ClockSampler(local)
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    t_start = torch.cuda.Event(enable_timing=True)
    t_stop = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for _ in range(args.steps):
        step()
    t_stop.record(stream)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    launches = castor.launch_count() - launches0
    ktimes = _kernel_times(N)
    N.load().h24_timing_enable(0)
    exhaustive, exact_scores, chunks = castor.quantize_stats(dev)
    elapsed_ms = t_start.elapsed_time(t_stop)
    if world > 1:
        t = torch.tensor([elapsed_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms = float(t.item())
    ms_per_step = elapsed_ms / args.steps
    value = atoms_total * args.steps / (elapsed_ms / 1e3) / 1e9

    # Per-kernel shares and rooflines (this rank's launches, CUDA events on the
    # launching stream over the timed region).
    peaks = _peaks()
    peak_t = peaks.get("bf16_tflops_sustained")
    peak_t_src = "measured sustained bf16 (MEASURED_PEAKS.json)"
    if peak_t is None:
        peak_t, peak_t_src = 1400.0, "fallback sustained bf16 1.4 PFLOP/s"
    peak_b = peaks.get("hbm_gbs")
    peak_b_src = "measured HBM copy (MEASURED_PEAKS.json)"
    if peak_b is None:
        peak_b, peak_b_src = 6650.0, "fallback HBM 6.65 TB/s"
    atoms_timed = atoms_rank * args.steps
    kern = {}
    for name, (ms, n) in ktimes.items():
        kern[name] = {"ms_total": ms, "launches": n, "ms_per_launch": ms / max(1, n),
                      "share_of_step": ms / max(1e-9, elapsed_ms), "atoms_per_launch": atoms_timed / max(1, n)}
    scr = kern["screen_kernel"]
    screen_tflops = SCREEN_FLOP_PER_ATOM * scr["atoms_per_launch"] / (scr["ms_per_launch"] / 1e3) / 1e12
    screen_roof = {"bound": "tensor", "kernel": "screen_kernel", "achieved": screen_tflops,
                   "peak": peak_t, "unit": "TFLOP/s", "frac": screen_tflops / peak_t,
                   "peak_source": peak_t_src, "flop_per_atom": SCREEN_FLOP_PER_ATOM,
                   "launch_ms_mean": scr["ms_per_launch"], "launches": scr["launches"],
                   "traffic": SCREEN_TRAFFIC_PER_ATOM * scr["atoms_per_launch"],
                   "traffic_source": "ncu dram bytes of one 262,144-atom launch, scaled to this "
                                     "launch's atoms (profiles/screen_kernel_262k.md)"}
    res_ = kern["rescore_kernel"]
    res_s = res_["ms_per_launch"] / 1e3
    rescore_gbs = RESCORE_BYTES_PER_ATOM_BF16 * res_["atoms_per_launch"] / res_s / 1e9
    sm_mhz = (clk or {}).get("sm_mhz") or (clk or {}).get("sm_max_mhz") or 1965.0
    issue_peak = torch.cuda.get_device_properties(dev).multi_processor_count * ISSUE_SLOTS_PER_SM \
        * sm_mhz * 1e6 / 1e9
    issue_rate = RESCORE_WARP_INST_PER_ATOM * res_["atoms_per_launch"] / res_s / 1e9
    rescore_roof = {"bound": "issue", "kernel": "rescore_kernel", "achieved": issue_rate,
                    "peak": issue_peak, "unit": "G warp-instructions/s", "frac": issue_rate / issue_peak,
                    "peak_source": f"SMs x {ISSUE_SLOTS_PER_SM} warp instructions per cycle x the "
                                   f"median SM clock sampled in the timed region ({sm_mhz:.0f} MHz)",
                    "warp_instructions_per_atom": RESCORE_WARP_INST_PER_ATOM,
                    "instructions_source": "ncu smsp__inst_executed.sum of one 262,144-atom launch "
                                           "(profiles/rescore_kernel_262k.md)",
                    "launch_ms_mean": res_["ms_per_launch"], "launches": res_["launches"],
                    "traffic": RESCORE_TRAFFIC_PER_ATOM * res_["atoms_per_launch"],
                    "traffic_source": "ncu dram bytes of one 262,144-atom launch, scaled to this "
                                      "launch's atoms (profiles/rescore_kernel_262k.md)",
                    "memory_floor": {"bound": "hbm", "bytes_per_atom": RESCORE_BYTES_PER_ATOM_BF16,
                                     "achieved": rescore_gbs, "peak": peak_b, "unit": "GB/s",
                                     "frac": rescore_gbs / peak_b, "peak_source": peak_b_src}}
    dominant = max(("screen_kernel", "rescore_kernel"), key=lambda k: kern[k]["ms_total"])
    roofline = screen_roof if dominant == "screen_kernel" else rescore_roof

    # Optional collective: the packed shards and scales gathered on every rank
    # (one all_gather_into_tensor each, NCCL over NVLink), timed on its own.
    gather = None
    if world > 1:
        pall = torch.empty(world * max_pb, dtype=torch.uint8, device=dev)
        sall = torch.empty(world * max_sb, dtype=torch.float16, device=dev)
        for _ in range(2):
            dist.all_gather_into_tensor(pall, pbuf)
            dist.all_gather_into_tensor(sall, sbuf)
        torch.cuda.synchronize()
        barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 5
        g0.record(stream)
        for _ in range(reps):
            dist.all_gather_into_tensor(pall, pbuf)
            dist.all_gather_into_tensor(sall, sbuf)
        g1.record(stream)
        torch.cuda.synchronize()
        gms = torch.tensor([g0.elapsed_time(g1) / reps], device=dev)
        dist.all_reduce(gms, op=dist.ReduceOp.MAX)
        # The gathered bytes of matrix 0 equal the single-GPU bytes.
        whole_p, whole_s = pack.quantize_layers([weights[0]])[0]
        got_p, got_s = [], []
        for r in range(world):
            s0, s1 = shard.shard_rows(*shapes[0], world, r)
            b0, b1 = shard.packed_range(s0, s1, shapes[0][1])
            got_p.append(pall[r * max_pb: r * max_pb + b1 - b0])
            got_s.append(sall[r * max_sb: r * max_sb + s1 - s0])
        ok = torch.equal(torch.cat(got_p), whole_p) and torch.equal(torch.cat(got_s), whole_s)
        gather = {"what": "all_gather_into_tensor of every rank's packed shards (and one of its "
                          "fp16 scales) of all 72 matrices, NCCL",
                  "ms": float(gms.item()), "bytes_gathered": world * (max_pb + 2 * max_sb),
                  "matrix0_equals_single_gpu_bytes": bool(ok),
                  "share_of_quantize_step": float(gms.item()) / ms_per_step}
        del pall, sall

    e2e = None
    if not args.skip_e2e:
        barrier()
        e2e = run_e2e(args, weights, shapes, ranges, dev, world)
        if world > 1:
            t = torch.tensor([e2e["ms_per_step"]], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e2e["ms_per_step"] = float(t.item())
            e2e["timing"] = "wall clock per rank around synchronised steps, max over ranks"
            for key in ("h2d_bytes_per_step", "d2h_bytes_per_step"):
                t = torch.tensor([e2e[key]], dtype=torch.float64, device=dev)
                dist.all_reduce(t)
                e2e[key] = int(t.item())
        e2e["value"] = atoms_total / (e2e["ms_per_step"] / 1e3) / 1e9

    extras = {}
    if rank == 0 and world == 1:
        del parts, outs
        torch.cuda.empty_cache()
        stress = None
        if not args.skip_stress:
            stress, sample = run_stress(args, dev)
        if not args.skip_cpu:
            extras["cpu_baseline"] = cpu_sample(12.0)
            if stress is not None:
                stress["host_check"] = cpu_stress_agreement(*sample)
        extras["stress"] = stress
        if not args.skip_components:
            extras["hbm_kernels"] = run_components(args)
            extras["training_projection"] = run_projection(dev)

    if rank == 0:
        out = {
            "metric": METRIC, "value": value, "unit": "G atoms/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic",
            "config": {"workload": WORKLOAD, "atoms_per_step": atoms_total, "matrices": len(shapes),
                       "atoms_per_rank": atoms_rank,
                       "packed_bytes_per_step": sum(((o * i // 24 + 3) // 4) * 9 for o, i in shapes),
                       "weight_bytes_per_step": sum(o * i * 2 for o, i in shapes),
                       "l2": "inputs larger than L2: 1.59 GB of bf16 weights read per step",
                       "compute": "bf16 weights read natively; bf16 x bf16 -> fp32 tcgen05 screening, "
                                  "fp32/fp64 rescore; sigma in torch's CUDA mean order"},
            "roofline": roofline,
            "rooflines": {"screen_kernel": screen_roof, "rescore_kernel": rescore_roof},
            "kernels": kern,
            "gpu_launches": launches,
            "clocks": clk,
            "search_stats": {"exhaustive_atoms": exhaustive, "exact_scores": exact_scores,
                             "flagged_32col_units": chunks, "atoms": atoms_timed,
                             "exhaustive_scan_equivalent_tflops":
                                 value * 1e9 * EXHAUSTIVE_FLOP_PER_ATOM / 1e12},
            "allgather": gather,
            "e2e": e2e,
            "cpu_baseline": extras.get("cpu_baseline"),
            "stress": extras.get("stress"),
            "hbm_kernels": extras.get("hbm_kernels"),
            "training_projection": extras.get("training_projection"),
        }
        print(json.dumps(out), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_e2e(args, weights, shapes, ranges, dev, world) -> dict:
    """The same step through the public API with host buffers: the bf16
    backbone as a model state_dict in page-locked host memory, packed by
    pack.quantize_state_dict (pack_checkpoint's tensor loop, pack.py:268-287:
    packed bytes and fp16 scales returned as host tensors) on one GPU, or on
    N ranks pack.quantize_layers_host for this rank's rows of every matrix;
    the host-to-device copies of the weights and the copies of the outputs
    back are inside the timed region.  The per-matrix drop-in
    pack._quantize_h24_layer loop is timed too, for context."""
    import torch
    from pollux_b200 import castor, pack
    names = [f"layers.{l}.{m}.weight" for l in range(len(shapes) // 4) for m in ("qkv", "o", "up", "down")]
    host_w = [w.cpu().pin_memory() for w in weights]
    state = dict(zip(names, host_w))
    torch.cuda.synchronize()

    def e2e_step():
        if world == 1:
            out = pack.quantize_state_dict(state)
            return [(out[n.replace(".weight", ".packed_weights")], out[n.replace(".weight", ".sigma_rows")])
                    for n in names]
        return pack.quantize_layers_host([(w, r0, r1) for w, (r0, r1) in zip(host_w, ranges)])

    def timed(fn, steps, warm):
        # The first calls of a process are slower (page-locked output buffers
        # and the device pool grow to their working set): steady state after
        # a few.  The warm-up keeps each call's outputs until the next call
        # returns, as the timed loop does, so that torch's page-locked host
        # cache already holds the two sets of output buffers that pattern
        # needs (pinning a new set inside the timed loop costs ~70 ms).
        res = None
        for _ in range(warm):
            res = fn()
        t0 = time.perf_counter()
        for _ in range(steps):
            res = fn()
        return (time.perf_counter() - t0) / steps, res

    # The page-locked host-to-device bandwidth this box gives at the moment
    # (PCIe links may be shared with other jobs), for reading the number.
    dev_w = [torch.empty_like(w, device=dev) for w in host_w]
    for _ in range(2):
        for h, d in zip(host_w, dev_w):
            d.copy_(h, non_blocking=True)
    torch.cuda.synchronize()
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0.record()
    for h, d in zip(host_w, dev_w):
        d.copy_(h, non_blocking=True)
    c1.record()
    c1.synchronize()
    h2d_gbps = sum(h.numel() * h.element_size() for h in host_w) / (c0.elapsed_time(c1) / 1e3) / 1e9
    del dev_w
    steps = max(1, min(args.steps, 5))
    dt, res = timed(e2e_step, steps, max(5, args.warmup))
    per_matrix = None
    if world == 1:
        cb = castor.get_h24_codebook("cpu", torch.float32)
        dtm, res_m = timed(lambda: [pack._quantize_h24_layer(w, cb) for w in host_w], min(steps, 3), 2)
        assert all(torch.equal(a[0], b[0]) and torch.equal(a[1], b[1]) for a, b in zip(res, res_m))
        per_matrix = {"api": "pack._quantize_h24_layer per matrix (bf16 host weights)", "ms_per_step": dtm * 1e3}
    h2d = sum((r1 - r0) * i * 2 for (r0, r1), (o, i) in zip(ranges, shapes))
    d2h = sum(p.numel() + s.numel() * 2 for p, s in res)
    del host_w, state
    return {"unit": "G atoms/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": dt * 1e3, "steps": steps, "h2d_GBps_measured": h2d_gbps,
            "api": ("pollux_b200.pack.quantize_state_dict on the 72-matrix bf16 state_dict" if world == 1
                    else "pollux_b200.pack.quantize_layers_host, this rank's rows of every matrix"),
            "per_matrix_drop_in": per_matrix}


def run_stress(args, dev):
    """Config 4: 2^24 stress atoms (seed 3) through the training rule
    (castor_quantize_leech's search): throughput, plus the GPU's choice on the
    reference's own stress fixtures (tests/golden/stress.npz: 4,096 atoms with
    the indices of pack.py's fp32 path and of castor's bf16 path) as the
    largest relative squared-distance excess over the reference's choice.
    Returns the report and a stratified sample for the host check."""
    import torch
    from pollux_b200 import castor, synth
    n = 1 << 24
    cb = castor.get_h24_codebook(dev, torch.float32)
    x, cat = synth.stress_atoms(n, cb, seed=3, device=dev, return_category=True)
    castor.quantize_indices(x[:1 << 16], 0)
    torch.cuda.synchronize()
    castor.quantize_stats(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 3
    e0.record()
    for _ in range(reps):
        idx = castor.quantize_indices(x, 0)
    e1.record()
    e1.synchronize()
    castor.device_check(dev)
    ms = e0.elapsed_time(e1) / reps
    exh, exact_scores, chunks = castor.quantize_stats(dev)
    rep = {"atoms": n, "rule": "training (castor_quantize_leech)", "ms": ms,
           "G_atoms_per_s": n / (ms / 1e3) / 1e9,
           "exhaustive_atoms_per_call": exh / reps, "exact_fp64_scores_per_atom": exact_scores / (reps * n),
           "flagged_32col_units_per_atom": chunks / (reps * n)}
    # Against the reference's fixtures: fp64 squared distances on the GPU.
    g = np.load(os.path.join(HERE, "tests", "golden", "stress.npz"))
    xg = torch.from_numpy(g["atoms"]).to(dev)
    cb64 = cb.double()
    for rule, key in ((1, "pack_rule_idx"), (0, "train_bf16_idx")):
        ours = castor.quantize_indices(xg, rule).long()
        ref = torch.from_numpy(g[key]).to(dev).long()
        d_o = ((xg.double() - cb64[ours]) ** 2).sum(1)
        d_r = ((xg.double() - cb64[ref]) ** 2).sum(1)
        rel = (d_o - d_r) / d_r.clamp_min(1e-30)
        rep[f"golden_{key}"] = {"agreement": float((ours == ref).float().mean()),
                                "max_rel_excess": float(rel.max()),
                                "min_rel_excess": float(rel.min())}
    # Stratified sample for the host check: 2^14 atoms of each category.
    gsel = torch.Generator(device=dev).manual_seed(4)
    sel = []
    for k in range(len(synth.STRESS_CATEGORIES)):
        pos = torch.nonzero(cat == k).flatten()
        sel.append(pos[torch.randperm(pos.numel(), generator=gsel, device=dev)[:1 << 14]])
    sel = torch.cat(sel)
    sample = (x[sel].cpu().numpy(), cat[sel].cpu().numpy(), idx[sel].cpu().numpy().astype(np.int64))
    del x, cat, idx
    torch.cuda.empty_cache()
    return rep, sample


def run_projection(dev) -> dict:
    """F3: the fused H24 block of pollux_step (row RMS, normalise, training-rule
    search, rescale into p.data) for the 48 config-2 matrices in one call."""
    import torch
    from pollux_b200 import castor, synth
    weights = synth.backbone_weights(2, device=dev)
    outs_p = [torch.empty_like(w) for w in weights]
    pairs = list(zip(outs_p, weights))
    castor.project_h24_many(pairs)
    torch.cuda.synchronize()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p0.record()
    for _ in range(3):
        castor.project_h24_many(pairs)
    p1.record()
    p1.synchronize()
    pms = p0.elapsed_time(p1) / 3
    atoms = sum(w.numel() // 24 for w in weights)
    return {"what": "pollux_step H24 block for all 48 config-2 fp32 matrices in one fused call",
            "ms": pms, "G_atoms_per_s": atoms / (pms / 1e3) / 1e9}


def run_search_only(args) -> None:
    """Search kernel alone on ``--search-atoms`` seeded N(0, 2) atoms (the
    scale of normalised weights); for profiling the screening kernel on a
    small case."""
    import torch
    from pollux_b200 import castor
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(7)
    x = torch.randn(args.search_atoms, 24, generator=g, device=dev) * 1.4142135
    if args.search_dtype == "bf16":
        x = x.to(torch.bfloat16)
    from pollux_b200 import _native as N
    for _ in range(args.warmup):
        castor.quantize_indices(x, 1)
    torch.cuda.synchronize()
    castor.quantize_stats(dev)
    N.load().h24_timing_enable(1)
    _kernel_times(N)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        castor.quantize_indices(x, 1)
    t1.record()
    torch.cuda.synchronize()
    castor.device_check(dev)
    kt = _kernel_times(N)
    N.load().h24_timing_enable(0)
    exhaustive, exact_scores, chunks = castor.quantize_stats(dev)
    ms = t0.elapsed_time(t1) / args.steps
    atoms_s = args.search_atoms / (ms / 1e3)
    n = args.search_atoms * args.steps
    print(json.dumps({"search_atoms": args.search_atoms, "dtype": args.search_dtype, "ms_per_call": ms,
                      "G_atoms_per_s": atoms_s / 1e9,
                      "screen_ms_per_call": kt["screen_kernel"][0] / args.steps,
                      "rescore_ms_per_call": kt["rescore_kernel"][0] / args.steps,
                      "prep_ms_per_call": kt["prep_kernel"][0] / args.steps,
                      "exhaustive_per_atom": exhaustive / n, "exact_scores_per_atom": exact_scores / n,
                      "flagged_32col_units_per_atom": chunks / n}), flush=True)


def run_components(args) -> dict:
    """HBM-bound kernels on config 5: the packed indices of 18 [7680,1920]
    layers (11,059,200 indices, uniform in [0,196560]) -- 18-bit pack of the
    int32 indices, unpack back to int32, and LUT dequant of all 18 layers to
    fp16 in one batched launch.  Each kernel is timed with CUDA events around
    a run of back-to-back calls that rotate over several buffer sets (pack and
    unpack: 8 sets, 552 MB; dequant: 2 sets of 531 MB of output), so no call
    finds its inputs in L2; the calls are replayed from one CUDA graph after
    an L2 flush, so the host's launch rate plays no part."""
    import ctypes
    import torch
    from pollux_b200 import castor, synth
    from pollux_b200 import _native as N
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    layers = 18
    rows, in_f = synth.CONFIG5_SHAPE
    per = rows * in_f // 24
    idx_l, sig_l = [], []
    for l in range(layers):
        i, sg = synth.config5_layer(seed=5 + l, device=dev)
        idx_l.append(i)
        sig_l.append(sg)
    idx = torch.cat(idx_l)
    n = idx.numel()
    sets = 8
    idxs = [idx] + [idx.roll(17 * k) for k in range(1, sets)]
    packs = [torch.empty(((n + 3) // 4) * 9, dtype=torch.uint8, device=dev) for _ in range(sets)]
    backs = [torch.empty(n, dtype=torch.int32, device=dev) for _ in range(sets)]
    outs = [[torch.empty(rows, in_f, dtype=torch.float16, device=dev) for _ in range(layers)]
            for _ in range(2)]
    bad = torch.zeros(1, dtype=torch.int32, device=dev)
    flush = torch.empty(512 << 20, dtype=torch.uint8, device=dev)
    lib = N.load()
    per_layer_bytes = per // 4 * 9

    def cur():
        """The current stream (a capture stream while a graph is recorded)."""
        return torch.cuda.current_stream(dev).cuda_stream

    def pack(k):
        N.check(lib.h24_pack(idxs[k].data_ptr(), n, packs[k].data_ptr(), cur()), "pack")

    def unpack(k):
        N.check(lib.h24_unpack(packs[k].data_ptr(), packs[k].numel() // 9, n, backs[k].data_ptr(),
                               cur()), "unpack")

    descs = []
    for k in range(2):
        L = (N.DequantLayer * layers)()
        for l in range(layers):
            L[l] = N.DequantLayer(packs[k].data_ptr() + l * per_layer_bytes, sig_l[l].data_ptr(),
                                  outs[k][l].data_ptr(), rows, in_f)
        descs.append(L)

    def dequant(k):
        N.check(lib.h24_dequant_batched(ctypes.cast(descs[k % 2], ctypes.c_void_p), layers,
                                        bad.data_ptr(), cur()), "dequant")

    def timed(fn, calls, reps):
        """Median ms per call of `calls` back-to-back calls fn(0..calls-1),
        captured once into a CUDA graph and replayed after an L2 flush."""
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):  # one eager run before capture
            for k in range(calls):
                fn(k)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for k in range(calls):
                fn(k)
        ts = []
        for i in range(reps + 2):
            flush.fill_(i & 0xFF)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            g.replay()
            e1.record()
            e1.synchronize()
            if i >= 2:
                ts.append(e0.elapsed_time(e1) / calls)
        del g
        return statistics.median(ts)

    # INT8 token embedding (PolluxConfig defaults: vocab 50688 x n_embd 1920),
    # two buffer sets of 389 MB of fp32 each.
    vocab, d = 50688, 1920
    emb_w = [torch.randn(vocab, d, device=dev) * 0.02 for _ in range(2)]
    emb_q = [torch.empty(vocab, d, dtype=torch.int8, device=dev) for _ in range(2)]
    emb_mu = [torch.empty(vocab, dtype=torch.float16, device=dev) for _ in range(2)]
    emb_out = [torch.empty(vocab, d, dtype=torch.float16, device=dev) for _ in range(2)]

    def int8_quant(k):
        N.check(lib.h24_int8_quantize(emb_w[k].data_ptr(), vocab, d, emb_q[k].data_ptr(),
                                      emb_mu[k].data_ptr(), cur()), "int8_quantize")

    def int8_deq(k):
        N.check(lib.h24_int8_dequant(emb_q[k].data_ptr(), emb_mu[k].data_ptr(), vocab, d,
                                     emb_out[k].data_ptr(), cur()), "int8_dequant")

    # Decode through the 18 config-5 layers: LUT GEMV straight from the packed
    # bytes vs a dense fp16 GEMV (cuBLAS) on the materialised weights.
    xs = {b: torch.randn(b, in_f, device=dev) for b in (1, 8)}
    ys = {b: torch.empty(b, rows, device=dev) for b in (1, 8)}
    x16 = {b: xs[b].half() for b in (1, 8)}

    def lut_sweep(b):
        def run(k):
            for l in range(layers):
                N.check(lib.h24_lut_gemv(packs[k].data_ptr() + l * per_layer_bytes, sig_l[l].data_ptr(),
                                         rows, in_f, xs[b].data_ptr(), b, ys[b].data_ptr(),
                                         bad.data_ptr(), cur()), "lut_gemv")
        return run

    ys16 = {b: torch.empty(b, rows, dtype=torch.float16, device=dev) for b in (1, 8)}

    def dense_sweep(b):
        def run(k):
            for l in range(layers):
                torch.matmul(x16[b], outs[k % 2][l].t(), out=ys16[b])
        return run

    reps = max(3, args.steps)
    # Fill every packed buffer before anything reads them.
    for k in range(sets):
        pack(k)
    torch.cuda.synchronize()
    dequant(0)
    dequant(1)
    t_lut1 = timed(lut_sweep(1), 2, reps)
    t_lut8 = timed(lut_sweep(8), 2, reps)
    t_dense1 = timed(dense_sweep(1), 2, reps)
    t_dense8 = timed(dense_sweep(8), 2, reps)
    t_pack = timed(pack, sets, reps)
    t_unpack = timed(unpack, sets, reps)
    t_deq = timed(dequant, 2, reps)
    t_i8q = timed(int8_quant, 2, reps)
    t_i8d = timed(int8_deq, 2, reps)
    torch.cuda.synchronize()
    for k in range(sets):
        assert torch.equal(backs[k], idxs[k]), "pack/unpack round trip failed"
    assert int(bad.item()) == 0
    peak = 6557.1
    try:
        with open(os.path.join(HERE, "MEASURED_PEAKS.json")) as f:
            peak = float(json.load(f)["hbm_gbs"])
    except (OSError, ValueError, KeyError):
        pass
    pack_bytes = n * 4 + packs[0].numel()
    deq_bytes = packs[0].numel() + layers * rows * 2 + layers * rows * in_f * 2
    res = {}
    i8q_bytes = vocab * d * 5 + vocab * 2      # fp32 in, int8 + fp16 scales out
    i8d_bytes = vocab * d * 3 + vocab * 2      # int8 + scales in, fp16 out
    for name, t, b in (("pack", t_pack, pack_bytes), ("unpack", t_unpack, pack_bytes),
                       ("dequant", t_deq, deq_bytes), ("int8_quantize", t_i8q, i8q_bytes),
                       ("int8_dequant", t_i8d, i8d_bytes)):
        gbs = b / (t / 1e3) / 1e9
        res[name] = {"ms": t, "algorithmic_bytes": b, "GB_per_s": gbs, "frac_of_measured_hbm": gbs / peak}
    wbytes = layers * rows * in_f * 2
    res["lut_gemv"] = {
        "what": "y = x @ W.T through all 18 config-5 layers, W never materialised (fp32 x, "
                "fp32 products); against torch.matmul of the materialised fp16 weights (cuBLAS); "
                "both sweeps replayed from CUDA graphs",
        "batch1_ms": t_lut1, "batch8_ms": t_lut8,
        "dense_fp16_batch1_ms": t_dense1, "dense_fp16_batch8_ms": t_dense8,
        "dense_equivalent_GB_per_s_batch1": wbytes / (t_lut1 / 1e3) / 1e9,
        "packed_bytes": layers * per_layer_bytes, "fp16_weight_bytes": wbytes}
    res["workload"] = ("config5: 18 layers x [7680,1920], 11,059,200 uniform indices; pack int32->18-bit, "
                       "unpack 18-bit->int32, batched LUT dequant to fp16; INT8 embedding "
                       "[50688,1920] quantize and dequant; back-to-back calls over "
                       "rotating buffer sets larger than L2, after an L2 flush")
    res["hbm_peak_gbs"] = peak
    return res


def run_torch_reference(args) -> None:
    """Secondary comparator, not a bench line: the reference's own GPU search
    for the pack rule, pack._quantize_h24_layer on a CUDA tensor (pack.py:
    159-178: chunks of 4096 atoms, an fp32 torch.matmul against all 196,560
    kissing points, the row maximum, the norm test), written here as the same
    torch operations and timed on config-3 matrix 0 ([5760, 1920], 460,800
    atoms) with CUDA events; also the share of its indices that equal the
    library's exact ones.  Prints one JSON line."""
    import math
    import torch
    from pollux_b200 import castor, pack, synth
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    kp = castor.get_h24_codebook(dev, torch.float32)[1:].contiguous()
    w = synth.backbone_weights(3, device=dev, shapes=[synth.CONFIG3_LAYER_SHAPES[0]])[0]

    def search(weight):
        wf = weight.detach().float()
        atoms = wf.reshape(-1, 24)
        sig = (torch.sqrt(wf.pow(2).mean(-1) + 1e-8) * math.sqrt(12.0)).clamp_min(1e-8)
        idx = torch.zeros(atoms.shape[0], dtype=torch.long, device=dev)
        for i in range(0, atoms.shape[0], 4096):
            a = atoms[i:i + 4096]
            _, best = torch.matmul(a, kp.t()).max(dim=-1)
            idx[i:i + 4096] = (best + 1).masked_fill(a.norm(dim=-1) < 1e-8, 0)
        return idx, sig

    search(w[:256])
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    idx, _ = search(w)
    e1.record()
    e1.synchronize()
    ms = e0.elapsed_time(e1)
    n = w.numel() // 24
    packed, _ = pack.quantize_layers([w])[0]
    ours = castor.unpack_indices(packed, n).long()
    rate = n / (ms / 1e3)
    print(json.dumps({"what": "the reference's GPU pack-rule search (fp32 matmul chunks of 4096 + max) as torch ops",
                      "matrix": list(w.shape), "atoms": n, "ms": ms, "G_atoms_per_s": rate / 1e9,
                      "config3_backbone_s": 33177600 / rate, "tf32": torch.backends.cuda.matmul.allow_tf32,
                      "index_agreement_with_library": float((ours == idx).float().mean())}), flush=True)


def run_lut_only(args) -> None:
    """Profile mode: the LUT GEMV alone through the 18 config-5 layers (one
    25 MB packed set, fp32 x of batch --lut-batch), CUDA events around
    --steps eager sweeps after --warmup sweeps; prints one JSON line."""
    import torch
    from pollux_b200 import castor, synth
    from pollux_b200 import _native as N
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    layers = 18
    rows, in_f = synth.CONFIG5_SHAPE
    packs, sigs = [], []
    for l in range(layers):
        i, sg = synth.config5_layer(seed=5 + l, device=dev)
        packs.append(castor.pack_indices(i))
        sigs.append(sg)
    b = args.lut_batch
    x = torch.randn(b, in_f, device=dev)
    y = torch.empty(b, rows, device=dev)
    bad = torch.zeros(1, dtype=torch.int32, device=dev)
    lib = N.load()
    st = torch.cuda.current_stream(dev).cuda_stream

    def sweep():
        for l in range(layers):
            N.check(lib.h24_lut_gemv(packs[l].data_ptr(), sigs[l].data_ptr(), rows, in_f, x.data_ptr(), b,
                                     y.data_ptr(), bad.data_ptr(), st), "lut_gemv")

    for _ in range(args.warmup):
        sweep()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        sweep()
    e1.record()
    e1.synchronize()
    assert int(bad.item()) == 0
    print(json.dumps({"lut_gemv_batch": b, "layers": layers, "shape": [rows, in_f],
                      "ms_per_sweep": e0.elapsed_time(e1) / args.steps}), flush=True)


def main():
    # libh24 is built from this checkout's sources (incremental; a no-op when
    # the library is current).
    from pollux_b200 import build as _build
    _build.build()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--skip-e2e", action="store_true")
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--skip-stress", action="store_true")
    ap.add_argument("--search-atoms", type=int, default=0,
                    help="profile mode: time only the search on this many atoms")
    ap.add_argument("--search-dtype", choices=["f32", "bf16"], default="f32")
    ap.add_argument("--components", action="store_true",
                    help="time the HBM-bound kernels (pack/unpack/dequant) on config 5 only")
    ap.add_argument("--skip-components", action="store_true")
    ap.add_argument("--lut-only", action="store_true",
                    help="profile mode: time only the LUT GEMV sweep over the config-5 layers")
    ap.add_argument("--lut-batch", type=int, default=1)
    ap.add_argument("--torch-reference", action="store_true",
                    help="time the reference's GPU search as torch ops on one config-3 matrix (a comparator)")
    args = ap.parse_args()
    if args.torch_reference:
        run_torch_reference(args)
    elif args.lut_only:
        run_lut_only(args)
    elif args.search_atoms:
        run_search_only(args)
    elif args.components:
        print(json.dumps(run_components(args)), flush=True)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
