#!/usr/bin/env python3
"""bench.py -- EXL3 trellis quantizer throughput on B200.

Metric: trellis-encoded weights/s (Viterbi + BlockLDLQ) at K=4.
Workload (one "step"): quantize_linear of one configuration-2 projection --
5120x5120 bf16 weight ~N(0, 0.02^2) with 0.1% outliers x10, Hessian from 4096
synthetic heavy-tailed activation rows, random-sign Hadamard rotation, damped
block-LDL, full BlockLDLQ sweep with the tail-biting trellis encode (K=4,
mul1, quantize_linear defaults: pivot 128, margin 0), packing and W_hat.

  value : weights/s with W and H resident in HBM (CUDA events around the
          timed steps, max over ranks)
  e2e   : same metric through the public API from pinned host buffers, the
          host->device copy of W and H and the device->host copy of the
          results inside every timed step
  N > 1 : one process per GPU, each quantizing its own projection (seeded per
          rank, no collective on the data path): weak scaling -- the layer-
          sharded way a stack of projections runs.  "per_layer" adds the time
          of ONE projection with its output columns split over the N ranks
          (exl3b.shard; all-gather of the finished tensors included);
          "per_layer_c5" the time of one 27B-shape layer (config 5 shapes and
          mixed K) with its output channels split over the N ranks
          (exl3b.stack.quantize_layer_split), at every N including 1

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--config c2|c3|c4] [--K k]

The default line is configuration 2 (the driver's bench line).  --config c3
(fused q/k/v module, K = [5, 7, 7], one shared Hessian) and --config c4
(17408 -> 5120 down projection at --K) print the same line for those
workloads.  "kernels" adds each device stage's roofline: the fused tile kernel
(fp32 lanes: 3 rounded fp32 ops per add-compare-select), the tcgen05 feedback
GEMM (useful FLOP vs the TF32 tensor rate), the Hadamard rotations (HBM bytes)
and the block LDL (k^3/3 FLOP against the fp32 FMA rate, although its trailing
updates run on the tensor cores).

--impl reference times the reference algorithm's CPU implementation (the C/numpy
restatement under oracle/; the reference itself is Python and does not travel)
on the host cores: each step is one k-block launch of the same projection's
LDLQ sweep (320 tiles), rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "exl3xpu-mixedk_b200")
for _p in (REPO, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "trellis-encoded weights/s (Viterbi+LDLQ) at K=4"
UNIT = "weights/s"
K_BITS = 4
DIM = 5120
# Algorithmic work per weight (one trellis step per weight and pass, 2 passes
# at margin 0): 2 x 2^16 add-compare-selects, counted as 2 fp32 lane ops each
# (the add and the compare-select): 262144 ops per weight.  This is the
# roofline's `achieved`.  Bit-exactness with the reference's fp32 "sq" emit
# needs 3 correctly rounded fp32 operations per add-compare-select (f - x,
# its square, + best; fusing any two changes the rounding) with the minimum on
# the ALU pipe beside them: that fp32-pipe floor is reported as a second
# fraction.  The fp32 pipe retires 128 lane operations per SM per clock (the
# packed f32x2 forms issue at half rate: they save issue slots, not fp32
# throughput).
OPS_PER_WEIGHT = 2 * 65536 * 2
FLOOR_OPS_PER_WEIGHT = 2 * 65536 * 3
FP32_NOTE = ("2 ops (add, compare-select) per add-compare-select, 2 x 2^16 per weight; "
             "peak = SMs x 128 fp32 lanes x max SM clock")
# DRAM traffic of the tile kernel per encoded weight, K = 4: dram__bytes_read.sum +
# dram__bytes_write.sum of one ldlq_lazy_kernel<4> launch of the 2048 x 2048
# profiling case (4096 tiles, 1048576 weights), divided by its weights; the bench
# scales it to a full launch (traffic grows with the tiles: rows per tile are
# fixed).  Mostly the lazy-argmin rows (2^(18-K) bytes per traced step).
TRAFFIC_BYTES_PER_WEIGHT_K4 = 26822
WORKLOAD = ("config 2: single dense projection 5120x5120 bf16 ~N(0,0.02^2) + 0.1% x10 "
            "outliers; H = A^T A/4096, A Student-t(4) x lognormal(1) channel scales; "
            "random-sign Hadamard, damped block-LDL, full BlockLDLQ + tail-biting "
            "Viterbi K=4 mul1 (pivot 128, margin 0), pack, W_hat")


def _env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def _measured_peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except OSError:
        return {}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.proc = None
        self.lines = []
        self.t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self, gpus):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.t:
            self.t.join(timeout=2)
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                idx = int(f[0])
            except ValueError:
                continue
            if idx not in gpus:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return None
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def _cpu_sample(Wq, Lfac, lut, nblocks, warm=0, nthreads=None):
    """Time `nblocks` k-blocks of the oracle sweep (after `warm` untimed ones);
    returns (seconds per block list, threads)."""
    from oracle import exl3_oracle as oracle
    nth = nthreads or (os.cpu_count() or 1)
    gen = oracle.ldlq_viterbi_steps(Wq, Lfac, lut, K_BITS, pivot=128, margin=0,
                                    nthreads=nth)
    times = []
    for j in range(warm + nblocks):
        t0 = time.perf_counter()
        next(gen)
        dt = time.perf_counter() - t0
        if j >= warm:
            times.append(dt)
    return times, nth


def _cpu_problem():
    """Config-2 problem prepared by the oracle on the host (untimed)."""
    import numpy as np
    import torch
    from exl3b import synth
    from oracle import exl3_oracle as oracle
    # the same seeded inputs as our arm on a GPU box; on the host without one
    # (the CPU test of this arm) torch's CPU generator gives other values of
    # the same distributions
    W, H = synth.config2(device="cuda" if torch.cuda.is_available() else "cpu")
    W = W.float().cpu().numpy()
    H = H.cpu().numpy()
    lut = oracle.code_lut("exl3_mul1")
    suh = oracle.sign_vec(DIM, 20261011).astype(np.float16)
    svh = oracle.sign_vec(DIM, 20261012).astype(np.float16)
    h = oracle.hadamard128()
    Wi = oracle.to_inner(np.ascontiguousarray(W.T), suh, svh, h)
    Wscale = np.float32(np.sqrt(np.float32(np.mean(Wi.astype(np.float64) ** 2)))) \
        / oracle.lut_rms(lut)
    Wq = (Wi / np.float32(Wscale)).astype(np.float32)
    G = oracle.rotate_hessian(H, suh, h)
    G[np.diag_indices_from(G)] += np.float32(0.01) * np.float32(np.mean(np.diagonal(G)))
    Lfac, _ = oracle.block_LDL(G, 16)
    del torch
    return Wq, Lfac.astype(np.float32), lut


def _workload(args, rank, dev):
    """(label, metric, weights, device inputs, step(inputs, out_device))."""
    from exl3b import api, synth
    if args.config == "c3":
        Ws, H, Ks = synth.config3(device=dev, seed_offset=100 * rank)
        label = ("config 3: fused q/k/v module, q 5120->6144, k/v 5120->1024 bf16 "
                 "~N(0,0.02^2) + outliers, one shared H (4096 heavy-tailed rows), "
                 "K = [5, 7, 7] mul1, one block-LDL + one sweep over the members")
        metric = "trellis-encoded weights/s (Viterbi+LDLQ) at K=[5,7,7]"

        def step(inp, od):
            return api.quantize_linear_fused(inp[0], inp[1], Ks=Ks, device=dev, out_device=od)
        return label, metric, sum(W.numel() for W in Ws), [Ws, H], step, \
            {"k": 5120, "n": [6144, 1024, 1024], "K": Ks}
    if args.config == "c4":
        W, H = synth.config4(device=dev, seed_w=7 + 100 * rank, seed_h=8 + 100 * rank)
        K = args.K
        label = (f"config 4: MLP down projection 17408->5120 bf16 ~N(0,0.015^2) + outliers, "
                 f"H of dim 17408 (4096 heavy-tailed rows), K={K} mul1, pivot 128, margin 0")
        metric = f"trellis-encoded weights/s (Viterbi+LDLQ) at K={K}"

        def step(inp, od):
            return api.quantize_linear(inp[0], inp[1], K=K, device=dev, out_device=od)
        return label, metric, W.numel(), [W, H], step, {"k": 17408, "n": 5120, "K": K}
    if args.dim == DIM:
        W, H = synth.config2(seed_w=1 + 100 * rank, seed_h=2 + 100 * rank, device=dev)
        label = WORKLOAD
    else:
        W = synth.weight(args.dim, args.dim, 0.02, 1 + 100 * rank, dev)
        H = synth.hessian(args.dim, 2 + 100 * rank, dev)
        label = f"{args.dim}x{args.dim} profiling case (not a bench line)"

    def step(inp, od):
        return api.quantize_linear(inp[0], inp[1], K=K_BITS, device=dev, out_device=od)
    return label, METRIC, W.numel(), [W, H], step, {"k": args.dim, "n": args.dim, "K": K_BITS}


def _split_leg(args, dev, world, local, rank, barrier):
    """Per-layer time of ONE projection (the workload's, same seeds on every
    rank) with its output columns split over the N ranks (exl3b.shard: each
    rank transforms W and factors H itself, sweeps its 128-aligned column
    range; the finished trellis and W_hat are NCCL all-gathered inside the
    timed region).  CUDA events, max over ranks.  None for the fused c3
    module (its columns span three segments of different K)."""
    import torch
    import torch.distributed as dist
    from exl3b import shard, synth
    if args.config == "c3" or args.dim != DIM:
        return None
    if args.config == "c4":
        W, H = synth.config4(device=dev)
        K = args.K
    else:
        W, H = synth.config2(device=dev)
        K = K_BITS

    def run():
        return shard.quantize_linear_split(W, H, K=K, out_device=dev)
    for _ in range(max(args.warmup, 1)):
        run()
    barrier()
    s = torch.cuda.current_stream(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(args.steps):
        r = run()
    e1.record(s)
    barrier()
    ms = torch.tensor([e0.elapsed_time(e1) / args.steps], dtype=torch.float64, device=dev)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms.item())
    cols = shard.column_ranges(W.shape[0], world)
    del r
    return {"split": "output columns of one projection, one 128-aligned range per rank; "
                     "each rank transforms W and factors H itself; NCCL all-gather of "
                     "the trellis and W_hat inside the timed region",
            "n_gpus": world, "ms_per_layer": ms, "weights_per_s": W.numel() / (ms / 1e3),
            "columns_per_rank": [b - a for a, b in cols],
            "column_tiles_per_rank": [(b - a) // 16 for a, b in cols]}


def _layer_leg(args, dev, world, barrier):
    """Per-layer time of one 27B-shape layer (config 5: q/k/v, o, gate/up,
    down at the SC5 mixed K = 4..7, seeded synthetic weights and Hessians)
    split over the N ranks (exl3b.stack.quantize_layer_split: channel ranges
    chosen by a per-rank time model, NCCL all-gather of the trellises inside
    the timed region; N = 1: the whole layer on one GPU).  One warm-up layer,
    then layers 1 .. L timed with CUDA events, max over ranks.  Weight and
    Hessian synthesis are inside the time, as they are for the stack driver."""
    import torch
    import torch.distributed as dist
    from exl3b import stack, synth
    if args.config != "c2" or args.dim != DIM or args.no_layer:
        return None
    nl = max(1, min(args.steps, 2))
    stack.quantize_layer_split(0, dev)
    barrier()
    s = torch.cuda.current_stream(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for layer in range(1, nl + 1):
        stack.quantize_layer_split(layer, dev)
    e1.record(s)
    barrier()
    ms = torch.tensor([e0.elapsed_time(e1) / nl], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms.item())
    return {"layer": "27B-shape layer (config 5 shapes, SC5 K: q5 k7 v7 o6 gate5 up5 down4)",
            "split": f"output channels over {world} rank(s), time-model cuts, NCCL all-gather",
            "n_gpus": world, "layers_timed": nl, "seconds_per_layer": ms / 1e3,
            "weights_per_s": synth.stack_weights_per_layer() / (ms / 1e3)}


def _to_host(inp):
    if isinstance(inp, list):
        return [_to_host(x) for x in inp]
    return inp.cpu().pin_memory()


def _nbytes(x):
    if isinstance(x, (list, tuple)):
        return sum(_nbytes(y) for y in x)
    return x.numel() * x.element_size()


def _result_bytes(r):
    if isinstance(r, list):
        return sum(_result_bytes(x) for x in r)
    return sum(r[k].numel() * r[k].element_size() for k in ("W_hat", "trellis", "suh", "svh"))


def _prof(L, kind):
    import ctypes
    from exl3b import native
    ms, n, u = ctypes.c_double(0.0), ctypes.c_longlong(0), ctypes.c_double(0.0)
    native.check("exl3b_profile_end",
                 L.exl3b_profile_end(kind, ctypes.byref(ms), ctypes.byref(n), ctypes.byref(u)))
    return ms.value, n.value, u.value


def _kernels(L, steps, step_ms, sms, peaks):
    """Per-stage roofline from the library's per-launch events (kinds 0, 1, 3, 4)."""
    mhz = float(peaks.get("sm_max_mhz", 1965.0))
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    bf16 = float(peaks.get("bf16_tflops", 1590.0))
    src = "MEASURED_PEAKS.json" if peaks else "fallback"
    out = {}
    specs = [
        (0, "ldlq_tile", "fp32", "Gop/s", lambda u: u * OPS_PER_WEIGHT / 1e9,
         sms * 128 * mhz * 1e6 / 1e9,
         f"{sms} SMs x 128 fp32 lanes x {mhz:.0f} MHz; {FP32_NOTE}"),
        (1, "feedback_gemm_tcgen05", "tensor", "TFLOP/s", lambda u: u / 1e12, bf16 / 2.0,
         f"TF32 dense = bf16 dense / 2 of {src} (useful FLOP; 3xTF32 issues 3 MMAs per "
         "useful product, so frac <= 1/3)"),
        (3, "hadamard_rotation", "hbm", "GB/s", lambda u: u / 1e9, hbm,
         f"HBM copy bandwidth of {src} (algorithmic bytes: read input + write output once)"),
        (4, "block_ldl", "fp32", "TFLOP/s", lambda u: u / 1e12, sms * 256 * mhz * 1e6 / 1e12,
         f"{sms} SMs x 128 FMA lanes x 2 x {mhz:.0f} MHz; k^3/3 FLOP"),
    ]
    for kind, name, bound, unit, conv, peak, note in specs:
        ms, n, u = _prof(L, kind)
        if n == 0:
            continue
        ach = conv(u) / (ms / 1e3) if ms > 0 else None
        out[name] = {"bound": bound, "ms_per_step": ms / steps, "launches_per_step": n / steps,
                     "share_of_step": (ms / steps) / step_ms if step_ms else None,
                     "achieved": ach, "peak": peak, "unit": unit,
                     "frac": (ach / peak) if ach is not None else None, "peak_source": note}
    return out


def run_reference(args, rank):
    if rank != 0:
        return 0
    Wq, Lfac, lut = _cpu_problem()
    times, nth = _cpu_sample(Wq, Lfac, lut, args.steps, warm=args.warmup)
    per_block_w = (DIM // 16) * 256
    t = sum(times) / len(times)
    v = per_block_w / t
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": t * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "k": DIM, "n": DIM, "K": K_BITS,
                   "step": "one k-block launch (320 tiles) of the sweep"},
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": nth, "kind": "port",
                         "sample": f"{args.steps} consecutive k-blocks (320 tiles each, "
                                   "right to left) of the config-2 LDLQ sweep after "
                                   f"{args.warmup} warm-up blocks; one-off rotation and "
                                   "LDL excluded (<1% of the CPU time)"},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    _emit(line)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer e2e leg")
    ap.add_argument("--no-layer", action="store_true",
                    help="skip the per-layer leg of one config-5 layer split over the ranks")
    ap.add_argument("--config", default="c2", choices=["c2", "c3", "c4"],
                    help="workload: c2 (default bench line), c3 fused mixed-K qkv, c4 at --K")
    ap.add_argument("--K", type=int, default=4, help="bits per weight for --config c4")
    ap.add_argument("--dim", type=int, default=DIM,
                    help="projection size (default 5120 = config 2; smaller sizes are "
                         "for profiler captures, not bench lines)")
    args = ap.parse_args()
    rank = _env_int("RANK", 0)
    world = _env_int("WORLD_SIZE", 1)
    local = _env_int("LOCAL_RANK", 0)
    if args.impl == "reference":
        return run_reference(args, rank)

    import torch
    import torch.distributed as dist
    from datetime import timedelta
    from exl3b import native

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=dev)
    L = native.lib()

    label, metric, weights, inputs, run_step, shape = _workload(args, rank, dev)
    torch.cuda.synchronize()

    def step():
        return run_step(inputs, dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step()
    barrier()

    sampler = ClockSampler() if rank == 0 else None
    if sampler:
        sampler.start()
    s = torch.cuda.current_stream(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    n0 = L.exl3b_launch_count()
    L.exl3b_profile_begin()
    barrier()
    e0.record(s)
    for _ in range(args.steps):
        r = step()
    e1.record(s)
    barrier()
    clocks = sampler.stop(set(range(max(world, 1)))) if sampler else None
    launches = (L.exl3b_launch_count() - n0) // args.steps
    ms = e0.elapsed_time(e1) / args.steps
    peaks = _measured_peaks()
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    kernels = _kernels(L, args.steps, ms, sms, peaks)
    ms_tile, n_tile, u_tile = _prof(L, 0)
    t_max = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
    ms = float(t_max.item())
    value = world * weights / (ms / 1e3)
    # per-layer time with one projection split over the ranks (N = 1: the
    # step itself, one whole projection on one GPU)
    per_layer = _split_leg(args, dev, world, local, rank, barrier) if world > 1 else None
    layer_c5 = _layer_leg(args, dev, world, barrier)

    # ---- e2e: public API from pinned host buffers, copies inside the step
    ms_e2e = float("nan")
    h2d = d2h = 0
    del r
    if not args.no_e2e:
        host = _to_host(inputs)
        # the same W warm-up steps as the resident leg; holding each result
        # while the next step runs, like the timed loop, also lets the pinned
        # host allocator settle on its two result buffers before timing
        rr = None
        for _ in range(max(args.warmup, 1)):
            rr = run_step(host, "cpu")
        barrier()
        e2 = torch.cuda.Event(enable_timing=True)
        e3 = torch.cuda.Event(enable_timing=True)
        e2.record(s)
        for _ in range(args.steps):
            rr = run_step(host, "cpu")
        e3.record(s)
        barrier()
        ms_e2e = e2.elapsed_time(e3) / args.steps
        h2d = _nbytes(host)
        d2h = _result_bytes(rr)
        del rr
    t2 = torch.tensor([ms_e2e], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t2, op=dist.ReduceOp.MAX)
    ms_e2e = float(t2.item())

    # ---- roofline of the dominant kernel (fused LDLQ tile kernel)
    mhz = float(peaks.get("sm_max_mhz", 1965.0))
    peak_ops = sms * 128 * mhz * 1e6 / 1e9           # Gop/s
    tile_ms_avg = ms_tile / max(n_tile, 1)
    w_per_launch = u_tile / max(n_tile, 1)
    achieved = w_per_launch * OPS_PER_WEIGHT / (tile_ms_avg / 1e3) / 1e9
    floor_achieved = w_per_launch * FLOOR_OPS_PER_WEIGHT / (tile_ms_avg / 1e3) / 1e9
    tpw = TRAFFIC_BYTES_PER_WEIGHT_K4 if shape.get("K") == 4 else None
    roofline = {
        "kernel": "LDLQ tile kernel (fused feedback + tail-biting Viterbi + write-back; "
                  "ldlq_lazy_kernel for launches of >= 2 tiles per SM; ldlq_solo_kernel where the "
                  "column tiles do not fill the SMs)",
        "bound": "fp32", "achieved": achieved, "peak": peak_ops, "unit": "Gop/s",
        "frac": achieved / peak_ops,
        "peak_source": f"{sms} SMs x 128 fp32 lanes x {mhz:.0f} MHz (sm_max_mhz of "
                       f"MEASURED_PEAKS.json); {FP32_NOTE}",
        "ops_per_weight": OPS_PER_WEIGHT,
        "frac_fp32_floor": floor_achieved / peak_ops,
        "fp32_floor_note": "3 correctly rounded fp32 ops per add-compare-select "
                           "(393216 per weight), the least a bit-exact encoder executes",
        "launches_per_step": n_tile / args.steps,
        "avg_launch_ms": tile_ms_avg,
        "share_of_step": ms_tile / args.steps / ms if ms else None,
        "traffic": (tpw * w_per_launch) if tpw else None,
        "traffic_unit": "bytes per launch (ncu DRAM bytes per weight of the 2048^2 "
                        "profiling launch x weights per launch)",
        "algorithmic_bytes_per_launch": w_per_launch * 2 * 2 ** (16 - shape["K"]) *
                                        shape["K"] / 8 if isinstance(shape.get("K"), int)
                                        else None,
    }

    in_bytes = _nbytes(inputs)
    config = {"workload": label, **shape,
              "per_rank": "one independent problem per rank (seeds offset by 100 r)",
              "l2": f"inputs larger than L2 ({in_bytes / 1e6:.0f} MB of W and H per step, "
                    "plus the sweep's intermediates)",
              "parallelism": f"{world} independent ranks"}
    if args.config != "c2":
        config["config"] = args.config
    line = {
        "metric": metric, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": config,
        "e2e": {"value": world * weights / (ms_e2e / 1e3), "unit": UNIT,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": ms_e2e},
        "gpu_launches": int(launches),
        "roofline": roofline,
        "kernels": kernels,
        "clocks": clocks,
        "per_layer_s": (per_layer["ms_per_layer"] / 1e3) if per_layer else ms / 1e3,
        "per_layer": per_layer if per_layer else {
            "split": "none: one whole projection per GPU (N = 1, or a fused module)",
            "n_gpus": world, "ms_per_layer": ms, "weights_per_s": weights / (ms / 1e3)},
    }
    if layer_c5 is not None:
        line["per_layer_c5"] = layer_c5
    if world > 1:
        dist.barrier(device_ids=[local])
    if (rank == 0 and world == 1 and not args.no_cpu_baseline and args.dim == DIM
            and args.config == "c2"):
        Wq, Lfac, lut = _cpu_problem()
        times, nth = _cpu_sample(Wq, Lfac, lut, 2, warm=1)
        t = sum(times) / len(times)
        line["cpu_baseline"] = {
            "value": (DIM // 16) * 256 / t, "unit": UNIT, "cores": nth, "kind": "port",
            "sample": "2 k-blocks (320 tiles each) of the config-2 LDLQ sweep after 1 "
                      "warm-up block, oracle C/numpy restatement, all host threads; "
                      "one-off rotation and LDL excluded (<1% of CPU time)"}
    if rank == 0:
        _emit(line)
    if world > 1:
        dist.destroy_process_group()
    return 0


def _stdout_for_json() -> int:
    """Keep stdout for the one JSON line: duplicate the real stdout and point
    file descriptor 1 at stderr, so that whatever the native libraries write
    there (NCCL's version banner at communicator set-up, library logs) lands
    on stderr.  Returns the duplicated descriptor."""
    sys.stdout.flush()
    fd = os.dup(1)
    os.dup2(2, 1)
    return fd


_JSON_FD = None


def _emit(line: dict):
    data = (json.dumps(line) + "\n").encode()
    if _JSON_FD is None:
        sys.stdout.write(data.decode())
        sys.stdout.flush()
    else:
        os.write(_JSON_FD, data)


if __name__ == "__main__":
    _JSON_FD = _stdout_for_json()
    sys.exit(main())
