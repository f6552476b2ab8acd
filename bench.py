"""Benchmark of the B200 GEMM engine: one JSON line on rank 0.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl kl|reference] [--workload NAME]

A step is one GEMM over the workload's operands. The default workload is the 8192^3 bf16 GEMM
(N(0,1)*0.02 inputs, seed 2), sharded along N over the ranks: rank r owns B rows
[r*N/g, (r+1)*N/g) and produces C[:, shard] (no collective on the data path); `value` is the
whole-job TFLOP/s, the total flops over the max-over-ranks device time. The operands (268 MB)
exceed the 126 MB L2, so no flush runs between steps.

  value      device time of K kl_gemm launches on resident inputs (CUDA events on the stream).
  e2e        the same through the public host-buffer API (kl_gemm_host): every step copies A and B
             in from pinned host memory and C back out, overlapped with the GEMM in column blocks.
  roofline   the GEMM kernel's achieved TFLOP/s against the measured dense bf16 (or fp8) peak.
  cpu_baseline  the CPU GEMM (fp32 accumulate, all host threads) on a bounded row slab.
  workloads  the other two targets on the same line: the fp8 GEMM (16384 x 16384 x 8192 e4m3,
             per-tensor scales, N-sharded like the headline) against twice the measured bf16
             peak, and (one GPU) the decode shapes M = 16 / 64 / 128, N = 28672, K = 8192 bf16
             against the measured copy bandwidth. Their operands are drawn on the device
             (torch's generator, the same distributions and seeds as the workload definitions).
  gather_check  (N > 1) the fused gather's full C compared bit for bit with the NCCL-gathered C.
`--impl reference` times only the reference arm: the CPU GEMM restatement (the reference ships no
GEMM of its own), rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

DEFAULT_WORKLOAD = "c3_8192_bf16"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


class ClockSampler:
    """SM clock and throttle reasons sampled through NVML (what nvidia-smi reads) every ~2 ms in a
    background thread while the timed region runs, so even a short region gets samples."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4}

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self.max_mhz = None
        self._stop = None

    def __enter__(self):
        import threading

        if self.index is None:  # sampling off
            return self
        try:
            import pynvml

            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            get_reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
        except Exception:
            return self
        self._stop = threading.Event()

        def run():
            while not self._stop.is_set():
                try:
                    mhz = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                    reasons = get_reasons(h)
                    self.samples.append((float(mhz), int(reasons)))
                except Exception:
                    pass
                self._stop.wait(0.0005)

        self._thread = threading.Thread(target=run, daemon=True)
        self._thread.start()
        time.sleep(0.01)
        return self

    def __exit__(self, *exc):
        if self._stop is not None:
            self._stop.set()
            self._thread.join(timeout=2)

    def summary(self):
        sm = [m for m, _ in self.samples]
        reasons = sorted({name for _, r in self.samples for name, bit in self.REASONS.items() if r & bit})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz, "reasons": reasons,
                "samples": len(sm), "source": "NVML (nvidia-smi's clocks.sm and clocks_event_reasons)"}


def cpu_baseline(w, budget_s: float = 6.0):
    """fp32-accumulate CPU GEMM on a row slab of A, doubled until it takes >= budget_s / 3."""
    from maia_b200 import workloads as wl
    from oracle import gemm as og

    threads = og.threads_default()
    rows = 16
    while True:
        a, b, sa, sb = wl.make_inputs(w, rows_a=rows)
        t0 = time.perf_counter()
        if w.dtype == "nvfp4":
            og.gemm_nv_f32(a, b, sa[0], sb[0], sa[1] * sb[1], threads=threads)
        elif w.dtype in wl.MX_ELEMENT:
            og.gemm_mx_f32(a, b, sa, sb, wl.MX_ELEMENT[w.dtype], threads=threads)
        else:
            og.gemm_f32(a, b, sa * sb, threads=threads)
        dt = time.perf_counter() - t0
        if dt >= budget_s / 3 or rows >= w.m:
            break
        rows = min(w.m, rows * 2 if dt > 0.05 else rows * 8)
    tflops = 2.0 * rows * w.n * w.k / dt / 1e12
    return {"value": tflops, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"rows [0,{rows}) of A x all of B ({rows}x{w.n}x{w.k}, {w.dtype}, fp32 accumulate), {dt:.2f} s"}


METRIC = "GEMM TFLOP/s per B200 and % of tcgen05 dense peak"


def timed(fn, steps: int, warmup: int, stream, device, sync, settle_s: float = 0.0, sample_clocks: bool = True):
    """Device time per call of fn (CUDA events on `stream`, after `warmup` untimed calls), with the
    NVML clock samples taken meanwhile. settle_s: an idle pause first, so that a workload does not
    start in the power state the previous one left. sample_clocks=False leaves the sampling thread
    out: a step that queues many small launches from Python (the NCCL gather path) is host-bound,
    and a thread polling NVML in every rank's process slows that host work down."""
    import torch

    if settle_s > 0:
        sync()
        time.sleep(settle_s)
    for _ in range(max(warmup, 3)):
        fn()
    sync()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device.index if sample_clocks else None) as clocks:
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        sync()
    return e0.elapsed_time(e1) / steps, clocks.summary()


def extra_workloads(world, rank, dev, dist, peaks, peak_src, sync, max_over_ranks):
    """The fp8 GEMM (every rank, N-sharded) and the decode shapes (rank 0 of a one-GPU run) on
    device-drawn operands; one entry each for the JSON line's `workloads`."""
    import torch

    import maia_b200 as kl
    from maia_b200 import sharding
    from maia_b200 import workloads as wl

    out = {}
    stream = torch.cuda.current_stream(dev)

    def normal(rows, cols, seed, scale):
        g = torch.Generator(device=dev).manual_seed(seed)
        x = torch.randn((rows, cols), generator=g, device=dev, dtype=torch.float32)
        return x.mul_(scale) if scale != 1.0 else x

    if world == 1:
        # Decode shapes: weights N(0,1) * 0.02, activations N(0,1), bf16 in and out; the skinny
        # kernel or the one-CTA tile kernel, whichever KL_ALGO_AUTO picks (the library default).
        w0 = wl.C5[16]
        wgt = normal(w0.n, w0.k, w0.seed * 1000 + 1, w0.b_scale).to(torch.bfloat16)
        for m, w in wl.C5.items():
            x = normal(m, w.k, w.seed * 1000 + 0, w.a_scale).to(torch.bfloat16)
            y = torch.empty((m, w.n), dtype=torch.bfloat16, device=dev)
            # Two activation buffers taken in turn (the second a copy of the first), so that no step
            # finds its activations in L2 from the step before; the weights (470 MB) exceed L2 anyway.
            x2, y2 = x.clone(), torch.empty_like(y)
            launches = [kl.gemm_launcher(x, wgt, y), kl.gemm_launcher(x2, wgt, y2)]
            turn = [0]

            def decode_step():
                launches[turn[0]]()
                turn[0] ^= 1

            steps = 300
            ms, clocks = timed(decode_step, steps, 10, stream, dev, sync, settle_s=1.0)
            if kl.read_status() != 0:
                raise RuntimeError("a device-side wait timed out in the decode workload")
            alg = (m * w.k + w.n * w.k) * 2 + m * w.n * 2
            achieved = alg / (ms * 1e-3) / 1e9
            out[w.name] = {
                "value": achieved, "unit": "GB/s", "ms_per_step": ms, "steps": steps, "warmup": 10, "n_gpus": 1,
                "dtype": "bf16", "tflops": w.flops / (ms * 1e-3) / 1e12,
                "route": {kl.ALGO_SKINNY: "skinny", kl.ALGO_1CTA: "one-CTA tile kernel",
                          kl.ALGO_2CTA: "CTA-pair tile kernel"}[kl.resolve_algo(x, wgt, y)],
                "data": "weights N(0,1)*0.02, activations N(0,1), drawn on the device (seeds 4001 / 4000)",
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                             "frac": achieved / peaks["hbm_gbs"], "peak_source": f"{peak_src} hbm_gbs",
                             "algorithmic_bytes_per_launch": alg},
                "clocks": clocks,
                "gpu_launches": steps,
                "l2": "weights (470 MB) exceed L2 (no flush); two activation buffers in turn", "settle_s": 1.0,
            }
        del wgt
        torch.cuda.empty_cache()
    # fp8 e4m3, per-tensor scales amax / 448, scale_a * scale_b applied in the epilogue, bf16 C.
    w = wl.C4
    n_lo, n_hi = sharding.shard_range(w.n, world, rank, align=256)
    xa = normal(w.m, w.k, w.seed * 1000 + 0, w.a_scale)
    sa = xa.abs().max() / 448.0
    a = (xa / sa).to(torch.float8_e4m3fn)
    del xa
    xb = normal(w.n, w.k, w.seed * 1000 + 1, w.b_scale)
    sb = xb.abs().max() / 448.0
    b = (xb[n_lo:n_hi] / sb).to(torch.float8_e4m3fn)
    del xb
    scale_a = sa.reshape(1).float()
    scale_b = sb.reshape(1).float()
    c = torch.empty((w.m, n_hi - n_lo), dtype=torch.bfloat16, device=dev)
    steps = 40
    ms, clocks = timed(kl.gemm_launcher(a, b, c, scale_a=scale_a, scale_b=scale_b), steps, 3, stream, dev, sync,
                       settle_s=1.0)
    in_kernel = kl.clock_probe(a, b, c, scale_a=scale_a, scale_b=scale_b)
    if kl.read_status() != 0:
        raise RuntimeError("a device-side wait timed out in the fp8 workload")
    ms_all = max_over_ranks(ms)
    per_rank = 2.0 * w.m * (n_hi - n_lo) * w.k
    achieved = per_rank / (ms * 1e-3) / 1e12
    peak = 2.0 * peaks["bf16_tflops"]
    out[w.name] = {
        "value": w.flops / (ms_all * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms_all, "steps": steps,
        "warmup": 3, "n_gpus": world, "dtype": "e4m3", "out": "bf16",
        "data": "N(0,1) drawn on the device (torch generator, seeds 3000 / 3001), per-tensor amax/448 scales",
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                     "peak_source": f"{peak_src} 2 x bf16_tflops (burst; the dense fp8 rate is twice bf16)",
                     "algorithmic_flops_per_launch": per_rank},
        "clocks": dict(clocks, in_kernel=in_kernel),
        "gpu_launches": steps, "settle_s": 1.0,
    }
    del a, b, c
    torch.cuda.empty_cache()

    return out


def config_of(w, args, world):
    """The `config` both arms report: the workload and the launch knobs."""
    par = f"N-sharded x{world}" if not getattr(args, "shard_of", 0) else f"shard 0 of {args.shard_of} on one GPU"
    return {"workload": w.name, "m": w.m, "n": w.n, "k": w.k, "out": w.out,
            "parallelism": par, "output": "C[:, shard] per rank (no gather)",
            "l2": "operands exceed L2 (no flush)", "algo": args.algo, "group_m": args.group_m,
            "prefetch": args.prefetch, "variant": args.variant, "max_ctas": args.max_ctas, "stream_k": args.stream_k}


def run_reference(args, w):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    base = None
    vals = []
    for i in range(args.warmup + args.steps):
        r = cpu_baseline(w, budget_s=3.0)
        if i >= args.warmup:
            vals.append(r["value"])
            base = r
    v = statistics.median(vals)
    base["value"] = v
    # The same metric, unit and config as the kl arm; what is timed is the CPU reference GEMM
    # (the oracle's fp32 restatement) on a row slab, as `cpu_baseline.sample` says.
    line = {"metric": METRIC, "value": v, "unit": "TFLOP/s",
            "impl": "reference", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 2.0 * w.m * w.n * w.k / (v * 1e12) * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": w.dtype, "data": "synthetic",
            "config": config_of(w, args, args.gpus), "cpu_baseline": base,
            "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["kl", "reference"], default="kl")
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD)
    ap.add_argument("--algo", type=int, default=0, help="kl_algo (0 = library default)")
    ap.add_argument("--group-m", type=int, default=0)
    ap.add_argument("--prefetch", type=int, default=0, help="L2 prefetch distance (0 = library default, -1 = off)")
    ap.add_argument("--variant", type=int, default=0, help="kl_gemm_desc.variant (0 = library default)")
    ap.add_argument("--max-ctas", type=int, default=0, help="cap on resident CTAs (0 = library default)")
    ap.add_argument("--chunks", type=int, default=0, help="e2e column blocks of kl_gemm_host (0 = library default)")
    ap.add_argument("--stream-k", type=int, default=0, choices=[-1, 0, 1],
                    help="tile kernels' split tail: 0 = library default, 1 = always, -1 = whole tiles")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--shard-of", type=int, default=0,
                    help="one GPU only: time the first column shard of a G-way N-split (the GEMM one rank of "
                         "G runs), for profiling the sharded kernel without a multi-rank launch")
    ap.add_argument("--no-extra-workloads", action="store_true",
                    help="skip the fp8 and decode entries of `workloads` (run by default with the headline workload)")
    args = ap.parse_args()

    from maia_b200 import workloads as wl

    w = wl.ALL[args.workload]
    if args.impl == "reference":
        return run_reference(args, w)

    import numpy as np
    import torch

    import maia_b200 as kl

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    # Inputs: full A, this rank's N-shard of B (host-generated, seeded, then pinned).
    from maia_b200 import sharding

    a_bits, b_bits, sa, sb = wl.make_inputs(w)
    split = world
    if args.shard_of > 0:
        if world != 1:
            raise SystemExit("--shard-of runs on one GPU")
        split = args.shard_of
    n_lo, n_hi = sharding.shard_range(w.n, split, rank, align=256)
    b_bits = np.ascontiguousarray(b_bits[n_lo:n_hi])
    mx = w.dtype in ("mxfp8", "mxfp6", "mxfp4", "nvfp4")
    vec = 16 if w.dtype == "nvfp4" else 32
    gscale = None
    if w.dtype == "nvfp4":  # (block scales, per-tensor scale) pairs
        (sa, ga), (sb, gb) = sa, sb
        gscale = (ga, gb)
    if mx:
        sb = np.ascontiguousarray(sb[n_lo:n_hi])
    nshard = n_hi - n_lo
    np_view = np.int16 if w.dtype == "bf16" else np.uint8
    # Packed fp6 has no torch dtype: its bytes travel as uint8 with ab_type naming the format.
    tdt = {"bf16": torch.bfloat16, "mxfp4": torch.float4_e2m1fn_x2, "nvfp4": torch.float4_e2m1fn_x2,
           "mxfp6": torch.uint8}.get(w.dtype, torch.float8_e4m3fn)
    odt = torch.bfloat16 if w.out == "bf16" else torch.float32
    a_host = torch.from_numpy(a_bits.view(np_view)).view(tdt).pin_memory()
    b_host = torch.from_numpy(b_bits.view(np_view)).view(tdt).pin_memory()
    del a_bits, b_bits
    a = a_host.to(dev)
    b = b_host.to(dev)
    c = torch.empty((w.m, nshard), dtype=odt, device=dev)
    c_host = torch.empty((w.m, nshard), dtype=odt).pin_memory()
    scale_a = scale_b = None
    sfa = sfb = sfa_host = sfb_host = None
    if w.dtype == "e4m3":
        scale_a = torch.tensor([sa], dtype=torch.float32, device=dev)
        scale_b = torch.tensor([sb], dtype=torch.float32, device=dev)
    if gscale is not None:
        scale_a = torch.tensor([gscale[0]], dtype=torch.float32, device=dev)
        scale_b = torch.tensor([gscale[1]], dtype=torch.float32, device=dev)
    if mx:
        # Block scales, repacked on the device into the blocked layout (untimed setup).
        sfa = kl.pack_block_scales(torch.from_numpy(sa).to(dev), w.k, vec)
        sfb = kl.pack_block_scales(torch.from_numpy(sb).to(dev), w.k, vec)
        sfa_host = sfa.cpu().pin_memory()
        sfb_host = sfb.cpu().pin_memory()
    stream = torch.cuda.current_stream(dev)
    kw = dict(scale_a=scale_a, scale_b=scale_b, algo=args.algo, group_m=args.group_m, prefetch=args.prefetch,
              variant=args.variant, max_ctas=args.max_ctas, sfa=sfa, sfb=sfb, scale_vec=vec,
              ab_type=wl.MX_ELEMENT[w.dtype] if w.dtype == "mxfp6" else None, stream_k=args.stream_k)

    step = kl.gemm_launcher(a, b, c, **kw)  # one kl_gemm per call, the descriptor built once
    # The kernel the launches run: its family and C tile (kl_gemm_resolve_algo / _tile).
    route = {kl.ALGO_SKINNY: "skinny (stream-K)", kl.ALGO_1CTA: "one CTA", kl.ALGO_2CTA: "CTA pair"}[
        kl.resolve_algo(a, b, c, **kw)]
    tile_m, tile_n = kl.resolve_tile(a, b, c, **kw)
    kernel = f"{route}, {tile_m} x {tile_n} tiles" if tile_m else route

    def barrier():
        torch.cuda.synchronize(dev)
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def max_over_ranks(x: float) -> float:
        return sharding.max_over_ranks(x, dist, dev)

    # ---- device-resident timing
    for _ in range(max(args.warmup, 3)):
        step()
    kl.read_status()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        barrier()
    dev_ms = ev0.elapsed_time(ev1) / args.steps
    in_kernel = None
    if w.m > 256 and args.algo in (0, kl.ALGO_1CTA, kl.ALGO_2CTA):
        # One more launch, right after the timed ones, with every CTA stamping clock64 and
        # %globaltimer: the SM clock the kernel really ran at (NVML may report the boost target).
        in_kernel = kl.clock_probe(a, b, c, scale_a=scale_a, scale_b=scale_b, algo=args.algo, group_m=args.group_m,
                                   sfa=sfa, sfb=sfb, scale_vec=vec, ab_type=kw["ab_type"])
    if kl.read_status() != 0:
        raise RuntimeError("a device-side wait timed out during the benchmark")
    dev_ms = max_over_ranks(dev_ms)
    flops_total = 2.0 * w.m * (w.n if split == world else n_hi - n_lo) * w.k
    value = flops_total / (dev_ms * 1e-3) / 1e12

    # ---- N > 1: the same GEMM followed by the NCCL all-gather of C (where the full C is needed). The
    # gather legs run before the end-to-end leg, whose NCCL all-gather of A runs on a side stream.
    gather = None
    gather_check = None
    if dist is not None:
        # Buffers of the NCCL path made once, so that a step queues the GEMM, the collective and one
        # re-layout copy, and allocates nothing.
        g_out = torch.empty((w.m, w.n), dtype=odt, device=dev)
        g_work = torch.empty((world, w.m, max(sharding.shard_range(w.n, world, r, align=256)[1] -
                                              sharding.shard_range(w.n, world, r, align=256)[0]
                                              for r in range(world))), dtype=odt, device=dev)

        def gather_step():
            step()
            sharding.gather_columns(c, w.n, dist, align=256, out=g_out, work=g_work)

        for _ in range(max(args.warmup, 3)):
            gather_step()
        barrier()
        # The gather legs are short (0.1-0.6 ms a step): at least 50 timed steps each, back to back after
        # their own warm-up (they are reported beside `value`, not as it).
        g_steps = max(args.steps, 50)
        g_ms, _ = timed(gather_step, g_steps, 0, stream, dev, barrier, sample_clocks=False)
        g_ms = max_over_ranks(g_ms)
        gather = {"value": flops_total / (g_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": g_ms,
                  "what": "kl_gemm + NCCL all-gather of C and re-layout to [M, N] on every rank (buffers made once)",
                  "steps": g_steps}

        # The same result with the gather fused into the GEMM: every tile is also TMA-stored into
        # the other ranks' copies of C over NVLink (kl_gemm_gather).
        shared = sharding.SharedC(w.m, w.n, odt, dev, dist)
        c_view = shared.full[:, n_lo:n_hi]
        peers = shared.peer_ptrs(n_lo)

        def fused_step():
            kl.gemm_gather(a, b, c_view, peers, scale_a=scale_a, scale_b=scale_b, algo=args.algo, sfa=sfa, sfb=sfb,
                           scale_vec=vec, stream_k=args.stream_k)

        for _ in range(max(args.warmup, 3)):
            fused_step()
        barrier()
        f_ms, _ = timed(fused_step, g_steps, 0, stream, dev, barrier, sample_clocks=False)
        f_ms = max_over_ranks(f_ms)
        gather["fused"] = {"value": flops_total / (f_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": f_ms,
                           "what": "kl_gemm_gather: tiles stored to every rank's C by the GEMM epilogue (P2P over NVLink)",
                           "steps": g_steps}
        # Outside the timed region: every rank's kernels have finished (barrier), so its copy of the
        # full C is complete. Compare it with the NCCL-gathered C of the plain GEMM, bit for bit (the
        # same kernel and schedule produce both), on every rank.
        barrier()
        kl.gemm(a, b, c, **kw)
        want = sharding.gather_columns(c, w.n, dist, align=256)
        torch.cuda.synchronize(dev)
        bits = torch.int16 if odt == torch.bfloat16 else torch.int32
        same = torch.equal(shared.full.view(bits), want.view(bits))
        diff = (shared.full.float() - want.float()).abs().max() / want.float().abs().max().clamp_min(1e-30)
        flags = torch.tensor([1.0 if same else 0.0, float(diff)], dtype=torch.float64, device=dev)
        lo = flags[:1].clone()
        dist.all_reduce(lo, op=dist.ReduceOp.MIN)
        hi = flags[1:].clone()
        dist.all_reduce(hi, op=dist.ReduceOp.MAX)
        gather_check = {"fused_vs_nccl_bitexact": bool(lo.item() == 1.0), "max_rel_diff": float(hi.item()),
                        "ranks": world}
        barrier()
        shared.close()

        # The same through an NVLink multicast object: each tile stored once, the switch delivering it
        # to every rank's C (kl_gemm_gather_multicast).
        mcc = sharding.MulticastC(w.m, w.n, odt, dev, dist)
        mc_bad = None
        if mcc.available:
            mc_view = mcc.full[:, n_lo:n_hi]
            mc_addr = mcc.mc_ptr(n_lo)

            def mc_step():
                kl.gemm_gather_multicast(a, b, mc_view, mc_addr, scale_a=scale_a, scale_b=scale_b, algo=args.algo,
                                         sfa=sfa, sfb=sfb, scale_vec=vec, stream_k=args.stream_k)

            m_ms, _ = timed(mc_step, g_steps, args.warmup, stream, dev, barrier, sample_clocks=False)
            m_ms = max_over_ranks(m_ms)
            barrier()
            same = torch.equal(mcc.full.view(bits), want.view(bits))
            mdiff = float((mcc.full.float() - want.float()).abs().max() / want.float().abs().max().clamp_min(1e-30))
            flags = torch.tensor([1.0 if same else 0.0], dtype=torch.float64, device=dev)
            dist.all_reduce(flags, op=dist.ReduceOp.MIN)
            md = torch.tensor([mdiff], dtype=torch.float64, device=dev)
            dist.all_reduce(md, op=dist.ReduceOp.MAX)
            gather_check["multicast_vs_nccl_bitexact"] = bool(flags.item() == 1.0)
            gather_check["multicast_max_rel_diff"] = float(md.item())
            mc_bad = float(md.item()) > 1e-2
            gather["multicast"] = {"value": flops_total / (m_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": m_ms,
                                   "what": "kl_gemm_gather_multicast: each tile stored once through an NVLink "
                                           "multicast address (multimem.st), the switch writing every rank's C",
                                   "steps": g_steps}
        else:
            gather["multicast"] = {"unavailable": mcc.reason}
        mcc.close()
        del want, g_out, g_work
        barrier()
        if float(hi.item()) > 1e-2 or mc_bad:
            raise RuntimeError(f"a fused gather's C differs from the NCCL-gathered C: {gather_check}")

    # ---- end to end through the public API with host buffers
    d2h = c.numel() * c.element_size()
    e2e_how = "kl_gemm_host: all of A and this rank's B copied in, C's block copied out, pipelined over column blocks"
    if dist is not None and not mx:
        # Each rank copies only its slab of A's rows in and the ranks all-gather A over NVLink, while
        # the B shard streams in (sharding.HostShardedGemm over kl_gemm_host_b).
        hs = sharding.HostShardedGemm(w.m, nshard, w.k, tdt, odt, dev, dist)
        s_lo, s_hi = hs.slab_rows()
        a_slab_host = a_host[s_lo:s_hi]
        h2d = a_slab_host.numel() * a_slab_host.element_size() + b_host.numel() * b_host.element_size()
        e2e_how = ("sharding.HostShardedGemm: this rank's slab of A's rows copied in and all-gathered over NVLink "
                   "(NCCL), B's shard streamed in and C's block out through kl_gemm_host_b")

        def e2e_step():
            hs(a_slab_host, b_host, c_host, scale_a=scale_a, scale_b=scale_b, algo=args.algo, chunks=args.chunks,
               stream_k=args.stream_k)
    else:
        h2d = a_host.numel() * a_host.element_size() + b_host.numel() * b_host.element_size()
        if mx:
            h2d += sfa_host.numel() + sfb_host.numel()

        def e2e_step():
            # The host-buffer entry point: copies in, GEMM and copy out, pipelined over column blocks.
            kl.gemm_host(a_host, b_host, c_host, a, b, c, scale_a=scale_a, scale_b=scale_b, algo=args.algo,
                         sfa=sfa_host, sfb=sfb_host, scale_vec=vec, chunks=args.chunks, ab_type=kw["ab_type"],
                         stream_k=args.stream_k)

    for _ in range(max(args.warmup, 3)):
        e2e_step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    # Outside the timed region: the host-side C of the last step against the device-resident GEMM's C
    # (column blocks may split the tail differently, so agreement is to fp32 rounding, not bits).
    if not mx:
        step()
        torch.cuda.synchronize(dev)
        ref_c = c.float()
        e2e_diff = float((c_host.to(dev).float() - ref_c).abs().max() / ref_c.abs().max().clamp_min(1e-30))
        if e2e_diff > 1e-2:
            raise RuntimeError(f"the host-buffer path's C differs from the device GEMM's: {e2e_diff:.3e}")
        del ref_c
    else:
        e2e_diff = None

    peaks, peak_src = load_peaks()
    extra = None
    if args.workload == DEFAULT_WORKLOAD and not args.no_extra_workloads and not args.shard_of:
        del a, b
        torch.cuda.empty_cache()
        extra = extra_workloads(world, rank, dev, dist, peaks, peak_src, barrier, max_over_ranks)
    per_rank_flops = 2.0 * w.m * nshard * w.k
    memory_bound = w.m <= 256
    if memory_bound:
        # Decode shapes: every operand byte moved once, against the measured copy bandwidth.
        alg_bytes = int((w.m * w.k + nshard * w.k) * w.in_bytes) + w.m * nshard * w.out_bytes + \
            (w.m + nshard) * -(-w.k // vec) * mx
        roofline = {"bound": "hbm", "achieved": alg_bytes / (dev_ms * 1e-3) / 1e9, "peak": peaks["hbm_gbs"],
                    "unit": "GB/s", "peak_source": f"{peak_src} hbm_gbs", "algorithmic_bytes_per_launch": alg_bytes}
    else:
        peak = peaks["bf16_tflops"] * {"bf16": 1.0, "mxfp4": 4.0, "nvfp4": 4.0}.get(w.dtype, 2.0)
        roofline = {"bound": "tensor", "achieved": per_rank_flops / (dev_ms * 1e-3) / 1e12, "peak": peak,
                    "unit": "TFLOP/s",
                    "peak_source": f"{peak_src} " + ("bf16_tflops (burst)" if w.dtype == "bf16" else
                                                     "4 x bf16_tflops (burst; the dense fp4 rate is four times bf16)"
                                                     if w.dtype in ("mxfp4", "nvfp4") else
                                                     "2 x bf16_tflops (burst; the fp8, MXFP8 and MXFP6 dense "
                                                     "rate is twice bf16)"),
                    "algorithmic_flops_per_launch": per_rank_flops}
    roofline["frac"] = roofline["achieved"] / roofline["peak"]
    traffic = None
    tf = ROOT / "profiles" / f"traffic_{w.name}.json"
    if tf.exists() and world == 1:
        traffic = json.loads(tf.read_text()).get("dram_bytes_per_launch")
    roofline["traffic"] = traffic

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": dev_ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": w.dtype, "data": "synthetic",
            "config": dict(config_of(w, args, world), kernel=kernel),
            "e2e": {"value": flops_total / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms, "what": e2e_how,
                    "max_rel_diff_vs_device": e2e_diff},
            "roofline": roofline,
            "gpu_launches": args.steps,
            "gemm_plus_allgather": gather,
            "gather_check": gather_check,
            "clocks": dict(clocks.summary(), in_kernel=in_kernel),
            "workloads": extra,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(w)
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
