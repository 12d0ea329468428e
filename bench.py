"""MonarchAttention forward benchmark (B200).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME]
                    [--impl ours|reference]

One step = one MonarchAttention forward over the configuration's whole batch
(default: the north-star config, E=4 H=16 N=16384 d=128 b=128 T=2 bf16).
Under torchrun the E*H heads of that ONE workload are split across the ranks
(contiguous ranges, whole batch rows when E is a multiple of the rank count;
every (e, h) is independent, so there is no collective on the data path):
strong scaling, value = the workload's tokens / max-over-ranks time.  After
timing, the output shards are all-gathered over NCCL and rank 0 checks them
bit for bit against its own single-GPU forward of the whole workload.

``--impl reference`` times the reference algorithm on the host CPU instead:
the reference is Python (ma/ma_torch.py) and cannot be installed on the GPU
box, so its CPU restatement in oracle/ma_oracle.py runs on all host cores
(rank 0 only) over every head of the workload in every step.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "MA fwd ms & tokens/s at N=16K d=128 H=16 bf16; % of HBM/tensor roofline"
L2_BYTES = 126 * 1024 * 1024
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default=None)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--kernel", default=None, help="force a kernel family: generic | tc")
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0,
                    help="target CPU time of the cpu_baseline sample")
    ap.add_argument("--E", type=int, default=None, help="override the batch size (profiling)")
    ap.add_argument("--H", type=int, default=None, help="override the head count (profiling)")
    return ap.parse_args()


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


# ---------------------------------------------------------------------------
# CPU legs: the oracle port of ma/ma_torch.py on host cores
# ---------------------------------------------------------------------------
def cpu_sample(cfg, heads: int, threads: int, inputs=None):
    """Run the oracle on `heads` (e, h) pairs of cfg in parallel; return seconds."""
    import numpy as np
    from concurrent.futures import ThreadPoolExecutor
    from oracle.ma_oracle import monarch_attention_oracle
    try:
        from threadpoolctl import threadpool_limits
    except ImportError:  # pragma: no cover
        threadpool_limits = None
    if inputs is None:
        inputs = cpu_inputs(cfg, heads)
    q, k, v, mask, dt = inputs

    def one(i):
        e = i // cfg.H if mask is not None else 0
        m = None if mask is None else mask[e:e + 1]
        return monarch_attention_oracle(q[i:i + 1, None], k[i:i + 1, None], v[i:i + 1, None],
                                        m, cfg.T, cfg.B, cfg.pre_pad, dt)

    import contextlib
    # one BLAS thread per worker: the parallelism is over heads
    ctx = threadpool_limits(limits=1) if threadpool_limits else contextlib.nullcontext()
    with ctx:
        t0 = time.perf_counter()
        with ThreadPoolExecutor(max_workers=threads) as ex:
            list(ex.map(one, range(heads)))
        return time.perf_counter() - t0


def cpu_inputs(cfg, heads):
    """`heads` seeded (e, h) slices of cfg's inputs, as float32 numpy arrays
    (16-bit / e4m3 values rounded exactly as the GPU sees them)."""
    import numpy as np
    import torch
    from monarch_attention_b200.configs import dequantize_e4m3, make_inputs
    small = cfg.with_(E=max(1, math.ceil(heads / cfg.H)), H=cfg.H)
    q, k, v, mask, scales = make_inputs(small, device="cpu")
    if scales is not None:
        q, k, v = (dequantize_e4m3(t, s) for t, s in zip((q, k, v), scales))
    flat = [t.float().reshape(-1, cfg.N, t.shape[-1])[:heads].numpy() for t in (q, k, v)]
    dt = {"f32": "f32", "f16": "f16", "bf16": "bf16", "e4m3": "f32"}[cfg.dtype]
    mk = None if mask is None else mask.numpy()
    return flat[0], flat[1], flat[2], mk, dt


def cpu_rate(cfg, threads, target_s, first_heads=None):
    """Heads/s of the oracle on `threads` host threads, sampled for ~target_s."""
    heads = first_heads or threads
    inputs = cpu_inputs(cfg, heads)
    t = cpu_sample(cfg, heads, threads, inputs)
    reps = max(1, min(8, int(target_s / max(t, 1e-3))))
    if reps > 1:
        heads2 = min(heads * reps, cfg.E * cfg.H)
        inputs = cpu_inputs(cfg, heads2)
        t = cpu_sample(cfg, heads2, threads, inputs)
        heads = heads2
    return heads / t, heads, t


def run_reference(args, cfg, rank, world):
    """The reference arm: every step runs the oracle port over ALL E*H heads of
    the workload on the host cores (no sampling, no extrapolation)."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    heads = cfg.E * cfg.H
    inputs = cpu_inputs(cfg, heads)
    for _ in range(args.warmup):
        cpu_sample(cfg, heads, threads, inputs)
    times = []
    for _ in range(args.steps):
        times.append(cpu_sample(cfg, heads, threads, inputs))
    step = sum(times) / len(times)
    tokens = cfg.E * cfg.N
    value = tokens / step
    sample = (f"every step: all {heads} (e,h) heads of {cfg.name} on {threads} host threads "
              f"(oracle port of ma/ma_torch.py, {cfg.dtype} rounding emulated), "
              f"{args.steps} timed steps")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": step * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": cfg.dtype, "data": "synthetic (seeded iid normal)",
        "config": config_dict(cfg, max(world, args.gpus)),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU leg
# ---------------------------------------------------------------------------
def input_bytes(cfg):
    in_b = {"f32": 4, "f16": 2, "bf16": 2, "e4m3": 1}[cfg.dtype]
    return cfg.E * cfg.H * cfg.N * (2 * cfg.D + cfg.dv) * in_b


def shard_input_bytes(cfg, world):
    """Input bytes of the largest per-GPU shard at `world` GPUs."""
    from monarch_attention_b200.shard import shard_range
    most = max(b - a for a, b in (shard_range(cfg.E, cfg.H, world, r) for r in range(world)))
    return input_bytes(cfg) * most // (cfg.E * cfg.H)


def needs_flush(cfg, world):
    """Per-GPU inputs smaller than 2x L2 could stay cached between steps."""
    return shard_input_bytes(cfg, world) < 2 * L2_BYTES


def l2_note(cfg, world):
    """How the GPU arm keeps L2 from carrying inputs between timed steps (a
    property of the workload and the GPU count; identical in both arms)."""
    mib = shard_input_bytes(cfg, world) / 2**20
    if needs_flush(cfg, world):
        return (f"per-GPU inputs {mib:.0f} MiB < 2x L2: L2 flushed between timed steps "
                "(256 MB write, outside the events)")
    return f"per-GPU inputs {mib:.0f} MiB, larger than 2x the 126 MiB L2 (no flush)"


def config_dict(cfg, world):
    """The workload (identical in the GPU arm and the reference arm)."""
    return {"workload": cfg.name, "E": cfg.E, "H": cfg.H, "N": cfg.N, "D": cfg.D,
            "Dv": cfg.dv, "block_size": cfg.B, "num_steps": cfg.T,
            "mask": cfg.mask_min_len is not None, "pre_pad": cfg.pre_pad, "dtype": cfg.dtype,
            "l2": l2_note(cfg, world)}


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during a region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = os.path.join("/tmp", f"ma_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=self.f, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        # wait (at most 5 s) for the first sample: with one sampler per rank
        # starting at once, nvidia-smi's start-up can outlast a short timed
        # region, which then had no sample at all
        t0 = time.time()
        while time.time() - t0 < 5.0 and self.proc.poll() is None:
            if os.path.getsize(self.path) > 0:
                break
            time.sleep(0.02)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.12)  # let the samples taken at the end of the region land
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.f.close()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        try:
            os.remove(self.path)
        except OSError:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        sm = []
        for r in rows:
            try:
                sm.append(float(r[1]))
            except ValueError:
                pass
            for i, n in enumerate(names):
                if r[5 + i].lower().startswith("active"):
                    reasons.add(n)
        sm.sort()
        try:
            smax = float(rows[-1][2])
        except ValueError:
            smax = None
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(rows)}


def flops_and_bytes(cfg):
    """Algorithmic FLOPs and HBM bytes of one forward (padded length for FLOPs)."""
    M = cfg.M
    Np = M * cfg.B
    D, Dv, B, T = cfg.D, cfg.dv, cfg.B, cfg.T
    per_head = ((T - 1) * (4 * Np * B * D + 4 * Np * M * D) + 4 * Np * B * D
                + 2 * Np * B * Dv + 2 * Np * M * D + 2 * Np * M * Dv)
    heads = cfg.E * cfg.H
    in_b = {"f32": 4, "f16": 2, "bf16": 2, "e4m3": 1}[cfg.dtype]
    out_b = 4 if cfg.dtype == "f32" else 2
    mask_b = cfg.E * cfg.N if cfg.mask_min_len is not None else 0
    byts = heads * cfg.N * (2 * D + Dv) * in_b + heads * cfg.N * Dv * out_b + mask_b
    return float(heads * per_head), float(byts)


def run_gpu(args, cfg, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    import monarch_attention_b200 as mab
    from monarch_attention_b200 import _lib
    from monarch_attention_b200.configs import make_inputs
    from monarch_attention_b200.shard import gather_shards, shard_problem

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev,
                                timeout=datetime.timedelta(seconds=120))

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # ONE workload for every world size (same seed on every rank; the CUDA
    # generator gives the same numbers on every device), split by heads
    fq, fk, fv, fmask, fscales = make_inputs(cfg, device=dev)
    q, k, v, mask, scales, (h0, h1) = shard_problem(fq, fk, fv, fmask, fscales, world, rank)
    keep_full = world > 1 and rank == 0  # rank 0 re-runs the whole workload to verify
    if not keep_full:
        fq = fk = fv = fmask = fscales = None
    torch.cuda.empty_cache()
    impl = args.kernel
    Eh, Hh = q.shape[0], q.shape[1]
    out = torch.empty((Eh, Hh, cfg.N, cfg.dv),
                      dtype=torch.bfloat16 if cfg.dtype == "e4m3" else q.dtype, device=dev)
    kernel_family = mab.selected_impl(q, k, v, mask, cfg.T, cfg.B, cfg.pre_pad, impl=impl)

    def fwd():
        return mab.monarch_attention(q, k, v, mask, cfg.T, cfg.B, cfg.pre_pad, impl=impl,
                                     scales=scales, out=out)

    # flush when the largest per-GPU shard could stay in L2 (the same decision
    # on every rank)
    flush = needs_flush(cfg, world)
    scrub = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev) if flush else None

    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        fwd()
    launches_per_fwd = _lib.load().ma_last_launch_count()
    barrier()
    clocks = ClockSampler(local_rank)
    clocks.start()
    time.sleep(0.15)
    barrier()
    if flush:
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
        for i in range(args.steps):
            scrub.fill_(float(i))
            evs[i][0].record(stream)
            fwd()
            evs[i][1].record(stream)
        barrier()
        elapsed = sum(a.elapsed_time(b) for a, b in evs)
    else:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            fwd()
        e1.record(stream)
        barrier()
        elapsed = e0.elapsed_time(e1)
    clk = clocks.stop()
    status = mab.read_status(dev)
    t = torch.tensor([elapsed], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_total = float(t.item())
    ms_step = ms_total / args.steps
    tokens_step = cfg.E * cfg.N  # the whole workload, whatever the rank count
    value = tokens_step / (ms_step / 1e3)

    # ---- end to end through the public API: host (pinned) -> device -> host.
    # Every step copies its inputs in and its result out inside the timed
    # region; the copies run on their own streams with two buffer sets, so
    # step i+1's input copy and step i-1's result copy overlap step i's
    # forward (a serving pipeline; PCIe carries both directions at once).
    # Each rank copies its own shard over its own link.
    e2e = None
    if not args.no_e2e:
        hq, hk, hv = (x.cpu().pin_memory() for x in (q, k, v))
        hm = None if mask is None else mask.cpu().pin_memory()
        hsc = None if scales is None else tuple(s.cpu() for s in scales)
        hout = [torch.empty(out.shape, dtype=out.dtype).pin_memory() for _ in range(2)]
        dbuf = [[torch.empty_like(x) for x in (q, k, v)] for _ in range(2)]
        dm = [None if mask is None else torch.empty_like(mask) for _ in range(2)]
        dsc = [None if scales is None else [torch.empty_like(s) for s in scales] for _ in range(2)]
        dout = [torch.empty_like(out) for _ in range(2)]
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        ev_in = [torch.cuda.Event() for _ in range(2)]
        ev_fwd = [torch.cuda.Event() for _ in range(2)]
        ev_out = [torch.cuda.Event() for _ in range(2)]
        n_e2e = args.e2e_steps or max(3, min(args.steps, 10))

        def e2e_steps(n):
            for i in range(n):
                b = i % 2
                with torch.cuda.stream(s_in):
                    if i >= 2:
                        s_in.wait_event(ev_fwd[b])  # the forward of step i-2 read buffer b
                    for d, h in zip(dbuf[b], (hq, hk, hv)):
                        d.copy_(h, non_blocking=True)
                    if hm is not None:
                        dm[b].copy_(hm, non_blocking=True)
                    if hsc is not None:
                        for d, h in zip(dsc[b], hsc):
                            d.copy_(h, non_blocking=True)
                    ev_in[b].record(s_in)
                stream.wait_event(ev_in[b])
                if i >= 2:
                    stream.wait_event(ev_out[b])  # the result of step i-2 was read out
                mab.monarch_attention(*dbuf[b], dm[b], cfg.T, cfg.B, cfg.pre_pad, impl=impl,
                                      scales=None if dsc[b] is None else tuple(dsc[b]),
                                      out=dout[b])
                ev_fwd[b].record(stream)
                with torch.cuda.stream(s_out):
                    s_out.wait_event(ev_fwd[b])
                    hout[b].copy_(dout[b], non_blocking=True)
                    ev_out[b].record(s_out)

        e2e_steps(2)
        torch.cuda.synchronize()
        barrier()
        a, b_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(s_in)
        e2e_steps(n_e2e)
        s_out.wait_stream(stream)
        s_out.wait_stream(s_in)
        b_.record(s_out)
        barrier()
        te = torch.tensor([a.elapsed_time(b_)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e_ms = float(te.item()) / n_e2e
        h2d = sum(x.numel() * x.element_size() for x in (hq, hk, hv))
        h2d += 0 if hm is None else hm.numel() * hm.element_size()
        h2d += 0 if hsc is None else sum(x.numel() * x.element_size() for x in hsc)
        d2h = hout[0].numel() * hout[0].element_size()
        if world > 1:  # whole-job bytes: the sum over ranks
            tb = torch.tensor([h2d, d2h], dtype=torch.float64, device=dev)
            dist.all_reduce(tb)
            h2d, d2h = int(tb[0].item()), int(tb[1].item())
        e2e = {"value": tokens_step / (e2e_ms / 1e3), "unit": "tokens/s",
               "ms_per_step": e2e_ms, "steps": n_e2e, "pipelined": "double-buffered copy streams",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h}
        del hq, hk, hv, hm, hout, dbuf, dm, dsc, dout

    # ---- verification (after timing): NCCL all-gather of the output shards;
    # rank 0 compares them bit for bit with its own forward of the whole
    # workload on one GPU (a head's result does not depend on which heads
    # share its launch)
    verify = None
    if world > 1:
        from monarch_attention_b200.shard import shard_range
        full = gather_shards(out, cfg.E, cfg.H)
        if rank == 0:
            ref = mab.monarch_attention(fq, fk, fv, fmask, cfg.T, cfg.B, cfg.pre_pad, impl=impl,
                                        scales=fscales)
            torch.cuda.synchronize()
            fl = full.reshape(cfg.E * cfg.H, cfg.N, cfg.dv)
            ref = ref.reshape(cfg.E * cfg.H, cfg.N, cfg.dv)
            sizes = [shard_range(cfg.E, cfg.H, world, r) for r in range(world)]
            same = [bool(torch.equal(fl[a:b], ref[a:b])) for a, b in sizes]
            verify = {"heads": cfg.E * cfg.H, "gathered_bytes": full.numel() * full.element_size(),
                      "bit_exact_per_rank": same, "all_bit_exact": all(same),
                      "all_finite": bool(torch.isfinite(full.float()).all().item()),
                      "status": mab.read_status(dev)}
            del ref, fl
        del full
        barrier()

    # ---- roofline of the dominant kernel (one forward = one launch on tc)
    peaks, peak_src = load_peaks()
    flop, byts = flops_and_bytes(cfg)  # the whole workload (all ranks)
    t_s = ms_step / 1e3
    if cfg.dtype == "f32":
        peak_flops = 148 * 128 * 2 * 1.965e9
        peak_note = "FFMA peak 148 SM x 128 lanes x 2 x 1.965 GHz (fp32 config)"
    else:
        peak_flops = peaks["bf16_tflops"] * 1e12 * (2 if cfg.dtype == "e4m3" else 1)
        peak_note = f"bf16 dense burst, {peak_src}" + (" x2 (fp8 assumed)" if cfg.dtype == "e4m3" else "")
    peak_flops *= world
    hbm = peaks["hbm_gbs"] * 1e9 * world
    t_flop, t_hbm = flop / peak_flops, byts / hbm
    if t_flop >= t_hbm:
        roof = {"bound": "tensor", "achieved": flop / t_s / 1e12, "peak": peak_flops / 1e12,
                "unit": "TFLOP/s"}
    else:
        roof = {"bound": "hbm", "achieved": byts / t_s / 1e9, "peak": hbm / 1e9, "unit": "GB/s"}
    roof["frac"] = roof["achieved"] / roof["peak"]
    roof["peak_source"] = (peak_note if roof["bound"] == "tensor" else f"hbm copy, {peak_src}") + \
        (f", x {world} GPUs" if world > 1 else "")
    traffic = load_traffic(cfg.name, kernel_family)
    roof["traffic"] = None if traffic is None else traffic / world  # per launch (one rank's)
    roof["t_star_us"] = max(t_flop, t_hbm) * 1e6
    roof["algorithmic_flop_per_launch"] = flop / world
    roof["algorithmic_bytes_per_launch"] = byts / world

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        rate, heads, secs = cpu_rate(cfg, threads, args.cpu_seconds)
        full_s = (cfg.E * cfg.H) / rate
        cpu = {"value": cfg.E * cfg.N / full_s, "unit": "tokens/s", "cores": threads,
               "kind": "port",
               "sample": f"{heads} of the {cfg.E * cfg.H} (e,h) heads of {cfg.name} in "
                         f"{secs:.1f} s on {threads} host threads (oracle port of "
                         f"ma/ma_torch.py), per-head rate scaled to the batch"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": cfg.dtype, "data": "synthetic (seeded iid normal)",
            "config": config_dict(cfg, world),
            "kernel": kernel_family,
            "parallelism": (f"E*H = {cfg.E * cfg.H} heads split over {world} GPU(s), "
                            f"{h1 - h0} heads on rank 0; no collective on the data path"),
            "roofline": roof, "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": launches_per_fwd * args.steps, "clocks": clk,
            "device_status": status,
        }
        if verify is not None:
            line["verify"] = verify
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def load_traffic(name, kernel):
    """DRAM bytes per launch of the dominant kernel from a committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(path):
        return None
    with open(path) as f:
        d = json.load(f)
    ent = d.get(f"{name}/{kernel}")
    return None if ent is None else ent.get("dram_bytes_per_launch")


def main():
    args = parse()
    from monarch_attention_b200.configs import CONFIGS, NORTH_STAR
    cfg = CONFIGS[args.config or NORTH_STAR]
    if args.E or args.H:
        cfg = cfg.with_(E=args.E or cfg.E, H=args.H or cfg.H)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, cfg, rank, world)
        return
    run_gpu(args, cfg, rank, world, local_rank)


if __name__ == "__main__":
    main()
