#!/usr/bin/env python
"""Benchmark of the Cherimoya hot path on B200.

Workload (one "step"): the default 9-layer Cherimoya (n_filters 128,
expansion 2, one unstranded track; random-init weights from seed 0) runs
its full forward -- stem, 9 Cheri Blocks, profile and count heads -- over
a batch of 1024 uniform random one-hot 2114-bp sequences per GPU, in bf16
mode (bf16 residual stream, fp32 LayerNorm statistics and accumulation).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun, one rank per GPU, each rank its own batch
(weak scaling, no collective on the data path). Prints one JSON line on
rank 0. `value` = sequences/s of the whole job with inputs resident in
HBM; `e2e` = the same through the public API (`model(X)`) with host
inputs copied in and outputs copied out inside the timed region; `ism` =
on-device saturation-mutagenesis mutants/s; `roofline` = the MLP kernel's
achieved tensor FLOP/s over the measured bf16 peak; `cpu_baseline` = the
oracle (the upstream PyTorch CPU path restated) on the host cores.

--impl reference times the upstream algorithm's CPU implementation (the
oracle port) on the same workload, a bounded sample of sequences per step,
on rank 0 only.
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "seqs/sec fwd (2114bp, 9-layer) & ISM mutants/sec at 1/2/4/8 B200; % roofline"
MLP_DRAM_BYTES_PER_SEQ = (138.728704e6 + 94.934528e6) / 256   # measured, bf16 mode
L = 2114
C, H, N_LAYERS = 128, 256, 9
# algorithmic work per sequence of the default model (one track)
MLP_FLOP_PER_SEQ = 4 * C * H * L * N_LAYERS                 # 2,493,775,872
FLOP_PER_SEQ = MLP_FLOP_PER_SEQ + 2 * 84 * C * L + 6 * C * L * N_LAYERS + 2 * C * 75 * 1000
IN_BYTES_PER_SEQ = 4 * 4 * L                                  # fp32 one-hot
OUT_BYTES_PER_SEQ = 4 * (1000 + 1)
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    except Exception:
        return PEAKS_FALLBACK, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), "--query-gpu=" + self.QUERY,
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.1)
        self.proc.terminate()
        try:
            self.proc.wait(5)
        except Exception:
            self.proc.kill()
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
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "samples": len(sm),
                "reasons": sorted(reasons)}


def dist_setup():
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl" if torch.cuda.is_available() else "gloo",
                                timeout=datetime.timedelta(seconds=120))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v, world, device):
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(v)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def make_inputs(batch, seed):
    import torch
    from oracle.cherimoya_oracle import one_hot  # input generator only
    g = torch.Generator().manual_seed(seed)
    return one_hot(torch.randint(0, 4, (batch, L), generator=g))


def cpu_forward_rate(n_seqs, min_seconds=10.0, max_reps=8):
    """Oracle (upstream PyTorch CPU path restated) fp32 forward on the host
    cores: sequences/s over a bounded sample of n_seqs sequences."""
    import torch
    from oracle import cherimoya_oracle as O
    import cherimoya_b200 as cb
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    torch.manual_seed(0)
    m = cb.Cherimoya(compile=False)
    sd = {k: v.clone() for k, v in m.state_dict().items()}
    cfg = m._init_kwargs()
    X = make_inputs(n_seqs, 1)
    with torch.no_grad():
        O.forward(sd, cfg, X)                       # warm-up
        times, t_all = [], time.perf_counter()
        while len(times) < max_reps:
            t0 = time.perf_counter()
            O.forward(sd, cfg, X)
            times.append(time.perf_counter() - t0)
            if time.perf_counter() - t_all >= min_seconds and len(times) >= 2:
                break
    return n_seqs / statistics.median(times), cores, len(times)


def run_reference(args, world, rank):
    """--impl reference: the upstream algorithm's CPU path (oracle port)."""
    if rank != 0:
        return
    import torch
    from oracle import cherimoya_oracle as O
    import cherimoya_b200 as cb
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    torch.manual_seed(0)
    m = cb.Cherimoya(compile=False)
    sd = {k: v.clone() for k, v in m.state_dict().items()}
    cfg = m._init_kwargs()
    sample = args.ref_sample
    X = make_inputs(sample, 1)
    with torch.no_grad():
        for _ in range(args.warmup):
            O.forward(sd, cfg, X)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            O.forward(sd, cfg, X)
        dt = time.perf_counter() - t0
    value = sample * args.steps / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "seqs/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * dt / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(args, world),
        "cpu_baseline": {"value": value, "unit": "seqs/s", "cores": cores, "kind": "port",
                         "sample": "{} of the batch's sequences per step, fp32 eager "
                                   "no_grad".format(sample)},
        "e2e": {"value": value, "unit": "seqs/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_config(args, world):
    return {
        "workload": "default 9-layer Cherimoya forward (n_filters 128, expansion 2, 1 track, "
                    "random init seed 0), batch {} per GPU of uniform random one-hot {}-bp "
                    "sequences, {} mode".format(args.batch, L, args.mode),
        "global_batch": args.batch * world, "seq_len": L, "parallelism": "dp{}".format(world),
        "l2": "256 MiB buffer written between timed steps (outside the step events)",
    }


def run_ours(args, world, rank, local):
    import torch
    import cherimoya_b200 as cb
    from cherimoya_b200 import _lib, ops

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    torch.manual_seed(0)
    model = cb.Cherimoya(compile=False, precision=args.mode).eval().to(dev)
    X = make_inputs(args.batch, 1 + rank).to(dev)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    lib = _lib.load()

    with torch.no_grad():
        for _ in range(args.warmup):
            model(X)
        torch.cuda.synchronize()
        launches_per_step = ops.last_launch_count()

        # ---- device-resident timed region
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        sampler = ClockSampler(local)
        barrier(world)
        torch.cuda.synchronize()
        sampler.start()
        _lib.timing_collect()
        _lib.timing_enable(True)
        for k in range(args.steps):
            flush.zero_()
            starts[k].record()
            model(X)
            ends[k].record()
        torch.cuda.synchronize()
        _lib.timing_enable(False)
        barrier(world)
        clocks = sampler.stop()
        per_class = _lib.timing_collect()
        step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
        dev_ms = sum(step_ms)
        dev_ms_max = max_over_ranks(dev_ms, world, dev)
        value = world * args.batch * args.steps / (dev_ms_max / 1000.0)

        # ---- end to end through the public API, host buffers: every step copies
        # its one-hot input from pinned host memory and reads its outputs back.
        # The copy of step k+1's input runs on a second stream while step k
        # computes (two device input buffers), as a serving loop would.
        e2e = None
        if not args.no_e2e:
            Xh = make_inputs(args.batch, 1 + rank).pin_memory()
            ph = torch.empty((args.batch, 1, L - 2 * model.trimming), dtype=torch.float32,
                             pin_memory=True)
            ch = torch.empty((args.batch, 1), dtype=torch.float32, pin_memory=True)
            xd = [torch.empty_like(Xh, device=dev) for _ in range(2)]
            copy_stream = torch.cuda.Stream(device=dev)
            compute = torch.cuda.current_stream(dev)

            def run_steps(n):
                copied = [torch.cuda.Event() for _ in range(2)]
                consumed = [torch.cuda.Event() for _ in range(2)]
                with torch.cuda.stream(copy_stream):
                    copy_stream.wait_stream(compute)       # after the start event
                    xd[0].copy_(Xh, non_blocking=True)
                    copied[0].record(copy_stream)
                for k in range(n):
                    b = k % 2
                    if k + 1 < n:
                        nb = (k + 1) % 2
                        with torch.cuda.stream(copy_stream):
                            if k >= 1:
                                copy_stream.wait_event(consumed[nb])
                            xd[nb].copy_(Xh, non_blocking=True)
                            copied[nb].record(copy_stream)
                    compute.wait_event(copied[b])
                    p, c = model(xd[b])
                    consumed[b].record(compute)
                    ph.copy_(p, non_blocking=True)
                    ch.copy_(c, non_blocking=True)

            run_steps(args.warmup)
            torch.cuda.synchronize()
            barrier(world)
            e_s = torch.cuda.Event(enable_timing=True)
            e_e = torch.cuda.Event(enable_timing=True)
            e_s.record()
            run_steps(args.steps)
            e_e.record()
            torch.cuda.synchronize()
            barrier(world)
            e2e_ms = max_over_ranks(e_s.elapsed_time(e_e), world, dev)
            e2e = {"value": world * args.batch * args.steps / (e2e_ms / 1000.0),
                   "unit": "seqs/s", "h2d_bytes_per_step": Xh.numel() * Xh.element_size(),
                   "d2h_bytes_per_step": ph.numel() * 4 + ch.numel() * 4,
                   "api": "Cherimoya.forward(X) on pinned host one-hot fp32 input; the "
                          "next step's H2D copy overlaps the current step"}

        # ---- saturation mutagenesis (sharded by sequence, weak scaling)
        ism = None
        if args.ism_seqs > 0:
            bases = torch.randint(0, 4, (args.ism_seqs, L),
                                  generator=torch.Generator().manual_seed(100 + rank))
            bases = bases.to(torch.int8).to(dev)
            cb.saturation_mutagenesis(model, bases[:1], 1000, 1010)     # warm-up
            torch.cuda.synchronize()
            barrier(world)
            i_s = torch.cuda.Event(enable_timing=True)
            i_e = torch.cuda.Event(enable_timing=True)
            i_s.record()
            d, j = cb.saturation_mutagenesis(model, bases, 0, L, mutant_batch=args.batch)
            i_e.record()
            torch.cuda.synchronize()
            barrier(world)
            ism_ms = max_over_ranks(i_s.elapsed_time(i_e), world, dev)
            n_mut = world * args.ism_seqs * 3 * L
            ism = {"value": n_mut / (ism_ms / 1000.0), "unit": "mutants/s",
                   "mutants": n_mut, "ms": ism_ms,
                   "workload": "{} random 2114-bp sequences per GPU x all 3x2114 single-base "
                               "substitutions, delta log-count + profile JSD per mutant, "
                               "{} mode".format(args.ism_seqs, args.mode)}

    peaks, peak_src = load_peaks()
    mlp_ms, mlp_n = per_class["mlp"]
    mlp_avg_ms = mlp_ms / max(mlp_n, 1)
    mlp_flop = 4.0 * C * H * L * args.batch                 # one layer, one launch
    achieved = mlp_flop / (mlp_avg_ms / 1000.0) / 1e12
    peak = peaks["bf16_tflops_sustained"]
    model_tflops = value / world * FLOP_PER_SEQ / 1e12
    roofline = {
        "bound": "tensor", "kernel": "mlp_kernel (tcgen05 conv+LN+MLP+residual, one layer)",
        "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
        "peak_source": "{} bf16_tflops_sustained".format(peak_src),
        "frac_of_burst": achieved / peaks["bf16_tflops"],
        # DRAM bytes of one MLP launch: ncu dram__bytes_read.sum + write.sum of the
        # layer-0 launch at batch 256 (138.73 MB + 94.93 MB), scaled by the
        # sequences processed
        "traffic": (MLP_DRAM_BYTES_PER_SEQ * args.batch) if args.mode == "bf16" else None,
        "traffic_unit": "bytes per launch",
        "algorithmic_bytes": 2.0 * L * C * (2 if args.mode == "bf16" else 4) * args.batch,
        "flop_per_launch": mlp_flop, "avg_launch_ms": mlp_avg_ms,
        "whole_forward_tflops_per_gpu": model_tflops,
        "whole_forward_frac": model_tflops / peak,
        "kernel_share": {k: v[0] / max(dev_ms, 1e-9) for k, v in per_class.items() if v[1]},
    }
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        rate, cores, reps = cpu_forward_rate(args.cpu_sample)
        cpu = {"value": rate, "unit": "seqs/s", "cores": cores, "kind": "port",
               "sample": "{} sequences, fp32 eager no_grad, median of {} reps".format(
                   args.cpu_sample, reps)}
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "seqs/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": dev_ms_max / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16" if args.mode == "bf16" else "f32", "data": "synthetic",
            "config": workload_config(args, world),
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "ism": ism,
            "clocks": clocks, "gpu_launches": launches_per_step * args.steps,
        }
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=int(os.environ.get("WORLD_SIZE", "1")))
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=1024)
    ap.add_argument("--mode", choices=["bf16", "fp32"], default="bf16")
    ap.add_argument("--ism-seqs", type=int, default=4)
    ap.add_argument("--cpu-sample", type=int, default=32)
    ap.add_argument("--ref-sample", type=int, default=16)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    args = ap.parse_args()
    world, rank, local = dist_setup()
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
