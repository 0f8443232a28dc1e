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
HBM, timed without per-kernel instrumentation; `e2e` = the same through
the public API (`model(X)`) with host inputs copied in and outputs copied
out inside the timed region; `ism` = saturation mutagenesis of 256
sequences x all 3 x 2114 substitutions, sharded over the ranks, with the
H2D copy of the bases and the all-gather + D2H of the scores inside the
timed region (mutants/s); `roofline` = the dominant kernel's achieved
tensor FLOP/s over the measured burst bf16 peak (a millisecond-long
step), with the whole forward's fraction beside it; `cpu_baseline` = the
upstream package's CPU forward on the host cores.

--impl reference times the upstream package's own CPU forward (the
reference's pure-PyTorch path, imported from baseline/_ref by
oracle/upstream.py; the oracle port when that install is absent) on the
same workload, a bounded sample of sequences per step, on rank 0 only.

--impl reference-gpu (opt-in, not part of the default runs) times the
upstream package's own CUDA inference path on this GPU: its Triton fused
Cheri Block kernels (upstream cherimoya/cheri.py:490-754) under
torch.no_grad(), compile=False, bf16 autocast, same weights and inputs,
inputs resident on the device.

--workload selects the model and input set (the default is the one above):
  forward    default 9-layer model, uniform random sequences, batch 1024
  multitask  the same backbone with 1 unstranded + 4 stranded tracks
             (signal_groups [1, 2, 2, 2, 2]: 9 profile tracks, 5 count
             heads), batch 2048, per-sequence GC fraction uniform in
             [0.35, 0.65]
  variant    12-layer n_filters 256 model (trimming 557), ref/alt pairs
             differing by one SNV at the centre position (alt uniform among
             the 3 other bases), 512 pairs per GPU per step; unit pairs/s
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
# DRAM bytes (read + write) of one default-width MLP launch per sequence, bf16:
# mean of the nine launches of one forward under ncu at batch 256
# (profiles/mlp_ws_dram_all_layers_bf16_b256.md)
MLP_DRAM_BYTES_PER_SEQ = 230.26e6 / 256
L = 2114
WORKLOADS = {
    # name: (model kwargs, default batch per GPU, input seed base, unit)
    "forward": ({}, 1024, 1, "seqs/s"),
    "multitask": ({"signal_groups": [1, 2, 2, 2, 2]}, 2048, 2, "seqs/s"),
    "variant": ({"n_filters": 256, "n_layers": 12, "trimming": 557}, 512, 3, "pairs/s"),
}


def flop_per_seq(model):
    """Algorithmic FLOP of one forward: MLP 4 C H L per layer, stem 2*84 C L,
    depthwise conv 6 C L per layer, profile head 2 C 75 n_out over the
    trimmed window (2,573,047,296 for the default model)."""
    C, H, nl = model.n_filters, model.n_filters * model.expansion, model.n_layers
    l_out = L - 2 * model.trimming
    return (4 * C * H * L * nl + 2 * 84 * C * L + 6 * C * L * nl
            + 2 * C * 75 * model.n_outputs * l_out)


def mlp_flop_per_seq(model):
    return 4 * model.n_filters * model.n_filters * model.expansion * L * model.n_layers


REF_WHAT = {"reference": "upstream cherimoya 0.2.1 Cherimoya.forward (baseline/_ref)",
            "port": "oracle restatement of the upstream CPU path"}
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
        if not self.lines:
            # a timed region shorter than the sampling interval: one reading
            # taken right after it
            try:
                out = subprocess.run(
                    ["nvidia-smi", "-i", str(self.index), "--query-gpu=" + self.QUERY,
                     "--format=csv,noheader,nounits"],
                    capture_output=True, text=True, timeout=20).stdout
                self.lines = [ln.strip() for ln in out.splitlines() if ln.strip()]
            except Exception:
                pass
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


def make_bases(workload, batch, seed):
    """Input bases (0..3 = A, C, G, T) of a workload: a tuple of (batch, L)
    int64 tensors, one per model input (ref and alt for variant pairs)."""
    import torch
    g = torch.Generator().manual_seed(seed)
    if workload == "multitask":
        # per-sequence GC fraction gc ~ U(0.35, 0.65); C and G each gc / 2
        gc = 0.35 + 0.3 * torch.rand(batch, 1, generator=g)
        u = torch.rand(batch, L, generator=g)
        bases = torch.where(u < gc / 2, 1, torch.where(u < gc, 2,
                            torch.where(u < gc + (1 - gc) / 2, 0, 3)))
        return (bases,)
    ref = torch.randint(0, 4, (batch, L), generator=g)
    if workload != "variant":
        return (ref,)
    alt = ref.clone()
    c = L // 2
    alt[:, c] = (ref[:, c] + torch.randint(1, 4, (batch,), generator=g)) % 4
    return (ref, alt)


def build_model(args):
    import torch
    import cherimoya_b200 as cb
    torch.manual_seed(0)
    return cb.Cherimoya(compile=False, precision=args.mode, **WORKLOADS[args.workload][0])


def reference_step(args, n):
    """The reference's fp32 CPU work for n units of the workload: (a callable
    running it once, kind). kind "reference": the upstream package itself
    (eager ``Cherimoya.forward`` under no_grad, compile=False; upstream
    cherimoya/cherimoya.py:340-400 with cheri.py:84-98 for the blocks),
    loaded with the same state_dict as the engine's model; kind "port": the
    oracle's restatement, when no upstream install is present."""
    import torch
    from oracle import cherimoya_oracle as O
    from oracle import upstream
    m = build_model(args)
    sd = {k: v.detach().float().clone() for k, v in m.state_dict().items()}
    cfg = m._init_kwargs()
    seed = WORKLOADS[args.workload][2]
    inputs = make_bases(args.workload, n, seed)
    if upstream.available():
        ref = upstream.import_upstream()
        um = ref.Cherimoya(**cfg, compile=False).eval()
        um.load_state_dict(sd)
        if args.workload == "variant":
            Xr, Xa = O.one_hot(inputs[0]), O.one_hot(inputs[1])

            def run_pairs():
                p_r, c_r = um(Xr)
                p_a, c_a = um(Xa)
                pr = torch.softmax(p_r.reshape(n, -1), dim=-1)
                return c_a - c_r, ref.performance.jensen_shannon_distance(
                    p_a.reshape(n, -1), pr)
            return run_pairs, "reference"
        X = O.one_hot(inputs[0])
        return (lambda: um(X)), "reference"
    if args.workload == "variant":
        return (lambda: O.variant_scores(sd, cfg, inputs[0], inputs[1])), "port"
    X = O.one_hot(inputs[0])
    return (lambda: O.forward(sd, cfg, X)), "port"


def cpu_forward_rate(args, n_units, min_seconds=10.0, max_reps=8):
    """Reference fp32 rate on the host cores, units/s over a bounded sample
    of n_units units (sequences, or pairs for the variant workload)."""
    import torch
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    run, kind = reference_step(args, n_units)
    with torch.no_grad():
        run()                                       # warm-up
        times, t_all = [], time.perf_counter()
        while len(times) < max_reps:
            t0 = time.perf_counter()
            run()
            times.append(time.perf_counter() - t0)
            if time.perf_counter() - t_all >= min_seconds and len(times) >= 2:
                break
    return n_units / statistics.median(times), cores, len(times), kind


def run_reference(args, world, rank):
    """--impl reference: the upstream package's CPU path on the host cores."""
    if rank != 0:
        return
    import torch
    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    sample = args.ref_sample
    run, kind = reference_step(args, sample)
    unit = WORKLOADS[args.workload][3]
    with torch.no_grad():
        for _ in range(args.warmup):
            run()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            run()
        dt = time.perf_counter() - t0
    value = sample * args.steps / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": unit,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * dt / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(args, world),
        "cpu_baseline": {"value": value, "unit": unit, "cores": cores, "kind": kind,
                         "sample": "{} of the batch's {} per step, fp32 eager no_grad, "
                                   "{}".format(sample, unit.split("/")[0], REF_WHAT[kind])},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_reference_gpu(args, world, rank, local):
    """--impl reference-gpu: the upstream package's Triton inference path on
    this GPU (rank 0 only), device-resident inputs, CUDA-event timing."""
    if rank != 0:
        return
    import torch
    from oracle import upstream
    from oracle.cherimoya_oracle import one_hot
    if not upstream.available():
        print(json.dumps({"impl": "reference-gpu",
                          "unavailable": "upstream package not installed in baseline/_ref"}))
        return
    ref = upstream.import_upstream()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    m = build_model(args)
    cfg = m._init_kwargs()
    um = ref.Cherimoya(**cfg, compile=False)
    um.load_state_dict(m.state_dict())
    um = um.eval().to(dev)
    seed = WORKLOADS[args.workload][2]
    X = one_hot(make_bases(args.workload, args.batch, seed)[0]).to(dev)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    amp = torch.autocast("cuda", dtype=torch.bfloat16, enabled=args.mode == "bf16")
    with torch.no_grad(), amp:
        for _ in range(max(args.warmup, 3)):
            um(X)
        torch.cuda.synchronize()
        ms = []
        for _ in range(args.steps):
            flush.zero_()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            um(X)
            e1.record()
            torch.cuda.synchronize()
            ms.append(e0.elapsed_time(e1))
    total = sum(ms)
    line = {
        "impl": "reference-gpu", "metric": METRIC, "value": args.batch * args.steps / (total / 1e3),
        "unit": WORKLOADS[args.workload][3], "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": total / args.steps, "higher_is_better": True,
        "dtype": args.mode, "data": "synthetic", "config": workload_config(args, 1),
        "what": "upstream cherimoya 0.2.1 Cherimoya.forward on CUDA (Triton fused Cheri Block "
                "inference kernels), no_grad, compile=False, {} autocast".format(args.mode),
    }
    print(json.dumps(line), flush=True)


def time_other_workload(name, args, world, rank, dev, steps=5, warmup=3):
    """Device-resident throughput of another workload's step (per GPU batch
    of that workload, weak scaling, max over ranks): the multi-task backbone
    (seq/s) and the 12-layer n_filters-256 variant scoring (pairs/s)."""
    import copy
    import torch
    import cherimoya_b200 as cb
    from oracle.cherimoya_oracle import one_hot  # input generator only
    wargs = copy.copy(args)
    wargs.workload = name
    batch = WORKLOADS[name][1]
    wargs.batch = batch
    model = build_model(wargs).eval().to(dev)
    xs = [one_hot(b).to(dev) for b in make_bases(name, batch, WORKLOADS[name][2] + rank)]

    def step():
        if name == "variant":
            return cb.variant_effect(model, xs[0], xs[1])
        return model(xs[0])

    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    with torch.no_grad():
        for _ in range(warmup):
            step()
        torch.cuda.synchronize()
        barrier(world)
        ms = 0.0
        for _ in range(steps):
            flush.zero_()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            step()
            e1.record()
            torch.cuda.synchronize()
            ms += e0.elapsed_time(e1)
        barrier(world)
    ms = max_over_ranks(ms, world, dev)
    del model, xs, flush
    torch.cuda.empty_cache()
    return {"value": world * batch * steps / (ms / 1000.0), "unit": WORKLOADS[name][3],
            "ms_per_step": ms / steps, "steps": steps, "batch_per_gpu": batch,
            "workload": workload_config(wargs, world)["workload"]}


def workload_config(args, world):
    if args.workload == "multitask":
        what = ("9-layer Cherimoya forward, signal_groups [1, 2, 2, 2, 2] (9 profile tracks, "
                "5 count heads; random init seed 0), batch {} per GPU of one-hot {}-bp "
                "sequences with per-sequence GC fraction uniform in [0.35, 0.65], {} mode")
    elif args.workload == "variant":
        what = ("ref/alt variant scoring (delta log-count + profile JSD per pair) with the "
                "12-layer n_filters 256 Cherimoya (trimming 557, random init seed 0), {} "
                "pairs per GPU of uniform random one-hot {}-bp sequences, alt = one SNV at "
                "the centre, {} mode")
    else:
        what = ("default 9-layer Cherimoya forward (n_filters 128, expansion 2, 1 track, "
                "random init seed 0), batch {} per GPU of uniform random one-hot {}-bp "
                "sequences, {} mode")
    return {
        "workload": what.format(args.batch, L, args.mode),
        "global_batch": args.batch * world, "seq_len": L, "parallelism": "dp{}".format(world),
        "l2": "256 MiB buffer written between timed steps (outside the step events)",
    }


def run_ours(args, world, rank, local):
    import torch
    import cherimoya_b200 as cb
    from cherimoya_b200 import _lib, ops
    from oracle.cherimoya_oracle import one_hot  # input generator only

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    model = build_model(args).eval().to(dev)
    variant = args.workload == "variant"
    unit = WORKLOADS[args.workload][3]
    # host inputs: one-hot fp32, (batch, 4, L) each (ref and alt for pairs)
    host_in = [one_hot(b) for b in make_bases(args.workload, args.batch,
                                              WORKLOADS[args.workload][2] + rank)]
    dev_in = [x.to(dev) for x in host_in]
    forwards = len(host_in)                       # model forwards per unit

    def step(xs):
        if variant:
            return cb.variant_effect(model, xs[0], xs[1])
        return model(xs[0])

    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    lib = _lib.load()

    with torch.no_grad():
        for _ in range(args.warmup):
            step(dev_in)
        torch.cuda.synchronize()
        launches_per_step = ops.last_launch_count()

        # ---- device-resident timed region
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        sampler = ClockSampler(local)
        barrier(world)
        torch.cuda.synchronize()
        sampler.start()
        for k in range(args.steps):
            flush.zero_()
            starts[k].record()
            step(dev_in)
            ends[k].record()
        torch.cuda.synchronize()
        barrier(world)
        clocks = sampler.stop()
        step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
        dev_ms = sum(step_ms)
        dev_ms_max = max_over_ranks(dev_ms, world, dev)
        value = world * args.batch * args.steps / (dev_ms_max / 1000.0)

        # ---- per-kernel shares: a separate instrumented pass (CUDA events
        # around every launch, on the launching stream), never the headline
        n_inst = max(1, min(args.steps, 5))
        _lib.timing_collect()
        _lib.timing_enable(True)
        inst_ms = 0.0
        for _ in range(n_inst):
            flush.zero_()
            i0 = torch.cuda.Event(enable_timing=True)
            i1 = torch.cuda.Event(enable_timing=True)
            i0.record()
            step(dev_in)
            i1.record()
            torch.cuda.synchronize()
            inst_ms += i0.elapsed_time(i1)
        _lib.timing_enable(False)
        per_class = _lib.timing_collect()

        # ---- end to end through the public API, host buffers: every step copies
        # its one-hot inputs from pinned host memory and reads its outputs back.
        # The copy of step k+1's inputs runs on a second stream while step k
        # computes (two device buffers per input), as a serving loop would.
        e2e = None
        if not args.no_e2e:
            hin = [x.pin_memory() for x in host_in]
            outs = step(dev_in)
            hout = [torch.empty(o.shape, dtype=o.dtype, pin_memory=True) for o in outs]
            xd = [[torch.empty_like(x, device=dev) for x in hin] for _ in range(2)]
            copy_stream = torch.cuda.Stream(device=dev)
            compute = torch.cuda.current_stream(dev)

            def copy_in(b):
                for dst, src in zip(xd[b], hin):
                    dst.copy_(src, non_blocking=True)

            def run_steps(n):
                # copy stream: input H2D of the next step and output D2H of the
                # finished one, both overlapping the compute of the current step
                copied = [torch.cuda.Event() for _ in range(2)]
                consumed = [torch.cuda.Event() for _ in range(2)]
                with torch.cuda.stream(copy_stream):
                    copy_stream.wait_stream(compute)       # after the start event
                    copy_in(0)
                    copied[0].record(copy_stream)
                for k in range(n):
                    b = k % 2
                    if k + 1 < n:
                        nb = (k + 1) % 2
                        with torch.cuda.stream(copy_stream):
                            if k >= 1:
                                copy_stream.wait_event(consumed[nb])
                            copy_in(nb)
                            copied[nb].record(copy_stream)
                    compute.wait_event(copied[b])
                    res = step(xd[b])
                    consumed[b].record(compute)
                    with torch.cuda.stream(copy_stream):
                        copy_stream.wait_event(consumed[b])
                        for h, o in zip(hout, res):
                            o.record_stream(copy_stream)
                            h.copy_(o, non_blocking=True)
                compute.wait_stream(copy_stream)           # before the end event

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
            api = ("cherimoya_b200.variant_effect(model, X_ref, X_alt)" if variant
                   else "Cherimoya.forward(X)")
            e2e = {"value": world * args.batch * args.steps / (e2e_ms / 1000.0),
                   "unit": unit, "h2d_bytes_per_step": sum(x.numel() * x.element_size()
                                                           for x in hin),
                   "d2h_bytes_per_step": sum(h.numel() * h.element_size() for h in hout),
                   "api": api + " on pinned host one-hot fp32 input; the next step's "
                                "H2D copy overlaps the current step"}

        # ---- saturation mutagenesis: 256 sequences x all 3 x 2114 single-base
        # substitutions (1,623,552 mutants), the sequences split into contiguous
        # shards over the ranks. Timed per rank from the H2D copy of its shard's
        # bases (pinned host int8) through the all-gather of every rank's scores
        # and their D2H copy into pinned host memory on rank 0.
        ism = None
        if args.ism_seqs > 0 and args.workload == "forward":
            from cherimoya_b200.ism import gather_shards, shard_range
            n_seq = args.ism_seqs
            all_bases = torch.randint(0, 4, (n_seq, L),
                                      generator=torch.Generator().manual_seed(100))
            lo, hi = shard_range(n_seq, rank, world)
            h_bases = all_bases[lo:hi].to(torch.int8).pin_memory()
            warm = h_bases[:1].to(dev)
            cb.saturation_mutagenesis(model, warm, 1000, 1010)         # warm-up
            h_d = h_j = None
            if rank == 0:
                h_d = torch.empty((n_seq, model.n_groups, 4, L), dtype=torch.float32,
                                  pin_memory=True)
                h_j = torch.empty((n_seq, 4, L), dtype=torch.float32, pin_memory=True)
            torch.cuda.synchronize()
            barrier(world)
            i_s = torch.cuda.Event(enable_timing=True)
            i_e = torch.cuda.Event(enable_timing=True)
            i_s.record()
            d_bases = h_bases.to(dev, non_blocking=True)
            d, j = cb.saturation_mutagenesis(model, d_bases, 0, L, mutant_batch=4096)
            if world > 1:
                d, j = gather_shards(d, n_seq), gather_shards(j, n_seq)
            if rank == 0:
                h_d.copy_(d, non_blocking=True)
                h_j.copy_(j, non_blocking=True)
            i_e.record()
            torch.cuda.synchronize()
            barrier(world)
            ism_ms = max_over_ranks(i_s.elapsed_time(i_e), world, dev)
            n_mut = n_seq * 3 * L
            ism = {"value": n_mut / (ism_ms / 1000.0), "unit": "mutants/s",
                   "mutants": n_mut, "ms": ism_ms, "n_gpus": world,
                   "scaling": "strong",
                   "h2d_bytes": n_seq * L, "d2h_bytes": 4 * n_seq * L * (model.n_groups + 1) * 4,
                   "workload": "{} random 2114-bp sequences (global, split over {} GPU(s)) x all "
                               "3x2114 single-base substitutions, delta log-count + profile JSD "
                               "per mutant, {} mode; H2D of bases, all-gather and D2H of the "
                               "scores inside the timed region".format(n_seq, world, args.mode)}

        # ---- the multi-task and variant-scoring configurations, a few
        # device-resident steps each (part of the default forward run)
        others = None
        if args.workload == "forward" and not args.no_other_configs:
            others = {name: time_other_workload(name, args, world, rank, dev)
                      for name in ("multitask", "variant")}

        # ---- variant scoring of --variant-pairs ref/alt pairs in total (the
        # variant configuration as stated: 1M pairs), split into contiguous shards
        # over the ranks; timed per rank from the H2D copy of its shard's bases
        # (pinned host int8, ref and alt) through the all-gather of every rank's
        # scores and their D2H copy on rank 0
        var_run = None
        if variant and args.variant_pairs > 0:
            from cherimoya_b200.ism import gather_shards, shard_range
            n_tot = args.variant_pairs
            lo, hi = shard_range(n_tot, rank, world)
            n_loc = hi - lo
            g = torch.Generator().manual_seed(3000 + rank)
            ref_b = torch.randint(0, 4, (n_loc, L), generator=g, dtype=torch.int8)
            alt_b = ref_b.clone()
            c = L // 2
            alt_b[:, c] = ((ref_b[:, c].long() + torch.randint(1, 4, (n_loc,), generator=g))
                           % 4).to(torch.int8)
            h_ref, h_alt = ref_b.pin_memory(), alt_b.pin_memory()
            cb.variant_effect(model, h_ref[:8].to(dev), h_alt[:8].to(dev))       # warm-up
            h_vd = h_vj = None
            if rank == 0:
                h_vd = torch.empty((n_tot, model.n_groups), dtype=torch.float32,
                                   pin_memory=True)
                h_vj = torch.empty((n_tot,), dtype=torch.float32, pin_memory=True)
            torch.cuda.synchronize()
            barrier(world)
            v_s = torch.cuda.Event(enable_timing=True)
            v_e = torch.cuda.Event(enable_timing=True)
            v_s.record()
            d_ref = h_ref.to(dev, non_blocking=True)
            d_alt = h_alt.to(dev, non_blocking=True)
            vd, vj = cb.variant_effect(model, d_ref, d_alt)
            if world > 1:
                vd, vj = gather_shards(vd, n_tot), gather_shards(vj, n_tot)
            if rank == 0:
                h_vd.copy_(vd, non_blocking=True)
                h_vj.copy_(vj, non_blocking=True)
            v_e.record()
            torch.cuda.synchronize()
            barrier(world)
            v_ms = max_over_ranks(v_s.elapsed_time(v_e), world, dev)
            var_run = {"value": n_tot / (v_ms / 1000.0), "unit": "pairs/s", "pairs": n_tot,
                       "ms": v_ms, "n_gpus": world, "scaling": "strong",
                       "h2d_bytes": 2 * n_tot * L, "d2h_bytes": 4 * n_tot * (model.n_groups + 1),
                       "workload": "{} random 2114-bp ref/alt pairs (global, split over {} "
                                   "GPU(s)), alt = one SNV at the centre, delta log-count + "
                                   "profile JSD per pair, {} mode; H2D of bases, all-gather "
                                   "and D2H of the scores inside the timed region".format(
                                       n_tot, world, args.mode)}

    peaks, peak_src = load_peaks()
    mlp_ms, mlp_n = per_class["mlp"]
    mlp_avg_ms = mlp_ms / max(mlp_n, 1)
    # tensor work of the MLP launches of the instrumented steps over their
    # device time (events on the launching stream around every launch)
    mlp_flop_step = mlp_flop_per_seq(model) * forwards * args.batch
    achieved = mlp_flop_step * n_inst / (mlp_ms / 1000.0) / 1e12
    # a millisecond-long step runs at the burst clock: the burst peak applies
    peak = peaks["bf16_tflops"]
    model_tflops = value / world * forwards * flop_per_seq(model) / 1e12
    default_width = model.n_filters == 128 and model.expansion == 2
    C, H = model.n_filters, model.n_filters * model.expansion
    roofline = {
        "bound": "tensor",
        "kernel": ("mlp_ws_kernel" if default_width
                   else "mlp_wide_kernel" if C == 256 and args.mode == "bf16"
                   else "mlp_stream_kernel") + " (tcgen05 conv+LN+MLP+residual, one layer)",
        "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
        "peak_source": "{} bf16_tflops (burst)".format(peak_src),
        "frac_of_sustained": achieved / peaks["bf16_tflops_sustained"],
        # DRAM bytes of one MLP launch of the default-width backbone: ncu
        # dram__bytes_read.sum + write.sum averaged over the nine launches of
        # a forward at batch 256, scaled by the sequences processed
        "traffic": (MLP_DRAM_BYTES_PER_SEQ * args.batch
                    if args.mode == "bf16" and default_width and not variant else None),
        "traffic_unit": "bytes per launch",
        "algorithmic_bytes": 2.0 * L * C * (2 if args.mode == "bf16" else 4) * args.batch,
        "flop_per_launch": 4.0 * C * H * L * args.batch, "avg_launch_ms": mlp_avg_ms,
        "whole_forward": {
            "tflops_per_gpu": model_tflops, "flop_per_unit": forwards * flop_per_seq(model),
            "frac": model_tflops / peak,
            "frac_of_sustained": model_tflops / peaks["bf16_tflops_sustained"]},
        "kernel_share": {k: v[0] / max(inst_ms, 1e-9) for k, v in per_class.items() if v[1]},
        "instrumented_steps": n_inst,
    }
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        n_cpu = args.cpu_sample if not variant else max(1, args.cpu_sample // 8)
        rate, cores, reps, kind = cpu_forward_rate(args, n_cpu)
        cpu = {"value": rate, "unit": unit, "cores": cores, "kind": kind,
               "sample": "{} {}, fp32 eager no_grad, median of {} reps, {}".format(
                   n_cpu, unit.split("/")[0], reps, REF_WHAT[kind])}
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": dev_ms_max / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16" if args.mode == "bf16" else "f32", "data": "synthetic",
            "config": workload_config(args, world),
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "ism": ism,
            "variant_pairs": var_run, "other_configs": others,
            "clocks": clocks, "gpu_launches": launches_per_step * args.steps,
        }
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=int(os.environ.get("WORLD_SIZE", "1")))
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference", "reference-gpu"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="forward")
    ap.add_argument("--batch", type=int, default=None,
                    help="units per GPU per step (default: the workload's)")
    ap.add_argument("--mode", choices=["bf16", "fp32"], default="bf16")
    ap.add_argument("--ism-seqs", type=int, default=256,
                    help="ISM sequences in total, split over the ranks (0: skip)")
    ap.add_argument("--variant-pairs", type=int, default=0,
                    help="variant workload: also score this many pairs in total, split "
                         "over the ranks, with host I/O timed (0: skip)")
    ap.add_argument("--cpu-sample", type=int, default=32)
    ap.add_argument("--ref-sample", type=int, default=16)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-other-configs", action="store_true",
                    help="forward workload: skip timing the multi-task and variant steps")
    args = ap.parse_args()
    if args.batch is None:
        args.batch = WORKLOADS[args.workload][1]
    world, rank, local = dist_setup()
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        elif args.impl == "reference-gpu":
            run_reference_gpu(args, world, rank, local)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
