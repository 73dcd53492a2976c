#!/usr/bin/env python
"""Benchmark: Gaussian-field delta-W render, forward + backward, whole SD1.5 UNet.

Workload: the 128 attention-projection fields of an SD1.5
UNet (widths 320/640/1280, cross-attention k/v 768 wide; 93,511,680 delta
elements), K=256 Gaussians each with config 1's distributions, seeded synthetic
parameters and upstream gradients (no dataset exists for this path).  One step =
forward render of every field (bf16 delta, fp32 accumulation) + all-gather of
the bf16 delta across ranks + backward (fp32 dL/d(delta) -> d_mu, d_chol_raw,
d_amp).  Fields are partitioned across ranks by measured render cost; the total
work is fixed as N grows (strong scaling).

Metric: delta elements rendered forward+backward per second, whole job.
value  -- device time of the step, inputs resident in HBM (CUDA events, max over ranks)
e2e    -- the same step through the whole-model API (guass_b200.batched /
          partition) with this rank's packed parameters and dL/d(delta) copied
          from pinned host memory and the packed gradients copied back, every
          step
e2e_dropin_per_layer -- the same, one call per layer through the drop-in API
          (guass_b200.cuda_field), as GUASS's own layers would call it
cpu_baseline / --impl reference -- the CPU oracle (a C restatement of the
          reference kernels, OpenMP over all host cores) on a bounded sample

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
       (N > 1 under torch.distributed.run; one process per GPU)
"""
from __future__ import annotations

import argparse
import ctypes
import csv
import io
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

METRIC = "Gaussian-field dW fwd+bwd elements/s (whole SD1.5 UNet, 128 projections, K=256)"
UNIT = "elements/s"
# FMA-pipe operations per (element, Gaussian) evaluation, per the survey's
# roofline definition (forward ~9, backward ~25).


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="budget of the CPU-baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--exchange", choices=["auto", "multicast", "fused", "nccl"], default="auto",
                    help="delta exchange for N > 1 (auto = nccl; multicast = NVLink multicast publish after each "
                         "render group; fused = the render kernel stores through the multicast address)")
    ap.add_argument("--groups", type=int, default=4, help="forward field groups per rank (multicast exchange)")
    ap.add_argument("--workload", choices=["cfg3", "cfg4"], default="cfg3",
                    help="cfg3: whole-UNet batched render (default, the headline); cfg4: data-parallel "
                         "SD1.5-UNet adapter training step")
    ap.add_argument("--adapter-apply", choices=["fused", "reference", "dropin"], default="fused",
                    help="cfg4: one batched render and one GEMM on W0+delta (fused); one batched render and the "
                         "reference layer's base GEMM + row-chunked delta GEMMs (reference); every layer rendering "
                         "itself through the drop-in runtime, the reference's call pattern (dropin)")
    ap.add_argument("--batch", type=int, default=4, help="cfg4: samples per GPU")
    ap.add_argument("--bwd-exp", choices=["expf", "ex2"], default="ex2",
                    help="backward basis: the base-2 hardware approximation (GF_CFG_BWD_EXP2, default; held to the "
                         "same gradient tolerance) or CUDA expf as the reference; the line reports both")
    ap.add_argument("--fwd-exp", choices=["expf", "ex2"], default="ex2",
                    help="bf16 forward basis: the base-2 hardware approximation (GF_CFG_FWD_EXP2, default; within the "
                         "bf16 tolerance) or CUDA expf (the RNE cast of the reference's fp32 sum)")
    ap.add_argument("--no-configs", action="store_true", help="skip the cfg1/cfg2 single-field lines and the "
                    "reference-extension timings (N=1)")
    ap.add_argument("--fields", type=int, default=128,
                    help="cfg3 slice for profiling: this many of the 128 fields, spread over the UNet's widths")
    ap.add_argument("--profile-field", choices=["cfg1", "cfg2", "dense4096", "dense16384"], default=None,
                    help="with --profile-case: one field of that configuration instead of the cfg3 slice")
    ap.add_argument("--profile-case", action="store_true",
                    help="only run warm-up + steps of the workload eagerly and exit (the command that the ncu "
                         "summaries under profiles/ capture)")
    a = ap.parse_args()
    a.warmup = max(3, a.warmup)
    return a


# ---------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi clock/throttle samples every 50 ms while running."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.proc = None
        self.t0 = self.t1 = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def mark(self, which):
        setattr(self, which, time.time())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        rows = []
        for rec in csv.reader(io.StringIO(out)):
            if len(rec) < 10:
                continue
            try:
                ts = time.mktime(time.strptime(rec[0].strip().split(".")[0], "%Y/%m/%d %H:%M:%S"))
                rows.append((ts, [x.strip() for x in rec[1:]]))
            except ValueError:
                continue
        lo, hi = (self.t0 or 0) - 1.0, (self.t1 or time.time()) + 1.0
        win = [r for ts, r in rows if lo <= ts <= hi] or [r for _, r in rows]
        sm = [float(r[1]) for r in win if r[1].replace(".", "", 1).isdigit()]
        mx = [float(r[2]) for r in win if r[2].replace(".", "", 1).isdigit()]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for r in win for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        loaded = [s for s in sm if mx and s > 0.5 * max(mx)] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(win)}


# ---------------------------------------------------------------------------
def setup_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# ---------------------------------------------------------------------------
class UNetWorkload:
    """Fields of the whole UNet, partitioned; this rank's batch and buffers."""

    def __init__(self, rank: int, world: int, exchange: str = "auto", groups: int = 4, bwd_exp2: bool = False,
                 fwd_exp2: bool = False, num_fields: int = 128):
        from guass_b200 import synthetic
        from guass_b200.batched import FieldBatch, pack_fields
        from guass_b200.partition import PartitionedRenderer, field_costs

        self.rank, self.world = rank, world
        self.fields = synthetic.cfg3()
        if num_fields < len(self.fields):
            keep = sorted(interleaved_order(len(self.fields))[:max(1, num_fields)])
            self.fields = [self.fields[i] for i in keep]
        shapes = [(f.out_features, f.in_features, f.k) for f in self.fields]
        self.numels = [f.numel for f in self.fields]
        self.total_elements = sum(self.numels)
        # exact per-field cost from one binning pass over all fields
        full = FieldBatch(shapes)
        mu, chol, amp, _ = pack_fields(self.fields, device="cuda")
        while full.ensure_capacity(mu, chol, amp):
            pass
        full.forward(mu, chol, amp)
        tps = [full.tile_ptr_view(i).cpu() for i in range(len(shapes))]
        self.costs = field_costs(tps, [(s[0], s[1]) for s in shapes])
        self.total_evals = sum(self.costs)
        self.total_pairs = full.total_pairs()
        del full, mu, chol, amp
        use_mc = {"auto": False, "multicast": True, "fused": True, "nccl": False}[exchange]
        self.renderer = PartitionedRenderer(shapes, self.costs, rank, world, groups=groups, use_multicast=use_mc,
                                            fused=(exchange == "fused"), bwd_exp2=bwd_exp2,
                                            fwd_exp2=fwd_exp2)
        self.parts, self.own = self.renderer.parts, self.renderer.own
        self.layout, self.gathered = self.renderer.layout, self.renderer.gathered
        own_fields = [self.fields[i] for i in self.own]
        self.mu, self.chol, self.amp, self.grad = pack_fields(own_fields, device="cuda")
        self.renderer.ensure_capacity(self.mu, self.chol, self.amp)
        assert self.renderer.device_flags() == 0
        self.own_evals = sum(self.costs[i] for i in self.own)

    def step(self):
        self.renderer.step(self.mu, self.chol, self.amp, self.grad)


def run_device_timed(w: UNetWorkload, steps: int, warmup: int, world: int):
    from guass_b200 import _lib

    L = _lib.lib()
    for _ in range(warmup):
        w.step()
    torch.cuda.synchronize()
    # per step: the library's trace events in host call order (gfield.h, gf_trace_events)
    per_step = w.renderer.trace_events_per_step()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(per_step * steps)]
    for e in evs:
        e.record()
    torch.cuda.synchronize()
    handles = (ctypes.c_void_p * max(1, len(evs)))(*[e.cuda_event for e in evs])
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    _lib.check(L.gf_trace_events(handles, len(evs)))
    w.renderer.gather_events = [] if world > 1 else None
    start.record()
    for _ in range(steps):
        w.step()
    end.record()
    torch.cuda.synchronize()
    barrier(world)
    recorded = L.gf_trace_count()
    _lib.check(L.gf_trace_events(None, 0))
    assert recorded == len(evs), (recorded, len(evs))
    ms = start.elapsed_time(end) / steps
    per = {n: [] for n in ("bin", "render_fwd", "bwd_prep", "render_bwd", "bwd_finalize")}
    for s_ in range(steps if per_step else 0):
        for k, v in w.renderer.kernel_times(evs[per_step * s_: per_step * (s_ + 1)]).items():
            per[k].append(v)
    if world > 1:
        per["exchange_side_stream"] = [a.elapsed_time(b) for a, b in w.renderer.gather_events]
        w.renderer.gather_events = None
    kern = {k: (sum(v) / len(v) if v else 0.0) for k, v in per.items()}  # same keys on every rank
    return ms, kern


def run_graph_timed(w: UNetWorkload, steps: int, warmup: int, world: int) -> float:
    """The timed region: ``steps`` replays of the captured step."""
    w.renderer.capture(w.mu, w.chol, w.amp, w.grad, warmup=2)
    for _ in range(warmup):
        w.renderer.replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    start.record()
    for _ in range(steps):
        w.renderer.replay()
    end.record()
    torch.cuda.synchronize()
    barrier(world)
    return start.elapsed_time(end) / steps


def run_e2e_batched(w: UNetWorkload, steps: int, warmup: int, world: int):
    """The step through the whole-model API with host buffers: every step
    copies this rank's packed parameters and dL/d(delta) from pinned host
    memory, runs the partitioned render (the same ``renderer.step`` as the
    device-timed loop) and copies the packed gradients back.

    Double-buffered: two device input sets; step k+1's inputs are copied on
    a copy stream while step k computes (every step still moves all of its
    own bytes; the timed region starts before step 0's copy and ends after
    the last step's gradients have reached the host)."""
    h_in = [t.detach().cpu().pin_memory() for t in (w.mu, w.chol, w.amp, w.grad)]
    bufs = [tuple(t.clone() for t in (w.mu, w.chol, w.amp, w.grad)) for _ in range(2)]
    outs = w.renderer.step(*bufs[0])
    h_out = [[t.detach().cpu().pin_memory() for t in g] for g in outs]
    h2d = sum(t.numel() * t.element_size() for t in h_in)
    d2h = sum(t.numel() * t.element_size() for g in h_out for t in g)
    main = torch.cuda.current_stream()
    copy = torch.cuda.Stream()
    copied = [torch.cuda.Event(), torch.cuda.Event()]
    used = [torch.cuda.Event(), torch.cuda.Event()]

    def issue_copy(slot):
        with torch.cuda.stream(copy):
            copy.wait_event(used[slot])  # the step that last read this set is done
            for h, d in zip(h_in, bufs[slot]):
                d.copy_(h, non_blocking=True)
            copied[slot].record(copy)

    def run(n):
        copy.wait_stream(main)
        issue_copy(0)
        for k in range(n):
            slot = k % 2
            main.wait_event(copied[slot])
            if k + 1 < n:
                issue_copy(1 - slot)
            outs = w.renderer.step(*bufs[slot])
            used[slot].record(main)
            for hg, dg in zip(h_out, outs):
                for h, d in zip(hg, dg):
                    h.copy_(d, non_blocking=True)

    run(warmup)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    start.record()
    run(steps)
    end.record()
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(end) / steps, world)
    return ms, sum_over_ranks(h2d, world), sum_over_ranks(d2h, world)


def run_e2e_model(w: UNetWorkload, steps: int, warmup: int, world: int, mode: str):
    """The same step through GUASS's layer API: a model of this rank's
    projection layers (GaussianLinear's interface, guass_b200.sd15.
    GaussianProjection, with this workload's shapes and K), whose forward asks
    every layer for ``compute_delta_weight()`` as GaussianLinear.forward does
    (gaussian_linear.py:162-242), then one autograd backward with each layer's
    dL/d(delta).  ``mode`` "dropin": every layer renders itself through the
    drop-in runtime (gaussian_field_train, the reference's call pattern);
    "model_renderer": adapters.ModelRenderer serves every layer from one
    batched render per model forward.  Every step copies the layers'
    parameters and dL/d(delta) from pinned host memory and the parameter
    gradients back; the model runs all layer forwards before the backward."""
    from torch import nn

    from guass_b200 import sd15
    from guass_b200.adapters import ModelRenderer

    settings = sd15.AdapterSettings()
    layers = nn.ModuleList()
    for n, i in enumerate(w.own):
        f = w.fields[i]
        layers.append(sd15.GaussianProjection(f.in_features, f.out_features, False, f.k, seed=i,
                                              dtype=torch.bfloat16, settings=settings))

    class DeltaModel(nn.Module):
        def __init__(self, layers):
            super().__init__()
            self.layers = layers

        def forward(self):
            return [m.compute_delta_weight() for m in self.layers]

    model = DeltaModel(layers).cuda()
    if mode == "dropin":
        sd15.PerLayerRender({str(n): m for n, m in enumerate(layers)}).install()
    else:
        ModelRenderer(model, out_dtype=torch.bfloat16)
    params = [p for m in layers for p in (m.mu_raw, m.chol_raw, m.amp)]
    # dL/d(delta) in the dtype autograd hands each layer's delta (bf16 under
    # ModelRenderer, fp32 from the per-layer drop-in)
    with torch.no_grad():
        delta_dtype = model()[0].dtype

    def flat(tensors, dtype, pinned):
        n = sum(t.numel() for t in tensors)
        buf = torch.empty(n, dtype=dtype, pin_memory=True) if pinned else torch.empty(n, dtype=dtype, device="cuda")
        views, o = [], 0
        for t in tensors:
            views.append(buf[o:o + t.numel()].view(t.shape))
            o += t.numel()
        return buf, views

    # one pinned staging buffer per direction: three copies per step instead of
    # one per tensor (the layers' parameters stay separate nn.Parameters)
    h_params, h_pviews = flat(params, torch.float32, True)
    d_params, d_pviews = flat(params, torch.float32, False)
    for hv, p in zip(h_pviews, params):
        hv.copy_(p.detach().cpu())
    grads_src = [w.fields[i].grad.view(w.fields[i].out_features, w.fields[i].in_features) for i in w.own]
    h_grads, h_gviews = flat(grads_src, delta_dtype, True)
    for hv, g in zip(h_gviews, grads_src):
        hv.copy_(g)
    d_grads, d_gviews = flat(grads_src, delta_dtype, False)
    h_out, _ = flat(params, torch.float32, True)
    d_out, d_oviews = flat(params, torch.float32, False)
    h2d = h_params.numel() * 4 + h_grads.numel() * h_grads.element_size()
    d2h = h_out.numel() * 4

    def step():
        with torch.no_grad():
            d_params.copy_(h_params, non_blocking=True)
            torch._foreach_copy_(params, d_pviews)
            d_grads.copy_(h_grads, non_blocking=True)
        deltas = model()
        torch.autograd.backward(deltas, d_gviews)
        with torch.no_grad():
            torch._foreach_copy_(d_oviews, [p.grad for p in params])
            h_out.copy_(d_out, non_blocking=True)
        for p in params:
            p.grad = None

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    start.record()
    for _ in range(steps):
        step()
    end.record()
    torch.cuda.synchronize()
    barrier(world)
    ms = max_over_ranks(start.elapsed_time(end) / steps, world)
    return ms, sum_over_ranks(h2d, world), sum_over_ranks(d2h, world)


# ---------------------------------------------------------------------------
def cpu_oracle_sample(fields, budget_s: float, order=None):
    """Run the CPU oracle fwd+bwd over fields (in ``order``) until the time
    budget is used (at least one field).  Returns (elements, seconds, names)."""
    import oracle

    order = order if order is not None else list(range(len(fields)))
    done_el, done_t, names = 0, 0.0, []
    for i in order:
        f = fields[i]
        t0 = time.perf_counter()
        d, tp, ids = oracle.forward(f.row_coords, f.col_coords, f.mu, f.chol_raw, f.amp)
        oracle.backward(f.grad, f.row_coords, f.col_coords, f.mu, f.chol_raw, f.amp, tp, ids)
        done_t += time.perf_counter() - t0
        done_el += f.numel
        names.append(f.name)
        if done_t >= budget_s:
            break
    return done_el, done_t, names


def interleaved_order(n=128, stride=16):
    return [i for s in range(stride) for i in range(s, n, stride)]


def host_threads() -> int:
    """Every host core this process may run on.  Set explicitly: under
    torch.distributed.run OMP_NUM_THREADS defaults to 1, which would time the
    CPU path single-threaded at N > 1."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_baseline(fields, budget_s):
    import oracle

    oracle.build()
    oracle.set_threads(host_threads())
    threads = oracle.max_threads()
    el, t, names = cpu_oracle_sample(fields, budget_s, interleaved_order(len(fields)))
    return {"value": el / t, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{len(names)} of {len(fields)} fields ({el} elements, fwd+bwd) in {t:.2f} s, "
                      f"OpenMP x{threads} threads, C restatement of the reference kernels (oracle/)"}


def reference_arm(a, rank, world):
    """--impl reference: the reference algorithm on the host cores (the CPU
    oracle, since the reference's own CPU path is PyTorch code that cannot be
    shipped to the GPU box), bounded samples per step."""
    if rank != 0:
        return
    from guass_b200 import synthetic
    import oracle

    oracle.build()
    oracle.set_threads(host_threads())
    fields = synthetic.cfg3()
    order = interleaved_order(len(fields))
    per_step = max(1, len(fields) // 16)
    threads = oracle.max_threads()
    for s in range(a.warmup):
        sub = [order[(s * per_step + j) % len(order)] for j in range(per_step)]
        cpu_oracle_sample(fields, 1e9, sub)
    tot_el, tot_t = 0, 0.0
    for s in range(a.steps):
        sub = [order[(s * per_step + j) % len(order)] for j in range(per_step)]
        el, t, _ = cpu_oracle_sample(fields, 1e9, sub)
        tot_el += el
        tot_t += t
    value = tot_el / tot_t
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": 1e3 * tot_t / a.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, BASELINE cfg3 shapes)",
            "config": {"workload": "cfg3 whole-UNet, 128 projection fields, K=256", "sample_per_step":
                       f"{per_step} of 128 fields, fwd+bwd", "elements_per_step_avg": tot_el / a.steps},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": f"{per_step} fields per step x {a.steps} steps, OpenMP x{threads}"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# Rooflines.  The render kernels are neither a contraction nor HBM-bound (2-4
# bytes per element against ~14 evaluations of the basis per element); they
# are bound by one of three SM resources, per evaluation:
#   issue  -- warp-instruction issue, 4 warp instructions (128 thread
#             instructions) per SM per clock
#   fp32   -- the FP32 lanes, 128 lane-operations per SM per clock (a packed
#             f32x2 instruction is two operations)
#   sfu    -- MUFU (ex2), 16 per SM per clock
# The per-evaluation counts come from ncu instruction counters of the same
# kernel (profiles/<kernel>.json); achieved = count x evaluations / CUDA-event
# time of the launch, peak = SMs x rate x the SM clock sampled during the run.
PIPE_RATE = {"issue": 128, "fp32": 128, "sfu": 16}
PIPE_KEY = {"issue": "thread_inst", "fp32": "fp32_lane_ops", "sfu": "xu_thread_inst"}


def load_counters(name: str):
    p = ROOT / "profiles" / f"{name}.json"
    if not p.exists():
        return None
    try:
        return json.loads(p.read_text())
    except ValueError:
        return None


def kernel_name(kind: str, ex2: bool) -> str:
    return f"{kind}32_{'ex2' if ex2 else 'expf'}"


def pipe_roofline(name: str, evals: float, elements: float, ms: float, f_mhz: float, sm_count: int):
    prof = load_counters(name)
    if prof is None or ms <= 0:
        return None
    pipes = {}
    for pipe, rate in PIPE_RATE.items():
        per = float(prof["per_eval"][PIPE_KEY[pipe]])
        achieved = per * evals / (ms / 1e3) / 1e12
        peak = sm_count * rate * f_mhz * 1e6 / 1e12
        pipes[pipe] = {"ops_per_eval": per, "achieved": achieved, "peak": peak, "frac": achieved / peak}
    bound = max(pipes, key=lambda k: pipes[k]["frac"])
    per_el = prof.get("dram_bytes_per_element")
    return {"kernel": name, "bound": bound, "achieved": pipes[bound]["achieved"], "peak": pipes[bound]["peak"],
            "unit": "Tops/s", "frac": pipes[bound]["frac"],
            "traffic": per_el * elements if per_el is not None else None,
            "pipes": pipes, "counters": f"profiles/{name}.json",
            "definition": f"per-evaluation counts from ncu counters x {int(evals)} evaluations / CUDA-event launch "
                          f"time; peaks = {sm_count} SMs x (issue 128, fp32 128, sfu 16) per clock x {f_mhz:.0f} MHz "
                          "(sampled); bound = the resource with the largest fraction; traffic = ncu DRAM bytes "
                          "per delta element x elements"}


def step_roofline(evals_total, bytes_step, ms, sm_count, f_mhz, hbm_peak, world, fwd_name, bwd_name):
    """Whole-step bound: t_bound = sum over the two render kernels of their
    binding resource's time at peak (counter-derived), against HBM bytes / BW."""
    clk = f_mhz * 1e6
    terms = {"hbm_ms": bytes_step / (hbm_peak * 1e9 * world) * 1e3}
    t_kernels = 0.0
    for name in (fwd_name, bwd_name):
        prof = load_counters(name)
        if prof is None:
            return None
        t = max(float(prof["per_eval"][PIPE_KEY[p]]) * evals_total / (sm_count * r * clk * world)
                for p, r in PIPE_RATE.items())
        terms[name + "_ms"] = t * 1e3
        t_kernels += t * 1e3
    t_bound = max(terms["hbm_ms"], t_kernels)
    return {"t_bound_ms": t_bound, "t_measured_ms": ms, "frac": t_bound / ms, "terms": terms, "clock_mhz": f_mhz,
            "definition": "t_bound = max(HBM bytes / MEASURED_PEAKS hbm_gbs, sum over the forward and backward "
                          "render of their binding resource at peak) / t_measured"}


# ---------------------------------------------------------------------------
def time_single_field(f, fwd_exp2: bool, bwd_exp2: bool, out_dtype, steps: int, warmup: int):
    """One field (FieldBatch of 1): forward + backward per step, CUDA events."""
    from guass_b200 import _lib
    from guass_b200.batched import FieldBatch, pack_fields
    from guass_b200.partition import field_costs

    L = _lib.lib()
    b = FieldBatch([(f.out_features, f.in_features, f.k)], out_dtype=out_dtype, fwd_exp2=fwd_exp2,
                   bwd_exp2=bwd_exp2)
    mu, chol, amp, grad = pack_fields([f], device="cuda")
    while b.ensure_capacity(mu, chol, amp):
        pass
    evals = field_costs([b.tile_ptr_view(0).cpu()], [(f.out_features, f.in_features)])[0]

    def step():
        b.forward(mu, chol, amp)
        b.backward(grad, mu, chol, amp)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(7 * steps)]
    for e in evs:
        e.record()
    torch.cuda.synchronize()
    handles = (ctypes.c_void_p * len(evs))(*[e.cuda_event for e in evs])
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _lib.check(L.gf_trace_events(handles, len(evs)))
    start.record()
    for _ in range(steps):
        step()
    end.record()
    torch.cuda.synchronize()
    _lib.check(L.gf_trace_events(None, 0))
    assert b.device_flags() == 0
    ms = start.elapsed_time(end) / steps
    kern = {"bin": 0.0, "render_fwd": 0.0, "render_bwd": 0.0}
    for s_ in range(steps):
        e = evs[7 * s_: 7 * s_ + 7]
        kern["bin"] += e[0].elapsed_time(e[1]) / steps
        kern["render_fwd"] += e[1].elapsed_time(e[2]) / steps
        kern["render_bwd"] += e[4].elapsed_time(e[5]) / steps
    return ms, kern, evals


def time_reference_cuda(fields, out_bf16: bool, steps: int, warmup: int):
    """The reference's own CUDA extension (built unmodified into oracle/_ref),
    called per field as GaussianLinear does: forward (fp32 delta, + the layer's
    bf16 cast where the config stores bf16), then the training backward.
    CUDA events on the stream it uses (the current one); its host reads of
    the pair count are part of its time.  None when the build is absent."""
    try:
        from oracle import build_ref
        ext = build_ref.load()
    except (FileNotFoundError, ImportError, OSError):
        return None
    dev = [f.to("cuda") for f in fields]

    def step():
        for d in dev:
            delta, tp, ids = ext.gaussian_field_forward(d.row_coords, d.col_coords, d.mu, d.chol_raw, d.amp, 32, 32,
                                                        3.0, False, 80.0)
            if out_bf16:
                delta.to(torch.bfloat16)
            ext.gaussian_field_backward(d.grad, d.row_coords, d.col_coords, d.mu, d.chol_raw, d.amp, tp, ids, 32, 32,
                                        3.0, False, 80.0)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        step()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / steps


def time_dropin_train(f, steps: int, warmup: int):
    """The drop-in training call GUASS's layers make (gaussian_field_train,
    fp32 delta, its autograd backward) on one field: ms per forward+backward
    and the peak device memory it adds."""
    from guass_b200 import cuda_field

    d = f.to("cuda")
    mu, chol, amp = (t.clone().requires_grad_(True) for t in (d.mu, d.chol_raw, d.amp))

    def step():
        delta = cuda_field.gaussian_field_train(row_coords=d.row_coords, col_coords=d.col_coords, mu=mu,
                                                chol_raw=chol, amp=amp, tile_out=32, tile_in=32, sigma_multiplier=3.0)
        delta.backward(d.grad)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    base = torch.cuda.memory_allocated()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        step()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / steps, torch.cuda.max_memory_allocated() - base


def dense_rows(a, ns_per_eval_fwd: float):
    """Densified layers (1280x1280, K = 4096 and 16384).  The BIN stage emits
    and sorts (tile, id) pairs, so its cost follows the pair count, not K x
    tiles: each row reports it beside the step (``bin_share``).  The forward
    render is compared with its work at the whole-UNet rate per evaluation:
    one field is 1600 tiles, a launch too small to fill the GPU the way the
    91 k tiles of the UNet do (``small_launch_excess_share``)."""
    from guass_b200 import synthetic

    rows = {}
    for k in (4096, 16384):
        f = synthetic.densified(k)
        ms, kern, evals = time_single_field(f, a.fwd_exp == "ex2", a.bwd_exp == "ex2", torch.bfloat16, 20, 3)
        work_ms = evals * ns_per_eval_fwd * 1e-6
        t_ms, peak = time_dropin_train(f, 5, 2)
        rows[f"dense{k}"] = {
            "workload": f"1280x1280 field, K={k} (densified: log s ~ N(log(0.02*sqrt(1024/K)), 0.3)), bf16 delta",
            "ms_per_step": ms, "value": f.numel / (ms / 1e3), "unit": "elements/s", "evals": evals,
            "kernels_ms": kern, "render_fwd_at_unet_rate_ms": work_ms,
            "bin_share": kern["bin"] / ms,
            "small_launch_excess_share": max(0.0, kern["render_fwd"] - work_ms) / kern["render_fwd"],
            "dropin_train": {"ms_per_step": t_ms, "peak_bytes": peak,
                             "k_times_tiles_bound_bytes": 40 * k * 1600,
                             "path": "cuda_field.gaussian_field_train + autograd backward, fp32 delta"}}
    return rows


def single_field_configs(a, f_mhz, sm_count):
    """BASELINE configs 1 and 2 at N=1: one field each, forward + backward."""
    from guass_b200 import synthetic

    out = {}
    for name, f, out_dtype, dt in (("cfg1", synthetic.cfg1(), torch.bfloat16, "bf16"),
                                   ("cfg2", synthetic.cfg2(), torch.float32, "f32")):
        fx = a.fwd_exp == "ex2" and out_dtype == torch.bfloat16
        bx = a.bwd_exp == "ex2"
        steps = max(a.steps, 20)
        ms, kern, evals = time_single_field(f, fx, bx, out_dtype, steps, a.warmup)
        ms_ref_basis, _, _ = time_single_field(f, False, False, out_dtype, steps, a.warmup)
        ref_ms = time_reference_cuda([f], out_dtype == torch.bfloat16, max(3, steps // 4), 2)
        dom = max(("render_fwd", "render_bwd"), key=kern.get)
        kind = dom
        out[name] = {
            "workload": f"{name}: {f.out_features}x{f.in_features} field, K={f.k}, {dt} delta, f32 dL/d(delta)",
            "value": f.numel / (ms / 1e3), "unit": "elements/s", "ms_per_step": ms, "evals": evals,
            "forward_basis": "ex2.approx" if fx else "expf", "backward_basis": "ex2.approx" if bx else "expf",
            "kernels_ms": kern,
            "roofline": pipe_roofline(kernel_name(kind, fx if kind == "render_fwd" else bx), evals, f.numel,
                                      kern[dom], f_mhz, sm_count),
            "reference_basis_ms_per_step": ms_ref_basis,
            "ref_cuda": None if ref_ms is None else {
                "ms_per_step": ref_ms, "value": f.numel / (ref_ms / 1e3), "speedup": ref_ms / ms,
                "what": "reference extension (oracle/_ref, unmodified gaussian_peft/cuda_field/csrc) forward"
                        + (" + bf16 cast" if out_dtype == torch.bfloat16 else "") + " + backward, same inputs"},
        }
    return out


# ---------------------------------------------------------------------------
TRAIN_METRIC = "SD1.5-UNet Gaussian-adapter data-parallel training samples/s (128 projections, K=256)"


def train_arm(a, rank: int, world: int, local: int) -> None:
    """cfg4: one step = render every delta (batched), UNet forward + epsilon
    MSE, backward (batched render backward), one flat NCCL all-reduce of the
    Gaussian-parameter gradients, AdamW.  Weak scaling: a fixed batch per GPU."""
    from guass_b200 import _lib, sd15
    from guass_b200.adapters import BatchedAdapters
    from guass_b200.partition import field_costs

    L = _lib.lib()
    cfg = sd15.UNetConfig()
    torch.manual_seed(0)  # identical base weights on every rank
    with torch.device("cuda"):
        model = sd15.SD15UNet(cfg, dtype=torch.bfloat16)
    model.cuda()
    mods = model.adapters()
    if a.adapter_apply == "dropin":
        bank = sd15.PerLayerRender(mods)
    else:
        bank = BatchedAdapters(mods, out_dtype=torch.bfloat16, fused_weight=(a.adapter_apply == "fused"),
                               fast_exp=(a.fwd_exp == "ex2" and a.bwd_exp == "ex2"),
                               track_metadata=False)  # no per-step diagnostic read-back in the timed loop
    bank.install()
    tr = sd15.DataParallelTrainer(model, bank, world=world)
    inp = sd15.synthetic_inputs(cfg, a.batch, seed=1000 + rank, device="cuda")
    host = [t.cpu().pin_memory() for t in inp.tensors()]
    shapes = [(m.out_features, m.in_features) for m in mods.values()]

    for _ in range(a.warmup):
        tr.step(inp)
    torch.cuda.synchronize()
    nf = len(shapes)
    # exact evaluation count from one binning pass of the current parameters
    probe = bank if a.adapter_apply != "dropin" else BatchedAdapters(mods, track_metadata=False)
    with torch.no_grad():
        probe.render()
    assert probe.batch.device_flags() == 0
    tps = [probe.batch.tile_ptr_view(i).cpu() for i in range(nf)]
    evals = sum(field_costs(tps, shapes))
    elements = sum(o * i for o, i in shapes)
    del probe
    calls = nf if a.adapter_apply == "dropin" else 1  # library forward/backward calls per step

    sampler = ClockSampler() if local == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
        sampler.mark("t0")
    # per step and call: 3 trace events in the render forward, 4 in its backward (gfield.h,
    # gf_trace_events); all forward calls of a step come before its backward calls
    expected = 7 * calls * a.steps
    # headroom: a drop-in forward that outgrows its id buffer renders again (3 more events)
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(expected + (3 * calls * a.steps if calls > 1 else 0))]
    for e in evs:
        e.record()
    torch.cuda.synchronize()
    handles = (ctypes.c_void_p * len(evs))(*[e.cuda_event for e in evs])
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    _lib.check(L.gf_trace_events(handles, len(evs)))
    tr.allreduce_events = [] if world > 1 else None
    start.record()
    for _ in range(a.steps):
        loss = tr.step(inp)
    end.record()
    torch.cuda.synchronize()
    barrier(world)
    recorded = L.gf_trace_count()
    _lib.check(L.gf_trace_events(None, 0))
    if sampler:
        sampler.mark("t1")
    ms = max_over_ranks(start.elapsed_time(end) / a.steps, world)
    per = {"render_fwd": [], "render_bwd": [], "render_total": []}
    if recorded != expected:  # a re-render shifted the events: no per-kernel attribution
        assert calls > 1, (recorded, expected)
        per = {}
    for st in range(a.steps if per else 0):
        e = evs[7 * calls * st: 7 * calls * (st + 1)]
        fw = [e[3 * c: 3 * c + 3] for c in range(calls)]
        bw = [e[3 * calls + 4 * c: 3 * calls + 4 * c + 4] for c in range(calls)]
        per["render_fwd"].append(sum(f[1].elapsed_time(f[2]) for f in fw))
        per["render_bwd"].append(sum(b[1].elapsed_time(b[2]) for b in bw))
        per["render_total"].append(sum(f[0].elapsed_time(f[2]) for f in fw) + sum(b[0].elapsed_time(b[3]) for b in bw))
    ok = torch.tensor([1.0 if per else 0.0], device="cuda")
    if world > 1:
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    if ok.item() > 0:
        kern = {k: max_over_ranks(sum(v) / len(v), world) for k, v in per.items()}
    else:
        kern = {"unavailable": "a drop-in forward re-rendered for a larger id buffer inside the timed loop"}
    if tr.allreduce_events:
        kern["allreduce"] = max_over_ranks(sum(x.elapsed_time(y) for x, y in tr.allreduce_events)
                                           / len(tr.allreduce_events), world)
    tr.allreduce_events = None
    clocks = sampler.stop() if sampler else None
    assert torch.isfinite(loss).item()

    # end to end: this step's inputs copied from pinned host memory, the loss read back, every step
    d_in = inp.tensors()
    h2d = sum(t.numel() * t.element_size() for t in host)

    def e2e_step():
        for h, d in zip(host, d_in):
            d.copy_(h, non_blocking=True)
        return tr.step(inp).cpu()

    n_e2e = max(3, min(a.steps, 10))
    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(n_e2e):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / n_e2e, world)

    if rank == 0:
        sm_count = torch.cuda.get_device_properties(0).multi_processor_count
        f_mhz = (clocks or {}).get("sm_mhz") or 1965.0
        fast = a.adapter_apply != "dropin" and a.fwd_exp == "ex2" and a.bwd_exp == "ex2"
        roofline = None
        if "render_bwd" in kern:
            roofline = pipe_roofline(kernel_name("render_bwd", fast), evals, elements, kern["render_bwd"], f_mhz,
                                     sm_count)
            if roofline is not None and calls > 1:
                roofline["definition"] += " (summed over the per-layer launches)"
        samples = a.batch * world
        line = {
            "metric": TRAIN_METRIC, "value": samples / (ms / 1e3), "unit": "samples/s", "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded latents/text/noise ~ N(0,1), t ~ U{0..999}; random-init SD1.5-shaped UNet)",
            "config": {"workload": "cfg4 data-parallel adapter training step", "batch_per_gpu": a.batch,
                       "latent": [cfg.latent_channels, cfg.latent_size, cfg.latent_size],
                       "text": [cfg.text_tokens, cfg.cross_dim], "adapters": nf, "K": cfg.num_gaussians,
                       "delta_elements": elements, "evals": evals, "adapter_apply": a.adapter_apply,
                       "render_bases": "ex2.approx (forward and backward)" if fast else "expf",
                       "parallelism": f"dp{world}: flat NCCL all-reduce of Gaussian-parameter gradients"
                       if world > 1 else "single GPU", "optimizer": "AdamW on mu_raw/chol_raw/amp",
                       "l2": "no flush: the UNet step streams GBs of activations and weights"},
            "kernels_ms": kern, "render_share": kern["render_total"] / ms if "render_total" in kern else None,
            "roofline": roofline,
            "clocks": clocks,
            "e2e": {"value": samples / (e2e_ms / 1e3), "unit": "samples/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": int(h2d * world), "d2h_bytes_per_step": 4 * world,
                    "path": "DataParallelTrainer.step with latents/text/t/noise H2D from pinned memory "
                            "and the loss read back, every step"},
            "cpu_baseline": None,
            "gpu_launches": 5 * calls * a.steps * world,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main():
    a = parse_args()
    if a.impl == "reference" and a.workload == "cfg4":
        if int(os.environ.get("RANK", "0")) == 0:
            print(json.dumps({"impl": "reference", "unavailable": "cfg4 is a GPU training step of an SD1.5-sized "
                              "UNet; the reference's CPU path would take minutes per step. Its layer composition "
                              "is timed on the GPU with --adapter-apply reference"}), flush=True)
        return
    if a.workload == "cfg4":
        rank, world, local = setup_dist()
        train_arm(a, rank, world, local)
        return
    if a.impl == "reference":
        # host-only: no CUDA context, no process group; rank 0 alone works
        reference_arm(a, int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")))
        return
    rank, world, local = setup_dist()
    fx, bx = a.fwd_exp == "ex2", a.bwd_exp == "ex2"
    if a.profile_case and a.profile_field:
        from guass_b200 import synthetic
        from guass_b200.batched import FieldBatch, pack_fields

        name = a.profile_field
        f = synthetic.densified(int(name[5:])) if name.startswith("dense") else synthetic.CONFIGS[name]()
        out_dtype = torch.float32 if name == "cfg2" else torch.bfloat16
        b = FieldBatch([(f.out_features, f.in_features, f.k)], out_dtype=out_dtype, fwd_exp2=fx, bwd_exp2=bx)
        mu, chol, amp, grad = pack_fields([f], device="cuda")
        while b.ensure_capacity(mu, chol, amp):
            pass
        for _ in range(a.warmup + a.steps):
            b.forward(mu, chol, amp)
            b.backward(grad, mu, chol, amp)
        torch.cuda.synchronize()
        print(f"profile case: {name}, {f.numel} elements, {b.total_pairs()} pairs, {a.warmup + a.steps} steps",
              flush=True)
        return
    w = UNetWorkload(rank, world, a.exchange, a.groups, bwd_exp2=bx, fwd_exp2=fx, num_fields=a.fields)
    if a.profile_case:
        for _ in range(a.warmup + a.steps):
            w.step()
        torch.cuda.synchronize()
        if rank == 0:
            print(f"profile case: {len(w.fields)} fields, {w.total_elements} elements, {w.total_evals} evaluations, "
                  f"{a.warmup + a.steps} steps", flush=True)
        if world > 1:
            dist.destroy_process_group()
        return
    sampler = ClockSampler() if local == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
        sampler.mark("t0")
    # The same timing at every N: eager steps (a few dozen launches on two
    # streams), CUDA events, max over ranks.  NCCL collectives are never
    # captured into a graph (a captured all-gather hung process teardown on
    # this system); at N=1 a CUDA-graph replay is reported beside it.
    ms_local, kern = run_device_timed(w, a.steps, a.warmup, world)
    if sampler:
        sampler.mark("t1")
    ms = max_over_ranks(ms_local, world)
    kern_max = {k: max_over_ranks(v, world) for k, v in kern.items()}
    clocks = sampler.stop() if sampler else None
    value = w.total_elements / (ms / 1e3)
    graph_ms = None
    if world == 1 or w.renderer.symm is not None:
        graph_ms = max_over_ranks(run_graph_timed(w, a.steps, a.warmup, world), world)

    # the reference's arithmetic (expf in both passes) on the same workload
    ref_basis = None
    if fx or bx:
        for b in w.renderer.batches:
            b.set_bases(fwd_exp2=False, bwd_exp2=False)
        ms_e, kern_e = run_device_timed(w, max(3, a.steps // 2), a.warmup, world)
        ref_basis = {"ms_per_step": max_over_ranks(ms_e, world),
                     "kernels_ms": {k: max_over_ranks(v, world) for k, v in kern_e.items()}}
        ref_basis["value"] = w.total_elements / (ref_basis["ms_per_step"] / 1e3)
        for b in w.renderer.batches:
            b.set_bases(fwd_exp2=fx, bwd_exp2=bx)

    e2e = e2e_layer = None
    if not a.no_e2e:
        n_e2e = max(3, min(a.steps, 10))
        try:
            e2e_ms, h2d, d2h = run_e2e_batched(w, n_e2e, 2, world)
            e2e = {"value": w.total_elements / (e2e_ms / 1e3), "unit": UNIT, "ms_per_step": e2e_ms,
                   "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                   "path": "whole-model API (PartitionedRenderer over FieldBatch): packed params and fp32 "
                           "dL/d(delta) H2D from pinned memory, packed gradients D2H, every step; the next "
                           "step's inputs copy on a second stream while this step computes"}
        except Exception as exc:  # report, do not lose the device-timed line
            e2e = {"error": f"{type(exc).__name__}: {exc}"}
        e2e_layer = {}
        for mode, key in ((("dropin", "e2e_dropin_per_layer"), ("model_renderer", "e2e_model_renderer"))
                          if world == 1 else ()):
            try:
                e2e_ms, h2d, d2h = run_e2e_model(w, n_e2e, 2, world, mode)
                e2e_layer[key] = {
                    "value": w.total_elements / (e2e_ms / 1e3), "unit": UNIT, "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                    "path": ("GUASS layer API: every layer's compute_delta_weight() through "
                             "guass_b200.cuda_field.gaussian_field_train (one render per layer, the reference's call "
                             "pattern), fp32 delta" if mode == "dropin" else
                             "GUASS layer API with adapters.ModelRenderer: one batched render per model forward "
                             "(bf16 delta), one batched backward") +
                            "; layer params and dL/d(delta) (in the delta's dtype) H2D from one pinned staging "
                            "buffer each, gradients D2H through one, every step"}
            except Exception as exc:  # noqa: BLE001
                e2e_layer[key] = {"error": f"{type(exc).__name__}: {exc}"}

    sm_count = torch.cuda.get_device_properties(0).multi_processor_count
    f_mhz = (clocks or {}).get("sm_mhz") or 1965.0
    extra = {}
    cpu = None
    if rank == 0 and world == 1:
        if not a.no_configs:
            try:
                extra["configs"] = single_field_configs(a, f_mhz, sm_count)
            except Exception as exc:  # noqa: BLE001
                extra["configs"] = {"error": f"{type(exc).__name__}: {exc}"}
            ref_ms = time_reference_cuda(w.fields, True, 2, 1)
            try:
                extra["dense"] = dense_rows(a, kern_max["render_fwd"] / w.total_evals * 1e6)
            except Exception as exc:  # noqa: BLE001
                extra["dense"] = {"error": f"{type(exc).__name__}: {exc}"}
            if ref_ms is not None:
                extra["ref_cuda"] = {"ms_per_step": ref_ms, "value": w.total_elements / (ref_ms / 1e3),
                                     "speedup": ref_ms / ms,
                                     "what": "reference extension (oracle/_ref, unmodified gaussian_peft/cuda_field/"
                                             "csrc), per layer as GaussianLinear calls it: forward + bf16 cast + "
                                             "backward for each of the fields, same inputs, CUDA events"}
        if not a.no_cpu_baseline:
            cpu = cpu_baseline(w.fields, a.cpu_seconds)

    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return
    # the slowest rank's launch processes its share of the evaluations
    evals = w.total_evals if world == 1 else max(sum(w.costs[i] for i in p) for p in w.parts)
    elements = w.total_elements if world == 1 else max(sum(w.fields[i].numel for i in p) for p in w.parts)
    dom = max(("render_fwd", "render_bwd"), key=lambda k: kern_max[k])
    roofline = pipe_roofline(kernel_name(dom, fx if dom == "render_fwd" else bx), evals, elements, kern_max[dom],
                             f_mhz, sm_count)
    other = "render_fwd" if dom == "render_bwd" else "render_bwd"
    roofline_other = pipe_roofline(kernel_name(other, fx if other == "render_fwd" else bx), evals, elements,
                                   kern_max[other], f_mhz, sm_count)
    bytes_step = w.total_elements * (2 + 4)  # bf16 delta written + fp32 dL/d(delta) read
    with open(ROOT / "MEASURED_PEAKS.json") if (ROOT / "MEASURED_PEAKS.json").exists() else open(os.devnull) as fh:
        txt = fh.read()
    hbm_peak = json.loads(txt).get("hbm_gbs", 6650.0) if txt else 6650.0
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded; BASELINE cfg3 shapes and cfg1 distributions)",
        "config": {"workload": f"cfg3 whole-UNet batched render, {len(w.fields)} projection fields, K=256",
                   "elements": w.total_elements, "pairs": w.total_pairs, "evals": w.total_evals,
                   "delta_dtype": "bf16", "grad_dtype": "f32", "tile": "32x32", "sigma_multiplier": 3.0,
                   "forward_basis": "ex2.approx" if fx else "expf",
                   "backward_basis": "ex2.approx" if bx else "expf",
                   "clamp_quad": 80.0, "partition": f"LPT by render cost over {world} rank(s)",
                   "parallelism": f"layer-partition x{world} + {w.renderer.exchange} of bf16 delta "
                                  f"({w.layout.num_groups} field groups)" if world > 1 else "single GPU",
                   "l2": "no flush: each step writes 187 MB of delta and reads 374 MB of dL/d(delta) (> 126 MB L2)"},
        "kernels_ms": kern_max,
        "timing": "value and kernels_ms: eager steps with per-launch trace events (every N); graph_ms_per_step: "
                  "the same step replayed as one CUDA graph",
        "graph_ms_per_step": graph_ms,
        "roofline": roofline,
        "roofline_other_kernel": roofline_other,
        "roofline_step": step_roofline(w.total_evals, bytes_step, ms, sm_count, f_mhz, hbm_peak, world,
                                       kernel_name("render_fwd", fx), kernel_name("render_bwd", bx)),
        "roofline_hbm": {"achieved": bytes_step / (ms / 1e3) / 1e9, "peak": hbm_peak, "unit": "GB/s",
                         "frac": bytes_step / (ms / 1e3) / 1e9 / hbm_peak, "peak_source": "MEASURED_PEAKS.json hbm_gbs"},
        "reference_basis": ref_basis,
        "clocks": clocks,
        "e2e": e2e,
        **(e2e_layer or {}),
        "cpu_baseline": cpu,
        **extra,
        # per step: bin (+ the id lists when the render runs in field groups), per render call the
        # regular and the heavy-tile kernel, prep, backward render (regular + heavy), finalize
        # (+ one publish kernel per group of the multicast exchange)
        "gpu_launches": a.steps * world * (
            7 if world == 1 else (2 + 2 * (1 if w.renderer.fused else len(w.renderer.ranges)) + 4
                                  + (w.layout.num_groups if w.renderer.symm is not None and not w.renderer.fused
                                     else 0))),
    }
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
