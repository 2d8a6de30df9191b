"""Benchmark: FP64 loss + parameter-gradient evaluations per second on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg1]
                    [--impl ours|reference|reference-gpu] [--route F|B1|v8|v8+]

Default workload (cfg1): the Kovasznay stream-function net 2->64x4->2 on 16,384
interior points with full third-order Q10 jets plus 4,096 boundary points with
first-order rows, FP64, seeded synthetic points and Xavier-normal weights (seed 0).  One step is one complete loss + gradient
evaluation of a cfg1-sized point set per GPU.  With N GPUs (torchrun, one rank
per GPU) the global point set is N x cfg1, each rank evaluates its shard and one
NCCL all-reduce of the packed [gradient, loss] buffer completes the step (weak
scaling); ``value`` counts cfg1-sized shard evaluations of all ranks per second.
``--scaling strong`` shards the configuration's one point set over the N ranks
(``shard_bounds`` on interior and boundary points, global weights) and ``value``
counts complete evaluations of that set per second.

``--impl reference`` times the reference's own CPU implementation, its ``PackedPINN``
(installed into ``baseline/_ref/`` by ``baseline/install_reference.py``, run by
``baseline/reference_cpu.py`` with torch on all host threads), on the same point set;
where that is not installed, or for the 3-D configuration the reference has no head for,
the oracle port of ``PackedPINN`` is timed instead.  Rank 0 alone runs and prints.

``--impl reference-gpu --config ref16k`` times one of the reference's own GPU routes on
this GPU (``--route``: F, its published H100 headline route; B1; the v8 packed route;
or v8+, the v8 route with every opt-in fused hook), with the reference's kernels compiled from its sources into ``baseline/_ref/``
by ``baseline/build_reference_gpu.py`` and torch FP64 GEMMs between them, replayed from a
CUDA graph as the reference's benchmarks do.  Rank 0 alone runs it.
"""

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

REF16K_PUBLISHED_MS = 1.832
# the reference's published H100 replay times of its routes at 16,384 points
# (docs/cuda-h100-results.md:54-64); the v8 packed routes have none
REFERENCE_ROUTE_PUBLISHED_MS = {"F": 1.832, "B1": 1.954}
METRIC = "FP64 loss+param-gradient evals/sec"
# NVIDIA's published dense FP64 tensor-core figure for B200, beside the in-run probe
FP64_DATASHEET_TFLOPS = 40.0
UNIT = "evals/s"
# the reference arm: seconds of one full cfg1 evaluation of the reference's CPU path on the
# box's 16 cores (measured 0.61 s), and the wall time its timed run should stay within
REFERENCE_FULL_EVAL_S, REFERENCE_BUDGET_S = 0.65, 240.0


def parse():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=500)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--config", default="cfg1",
                    choices=["cfg0", "cfg1", "cfg2", "cfg3", "ref16k", "tgv64", "cfg1x64"],
                    help="tgv64 and cfg1x64 are not benchmark configurations: the 3-D 64-wide net whose kernels "
                         "the others do not reach, and cfg1's net on 64 times its points (1.3M)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "reference-gpu"])
    ap.add_argument("--route", default="F", choices=["F", "B1", "v8", "v8+"],
                    help="route of --impl reference-gpu")
    ap.add_argument("--scaling", default="weak", choices=["weak", "strong"],
                    help="weak: each rank evaluates a config-sized shard of an N x config set; strong: the "
                         "config's one point set is sharded over the N ranks")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile", action="store_true",
                    help="only W warm-up and K timed steps (for ncu launch lists); prints a short line")
    ap.add_argument("--points-divisor", type=int, default=1,
                    help="with --profile: 1/D of the configuration's points (small ncu captures of the same kernels)")
    return ap.parse_args()


def workload(config, scaling="weak"):
    from flashns_b200.problems import CONFIGS, config_options
    c = CONFIGS[config]
    head, order, _ = config_options(config)
    net = "-".join(str(w) for w in c["widths"][:2]) + f"x{len(c['widths']) - 2}-{c['widths'][-1]}"
    rows = "first-order boundary rows" if order else "value boundary rows"
    jets = f"Q{10 if c['widths'][0] == 2 else 20} interior jets"
    if scaling == "strong":
        return {"workload": f"{config}: {c['kind']} {c['interior']}+{c['boundary']} points in total, sharded over "
                            f"the GPUs, {head} head, {jets}, {rows}",
                "net": net, "interior_points": c["interior"], "boundary_points": c["boundary"], "head": head,
                "boundary_order": order}
    return {"workload": f"{config}: {c['kind']} {c['interior']}+{c['boundary']} points per GPU, {head} head, "
                        f"{jets}, {rows}",
            "net": net, "interior_points_per_gpu": c["interior"], "boundary_points_per_gpu": c["boundary"],
            "head": head, "boundary_order": order}


# ---------------------------------------------------------------------------- CPU side
def host_cores():
    """CPUs this process may run on (its affinity mask, which a container's cpuset
    narrows), not every CPU of the host."""
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def cpu_port_rate(config, steps, warmup, workers):
    """Oracle port of the reference CPU path on 1/8-point chunks over a process pool;
    returns (evals/s of the full set, median s/step, sample description)."""
    from flashns_b200.problems import config_options, config_parameters, config_points
    from oracle.cpu_baseline import timed_rate

    head, order, gamma = config_options(config)
    pts = config_points(config)
    ws, bs = config_parameters(config)
    problem = dict(x=pts.x.numpy(), ni=pts.interior_count, pw=pts.pde_weights.numpy(),
                   bw=pts.boundary_weights.numpy(), target=pts.target.numpy(), ws=[w.numpy() for w in ws],
                   bs=[b.numpy() for b in bs],
                   options=dict(head=head, nu=pts.viscosity, gamma=gamma, bc=5.0, boundary_order=order))
    parts = 8
    rate, med = timed_rate(problem, workers, steps, warmup, parts=parts)
    ni, nb = pts.interior_count, len(pts.x) - pts.interior_count
    sample = (f"{steps} timed steps; each evaluates one of {parts} point chunks ({ni // parts}+{nb // parts} points) "
              f"of the {config} set split over {workers} single-threaded NumPy processes; "
              f"evals/s = (1/{parts}) / median step time")
    return rate, med, sample


def reference_cpu_rate(config, steps, warmup, threads, parts=1):
    """The reference's own PackedPINN on `threads` host threads, in its own process
    (baseline/reference_cpu.py); returns its JSON line, or None when it is not installed
    or does not cover the configuration."""
    from baseline.reference_cpu import available
    from flashns_b200.problems import CONFIGS
    if not available() or CONFIGS[config]["kind"] == "taylor_green":
        return None
    cmd = [sys.executable, "-m", "baseline.reference_cpu", "--config", config, "--steps", str(steps),
           "--warmup", str(warmup), "--parts", str(parts), "--threads", str(threads)]
    result = subprocess.run(cmd, capture_output=True, text=True, cwd=ROOT, timeout=900)
    if result.returncode:
        raise RuntimeError(f"reference CPU arm failed:\n{result.stderr[-2000:]}")
    return json.loads(result.stdout.strip().splitlines()[-1])


def reference_cpu_sample(r, config):
    chunk = (f"one of {r['parts']} point chunks ({r['interior'] // r['parts']}+{r['boundary'] // r['parts']} "
             f"points) per step; evals/s = (1/{r['parts']}) / median step time" if r["parts"] > 1
             else "one complete evaluation per step; evals/s = 1 / median step time")
    head = ("the same (u, v, p) objective as the repo arm" if config == "ref16k" else
            "the (u, v, p) head (the reference has no stream-function head)")
    return (f"the reference's PackedPINN(layout='compact', seed='explicit') from {r['module']}, torch CPU FP64 "
            f"on {r['threads']} threads: {head} on the {config} point set, net {r['net']}, {r['rows']} packed "
            f"rows; {len(r['times_s'])} timed steps, {chunk}")


def kernel_source_sha():
    """sha256 over the CUDA sources and the C header (the build an ncu capture belongs to)."""
    import hashlib
    h = hashlib.sha256()
    for path in sorted((ROOT / "flashns_b200" / "csrc").glob("*.cu*")) + sorted((ROOT / "include").glob("*.h")):
        h.update(path.name.encode() + b"\0" + path.read_bytes())
    return h.hexdigest()


# ---------------------------------------------------------------------------- clocks
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index, path):
        self.path = path
        self.proc = None
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={index}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=open(path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, ValueError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            f = [v.strip() for v in line.split(",")]
            if len(f) < 10:
                continue
            try:
                rows.append(dict(sm=float(f[1]), max=float(f[2]), power=float(f[3]), util=float(f[4]),
                                 hw=f[6], hwt=f[7], swt=f[8], swp=f[9]))
            except ValueError:
                continue
        if not rows:
            return None
        load = [r for r in rows if r["util"] >= 50] or rows
        reasons = set()
        for r in load:
            for key, name in (("hw", "hw_slowdown"), ("hwt", "hw_thermal_slowdown"), ("swt", "sw_thermal_slowdown"),
                              ("swp", "sw_power_cap")):
                if r[key].lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r["sm"] for r in load), "sm_max_mhz": max(r["max"] for r in rows),
                "power_w_max": max(r["power"] for r in rows), "samples_under_load": len(load),
                "reasons": sorted(reasons)}


# ---------------------------------------------------------------------------- GPU side
def hbm_peak_gbs():
    """(GB/s, source): the driver-measured copy bandwidth of MEASURED_PEAKS.json, else the
    pool's earlier measurement of 6.65 TB/s."""
    try:
        value = float(json.loads((ROOT / "MEASURED_PEAKS.json").read_text())["hbm_gbs"])
        if value > 0:
            return value, "MEASURED_PEAKS.json hbm_gbs (measured)"
    except (OSError, ValueError, KeyError, TypeError):
        pass
    return 6650.0, "fallback 6.65 TB/s (no MEASURED_PEAKS.json)"


def fp64_peak(device_stream, torch):
    from flashns_b200 import _lib
    lib = _lib.library()
    sink = torch.zeros(1, dtype=torch.float64, device="cuda")
    flops = ctypes.c_double()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    run = lambda it: _lib.check(lib.flashns_b200_fp64_peak_probe(4 * sms, it, ctypes.c_void_p(sink.data_ptr()),
                                                                 ctypes.byref(flops),
                                                                 ctypes.c_void_p(device_stream.cuda_stream)),
                                "peak probe")
    run(64)
    best = 0.0
    for _ in range(3):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(device_stream)
        run(4096)
        e1.record(device_stream)
        e1.synchronize()
        best = max(best, flops.value / (e0.elapsed_time(e1) * 1e-3) / 1e12)
    return best


def kernel_times(ev, params, out, steps, stream, torch):
    """Per-kind average launch duration (ms) from events recorded between launches."""
    from flashns_b200 import _lib
    lib = ev.plan._lib
    n = ctypes.c_int()
    _lib.check(lib.flashns_b200_plan_launch_kinds(ev.plan.handle, None, 0, ctypes.byref(n)), "launch_kinds")
    kinds = (ctypes.c_int * n.value)()
    _lib.check(lib.flashns_b200_plan_launch_kinds(ev.plan.handle, kinds, n.value, ctypes.byref(n)), "launch_kinds")
    events = [[torch.cuda.Event(enable_timing=True) for _ in range(n.value + 1)] for _ in range(steps)]
    for row in events:  # torch creates the CUDA event at its first record
        for e in row:
            e.record(stream)
    torch.cuda.synchronize()
    ptr = lambda t: ctypes.c_void_p(t.data_ptr()) if t.numel() else None
    for s in range(steps):
        handles = (ctypes.c_void_p * (n.value + 1))(*[ctypes.c_void_p(e.cuda_event) for e in events[s]])
        rec = ctypes.c_int()
        _lib.check(lib.flashns_b200_eval_marked(ev.plan.handle, ptr(ev.x), ptr(params), ptr(ev.pde_weights),
                                                ptr(ev.boundary_weights), ptr(ev.target), ptr(out),
                                                ptr(ev.workspace), ev.workspace.numel() * 8,
                                                ctypes.c_void_p(stream.cuda_stream), handles, n.value + 1,
                                                ctypes.byref(rec)), "eval_marked")
    torch.cuda.synchronize()
    per = {}
    for s in range(steps):
        for i, k in enumerate(kinds):
            name = _lib.KERNEL_KINDS[k]
            per.setdefault(name, []).append(events[s][i].elapsed_time(events[s][i + 1]))
    counts = {}
    for k in kinds:
        counts[_lib.KERNEL_KINDS[k]] = counts.get(_lib.KERNEL_KINDS[k], 0) + 1
    return {k: {"launches_per_eval": counts[k], "avg_ms": statistics.mean(v), "total_ms_per_eval": sum(v) / steps}
            for k, v in per.items()}


def reference_gpu_arm(args, cfg, local):
    """One of the reference's GPU routes, CUDA-graph replayed on this GPU (rank 0 only)."""
    import torch
    from baseline.reference_routes import CapturedRoute, ReferenceKernels, available
    from flashns_b200.evaluator import PackedEvaluator, flat_parameters
    from flashns_b200.ns_seed import NSLoss
    from flashns_b200.problems import CONFIGS, config_options, config_parameters, config_points

    base = {"impl": "reference-gpu", "route": args.route}
    if args.config != "ref16k":
        return dict(base, unavailable="the reference's GPU routes implement the (u, v, p) head without boundary "
                                      "targets on dense routes; run --config ref16k")
    if not available():
        return dict(base, unavailable="reference kernels not built (python baseline/build_reference_gpu.py with "
                                      "FLASHNS_REFERENCE set)")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    kernels = ReferenceKernels()
    pts = config_points(args.config)
    head, order, gamma = config_options(args.config)
    ws_host, bs_host = config_parameters(args.config)
    dev = lambda t: t.to(device).contiguous()
    x, pw, bw, target = dev(pts.x), dev(pts.pde_weights), dev(pts.boundary_weights), dev(pts.target)
    ws, bs = [dev(w) for w in ws_host], [dev(b) for b in bs_host]
    route = CapturedRoute(args.route, x, pts.interior_count, pw, bw, target, ws, bs, kernels,
                          nu=pts.viscosity, gamma=gamma)
    stream = torch.cuda.current_stream(device)

    sampler = ClockSampler(local, "/tmp/flashns_clocks_reference.csv")
    t_end = time.perf_counter() + 1.0
    while time.perf_counter() < t_end:
        for _ in range(20):
            route.replay()
        torch.cuda.synchronize()
    for _ in range(max(args.warmup, 3)):
        route.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        route.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    ms_step = e0.elapsed_time(e1) / args.steps
    clocks = sampler.stop()

    # end to end as in our arm: pinned host inputs copied into the graph's static inputs,
    # one replay, the loss and gradient read back, a synchronize
    statics = [x] + ws + bs
    hosts = [t.cpu().pin_memory() for t in statics]
    outs = [route.loss] + list(route.grads)
    hout = [t.cpu().pin_memory() for t in outs]
    h2d = sum(t.numel() * 8 for t in hosts)
    d2h = sum(t.numel() * 8 for t in hout)

    def e2e_step():
        for d, h in zip(statics, hosts):
            d.copy_(h, non_blocking=True)
        route.refresh()
        route.replay()
        for h, d in zip(hout, outs):
            h.copy_(d, non_blocking=True)
        stream.synchronize()

    e2e_steps = max(1, min(args.steps, 200))
    for _ in range(3):
        e2e_step()
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps

    # agreement with this library's fused evaluation on the same inputs (not timed)
    loss, grads = route.replay()
    got = torch.cat([g.reshape(-1) for g in grads] + [loss.reshape(1)]).cpu()
    ev = PackedEvaluator(x, pts.interior_count, pw, bw, target, CONFIGS[args.config]["widths"], head=head,
                         boundary_order=order, loss=NSLoss(viscosity=pts.viscosity, gradient_weight=gamma,
                                                           boundary_weight=5.0), device=device)
    ours = ev(flat_parameters(ws_host, bs_host).to(device)).cpu()
    ratio = float(((got - ours).abs() / (2e-12 + 2e-11 * ours.abs())).max())
    rel = float((got - ours).norm() / ours.norm())

    value = 1e3 / ms_step
    published = REFERENCE_ROUTE_PUBLISHED_MS.get(args.route)
    libs = kernels.build["libraries"]
    return dict(base, **{
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": value / (1e3 / published) if published else None, "dtype": "f64",
        "data": "synthetic (the reference benchmark's recipe, as in --impl ours --config ref16k)",
        "config": cfg, "parallelism": "single",
        "e2e": {"value": 1e3 / e2e_ms, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "kernels_from": {k: {"sources": sorted(v["sources"]), "sha256": v["sha256"][:16]} for k, v in libs.items()},
        "cutlass": kernels.build.get("cutlass"),
        "agreement_with_flashns_b200": {"max_error_over_tolerance": ratio, "relative_l2": rel,
                                        "tolerance": "|a-b| <= 2e-12 + 2e-11|b|"},
        "clocks": clocks,
        "baseline_note": (f"vs_baseline: this route's published H100 time, {published} ms "
                          "(docs/cuda-h100-results.md:54-64)" if published else "no published time for this route"),
    })


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    cfg = workload(args.config, args.scaling)

    if args.impl == "reference-gpu":
        if rank == 0:
            print(json.dumps(reference_gpu_arm(args, cfg, local)), flush=True)
        return

    if args.impl == "reference":
        if rank != 0:
            return
        threads = host_cores()
        # full evaluations when the run fits a few minutes, else the fewest point chunks that
        # keep it there: every call of the reference's PackedPINN pays a fixed cost (about
        # 30 ms on 16 cores against 0.6 s for a whole cfg1 evaluation) once per chunk, so the
        # smaller the chunks the more the chunked rate understates the reference
        need = (args.steps + args.warmup) * REFERENCE_FULL_EVAL_S / REFERENCE_BUDGET_S
        parts = 1 if need <= 1 else min(64, 1 << math.ceil(math.log2(need)))
        ref = reference_cpu_rate(args.config, args.steps, args.warmup, threads, parts)
        if ref is not None:
            rate, kind, sample = ref["value"], "reference", reference_cpu_sample(ref, args.config)
            objective = (f"the reference's (u, v, p) head with the gradient-enhanced residual on value boundary "
                         f"rows, net {ref['net']}, same points and weights as the repo arm")
        else:
            rate, _, sample = cpu_port_rate(args.config, args.steps, args.warmup, threads)
            kind, objective = "port", "the oracle port of PackedPINN on the repo arm's exact objective"
        line = {"metric": METRIC, "value": rate, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 / rate, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic", "config": cfg,
                "reference_objective": objective,
                "cpu_baseline": {"value": rate, "unit": UNIT, "cores": threads, "kind": kind, "sample": sample},
                "e2e": {"value": rate, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta
    from flashns_b200.costs import checkpoint_bytes, evaluation_bytes, evaluation_costs, kernel_rooflines
    from flashns_b200.evaluator import PackedEvaluator, flat_parameters
    from flashns_b200.ns_seed import NSLoss
    from flashns_b200.problems import CONFIGS, config_options, config_parameters, config_points

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=device)
    c = CONFIGS[args.config]
    widths = c["widths"]
    # weak scaling: the global set is `world` x the config; each rank owns one config-sized shard
    if args.points_divisor != 1 and not args.profile:
        raise SystemExit("--points-divisor only applies to --profile runs")
    if world == 1:
        pts = config_points(args.config, divisor=args.points_divisor)
    elif args.scaling == "strong":  # the configuration's point set, sharded
        pts = config_points(args.config).shard(world, rank)
    else:  # weak: a world x config set, one config-sized shard per rank
        pts = config_points(args.config, scale=world).shard(world, rank)
    per_step = world if args.scaling == "weak" else 1  # configuration-sized evaluations per step
    head, order, gamma = config_options(args.config)
    loss = NSLoss(viscosity=pts.viscosity, gradient_weight=gamma, boundary_weight=5.0)
    ev = PackedEvaluator(pts.x, pts.interior_count, pts.pde_weights, pts.boundary_weights, pts.target, widths,
                         head=head, boundary_order=order, loss=loss, device=device)
    ws, bs = config_parameters(args.config)
    params_host = flat_parameters(ws, bs)
    params = params_host.to(device)
    out = torch.empty(ev.parameters + 1, dtype=torch.float64, device=device)
    stream = torch.cuda.current_stream()

    def step():
        ev(params, out)
        if world > 1:
            dist.all_reduce(out)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    if args.profile:
        for _ in range(args.warmup):
            step()
        barrier()
        for _ in range(args.steps):
            step()
        barrier()
        if world > 1:
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps({"profile": True, "config": args.config, "launches_per_step": ev.launches_per_call,
                              "interior": ev.ni, "boundary": ev.nb, "warmup": args.warmup, "steps": args.steps}),
                  flush=True)
        return

    sampler = ClockSampler(local, f"/tmp/flashns_clocks_{rank}.csv")
    # settle clocks under load for about a second; rank 0 decides per batch and every
    # rank follows, so all ranks issue the same collectives in the same order
    t_end = time.perf_counter() + 1.0
    go = torch.ones(1, dtype=torch.int32, device=device)
    while True:
        for _ in range(20):
            step()
        torch.cuda.synchronize()
        go.fill_(int(time.perf_counter() < t_end))
        if world > 1:
            dist.broadcast(go, 0)
        if not int(go):
            break
    for _ in range(max(args.warmup, 3)):
        step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    barrier()
    elapsed = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(elapsed, op=dist.ReduceOp.MAX)
    ms_step = float(elapsed) / args.steps
    clocks = sampler.stop()

    # end to end: every step copies all inputs (coordinates, weights, targets, parameters)
    # from one pinned host staging buffer to the device in a single transfer, evaluates,
    # all-reduces and reads [grad, loss] back to the host
    hin, din, dparams = ev.input_arena(params_host)
    hout = torch.empty(ev.parameters + 1, dtype=torch.float64).pin_memory()
    h2d = hin.numel() * 8
    d2h = hout.numel() * 8

    def e2e_step():
        din.copy_(hin, non_blocking=True)
        ev(dparams, out)
        if world > 1:
            dist.all_reduce(out)
        hout.copy_(out, non_blocking=True)
        stream.synchronize()

    e2e_steps = max(1, min(args.steps, 200))
    for _ in range(3):
        e2e_step()
    barrier()
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    barrier()
    e2e_ms = torch.tensor([e0.elapsed_time(e1) / e2e_steps], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)

    # per-kernel roofline (events between launches, separate from the headline timing)
    ktimes = kernel_times(ev, params, out, 20, stream, torch)
    peak = fp64_peak(stream, torch)
    costs = evaluation_costs(widths, ev.ni, ev.nb, head=head, boundary_order=order)
    dominant = max(ktimes, key=lambda k: ktimes[k]["total_ms_per_eval"])
    dom_flops = statistics.mean(costs["per_kind"][dominant])
    achieved = dom_flops / (ktimes[dominant]["avg_ms"] * 1e-3) / 1e12
    hbm_peak, hbm_source = hbm_peak_gbs()
    kernels = kernel_rooflines(ktimes, costs["per_kind"],
                               evaluation_bytes(widths, ev.ni, ev.nb, head=head, boundary_order=order), peak,
                               hbm_peak)
    # DRAM bytes of one launch of the dominant kernel from a committed ncu capture, used only
    # when that capture was taken of the kernel sources built here
    traffic, traffic_source = None, "no ncu capture of this configuration committed"
    tfile = ROOT / "profiles" / "traffic.json"
    if tfile.exists():
        try:
            record = json.loads(tfile.read_text())
            captured = record.get(args.config, {}).get(dominant)
            if captured is not None and record.get("kernel_source_sha") == kernel_source_sha():
                traffic = captured
                traffic_source = f"ncu capture of this build (profiles/traffic.json, sources {record['kernel_source_sha'][:12]})"
            elif captured is not None:
                traffic_source = "dropped: the committed ncu capture is of other kernel sources"
        except (ValueError, AttributeError, KeyError):
            traffic = None

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    cpu = port = None
    if world == 1 and not args.no_cpu_baseline:
        threads = host_cores()
        ref = reference_cpu_rate(args.config, 3, 1, threads)
        rate, med, sample = cpu_port_rate(args.config, 16, 2, threads)
        port = {"value": rate, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample}
        cpu = port if ref is None else {"value": ref["value"], "unit": UNIT, "cores": threads, "kind": "reference",
                                        "sample": reference_cpu_sample(ref, args.config)}
    step_tflops = costs["total"] / (ms_step * 1e-3) / 1e12
    value = per_step * 1e3 / ms_step
    if args.config == "ref16k":
        # the reference's own headline workload, published for its fused F route on H100
        # (1.832 ms per evaluation, CUDA-graph replay): the only config with a published number
        vs_baseline = value / (1e3 / REF16K_PUBLISHED_MS)
        data = ("synthetic (the reference benchmark's recipe: N(0, 0.4^2) coordinates, unweighted quadrature, "
                "weights N(0, 0.49/fan_in), biases N(0, 0.01))")
    else:
        vs_baseline = None
        data = "synthetic (seeded uniform Kovasznay points, analytic boundary targets, Xavier-normal weights seed 0)"
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": args.scaling,
        "vs_baseline": vs_baseline, "dtype": "f64", "data": data,
        "config": cfg,
        "parallelism": f"dp{world}" if world > 1 else "single",
        "l2": "working set (checkpoints + seeds) %.2f GB > 126 MB L2; no flush needed"
              % (checkpoint_bytes(widths, ev.ni, ev.nb, boundary_order=order) / 1e9),
        "e2e": {"value": per_step * 1e3 / float(e2e_ms), "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": ev.launches_per_call * args.steps,
        "roofline": {"bound": "tensor", "kernel": dominant, "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "traffic": traffic, "traffic_source": traffic_source,
                     "peak_source": "in-run FP64 DMMA m16n8k8 register-only probe (no FP64 entry in MEASURED_PEAKS.json)",
                     "frac_of_datasheet": achieved / FP64_DATASHEET_TFLOPS,
                     "datasheet_peak": FP64_DATASHEET_TFLOPS,
                     "flops_per_launch": dom_flops},
        "step_roofline": {"algorithmic_tflop_per_step": costs["total"] / 1e12, "achieved": step_tflops,
                          "frac": step_tflops / peak, "frac_of_datasheet": step_tflops / FP64_DATASHEET_TFLOPS},
        "kernels": kernels,
        "kernel_peaks": {"fp64_tflops": peak, "hbm_gbs": hbm_peak, "hbm_source": hbm_source,
                         "note": "per kind: CUDA-event mean launch time, algorithmic FLOPs and compulsory "
                                 "DRAM bytes per launch (flashns_b200/costs.py)"},
        "clocks": clocks,
    }
    if vs_baseline is not None:
        line["baseline_note"] = ("vs the reference's published fused-F replay on H100 80GB "
                                 "(docs/cuda-h100-results.md:54-64), other hardware")
    if cpu:
        line["cpu_baseline"] = cpu
    if port and cpu is not port:
        line["cpu_baseline_port"] = port
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
