"""Kovasznay time-to-accuracy solve: the 2-64x4-2 stream-function net on 16,384 + 4,096 points.

The reference's complete solve (experiments/pinn_solver/solve.py:77-167) replays a
CUDA-graph-captured loss + gradient evaluation as the closure of an Adam phase and a
strong-Wolfe ``torch.optim.LBFGS``.  Here the closure replays one captured
``flashns_b200_eval`` (plus the gradient all-reduce on several GPUs); acceptance is the
relative L2 error of (u, v) <= 1e-3 and of p <= 1e-2 against the analytic Kovasznay
fields on a 201 x 201 grid over the domain, evaluated with ``flashns_b200_fields``.

    python -m flashns_b200.solver                       # one GPU
    torchrun --nproc-per-node N -m flashns_b200.solver  # N GPUs (sample data parallelism)

The wall time includes setup (point generation, plans, graph capture), every closure
evaluation of the line searches and the acceptance checks.
"""

import argparse
import ctypes
import json
import math
import os
import time
from pathlib import Path

import torch
import torch.distributed as dist

from flashns_b200 import _lib
from flashns_b200.evaluator import FieldEvaluator, PackedEvaluator, flat_parameters, xavier_normal
from flashns_b200.lbfgs import DeviceLBFGS
from flashns_b200.ns_seed import NSLoss
from flashns_b200.problems import SAMPLINGS, kovasznay, kovasznay_exact


def acceptance_grid(n=201):
    xs = torch.linspace(-0.5, 1.0, n, dtype=torch.float64)
    ys = torch.linspace(-0.5, 1.5, n, dtype=torch.float64)
    gx, gy = torch.meshgrid(xs, ys, indexing="ij")
    return torch.stack((gx.reshape(-1), gy.reshape(-1)), 1)


class Acceptance:
    """Relative L2 errors of (u, v, p) on the grid against the analytic solution.  The
    stream-function head gives (u, v, p) = (psi_y, -psi_x, p) from first-order rows, the
    (u, v, p) head its raw outputs from value rows."""

    def __init__(self, widths, re, device, n=201, head="psi"):
        grid = acceptance_grid(n)
        u, v, p, _ = kovasznay_exact(grid, re)
        self.exact = torch.stack((u, v, p), 1).to(device)
        self.norm = self.exact.square().sum(0).sqrt()
        self.fields = FieldEvaluator(grid, widths, head=head, boundary_order=1 if head == "psi" else 0,
                                     device=device)

    def __call__(self, flat):
        f = self.fields(flat)
        err = (f - self.exact).square().sum(0).sqrt() / self.norm
        return [float(e) for e in err.cpu()]


def save_checkpoint(path, flat, meta):
    """Final parameters and the run description as a torch checkpoint (the record of
    experiments/pinn_solver/solve.py:255-266); returns the file's sha256."""
    import hashlib
    path = Path(path)
    torch.save({"flat_parameters": flat.detach().cpu(), **meta}, path)
    return hashlib.sha256(path.read_bytes()).hexdigest()


def load_checkpoint(path):
    return torch.load(Path(path), map_location="cpu", weights_only=True)


def solve(*, interior=16384, boundary=4096, widths=None, re=20.0, seed=1, init_seed=0,
          boundary_weight=5.0, tol_uv=1e-3, tol_p=1e-2, max_iterations=50000, check_every=100, history=50,
          adam_steps=3000, adam_lr=1e-3, grid=201, device=None, log=None, time_limit=None, optimizer="device",
          sampling="uniform", initial=None, return_parameters=False, head="psi", make_evaluator=None):
    """Solve to acceptance; returns the result dict (and the final parameters).

    ``head`` "psi": the stream-function net (psi, p), first-order boundary rows with (u, v, p)
    targets (the benchmark configuration); "uvp": the reference's (u, v, p) net with the
    gradient-enhanced residual (gradient weight 0.2) and (u, v, p) targets on value rows.
    ``make_evaluator(points, widths, head, boundary_order, loss, device)`` replaces the
    evaluation: an object with ``parameters`` (P) whose ``__call__(flat, out)`` writes
    ``[grad(P), loss]`` into ``out`` on the current stream, capturable in a CUDA graph."""
    start = time.perf_counter()
    world = dist.get_world_size() if dist.is_initialized() else 1
    rank = dist.get_rank() if dist.is_initialized() else 0
    device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    if head not in ("psi", "uvp"):
        raise ValueError("head must be 'psi' or 'uvp'")
    widths = list(widths) if widths is not None else [2, 64, 64, 64, 64, 2 if head == "psi" else 3]
    order = 1 if head == "psi" else 0
    # the first-order-row point set carries (u, v, p) targets and weights per boundary point,
    # which the (u, v, p) head's value rows use as they are
    pts = kovasznay(interior, boundary, re=re, seed=seed, boundary_order=1, sampling=sampling, device=device)
    loss = NSLoss(viscosity=1.0 / re, boundary_weight=boundary_weight)
    if make_evaluator is not None:
        ev = make_evaluator(pts, widths, head, order, loss, device)
    elif world > 1:
        from flashns_b200.distributed import DistributedEvaluator
        ev = DistributedEvaluator(pts, widths, head=head, boundary_order=order, loss=loss, device=device)
    else:
        ev = PackedEvaluator(pts.x, pts.interior_count, pts.pde_weights, pts.boundary_weights, pts.target, widths,
                             head=head, boundary_order=order, loss=loss, device=device)
    accept = Acceptance(widths, re, device, grid, head)
    ws, bs = xavier_normal(widths, init_seed)
    start_params = flat_parameters(ws, bs) if initial is None else initial.detach().to(torch.float64).reshape(-1)
    flat = torch.nn.Parameter(start_params.to(device).contiguous())
    out = torch.empty(ev.parameters + 1, dtype=torch.float64, device=device)
    # capture one evaluation (the parameter storage stays at the same address)
    stream = torch.cuda.Stream(device)
    stream.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(stream):
        for _ in range(3):
            ev(flat.data, out)
    torch.cuda.current_stream(device).wait_stream(stream)
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        ev(flat.data, out)
    grad_view, loss_view = out[:ev.parameters], out[ev.parameters]
    evaluations = [0]

    def closure():
        graph.replay()
        evaluations[0] += 1
        flat.grad = grad_view
        return loss_view

    torch.cuda.synchronize(device)
    setup = time.perf_counter() - start
    phases = {"adam_s": 0.0, "lbfgs_s": 0.0, "accept_s": 0.0}
    t_phase = time.perf_counter()
    if adam_steps:
        # Adam phase on the same captured closure (experiments/pinn_solver/solve.py:137-149),
        # one fused update kernel per step
        m, v = torch.zeros_like(flat.data), torch.zeros_like(flat.data)
        lib = _lib.library()
        ptr = lambda t: ctypes.c_void_p(t.data_ptr())
        launch_stream = ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
        for k in range(1, adam_steps + 1):
            graph.replay()
            _lib.check(lib.flashns_b200_adam_step(ptr(flat.data), ptr(grad_view), ptr(m), ptr(v), flat.numel(),
                                                  adam_lr, 0.9, 0.999, 1e-8, k, launch_stream), "adam_step")
        evaluations[0] += adam_steps
        torch.cuda.synchronize(device)
    phases["adam_s"] = time.perf_counter() - t_phase
    if optimizer == "device":
        lbfgs = DeviceLBFGS(flat.data, grad_view, loss_view, graph.replay, history=history,
                            capture_evaluate=lambda: ev(flat.data, out))
    else:
        lbfgs = torch.optim.LBFGS([flat], lr=1.0, max_iter=check_every, max_eval=int(check_every * 1.25),
                                  history_size=history, tolerance_grad=0.0, tolerance_change=0.0,
                                  line_search_fn="strong_wolfe")
    iterations, metrics, accepted = 0, None, False
    decision = torch.zeros(1, dtype=torch.int32, device=device)
    while iterations < max_iterations:
        t_phase = time.perf_counter()
        if optimizer == "device":
            lbfgs.step(check_every)
            iterations = lbfgs.iterations
            evaluations[0] = adam_steps + lbfgs.evaluations
        else:
            lbfgs.step(closure)
            iterations = lbfgs.state[lbfgs._params[0]]["n_iter"]
        t_accept = time.perf_counter()
        phases["lbfgs_s"] += t_accept - t_phase
        metrics = accept(flat.data)
        phases["accept_s"] += time.perf_counter() - t_accept
        accepted = metrics[0] <= tol_uv and metrics[1] <= tol_uv and metrics[2] <= tol_p
        # rank 0 decides whether to stop (accepted, diverged or out of time) and every rank
        # follows, so all ranks leave the loop after the same closure evaluations
        out_of_time = time_limit is not None and time.perf_counter() - start > time_limit
        decision.fill_(int(accepted or out_of_time or not all(math.isfinite(m) for m in metrics)))
        if world > 1:
            dist.broadcast(decision, 0)
        if log and rank == 0:
            log(json.dumps({"t": round(time.perf_counter() - start, 3), "iter": iterations, "evals": evaluations[0],
                            "loss": float(loss_view), "rel_l2_uvp": metrics}))
        if int(decision):
            break
    torch.cuda.synchronize(device)
    wall = time.perf_counter() - start
    del graph
    result = {"accepted": accepted, "wall_s": wall, "setup_s": setup, **phases, "optimizer": optimizer,
              "iterations": iterations,
              "evaluations": evaluations[0], "rel_l2_u": metrics[0], "rel_l2_v": metrics[1], "rel_l2_p": metrics[2],
              "final_loss": float(loss_view), "n_gpus": world, "interior": interior, "boundary": boundary,
              "widths": widths, "head": head, "re": re, "seed": seed, "init_seed": init_seed, "sampling": sampling}
    return (result, flat.detach().cpu()) if return_parameters else result


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--seed", type=int, default=1)
    ap.add_argument("--init-seed", type=int, default=0)
    ap.add_argument("--max-iterations", type=int, default=50000)
    ap.add_argument("--check-every", type=int, default=100)
    ap.add_argument("--boundary-weight", type=float, default=5.0)
    ap.add_argument("--adam-steps", type=int, default=3000)
    ap.add_argument("--history", type=int, default=50)
    ap.add_argument("--time-limit", type=float, default=None)
    ap.add_argument("--optimizer", choices=["device", "torch"], default="device")
    ap.add_argument("--sampling", choices=list(SAMPLINGS), default="uniform",
                    help="uniform: torch CPU generator; sobol / philox: drawn on the device")
    ap.add_argument("--initial", type=Path, default=None, help="start from a checkpoint's flat parameters")
    ap.add_argument("--head", choices=["psi", "uvp"], default="psi",
                    help="psi: stream-function net (the benchmark); uvp: the reference's (u, v, p) net")
    ap.add_argument("--output", type=Path, default=None,
                    help="write OUTPUT.pt (final parameters + run description) and OUTPUT.json (result)")
    ap.add_argument("--quiet", action="store_true")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    initial = load_checkpoint(args.initial)["flat_parameters"] if args.initial else None
    result, final = solve(seed=args.seed, init_seed=args.init_seed, max_iterations=args.max_iterations,
                          check_every=args.check_every, boundary_weight=args.boundary_weight,
                          adam_steps=args.adam_steps, history=args.history, time_limit=args.time_limit,
                          optimizer=args.optimizer, sampling=args.sampling, initial=initial, head=args.head,
                          log=None if args.quiet else lambda s: print(s, flush=True), return_parameters=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if int(os.environ.get("RANK", "0")) == 0:
        if args.output is not None:
            meta = {"problem": {"name": "kovasznay", "re": result["re"], "interior": result["interior"],
                                "boundary": result["boundary"], "widths": result["widths"],
                                "head": args.head, "sampling": args.sampling},
                    "protocol": {k: getattr(args, k) for k in ("adam_steps", "history", "check_every",
                                                               "boundary_weight", "max_iterations")},
                    "seed": args.seed, "init_seed": args.init_seed, "backend": "flashns_b200"}
            result["checkpoint_sha256"] = save_checkpoint(args.output.with_suffix(".pt"), final, meta)
            args.output.with_suffix(".json").write_text(json.dumps(result, indent=1) + "\n")
        print(json.dumps(result), flush=True)


if __name__ == "__main__":
    main()
