"""The Kovasznay solve with the reference's own GPU evaluation route as the closure, on the
same GPU and under the same optimizer as this library's solve: a same-machine
time-to-accuracy comparison.

    python -m baseline.reference_solve [--route v8+] [--seed 1]

The reference has only the (u, v, p) head, so both sides solve that objective: the
2-64x4-3 net, the gradient-enhanced residual (weight 0.2) on 16,384 interior points and
(u, v, p) targets on 4,096 value boundary rows, Re = 20, acceptance relative L2 of (u, v)
<= 1e-3 and of p <= 1e-2 on the 201 x 201 grid.  Everything but the evaluation is
``flashns_b200.solver.solve(head="uvp")`` (3,000 Adam steps, then the device L-BFGS with a
strong-Wolfe line search, acceptance every 100 iterations, one CUDA graph per evaluation).
The evaluation is the reference's packed route (``src/flashns/pinn_packed.py:93-191`` with
its v8 kernels, ``baseline/reference_routes.py``): ``v8+`` adds every opt-in fused hook,
its fastest route on this GPU.  This library's side of the comparison is
``python -m flashns_b200.solver --head uvp --seed S``.

Nothing in the product imports this module.
"""

import argparse
import json
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

from baseline.reference_routes import ReferenceKernels, available, packed_coordinates, packed_step  # noqa: E402


class ReferenceRouteEvaluator:
    """``__call__(flat, out)`` writes ``[grad(P), loss]`` of the reference's packed route,
    with the parameters read as views of ``flat``; capturable in a CUDA graph (the route's
    torch GEMMs and kernel launches all run on the current stream)."""

    def __init__(self, points, widths, head, boundary_order, loss, device, route="v8+"):
        if head != "uvp" or boundary_order != 0:
            raise ValueError("the reference's routes evaluate the (u, v, p) head on value boundary rows")
        if route not in ("v8", "v8+"):
            raise ValueError("the packed routes (v8, v8+) carry boundary rows")
        dev = lambda t: t.to(device).contiguous()
        self.x, self.pw, self.bw, self.target = dev(points.x), dev(points.pde_weights), \
            dev(points.boundary_weights), dev(points.target)
        self.ni = points.interior_count
        self.widths = list(widths)
        self.shapes = list(zip(self.widths, self.widths[1:]))
        self.parameters = sum(i * o for i, o in self.shapes) + sum(o for _, o in self.shapes)
        self.kernels = ReferenceKernels()
        self.inputs = packed_coordinates(self.x, self.ni)
        self.loss, self.hooks = loss, route == "v8+"

    def __call__(self, flat, out):
        ws, bs, o = [], [], 0
        for i, j in self.shapes:
            ws.append(flat[o:o + i * j].view(j, i))
            o += i * j
        for _, j in self.shapes:
            bs.append(flat[o:o + j])
            o += j
        total, grads = packed_step(self.x, self.ni, self.pw, self.bw, self.target, ws, bs, self.kernels,
                                   self.loss.viscosity, self.loss.gradient_weight, self.loss.boundary_weight,
                                   inputs=self.inputs, hooks=self.hooks)
        torch.cat([g.reshape(-1) for g in grads] + [total.reshape(1)], out=out)
        return out


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--route", default="v8+", choices=["v8", "v8+"])
    ap.add_argument("--seed", type=int, default=1)
    ap.add_argument("--adam-steps", type=int, default=3000)
    ap.add_argument("--max-iterations", type=int, default=50000)
    args = ap.parse_args()
    if not available():
        print(json.dumps({"impl": f"reference-{args.route}", "unavailable": "reference kernels not built"}))
        return
    from flashns_b200.solver import solve
    torch.cuda.set_device(0)
    make = lambda pts, widths, head, order, loss, device: ReferenceRouteEvaluator(pts, widths, head, order, loss,
                                                                                  device, args.route)
    result = solve(seed=args.seed, head="uvp", adam_steps=args.adam_steps, max_iterations=args.max_iterations,
                   make_evaluator=make)
    result["evaluation"] = f"reference {args.route} route (its kernels, torch FP64 GEMMs)"
    print(json.dumps(result), flush=True)


if __name__ == "__main__":
    main()
