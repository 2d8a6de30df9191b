"""Timed CPU reference arm: the reference's own ``PackedPINN`` on the host cores.

    python -m baseline.reference_cpu --config cfg1 --steps 5 --warmup 1 [--parts M] [--threads N]

Runs the reference package installed into ``baseline/_ref/`` by
``baseline/install_reference.py`` (``src/flashns/pinn_packed.py:15-191``, unchanged),
with ``layout="compact", seed="explicit"`` and torch's CPU FP64 kernels on
``torch.set_num_threads(N)`` threads, and prints one JSON line with the median time of
``--steps`` loss + parameter-gradient evaluations after ``--warmup`` untimed ones.  With
``--parts M`` each step evaluates one of M contiguous point chunks (step k takes chunk
k mod M, each a ``PackedPINN`` over 1/M of the interior and of the boundary points with
the global weights), so that a long run stays bounded; the rate is then
(1/M) / median step time in evaluations of the whole set per second.

The reference has only the (u, v, p) head with the gradient-enhanced residual on value
boundary rows, so the timed objective is that head on the configuration's own point set
and hidden layers: for cfg1 the 2-64x4-3 net on the same 16,384 interior + 4,096
boundary Kovasznay points with the same globally normalized weights, boundary targets
(u, v, p) from the analytic field on the raw outputs, Xavier-normal weights from seed 0.  Its packed rows (Q10 interior jets + one value row per
boundary point) are 167,936 against this library's 172,032 (first-order boundary rows);
the GEMM work differs by the 3rd output column and those rows, under 3 %.

Nothing in the product imports this module.  It runs as its own process so that the
reference's ``flashns`` package, not this repository's import alias of the same name,
is the one imported.
"""

import argparse
import json
import os
import statistics
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
REF = Path(__file__).resolve().parent / "_ref"


def available(directory=REF):
    return (Path(directory) / "flashns" / "pinn_packed.py").exists()


def reference_inputs(config):
    """(x, ni, pde_weights, boundary_weights[nb, 3], target[nb, 3], widths) of the uvp
    objective on the configuration's point set."""
    import torch

    sys.path.insert(1, str(ROOT))
    from flashns_b200.evaluator import xavier_normal  # seeded init only, no device code
    from flashns_b200.problems import CONFIGS, config_parameters, config_points
    c = CONFIGS[config]
    if c["kind"] == "reference_case":  # the reference's own headline workload, as it is
        pts = config_points(config)
        ws, bs = config_parameters(config)
        return (pts.x.contiguous(), pts.interior_count, pts.pde_weights.contiguous(),
                pts.boundary_weights.contiguous(), pts.target.contiguous(), ws, bs, list(c["widths"]),
                pts.viscosity)
    if c["kind"] != "kovasznay":
        raise ValueError("the reference CPU arm covers the 2-D configurations (the reference has no 3-D head)")
    # the first-order-row point set carries (u, v, p) targets and weights per boundary point
    pts = config_points(config, boundary_order=1)
    widths = list(c["widths"][:-1]) + [3]
    ws, bs = xavier_normal(widths, 0)
    return (pts.x.contiguous(), pts.interior_count, pts.pde_weights.contiguous(),
            pts.boundary_weights.contiguous(), pts.target.contiguous(), ws, bs, widths, pts.viscosity)


def run(config, steps, warmup, threads, parts=1):
    import torch

    torch.set_num_threads(threads)
    for name in [m for m in sys.modules if m == "flashns" or m.startswith("flashns.")]:
        del sys.modules[name]
    sys.path.insert(0, str(REF))
    from flashns.ns_seed import NSLoss
    from flashns.pinn_packed import PackedPINN
    import flashns.pinn_packed as module
    if not Path(module.__file__).resolve().is_relative_to(REF.resolve()):
        raise RuntimeError(f"imported {module.__file__}, not the reference package under {REF}")
    x, ni, pw, bw, target, ws, bs, widths, nu = reference_inputs(config)
    nb = len(x) - ni
    loss = NSLoss(viscosity=nu, gradient_weight=0.2, boundary_weight=5.0)
    chunks = []
    for k in range(parts):
        i0, i1 = ni * k // parts, ni * (k + 1) // parts
        b0, b1 = nb * k // parts, nb * (k + 1) // parts
        xs = torch.cat((x[i0:i1], x[ni + b0:ni + b1])).contiguous()
        chunks.append(PackedPINN(xs, i1 - i0, pw[i0:i1].contiguous(), bw[b0:b1].contiguous(),
                                 target[b0:b1].contiguous(), layout="compact", seed="explicit", loss=loss))
    for k in range(warmup):
        chunks[k % parts](ws, bs)
    times = []
    for k in range(steps):
        t0 = time.perf_counter()
        chunks[k % parts](ws, bs)
        times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return {"value": (1.0 / parts) / med, "unit": "evals/s", "median_s": med, "parts": parts, "times_s": times,
            "threads": threads, "net": "-".join(map(str, widths)), "interior": ni, "boundary": nb,
            "rows": ni * 10 + nb, "module": str(Path(module.__file__).relative_to(ROOT))}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--config", default="cfg1")
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--parts", type=int, default=1)
    ap.add_argument("--threads", type=int, default=None)
    args = ap.parse_args()
    if args.parts < 1 or args.steps < 1 or args.warmup < 0:
        sys.exit("--parts and --steps must be positive, --warmup non-negative")
    threads = args.threads or max(1, len(os.sched_getaffinity(0)))
    print(json.dumps(run(args.config, args.steps, args.warmup, threads, args.parts)), flush=True)


if __name__ == "__main__":
    main()
