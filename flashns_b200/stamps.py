"""Phase timings of the two-group kernels, from the instrumented library.

    python -m flashns_b200.build --stamps
    python -m flashns_b200.stamps [--config cfg1] [--evals 5] [--json]

``libflashns_b200_stamps.so`` is this library built with ``FLASHNS_B200_STAMPS``: the
leader thread of each 8-warp group of ``bwd_pingpong``, ``fwd_pingpong`` and
``head_pingpong`` writes ``%globaltimer`` at the phase boundaries of each of its half
tiles.  For every launch of those kernels in one evaluation this reports, per half tile
and in microseconds:

* backward: the wait for the seed tile and the turn, dgrad, the wait for H_l plus wgrad,
  and the VJP epilogue (the leader thread's share, to the group barrier);
* forward and the fused head: the wait for the input tile and the turn, the mainloop,
  and the epilogue (for the head: jet, output layer, seeds, output gradient and VJP);

and the share of each CTA's span during which one of its two groups held the tensor pipe
(its MMA phases), averaged over the CTAs.  The instrumentation changes register
allocation slightly (some variants spill a few dozen bytes), so the figures describe the
schedule rather than the product's exact timings; the product library has no stamps.
"""

import argparse
import ctypes
import json
import statistics

TILES, PHASES = 32, 5  # kStampTiles, kStampPhases of csrc/eval.cu
# kernel kind -> (phase names between consecutive stamps, the stamps bounding the MMA phase)
LAYOUT = {"backward": (("wait", "dgrad", "wait H + wgrad", "epilogue"), (1, 3)),
          "forward": (("wait", "mainloop", "epilogue"), (1, 2)),
          "forward_head": (("wait", "mainloop", "epilogue"), (1, 2))}


def summarize(stamps, kinds):
    """Per instrumented launch: mean phase durations (us) and mean MMA coverage of a CTA's
    span.  ``stamps``: int64 array [launches, ctas, 2, TILES, PHASES] of %globaltimer ns
    (0 = not written)."""
    rows = []
    for launch, kind in enumerate(kinds):
        if kind not in LAYOUT:
            continue
        names, (m0, m1) = LAYOUT[kind]
        last = len(names)
        phases = {n: [] for n in names}
        coverage = []
        for cta in stamps[launch]:
            mma, begin, end = 0, None, None
            for group in cta:
                for tile in group:
                    if not tile[0] or not tile[last]:
                        continue
                    for i, n in enumerate(names):
                        phases[n].append((int(tile[i + 1]) - int(tile[i])) / 1e3)
                    mma += int(tile[m1]) - int(tile[m0])
                    begin = int(tile[0]) if begin is None else min(begin, int(tile[0]))
                    end = int(tile[last]) if end is None else max(end, int(tile[last]))
            if begin is not None and end > begin:
                coverage.append(mma / (end - begin))
        if coverage:
            rows.append({"launch": launch, "kind": kind, "half_tiles": len(phases[names[0]]),
                         "us": {n: statistics.mean(v) for n, v in phases.items()},
                         "mma_share_of_cta_span": statistics.mean(coverage)})
    return rows


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--config", default="cfg1", choices=["cfg0", "cfg1", "cfg2", "cfg3", "ref16k"])
    ap.add_argument("--evals", type=int, default=5)
    ap.add_argument("--json", action="store_true")
    args = ap.parse_args()

    import torch

    from flashns_b200 import _lib, build
    from flashns_b200.evaluator import PackedEvaluator, flat_parameters
    from flashns_b200.ns_seed import NSLoss
    from flashns_b200.problems import CONFIGS, config_options, config_parameters, config_points

    if not build.STAMPS_LIBRARY.exists():
        raise SystemExit("build the instrumented library first: python -m flashns_b200.build --stamps")
    _lib.LIBRARY, _lib._library = build.STAMPS_LIBRARY, None
    lib = _lib.library()
    lib.flashns_b200_stamps_attach.argtypes = [ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int]
    lib.flashns_b200_stamps_attach.restype = ctypes.c_int
    lib.flashns_b200_stamps_per_launch.argtypes = [ctypes.c_longlong]
    lib.flashns_b200_stamps_per_launch.restype = ctypes.c_longlong
    if lib.flashns_b200_stamps_per_launch(1) != 2 * TILES * PHASES:
        raise SystemExit("stamp layout of the library and of this runner differ")

    device = torch.device("cuda", 0)
    pts = config_points(args.config)
    head, order, gamma = config_options(args.config)
    ev = PackedEvaluator(pts.x, pts.interior_count, pts.pde_weights, pts.boundary_weights, pts.target,
                         CONFIGS[args.config]["widths"], head=head, boundary_order=order,
                         loss=NSLoss(viscosity=pts.viscosity, gradient_weight=gamma, boundary_weight=5.0),
                         device=device)
    params = flat_parameters(*config_parameters(args.config)).to(device)
    out = torch.empty(ev.parameters + 1, dtype=torch.float64, device=device)
    n = ctypes.c_int()
    _lib.check(lib.flashns_b200_plan_launch_kinds(ev.plan.handle, None, 0, ctypes.byref(n)), "launch_kinds")
    kinds_c = (ctypes.c_int * n.value)()
    _lib.check(lib.flashns_b200_plan_launch_kinds(ev.plan.handle, kinds_c, n.value, ctypes.byref(n)), "launch_kinds")
    kinds = [_lib.KERNEL_KINDS[k] for k in kinds_c]
    ctas = 2 * torch.cuda.get_device_properties(device).multi_processor_count  # above any persistent grid
    buf = torch.zeros(n.value * lib.flashns_b200_stamps_per_launch(ctas), dtype=torch.int64, device=device)
    for _ in range(3):
        ev(params, out)
    _lib.check(lib.flashns_b200_stamps_attach(ctypes.c_void_p(buf.data_ptr()), ctas, n.value), "stamps_attach")
    results = []
    try:
        for _ in range(args.evals):
            buf.zero_()
            ev(params, out)
            torch.cuda.synchronize()
            results.append(summarize(buf.view(n.value, ctas, 2, TILES, PHASES).cpu().numpy(), kinds))
    finally:
        _lib.check(lib.flashns_b200_stamps_attach(None, 0, 0), "stamps_detach")
    # mean over the evaluations, launch by launch
    merged = []
    for i, first in enumerate(results[0]):
        same = [r[i] for r in results]
        merged.append({"launch": first["launch"], "kind": first["kind"], "half_tiles": first["half_tiles"],
                       "us": {k: statistics.mean(r["us"][k] for r in same) for k in first["us"]},
                       "mma_share_of_cta_span": statistics.mean(r["mma_share_of_cta_span"] for r in same)})
    if args.json:
        for row in merged:
            print(json.dumps(row))
        return
    print(f"{args.config}: phase means per half tile (us), {args.evals} evaluations, instrumented build\n")
    print("| launch | kernel | half tiles | phases (us) | MMA share of CTA span |\n|---|---|---|---|---|")
    for row in merged:
        phases = ", ".join(f"{k} {v:.2f}" for k, v in row["us"].items())
        print(f"| {row['launch']} | {row['kind']} | {row['half_tiles']} | {phases} | "
              f"{100 * row['mma_share_of_cta_span']:.1f} % |")


if __name__ == "__main__":
    main()
