"""Time the fused dense dgrad + jet VJP behind the reference's ABI on one GPU: this
library's ``flashns_stable_dgrad_vjp`` (DMMA mainloop, VJP epilogue) against the
reference's own (``experiments/cuda_jet_h100/stable_dgrad.cu:57-174``, a CUTLASS SM80
FP64 mainloop with the VJP in its epilogue, built from its sources into ``baseline/_ref/``
by ``baseline/build_reference_gpu.py``), on the same inputs.

    python -m baseline.dgrad_bench [--batch 16384] [--cout 64] [--cin 64] [--dim 2] [--iters 200]

Prints one JSON line per implementation: mean time per call over ``--iters`` calls after
20 warm-up calls (CUDA events on the launch stream), the algorithmic FP64 rate
(2 B Q cout cin for the GEMM, the VJP's generated formula flops per (sample, channel)),
and the agreement of the two outputs under ``|a-b| <= 2e-12 + 2e-11|b|``.  The reference's
published H100 time for this shape is 0.105 ms (docs/cuda-h100-results.md:112-120).
"""

import argparse
import ctypes
import json
import sys
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

VJP_FLOPS = {2: 103, 3: 255}  # generated jet VJP flops per (sample, channel), as flashns_b200/costs.py counts


def bind(path):
    lib = ctypes.CDLL(str(path))
    fn = lib.flashns_stable_dgrad_vjp
    fn.argtypes = [ctypes.c_int, ctypes.c_bool] + [ctypes.c_void_p] * 5 + [ctypes.c_int] * 3 + [ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return fn


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--batch", type=int, default=16384)
    ap.add_argument("--cout", type=int, default=64)
    ap.add_argument("--cin", type=int, default=64)
    ap.add_argument("--dim", type=int, default=2, choices=[2, 3])
    ap.add_argument("--iters", type=int, default=200)
    args = ap.parse_args()
    from flashns_b200 import _lib
    impls = {"flashns_b200": bind(_lib.LIBRARY)}
    ref = ROOT / "baseline" / "_ref" / "libdgrad_n64.so"
    if ref.exists():
        impls["reference_stable_dgrad"] = bind(ref)
    dev = torch.device("cuda", 0)
    q = 10 if args.dim == 2 else 20
    gen = torch.Generator(device="cpu").manual_seed(7)
    rnd = lambda *s: torch.randn(*s, generator=gen, dtype=torch.float64).to(dev)
    d = rnd(args.batch, q, args.cout)
    w = rnd(args.cout, args.cin) / args.cout ** 0.5
    h = torch.tanh(rnd(args.batch, q, args.cin) * 0.5)
    aux = torch.rand(args.batch, args.cin, generator=gen, dtype=torch.float64).to(dev)
    stream = torch.cuda.current_stream(dev)
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    outs = {}
    flops = 2.0 * args.batch * q * args.cout * args.cin + VJP_FLOPS[args.dim] * args.batch * args.cin
    for name, fn in impls.items():
        out = torch.empty(args.batch, q, args.cin, dtype=torch.float64, device=dev)
        call = lambda: fn(args.dim, True, p(d), p(w), p(h), p(aux), p(out), args.batch, args.cout, args.cin,
                          ctypes.c_void_p(stream.cuda_stream))
        for _ in range(20):
            if call():
                raise RuntimeError(f"{name}: launch failed")
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.iters):
            call()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.iters
        outs[name] = out
        print(json.dumps({"impl": name, "dim": args.dim, "batch": args.batch, "cout": args.cout, "cin": args.cin,
                          "ms": ms, "tflops": flops / (ms * 1e-3) / 1e12}), flush=True)
    if len(outs) == 2:
        a, b = outs["flashns_b200"], outs["reference_stable_dgrad"]
        ratio = float(((a - b).abs() / (2e-12 + 2e-11 * b.abs())).max())
        print(json.dumps({"agreement_max_error_over_tolerance": ratio}), flush=True)


if __name__ == "__main__":
    main()
