"""FP64 throughput of each instruction shape on this GPU: context for the FP64 roofline's
denominator (DMMA m16n8k8, which ``bench.py`` re-measures in every run).  Measurement
infrastructure beside the baselines; nothing in the product imports it.

    python -m baseline.fp64_peak [--iters 4096] [--repeats 3] [--json]

``flashns_b200_fp64_probe`` runs each kind at several launch shapes; the best of
``repeats`` CUDA-event timings per kind is reported in TFLOP/s, with the SM clock the
driver reports under load.

* register-only MMA chains (m8n8k4, m16n8k4, m16n8k8, m16n8k16) and DFMA chains:
  SMs x {1, 2, 4} CTAs of {128, 256, 512} threads (m16n8k8 runs at 256 threads, the
  in-run probe's shape);
* ``smem``: m16n8k8 fed from shared memory in the kernels' tile shape at 16 warps per SM
  (one 512-thread CTA, or two 256-thread CTAs), at 8 warps per SM (one 256-thread CTA) and
  at 4 warps per SM (one 128-thread CTA).
"""

import argparse
import ctypes
import json
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
from flashns_b200 import _lib  # noqa: E402

KINDS = {"m16n8k8": 0, "m8n8k4": 1, "m16n8k4": 2, "m16n8k16": 3, "dfma": 4, "smem": 5}


def launch_shapes(kind, sms):
    if kind == "smem":
        return [(sms, 512, "16 warps/SM, one 512-thread CTA"), (2 * sms, 256, "16 warps/SM, two 256-thread CTAs"),
                (sms, 256, "8 warps/SM, one 256-thread CTA"), (sms, 128, "4 warps/SM, one 128-thread CTA")]
    threads = (256,) if kind == "m16n8k8" else (128, 256, 512)
    return [(m * sms, t, f"{m} x {t}-thread CTAs per SM") for m in (1, 2, 4) for t in threads]


def measure(kind, blocks, threads, iters, repeats, stream):
    lib = _lib.library()
    sink = torch.zeros(1, dtype=torch.float64, device="cuda")
    flops = ctypes.c_double()

    def run(n):
        _lib.check(lib.flashns_b200_fp64_probe(KINDS[kind], blocks, threads, n, ctypes.c_void_p(sink.data_ptr()),
                                               ctypes.byref(flops), ctypes.c_void_p(stream.cuda_stream)),
                   "fp64_probe")

    run(max(1, iters // 64))  # warm-up
    best = 0.0
    for _ in range(repeats):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        run(iters)
        e1.record(stream)
        e1.synchronize()
        best = max(best, flops.value / (e0.elapsed_time(e1) * 1e-3) / 1e12)
    return best


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--iters", type=int, default=4096)
    ap.add_argument("--repeats", type=int, default=3)
    ap.add_argument("--json", action="store_true", help="one JSON line per measurement")
    args = ap.parse_args()
    props = torch.cuda.get_device_properties(0)
    sms = props.multi_processor_count
    stream = torch.cuda.current_stream()
    rows = []
    for kind in KINDS:
        for blocks, threads, shape in launch_shapes(kind, sms):
            tf = measure(kind, blocks, threads, args.iters, args.repeats, stream)
            rows.append({"kind": kind, "blocks": blocks, "threads": threads, "shape": shape, "tflops": tf})
            if args.json:
                print(json.dumps(rows[-1]), flush=True)
    print(f"\n{props.name}, {sms} SMs\n")
    print("| kind | best TFLOP/s | launch shape |\n|---|---|---|")
    for kind in KINDS:
        mine = [r for r in rows if r["kind"] == kind]
        if kind == "smem":
            for r in mine:
                print(f"| smem-fed m16n8k8 | {r['tflops']:.2f} | {r['shape']} |")
        else:
            r = max(mine, key=lambda r: r["tflops"])
            print(f"| {kind} | {r['tflops']:.2f} | {r['shape']} |")


if __name__ == "__main__":
    main()
