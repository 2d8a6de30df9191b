"""What slows the FP64 tensor pipe: the DMMA rate of 8 warps running the evaluation
kernels' shared-memory-fed m16n8k8 loop while the other 8 warps of the CTA run one kind of
other work (FP64 chains, ``exp``, shared loads, integer work, global stores of several
forms, bulk stores).  Measurement infrastructure beside the baselines; nothing in the
product imports it.

    python -m baseline.dmma_interference [--iters 4096]

Builds ``baseline/dmma_interference.cu`` with nvcc for sm_100a into ``baseline/_build/``
when the binary is missing or older than the source, runs it on the current GPU and
prints a Markdown table: the DMMA rate as a fraction of the full rate (64 cycles per
m16n8k8 per SM sub-partition) and the bytes the other warps stored per clock per SM.
"""

import argparse
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SOURCE = HERE / "dmma_interference.cu"
BINARY = HERE / "_build" / "dmma_interference"


def build():
    if BINARY.exists() and BINARY.stat().st_mtime >= SOURCE.stat().st_mtime:
        return BINARY
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    BINARY.parent.mkdir(exist_ok=True)
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17", str(SOURCE), "-o",
           str(BINARY)]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode:
        raise RuntimeError(f"nvcc failed:\n{result.stderr}")
    return BINARY


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--iters", type=int, default=4096, help="rounds of the DMMA loop per MMA warp")
    ap.add_argument("--build-only", action="store_true")
    args = ap.parse_args(argv)
    binary = build()
    if args.build_only:
        return 0
    return subprocess.run([str(binary), str(args.iters)]).returncode


if __name__ == "__main__":
    sys.exit(main())
