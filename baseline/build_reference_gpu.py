"""Build the reference's own GPU kernels for B200, from the reference's sources, into
``baseline/_ref/``: a same-hardware baseline for ``bench.py --impl reference-gpu``.

    FLASHNS_REFERENCE=/path/to/FlashNS python baseline/build_reference_gpu.py

Nothing here is part of the product and nothing in the product loads these files.
The sources are compiled where they lie in the reference checkout (nothing is copied),
with the reference's own flags:

* ``libflashns_v8.so``  <- ``experiments/pinn_v8/native.cu``
  (recipe ``experiments/pinn_v8/build.py:31-32``: ``-O3 --fmad=false``);
* ``libstable.so``      <- ``experiments/cuda_jet_h100/stable_kernels.cu``
  (recipe ``experiments/cuda_jet_h100/build.py:34-45``);
* ``libdgrad_n64.so``   <- ``experiments/cuda_jet_h100/stable_dgrad.cu`` with CUTLASS
  headers.  The reference pins CUTLASS v4.7.1 (``build.py:14``), which is not on this
  machine; the CUTLASS tree vendored by the installed ``flashinfer`` package is used, and
  its version is recorded.  The kernel uses only the CUTLASS 2.x SM80 FP64 GEMM mainloop.

The target is ``sm_100`` (the reference derives ``-arch=sm_<major><minor>`` from the
device).  ``build.json`` records every command, the sha256 of every source and library,
and the CUTLASS version; the bindings refuse a library whose hash differs.
"""

import hashlib
import importlib.util
import json
import os
import re
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
ARCH = "sm_100"


def cutlass_include():
    spec = importlib.util.find_spec("flashinfer")
    if spec is None or not spec.submodule_search_locations:
        return None, None
    path = Path(list(spec.submodule_search_locations)[0]) / "data" / "cutlass" / "include"
    header = path / "cutlass" / "version.h"
    if not header.exists():
        return None, None
    text = header.read_text()
    parts = [re.search(rf"#define CUTLASS_{k} (\d+)", text) for k in ("MAJOR", "MINOR", "PATCH")]
    version = ".".join(m.group(1) for m in parts) if all(parts) else "unknown"
    return path, version


def sha256(path):
    return hashlib.sha256(Path(path).read_bytes()).hexdigest()


def recipes(reference):
    v8 = reference / "experiments" / "pinn_v8"
    h100 = reference / "experiments" / "cuda_jet_h100"
    include, version = cutlass_include()
    common = ["-std=c++17", "-O3", "-shared", "-Xcompiler=-fPIC", f"-arch={ARCH}"]
    jobs = [
        ("flashns_v8", v8 / "native.cu", common + ["--fmad=false"],
         [v8 / n for n in ("native.cu", "residual_generated.cuh", "coordinate_jet.cuh", "coordinate_wgrad.cuh",
                           "coordinate_activation_wgrad.cuh")] + [h100 / "stable_jet.cuh"]),
        ("stable", h100 / "stable_kernels.cu", common + ["--expt-relaxed-constexpr", "-lineinfo"],
         [h100 / "stable_kernels.cu", h100 / "stable_jet.cuh"]),
    ]
    if include is not None:
        jobs.append(("dgrad_n64", h100 / "stable_dgrad.cu",
                     common + ["--expt-relaxed-constexpr", "-lineinfo", f"-I{include}"],
                     [h100 / "stable_dgrad.cu", h100 / "stable_jet.cuh"]))
    return jobs, version


def build(reference, out=OUT):
    reference = Path(reference)
    if not (reference / "experiments" / "pinn_v8" / "native.cu").exists():
        raise FileNotFoundError(f"no reference CUDA sources under {reference}")
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    out.mkdir(parents=True, exist_ok=True)
    jobs, version = recipes(reference)
    report = {"arch": ARCH, "cutlass": {"used": version, "pinned_by_reference": "4.7.1"}, "libraries": {}}
    for name, source, flags, inputs in jobs:
        library = out / f"lib{name}.so"
        command = [nvcc, *flags, str(source), "-o", str(library)]
        result = subprocess.run(command, capture_output=True, text=True)
        if result.returncode:
            raise RuntimeError(f"nvcc failed for {source.name}:\n{result.stderr}")
        report["libraries"][name] = {
            "file": library.name,
            "command": [Path(command[0]).name] + [str(c).replace(str(reference), "<reference>")
                                                  .replace(str(HERE.parent), ".") for c in command[1:]],
            "sources": {str(p.relative_to(reference)): sha256(p) for p in inputs},
            "sha256": sha256(library),
        }
    (out / "build.json").write_text(json.dumps(report, indent=2) + "\n")
    return report


def main():
    root = os.environ.get("FLASHNS_REFERENCE") or (sys.argv[1] if len(sys.argv) > 1 else None)
    if not root:
        sys.exit("set FLASHNS_REFERENCE (or pass the path) to the root of a FlashNS checkout")
    report = build(root)
    for name, item in report["libraries"].items():
        print(name, item["file"], item["sha256"][:16])


if __name__ == "__main__":
    main()
