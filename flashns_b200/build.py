"""Build ``libflashns_b200.so`` in-tree for sm_100a with nvcc.

    python -m flashns_b200.build          # incremental
    python -m flashns_b200.build --force

Objects go to ``flashns_b200/_build/``; the shared library is written next to
this file so that it travels with the source tree.
"""

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
LIBRARY = HERE / "libflashns_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
         "-diag-suppress", "177", f"-I{ROOT / 'include'}", f"-I{CSRC}"]


def nvcc():
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build flashns_b200")
    return path


def sources():
    return sorted(CSRC.glob("*.cu"))


def dependencies():
    return sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))


def _stale(target, inputs):
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(p.stat().st_mtime > t for p in inputs)


def build(force=False, verbose=False):
    out_dir, library, flags = BUILD, LIBRARY, FLAGS
    out_dir.mkdir(exist_ok=True)
    deps = dependencies()
    compiler = nvcc()
    jobs = []
    for src in sources():
        obj = out_dir / (src.stem + ".o")
        if force or _stale(obj, [src, *deps]):
            jobs.append((src, obj))

    def compile_one(job):
        src, obj = job
        cmd = [compiler, *ARCH, *flags, "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        result = subprocess.run(cmd, capture_output=True, text=True)
        if result.returncode:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{result.stderr}")
        return result.stderr

    with ThreadPoolExecutor(max(1, min(len(jobs), os.cpu_count() or 1))) as pool:
        logs = list(pool.map(compile_one, jobs))
    if verbose:
        for log in logs:
            sys.stderr.write(log)
    objects = [out_dir / (s.stem + ".o") for s in sources()]
    if force or jobs or _stale(library, objects):
        tmp = library.with_suffix(".so.tmp")
        cmd = [compiler, *ARCH, "-shared", "-Xcompiler", "-fPIC", *map(str, objects), "-o", str(tmp)]
        result = subprocess.run(cmd, capture_output=True, text=True)
        if result.returncode:
            raise RuntimeError(f"link failed:\n{result.stderr}")
        os.replace(tmp, library)
    return library


def main():
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    args = parser.parse_args()
    print(build(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    main()
