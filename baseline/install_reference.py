"""Install the reference's Python package into ``baseline/_ref/`` for the timed CPU
reference arm of ``bench.py`` (``--impl reference`` and the ``cpu_baseline`` leg).

    FLASHNS_REFERENCE=/path/to/FlashNS python baseline/install_reference.py

Nothing in the product imports what this writes; ``baseline/_ref/`` is git-ignored and
travels to the GPU machine beside the built libraries.

The contract's install is ``pip install --no-index --no-build-isolation --find-links
<wheelhouse> --target baseline/_ref <reference>``.  The reference's ``pyproject.toml``
builds with ``hatchling`` (``[tool.hatch.build.targets.wheel] packages =
["src/flashns"]``), which is not installed on this machine and cannot be fetched, so
that command stops in its build backend.  The wheel it would build holds exactly the
``src/flashns`` package; when pip fails this script places that package under
``baseline/_ref/flashns`` unchanged, which is what the wheel's install would do.  The
reference's runtime dependencies (torch, numpy) are the machine's own.  ``install.json``
records which route was taken and the sha256 of every installed file.
"""

import hashlib
import json
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
WHEELHOUSE = Path("/opt/wheelhouse")


def sha256(path):
    return hashlib.sha256(Path(path).read_bytes()).hexdigest()


def install(reference, out=OUT):
    reference = Path(reference)
    package = reference / "src" / "flashns"
    if not (package / "pinn_packed.py").exists():
        raise FileNotFoundError(f"no flashns package under {reference}")
    out.mkdir(parents=True, exist_ok=True)
    target = out / "flashns"
    if target.exists():
        shutil.rmtree(target)
    command = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
               "--find-links", str(WHEELHOUSE), "--target", str(out), str(reference)]
    pip = subprocess.run(command, capture_output=True, text=True, timeout=600)
    route = "pip"
    if pip.returncode or not (target / "pinn_packed.py").exists():
        route = "package copy (pip failed: %s)" % (pip.stderr.strip().splitlines() or ["no output"])[-1][:200]
        shutil.copytree(package, target, ignore=shutil.ignore_patterns("__pycache__", "*.pyc"))
    files = {str(p.relative_to(out)): sha256(p) for p in sorted(target.rglob("*.py"))}
    report = {"route": route, "source": "src/flashns", "files": files}
    (out / "install.json").write_text(json.dumps(report, indent=2) + "\n")
    return report


def main():
    root = os.environ.get("FLASHNS_REFERENCE") or (sys.argv[1] if len(sys.argv) > 1 else None)
    if not root:
        sys.exit("set FLASHNS_REFERENCE (or pass the path) to the root of a FlashNS checkout")
    report = install(root)
    print(report["route"], len(report["files"]), "files")


if __name__ == "__main__":
    main()
