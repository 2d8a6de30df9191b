"""CPU: the timed reference arm (baseline/reference_cpu.py) runs the reference's own
PackedPINN on the objective it claims, the (u, v, p) head on the configuration's point set:
its loss and gradient equal the oracle's on a small chunk, and its chunked timing covers
the whole set.  Skipped where the reference package is not installed in baseline/_ref/
(baseline/install_reference.py)."""

import json
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

from baseline.reference_cpu import available  # noqa: E402

pytestmark = pytest.mark.skipif(not available(), reason="reference package not installed in baseline/_ref")


def test_reference_arm_objective_matches_the_oracle():
    """One chunk of cfg0's point set through the reference's PackedPINN (in a child
    process, as the arm runs it) against the oracle's uvp evaluation of the same inputs."""
    code = """
import json, sys
sys.path.insert(0, {root!r})
import torch
from baseline.reference_cpu import REF, reference_inputs
sys.path.insert(0, str(REF))
from flashns.ns_seed import NSLoss
from flashns.pinn_packed import PackedPINN
x, ni, pw, bw, target, ws, bs, widths, nu = reference_inputs("cfg0")
nb = len(x) - ni
i1, b1 = ni // 16, nb // 16
xs = torch.cat((x[:i1], x[ni:ni + b1]))
step = PackedPINN(xs, i1, pw[:i1].contiguous(), bw[:b1].contiguous(), target[:b1].contiguous(),
                  layout="compact", seed="explicit", loss=NSLoss(viscosity=nu, gradient_weight=0.2, boundary_weight=5.0))
loss, grads = step(ws, bs)
print(json.dumps({{"loss": float(loss), "grad": torch.cat([g.reshape(-1) for g in grads]).tolist(),
                  "widths": widths, "nu": nu, "i1": i1, "b1": b1}}))
""".format(root=str(ROOT))
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, cwd=ROOT, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    got = json.loads(out.stdout.strip().splitlines()[-1])
    from baseline.reference_cpu import reference_inputs
    from oracle.evaluate import evaluate
    from tests.cases import close_ratio
    x, ni, pw, bw, target, ws, bs, widths, nu = reference_inputs("cfg0")
    i1, b1 = got["i1"], got["b1"]
    xs = np.concatenate((x[:i1].numpy(), x[ni:ni + b1].numpy()))
    loss, grads = evaluate(xs, i1, pw[:i1].numpy(), bw[:b1].numpy(), target[:b1].numpy(), [w.numpy() for w in ws],
                           [b.numpy() for b in bs], head="uvp", nu=nu, gamma=0.2, bc=5.0, boundary_order=0)
    assert got["widths"] == [2, 64, 64, 64, 64, 3]
    assert close_ratio(got["loss"], loss) <= 1.0
    assert close_ratio(np.array(got["grad"]), np.concatenate([g.reshape(-1) for g in grads])) <= 1.0


def test_reference_arm_chunks_cover_the_set():
    """With --parts M the arm's steps evaluate disjoint chunks that together are the set."""
    cmd = [sys.executable, "-m", "baseline.reference_cpu", "--config", "cfg0", "--steps", "2", "--warmup", "0",
           "--parts", "4", "--threads", "2"]
    out = subprocess.run(cmd, capture_output=True, text=True, cwd=ROOT, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    r = json.loads(out.stdout.strip().splitlines()[-1])
    assert r["parts"] == 4 and r["interior"] == 2048 and r["boundary"] == 512 and len(r["times_s"]) == 2
    assert r["value"] > 0 and r["module"].startswith("baseline/_ref/flashns/")
