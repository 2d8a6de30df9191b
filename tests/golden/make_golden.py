"""Generate golden vectors by running the reference FlashNS code on the CPU.

Run from the repository root with the reference checkout available:

    FLASHNS_REFERENCE=/path/to/FlashNS python tests/golden/make_golden.py

It imports the reference package (``src/flashns``) read-only and records, for
seeded inputs, the outputs of:

* ``TensorActivation`` forward / VJP on packed layouts  (``src/flashns/jet_packed.py:91-133``)
* ``explicit_seed`` and ``residuals``                   (``src/flashns/ns_seed.py:54-87``)
* ``PackedPINN(layout="compact", seed="explicit")``      (``src/flashns/pinn_packed.py:15-191``)
  and the reference's independent nested-AD ``nested_step``
  (``sources/flashns_v8_reference/tests/verify_math.py:65-83``)

The fixtures are small ``.npz`` files committed beside this script; the tests
compare the oracle and the CUDA path against them without the reference.
"""

import importlib.util
import math
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
if "FLASHNS_REFERENCE" not in os.environ:
    sys.exit("set FLASHNS_REFERENCE to the root of a FlashNS checkout (the directory holding src/flashns)")
REF = Path(os.environ["FLASHNS_REFERENCE"])
sys.path.insert(0, str(REF / "src"))

from flashns.jet_packed import PackedLayout, TensorActivation  # noqa: E402
from flashns.ns_seed import NSLoss, explicit_seed, residual_terms, residuals  # noqa: E402
from flashns.pinn_packed import PackedPINN  # noqa: E402

_spec = importlib.util.spec_from_file_location(
    "reference_verify_math", REF / "sources/flashns_v8_reference/tests/verify_math.py")
_verify = importlib.util.module_from_spec(_spec)
sys.path.insert(0, str(REF / "sources/flashns_v8_reference/src"))
_spec.loader.exec_module(_verify)


def activation_cases():
    out = {}
    rng = np.random.default_rng(20261201)
    k = 0
    for dim in (2, 3):
        for full, value in ((5, 3), (0, 3), (3, 0), (4, 2)):
            layout = PackedLayout(full, value, dim)
            z = rng.normal(size=(layout.rows, 7)) * 0.3
            if full >= 3:
                q = layout.q
                z[q, :] += 20.0       # saturated centres, as tests/test_jet_stable.py:13-15
                z[2 * q, :] -= 20.0
            if value >= 2:
                z[layout.full_rows + 1, :] += 30.0
            seed = rng.normal(size=z.shape)
            ops = TensorActivation(layout)
            zt = torch.tensor(z)
            h, a = ops.forward(zt)
            dz = ops.vjp(h, a, torch.tensor(seed))
            p = f"act{k}_"
            out.update({p + "meta": np.array([dim, full, value]), p + "z": z, p + "seed": seed,
                        p + "h": h.numpy(), p + "a1": a.numpy(), p + "dz": dz.numpy()})
            k += 1
    out["act_count"] = np.array(k)
    return out


def seed_cases():
    out = {}
    rng = np.random.default_rng(61402)
    k = 0
    for batch, scale in ((1, 0.01), (7, 0.4), (7, 3.0), (33, 0.4)):
        j = rng.normal(size=(batch, 10, 3)) * scale
        w = rng.uniform(0.1, 1.0, batch) / batch
        w[0] = 0.0
        for viscosity, gw in ((0.0, 0.2), (0.07, 0.2), (0.2, 0.2), (0.05, 0.5)):
            loss = NSLoss(viscosity=viscosity, gradient_weight=gw)
            value, gradient = explicit_seed(torch.tensor(j), torch.tensor(w), loss)
            r = residuals(torch.tensor(j), loss)
            p = f"seed{k}_"
            out.update({p + "jets": j, p + "w": w, p + "nu_gamma": np.array([viscosity, gw]),
                        p + "loss": np.array(float(value)), p + "seed": gradient.numpy(),
                        p + "res": r.numpy()})
            k += 1
    out["seed_count"] = np.array(k)
    for m, nu in enumerate((0.0, 0.05, 0.07, 0.2)):
        rows = [(r, c, i, j) for r, terms in enumerate(residual_terms(nu)) for c, i, j in terms]
        out[f"terms{m}_nu"] = np.array(nu)
        out[f"terms{m}"] = np.array(rows, dtype=np.float64)
    return out


def make_case(ni, nb, widths, seed, scale):
    rng = np.random.default_rng(seed)
    x = rng.normal(size=(ni + nb, 2)) * scale
    ws = [rng.normal(size=(o, i)) * 0.7 / math.sqrt(i) for i, o in zip(widths, widths[1:])]
    bs = [rng.normal(size=o) * 0.1 for o in widths[1:]]
    pw = rng.uniform(0.2, 1.2, size=ni) / max(ni, 1)
    if ni >= 2:
        pw[0] = 0.0
    bw = rng.uniform(0.2, 1.2, size=(nb, 3)) / max(nb, 1)
    if nb:
        bw[:-1, 2] = 0.0
    target = rng.normal(size=(nb, 3)) * 0.3
    return x, ws, bs, pw, bw, target


def pinn_cases():
    out = {}
    cases = [
        (5, 3, (2, 7, 6, 3), 123, 0.4, NSLoss()),
        (17, 5, (2, 32, 31, 3), 7, 0.4, NSLoss()),
        (3, 2, (2, 7, 6, 3), 11, 3.0, NSLoss()),
        (1, 0, (2, 7, 6, 3), 5, 0.4, NSLoss()),
        (0, 3, (2, 7, 6, 3), 6, 0.4, NSLoss()),
        (40, 12, (2, 16, 16, 16, 3), 99, 0.5, NSLoss(viscosity=0.05, gradient_weight=0.2, boundary_weight=5.0)),
        (24, 9, (2, 64, 64, 3), 4, 0.5, NSLoss()),
        (9, 4, (2, 20, 3), 8, 0.6, NSLoss(viscosity=0.2, gradient_weight=0.5, boundary_weight=2.0)),
    ]
    for k, (ni, nb, widths, seed, scale, loss) in enumerate(cases):
        x, ws, bs, pw, bw, target = make_case(ni, nb, widths, seed, scale)
        step = PackedPINN(torch.tensor(x), ni, torch.tensor(pw), torch.tensor(bw), torch.tensor(target),
                          layout="compact", seed="explicit", loss=loss)
        value, grads = step([torch.tensor(w) for w in ws], [torch.tensor(b) for b in bs])
        p = f"pinn{k}_"
        out.update({p + "x": x, p + "ni": np.array(ni), p + "widths": np.array(widths),
                    p + "pw": pw, p + "bw": bw, p + "target": target,
                    p + "loss_coeffs": np.array([loss.viscosity, loss.gradient_weight, loss.boundary_weight]),
                    p + "loss": np.array(float(value))})
        for i, w in enumerate(ws):
            out[p + f"W{i}"] = w
        for i, b in enumerate(bs):
            out[p + f"b{i}"] = b
        for i, g in enumerate(grads):
            out[p + f"g{i}"] = g.numpy()
        if loss == NSLoss() and len(widths) == 4:
            nv, ng = _verify.nested_step(x, ws, bs, ni, pw, bw, target)
            out[p + "nested_loss"] = np.array(nv)
            for i, g in enumerate(ng):
                out[p + f"nested_g{i}"] = g
    out["pinn_count"] = np.array(len(cases))
    return out


def main():
    np.savez_compressed(HERE / "reference_activation.npz", **activation_cases())
    np.savez_compressed(HERE / "reference_seed.npz", **seed_cases())
    np.savez_compressed(HERE / "reference_packed_pinn.npz", **pinn_cases())
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
