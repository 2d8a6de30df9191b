"""Seeded test cases shared by the CPU and GPU tests."""

import math

import numpy as np

GOLDEN = __import__("pathlib").Path(__file__).resolve().parent / "golden"


def close_ratio(actual, expected, atol=2e-12, rtol=2e-11):
    """max |a-b| / (atol + rtol |b|): the reference criterion
    (sources/flashns_v8_reference/tests/verify_math.py:35-41)."""
    a = np.asarray(actual, dtype=np.float64)
    b = np.asarray(expected, dtype=np.float64)
    assert a.shape == b.shape, (a.shape, b.shape)
    assert np.isfinite(a).all() and np.isfinite(b).all(), "non-finite values"
    return float(np.max(np.abs(a - b) / (atol + rtol * np.abs(b)), initial=0.0))


def rel_norm(actual, expected):
    a = np.asarray(actual, dtype=np.float64).ravel()
    b = np.asarray(expected, dtype=np.float64).ravel()
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / den) if den else float(np.linalg.norm(a))


def random_case(ni, nb, widths, *, head="uvp", boundary_order=0, seed=1, scale=0.4, zero_weights=True):
    """Random points, parameters (0.7/sqrt(fan_in)), unequal/partly zero weights."""
    rng = np.random.default_rng(seed)
    dim = widths[0]
    x = rng.normal(size=(ni + nb, dim)) * scale
    ws = [rng.normal(size=(o, i)) * 0.7 / math.sqrt(i) for i, o in zip(widths, widths[1:])]
    bs = [rng.normal(size=o) * 0.1 for o in widths[1:]]
    f = 3 if (head == "uvp" or boundary_order == 1) else 2
    pw = rng.uniform(0.2, 1.2, size=ni) / max(ni, 1)
    if zero_weights and ni >= 2:
        pw[0] = 0.0
    bw = rng.uniform(0.2, 1.2, size=(nb, f)) / max(nb, 1)
    if zero_weights and nb:
        bw[:-1, f - 1] = 0.0
    target = rng.normal(size=(nb, f)) * 0.3
    return dict(x=x, ni=ni, pw=pw, bw=bw, target=target, ws=ws, bs=bs)


def flat(ws, bs):
    return np.concatenate([w.reshape(-1) for w in ws] + [b.reshape(-1) for b in bs])


def golden_pinn_cases():
    g = np.load(GOLDEN / "reference_packed_pinn.npz")
    out = []
    for k in range(int(g["pinn_count"])):
        p = f"pinn{k}_"
        widths = [int(v) for v in g[p + "widths"]]
        n = len(widths) - 1
        nu, gamma, bc = (float(v) for v in g[p + "loss_coeffs"])
        out.append(dict(name=f"pinn{k}", x=g[p + "x"], ni=int(g[p + "ni"]), pw=g[p + "pw"], bw=g[p + "bw"],
                        target=g[p + "target"], widths=widths,
                        ws=[g[p + f"W{i}"] for i in range(n)], bs=[g[p + f"b{i}"] for i in range(n)],
                        nu=nu, gamma=gamma, bc=bc, loss=float(g[p + "loss"]),
                        grads=[g[p + f"g{i}"] for i in range(2 * n)]))
    return out
