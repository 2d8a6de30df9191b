"""Algorithmic FLOP and byte counts of one evaluation, per kernel kind.

GEMM work uses the true (unpadded) widths; pointwise work is counted from the
generated jet and residual formulas (each binary * + - / is one flop; tanh and
exp calls count zero, so the figures are lower bounds).
"""

import re
from functools import lru_cache

from flashns_b200 import codegen


def _ops(text):
    body = text[text.index("{") + 1:]
    body = re.sub(r"\b(tanh|exp|fabs)\(", "(", body)
    body = re.sub(r"(\[\s*[0-9]+\s*\])", "", body)  # array subscripts
    return len(re.findall(r"(?<=\s)[*+/-](?=\s)", body))


@lru_cache(None)
def jet_flops(dim, order):
    return _ops(codegen.jet_forward(dim, order)), _ops(codegen.jet_vjp(dim, order))


@lru_cache(None)
def seed_flops(head, dim):
    if head == "uvp":
        res, grp = codegen.residuals_uvp()
        text = codegen.residual_function("f", 2, 3, res, grp)
    else:
        res, grp = codegen.residuals_psi(dim)
        text = codegen.residual_function("f", dim, 2, res, grp)
    return _ops(text)


def padded_width(c):
    return 32 if c <= 32 else 64 if c <= 64 else 128


def fused_backward(widths, layer):
    """Mirror of the plan: square 64-wide hidden layers run dgrad + VJP + wgrad in one kernel."""
    return padded_width(widths[layer]) == 64 and padded_width(widths[layer + 1]) == 64


def fused_head(widths):
    """Mirror of the plan: a square 64-wide last hidden layer runs with the output layer."""
    nh = len(widths) - 2
    return nh >= 2 and padded_width(widths[nh]) == 64 and padded_width(widths[nh - 1]) == 64


def evaluation_costs(widths, ni, nb, *, head, boundary_order):
    """Dict kind -> list of per-launch FLOPs, in launch order, plus totals."""
    dim = widths[0]
    q = 10 if dim == 2 else 20
    qb = dim + 1 if boundary_order else 1
    rows = ni * q + nb * qb
    points = ni + nb
    nf = widths[-1]
    nh = len(widths) - 2
    f3, v3 = jet_flops(dim, 3)
    fb, vb = jet_flops(dim, 1 if boundary_order else 0)
    out = {"first": [], "forward": [], "head": [], "backward": [], "wgrad": []}
    c1 = widths[1]
    out["first"].append(ni * c1 * (2 * dim + f3) + nb * c1 * (2 * dim + fb))
    for l in range(1, nh):
        cin, cout = widths[l], widths[l + 1]
        out["forward"].append(2 * rows * cin * cout + points * cout + ni * cout * f3 + nb * cout * fb)
    c = widths[nh]
    out["head"].append(2 * rows * c * nf + points * nf + ni * seed_flops(head, dim) + nb * 6 * nf
                       + 2 * rows * nf * c + points * nf + 2 * rows * nf * c + ni * c * v3 + nb * c * vb)
    for l in range(nh - 1, 0, -1):
        cin, cout = widths[l], widths[l + 1]
        extra = points * cin * (2 * dim + 1) if l == 1 else 0
        wgrad = 2 * rows * cout * cin
        bwd = 2 * rows * cout * cin + ni * cin * v3 + nb * cin * vb + extra + points * cin
        if fused_backward(widths, l):
            out["backward"].append(bwd + wgrad)
        else:
            out["backward"].append(bwd)
            out["wgrad"].append(wgrad)
    if nh == 1:
        out["head"][0] += points * c1 * (2 * dim + 1)
    if fused_head(widths):
        out["forward_head"] = [out["forward"].pop() + out["head"].pop()]
    total = sum(sum(v) for v in out.values())
    gemm = 2 * rows * sum(a * b for a, b in zip(widths, widths[1:])) * 3 - 2 * rows * dim * c1
    return {"per_kind": out, "total": total, "gemm": gemm, "rows": rows}


def evaluation_bytes(widths, ni, nb, *, head, boundary_order):
    """Dict kind -> list of per-launch compulsory DRAM bytes, in the launch order of
    ``evaluation_costs``: every checkpoint, auxiliary and seed a launch must read or write
    once (FP64), plus its inputs (coordinates, objective weights and targets).  Weights,
    biases and the per-CTA partials are left out (KB against the MB-GB tensors).

    * first: x in; H_1 and a1_1 out.
    * forward l: H_l in; H_{l+1}, a1_{l+1} out.
    * head: H_L, a1_L, objective in; D_L out (with a single hidden layer: x in instead,
      bar_Z_1 contracted on chip).  forward_head (fused): H_{L-1} and the objective in,
      D_L out (H_L and a1_L stay on chip).
    * backward l: D_{l+1}, H_l, a1_l in; D_l out, except layer 1, whose bar_Z_1 is
      contracted with the coordinate jets (x in) and never stored.
    * wgrad l (when not fused into backward): D_{l+1} and H_l in.
    """
    dim = widths[0]
    q = 10 if dim == 2 else 20
    qb = dim + 1 if boundary_order else 1
    rows = ni * q + nb * qb
    points = ni + nb
    nh = len(widths) - 2
    f = 3 if (head == "uvp" or boundary_order) else 2
    objective = 8 * (ni + 2 * nb * f)
    x = 8 * points * dim
    hbytes = lambda c: 8 * rows * c
    abytes = lambda c: 8 * points * c
    out = {"first": [x + hbytes(widths[1]) + abytes(widths[1])], "forward": [], "head": [], "backward": [],
           "wgrad": []}
    for l in range(1, nh):
        out["forward"].append(hbytes(widths[l]) + hbytes(widths[l + 1]) + abytes(widths[l + 1]))
    c = widths[nh]
    # with one hidden layer the head also contracts bar_Z_1 with the coordinates (x in,
    # no seed out)
    out["head"].append(hbytes(c) + abytes(c) + objective + (x if nh == 1 else hbytes(c)))
    for l in range(nh - 1, 0, -1):
        cin, cout = widths[l], widths[l + 1]
        seeds_and_checkpoints = hbytes(cout) + hbytes(cin) + abytes(cin)
        # layer 1 reads the coordinates instead of writing bar_Z_1
        out["backward"].append(seeds_and_checkpoints + (x if l == 1 else hbytes(cin)))
        if not fused_backward(widths, l):
            out["wgrad"].append(hbytes(cout) + hbytes(cin))
    if fused_head(widths):
        out["forward"].pop()
        out["head"].pop()
        out["forward_head"] = [hbytes(widths[nh - 1]) + objective + hbytes(c)]
    return out


def kernel_rooflines(times, flops, dram_bytes, fp64_peak_tflops, hbm_peak_gbs):
    """Per kernel kind: achieved FP64 TFLOP/s and compulsory-traffic GB/s, each against its
    peak, from the mean launch time ``times[kind]["avg_ms"]`` and the mean per-launch
    figures of ``evaluation_costs`` / ``evaluation_bytes``.  Kinds without a model (the
    parameter packing, the final reduction) keep only their times."""
    out = {}
    for kind, t in times.items():
        row = dict(t)
        ms = t.get("avg_ms")
        if ms and flops.get(kind) and dram_bytes.get(kind):
            f = sum(flops[kind]) / len(flops[kind])
            b = sum(dram_bytes[kind]) / len(dram_bytes[kind])
            tflops, gbs = f / (ms * 1e-3) / 1e12, b / (ms * 1e-3) / 1e9
            row.update(tflops=tflops, fp64_frac=tflops / fp64_peak_tflops, gbs=gbs, hbm_frac=gbs / hbm_peak_gbs,
                       flops_per_launch=f, dram_bytes_per_launch=b)
        out[kind] = row
    return out


def checkpoint_bytes(widths, ni, nb, *, boundary_order):
    """Compulsory HBM bytes: each hidden checkpoint written and read once, a1 likewise,
    one seed buffer per hidden layer written and read, inputs and the gradient."""
    dim = widths[0]
    q = 10 if dim == 2 else 20
    qb = dim + 1 if boundary_order else 1
    rows = ni * q + nb * qb
    points = ni + nb
    hidden = widths[1:-1]
    p = sum(a * b + b for a, b in zip(widths, widths[1:]))
    b = sum(2 * 8 * (rows * c + points * c) for c in hidden)
    b += sum(2 * 8 * rows * c for c in hidden[:-1])
    return b + 8 * (points * dim + 2 * p)
