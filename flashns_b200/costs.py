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
