"""Emit the straight-line device math for jets and residual seeds.

The generated headers ``csrc/jets_generated.cuh`` and
``csrc/residual_generated.cuh`` are committed; ``python -m flashns_b200.codegen``
rewrites them and ``tests/test_codegen.py`` checks that they are current.

Jet math (factorial-normalized Taylor coefficients, basis order of
``src/flashns/jet_spec.py:30-41``):

* forward: ``h = a1*d - t*a1*d^2 + a1*(t^2-1/3)*d^3``, ``h_0 = tanh z_0``,
  ``a1 = (2r/(1+r^2))^2`` with ``r = exp(-|z_0|)``  (``src/flashns/jet_stable.py:14-19,62-76``)
* VJP: ``g = -(H*H)``, ``g_0 = a1``, ``zbar_b = sum_{a>=b} hbar_a g_{a-b}``
  (``src/flashns/jet_packed.py:76-88``)

Residual seeds: each residual is a polynomial in raw derivatives written from
the PDE (``src/flashns/ns_seed.py:26-43`` lists the same nine polynomials of the
(u, v, p) head in coefficient form).  Coefficients are affine in the viscosity
``nu``, so each monomial carries ``a + b*nu``.
"""

from functools import lru_cache
from itertools import product
from math import factorial, prod
from pathlib import Path

HERE = Path(__file__).resolve().parent


@lru_cache(None)
def basis(dim, order=3):
    full = sorted((a for a in product(range(4), repeat=dim) if sum(a) <= 3), key=lambda a: (sum(a), a))
    return tuple(a for a in full if sum(a) <= order)


def pairs(dim, order):
    b = basis(dim, order)
    lookup = {a: i for i, a in enumerate(b)}
    out = []
    for g in b:
        out.append(tuple((i, lookup[tuple(y - x for x, y in zip(a, g))])
                         for i, a in enumerate(b) if all(x <= y for x, y in zip(a, g))))
    return out


def _lit(v):
    s = repr(float(v))
    return s if ("e" in s or "." in s) else s + ".0"


# --------------------------------------------------------------------------- jets

def _sym_sum(terms, value):
    """Sum of value(i, j) over ordered pairs, each unordered pair computed once."""
    seen, parts = set(), []
    for i, j in terms:
        key = (min(i, j), max(i, j))
        if key in seen:
            continue
        seen.add(key)
        parts.append(value(i, j) if i == j else f"2.0 * ({value(i, j)})")
    return " + ".join(parts)


# Stable tanh and a1 from one exponential (all FP64 units are shared with the DMMA
# main loop, so every instruction of the epilogue counts):
#   r = exp(-|z0|), inv = 1/(1+r^2):  a1 = (2 r inv)^2 = sech^2 z0,  tanh|z0| = (1 - r^2) inv.
# (1 - r^2) carries an absolute rounding error of a few ulp(1); below |z0| = 2^-10 the odd
# Taylor series z (1 - z^2/3 + 2 z^4/15) (next term 17 z^7/315 < 1e-22 |z|) is used instead.
_STABLE = """  const double z0 = z[0];
  const double az = fabs(z0);
  const double r = exp(-az);
  const double r2 = r * r;
  const double inv = 1.0 / (1.0 + r2);
  const double v = 2.0 * r * inv;
  a1 = v * v;
  double ta = (1.0 - r2) * inv;
  if (az < 0x1p-10) {
    const double q = az * az;
    ta = az * (1.0 - q * (1.0 / 3.0 - q * (2.0 / 15.0)));
  }
  const double t = copysign(ta, z0);"""


def jet_forward(dim, order):
    b = basis(dim, order)
    q = len(b)
    name = f"jet_fwd_{dim}d{order}"
    L = [f"// tanh jet, dim {dim}, order {order}: {q} coefficients",
         f"__device__ __forceinline__ void {name}(const double* z, double* h, double& a1) {{",
         _STABLE,
         "  h[0] = t;"]
    if order >= 2:
        L.append("  const double a2 = -(t * a1);")
    if order >= 3:
        L.append("  const double a3 = a1 * (t * t - (1.0 / 3.0));")
    if order >= 2:
        pr = pairs(dim, order)
        for g, a in enumerate(b):
            if sum(a) >= 2:
                terms = [(i, j) for i, j in pr[g] if i != 0 and j != 0]
                L.append(f"  const double p2_{g} = {_sym_sum(terms, lambda i, j: f'z[{i}] * z[{j}]')};")
        for g, a in enumerate(b):
            if sum(a) == 3:
                terms = [(i, j) for i, j in pr[g] if sum(b[i]) == 2 and sum(b[j]) == 1]
                expr = " + ".join(f"p2_{i} * z[{j}]" for i, j in terms)
                L.append(f"  const double p3_{g} = {expr};")
    for g, a in enumerate(b):
        s = sum(a)
        if s == 1:
            L.append(f"  h[{g}] = a1 * z[{g}];")
        elif s == 2:
            L.append(f"  h[{g}] = a1 * z[{g}] + a2 * p2_{g};")
        elif s == 3:
            L.append(f"  h[{g}] = (a1 * z[{g}] + a2 * p2_{g}) + a3 * p3_{g};")
    L.append("}")
    return "\n".join(L)


def jet_vjp(dim, order):
    b = basis(dim, order)
    q = len(b)
    name = f"jet_vjp_{dim}d{order}"
    pr = pairs(dim, order)
    L = [f"// transpose of the tanh-jet Jacobian, dim {dim}, order {order}",
         f"__device__ __forceinline__ void {name}(const double* h, double a1, const double* hb, double* zb) {{"]
    if order == 0:
        L += ["  zb[0] = hb[0] * a1;", "}"]
        return "\n".join(L)
    # g_gamma = -(H*H)_gamma for |gamma|>=1
    for g in range(1, q):
        L.append(f"  const double g{g} = -({_sym_sum(pr[g], lambda i, j: f'h[{i}] * h[{j}]')});")
    L.append("  const double g0 = a1;")
    for beta in range(q):
        # zbar_beta = sum_{alpha >= beta} hb[alpha] * g[alpha - beta]
        terms = []
        for alpha in range(q):
            for i, j in pr[alpha]:
                if i == beta:
                    terms.append(f"hb[{alpha}] * g{j}")
        L.append(f"  zb[{beta}] = {' + '.join(terms)};")
    L.append("}")
    return "\n".join(L)


def jets_header():
    parts = ["// GENERATED by flashns_b200/codegen.py -- do not edit.",
             "#pragma once", "namespace flashns_b200 {"]
    for dim in (2, 3):
        for order in (0, 1, 3):
            parts.append(jet_forward(dim, order))
            parts.append(jet_vjp(dim, order))
    parts.append("}  // namespace flashns_b200")
    return "\n\n".join(parts) + "\n"


# ----------------------------------------------------------------- residual polynomials
# expression: {factors(tuple of (field, alpha)): (const, nu)}

def _add(*es):
    out = {}
    for e in es:
        for k, (a, b) in e.items():
            c = out.get(k, (0.0, 0.0))
            out[k] = (c[0] + a, c[1] + b)
    return {k: c for k, c in out.items() if c != (0.0, 0.0)}


def _mul(x, y):
    out = {}
    for kx, (ax, bx) in x.items():
        for ky, (ay, by) in y.items():
            if bx and by:
                raise ValueError("nu^2 term")
            k = tuple(sorted(kx + ky))
            c = out.get(k, (0.0, 0.0))
            out[k] = (c[0] + ax * ay, c[1] + ax * by + bx * ay)
    return {k: c for k, c in out.items() if c != (0.0, 0.0)}


def _scale_nu(e, s):
    """Multiply a nu-free expression by s*nu."""
    return {k: (0.0, a * s) for k, (a, b) in e.items()}


def _diff(e, axis):
    out = {}
    for k, (a, b) in e.items():
        for pos, (f, al) in enumerate(k):
            nl = list(al)
            nl[axis] += 1
            nk = tuple(sorted(k[:pos] + ((f, tuple(nl)),) + k[pos + 1:]))
            c = out.get(nk, (0.0, 0.0))
            out[nk] = (c[0] + a, c[1] + b)
    return {k: c for k, c in out.items() if c != (0.0, 0.0)}


def _d(dim, field, coeff, *axes):
    al = [0] * dim
    for x in axes:
        al[x] += 1
    return {((field, tuple(al)),): (coeff, 0.0)}


def residuals_uvp():
    X, Y = 0, 1
    U = lambda *a: _d(2, 0, 1.0, *a)
    V = lambda *a: _d(2, 1, 1.0, *a)
    P = lambda *a: _d(2, 2, 1.0, *a)
    ru = _add(_mul(U(), U(X)), _mul(V(), U(Y)), P(X), _scale_nu(_add(U(X, X), U(Y, Y)), -1.0))
    rv = _add(_mul(U(), V(X)), _mul(V(), V(Y)), P(Y), _scale_nu(_add(V(X, X), V(Y, Y)), -1.0))
    div = _add(U(X), V(Y))
    base = [ru, rv, div]
    return base + [_diff(r, X) for r in base] + [_diff(r, Y) for r in base], [0, 0, 0, 1, 1, 1, 1, 1, 1]


def residuals_psi(dim):
    X, Y = 0, 1
    u = lambda *a: _d(dim, 0, 1.0, Y, *a)
    v = lambda *a: _d(dim, 0, -1.0, X, *a)
    P = lambda *a: _d(dim, 1, 1.0, *a)
    ru = _add(_mul(u(), u(X)), _mul(v(), u(Y)), P(X), _scale_nu(_add(u(X, X), u(Y, Y)), -1.0))
    rv = _add(_mul(u(), v(X)), _mul(v(), v(Y)), P(Y), _scale_nu(_add(v(X, X), v(Y, Y)), -1.0))
    if dim == 3:
        ru = _add(ru, u(2))
        rv = _add(rv, v(2))
    return [ru, rv], [0, 0]


def residual_function(name, dim, nf, residuals, groups):
    """C++: loss of one interior point and the seed dy[Q*F] (coefficient-major)."""
    lookup = {a: i for i, a in enumerate(basis(dim))}
    q = len(basis(dim))
    L = [f"// interior residual loss + seed: dim {dim}, {nf} fields; y[i*{nf}+f] = coefficient i of field f",
         f"__device__ __forceinline__ double {name}(const double* y, double w, double nu, double gamma, double* dy) {{",
         f"  #pragma unroll\n  for (int k = 0; k < {q * nf}; ++k) dy[k] = 0.0;",
         "  double loss = 0.0;"]
    for k, (r, grp) in enumerate(zip(residuals, groups)):
        mons = []
        for key, (a, b) in sorted(r.items()):
            fac = 1.0
            slots = []
            for f, al in key:
                fac *= prod(factorial(v) for v in al)
                slots.append(lookup[al] * nf + f)
            mons.append(((a * fac, b * fac), slots))
        def coef(c):
            a, b = c
            if b == 0.0:
                return _lit(a)
            if a == 0.0:
                return f"({_lit(b)} * nu)"
            return f"({_lit(a)} + {_lit(b)} * nu)"
        expr = " + ".join(f"{coef(c)} * " + " * ".join(f"y[{s}]" for s in sl) for c, sl in mons)
        L.append(f"  const double r{k} = {expr};")
        scale = "w" if grp == 0 else "(w * gamma)"
        L.append(f"  const double d{k} = {scale} * r{k};")
        L.append(f"  loss += 0.5 * (d{k} * r{k});")
        for c, sl in mons:
            for pos, s in enumerate(sl):
                others = [f"y[{o}]" for i2, o in enumerate(sl) if i2 != pos]
                term = " * ".join([coef(c), f"d{k}"] + others)
                L.append(f"  dy[{s}] += {term};")
    L.append("  return loss;")
    L.append("}")
    return "\n".join(L)


def residual_values_function(name, dim, nf, residuals):
    lookup = {a: i for i, a in enumerate(basis(dim))}
    L = [f"__device__ __forceinline__ void {name}(const double* y, double nu, double* r) {{"]
    for k, res in enumerate(residuals):
        terms = []
        for key, (a, b) in sorted(res.items()):
            fac = 1.0
            slots = []
            for f, al in key:
                fac *= prod(factorial(v) for v in al)
                slots.append(lookup[al] * nf + f)
            c = _lit(a * fac) if b == 0.0 else (f"({_lit(b * fac)} * nu)" if a == 0.0 else f"({_lit(a * fac)} + {_lit(b * fac)} * nu)")
            terms.append(f"{c} * " + " * ".join(f"y[{s}]" for s in slots))
        L.append(f"  r[{k}] = {' + '.join(terms)};")
    L.append("}")
    return "\n".join(L)


def residual_header():
    parts = ["// GENERATED by flashns_b200/codegen.py -- do not edit.", "#pragma once",
             "namespace flashns_b200 {"]
    res, grp = residuals_uvp()
    parts.append(residual_function("seed_uvp_2d", 2, 3, res, grp))
    parts.append(residual_values_function("residuals_uvp_2d", 2, 3, res))
    for dim in (2, 3):
        res, grp = residuals_psi(dim)
        parts.append(residual_function(f"seed_psi_{dim}d", dim, 2, res, grp))
        parts.append(residual_values_function(f"residuals_psi_{dim}d", dim, 2, res))
    parts.append("}  // namespace flashns_b200")
    return "\n\n".join(parts) + "\n"


def outputs():
    return {HERE / "csrc" / "jets_generated.cuh": jets_header(),
            HERE / "csrc" / "residual_generated.cuh": residual_header()}


def main():
    for path, text in outputs().items():
        path.write_text(text)
        print("wrote", path)


if __name__ == "__main__":
    main()
