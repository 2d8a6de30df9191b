"""Seeded synthetic point sets of the benchmark configurations.

Kovasznay flow (steady 2-D NS, Re = 20 unless given): on [-0.5, 1] x [-0.5, 1.5],
``lambda = Re/2 - sqrt(Re^2/4 + 4 pi^2)``, ``nu = 1/Re`` and

    u = 1 - e^{lambda x} cos 2 pi y,   v = lambda/(2 pi) e^{lambda x} sin 2 pi y,
    p = (1 - e^{2 lambda x}) / 2,      psi = y - e^{lambda x} sin(2 pi y) / (2 pi)

Taylor-Green vortex (unsteady 2-D NS): on (x, y, t) in [0, 2 pi]^2 x [0, 1] with
``F = e^{-2 nu t}``: ``u = -cos x sin y F``, ``v = sin x cos y F``,
``p = -(cos 2x + cos 2y) F^2 / 4``, ``psi = cos x cos y F``.

Interior points are uniform; boundary points are uniform on the edges (Kovasznay:
equal counts per edge) or, for Taylor-Green, half on the initial slice t = 0 and
half on the four periodic faces.  The pressure gauge follows the reference solver
(experiments/pinn_solver/problem.py:101-107): exact p is imposed on the x = 1
outflow edge only for Kovasznay; for Taylor-Green on every boundary point.
Weights are globally normalized: 1/Ni for the PDE, 1/Nb for boundary velocity,
1/(points carrying the p target) for pressure.
"""

import math
from dataclasses import dataclass

import torch

from flashns_b200.distributed_contract import shard_bounds


@dataclass
class PointSet:
    x: torch.Tensor            # [ni + nb, dim], interior first
    interior_count: int
    pde_weights: torch.Tensor  # [ni]
    boundary_weights: torch.Tensor  # [nb, F]
    target: torch.Tensor       # [nb, F]
    dim: int
    viscosity: float
    name: str

    def shard(self, world, rank):
        """Rank's contiguous share of interior and of boundary points (weights stay global)."""
        ni = self.interior_count
        nb = len(self.x) - ni
        i0, i1 = shard_bounds(ni, world, rank)
        b0, b1 = shard_bounds(nb, world, rank)
        x = torch.cat((self.x[i0:i1], self.x[ni + b0:ni + b1]))
        return PointSet(x, i1 - i0, self.pde_weights[i0:i1], self.boundary_weights[b0:b1], self.target[b0:b1],
                        self.dim, self.viscosity, f"{self.name}[{rank}/{world}]")


def kovasznay_lambda(re):
    return re / 2 - math.sqrt(re * re / 4 + 4 * math.pi ** 2)


def kovasznay_exact(x, re=20.0):
    lam = kovasznay_lambda(re)
    e = torch.exp(lam * x[:, 0])
    a = 2 * math.pi * x[:, 1]
    u = 1 - e * torch.cos(a)
    v = lam / (2 * math.pi) * e * torch.sin(a)
    p = 0.5 * (1 - e * e)
    psi = x[:, 1] - e * torch.sin(a) / (2 * math.pi)
    return u, v, p, psi


SAMPLINGS = ("uniform", "sobol", "philox")


def sobol_engine(dim, seed, stream=0):
    """The scrambled Sobol engine of one point family: seeded by `seed` and `stream`, so
    separate families get independent sequences."""
    return torch.quasirandom.SobolEngine(dim, scramble=True, seed=seed * 1009 + stream)


def philox_key(seed, stream=0):
    """(key0, key1) of a family's Philox4x64-10 stream."""
    if not 0 <= seed < 2 ** 64 or not 0 <= stream < 2 ** 64:
        raise ValueError("philox sampling needs 0 <= seed, stream < 2^64")
    return seed, stream


def unit_samples(n, dim, gen, sampling, seed, stream=0):
    """n points in [0, 1)^dim on the host.

    * ``uniform``: torch's CPU generator `gen` (host only);
    * ``sobol``: scrambled Sobol from ``sobol_engine(dim, seed, stream)``;
    * ``philox``: Philox4x64-10 keyed by ``philox_key(seed, stream)``, the stream of
      ``numpy.random.Generator(numpy.random.Philox(key=key0 + 2^64 key1)).random()``.

    The device kernels draw the Sobol and Philox families bit for bit alike
    (``sample_points``)."""
    if sampling not in SAMPLINGS:
        raise ValueError(f"sampling must be one of {SAMPLINGS}")
    if n == 0:
        return torch.zeros(0, dim, dtype=torch.float64)
    if sampling == "uniform":
        return torch.rand(n, dim, generator=gen, dtype=torch.float64)
    if sampling == "sobol":
        return sobol_engine(dim, seed, stream).draw(n, dtype=torch.float64)
    import numpy as np
    k0, k1 = philox_key(seed, stream)
    rng = np.random.Generator(np.random.Philox(key=k0 + (k1 << 64)))
    return torch.from_numpy(rng.random((n, dim)))


def sample_points(n, dim, gen, sampling, seed, stream=0, *, lo=None, span=None, device=None):
    """[n, dim] points ``lo + span * u`` (u from ``unit_samples``; the product and the sum
    rounded separately; lo / span None drop them) on `device`.

    On a CUDA device the Sobol and Philox families are drawn there by
    ``flashns_b200_sobol_points`` / ``flashns_b200_philox_points``, bit-identical to the
    host; uniform points come from torch's CPU generator and are copied."""
    device = torch.device(device or "cpu")
    lo_t = None if lo is None else torch.tensor(lo, dtype=torch.float64)
    span_t = None if span is None else torch.tensor(span, dtype=torch.float64)
    for t in (lo_t, span_t):
        if t is not None and t.shape != (dim,):
            raise ValueError("lo and span need one value per coordinate")
    if device.type == "cuda" and sampling in ("sobol", "philox"):
        return _device_points(n, dim, sampling, seed, stream, lo_t, span_t, device)
    u = unit_samples(n, dim, gen, sampling, seed, stream)
    if span_t is not None:
        u = span_t * u
    if lo_t is not None:
        u = lo_t + u
    return u.to(device)


def _device_points(n, dim, sampling, seed, stream, lo, span, device):
    import ctypes

    from flashns_b200 import _lib
    out = torch.empty(n, dim, dtype=torch.float64, device=device)
    if n == 0:
        return out
    dbl = lambda t: None if t is None else (ctypes.c_double * dim)(*t.tolist())
    lib = _lib.library()
    with torch.cuda.device(device):
        s = ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)
        if sampling == "sobol":
            engine = sobol_engine(dim, seed, stream)
            dirs = engine.sobolstate.contiguous()
            shift = engine.shift.contiguous()
            status = lib.flashns_b200_sobol_points(ctypes.c_void_p(dirs.data_ptr()), ctypes.c_void_p(shift.data_ptr()),
                                                   dim, 0, n, dbl(lo), dbl(span), ctypes.c_void_p(out.data_ptr()), dim,
                                                   s)
        else:
            k0, k1 = philox_key(seed, stream)
            status = lib.flashns_b200_philox_points(k0, k1, dim, 0, n, dbl(lo), dbl(span),
                                                    ctypes.c_void_p(out.data_ptr()), dim, s)
    _lib.check(status, f"flashns_b200_{sampling}_points")
    return out


def kovasznay(interior, boundary, *, re=20.0, seed=1, boundary_order=1, sampling="uniform", device=None):
    """Kovasznay point set on `device` (default: the host).  With ``sobol`` or ``philox``
    sampling on a CUDA device the points are drawn there (``sample_points``)."""
    gen = torch.Generator(device="cpu").manual_seed(seed)
    device = torch.device(device or "cpu")
    f64 = dict(dtype=torch.float64, device=device)
    xi = sample_points(interior, 2, gen, sampling, seed, lo=[-0.5, -0.5], span=[1.5, 2.0], device=device)
    counts = [boundary // 4 + (1 if k < boundary % 4 else 0) for k in range(4)]
    edges = []
    for k, n in enumerate(counts):
        lo, span = (-0.5, 1.5) if k < 2 else (-0.5, 2.0)
        s = sample_points(n, 1, gen, sampling, seed, stream=k + 1, lo=[lo], span=[span], device=device)
        fixed = torch.full_like(s, (-0.5, 1.5, -0.5, 1.0)[k])
        edges.append(torch.cat((s, fixed) if k < 2 else (fixed, s), 1))
    xb = torch.cat(edges)
    u, v, p, psi = kovasznay_exact(xb, re)
    outflow = torch.zeros(boundary, dtype=torch.bool, device=device)
    outflow[boundary - counts[3]:] = True
    wv = 1.0 / max(boundary, 1)
    wp = torch.zeros(boundary, **f64).masked_fill_(outflow, 1.0 / max(counts[3], 1))
    if boundary_order == 1:
        target = torch.stack((u, v, p), 1)
        weights = torch.stack((torch.full_like(u, wv), torch.full_like(u, wv), wp), 1)
    else:
        target = torch.stack((psi, p), 1)
        weights = torch.stack((torch.full_like(u, wv), wp), 1)
    pde = torch.full((interior,), 1.0 / max(interior, 1), **f64)
    return PointSet(torch.cat((xi, xb)), interior, pde, weights, target, 2, 1.0 / re,
                    f"kovasznay Re={re:g} {interior}+{boundary}")


def taylor_green_exact(x, nu=0.01):
    f = torch.exp(-2 * nu * x[:, 2])
    u = -torch.cos(x[:, 0]) * torch.sin(x[:, 1]) * f
    v = torch.sin(x[:, 0]) * torch.cos(x[:, 1]) * f
    p = -0.25 * (torch.cos(2 * x[:, 0]) + torch.cos(2 * x[:, 1])) * f * f
    psi = torch.cos(x[:, 0]) * torch.cos(x[:, 1]) * f
    return u, v, p, psi


def taylor_green(interior, boundary, *, nu=0.01, seed=1, boundary_order=1, sampling="uniform", device=None):
    """Taylor-Green point set on `device` (default: the host), drawn there with ``sobol``
    or ``philox`` sampling on a CUDA device."""
    gen = torch.Generator(device="cpu").manual_seed(seed)
    device = torch.device(device or "cpu")
    two_pi = 2 * math.pi
    xi = sample_points(interior, 3, gen, sampling, seed, span=[two_pi, two_pi, 1.0], device=device)
    n0 = boundary // 2
    init = sample_points(n0, 3, gen, sampling, seed, stream=1, span=[two_pi, two_pi, 0.0], device=device)
    side = sample_points(boundary - n0, 3, gen, sampling, seed, stream=2, span=[two_pi, two_pi, 1.0], device=device)
    face = torch.arange(boundary - n0, device=device) % 4
    for k, (axis, value) in enumerate(((0, 0.0), (0, two_pi), (1, 0.0), (1, two_pi))):
        side[:, axis] = torch.where(face == k, value, side[:, axis])
    xb = torch.cat((init, side))
    u, v, p, psi = taylor_green_exact(xb, nu)
    w = 1.0 / max(boundary, 1)
    if boundary_order == 1:
        target = torch.stack((u, v, p), 1)
        weights = torch.full((boundary, 3), w, dtype=torch.float64, device=device)
    else:
        target = torch.stack((psi, p), 1)
        weights = torch.full((boundary, 2), w, dtype=torch.float64, device=device)
    pde = torch.full((interior,), 1.0 / max(interior, 1), dtype=torch.float64, device=device)
    return PointSet(torch.cat((xi, xb)), interior, pde, weights, target, 3, nu,
                    f"taylor-green nu={nu:g} {interior}+{boundary}")


def reference_case(batch, *, seed=7510, scale=0.4):
    """The reference's own benchmark problem (uvp head, 2-64-64-3, dense Q10 points, no
    boundary rows, unweighted quadrature): coordinates N(0, scale^2), globally normalized
    weights 1/batch, nu = 0.07 (docs/cuda-h100-results.md "固定科学目标"; the generator
    recipe of experiments/cuda_jet_h100/common.py:44-80, restated)."""
    gen = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(batch, 2, generator=gen, dtype=torch.float64) * scale
    pde = torch.full((batch,), 1.0 / max(batch, 1), dtype=torch.float64)
    empty = torch.zeros(0, 3, dtype=torch.float64)
    return PointSet(x, batch, pde, empty, empty.clone(), 2, 0.07, f"reference case {batch}")


def reference_parameters(widths, seed=7510):
    """Weights N(0, 0.7^2 / fan_in), biases N(0, 0.1^2) (the reference benchmark's init)."""
    gen = torch.Generator(device="cpu").manual_seed(seed + 1)
    ws = [torch.randn(o, i, generator=gen, dtype=torch.float64) * (0.7 / math.sqrt(i))
          for i, o in zip(widths, widths[1:])]
    bs = [torch.randn(o, generator=gen, dtype=torch.float64) * 0.1 for o in widths[1:]]
    return ws, bs


# benchmark configurations: (builder, interior, boundary, widths); ref16k is the reference's
# own headline workload (its published H100 number: 1.832 ms per evaluation)
CONFIGS = {
    "cfg0": dict(kind="kovasznay", interior=2048, boundary=512, widths=[2, 64, 64, 64, 64, 2]),
    "cfg1": dict(kind="kovasznay", interior=16384, boundary=4096, widths=[2, 64, 64, 64, 64, 2]),
    "cfg2": dict(kind="kovasznay", interior=65536, boundary=16384, widths=[2] + [128] * 6 + [2]),
    "cfg3": dict(kind="taylor_green", interior=262144, boundary=65536, widths=[3] + [128] * 5 + [2]),
    "ref16k": dict(kind="reference_case", interior=16384, boundary=0, widths=[2, 64, 64, 3], head="uvp",
                   boundary_order=0, gamma=0.2, init="reference"),
    # not a benchmark configuration: a space-time net 64 wide, the one shape that runs the
    # 3-D 64-wide kernels (fwd_head, bwd_fused); for their profiles
    "tgv64": dict(kind="taylor_green", interior=16384, boundary=4096, widths=[3, 64, 64, 64, 64, 2]),
    # not a benchmark configuration: cfg1's net on 64 times its points (1,048,576 interior,
    # 262,144 boundary), the top of the 16K-1M range the throughput target names
    "cfg1x64": dict(kind="kovasznay", interior=1048576, boundary=262144, widths=[2, 64, 64, 64, 64, 2]),
}


def config_options(name):
    """(head, boundary_order, gradient weight gamma) of a configuration."""
    c = CONFIGS[name]
    return c.get("head", "psi"), c.get("boundary_order", 1), c.get("gamma", 0.2)


def config_parameters(name, seed=0):
    from flashns_b200.evaluator import xavier_normal
    c = CONFIGS[name]
    return reference_parameters(c["widths"]) if c.get("init") == "reference" else xavier_normal(c["widths"], seed)


def config_points(name, *, scale=1, seed=1, boundary_order=None, divisor=1):
    """The configuration's point set, `scale` times as many points (weak scaling), or
    1/`divisor` of them (small profiling cases of the same kernels)."""
    c = CONFIGS[name]
    ni, nb = c["interior"] * scale // divisor, c["boundary"] * scale // divisor
    if c["kind"] == "reference_case":
        return reference_case(ni)
    build = kovasznay if c["kind"] == "kovasznay" else taylor_green
    order = c.get("boundary_order", 1) if boundary_order is None else boundary_order
    return build(ni, nb, seed=seed, boundary_order=order)
