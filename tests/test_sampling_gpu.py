"""GPU: the data-preparation kernels against the libraries and restatements they follow,
bit for bit: scrambled Sobol against torch.quasirandom.SobolEngine, Philox4x64-10
against numpy.random.Generator(Philox), packed coordinate rows against the host
PackedLayout.coordinates, and whole point sets drawn on the device against the host.
Strided outputs are written inside sentinel guards that must stay untouched."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import sampling as ref

pytestmark = pytest.mark.gpu

SENTINEL = -3.25e300


def _dbl(values):
    return None if values is None else (ctypes.c_double * len(values))(*values)


def _affine(u, lo, span):
    if span is not None:
        u = np.asarray(span) * u
    if lo is not None:
        u = np.asarray(lo) + u
    return u


def _strided(n, dim, ld, device):
    buf = torch.full((n * ld + 2 * ld,), SENTINEL, dtype=torch.float64, device=device)
    return buf, buf[ld:ld + n * ld].view(n, ld)


def _untouched(buf, view, dim, ld):
    mask = torch.ones_like(buf, dtype=torch.bool)
    mask[ld:ld + view.shape[0] * ld].view(view.shape[0], ld)[:, :dim] = False
    return bool((buf[mask] == SENTINEL).all())


SOBOL = [(1, 5, 0, 1000, None, None, 1), (2, 1009, 0, 4097, [-0.5, -0.5], [1.5, 2.0], 3),
         (3, 77, 1, 3000, None, [6.25, 6.25, 0.0], 3), (3, 12, 1000, 777, [0.1, 0.2, 0.3], None, 5),
         (8, 4, 0, 1, None, None, 8), (2, 3, 65535, 2, None, None, 2)]


@pytest.mark.parametrize("dim,seed,first,n,lo,span,ld", SOBOL)
def test_sobol_points_match_torch_engine(cuda, dim, seed, first, n, lo, span, ld):
    from flashns_b200 import _lib
    engine = torch.quasirandom.SobolEngine(dim, scramble=True, seed=seed)
    dirs, shift = engine.sobolstate.contiguous(), engine.shift.contiguous()
    if first:
        engine.fast_forward(first)
    expected = _affine(engine.draw(n, dtype=torch.float64).numpy(), lo, span)
    buf, view = _strided(n, dim, ld, cuda)
    status = _lib.library().flashns_b200_sobol_points(
        ctypes.c_void_p(dirs.data_ptr()), ctypes.c_void_p(shift.data_ptr()), dim, first, n, _dbl(lo), _dbl(span),
        ctypes.c_void_p(view.data_ptr()), ld, ctypes.c_void_p(torch.cuda.current_stream(cuda).cuda_stream))
    assert status == 0
    torch.cuda.synchronize()
    np.testing.assert_array_equal(view[:, :dim].cpu().numpy(), expected)
    np.testing.assert_array_equal(view[:, :dim].cpu().numpy(),
                                  _affine(ref.sobol_points(dirs.numpy(), shift.numpy(), first, n), lo, span))
    assert _untouched(buf, view, dim, ld)


PHILOX = [(0, 0, 1, 0, 1001), (12345, 7, 2, 0, 333), (99, 1, 3, 5, 400), ((1 << 64) - 1, 3, 3, 1, 17),
          (5, 0, 8, 3, 9)]


@pytest.mark.parametrize("key0,key1,dim,first,n", PHILOX)
def test_philox_points_match_numpy_generator(cuda, key0, key1, dim, first, n):
    from flashns_b200 import _lib
    gen = np.random.Generator(np.random.Philox(key=key0 + (key1 << 64)))
    if first:
        gen.random((first, dim))
    lo, span = [-1.0] * dim, [2.0] * dim
    expected = _affine(gen.random((n, dim)), lo, span)
    ld = dim + 1
    buf, view = _strided(n, dim, ld, cuda)
    status = _lib.library().flashns_b200_philox_points(
        key0, key1, dim, first, n, _dbl(lo), _dbl(span), ctypes.c_void_p(view.data_ptr()), ld,
        ctypes.c_void_p(torch.cuda.current_stream(cuda).cuda_stream))
    assert status == 0
    torch.cuda.synchronize()
    np.testing.assert_array_equal(view[:, :dim].cpu().numpy(), expected)
    assert _untouched(buf, view, dim, ld)


@pytest.mark.parametrize("dim,nf,nv", [(2, 333, 97), (3, 91, 37), (2, 0, 5), (3, 7, 0), (2, 0, 0)])
def test_pack_coordinates_match_host_layout(cuda, dim, nf, nv):
    from flashns_b200.jet_packed import PackedLayout
    x = torch.rand(nf + nv, dim, dtype=torch.float64, generator=torch.Generator().manual_seed(nf + nv))
    x[::7] = -x[::7]
    layout = PackedLayout(nf, nv, dim)
    got = layout.coordinates(x.to(cuda))
    torch.cuda.synchronize()
    assert torch.equal(got.cpu(), layout.coordinates(x))
    np.testing.assert_array_equal(got.cpu().numpy(), ref.packed_coordinates(x.numpy(), nf, dim))


@pytest.mark.parametrize("sampling", ["sobol", "philox"])
@pytest.mark.parametrize("order", [0, 1])
def test_point_sets_drawn_on_device_match_host(cuda, sampling, order):
    from flashns_b200.problems import kovasznay, taylor_green
    for build, ni, nb in ((kovasznay, 1001, 403), (taylor_green, 517, 130)):
        host = build(ni, nb, seed=3, boundary_order=order, sampling=sampling)
        dev = build(ni, nb, seed=3, boundary_order=order, sampling=sampling, device=cuda)
        assert dev.x.is_cuda and dev.target.is_cuda
        assert torch.equal(dev.x.cpu(), host.x)
        assert torch.equal(dev.pde_weights.cpu(), host.pde_weights)
        assert torch.equal(dev.boundary_weights.cpu(), host.boundary_weights)
        # analytic targets through the device's exp / sin / cos: last-bit differences only
        np.testing.assert_allclose(dev.target.cpu().numpy(), host.target.numpy(), rtol=1e-14, atol=1e-15)


def test_device_point_set_evaluates_like_host(cuda):
    from flashns_b200.evaluator import PackedEvaluator, flat_parameters, xavier_normal
    from flashns_b200.ns_seed import NSLoss
    from flashns_b200.problems import kovasznay
    widths = [2, 64, 64, 64, 2]
    ws, bs = xavier_normal(widths, 0)
    p = flat_parameters(ws, bs).to(cuda)
    out = []
    for device in (None, cuda):
        pts = kovasznay(700, 180, seed=5, sampling="sobol", device=device)
        ev = PackedEvaluator(pts.x, pts.interior_count, pts.pde_weights, pts.boundary_weights, pts.target, widths,
                             head="psi", boundary_order=1, loss=NSLoss(pts.viscosity, 0.0, 5.0), device=cuda)
        out.append(ev(p).cpu())
    np.testing.assert_allclose(out[1].numpy(), out[0].numpy(), rtol=1e-12, atol=1e-14)
