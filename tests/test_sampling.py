"""CPU: the restatements of the device samplers are pinned to the libraries they follow
(torch.quasirandom.SobolEngine, numpy.random.Philox), the host point sets keep their
sampling contract, and the sampling entry points reject bad arguments before any CUDA
call."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import sampling as ref


@pytest.mark.parametrize("dim,seed", [(1, 5), (2, 1009), (3, 77), (8, 4)])
def test_sobol_restatement_matches_torch_engine(dim, seed):
    engine = torch.quasirandom.SobolEngine(dim, scramble=True, seed=seed)
    dirs, shift = engine.sobolstate.numpy(), engine.shift.numpy()
    first = engine.draw(1000, dtype=torch.float64).numpy()
    more = engine.draw(37, dtype=torch.float64).numpy()
    np.testing.assert_array_equal(ref.sobol_points(dirs, shift, 0, 1000), first)
    np.testing.assert_array_equal(ref.sobol_points(dirs, shift, 1000, 37), more)


def test_philox_restatement_matches_numpy():
    for key in (0, 12345, 3 + (7 << 64), (1 << 64) - 1):
        k0, k1 = key & ref.MASK64, key >> 64
        raw = [int(w) for w in np.random.Philox(key=key).random_raw(13)]
        assert ref.philox_words(k0, k1, 0, 13) == raw
        gen = np.random.Generator(np.random.Philox(key=key))
        head = gen.random((5, 3))
        tail = gen.random((4, 3))
        np.testing.assert_array_equal(ref.philox_uniform(k0, k1, 3, 0, 5), head)
        np.testing.assert_array_equal(ref.philox_uniform(k0, k1, 3, 5, 4), tail)


def test_packed_coordinates_restatement_matches_layout():
    from flashns_b200.jet_packed import PackedLayout
    for dim, nf, nv in ((2, 5, 3), (3, 4, 0), (2, 0, 6)):
        x = torch.rand(nf + nv, dim, dtype=torch.float64, generator=torch.Generator().manual_seed(dim + nf))
        got = PackedLayout(nf, nv, dim).coordinates(x).numpy()
        np.testing.assert_array_equal(ref.packed_coordinates(x.numpy(), nf, dim), got)


def test_host_philox_points_follow_numpy_stream():
    from flashns_b200.problems import kovasznay, sample_points
    got = sample_points(50, 2, None, "philox", 9, stream=3, lo=[-0.5, -0.5], span=[1.5, 2.0])
    u = np.random.Generator(np.random.Philox(key=9 + (3 << 64))).random((50, 2))
    np.testing.assert_array_equal(got.numpy(), np.array([-0.5, -0.5]) + np.array([1.5, 2.0]) * u)
    a, b = kovasznay(64, 20, seed=9, sampling="philox"), kovasznay(64, 20, seed=9, sampling="philox")
    assert torch.equal(a.x, b.x)
    assert not torch.equal(a.x, kovasznay(64, 20, seed=10, sampling="philox").x)
    with pytest.raises(ValueError):
        kovasznay(8, 4, sampling="mersenne")


def test_sampling_entry_points_reject_bad_arguments():
    from flashns_b200 import _lib
    lib = _lib.library()
    invalid = 1  # cudaErrorInvalidValue
    dirs = (ctypes.c_int64 * 90)(*([1] * 90))
    shift = (ctypes.c_int64 * 3)(0, 1, 2)
    out = ctypes.c_void_p(16)  # never written: every call below returns before a launch
    sobol = lambda dim, first, n, ld, d=dirs, s=shift: lib.flashns_b200_sobol_points(d, s, dim, first, n, None, None,
                                                                                     out, ld, None)
    assert sobol(0, 0, 4, 1) == invalid
    assert sobol(9, 0, 4, 9) == invalid
    assert sobol(2, 0, 4, 1) == invalid                 # ld < dim
    assert sobol(2, -1, 4, 2) == invalid
    assert sobol(2, (1 << 30) - 3, 4, 2) == invalid     # past the engine's 2^30 points
    assert sobol(2, 0, 4, 2, d=None) == invalid
    bad = (ctypes.c_int64 * 90)(*([1 << 30] * 90))
    assert sobol(2, 0, 4, 2, d=bad) == invalid          # direction numbers wider than 30 bits
    assert sobol(2, 5, 0, 2) == 0                       # nothing to draw
    philox = lambda dim, first, n, ld: lib.flashns_b200_philox_points(1, 2, dim, first, n, None, None, out, ld, None)
    assert philox(0, 0, 4, 1) == invalid
    assert philox(3, 0, -1, 3) == invalid
    assert philox(3, 1 << 60, 4, 3) == invalid
    assert philox(3, 0, 0, 3) == 0
    assert lib.flashns_b200_pack_coordinates(None, 0, 0, 2, None, None) == 0
    assert lib.flashns_b200_pack_coordinates(None, 3, 0, 2, None, None) == invalid
    assert lib.flashns_b200_pack_coordinates(None, -1, 0, 2, None, None) == invalid
