"""CPU: host-side contracts mirrored from the reference tests
(tests/test_jet_spec.py, tests/test_distributed_contract.py, tests/test_pinn_v8.py:128-134)."""

import math

import numpy as np
import pytest
import torch

from flashns_b200.distributed_contract import global_normalization, parameter_count, shard_bounds
from flashns_b200.jet_spec import JetSpec


@pytest.mark.parametrize("dim,q", [(2, 10), (3, 20)])
def test_full_jet_recovery_and_cotangent_duality(dim, q):
    spec = JetSpec(dim)
    assert spec.q == q and spec.coefficient_order[0] == (0,) * dim
    coefficients = np.zeros(q)
    cube = (3,) + (0,) * (dim - 1)
    mixed = (1, 2) + (0,) * (dim - 2)
    coefficients[spec.coefficient_order.index(cube)] = 1
    coefficients[spec.coefficient_order.index(mixed)] = 2
    derivatives = spec.recover_raw_derivatives(coefficients)
    assert derivatives[spec.coefficient_order.index(cube)] == 6
    assert derivatives[spec.coefficient_order.index(mixed)] == 4
    raw_seed = np.arange(q) / 7
    assert np.dot(raw_seed, derivatives) == pytest.approx(np.dot(spec.pullback_raw_derivative_seed(raw_seed), coefficients))
    assert spec.truncated_q(1) == dim + 1 and spec.truncated_q(0) == 1


@pytest.mark.parametrize("operation", ["hvp", "double_backward", "c13", "nonlocal_loss"])
def test_unsupported_transforms_are_explicit(operation):
    with pytest.raises(NotImplementedError, match=operation):
        JetSpec(3).require_operation(operation)


def test_basis_matches_device_unit_rows():
    from flashns_b200 import codegen
    for dim in (2, 3):
        basis = JetSpec(dim).coefficient_order
        assert basis == codegen.basis(dim)
        for axis in range(dim):
            unit = tuple(int(j == axis) for j in range(dim))
            assert basis.index(unit) == dim - axis  # unit_row<DIM>(axis) in csrc/common.cuh


@pytest.mark.parametrize("points,world", [(17, 1), (17, 2), (17, 4), (3, 4), (0, 4)])
def test_shards_cover_global_ids_once_including_empty_ranks(points, world):
    shards = [list(range(*shard_bounds(points, world, rank))) for rank in range(world)]
    assert [i for shard in shards for i in shard] == list(range(points))
    assert max(map(len, shards)) - min(map(len, shards)) <= 1


@pytest.mark.parametrize("points,world", [(17, 4), (3, 4)])
def test_weighted_local_sums_have_one_global_denominator(points, world):
    weights = [0.5 + (i % 7) / 8 for i in range(points)]
    derivative = [math.cos(i / 3) for i in range(points)]
    z = global_normalization(weights)
    expected = math.fsum(w * d for w, d in zip(weights, derivative)) / z
    partials = [math.fsum(weights[i] * derivative[i] for i in range(*shard_bounds(points, world, r))) / z
                for r in range(world)]
    assert math.fsum(partials) == pytest.approx(expected, abs=1e-15)


def test_model_gradient_payload_comes_from_parameters():
    assert parameter_count([2, 64, 64, 3]) == 4547
    assert parameter_count([2, 64, 64, 64, 64, 2]) == 12802
    assert parameter_count([2] + [128] * 6 + [2]) == 83202
    assert parameter_count([3] + [128] * 5 + [2]) == 66818


@pytest.mark.parametrize("weights", [[0, 0], [1, -1], [float("nan")], [float("inf")]])
def test_invalid_global_weights_rejected(weights):
    with pytest.raises(ValueError):
        global_normalization(weights)


def test_problem_generators_and_shards():
    from flashns_b200.problems import config_points, kovasznay, taylor_green
    k = kovasznay(100, 40)
    assert k.x.shape == (140, 2) and k.target.shape == (40, 3)
    assert abs(float(k.pde_weights.sum()) - 1) < 1e-14
    assert abs(float(k.boundary_weights[:, 0].sum()) - 1) < 1e-14
    assert abs(float(k.boundary_weights[:, 2].sum()) - 1) < 1e-14
    assert bool((k.x[:100, 0] >= -0.5).all() and (k.x[:100, 0] <= 1.0).all())
    t = taylor_green(64, 32)
    assert t.x.shape == (96, 3) and bool((t.x[64:64 + 16, 2] == 0).all())
    g = config_points("cfg1", scale=4)
    parts = [g.shard(4, r) for r in range(4)]
    assert sum(p.interior_count for p in parts) == g.interior_count
    assert sum(len(p.x) for p in parts) == len(g.x)
    assert abs(sum(float(p.pde_weights.sum()) for p in parts) - 1) < 1e-12


def test_residual_terms_match_reference_table():
    """ns_seed.residual_terms (derived from the PDE) equals the reference table
    (src/flashns/ns_seed.py:26-43, recorded in tests/golden) as polynomials."""
    from tests.cases import GOLDEN
    from flashns_b200.ns_seed import residual_terms
    g = np.load(GOLDEN / "reference_seed.npz")

    def norm(terms):
        d = {}
        for c, i, j in terms:
            i, j = int(i), int(j)
            k = (min(i, j), max(i, j)) if j >= 0 else (i, -1)
            d[k] = d.get(k, 0.0) + c
        return {k: round(v, 12) for k, v in d.items()}

    for m in range(4):
        nu = float(g[f"terms{m}_nu"])
        rows = g[f"terms{m}"]
        ref = [[(c, i, j) for r2, c, i, j in rows if int(r2) == r] for r in range(9)]
        mine = residual_terms(nu)
        assert len(mine) == 9
        for a, b in zip(mine, ref):
            assert norm(a) == norm(b)


def test_sobol_sampling_is_seeded_and_in_domain():
    """Scrambled-Sobol point sets (the reference's data kind): deterministic per seed,
    inside the domain, boundary points on the edges / faces, weights normalized."""
    import torch
    from flashns_b200.problems import kovasznay, taylor_green
    a = kovasznay(512, 128, seed=3, sampling="sobol")
    b = kovasznay(512, 128, seed=3, sampling="sobol")
    c = kovasznay(512, 128, seed=4, sampling="sobol")
    assert torch.equal(a.x, b.x) and not torch.equal(a.x, c.x)
    xi = a.x[:512]
    assert float(xi[:, 0].min()) >= -0.5 and float(xi[:, 0].max()) < 1.0
    assert float(xi[:, 1].min()) >= -0.5 and float(xi[:, 1].max()) < 1.5
    xb = a.x[512:]
    on_edge = (xb[:, 0] == -0.5) | (xb[:, 0] == 1.0) | (xb[:, 1] == -0.5) | (xb[:, 1] == 1.5)
    assert bool(on_edge.all())
    assert abs(float(a.pde_weights.sum()) - 1.0) < 1e-12
    t = taylor_green(256, 64, seed=2, sampling="sobol")
    assert t.x.shape == (320, 3) and float(t.x[256:288, 2].abs().max()) == 0.0  # initial slab t = 0


def test_solver_checkpoint_round_trip(tmp_path):
    """OUTPUT.pt holds the final flat parameters and the run description; its sha256 is
    what the solver reports."""
    import hashlib
    import torch
    from flashns_b200.solver import load_checkpoint, save_checkpoint
    flat = torch.linspace(-1.0, 1.0, 12802, dtype=torch.float64)
    meta = {"problem": {"name": "kovasznay", "re": 20.0}, "protocol": {"adam_steps": 3000}, "seed": 1}
    digest = save_checkpoint(tmp_path / "run.pt", flat, meta)
    assert digest == hashlib.sha256((tmp_path / "run.pt").read_bytes()).hexdigest()
    back = load_checkpoint(tmp_path / "run.pt")
    assert torch.equal(back["flat_parameters"], flat) and back["problem"]["re"] == 20.0 and back["seed"] == 1


def test_jet_multiply_and_manifest():
    """jet_stable.multiply is the truncated Cauchy product of the oracle
    (src/flashns/jet_stable.py:52-59); the activation manifest keeps the reference's keys."""
    import numpy as np
    import torch

    from flashns_b200 import jet_packed, jet_stable
    from oracle import jets as J
    for dim in (2, 3):
        gen = torch.Generator().manual_seed(dim)
        a = torch.randn(7, J.q(dim), 3, dtype=torch.float64, generator=gen)
        b = torch.randn(7, J.q(dim), 3, dtype=torch.float64, generator=gen)
        np.testing.assert_allclose(jet_stable.multiply(a, b, dim).numpy(), J.cauchy(a.numpy(), b.numpy(), dim, 3),
                                   rtol=1e-15, atol=1e-15)
    m = jet_stable.manifest(2, "a" * 64)
    assert m["activation_aux_state"]["strategy"] == "stable_aux_a1" and m["q"] == 10
    assert jet_packed.stable_a1 is jet_stable.stable_a1


def test_foreign_stage_hooks_are_named():
    """PackedPINN calls no stage hook (its fused kernels contain the stages); this
    library's own hooks are recognized, any other callable is reported so the drop-in
    can refuse it instead of dropping a caller-defined stage silently."""
    from flashns_b200.jet_packed import TensorActivation
    from flashns_b200.native import Native, NativeCUDA
    from flashns_b200.ns_seed import per_point_loss
    from flashns_b200.pinn_packed import HOOKS, foreign_hooks
    from flashns_b200 import _lib
    if not _lib.LIBRARY.exists():
        pytest.skip("library not built")
    nat, dense = NativeCUDA(), Native()
    own = dict(activation_factory=nat.activation_factory, cuda_seed=nat.seed, residual_reference=per_point_loss,
               tail_dgrad_vjp=nat.tail_dgrad_vjp, coordinate_affine=nat.coordinate_affine,
               first_affine_activation=nat.coordinate_affine_activation, coordinate_wgrad=nat.coordinate_wgrad,
               first_activation_wgrad=nat.coordinate_activation_wgrad)
    assert set(own) == set(HOOKS)
    assert foreign_hooks(**own) == []
    assert foreign_hooks(activation_factory=TensorActivation, coordinate_wgrad=None) == []
    assert foreign_hooks(activation_factory=dense.forward) == []
    mine = lambda *a, **k: None
    assert foreign_hooks(activation_factory=TensorActivation, coordinate_affine=mine, cuda_seed=mine) == [
        "coordinate_affine", "cuda_seed"]


def test_packed_pinn_refuses_a_foreign_residual_before_any_device_work():
    """A caller-defined residual (seed="autograd") or CUDA seed (seed="cuda") is what the
    reference would call (src/flashns/pinn_packed.py:136-146); the drop-in raises
    NotImplementedError at construction, on any device, rather than ignore it."""
    from flashns_b200.pinn_packed import PackedPINN
    x = torch.zeros(3, 2, dtype=torch.float64)
    args = (x, 2, torch.full((2,), 0.5, dtype=torch.float64), torch.ones(1, 3, dtype=torch.float64),
            torch.zeros(1, 3, dtype=torch.float64))
    mine = lambda *a, **k: None
    with pytest.raises(NotImplementedError, match="residual_reference"):
        PackedPINN(*args, seed="autograd", residual_reference=mine)
    with pytest.raises(NotImplementedError, match="cuda_seed"):
        PackedPINN(*args, seed="cuda", cuda_seed=mine)
    with pytest.raises(NotImplementedError, match="activation_factory"):
        PackedPINN(*args, activation_factory=mine)
    with pytest.raises(ValueError, match="CUDA tensors"):  # no foreign hook: the CPU tensors are refused
        PackedPINN(*args, seed="autograd", residual_reference=None)


def test_compulsory_bytes_per_kernel_match_the_cfg1_profile():
    """The per-launch DRAM model reproduces the compulsory figures of the cfg1 kernels
    (backward 281 MB, forward 191 MB, fused head 180 MB of seeds and checkpoints) and
    lines up launch for launch with the FLOP model for every width pattern."""
    from flashns_b200.costs import evaluation_bytes, evaluation_costs, kernel_rooflines
    b = evaluation_bytes([2, 64, 64, 64, 64, 2], 16384, 4096, head="psi", boundary_order=1)
    mb = lambda v: round(v / 1e6)
    assert [mb(v) for v in b["backward"][:2]] == [281, 281] and [mb(v) for v in b["forward"]] == [191, 191]
    assert mb(b["forward_head"][0]) == 181 and mb(b["first"][0]) == 101
    for widths, head, order in (([2, 128, 128, 128, 2], "psi", 1), ([3] + [128] * 5 + [2], "psi", 1),
                                ([2, 64, 64, 3], "uvp", 0), ([2, 20, 3], "uvp", 0), ([2, 30, 64, 64, 2], "psi", 0)):
        c = evaluation_costs(widths, 100, 10, head=head, boundary_order=order)["per_kind"]
        d = evaluation_bytes(widths, 100, 10, head=head, boundary_order=order)
        assert {k: len(v) for k, v in c.items() if v} == {k: len(v) for k, v in d.items() if v}, widths
    flops = evaluation_costs([2, 64, 64, 64, 64, 2], 16384, 4096, head="psi", boundary_order=1)["per_kind"]
    times = {"backward": {"avg_ms": 0.1158, "launches_per_eval": 3}, "reduce": {"avg_ms": 0.0101}}
    r = kernel_rooflines(times, flops, b, 37.1, 6552.6)
    assert 25 < r["backward"]["tflops"] < 27 and abs(r["backward"]["fp64_frac"] - r["backward"]["tflops"] / 37.1) < 1e-12
    assert 2000 < r["backward"]["gbs"] < 2500 and r["reduce"] == {"avg_ms": 0.0101}


def test_bench_configurations_are_the_configuration_table():
    """bench.py --config offers exactly the configurations of flashns_b200.problems, and the
    two profile-only ones have the sizes their profiles state."""
    import re
    from pathlib import Path

    from flashns_b200.problems import CONFIGS, config_points
    src = (Path(__file__).resolve().parent.parent / "bench.py").read_text()
    m = re.search(r'"--config", default="cfg1",\s*choices=\[([^\]]*)\]', src)
    assert m, "bench.py --config choices not found"
    assert set(re.findall(r'"([a-z0-9]+)"', m.group(1))) == set(CONFIGS)
    assert CONFIGS["tgv64"]["widths"] == [3, 64, 64, 64, 64, 2]
    big = config_points("cfg1x64")
    assert big.interior_count == 1 << 20 and len(big.x) == (1 << 20) + (1 << 18)
    assert CONFIGS["cfg1x64"]["widths"] == CONFIGS["cfg1"]["widths"]
