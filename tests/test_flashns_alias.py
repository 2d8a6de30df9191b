"""CPU: the reference's import paths (``flashns.*``) resolve to this library's modules and
carry every name of the evaluation path's Python API."""

import importlib

import pytest

API = {
    "jet_spec": ["JetSpec"],
    "jet_stable": ["stable_a1", "stable_tanh", "tanh_jet", "tanh_vjp", "multiply", "product_pairs", "manifest"],
    "jet_packed": ["PackedLayout", "TensorActivation", "stable_a1", "full_vjp", "convolution_terms"],
    "ns_seed": ["NSLoss", "residual_terms", "residuals", "per_point_loss", "explicit_seed", "compile_seed",
                "validate_weights"],
    "pinn_packed": ["PackedPINN"],
    "distributed_contract": ["shard_bounds", "global_normalization", "parameter_count"],
}


@pytest.mark.parametrize("module", sorted(API))
def test_reference_import_paths_resolve_to_this_library(module):
    ref_name = importlib.import_module(f"flashns.{module}")
    assert ref_name is importlib.import_module(f"flashns_b200.{module}")
    for name in API[module]:
        assert callable(getattr(ref_name, name)), (module, name)


def test_from_imports_and_package_attributes():
    import flashns
    import flashns_b200.pinn_packed
    from flashns.distributed_contract import shard_bounds
    from flashns.jet_spec import JetSpec
    from flashns.pinn_packed import PackedPINN
    assert PackedPINN is flashns_b200.pinn_packed.PackedPINN
    assert flashns.ns_seed.NSLoss().viscosity == 0.07
    assert JetSpec(2).coefficient_order[:3] == ((0, 0), (0, 1), (1, 0))
    assert [shard_bounds(10, 3, r) for r in range(3)] == [(0, 3), (3, 6), (6, 10)]
    assert set(flashns.MODULES) == set(API)
