"""GPU: PackedPINN fixes its point set at construction, as the reference's does
(the reference's tests/test_coordinate_affine.py:37-70 moves x in place after
construction and expects unchanged results over several parameter updates)."""

import numpy as np
import pytest
import torch

from tests.cases import close_ratio, random_case

pytestmark = pytest.mark.gpu


def test_point_set_fixed_at_construction(cuda):
    from flashns_b200.pinn_packed import PackedPINN
    c = random_case(7, 3, [2, 7, 5, 3], seed=6422)
    t = lambda a: torch.tensor(np.asarray(a), dtype=torch.float64, device=cuda)
    x = t(c["x"])
    step = PackedPINN(x, 7, t(c["pw"]), t(c["bw"]), t(c["target"]))
    fresh = PackedPINN(t(c["x"]), 7, t(c["pw"]), t(c["bw"]), t(c["target"]))
    x.add_(100.0)  # the caller moves its points after construction
    ws, bs = [t(w) for w in c["ws"]], [t(b) for b in c["bs"]]
    for _ in range(3):
        loss_a, grads_a = step(ws, bs)
        loss_b, grads_b = fresh(ws, bs)
        assert close_ratio(float(loss_a), float(loss_b)) <= 1
        for a, b in zip(grads_a, grads_b):
            assert close_ratio(a.cpu(), b.cpu()) <= 1
        with torch.no_grad():
            for p, g in zip(ws + bs, grads_a):
                p.add_(g, alpha=-1e-3)


def test_caller_defined_hooks_are_refused(cuda):
    """A stage hook that is not this library's own cannot be called by the fused drop-in;
    construction refuses it instead of dropping it silently.  Its own hooks are accepted
    (the fused kernels contain their stages) and recorded as not called."""
    from flashns_b200.native import NativeCUDA
    from flashns_b200.pinn_packed import PackedPINN
    c = random_case(5, 2, [2, 6, 3], seed=3)
    t = lambda a: torch.tensor(np.asarray(a), dtype=torch.float64, device=cuda)
    args = (t(c["x"]), 5, t(c["pw"]), t(c["bw"]), t(c["target"]))
    with pytest.raises(NotImplementedError, match="coordinate_affine"):
        PackedPINN(*args, coordinate_affine=lambda *a: None)
    with pytest.raises(NotImplementedError, match="residual_reference"):
        PackedPINN(*args, seed="autograd", residual_reference=lambda *a: None)
    nat = NativeCUDA()
    quiet = PackedPINN(*args, seed="cuda", activation_factory=nat.activation_factory, cuda_seed=nat.seed,
                       tail_dgrad_vjp=nat.tail_dgrad_vjp)
    assert quiet.metadata["hooks_not_called"] == ["activation_factory", "cuda_seed", "tail_dgrad_vjp"]
    loss, grads = quiet([t(w) for w in c["ws"]], [t(b) for b in c["bs"]])
    assert torch.isfinite(loss) and len(grads) == 4
