"""GPU: the reference-ABI hooks and the PackedPINN drop-in against the reference golden
vectors and the oracle.  ``staged_step`` composes the hooks the way the reference's
PackedPINN does (src/flashns/pinn_packed.py:108-190): torch GEMMs between hook calls."""

import numpy as np
import pytest
import torch

from tests.cases import GOLDEN, close_ratio, golden_pinn_cases, random_case

pytestmark = pytest.mark.gpu


def T(a, dev):
    return torch.tensor(np.asarray(a), dtype=torch.float64, device=dev)


def test_packed_activation_matches_reference(cuda):
    from flashns_b200.jet_packed import PackedLayout, TensorActivation
    a = np.load(GOLDEN / "reference_activation.npz")
    for k in range(int(a["act_count"])):
        p = f"act{k}_"
        dim, full, value = (int(v) for v in a[p + "meta"])
        ops = TensorActivation(PackedLayout(full, value, dim))
        h, aux = ops.forward(T(a[p + "z"], cuda))
        dz = ops.vjp(h, aux, T(a[p + "seed"], cuda))
        assert close_ratio(h.cpu(), a[p + "h"]) <= 1
        assert close_ratio(aux.cpu(), a[p + "a1"]) <= 1
        assert close_ratio(dz.cpu(), a[p + "dz"]) <= 1


def test_dense_activation_and_dgrad_match_oracle(cuda):
    from flashns_b200.native import Native
    from oracle import jets as J
    rng = np.random.default_rng(5)
    nat = Native()
    for dim in (2, 3):
        q = J.q(dim)
        z = rng.normal(size=(9, q, 13)) * 0.4
        z[1, 0] += 20.0
        h, a1 = J.tanh_jet(z, dim)
        hb = rng.normal(size=z.shape)
        hg, ag = nat.forward(T(z, cuda), dim)
        assert close_ratio(hg.cpu(), h) <= 1 and close_ratio(ag.cpu(), a1) <= 1
        assert close_ratio(nat.vjp(hg, ag, T(hb, cuda), dim).cpu(), J.tanh_vjp(h, a1, hb, dim)) <= 1
        for cout in (3, 11):
            d = rng.normal(size=(9, q, cout))
            w = rng.normal(size=(cout, 13))
            dh = d @ w
            expect = J.tanh_vjp(h, a1, dh, dim)
            for backend in ("B1", "F", "F3", "U3"):
                got = nat.dgrad(T(d, cuda), T(w, cuda), hg, ag, dim, backend)
                assert close_ratio(got.cpu(), expect) <= 1, (dim, cout, backend)


def test_seed_and_residuals_match_reference(cuda):
    from flashns_b200.ns_seed import NSLoss, explicit_seed, per_point_loss, residuals
    s = np.load(GOLDEN / "reference_seed.npz")
    for k in range(int(s["seed_count"])):
        p = f"seed{k}_"
        nu, gamma = (float(v) for v in s[p + "nu_gamma"])
        loss = NSLoss(viscosity=nu, gradient_weight=gamma)
        jets, w = T(s[p + "jets"], cuda), T(s[p + "w"], cuda)
        value, seed = explicit_seed(jets, w, loss)
        assert close_ratio(float(value), float(s[p + "loss"])) <= 1
        assert close_ratio(seed.cpu(), s[p + "seed"]) <= 1
        assert close_ratio(residuals(jets, loss).cpu(), s[p + "res"]) <= 1
        assert close_ratio(float((w * per_point_loss(jets, loss)).sum()), float(s[p + "loss"])) <= 1


def staged_step(x, ni, pw, bw, target, ws, bs, loss, native):
    """The reference's hook-driven compact evaluation (pinn_packed.py:108-190) on these hooks."""
    from flashns_b200.jet_packed import PackedLayout
    layout = PackedLayout(ni, len(x) - ni, 2)
    zero = layout.zero_rows(x.device)
    act = native.activation_factory(layout)
    h, a1 = native.coordinate_affine_activation(layout, x, ws[0], bs[0])
    saved, aux = [layout.coordinates(x), h], [a1]
    for layer in range(1, len(ws)):
        z = h @ ws[layer].T
        z[zero] += bs[layer]
        if layer + 1 < len(ws):
            h, a1 = act.forward(z)
            aux.append(a1)
        else:
            h = z
        saved.append(h)
    interior = saved[-1][:ni * 10].view(ni, 10, 3)
    boundary = saved[-1][zero][ni:]
    total, di, db = native.seed(interior.contiguous(), boundary, pw, bw, target, loss)
    d = torch.zeros_like(saved[-1])
    d[:ni * 10] = di.reshape(ni * 10, 3)
    d[zero[ni:]] += db
    dws, dbs = [None] * len(ws), [None] * len(ws)
    for layer in reversed(range(len(ws))):
        if layer == 0:
            dws[0], dbs[0] = native.coordinate_wgrad(layout, x, d)
            break
        dws[layer] = d.T @ saved[layer]
        dbs[layer] = d[zero].sum(0)
        if layer == 1:
            dh = d @ ws[1]
            dws[0], dbs[0] = native.coordinate_activation_wgrad(layout, x, saved[1], aux[0], dh)
            break
        if layer == len(ws) - 1:
            d = native.tail_dgrad_vjp(layout, d.contiguous(), ws[layer], saved[layer], aux[layer - 1])
        else:
            d = act.vjp(saved[layer], aux[layer - 1], (d @ ws[layer]).contiguous())
    return total, dws + dbs


@pytest.mark.parametrize("k", range(8))
def test_hooks_compose_to_reference_packed_pinn(cuda, k):
    from flashns_b200.native import NativeCUDA
    from flashns_b200.ns_seed import NSLoss
    c = golden_pinn_cases()[k]
    if len(c["widths"]) < 4:
        pytest.skip("the staged path needs two hidden layers")
    loss = NSLoss(c["nu"], c["gamma"], c["bc"])
    total, grads = staged_step(T(c["x"], cuda), c["ni"], T(c["pw"], cuda), T(c["bw"], cuda), T(c["target"], cuda),
                               [T(w, cuda) for w in c["ws"]], [T(b, cuda) for b in c["bs"]], loss, NativeCUDA())
    assert close_ratio(float(total), c["loss"]) <= 1
    for got, exp in zip(grads, c["grads"]):
        assert close_ratio(got.cpu(), exp) <= 1


@pytest.mark.parametrize("layout", ["dense", "split", "compact"])
def test_packed_pinn_dropin_matches_reference(cuda, layout):
    from flashns_b200.ns_seed import NSLoss
    from flashns_b200.pinn_packed import PackedPINN
    for c in golden_pinn_cases():
        loss = NSLoss(c["nu"], c["gamma"], c["bc"])
        step = PackedPINN(T(c["x"], cuda), c["ni"], T(c["pw"], cuda), T(c["bw"], cuda), T(c["target"], cuda),
                          layout=layout, seed="explicit", loss=loss)
        total, grads = step([T(w, cuda) for w in c["ws"]], [T(b, cuda) for b in c["bs"]])
        assert close_ratio(float(total), c["loss"]) <= 1
        assert len(grads) == len(c["grads"])
        for got, exp in zip(grads, c["grads"]):
            assert tuple(got.shape) == exp.shape
            assert close_ratio(got.cpu(), exp) <= 1


def test_packed_pinn_adam_updates_track_reference_oracle(cuda):
    """Three Adam updates through the drop-in stay on the oracle's trajectory
    (the reference pattern of tests/test_pinn_v8.py:88-109)."""
    from flashns_b200.ns_seed import NSLoss
    from flashns_b200.pinn_packed import PackedPINN
    from oracle.evaluate import evaluate
    c = random_case(13, 5, [2, 24, 20, 3], seed=821)
    c["x"][-1] = c["x"][-2]  # repeated boundary point
    step = PackedPINN(T(c["x"], cuda), 13, T(c["pw"], cuda), T(c["bw"], cuda), T(c["target"], cuda))
    ps = [T(p, cuda).requires_grad_() for p in c["ws"] + c["bs"]]
    refs = [torch.tensor(p, requires_grad=True) for p in c["ws"] + c["bs"]]
    opt, ropt = torch.optim.Adam(ps, lr=1e-3), torch.optim.Adam(refs, lr=1e-3)
    for _ in range(3):
        total, grads = step(ps[:3], ps[3:])
        rp = [p.detach().numpy() for p in refs]
        rl, rg = evaluate(c["x"], 13, c["pw"], c["bw"], c["target"], rp[:3], rp[3:], head="uvp")
        assert close_ratio(float(total), rl) <= 1
        for p, g, r, e in zip(ps, grads, refs, rg):
            p.grad = g.clone()
            r.grad = torch.tensor(e)
        opt.step()
        ropt.step()
        for p, r in zip(ps, refs):
            assert close_ratio(p.detach().cpu(), r.detach()) <= 1


def test_coordinate_hooks_handle_empty_and_value_only(cuda):
    from flashns_b200.jet_packed import PackedLayout
    from flashns_b200.native import NativeCUDA
    nat = NativeCUDA()
    for full, value in ((0, 0), (0, 5), (3, 0)):
        layout = PackedLayout(full, value, 2)
        x = torch.randn(layout.points, 2, dtype=torch.float64, device=cuda)
        d = torch.randn(layout.rows, 7, dtype=torch.float64, device=cuda)
        dw, db = nat.coordinate_wgrad(layout, x, d)
        zero = layout.zero_rows(cuda)
        coords = layout.coordinates(x)
        assert close_ratio(dw.cpu(), (d.T @ coords).cpu()) <= 1
        assert close_ratio(db.cpu(), d[zero].sum(0).cpu()) <= 1


def test_hopper_plan_names_match_oracle(cuda):
    """flashns_hopper_create / _launch / _destroy (the reference's Hopper plan ABI,
    experiments/cuda_jet_hopper/hopper.cu:287-353): D W, fused with the jet VJP or not, on
    the oracle; resources fills the nine values the reference's binding reads."""
    import ctypes

    import torch

    from flashns_b200 import _lib
    from oracle import jets as J
    lib = _lib.library()
    assert lib.flashns_hopper_initialize() == 0
    for dim in (2, 3):
        for fused in (False, True):
            vals = (ctypes.c_longlong * 9)()
            assert lib.flashns_hopper_resources(dim, fused, vals) == 0
            assert vals[1] > 0 and vals[0] > 0 and vals[5] >= 1
    rng = np.random.default_rng(11)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda).cuda_stream)
    for dim in (2, 3):
        q = J.q(dim)
        for cout, cin in ((32, 64), (64, 32), (64, 64)):
            batch = 37
            z = rng.normal(size=(batch, q, cin)) * 0.4
            h, a1 = J.tanh_jet(z, dim)
            d = rng.normal(size=(batch, q, cout))
            w = rng.normal(size=(cout, cin)) / np.sqrt(cout)
            dg, wg, hg, ag = (T(v, cuda) for v in (d, w, h, a1))
            plan = ctypes.c_void_p()
            assert lib.flashns_hopper_create(dim, _lib_ptr(dg), _lib_ptr(wg), batch, cout, cin, ctypes.byref(plan)) == 0
            try:
                for fused in (False, True):
                    out = torch.full((batch, q, cin), float("nan"), dtype=torch.float64, device=cuda)
                    assert lib.flashns_hopper_launch(plan, dim, fused, _lib_ptr(hg), _lib_ptr(ag), _lib_ptr(out),
                                                     stream) == 0
                    torch.cuda.synchronize()
                    expect = J.tanh_vjp(h, a1, d @ w, dim) if fused else d @ w
                    assert close_ratio(out.cpu(), expect) <= 1, (dim, cout, cin, fused)
                # a plan is tied to its jet size: the other dimension is refused
                out = torch.empty((batch, q, cin), dtype=torch.float64, device=cuda)
                assert lib.flashns_hopper_launch(plan, 5 - dim, False, None, None, _lib_ptr(out), stream) == 1
            finally:
                lib.flashns_hopper_destroy(plan)


def _lib_ptr(t):
    import ctypes
    return ctypes.c_void_p(t.data_ptr())
