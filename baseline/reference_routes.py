"""The reference's GPU routes for one FP64 loss + parameter-gradient evaluation, on the
reference's own compiled kernels (``baseline/_ref/``, built by
``baseline/build_reference_gpu.py``): the same-hardware baseline of
``bench.py --impl reference-gpu``.

The reference drives its kernels from Python with torch FP64 GEMMs in between.  That
Python does not travel to a GPU machine, so the orchestration is restated here, step for
step, from the reference files cited on each function; the kernels are the reference's.

Routes (all for the reference's (u, v, p) head with the gradient-enhanced residual, 2-D):

* ``F``  -- the route of the reference's published H100 headline: dense ``[B, Q, C]`` jets,
  torch GEMMs for the affine layers and weight gradients, ``flashns_stable_activation``,
  the interior seed by torch autograd of the residual, and the CUTLASS dgrad with the
  jet VJP fused into its epilogue (``flashns_stable_dgrad_vjp``);
* ``B1`` -- the same with the dgrad as a torch GEMM followed by the activation VJP kernel;
* ``v8`` -- the packed compact layout of ``PackedPINN`` with the v8 kernels: packed
  activation, the CUDA residual seed (``flashns_v8_loss_seed``), torch GEMMs between them
  (the v8 benchmark's configuration, ``experiments/pinn_v8/benchmark.py:45``);
* ``v8+`` -- the same with every opt-in v8 hook of ``PackedPINN``: the first affine layer
  fused with its activation, the first activation's VJP fused with the coordinate weight
  gradient, and the fused 3-output tail (F3).

Every route is captured once in a CUDA graph and replayed, as the reference's own
benchmarks do.  Nothing in the product imports this module.
"""

import ctypes
import hashlib
import json
import math
from pathlib import Path

import torch

from flashns_b200.jet_spec import JetSpec

LIBRARIES = Path(__file__).resolve().parent / "_ref"
ROUTES = ("F", "B1", "v8", "v8+")


def _sha256(path):
    return hashlib.sha256(Path(path).read_bytes()).hexdigest()


def available(directory=LIBRARIES):
    return (Path(directory) / "build.json").exists()


class ReferenceKernels:
    """ctypes bindings of the reference's compiled kernels, with the argument order of the
    reference's own bindings (``experiments/cuda_jet_h100/gpu.py:16-47`` for the dense
    kernels, ``experiments/pinn_v8/native.py:11-49`` for the packed ones).  Shapes are
    checked before every launch, as those bindings do, so a kernel never sees a buffer
    smaller than its sizes say."""

    def __init__(self, directory=LIBRARIES):
        directory = Path(directory)
        self.build = json.loads((directory / "build.json").read_text())
        libs = {}
        for name, item in self.build["libraries"].items():
            path = directory / item["file"]
            if _sha256(path) != item["sha256"]:
                raise RuntimeError(f"reference library changed since its build: {path.name}")
            libs[name] = ctypes.CDLL(str(path))
        if "dgrad_n64" not in libs:
            raise RuntimeError("the CUTLASS dgrad library was not built (no CUTLASS headers at build time)")
        ptr, i32, i64, size, flag = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t, ctypes.c_bool
        self._activation = libs["stable"].flashns_stable_activation
        self._activation.argtypes = [i32, flag] + [ptr] * 5 + [size, size, ptr]
        self._dgrad = libs["dgrad_n64"].flashns_stable_dgrad_vjp
        self._dgrad.argtypes = [i32, flag] + [ptr] * 5 + [i32] * 3 + [ptr]
        self._packed = libs["flashns_v8"].flashns_v8_activation
        self._packed.argtypes = [i32, i32] + [ptr] * 5 + [i64, i64, i32, ptr]
        self._seed = libs["flashns_v8"].flashns_v8_loss_seed
        self._seed.argtypes = [ptr] * 8 + [i64] * 3 + [ctypes.c_double] * 3 + [ptr]
        self._first = libs["flashns_v8"].flashns_v8_coordinate_affine_activation
        self._first.argtypes = [i32] + [ptr] * 5 + [i64, i64, i32, ptr]
        self._first_wgrad = libs["flashns_v8"].flashns_v8_coordinate_activation_wgrad
        self._first_wgrad.argtypes = [i32] + [ptr] * 7 + [i64, i64, i32, ptr]
        self._tail = libs["flashns_v8"].flashns_v8_tail3
        self._tail.argtypes = [i32, i32] + [ptr] * 5 + [i64, i64, i32, ptr]
        for f in (self._activation, self._dgrad, self._packed, self._seed, self._first, self._first_wgrad, self._tail):
            f.restype = ctypes.c_int

    @staticmethod
    def _check(tensors):
        device = tensors[0].device
        for t in tensors:
            if not t.is_cuda or t.dtype != torch.float64 or t.device != device or not t.is_contiguous():
                raise ValueError("contiguous FP64 CUDA tensors on one device required")

    @staticmethod
    def _call(function, args, tensors):
        with torch.cuda.device(tensors[0].device):
            stream = torch.cuda.current_stream()
            status = function(*args, ctypes.c_void_p(stream.cuda_stream))
        if status:
            raise RuntimeError(f"reference kernel returned CUDA error {status}")

    # dense [B, Q, C] jets (experiments/cuda_jet_h100/gpu.py:74-169)
    def forward(self, z, dim):
        self._check((z,))
        if z.ndim != 3 or z.shape[1] != JetSpec(dim).q:
            raise ValueError("expected [B, Q, C] jets")
        h, a1 = torch.empty_like(z), z.new_empty((z.shape[0], z.shape[2]))
        self._call(self._activation, [dim, False, z.data_ptr(), None, None, h.data_ptr(), a1.data_ptr(),
                                      z.shape[0], z.shape[2]], (z, h, a1))
        return h, a1

    def vjp(self, h, a1, hbar, dim):
        self._check((h, a1, hbar))
        if h.ndim != 3 or h.shape[1] != JetSpec(dim).q or hbar.shape != h.shape or a1.shape != (h.shape[0], h.shape[2]):
            raise ValueError("expected H, bar_H [B, Q, C] and a1 [B, C]")
        out = torch.empty_like(h)
        # argument order (value, adjoint, aux_in): stable_kernels.cu:94-97
        self._call(self._activation, [dim, True, h.data_ptr(), hbar.data_ptr(), a1.data_ptr(), out.data_ptr(), None,
                                      h.shape[0], h.shape[2]], (h, a1, hbar, out))
        return out

    def dgrad(self, d, w, h, a1, dim, backend):
        """bar_Z of the layer below: (D W) pulled back through the stable tanh jet."""
        self._check((d, w, h, a1))
        q = JetSpec(dim).q
        if (d.ndim != 3 or d.shape[1] != q or w.ndim != 2 or d.shape[2] != w.shape[0]
                or h.shape != (d.shape[0], q, w.shape[1]) or a1.shape != (d.shape[0], w.shape[1])):
            raise ValueError("expected D [B, Q, Cout], W [Cout, Cin], H [B, Q, Cin], a1 [B, Cin]")
        if backend == "B1":
            return self.vjp(h, a1, d @ w, dim)
        if backend != "F":
            raise ValueError("dense backends: B1, F")
        if d.shape[0] > (2**31 - 1) // 20 or w.shape[1] > 64 * 65535:
            raise ValueError("CUTLASS integer or grid dimension limit exceeded")
        out = torch.empty_like(h)
        self._call(self._dgrad, [dim, True, d.data_ptr(), w.data_ptr(), h.data_ptr(), a1.data_ptr(), out.data_ptr(),
                                 d.shape[0], w.shape[0], w.shape[1]], (d, w, h, a1, out))
        return out

    # packed rows [full x Q ; value x 1] (experiments/pinn_v8/native.py:66-97, 202-221)
    def packed_forward(self, full, value, dim, z):
        self._check((z,))
        if z.ndim != 2 or z.shape[0] != full * JetSpec(dim).q + value:
            raise ValueError("packed row count mismatch")
        h, a1 = torch.empty_like(z), z.new_empty((full + value, z.shape[1]))
        self._call(self._packed, [dim, 0, z.data_ptr(), None, None, h.data_ptr(), a1.data_ptr(), full, value,
                                  z.shape[1]], (z, h, a1))
        return h, a1

    def packed_vjp(self, full, value, dim, h, a1, hbar):
        self._check((h, a1, hbar))
        if (h.ndim != 2 or h.shape[0] != full * JetSpec(dim).q + value or hbar.shape != h.shape
                or a1.shape != (full + value, h.shape[1])):
            raise ValueError("packed H / a1 / bar_H shape mismatch")
        out = torch.empty_like(h)
        self._call(self._packed, [dim, 1, h.data_ptr(), a1.data_ptr(), hbar.data_ptr(), out.data_ptr(), None, full,
                                  value, h.shape[1]], (h, a1, hbar, out))
        return out

    def first_affine_activation(self, full, value, dim, x, w, b):
        """H_1, a1_1 of the packed rows straight from the coordinates
        (``experiments/pinn_v8/native.py:102-131``)."""
        self._check((x, w, b))
        c = w.shape[0]
        if x.shape != (full + value, dim) or w.shape != (c, dim) or b.shape != (c,):
            raise ValueError("expected x [points, dim], W [C, dim], b [C]")
        h, a1 = x.new_empty((full * JetSpec(dim).q + value, c)), x.new_empty((full + value, c))
        self._call(self._first, [dim, x.data_ptr(), w.data_ptr(), b.data_ptr(), h.data_ptr(), a1.data_ptr(), full,
                                 value, c], (x,))
        return h, a1

    def first_activation_wgrad(self, full, value, dim, x, h, a1, hbar):
        """dW_0, db_0 from bar_H_1 through the first activation's VJP
        (``experiments/pinn_v8/native.py:156-176``)."""
        self._check((x, h, a1, hbar))
        c = h.shape[1]
        if (x.shape != (full + value, dim) or h.shape != (full * JetSpec(dim).q + value, c) or hbar.shape != h.shape
                or a1.shape != (full + value, c)):
            raise ValueError("expected x [points, dim], H / bar_H [rows, C], a1 [points, C]")
        partials = h.new_empty(((full + value + 7) // 8, c, dim + 1))
        dw, db = h.new_empty((c, dim)), h.new_empty((c,))
        self._call(self._first_wgrad, [dim, h.data_ptr(), a1.data_ptr(), hbar.data_ptr(), x.data_ptr(),
                                       partials.data_ptr(), dw.data_ptr(), db.data_ptr(), full, value, c], (x,))
        return dw, db

    def tail3(self, full, value, dim, d, w, h, a1):
        """bar_Z of the last hidden layer from D [rows, 3] in one kernel, F3
        (``experiments/pinn_v8/native.py:178-200``)."""
        self._check((d, w, h, a1))
        c = h.shape[1]
        rows = full * JetSpec(dim).q + value
        if d.shape != (rows, 3) or w.shape != (3, c) or h.shape != (rows, c) or a1.shape != (full + value, c):
            raise ValueError("expected D [rows, 3], W [3, C], H [rows, C], a1 [points, C]")
        out = torch.empty_like(h)
        self._call(self._tail, [dim, 1, d.data_ptr(), w.data_ptr(), h.data_ptr(), a1.data_ptr(), out.data_ptr(), full,
                                value, c], (d,))
        return out

    def seed(self, jets, boundary, pde_weights, boundary_weights, target, nu, gamma, bc):
        ni, nb = len(jets), len(boundary)
        self._check((jets, pde_weights))
        if jets.shape != (ni, 10, 3) or pde_weights.shape != (ni,):
            raise ValueError("expected interior jets [N, 10, 3] and weights [N]")
        if boundary.shape != (nb, 3) or boundary_weights.shape != (nb, 3) or target.shape != (nb, 3):
            raise ValueError("expected boundary values, weights and targets [Nb, 3]")
        if nb:
            self._check((jets, boundary, boundary_weights, target))
        di, db = torch.empty_like(jets), jets.new_empty((nb, 3))
        partial = jets.new_empty(((ni + nb + 127) // 128,))
        tensors = (jets, boundary, pde_weights, boundary_weights, target, di, db, partial)
        ptrs = [t.data_ptr() if t.numel() else None for t in tensors]
        self._call(self._seed, ptrs + [ni, nb, 3, float(nu), float(gamma), float(bc)], (jets,))
        return partial.sum(), di, db


# ------------------------------------------------------------------------- the residual
def uvp_residual_per_point(jets, nu=0.07, gamma=0.2):
    """Per-point gradient-enhanced loss of (u, v, p) Taylor jets ``[N, 10, 3]`` as torch
    operations (for autograd), after ``experiments/cuda_jet_h100/common.py:99-146``:
    ``0.5 * sum over alpha in {0, d/dx, d/dy} of w_alpha (r_u^2 + r_v^2 + div^2)``, with
    w_0 = 1 and ``gamma`` for the two first-order coefficients."""
    order = JetSpec(2).coefficient_order
    slot = {a: k for k, a in enumerate(order)}

    def coef(field, a):
        return jets[:, slot[a], field]

    def diff(field, a, axis, times=1):
        # raw derivative of the Taylor coefficient: (a_axis + times)! / a_axis! * c[a + times e_axis]
        b = tuple(v + times if i == axis else v for i, v in enumerate(a))
        return (math.factorial(b[axis]) / math.factorial(a[axis])) * coef(field, b)

    total = 0.0
    for alpha in ((0, 0), (1, 0), (0, 1)):
        conv_u = conv_v = 0.0
        for beta in order:
            if beta[0] > alpha[0] or beta[1] > alpha[1]:
                continue
            rest = (alpha[0] - beta[0], alpha[1] - beta[1])
            u, v = coef(0, beta), coef(1, beta)
            conv_u = conv_u + u * diff(0, rest, 0) + v * diff(0, rest, 1)
            conv_v = conv_v + u * diff(1, rest, 0) + v * diff(1, rest, 1)
        r_u = conv_u + diff(2, alpha, 0) - nu * (diff(0, alpha, 0, 2) + diff(0, alpha, 1, 2))
        r_v = conv_v + diff(2, alpha, 1) - nu * (diff(1, alpha, 0, 2) + diff(1, alpha, 1, 2))
        div = diff(0, alpha, 0) + diff(1, alpha, 1)
        total = total + (1.0 if alpha == (0, 0) else gamma) * (r_u.square() + r_v.square() + div.square())
    return 0.5 * total


def coordinate_jets(x):
    """Dense input jets ``[B, Q, d]`` of coordinates: order 0 is x, the first-order
    coefficient of each axis is 1 (``experiments/cuda_jet/input/jet_reference.py:54-63``)."""
    dim = x.shape[1]
    order = JetSpec(dim).coefficient_order
    out = x.new_zeros((x.shape[0], len(order), dim))
    out[:, 0] = x
    for axis in range(dim):
        out[:, order.index(tuple(int(i == axis) for i in range(dim))), axis] = 1.0
    return out


def packed_coordinates(x, full):
    """Packed input rows ``[full x Q ; value x 1]`` of coordinates
    (``src/flashns/jet_packed.py:43-53``)."""
    dim = x.shape[1]
    order = JetSpec(dim).coefficient_order
    q = len(order)
    dense = coordinate_jets(x[:full]).reshape(full * q, dim)
    return torch.cat((dense, x[full:]))


def zero_rows(full, value, q, device):
    return torch.cat((torch.arange(0, full * q, q, device=device),
                      torch.arange(full * q, full * q + value, device=device)))


# ------------------------------------------------------------------------- the routes
def dense_step(x, quadrature, denominator, ws, bs, kernels, backend, nu=0.07, gamma=0.2):
    """One evaluation of the dense route (``experiments/cuda_jet_h100/common.py:149-190``):
    returns ``(loss, [dW_0..dW_L, db_0..db_L])``."""
    with torch.no_grad():
        h = coordinate_jets(x)
        saved, aux = [h], [None]
        for layer, (w, b) in enumerate(zip(ws, bs)):
            z = h @ w.T
            z[:, 0] += b
            if layer + 1 < len(ws):
                h, a1 = kernels.forward(z, 2)
            else:
                h, a1 = z, None
            saved.append(h)
            aux.append(a1)
    leaf = h.detach().requires_grad_()
    with torch.enable_grad():
        loss = (quadrature * uvp_residual_per_point(leaf, nu, gamma)).sum() / denominator
        (d,) = torch.autograd.grad(loss, leaf)
    dws, dbs = [None] * len(ws), [None] * len(ws)
    with torch.no_grad():
        for layer in reversed(range(len(ws))):
            dws[layer] = d.flatten(0, 1).T @ saved[layer].flatten(0, 1)
            dbs[layer] = d[:, 0].sum(0)
            if layer:
                d = kernels.dgrad(d, ws[layer], saved[layer], aux[layer], 2, backend)
    return loss.detach(), dws + dbs


def packed_step(x, ni, pde_weights, boundary_weights, target, ws, bs, kernels, nu=0.07, gamma=0.2, bc=5.0,
                inputs=None, hooks=False):
    """One evaluation of the v8 compact route: ``PackedPINN(layout="compact", seed="cuda")``
    with the v8 activation hooks (``src/flashns/pinn_packed.py:93-191``,
    ``experiments/pinn_v8/runtime.py:62-87``).  ``inputs`` are the packed coordinate rows,
    which ``PackedPINN`` builds once at construction (``pinn_packed.py:60-72``); they are
    built here when not given.  ``hooks`` adds the opt-in ``first_affine_activation``,
    ``first_activation_wgrad`` and ``tail_dgrad_vjp`` (F3) hooks (``pinn_packed.py:108-113,
    172-186``)."""
    nb = len(x) - ni
    q = 10
    last = len(ws) - 1
    with torch.no_grad():
        zero = zero_rows(ni, nb, q, x.device)
        h = packed_coordinates(x, ni) if inputs is None else inputs
        saved, aux = [h], []
        for layer, (w, b) in enumerate(zip(ws, bs)):
            if hooks and layer == 0 and last > 0:
                h, a1 = kernels.first_affine_activation(ni, nb, 2, x, w, b)
                aux.append(a1)
                saved.append(h)
                continue
            z = h @ w.T
            z[zero] += b
            if layer < last:
                h, a1 = kernels.packed_forward(ni, nb, 2, z)
                aux.append(a1)
            else:
                h = z
            saved.append(h)
        interior = saved[-1][:ni * q].view(ni, q, 3)
        boundary = saved[-1][zero[ni:]]
        total, di, db = kernels.seed(interior, boundary, pde_weights, boundary_weights, target, nu, gamma, bc)
        d = torch.zeros_like(saved[-1])
        d[:ni * q] = di.reshape(ni * q, 3)
        d[zero[ni:]] += db
        dws, dbs = [None] * len(ws), [None] * len(ws)
        for layer in reversed(range(len(ws))):
            dws[layer] = d.T @ saved[layer]
            dbs[layer] = d[zero].sum(0)
            if not layer:
                break
            if hooks and layer == 1:
                dws[0], dbs[0] = kernels.first_activation_wgrad(ni, nb, 2, x, saved[1], aux[0], d @ ws[1])
                break
            if hooks and layer == last and ws[layer].shape[0] == 3:
                d = kernels.tail3(ni, nb, 2, d, ws[layer], saved[layer], aux[layer - 1])
            else:
                d = kernels.packed_vjp(ni, nb, 2, saved[layer], aux[layer - 1], d @ ws[layer])
    return total, dws + dbs


class CapturedRoute:
    """A route captured once in a CUDA graph and replayed
    (``experiments/cuda_jet_h100/graph_experiment.py:29-60``,
    ``experiments/pinn_v8/runtime.py:90-117``).  ``x`` and the parameters are static
    inputs: overwrite them in place, then call ``refresh()``, before a replay."""

    def __init__(self, route, x, ni, pde_weights, boundary_weights, target, ws, bs, kernels, *, nu, gamma, bc=5.0):
        if route not in ROUTES:
            raise ValueError(f"route must be one of {ROUTES}")
        if route in ("F", "B1") and len(x) != ni:
            raise ValueError("the dense routes have no boundary rows")
        self.x, self.ni, self.ws, self.bs = x, ni, ws, bs
        self.inputs = None
        if route in ("v8", "v8+"):
            # packed coordinate rows are a static input, as in PackedPINN
            self.inputs = packed_coordinates(x, ni)
            self.step = lambda: packed_step(x, ni, pde_weights, boundary_weights, target, ws, bs, kernels, nu, gamma,
                                            bc, inputs=self.inputs, hooks=route == "v8+")
        else:
            # the dense routes weight the points by quadrature / denominator; the packed
            # weights are already globally normalized, so quadrature = weights, denominator = 1
            self.step = lambda: dense_step(x, pde_weights, 1.0, ws, bs, kernels, route, nu, gamma)
        self.stream = torch.cuda.Stream(x.device)
        self.stream.wait_stream(torch.cuda.current_stream(x.device))
        with torch.cuda.stream(self.stream):
            for _ in range(5):
                self.step()
        torch.cuda.current_stream(x.device).wait_stream(self.stream)
        torch.cuda.synchronize(x.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=self.stream):
            self.loss, self.grads = self.step()

    def refresh(self):
        """Rebuild the static packed coordinate rows after ``x`` changed (v8 route)."""
        if self.inputs is not None:
            self.inputs.copy_(packed_coordinates(self.x, self.ni))

    def replay(self):
        self.graph.replay()
        return self.loss, self.grads
