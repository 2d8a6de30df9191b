"""Hook providers with the reference's binding interface, on this library's kernels.

``NativeCUDA`` has the methods of ``experiments/pinn_v8/native.py:11-221`` (packed
layout hooks for ``PackedPINN``) and ``Native`` those of
``experiments/cuda_jet_h100/gpu.py`` (dense ``[B,Q,C]`` activation, VJP and dgrad).
Launches are asynchronous on the current stream; shape/dtype errors raise
``ValueError``, nonzero CUDA statuses ``RuntimeError``.
"""

import ctypes

import torch

from flashns_b200 import _lib
from flashns_b200.jet_spec import JetSpec


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None and t.numel() else None


def _launch(name, args, tensors):
    lib = _lib.library()
    with torch.cuda.device(tensors[0].device):
        stream = torch.cuda.current_stream()
        status = getattr(lib, name)(*args, ctypes.c_void_p(stream.cuda_stream))
        for t in tensors:
            if t is not None and t.numel():
                t.record_stream(stream)
    if status:
        raise RuntimeError(f"{name} returned CUDA error {status}")


def _check(tensors):
    device = tensors[0].device
    for t in tensors:
        if not t.is_cuda or t.dtype != torch.float64 or t.device != device:
            raise ValueError("same-device CUDA FP64 tensors required")
        if not t.is_contiguous():
            raise ValueError("contiguous tensors required")
        if torch.is_grad_enabled() and t.requires_grad:
            raise NotImplementedError("manual parameter VJP; double backward/HVP unsupported")


class _PackedActivation:
    def __init__(self, layout):
        self.layout = layout

    def forward(self, value):
        layout = self.layout
        _check((value,))
        layout.check(value)
        out = torch.empty_like(value)
        aux = value.new_empty((layout.points, value.shape[1]))
        _launch("flashns_v8_activation", [layout.dimension, 0, _ptr(value), None, None, _ptr(out), _ptr(aux),
                                          layout.full_points, layout.value_points, value.shape[1]],
                (value, out, aux))
        return out, aux

    def vjp(self, hidden, aux, seed):
        layout = self.layout
        _check((hidden, aux, seed))
        layout.check(hidden)
        layout.check(seed)
        if aux.shape != (layout.points, hidden.shape[1]) or seed.shape != hidden.shape:
            raise ValueError("auxiliary/adjoint shape mismatch")
        out = torch.empty_like(hidden)
        _launch("flashns_v8_activation", [layout.dimension, 1, _ptr(hidden), _ptr(aux), _ptr(seed), _ptr(out), None,
                                          layout.full_points, layout.value_points, hidden.shape[1]],
                (hidden, aux, seed, out))
        return out


class NativeCUDA:
    """Packed-layout hooks (``experiments/pinn_v8/native.py:11-221``)."""

    def __init__(self, build_directory=None):
        _lib.library()
        self.metadata = {"library": str(_lib.LIBRARY), "precision": "FP64", "arch": "sm_100a"}

    def activation_factory(self, layout):
        return _PackedActivation(layout)

    def coordinate_affine(self, layout, coordinates, weight, bias):
        return self._coordinate_affine(layout, coordinates, weight, bias, activation=False)

    def coordinate_affine_activation(self, layout, coordinates, weight, bias):
        return self._coordinate_affine(layout, coordinates, weight, bias, activation=True)

    def _coordinate_affine(self, layout, coordinates, weight, bias, *, activation):
        tensors = (coordinates, weight, bias)
        _check(tensors)
        if coordinates.shape != (layout.points, layout.dimension) or weight.ndim != 2:
            raise ValueError("coordinates must match the physical-coordinate layout")
        channels = weight.shape[0]
        if channels < 1 or weight.shape[1] != layout.dimension or bias.shape != (channels,):
            raise ValueError("expected W[C,dimension], bias[C]")
        out = coordinates.new_empty((layout.rows, channels))
        if activation:
            aux = coordinates.new_empty((layout.points, channels))
            _launch("flashns_v8_coordinate_affine_activation",
                    [layout.dimension, *map(_ptr, tensors), _ptr(out), _ptr(aux), layout.full_points,
                     layout.value_points, channels], (*tensors, out, aux))
            return out, aux
        _launch("flashns_v8_coordinate_affine", [layout.dimension, *map(_ptr, tensors), _ptr(out), layout.full_points,
                                                 layout.value_points, channels], (*tensors, out))
        return out

    def coordinate_wgrad(self, layout, coordinates, derivative):
        tensors = (coordinates, derivative)
        _check(tensors)
        layout.check(derivative)
        channels = derivative.shape[1]
        if coordinates.shape != (layout.points, layout.dimension):
            raise ValueError("expected coordinates[points,dimension], bar_Z[rows,C]")
        partials = derivative.new_empty(((layout.points + 7) // 8, channels, layout.dimension + 1))
        dw = derivative.new_empty((channels, layout.dimension))
        db = derivative.new_empty((channels,))
        _launch("flashns_v8_coordinate_wgrad", [layout.dimension, _ptr(derivative), _ptr(coordinates), _ptr(partials),
                                                _ptr(dw), _ptr(db), layout.full_points, layout.value_points, channels],
                (*tensors, partials, dw, db))
        return dw, db

    def coordinate_activation_wgrad(self, layout, coordinates, hidden, aux, seed):
        tensors = (coordinates, hidden, aux, seed)
        _check(tensors)
        layout.check(hidden)
        layout.check(seed)
        channels = hidden.shape[1]
        if coordinates.shape != (layout.points, layout.dimension) or seed.shape != hidden.shape \
                or aux.shape != (layout.points, channels):
            raise ValueError("expected x[points,dimension], H/bar_H[rows,C], a1[points,C]")
        partials = hidden.new_empty(((layout.points + 7) // 8, channels, layout.dimension + 1))
        dw, db = hidden.new_empty((channels, layout.dimension)), hidden.new_empty((channels,))
        _launch("flashns_v8_coordinate_activation_wgrad",
                [layout.dimension, _ptr(hidden), _ptr(aux), _ptr(seed), _ptr(coordinates), _ptr(partials), _ptr(dw),
                 _ptr(db), layout.full_points, layout.value_points, channels], (*tensors, partials, dw, db))
        return dw, db

    def tail_dgrad_vjp(self, layout, d, weight, hidden, aux, *, backend="F3"):
        if backend not in ("U3", "F3"):
            raise ValueError("packed tail backend must be U3 or F3")
        tensors = (d, weight, hidden, aux)
        _check(tensors)
        layout.check(d)
        layout.check(hidden)
        channels = hidden.shape[1]
        if d.shape != (layout.rows, 3) or weight.shape != (3, channels) or aux.shape != (layout.points, channels):
            raise ValueError("expected D[rows,3], W[3,C], H[rows,C], aux[points,C]")
        out = torch.empty_like(hidden)
        _launch("flashns_v8_tail3", [layout.dimension, int(backend == "F3"), *map(_ptr, tensors), _ptr(out),
                                     layout.full_points, layout.value_points, channels], (*tensors, out))
        if backend == "U3":
            return self.activation_factory(layout).vjp(hidden, aux, out)
        return out

    def seed(self, jets, boundary, pde_weights, boundary_weights, target, loss):
        ni, nb = len(jets), len(boundary)
        for t in (jets, boundary, pde_weights, boundary_weights, target):
            if not t.is_cuda or t.dtype != torch.float64 or t.device != jets.device:
                raise ValueError("same-device CUDA FP64 tensors required")
        if jets.shape != (ni, 10, 3) or boundary.shape != (nb, 3) or boundary.stride(-1) != 1:
            raise ValueError("2-D Q10 interior and contiguous-channel boundary fields required")
        if nb > 1 and boundary.stride(0) < 3:
            raise ValueError("boundary rows must not overlap or broadcast")
        if pde_weights.shape != (ni,) or boundary_weights.shape != (nb, 3) or target.shape != (nb, 3):
            raise ValueError("objective shape mismatch")
        if not all(t.is_contiguous() for t in (jets, pde_weights, boundary_weights, target)):
            raise ValueError("contiguous jet/weight/target storage required")
        di, db = torch.empty_like(jets), boundary.new_empty((nb, 3))
        partial = jets.new_empty(((ni + nb + 127) // 128,))
        boundary_ptr = ctypes.c_void_p(boundary.data_ptr()) if nb else None
        _launch("flashns_v8_loss_seed",
                [_ptr(jets), boundary_ptr, _ptr(pde_weights), _ptr(boundary_weights), _ptr(target), _ptr(di), _ptr(db),
                 _ptr(partial), ni, nb, max(3, boundary.stride(0)) if nb else 3, loss.viscosity,
                 loss.gradient_weight, loss.boundary_weight], (jets, pde_weights, boundary_weights, target, di, db,
                                                               partial))
        return partial.sum(), di, db


class Native:
    """Dense ``[B,Q,C]`` hooks (``experiments/cuda_jet_h100/gpu.py``): forward, vjp, dgrad."""

    BACKENDS = ("B1", "F", "F_n32", "U3", "F3")

    def __init__(self, *args, **kwargs):
        _lib.library()

    def forward(self, value, dim):
        q = JetSpec(dim).q
        _check((value,))
        if value.ndim != 3 or value.shape[1] != q:
            raise ValueError("expected canonical full [B,Q,C] jets")
        hidden = torch.empty_like(value)
        aux = value.new_empty((value.shape[0], value.shape[2]))
        _launch("flashns_stable_activation", [dim, False, _ptr(value), None, None, _ptr(hidden), _ptr(aux),
                                              value.shape[0], value.shape[2]], (value, hidden, aux))
        return hidden, aux

    def vjp(self, hidden, aux, adjoint, dim):
        q = JetSpec(dim).q
        _check((hidden, aux, adjoint))
        if hidden.ndim != 3 or hidden.shape[1] != q or adjoint.shape != hidden.shape \
                or aux.shape != (hidden.shape[0], hidden.shape[2]):
            raise ValueError("incompatible full jets, auxiliary state or adjoint")
        out = torch.empty_like(hidden)
        _launch("flashns_stable_activation", [dim, True, _ptr(hidden), _ptr(adjoint), _ptr(aux), _ptr(out), None,
                                              hidden.shape[0], hidden.shape[2]], (hidden, aux, adjoint, out))
        return out

    def dgrad(self, d, weight, hidden, aux, dim, backend="B1"):
        if backend not in self.BACKENDS:
            raise ValueError(f"unknown backend {backend}")
        q = JetSpec(dim).q
        _check((d, weight, hidden, aux))
        if d.ndim != 3 or d.shape[1] != q or weight.ndim != 2 or d.shape[2] != weight.shape[0] \
                or hidden.shape != (d.shape[0], q, weight.shape[1]) or aux.shape != (d.shape[0], weight.shape[1]) \
                or weight.shape[0] == 0:
            raise ValueError("expected D[B,Q,Cout], W[Cout,Cin], H[B,Q,Cin], aux[B,Cin]")
        out = torch.empty_like(hidden)
        tensors = (d, weight, hidden, aux, out)
        if backend in ("U3", "F3") and weight.shape[0] == 3:
            _launch("flashns_stable_tail3", [dim, backend == "F3", *map(_ptr, tensors), d.shape[0], weight.shape[1]],
                    tensors)
            return out if backend == "F3" else self.vjp(hidden, aux, out, dim)
        fused = backend.startswith("F")
        _launch("flashns_stable_dgrad_vjp", [dim, fused, *map(_ptr, tensors), d.shape[0], weight.shape[0],
                                             weight.shape[1]], tensors)
        return out if fused else self.vjp(hidden, aux, out, dim)
