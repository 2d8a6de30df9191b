"""Packed full-jet / value-row layout and its CUDA activation (API of ``src/flashns/jet_packed.py``).

``PackedLayout`` keeps the reference contract (``jet_packed.py:12-59``).  The compute
entry points run this library's kernels: ``TensorActivation`` (the reference's name
for the activation object, ``jet_packed.py:91-133``) and ``full_vjp`` launch the packed
and dense stable-tanh kernels.
"""

from dataclasses import dataclass
from functools import lru_cache

import torch

from flashns_b200.jet_spec import JetSpec
from flashns_b200.jet_stable import stable_a1  # noqa: F401  (the reference exports it here too)


@dataclass(frozen=True)
class PackedLayout:
    full_points: int
    value_points: int
    dimension: int = 2

    def __post_init__(self):
        if any(type(n) is not int or n < 0 for n in (self.full_points, self.value_points)):
            raise ValueError("nonnegative integer point counts required")
        JetSpec(self.dimension)

    @property
    def q(self):
        return JetSpec(self.dimension).q

    @property
    def points(self):
        return self.full_points + self.value_points

    @property
    def full_rows(self):
        return self.full_points * self.q

    @property
    def rows(self):
        return self.full_rows + self.value_points

    def zero_rows(self, device):
        return torch.cat((torch.arange(0, self.full_rows, self.q, device=device),
                          torch.arange(self.full_rows, self.rows, device=device))).long()

    def coordinates(self, x):
        """Input jets of the coordinates (order-0 value, unit first-order coefficients)."""
        if x.shape != (self.points, self.dimension) or x.dtype != torch.float64:
            raise ValueError("FP64 coordinates must match the layout")
        if x.is_cuda:  # one kernel (flashns_b200_pack_coordinates), same values
            import ctypes

            from flashns_b200 import _lib
            x = x.contiguous()
            result = torch.empty((self.rows, self.dimension), dtype=torch.float64, device=x.device)
            with torch.cuda.device(x.device):
                stream = ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)
                _lib.check(_lib.library().flashns_b200_pack_coordinates(
                    ctypes.c_void_p(x.data_ptr()), self.full_points, self.value_points, self.dimension,
                    ctypes.c_void_p(result.data_ptr()), stream), "flashns_b200_pack_coordinates")
            return result
        result = x.new_zeros((self.rows, self.dimension))
        result[self.zero_rows(x.device)] = x
        order = JetSpec(self.dimension).coefficient_order
        full = result[:self.full_rows].view(self.full_points, self.q, self.dimension)
        for axis in range(self.dimension):
            full[:, order.index(tuple(int(axis == j) for j in range(self.dimension))), axis] = 1.0
        return result

    def check(self, tensor):
        if tensor.ndim != 2 or tensor.shape[0] != self.rows or tensor.shape[1] < 1:
            raise ValueError("packed row/channel shape mismatch")
        if tensor.dtype != torch.float64 or not tensor.is_contiguous():
            raise ValueError("contiguous FP64 packed storage required")


@lru_cache(None)
def convolution_terms(dimension):
    """For each alpha: the (beta, alpha-beta) index pairs of the truncated Cauchy product."""
    indices = JetSpec(dimension).coefficient_order
    lookup = {a: k for k, a in enumerate(indices)}
    return tuple(tuple((i, lookup[tuple(x - y for x, y in zip(a, b))])
                       for i, b in enumerate(indices) if all(y <= x for x, y in zip(a, b)))
                 for a in indices)


def full_vjp(hidden, auxiliary, seed, dimension):
    """Jet VJP of full ``[N, Q, C]`` jets on the GPU (``jet_packed.py:76-88``)."""
    from flashns_b200.native import Native
    return Native().vjp(hidden.contiguous(), auxiliary.contiguous(), seed.contiguous(), dimension)


class TensorActivation:
    """Packed stable-tanh activation: ``forward(Z) -> (H, a1)``, ``vjp(H, a1, bar_H) -> bar_Z``.

    ``compiled`` / ``compile_options`` are accepted for signature compatibility; the
    kernels are always the compiled CUDA path.
    """

    def __init__(self, layout, *, compiled=False, compile_options=None):
        from flashns_b200.native import NativeCUDA
        self.layout = layout
        impl = NativeCUDA().activation_factory(layout)
        self.forward = impl.forward
        self.vjp = impl.vjp
