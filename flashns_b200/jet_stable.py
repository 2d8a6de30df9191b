"""Stable tanh jets (API of ``src/flashns/jet_stable.py``).

``tanh_jet`` and ``tanh_vjp`` run the dense CUDA kernels on ``[B, Q, C]`` jets.
``stable_a1`` / ``stable_tanh`` (an autograd function whose derivative is the stable
``sech^2``) are device-agnostic tensor helpers for nested-derivative validation, as in
the reference (``jet_stable.py:1-5``); they are not on the evaluation path.
"""

from functools import lru_cache

import torch

from flashns_b200.jet_spec import JetSpec


def stable_a1(z0):
    r = torch.exp(torch.where(z0 >= 0, -z0, z0))
    v = (2 * r) / (1 + r * r)
    return v * v


class _StableTanh(torch.autograd.Function):
    @staticmethod
    def forward(ctx, value):
        ctx.save_for_backward(value)
        return value.tanh()

    @staticmethod
    def backward(ctx, adjoint):
        (value,) = ctx.saved_tensors
        return adjoint * stable_a1(value)


def stable_tanh(value):
    return _StableTanh.apply(value)


@lru_cache
def product_pairs(dim):
    indices = JetSpec(dim).coefficient_order
    lookup = {a: i for i, a in enumerate(indices)}
    return tuple(tuple((j, lookup[tuple(x - y for x, y in zip(a, b))]) for j, b in enumerate(indices)
                       if all(y <= x for x, y in zip(a, b))) for a in indices)


def tanh_jet(z, dim):
    """Stable tanh composition of full ``[B, Q, C]`` jets on the GPU: ``(H, a1)``."""
    from flashns_b200.native import Native
    if z.ndim != 3 or z.shape[1] != JetSpec(dim).q:
        raise ValueError("expected [B,Q,C] full jets")
    return Native().forward(z.contiguous(), dim)


def tanh_vjp(hidden, aux, adjoint, dim):
    from flashns_b200.native import Native
    return Native().vjp(hidden.contiguous(), aux.contiguous(), adjoint.contiguous(), dim)
