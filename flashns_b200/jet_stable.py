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


@lru_cache
def _product_index(dim, device):
    """(alpha, j, k) index triples of the truncated Cauchy product, as device tensors."""
    triples = [(alpha, j, k) for alpha, terms in enumerate(product_pairs(dim)) for j, k in terms]
    t = torch.tensor(triples, dtype=torch.long, device=device).T
    return t[0], t[1], t[2]


def multiply(a, b, dim):
    """Truncated Cauchy product of ``[B, Q, ...]`` jets: ``(a b)_alpha = sum a_beta b_(alpha-beta)``
    (``src/flashns/jet_stable.py:52-59``).  A tensor helper for validation, like
    ``stable_tanh``; the evaluation kernels form their products in registers."""
    q = JetSpec(dim).q
    if a.shape != b.shape or a.ndim < 2 or a.shape[1] != q:
        raise ValueError("expected two [B,Q,...] jets of the same shape")
    alpha, j, k = _product_index(dim, a.device)
    out = a.new_zeros(a.shape)
    return out.index_add_(1, alpha, a[:, j] * b[:, k])


def tanh_jet(z, dim):
    """Stable tanh composition of full ``[B, Q, C]`` jets on the GPU: ``(H, a1)``."""
    from flashns_b200.native import Native
    if z.ndim != 3 or z.shape[1] != JetSpec(dim).q:
        raise ValueError("expected [B,Q,C] full jets")
    return Native().forward(z.contiguous(), dim)


def tanh_vjp(hidden, aux, adjoint, dim):
    from flashns_b200.native import Native
    return Native().vjp(hidden.contiguous(), aux.contiguous(), adjoint.contiguous(), dim)


def manifest(dim, source_hash):
    """The jet spec's manifest plus the activation's stored auxiliary state
    (``src/flashns/jet_stable.py:101-110``; the keys are the reference's so manifests
    compare across the two builds)."""
    value = JetSpec(dim).manifest(generated_source_hash=source_hash)
    value["activation_aux_state"] = {
        "strategy": "stable_aux_a1",
        "activation_revision": 2,
        "stored": ["H[B,Q,C]", "a1[B,C]"],
        "a1_rule": "(2*exp(-abs(Z0))/(1+exp(-2*abs(Z0))))^2",
        "tail_accuracy": "declared by per-device high-precision tests; relative accuracy not promised after "
                         "subnormal quantization",
    }
    return value
