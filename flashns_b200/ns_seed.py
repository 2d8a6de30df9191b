"""Objective coefficients and the CUDA residual seed (API of ``src/flashns/ns_seed.py``).

``NSLoss``, ``residual_terms`` and ``validate_weights`` keep the reference names
and meaning (``src/flashns/ns_seed.py:13-51``).  The compute entry points
(``residuals``, ``per_point_loss``, ``explicit_seed``, ``compile_seed``) run the
generated seed kernels of ``libflashns_b200.so`` on CUDA tensors.
"""

from dataclasses import dataclass
from math import isfinite

import torch


@dataclass(frozen=True)
class NSLoss:
    viscosity: float = 0.07
    gradient_weight: float = 0.2
    boundary_weight: float = 5.0

    def __post_init__(self):
        if any(not isfinite(v) or v < 0 for v in (self.viscosity, self.gradient_weight, self.boundary_weight)):
            raise ValueError("finite nonnegative objective coefficients required")


def validate_weights(weights, shape, *, device):
    """Call during preparation, outside CUDA Graph capture and timed replay."""
    if weights.shape != shape or weights.dtype != torch.float64 or weights.device != torch.device(device):
        raise ValueError("FP64 weights with the expected shape/device required")
    if not bool(torch.isfinite(weights).all()) or bool((weights < 0).any()):
        raise ValueError("finite nonnegative globally normalized weights required")


def residual_terms(viscosity=0.07):
    """The nine (u, v, p) residual polynomials as (coefficient, i, j) terms, ``i = 3*q + field``,
    ``j = -1`` for a linear term (the format of ``src/flashns/ns_seed.py:26-43``), derived
    from the PDE by ``flashns_b200.codegen``."""
    from flashns_b200 import codegen
    from math import factorial, prod
    lookup = {a: i for i, a in enumerate(codegen.basis(2))}
    out = []
    for expr in codegen.residuals_uvp()[0]:
        terms = []
        for key, (a, b) in sorted(expr.items()):
            coef = (a + b * viscosity) * prod(prod(factorial(v) for v in al) for _, al in key)
            slots = [3 * lookup[al] + f for f, al in key]
            terms.append((coef, slots[0], slots[1] if len(slots) > 1 else -1))
        out.append(tuple(terms))
    return tuple(out)


def _residuals_cuda(jets, head, nu):
    import ctypes
    from flashns_b200 import _lib
    q = jets.shape[1]
    dim = 2 if q == 10 else 3
    r = 9 if head == "uvp" else 2
    out = jets.new_empty((jets.shape[0], r))
    lib = _lib.library()
    with torch.cuda.device(jets.device):
        stream = torch.cuda.current_stream()
        status = lib.flashns_b200_residuals(0 if head == "uvp" else 1, dim,
                                            ctypes.c_void_p(jets.data_ptr()) if jets.numel() else None, float(nu),
                                            ctypes.c_void_p(out.data_ptr()) if out.numel() else None, jets.shape[0],
                                            ctypes.c_void_p(stream.cuda_stream))
    _lib.check(status, "flashns_b200_residuals")
    return out


def residuals(jets, loss=NSLoss()):
    """The nine residuals of FP64 ``[N, 10, 3]`` (u, v, p) jets on the GPU."""
    if jets.ndim != 3 or jets.shape[1:] != (10, 3) or jets.dtype != torch.float64:
        raise ValueError("expected FP64 [N,10,3] jets of u,v,p")
    if not jets.is_cuda:
        raise ValueError("CUDA tensors required")
    return _residuals_cuda(jets.contiguous(), "uvp", loss.viscosity)


def per_point_loss(jets, loss=NSLoss()):
    r = residuals(jets, loss)
    return 0.5 * (r[:, :3].square().sum(1) + loss.gradient_weight * r[:, 3:].square().sum(1))


def explicit_seed(jets, weights, loss=NSLoss(), *, validate=True):
    """``(loss, d loss / d jets)`` of the interior objective (``src/flashns/ns_seed.py:72-91``)."""
    from flashns_b200.native import NativeCUDA
    if validate:
        validate_weights(weights, (len(jets),), device=jets.device)
    empty = jets.new_empty((0, 3))
    total, seed, _ = NativeCUDA().seed(jets.contiguous(), empty, weights.contiguous(), empty, empty, loss)
    return total, seed


def compile_seed(loss=NSLoss(), **compile_options):
    """The seed as a callable ``(jets, weights) -> (loss, seed)``; the CUDA kernel is already
    compiled, so ``compile_options`` are accepted and ignored.  Validate inputs before capture."""
    return lambda jets, weights: explicit_seed(jets, weights, loss, validate=False)
