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
