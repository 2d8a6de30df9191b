"""Drop-in ``PackedPINN`` (API of ``src/flashns/pinn_packed.py:15-191``).

Construction validates and prepares the point set once (``pinn_packed.py:16-88``);
``__call__(weights, biases) -> (loss, [dW_0..dW_L, db_0..db_L])`` runs one fused FP64
evaluation (``flashns_b200_eval``) on the current CUDA stream.  Every ``layout``
(dense / split / compact) and ``seed`` mode of the reference describes the same
objective; all of them evaluate through the compact fused kernels.  The stage hooks
(``activation_factory``, ``cuda_seed``, ``tail_dgrad_vjp``, ``coordinate_*``,
``first_*``) are accepted when they are this library's own (``TensorActivation``, the
methods of ``flashns_b200.native``): the fused kernels already contain every stage they
replace, so they are recorded in ``metadata`` and not called.  Any other hook -- a
caller-defined stage or residual, or another library's kernels -- raises
``NotImplementedError`` at construction, because the reference would call it
(``src/flashns/pinn_packed.py:108-190``) and the fused kernels cannot.

Extensions: ``head="psi"`` (stream-function net, outputs (psi, p)), 3-D coordinates
(x, y, t) for the psi head, and ``boundary_order=1`` (first-order boundary rows with
(u, v, p) targets).
"""

from contextlib import nullcontext

import torch

from flashns_b200.evaluator import PackedEvaluator, output_width, target_width
from flashns_b200.ns_seed import NSLoss, validate_weights

HOOKS = ("activation_factory", "cuda_seed", "residual_reference", "tail_dgrad_vjp", "coordinate_affine",
         "first_affine_activation", "coordinate_wgrad", "first_activation_wgrad")


def foreign_hooks(**hooks):
    """Names of the supplied stage hooks that are not this library's own.

    The fused kernels contain every stage a hook replaces, so this library's hooks
    (``TensorActivation`` and the methods of ``flashns_b200.native.NativeCUDA`` /
    ``Native``) change nothing.  Any other callable -- the reference's own equivalent
    hooks included -- is not called either; ``PackedPINN`` warns about those, because a
    caller-defined stage or residual would silently not take effect."""
    from flashns_b200.jet_packed import TensorActivation
    from flashns_b200.native import Native, NativeCUDA
    from flashns_b200.ns_seed import per_point_loss
    foreign = []
    for name, hook in hooks.items():
        if hook is None or hook is TensorActivation or hook is per_point_loss:
            continue
        if isinstance(getattr(hook, "__self__", None), (NativeCUDA, Native)):
            continue
        foreign.append(name)
    return foreign


class PackedPINN:
    def __init__(self, x, interior_count, pde_weights, boundary_weights, target, *, layout="compact",
                 seed="explicit", activation_factory=None, cuda_seed=None, residual_reference=None, loss=NSLoss(),
                 compiled_options=None, trace=False, tail_dgrad_vjp=None, coordinate_affine=None,
                 first_affine_activation=None, coordinate_wgrad=None, first_activation_wgrad=None,
                 head="uvp", boundary_order=0):
        if head not in ("uvp", "psi"):
            raise ValueError("head must be 'uvp' or 'psi'")
        dims = (2,) if head == "uvp" else (2, 3)
        if x.ndim != 2 or x.shape[1] not in dims or x.dtype != torch.float64:
            raise ValueError("the fixed NS residual requires FP64 2-D coordinates" if head == "uvp"
                             else "FP64 2-D or 3-D coordinates required")
        if type(interior_count) is not int or not 0 <= interior_count <= len(x):
            raise ValueError("invalid interior split")
        if layout not in ("dense", "split", "compact") or seed not in ("autograd", "explicit", "compiled", "cuda"):
            raise ValueError("unsupported layout or seed mode")
        if seed == "cuda" and cuda_seed is None:
            raise ValueError("CUDA seed implementation required")
        for name, hook in (("tail_dgrad_vjp", tail_dgrad_vjp), ("coordinate_affine", coordinate_affine),
                           ("first_affine_activation", first_affine_activation),
                           ("coordinate_wgrad", coordinate_wgrad), ("first_activation_wgrad", first_activation_wgrad)):
            if hook is not None and not callable(hook):
                raise ValueError(f"{name} must be callable or None")
        # the reference calls residual_reference only for seed="autograd" and cuda_seed
        # only for seed="cuda" (src/flashns/pinn_packed.py:136-146)
        foreign = foreign_hooks(
            activation_factory=activation_factory, cuda_seed=cuda_seed if seed == "cuda" else None,
            residual_reference=residual_reference if seed == "autograd" else None, tail_dgrad_vjp=tail_dgrad_vjp,
            coordinate_affine=coordinate_affine, first_affine_activation=first_affine_activation,
            coordinate_wgrad=coordinate_wgrad, first_activation_wgrad=first_activation_wgrad)
        if foreign:
            raise NotImplementedError(
                f"flashns_b200 PackedPINN evaluates every stage in its fused kernels and cannot call the "
                f"supplied {', '.join(foreign)} hook(s); pass None (or this library's own hooks) to evaluate "
                f"the NSLoss objective")
        if not x.is_cuda:
            raise ValueError("flashns_b200 evaluates on CUDA tensors (no CPU path)")
        self.ni, self.nb = interior_count, len(x) - interior_count
        f = target_width(head, boundary_order)
        validate_weights(pde_weights, (self.ni,), device=x.device)
        validate_weights(boundary_weights, (self.nb, f), device=x.device)
        if target.shape != (self.nb, f) or target.dtype != torch.float64 or target.device != x.device:
            raise ValueError("boundary target shape/dtype/device mismatch")
        if not bool(torch.isfinite(x).all()) or not bool(torch.isfinite(target).all()):
            raise ValueError("finite coordinates and targets required")
        # the point set is fixed at construction, as the reference's packed inputs are
        # (pinn_packed.py:60-66): a later in-place change of `x` does not reach this object;
        # weights and targets are kept by reference, as there
        self.x = x.detach().clone(memory_format=torch.contiguous_format)
        self.pde_weights = pde_weights.detach().contiguous()
        self.boundary_weights = boundary_weights.detach().contiguous()
        self.target = target.detach().contiguous()
        self.mode, self.seed_mode, self.loss, self.head = layout, seed, loss, head
        self.boundary_order, self.trace = boundary_order, trace
        self._evaluators = {}
        dim = x.shape[1]
        q = 10 if dim == 2 else 20
        self.metadata = {
            "layout": layout, "seed": seed, "full_order": 3, "dimension": dim, "head": head,
            "boundary_order": boundary_order, "interior_count": self.ni, "boundary_count": self.nb,
            "segment_rows": [self.ni * q + self.nb * (dim + 1 if boundary_order else 1)],
            "packed_rows_total": self.ni * q + self.nb * (dim + 1 if boundary_order else 1),
            "precision": "FP64 stable_aux_a1", "weights": "already globally normalized",
            "supports_hvp_or_double_backward": False, "implementation": "flashns_b200 fused sm_100a kernels",
            "tail_dgrad_vjp_enabled": tail_dgrad_vjp is not None,
            "coordinate_affine_enabled": coordinate_affine is not None,
            "first_affine_activation_enabled": first_affine_activation is not None,
            "coordinate_wgrad_enabled": coordinate_wgrad is not None,
            "first_activation_wgrad_enabled": first_activation_wgrad is not None,
            "hooks_not_called": [name for name, hook in (
                ("activation_factory", activation_factory), ("cuda_seed", cuda_seed),
                ("residual_reference", residual_reference), ("tail_dgrad_vjp", tail_dgrad_vjp),
                ("coordinate_affine", coordinate_affine), ("first_affine_activation", first_affine_activation),
                ("coordinate_wgrad", coordinate_wgrad), ("first_activation_wgrad", first_activation_wgrad))
                if hook is not None],
        }

    def region(self, name):
        return torch.profiler.record_function("flashns_b200::" + name) if self.trace else nullcontext()

    def evaluator(self, widths):
        key = tuple(widths)
        if key not in self._evaluators:
            self._evaluators[key] = PackedEvaluator(self.x, self.ni, self.pde_weights, self.boundary_weights,
                                                    self.target, list(widths), head=self.head,
                                                    boundary_order=self.boundary_order, loss=self.loss,
                                                    device=self.x.device)
        return self._evaluators[key]

    def __call__(self, weights, biases):
        nf = output_width(self.head)
        if not weights or len(weights) != len(biases) or weights[-1].shape[0] != nf:
            raise ValueError(f"matching affine layers with {nf} final outputs required")
        cin = self.x.shape[1]
        widths = [cin]
        for weight, bias in zip(weights, biases):
            if weight.ndim != 2 or weight.shape[1] != cin or bias.shape != (weight.shape[0],):
                raise ValueError("incompatible affine layer")
            if any(t.dtype != torch.float64 or t.device != self.x.device for t in (weight, bias)):
                raise ValueError("all parameters must be FP64 on the data device")
            cin = weight.shape[0]
            widths.append(cin)
        ev = self.evaluator(widths)
        with torch.no_grad(), self.region("evaluation"):
            flat = torch.cat([w.detach().reshape(-1) for w in weights] + [b.detach().reshape(-1) for b in biases])
            out = ev(flat)
        total, grads = ev.split(out)
        return total, grads
