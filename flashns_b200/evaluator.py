"""Fused FP64 loss + parameter-gradient evaluation on one GPU.

``PackedEvaluator`` owns a plan of the C ABI (``flashns_b200_plan_create``), the
device copies of the point set and a caller-side workspace; each call launches
the fused kernel chain (``flashns_b200_eval``) on the current CUDA stream and
returns ``[grad(P), loss]`` in one contiguous FP64 buffer -- the layout the
multi-GPU all-reduce uses directly.
"""

import ctypes
import math

import torch

from flashns_b200 import _lib
from flashns_b200.ns_seed import NSLoss

HEADS = {"uvp": 0, "psi": 1}


def output_width(head):
    return 3 if head == "uvp" else 2


def target_width(head, boundary_order):
    return 3 if (head == "uvp" or boundary_order == 1) else 2


def parameter_count(widths):
    return sum(i * o + o for i, o in zip(widths, widths[1:]))


class Plan:
    """Host-side plan of one packed geometry (no device allocation)."""

    def __init__(self, dim, head, boundary_order, widths, interior, boundary, loss):
        lib = _lib.library()
        arr = (ctypes.c_int * len(widths))(*widths)
        handle = ctypes.c_void_p()
        _lib.check(lib.flashns_b200_plan_create(dim, HEADS[head], boundary_order, len(widths) - 1, arr,
                                                interior, boundary, loss.viscosity, loss.gradient_weight,
                                                loss.boundary_weight, ctypes.byref(handle)),
                   "flashns_b200_plan_create")
        self.handle = handle
        self._lib = lib
        size = ctypes.c_size_t()
        _lib.check(lib.flashns_b200_plan_workspace_bytes(handle, ctypes.byref(size)), "workspace_bytes")
        self.workspace_bytes = size.value
        count = ctypes.c_int64()
        _lib.check(lib.flashns_b200_plan_parameter_count(handle, ctypes.byref(count)), "parameter_count")
        self.parameters = count.value
        launches = ctypes.c_int()
        _lib.check(lib.flashns_b200_plan_launch_count(handle, ctypes.byref(launches)), "launch_count")
        self.launches = launches.value

    def __del__(self):
        handle = getattr(self, "handle", None)
        if handle is not None and handle.value:
            self._lib.flashns_b200_plan_destroy(handle)
            self.handle = None


class PackedEvaluator:
    """Loss and gradient of the packed PINN objective for a fixed point set.

    ``x[:interior_count]`` carry full third-order jets (Q=10 in 2-D, Q=20 in 3-D);
    the remaining points are boundary points with value rows (``boundary_order=0``,
    the reference layout) or first-order rows (``boundary_order=1``, psi head).
    """

    def __init__(self, x, interior_count, pde_weights, boundary_weights, target, widths, *,
                 head="uvp", boundary_order=0, loss=NSLoss(), device=None):
        if head not in HEADS:
            raise ValueError("head must be 'uvp' or 'psi'")
        if boundary_order not in (0, 1) or (head == "uvp" and boundary_order):
            raise ValueError("boundary_order must be 0 (uvp) or 0/1 (psi)")
        device = torch.device(device if device is not None else (x.device if x.is_cuda else "cuda"))
        if device.type != "cuda":
            raise ValueError("flashns_b200 evaluates on CUDA devices only")
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        if x.ndim != 2 or x.shape[1] not in (2, 3) or x.dtype != torch.float64:
            raise ValueError("FP64 coordinates [points, 2|3] required")
        dim = x.shape[1]
        if head == "uvp" and dim != 2:
            raise ValueError("the (u, v, p) head is two-dimensional")
        widths = [int(w) for w in widths]
        if len(widths) < 3 or widths[0] != dim or widths[-1] != output_width(head):
            raise ValueError(f"widths must be [{dim}, hidden..., {output_width(head)}] with >= 1 hidden layer")
        if any(w < 1 or w > 128 for w in widths[1:-1]):
            raise ValueError("hidden widths must lie in 1..128")
        ni = int(interior_count)
        if not 0 <= ni <= len(x):
            raise ValueError("invalid interior split")
        nb = len(x) - ni
        f = target_width(head, boundary_order)
        if pde_weights.shape != (ni,) or boundary_weights.shape != (nb, f) or target.shape != (nb, f):
            raise ValueError(f"expected pde_weights[{ni}], boundary_weights/target[{nb},{f}]")
        for t in (pde_weights, boundary_weights, target):
            if t.dtype != torch.float64:
                raise ValueError("FP64 objective tensors required")
        if not bool(torch.isfinite(x).all()) or not bool(torch.isfinite(target).all()):
            raise ValueError("finite coordinates and targets required")
        for w in (pde_weights, boundary_weights):
            if not bool(torch.isfinite(w).all()) or bool((w < 0).any()):
                raise ValueError("finite nonnegative globally normalized weights required")
        self.dim, self.head, self.boundary_order, self.loss = dim, head, boundary_order, loss
        self.widths, self.ni, self.nb, self.device = widths, ni, nb, device
        with torch.cuda.device(device):
            self.plan = Plan(dim, head, boundary_order, widths, ni, nb, loss)
            to = lambda t: t.detach().to(device=device, dtype=torch.float64).contiguous()
            self.x, self.pde_weights = to(x), to(pde_weights)
            self.boundary_weights, self.target = to(boundary_weights), to(target)
            self.workspace = torch.empty(max(1, (self.plan.workspace_bytes + 7) // 8), dtype=torch.float64,
                                         device=device)
        self.parameters = self.plan.parameters
        self.launches_per_call = self.plan.launches

    def __call__(self, flat, out=None):
        """Evaluate at the flat parameters ``[W_0..W_L, b_0..b_L]``; return ``out[P+1]``."""
        if flat.shape != (self.parameters,) or flat.dtype != torch.float64 or flat.device != self.device:
            raise ValueError(f"flat FP64 parameters [{self.parameters}] on {self.device} required")
        if not flat.is_contiguous():
            raise ValueError("contiguous parameters required")
        if flat.data_ptr() % 16:
            flat = flat.clone()  # the C ABI reads parameters from a 16-byte boundary
        if torch.is_grad_enabled() and flat.requires_grad:
            raise NotImplementedError("manual parameter VJP; double backward/HVP unsupported")
        if out is None:
            out = torch.empty(self.parameters + 1, dtype=torch.float64, device=self.device)
        elif out.shape != (self.parameters + 1,) or out.dtype != torch.float64 or out.device != self.device \
                or not out.is_contiguous():
            raise ValueError("out must be a contiguous FP64 [P+1] tensor on the device")
        lib = self.plan._lib
        with torch.cuda.device(self.device):
            stream = torch.cuda.current_stream()
            ptr = lambda t: ctypes.c_void_p(t.data_ptr()) if t.numel() else None
            status = lib.flashns_b200_eval(self.plan.handle, ptr(self.x), ptr(flat), ptr(self.pde_weights),
                                           ptr(self.boundary_weights), ptr(self.target), ptr(out),
                                           ptr(self.workspace), self.workspace.numel() * 8,
                                           ctypes.c_void_p(stream.cuda_stream))
        _lib.check(status, "flashns_b200_eval")
        return out

    def input_arena(self, flat):
        """Stage every input of a step in one buffer pair: a pinned host buffer and a device
        buffer, both ``[x | pde_weights | boundary_weights | target | parameters]`` with each
        segment starting on a 16-byte boundary.  The evaluator's inputs become views of the
        device buffer, so one host-to-device copy refreshes all of them.  Returns
        ``(host, device, parameters view)``; ``flat`` is copied into both buffers."""
        parts = [self.x, self.pde_weights, self.boundary_weights, self.target,
                 flat.detach().to(dtype=torch.float64).reshape(-1)]
        if parts[-1].numel() != self.parameters:
            raise ValueError(f"flat FP64 parameters [{self.parameters}] required")
        sizes = [t.numel() for t in parts]
        offsets, off = [], 0
        for n in sizes:
            offsets.append(off)
            off += n + (n & 1)  # even number of doubles: every segment 16-byte aligned
        device = torch.empty(max(off, 2), dtype=torch.float64, device=self.device)
        views = [device[o:o + n] for o, n in zip(offsets, sizes)]
        for v, t in zip(views, parts):
            v.copy_(t.reshape(-1))
        shapes = [t.shape for t in parts[:4]]
        self.x, self.pde_weights, self.boundary_weights, self.target = (
            v.view(shape) for v, shape in zip(views[:4], shapes))
        host = device.cpu().pin_memory()
        return host, device, views[4]

    def split(self, out):
        """Views ``(loss, [dW_0..dW_L, db_0..db_L])`` of an output buffer."""
        grads, offset = [], 0
        pairs = list(zip(self.widths, self.widths[1:]))
        for i, o in pairs:
            grads.append(out[offset:offset + i * o].view(o, i))
            offset += i * o
        for _, o in pairs:
            grads.append(out[offset:offset + o])
            offset += o
        return out[self.parameters], grads


def flat_parameters(weights, biases):
    return torch.cat([w.reshape(-1) for w in weights] + [b.reshape(-1) for b in biases])


def xavier_normal(widths, seed, dtype=torch.float64):
    """Xavier-normal weights (std sqrt(2/(fan_in+fan_out))), zero biases, from a seeded CPU generator."""
    gen = torch.Generator(device="cpu").manual_seed(seed)
    weights = [torch.randn(o, i, generator=gen, dtype=dtype) * math.sqrt(2.0 / (i + o))
               for i, o in zip(widths, widths[1:])]
    biases = [torch.zeros(o, dtype=dtype) for o in widths[1:]]
    return weights, biases


class FieldEvaluator:
    """Forward-only (u, v, p) -- or the raw outputs with value rows -- at a fixed point set
    (the acceptance grid of a solve): ``__call__(flat) -> fields [points, F]``."""

    def __init__(self, x, widths, *, head="psi", boundary_order=1, device=None):
        device = torch.device(device if device is not None else (x.device if x.is_cuda else "cuda"))
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        if x.ndim != 2 or x.dtype != torch.float64:
            raise ValueError("FP64 coordinates [points, dim] required")
        self.widths, self.head, self.device = [int(w) for w in widths], head, device
        with torch.cuda.device(device):
            self.plan = Plan(x.shape[1], head, boundary_order, self.widths, 0, len(x), NSLoss())
            self.x = x.detach().to(device).contiguous()
            self.workspace = torch.empty(max(1, (self.plan.workspace_bytes + 7) // 8), dtype=torch.float64,
                                         device=device)
        self.width = target_width(head, boundary_order)
        self.parameters = self.plan.parameters

    def __call__(self, flat, out=None):
        if flat.shape != (self.parameters,) or flat.dtype != torch.float64 or flat.device != self.device:
            raise ValueError(f"flat FP64 parameters [{self.parameters}] on {self.device} required")
        if out is None:
            out = torch.empty((len(self.x), self.width), dtype=torch.float64, device=self.device)
        elif out.shape != (len(self.x), self.width) or out.dtype != torch.float64 or out.device != self.device \
                or not out.is_contiguous():
            raise ValueError(f"out must be a contiguous FP64 [{len(self.x)}, {self.width}] tensor on the device")
        flat = flat.contiguous()
        lib = self.plan._lib
        with torch.cuda.device(self.device):
            stream = torch.cuda.current_stream()
            status = lib.flashns_b200_fields(self.plan.handle, ctypes.c_void_p(self.x.data_ptr()),
                                             ctypes.c_void_p(flat.data_ptr()),
                                             ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(self.workspace.data_ptr()),
                                             self.workspace.numel() * 8, ctypes.c_void_p(stream.cuda_stream))
        _lib.check(status, "flashns_b200_fields")
        return out
