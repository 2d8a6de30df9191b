"""Independent nested-autograd loss + gradient (torch, CPU, FP64).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

No jets: fields are evaluated pointwise and every spatial derivative is taken
by nested ``torch.autograd.grad``, in the manner of ``nested_step``
(``sources/flashns_v8_reference/tests/verify_math.py:65-83``) and
``nested_reference`` (``experiments/cuda_jet_h100/common.py:192-227``).  It pins the
jet oracle for both heads, including the stream-function head that has no
counterpart in the reference.
"""

import torch


def _stable_a1(z):
    r = torch.exp(torch.where(z >= 0, -z, z))
    return ((2 * r) / (1 + r * r)) ** 2


class _StableTanh(torch.autograd.Function):
    # Backward uses the stable auxiliary, as ``src/flashns/jet_stable.py:22-34``.
    @staticmethod
    def forward(ctx, z):
        ctx.save_for_backward(z)
        return torch.tanh(z)

    @staticmethod
    def backward(ctx, g):
        (z,) = ctx.saved_tensors
        return g * _stable_a1(z)


def field(x, ws, bs):
    h = x
    for layer, (w, b) in enumerate(zip(ws, bs)):
        h = h @ w.T + b
        if layer + 1 < len(ws):
            h = _StableTanh.apply(h)
    return h


def nested_step(x, ni, pde_weights, boundary_weights, target, weights, biases, *,
                head="uvp", nu=0.07, gamma=0.2, bc=5.0, boundary_order=0):
    dt = torch.float64
    ps = [torch.tensor(p, dtype=dt, requires_grad=True) for p in list(weights) + list(biases)]
    ws, bs = ps[:len(weights)], ps[len(weights):]
    x = torch.as_tensor(x, dtype=dt)
    dim = x.shape[1]
    loss = sum(p.sum() * 0 for p in ps)

    def grad(y, wrt):
        return torch.autograd.grad(y.sum(), wrt, create_graph=True, retain_graph=True)[0]

    if ni:
        xx = x[:ni].clone().requires_grad_()
        out = field(xx, ws, bs)
        g = lambda y: grad(y, xx)
        if head == "uvp":
            u, v, p = out.unbind(-1)
            gu, gv, gp = g(u), g(v), g(p)
            ru = u * gu[:, 0] + v * gu[:, 1] + gp[:, 0] - nu * (g(gu[:, 0])[:, 0] + g(gu[:, 1])[:, 1])
            rv = u * gv[:, 0] + v * gv[:, 1] + gp[:, 1] - nu * (g(gv[:, 0])[:, 0] + g(gv[:, 1])[:, 1])
            div = gu[:, 0] + gv[:, 1]
            per = 0.5 * (ru ** 2 + rv ** 2 + div ** 2 + gamma * (
                g(ru).square().sum(-1) + g(rv).square().sum(-1) + g(div).square().sum(-1)))
        else:
            psi, p = out.unbind(-1)
            gpsi, gp = g(psi), g(p)
            u, v = gpsi[:, 1], -gpsi[:, 0]
            gu, gv = g(u), g(v)
            ru = u * gu[:, 0] + v * gu[:, 1] + gp[:, 0] - nu * (g(gu[:, 0])[:, 0] + g(gu[:, 1])[:, 1])
            rv = u * gv[:, 0] + v * gv[:, 1] + gp[:, 1] - nu * (g(gv[:, 0])[:, 0] + g(gv[:, 1])[:, 1])
            if dim == 3:
                ru = ru + gu[:, 2]
                rv = rv + gv[:, 2]
            per = 0.5 * (ru ** 2 + rv ** 2)
        loss = loss + (torch.as_tensor(pde_weights, dtype=dt) * per).sum()
    if len(x) > ni:
        xb = x[ni:].clone().requires_grad_()
        out = field(xb, ws, bs)
        if boundary_order == 0:
            fields = out
        else:
            gpsi = grad(out[:, 0], xb)
            fields = torch.stack((gpsi[:, 1], -gpsi[:, 0], out[:, 1]), -1)
        err = fields - torch.as_tensor(target, dtype=dt)
        loss = loss + bc * (torch.as_tensor(boundary_weights, dtype=dt) * err ** 2).sum()
    grads = torch.autograd.grad(loss, ps)
    return float(loss.detach()), [p.detach().numpy() for p in grads]
