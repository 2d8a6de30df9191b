"""Sample data parallelism: one shard of points per rank, one all-reduce per evaluation.

Restates the reference's sample-DP evaluation (experiments/cuda_jet_v5/distributed.py:53-101,
src/flashns/distributed_contract.py:7-20) for the fused evaluator:

* every rank takes ``shard_bounds`` of the interior points and of the boundary points
  (weights are globally normalized before sharding, so local sums add up);
* each rank evaluates its shard into the packed FP64 buffer ``[grad(P), loss]``;
* one ``all_reduce(SUM)`` of that buffer (NCCL over NVLink on GPUs) gives every rank the
  identical global gradient and loss.  A NaN/Inf on any rank reaches every rank through
  the sum, which replaces the reference's separate finite-flag collective
  (distributed.py:76-81); ``finite(out)`` is the unanimous check.

For bitwise run-to-run reproducibility fix NCCL's algorithm and protocol (e.g.
``NCCL_ALGO=Ring NCCL_PROTO=Simple``); the sum order is then fixed.
"""

import torch
import torch.distributed as dist

from flashns_b200.problems import PointSet


class DistributedEvaluator:
    """``__call__(flat) -> out[P+1]`` with the global gradient and loss on every rank.

    ``points`` is the GLOBAL point set (every rank builds the same one from a seed);
    ``local_factory(shard) -> callable(flat, out)`` builds the per-rank evaluator (by
    default a CUDA ``PackedEvaluator`` on ``device``).
    """

    def __init__(self, points: PointSet, widths, *, head="psi", boundary_order=1, loss=None, device=None,
                 group=None, local_factory=None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.shard = points.shard(self.world, self.rank)
        if local_factory is None:
            from flashns_b200.evaluator import PackedEvaluator
            from flashns_b200.ns_seed import NSLoss
            loss = loss or NSLoss(viscosity=points.viscosity)
            s = self.shard
            ev = PackedEvaluator(s.x, s.interior_count, s.pde_weights, s.boundary_weights, s.target, widths,
                                 head=head, boundary_order=boundary_order, loss=loss, device=device)
            self.local = ev
            self.parameters = ev.parameters
        else:
            self.local = local_factory(self.shard)
            self.parameters = sum(i * o + o for i, o in zip(widths, widths[1:]))

    def __call__(self, flat, out=None):
        out = self.local(flat, out)
        if self.world > 1:
            dist.all_reduce(out, op=dist.ReduceOp.SUM, group=self.group)
        return out

    @staticmethod
    def finite(out):
        """Unanimous: the reduced buffer is finite on every rank or on none."""
        return bool(torch.isfinite(out).all())
