"""GPU (NCCL, 2 ranks on 2 GPUs; skipped with fewer): the sharded evaluation with one
all-reduce equals the single-GPU evaluation of the whole point set and the oracle.  The
shards split 4,099 interior and 1,031 boundary points 2,049 / 2,050 and 515 / 516, so both
shard boundaries cut through a tile of the kernels."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, queue):
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from flashns_b200.distributed import DistributedEvaluator
        from flashns_b200.evaluator import flat_parameters, xavier_normal
        from flashns_b200.problems import kovasznay
        widths = [2, 64, 64, 64, 2]
        pts = kovasznay(4099, 1031, seed=3)
        ev = DistributedEvaluator(pts, widths, head="psi", boundary_order=1, device=torch.device("cuda", rank))
        ws, bs = xavier_normal(widths, 0)
        out = ev(flat_parameters(ws, bs).cuda(rank)).cpu().numpy()
        queue.put((rank, out))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_gpu_allreduce_matches_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from flashns_b200.evaluator import PackedEvaluator, flat_parameters, xavier_normal
    from flashns_b200.ns_seed import NSLoss
    from flashns_b200.problems import kovasznay
    widths = [2, 64, 64, 64, 2]
    pts = kovasznay(4099, 1031, seed=3)
    single = PackedEvaluator(pts.x, pts.interior_count, pts.pde_weights, pts.boundary_weights, pts.target, widths,
                             head="psi", boundary_order=1, loss=NSLoss(pts.viscosity), device="cuda:0")
    ws, bs = xavier_normal(widths, 0)
    expected = single(flat_parameters(ws, bs).cuda(0)).cpu().numpy()
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    outs = dict(queue.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert np.array_equal(outs[0], outs[1])  # identical bytes on every rank
    rel = np.linalg.norm(outs[0] - expected) / np.linalg.norm(expected)
    assert rel <= 1e-12
    from oracle.evaluate import evaluate
    from tests.cases import close_ratio, rel_norm
    loss, grads = evaluate(pts.x.numpy(), pts.interior_count, pts.pde_weights.numpy(), pts.boundary_weights.numpy(),
                           pts.target.numpy(), [w.numpy() for w in ws], [b.numpy() for b in bs], head="psi",
                           nu=pts.viscosity, boundary_order=1)
    reference = np.concatenate([g.reshape(-1) for g in grads] + [[loss]])
    assert close_ratio(outs[0], reference) <= 1.0
    assert rel_norm(outs[0], reference) <= 1e-10
