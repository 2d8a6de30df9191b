"""CPU (gloo, world size 2): the data-parallel reduction gives every rank the
single-process loss and gradient, and a non-finite value on one rank reaches all."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_factory(widths, params, poison_rank=None):
    """Local evaluator on the CPU oracle (test stand-in for the CUDA evaluator)."""
    from oracle.evaluate import evaluate

    def factory(shard):
        def run(flat, out=None):
            n = len(widths) - 1
            sizes = [i * o for i, o in zip(widths, widths[1:])]
            f = flat.numpy()
            ws, off = [], 0
            for (i, o), sz in zip(zip(widths, widths[1:]), sizes):
                ws.append(f[off:off + sz].reshape(o, i)); off += sz
            bs = []
            for o in widths[1:]:
                bs.append(f[off:off + o]); off += o
            loss, grads = evaluate(shard.x.numpy(), shard.interior_count, shard.pde_weights.numpy(),
                                   shard.boundary_weights.numpy(), shard.target.numpy(), ws, bs, head="psi",
                                   nu=shard.viscosity, boundary_order=1)
            res = torch.tensor(np.concatenate([g.reshape(-1) for g in grads] + [[loss]]))
            if poison_rank is not None and dist.get_rank() == poison_rank:
                res[3] = float("nan")
            return res
        return run
    return factory


def _worker(rank, world, port, widths, params, expected, poison, queue, points=(37, 13)):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from flashns_b200.distributed import DistributedEvaluator
        from flashns_b200.problems import kovasznay
        pts = kovasznay(*points, seed=4)
        ev = DistributedEvaluator(pts, widths, local_factory=_oracle_factory(widths, params, poison))
        out = ev(torch.tensor(params))
        if poison is None:
            err = float(np.max(np.abs(out.numpy() - expected) / (2e-12 + 2e-11 * np.abs(expected))))
            queue.put((rank, "ok", err, DistributedEvaluator.finite(out)))
        else:
            queue.put((rank, "poison", 0.0, DistributedEvaluator.finite(out)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("poison,world,points", [(None, 2, (37, 13)), (1, 2, (37, 13)), (None, 3, (2, 1)),
                                                 (None, 3, (17, 5))])
def test_rank_reduction_matches_single_process(poison, world, points):
    """World 2, with and without a NaN injected on rank 1; world 3 with an entirely empty
    shard on rank 0 (2 + 1 points) and with uneven shards (17 + 5 points), as the
    reference's experiments/cuda_jet_v5/distributed.py:431-442 exercises."""
    from flashns_b200.evaluator import flat_parameters, xavier_normal
    from flashns_b200.problems import kovasznay
    from oracle.evaluate import evaluate
    widths = [2, 12, 10, 2]
    ws, bs = xavier_normal(widths, 0)
    params = flat_parameters(ws, bs).numpy()
    pts = kovasznay(*points, seed=4)
    loss, grads = evaluate(pts.x.numpy(), pts.interior_count, pts.pde_weights.numpy(), pts.boundary_weights.numpy(),
                           pts.target.numpy(), [w.numpy() for w in ws], [b.numpy() for b in bs], head="psi",
                           nu=pts.viscosity, boundary_order=1)
    expected = np.concatenate([g.reshape(-1) for g in grads] + [[loss]])
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, widths, params, expected, poison, queue, points))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [queue.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, kind, err, finite in results:
        if poison is None:
            assert err <= 1.0 and finite
        else:
            assert not finite  # every rank sees the poisoned value


def test_shards_partition_points_and_weights():
    from flashns_b200.problems import kovasznay
    pts = kovasznay(101, 37, seed=2)
    for world in (1, 2, 3, 8):
        shards = [pts.shard(world, r) for r in range(world)]
        assert sum(s.interior_count for s in shards) == 101
        assert sum(len(s.x) for s in shards) == 138
        assert abs(sum(float(s.pde_weights.sum()) for s in shards) - float(pts.pde_weights.sum())) < 1e-14
        xs = torch.cat([s.x[:s.interior_count] for s in shards])
        assert torch.equal(xs, pts.x[:101])


def _leaving_worker(rank, world, port, widths, params, queue):
    """Rank 1 dies between evaluations without a word to the group; rank 0's next
    evaluation must end with an error (peer gone or the group's timeout), not hang."""
    import time
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    from flashns_b200.distributed import DistributedEvaluator
    from flashns_b200.problems import kovasznay
    ev = DistributedEvaluator(kovasznay(37, 13, seed=4), widths, local_factory=_oracle_factory(widths, params))
    ev(torch.tensor(params))  # one evaluation together
    if rank == 1:
        queue.put((rank, "left", 0.0))
        queue.close()
        queue.join_thread()
        os._exit(3)
    t0 = time.monotonic()
    try:
        ev(torch.tensor(params))
        outcome = "no error"
    except Exception:  # noqa: BLE001 -- any error of the broken collective is the expected outcome
        outcome = "error"
    queue.put((rank, outcome, time.monotonic() - t0))
    queue.close()
    queue.join_thread()
    os._exit(0)  # the group is broken: skip its teardown


def test_a_rank_that_leaves_ends_the_others_evaluation_with_an_error():
    from flashns_b200.evaluator import flat_parameters, xavier_normal
    widths = [2, 8, 2]
    params = flat_parameters(*xavier_normal(widths, 0)).numpy()
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaving_worker, args=(r, 2, port, widths, params, queue)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        results = dict((r, (kind, secs)) for r, kind, secs in (queue.get(timeout=120) for _ in procs))
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    assert results[1][0] == "left" and procs[1].exitcode == 3
    kind, secs = results[0]
    assert kind == "error" and secs < 60 and procs[0].exitcode == 0
