"""Timed CPU baseline: the oracle port of ``PackedPINN`` on all host cores.

TEST AND CPU-BASELINE INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): used by the
``cpu_baseline`` and ``--impl reference`` legs of ``bench.py``.  Points are
independent, so a sample of the point set is split over a ``spawn`` process pool
(one single-threaded NumPy worker per core); the chunk losses and gradients are
summed, as a data-parallel CPU evaluation would.
"""

import multiprocessing as mp
import os
import statistics
import time

_STATE = {}


def _init(problem):
    _STATE.update(problem)


def _work(task):
    from oracle.evaluate import evaluate
    i0, i1, b0, b1 = task
    s = _STATE
    import numpy as np
    ni = s["ni"]
    xs = np.concatenate((s["x"][i0:i1], s["x"][ni + b0:ni + b1]))
    loss, grads = evaluate(xs, i1 - i0, s["pw"][i0:i1], s["bw"][b0:b1], s["target"][b0:b1], s["ws"], s["bs"],
                           **s["options"])
    return loss, grads


class CpuPool:
    def __init__(self, problem, workers):
        self.problem = problem
        self.workers = workers
        saved = {k: os.environ.get(k) for k in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS")}
        for k in saved:
            os.environ[k] = "1"
        try:
            self.pool = mp.get_context("spawn").Pool(workers, initializer=_init, initargs=(problem,))
        finally:
            for k, v in saved.items():
                if v is None:
                    os.environ.pop(k, None)
                else:
                    os.environ[k] = v

    def evaluate_fraction(self, part, parts):
        """Evaluate point chunk ``part`` of ``parts`` split over all workers; return (loss, grads)."""
        ni = self.problem["ni"]
        nb = len(self.problem["x"]) - ni
        i0, i1 = ni * part // parts, ni * (part + 1) // parts
        b0, b1 = nb * part // parts, nb * (part + 1) // parts
        w = self.workers
        tasks = [(i0 + (i1 - i0) * k // w, i0 + (i1 - i0) * (k + 1) // w,
                  b0 + (b1 - b0) * k // w, b0 + (b1 - b0) * (k + 1) // w) for k in range(w)]
        results = self.pool.map(_work, tasks)
        loss = sum(r[0] for r in results)
        grads = [sum(r[1][i] for r in results) for i in range(len(results[0][1]))]
        return loss, grads

    def close(self):
        self.pool.terminate()
        self.pool.join()


def timed_rate(problem, workers, steps, warmup, parts=8):
    """CPU evaluations/s of the full point set from ``steps`` timed chunk evaluations."""
    pool = CpuPool(problem, workers)
    try:
        for k in range(warmup):
            pool.evaluate_fraction(k % parts, parts)
        times = []
        for k in range(steps):
            t0 = time.perf_counter()
            pool.evaluate_fraction(k % parts, parts)
            times.append(time.perf_counter() - t0)
    finally:
        pool.close()
    med = statistics.median(times)
    return (1.0 / parts) / med, med
