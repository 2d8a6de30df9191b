"""Restatements of the device data-preparation kernels (``flashns_b200/csrc/sampling.cu``).

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

* ``sobol_points``: point k of a scrambled Sobol engine as shift ^ XOR of the direction
  numbers picked by the bits of gray(k), in closed form instead of the engine's point by
  point Gray-code update.  The reference solver samples with
  ``torch.quasirandom.SobolEngine(dim, scramble=True, seed)``
  (experiments/pinn_solver/problem.py:68-99); the tests pin this restatement to that
  engine, including its first point, which the engine divides in single precision.
* ``philox4x64_10`` / ``philox_uniform``: Philox4x64-10 (Salmon, Moraes, Dror and Shaw,
  SC 2011) in Python integers; pinned to ``numpy.random.Philox``'s raw words and to
  ``numpy.random.Generator.random()``.
* ``packed_coordinates``: ``PackedLayout.coordinates`` (src/flashns/jet_packed.py:43-53)
  in NumPy.
"""

from math import comb

import numpy as np

SOBOL_BITS = 30
MASK64 = (1 << 64) - 1
PHILOX_M = (0xD2E7470EE14C6C93, 0xCA5A826395121157)
PHILOX_W = (0x9E3779B97F4A7C15, 0xBB67AE8584CAA73B)


def sobol_points(directions, shift, first, n):
    """[n, dim] unit points first .. first+n-1 from scrambled direction numbers
    ``directions`` [dim][30] and digital ``shift`` [dim]."""
    directions = np.asarray(directions, dtype=np.int64)
    shift = np.asarray(shift, dtype=np.int64)
    k = np.arange(first, first + n, dtype=np.int64)
    g = k ^ (k >> 1)
    q = np.repeat(shift[None, :], n, 0)
    for b in range(SOBOL_BITS):
        picked = ((g >> b) & 1).astype(bool)
        q[picked] ^= directions[:, b][None, :]
    out = q.astype(np.float64) * 2.0 ** -SOBOL_BITS
    if first == 0 and n:
        out[0] = (shift.astype(np.float32) / np.float32(2 ** SOBOL_BITS)).astype(np.float64)
    return out


def philox4x64_10(counter, key):
    """Ten Philox4x64 rounds of a 4-word counter under a 2-word key (Python ints)."""
    x = [int(c) & MASK64 for c in counter]
    k0, k1 = (int(k) & MASK64 for k in key)
    for _ in range(10):
        p0, p1 = PHILOX_M[0] * x[0], PHILOX_M[1] * x[2]
        x = [(p1 >> 64) ^ x[1] ^ k0, p1 & MASK64, (p0 >> 64) ^ x[3] ^ k1, p0 & MASK64]
        k0, k1 = (k0 + PHILOX_W[0]) & MASK64, (k1 + PHILOX_W[1]) & MASK64
    return x


def philox_words(key0, key1, first_word, count):
    """Words first_word .. first_word+count-1 of a key's stream: word j is lane j % 4 of
    counter block j // 4 + 1."""
    out, cache = [], {}
    for j in range(first_word, first_word + count):
        blk = j // 4
        if blk not in cache:
            cache = {blk: philox4x64_10((blk + 1, 0, 0, 0), (key0, key1))}
        out.append(cache[blk][j % 4])
    return out


def philox_uniform(key0, key1, dim, first, n):
    """[n, dim] doubles (word >> 11) * 2^-53, point first .. first+n-1."""
    words = philox_words(key0, key1, first * dim, n * dim)
    return np.array([(w >> 11) * 2.0 ** -53 for w in words], dtype=np.float64).reshape(n, dim)


def packed_coordinates(x, full_points, dim):
    """Input jets of the coordinates: full points as Q rows (value, then a 1 in the unit row
    dim - a of each axis a), value-only points as one row."""
    x = np.asarray(x, dtype=np.float64)
    q = comb(dim + 3, 3)
    full = np.zeros((full_points, q, dim))
    full[:, 0, :] = x[:full_points]
    for a in range(dim):
        full[:, dim - a, a] = 1.0
    return np.concatenate((full.reshape(full_points * q, dim), x[full_points:]))
