// Data preparation on the device: seeded collocation points and the packed coordinate
// rows of a point set.
//
// * Scrambled Sobol points, bit-identical to torch.quasirandom.SobolEngine(dim,
//   scramble=True, seed).draw(), which the reference solver samples with
//   (experiments/pinn_solver/problem.py:68-99).  The engine's scrambled direction numbers
//   and digital shift are per-seed constants (dim x 30 words) that the host takes from the
//   engine; point k is then independent of every other point: the Gray-code recurrence
//   the engine runs point after point equals shift ^ XOR of the direction numbers selected
//   by the bits of gray(k) = k ^ (k >> 1), so one thread writes one coordinate.
// * Counter-based uniforms: Philox4x64-10 (Salmon, Moraes, Dror and Shaw, "Parallel
//   random numbers: as easy as 1, 2, 3", SC 2011), word j of the key's stream taken from
//   counter block j / 4 + 1, lane j % 4, and mapped to [0, 1) as (word >> 11) * 2^-53.
//   That is the stream numpy.random.Generator(numpy.random.Philox(key)).random() draws.
// * PackedLayout.coordinates (src/flashns/jet_packed.py:43-53): the input jets of the
//   coordinates, full points as Q rows (value row, then one unit row per axis) and
//   value-only points as one row.
//
// Points map to the domain as lo + span * u with the product and the sum rounded
// separately (no FMA contraction), so the coordinates match the host's tensor arithmetic
// bit for bit.
#include <cstdint>

#include "common.cuh"
#include "flashns_b200.h"

namespace flashns_b200 {
namespace {

constexpr int kSobolBits = 30;  // torch.quasirandom.SobolEngine.MAXBIT
constexpr int kMaxSampleDim = 8;
constexpr int kSampleThreads = 256;

// Philox4x64 round multipliers and key increments (the published constants)
constexpr uint64_t kPhiloxM0 = 0xD2E7470EE14C6C93ull, kPhiloxM1 = 0xCA5A826395121157ull;
constexpr uint64_t kPhiloxW0 = 0x9E3779B97F4A7C15ull, kPhiloxW1 = 0xBB67AE8584CAA73Bull;

struct SobolTable {
  uint32_t v[kMaxSampleDim][kSobolBits];  // scrambled direction numbers per coordinate
  uint32_t shift[kMaxSampleDim];          // digital shift (the engine's first point)
};

// out = (lo ? lo : 0) + (span ? span * u : u); flags say which of lo / span apply
struct DomainMap {
  double lo[kMaxSampleDim], span[kMaxSampleDim];
  int has_lo, has_span;
};

__device__ __forceinline__ double to_domain(const DomainMap& m, int d, double u) {
  const double s = m.has_span ? __dmul_rn(m.span[d], u) : u;
  return m.has_lo ? __dadd_rn(m.lo[d], s) : s;
}

__device__ __forceinline__ int64_t grid_stride() { return int64_t(gridDim.x) * blockDim.x; }

__global__ void __launch_bounds__(kSampleThreads)
    sobol_points(const __grid_constant__ SobolTable tab, const __grid_constant__ DomainMap map, int dim,
                 int64_t first, int64_t n, double* __restrict__ out, int64_t ld) {
  for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < n * dim; e += grid_stride()) {
    const int64_t i = e / dim;
    const int d = int(e % dim);
    const uint64_t k = uint64_t(first + i);
    double u;
    if (k == 0) {
      // the engine's first point is its shift divided by 2^30 in single precision
      u = double(__uint2float_rn(tab.shift[d]) * 0x1p-30f);
    } else {
      const uint64_t g = k ^ (k >> 1);
      uint32_t q = tab.shift[d];
#pragma unroll
      for (int b = 0; b < kSobolBits; ++b)
        if ((g >> b) & 1u) q ^= tab.v[d][b];
      u = double(q) * 0x1p-30;
    }
    out[i * ld + d] = to_domain(map, d, u);
  }
}

__device__ __forceinline__ void philox4x64_10(uint64_t c[4], uint64_t k0, uint64_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint64_t hi0 = __umul64hi(kPhiloxM0, c[0]), lo0 = kPhiloxM0 * c[0];
    const uint64_t hi1 = __umul64hi(kPhiloxM1, c[2]), lo1 = kPhiloxM1 * c[2];
    c[0] = hi1 ^ c[1] ^ k0;
    c[1] = lo1;
    c[2] = hi0 ^ c[3] ^ k1;
    c[3] = lo0;
    k0 += kPhiloxW0;
    k1 += kPhiloxW1;
  }
}

// one thread per counter block: the block's four words are the stream's words
// 4 * blk .. 4 * blk + 3; those inside [w0, w1) become coordinates
__global__ void __launch_bounds__(kSampleThreads)
    philox_points(uint64_t key0, uint64_t key1, const __grid_constant__ DomainMap map, int dim, int64_t first,
                  int64_t n, double* __restrict__ out, int64_t ld) {
  const int64_t w0 = first * dim, w1 = (first + n) * dim;
  const int64_t b0 = w0 / 4, nblocks = (w1 - 1) / 4 - b0 + 1;
  for (int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; t < nblocks; t += grid_stride()) {
    const int64_t blk = b0 + t;
    uint64_t c[4] = {uint64_t(blk) + 1u, 0u, 0u, 0u};
    philox4x64_10(c, key0, key1);
#pragma unroll
    for (int lane = 0; lane < 4; ++lane) {
      const int64_t j = 4 * blk + lane;
      if (j < w0 || j >= w1) continue;
      const int64_t i = j / dim - first;
      const int d = int(j % dim);
      out[i * ld + d] = to_domain(map, d, double(c[lane] >> 11) * 0x1p-53);
    }
  }
}

// packed input jets: rows [full_points x Q ; value_points], Q = C(dim + 3, 3); the unit
// row of axis a is coefficient dim - a (basis sorted by total order, then multi-index)
__global__ void __launch_bounds__(kSampleThreads)
    pack_coordinates(const double* __restrict__ x, int64_t full_points, int64_t value_points, int dim, int q,
                     double* __restrict__ out) {
  const int64_t full_rows = full_points * q, total = (full_rows + value_points) * dim;
  for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < total; e += grid_stride()) {
    const int64_t r = e / dim;
    const int c = int(e % dim);
    double v;
    if (r < full_rows) {
      const int64_t p = r / q;
      const int s = int(r % q);
      v = s == 0 ? x[p * dim + c] : (s == dim - c ? 1.0 : 0.0);
    } else {
      v = x[(full_points + (r - full_rows)) * dim + c];
    }
    out[e] = v;
  }
}

unsigned sample_grid(int64_t work) {
  const int64_t blocks = (work + kSampleThreads - 1) / kSampleThreads;
  return unsigned(blocks < 148 * 16 ? (blocks > 0 ? blocks : 1) : 148 * 16);
}

bool domain_map(int dim, const double* lo, const double* span, DomainMap& m) {
  m = DomainMap{};
  m.has_lo = lo != nullptr;
  m.has_span = span != nullptr;
  for (int d = 0; d < dim; ++d) {
    m.lo[d] = lo ? lo[d] : 0.0;
    m.span[d] = span ? span[d] : 1.0;
  }
  return true;
}

}  // namespace
}  // namespace flashns_b200

using namespace flashns_b200;

extern "C" {

int flashns_b200_sobol_points(const int64_t* directions, const int64_t* shift, int dim, int64_t first, int64_t n,
                              const double* lo, const double* span, double* out, int64_t ld, cudaStream_t stream) {
  if (!directions || !shift || dim < 1 || dim > kMaxSampleDim || first < 0 || n < 0 || ld < dim ||
      first > (int64_t(1) << kSobolBits) - n || (n > 0 && !out))
    return int(cudaErrorInvalidValue);
  SobolTable tab{};
  for (int d = 0; d < dim; ++d) {
    if (shift[d] < 0 || shift[d] >= (int64_t(1) << kSobolBits)) return int(cudaErrorInvalidValue);
    tab.shift[d] = uint32_t(shift[d]);
    for (int b = 0; b < kSobolBits; ++b) {
      const int64_t v = directions[int64_t(d) * kSobolBits + b];
      if (v < 0 || v >= (int64_t(1) << kSobolBits)) return int(cudaErrorInvalidValue);
      tab.v[d][b] = uint32_t(v);
    }
  }
  if (n == 0) return int(cudaSuccess);
  DomainMap map;
  domain_map(dim, lo, span, map);
  sobol_points<<<sample_grid(n * dim), kSampleThreads, 0, stream>>>(tab, map, dim, first, n, out, ld);
  return int(cudaGetLastError());
}

int flashns_b200_philox_points(uint64_t key0, uint64_t key1, int dim, int64_t first, int64_t n, const double* lo,
                               const double* span, double* out, int64_t ld, cudaStream_t stream) {
  if (dim < 1 || dim > kMaxSampleDim || first < 0 || n < 0 || ld < dim || (n > 0 && !out) ||
      first > (int64_t(1) << 58) / dim - n)
    return int(cudaErrorInvalidValue);
  if (n == 0) return int(cudaSuccess);
  DomainMap map;
  domain_map(dim, lo, span, map);
  philox_points<<<sample_grid(n * dim / 4 + 2), kSampleThreads, 0, stream>>>(key0, key1, map, dim, first, n, out,
                                                                               ld);
  return int(cudaGetLastError());
}

int flashns_b200_pack_coordinates(const double* x, int64_t full_points, int64_t value_points, int dim, double* out,
                                  cudaStream_t stream) {
  if (dim < 1 || dim > kMaxSampleDim || full_points < 0 || value_points < 0) return int(cudaErrorInvalidValue);
  const int q = (dim + 1) * (dim + 2) * (dim + 3) / 6;
  const int64_t total = (full_points * q + value_points) * dim;
  if (total == 0) return int(cudaSuccess);
  if (!x || !out) return int(cudaErrorInvalidValue);
  pack_coordinates<<<sample_grid(total), kSampleThreads, 0, stream>>>(x, full_points, value_points, dim, q, out);
  return int(cudaGetLastError());
}

}  // extern "C"
