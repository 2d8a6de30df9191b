// Device vector kernels of the L-BFGS solver (flashns_b200/lbfgs.py): the history
// products of the compact quasi-Newton representation and the line-search updates.
// All reductions are fixed-order (one block per dot product, fixed tree), so repeated
// solves are bitwise reproducible.
#include <cstdint>

#include "common.cuh"
#include "flashns_b200.h"

namespace flashns_b200 {
namespace {

constexpr int kVecThreads = 256;

// out[r] = rows[r] . v for r < k (rows: [k][n] with row stride `stride`), one block per row
__global__ void __launch_bounds__(kVecThreads)
    row_dots(const double* __restrict__ rows, int64_t stride, const double* __restrict__ v, double* __restrict__ out,
             int64_t n) {
  __shared__ double red[kVecThreads];
  const double* row = rows + int64_t(blockIdx.x) * stride;
  double acc[4] = {0.0, 0.0, 0.0, 0.0};
  int64_t j = threadIdx.x;
  for (; j + 3 * kVecThreads < n; j += 4 * kVecThreads) {
#pragma unroll
    for (int u = 0; u < 4; ++u) acc[u] += row[j + u * kVecThreads] * v[j + u * kVecThreads];
  }
  for (int u = 0; j < n; j += kVecThreads, ++u) acc[u] += row[j] * v[j];
  red[threadIdx.x] = (acc[0] + acc[1]) + (acc[2] + acc[3]);
  __syncthreads();
  for (int s = kVecThreads / 2; s > 0; s >>= 1) {
    if (threadIdx.x < s) red[threadIdx.x] += red[threadIdx.x + s];
    __syncthreads();
  }
  if (threadIdx.x == 0) out[blockIdx.x] = red[0];
}

// d = -(gamma g + sum_i cs[i] S[i] + sum_i cy[i] Y[i])
__global__ void __launch_bounds__(kVecThreads)
    combine(const double* __restrict__ S, const double* __restrict__ Y, int64_t stride, const int* __restrict__ order,
            int k, const double* __restrict__ cs, const double* __restrict__ cy, const double* __restrict__ g,
            double gamma, double* __restrict__ d, int64_t n) {
  for (int64_t j = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; j < n; j += int64_t(gridDim.x) * blockDim.x) {
    double acc = gamma * g[j];
    for (int i = 0; i < k; ++i) {
      const int64_t r = int64_t(order[i]) * stride;
      acc += cs[i] * S[r + j] + cy[i] * Y[r + j];
    }
    d[j] = -acc;
  }
}

// x = x0 + t d
__global__ void __launch_bounds__(kVecThreads)
    axpy(const double* __restrict__ x0, double t, const double* __restrict__ d, double* __restrict__ x, int64_t n) {
  for (int64_t j = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; j < n; j += int64_t(gridDim.x) * blockDim.x)
    x[j] = x0[j] + t * d[j];
}

// s = x - x0, y = g - g0 (the new curvature pair)
__global__ void __launch_bounds__(kVecThreads)
    pair(const double* __restrict__ x, const double* __restrict__ x0, const double* __restrict__ g,
         const double* __restrict__ g0, double* __restrict__ s, double* __restrict__ y, int64_t n) {
  for (int64_t j = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; j < n; j += int64_t(gridDim.x) * blockDim.x) {
    s[j] = x[j] - x0[j];
    y[j] = g[j] - g0[j];
  }
}

unsigned vec_grid(int64_t n) {
  const int64_t b = (n + kVecThreads - 1) / kVecThreads;
  return unsigned(b < 148 * 8 ? (b > 0 ? b : 1) : 148 * 8);
}

}  // namespace
}  // namespace flashns_b200

using namespace flashns_b200;

extern "C" {

int flashns_b200_row_dots(const double* rows, int64_t stride, int k, const double* v, double* out, int64_t n,
                          cudaStream_t stream) {
  if (k < 0 || n < 0 || stride < n) return int(cudaErrorInvalidValue);
  if (k == 0) return int(cudaSuccess);
  if (!rows || !v || !out) return int(cudaErrorInvalidValue);
  row_dots<<<unsigned(k), kVecThreads, 0, stream>>>(rows, stride, v, out, n);
  return int(cudaGetLastError());
}

int flashns_b200_lbfgs_combine(const double* S, const double* Y, int64_t stride, const int* order, int k,
                               const double* cs, const double* cy, const double* g, double gamma, double* d, int64_t n,
                               cudaStream_t stream) {
  if (k < 0 || n < 0 || stride < n || !g || !d || (k && (!S || !Y || !order || !cs || !cy)))
    return int(cudaErrorInvalidValue);
  if (n == 0) return int(cudaSuccess);
  combine<<<vec_grid(n), kVecThreads, 0, stream>>>(S, Y, stride, order, k, cs, cy, g, gamma, d, n);
  return int(cudaGetLastError());
}

int flashns_b200_axpy(const double* x0, double t, const double* d, double* x, int64_t n, cudaStream_t stream) {
  if (n < 0 || (n && (!x0 || !d || !x))) return int(cudaErrorInvalidValue);
  if (n == 0) return int(cudaSuccess);
  axpy<<<vec_grid(n), kVecThreads, 0, stream>>>(x0, t, d, x, n);
  return int(cudaGetLastError());
}

int flashns_b200_lbfgs_pair(const double* x, const double* x0, const double* g, const double* g0, double* s, double* y,
                            int64_t n, cudaStream_t stream) {
  if (n < 0 || (n && (!x || !x0 || !g || !g0 || !s || !y))) return int(cudaErrorInvalidValue);
  if (n == 0) return int(cudaSuccess);
  pair<<<vec_grid(n), kVecThreads, 0, stream>>>(x, x0, g, g0, s, y, n);
  return int(cudaGetLastError());
}

}  // extern "C"
