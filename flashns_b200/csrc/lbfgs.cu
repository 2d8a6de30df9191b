// Device kernels of the L-BFGS solver (flashns_b200/lbfgs.py): the curvature-pair ring,
// the compact quasi-Newton coefficients, the search direction and the line-search updates.
// All reductions are fixed-order (one block per dot product, fixed tree), so repeated
// solves are bitwise reproducible.
#include <cmath>
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

// ---- device-resident L-BFGS state: pairs in a ring of `slots` = history + 1 physical rows
// (one spare).  state = {k stored pairs, h spare slot, have_pair, 0}; the stored pairs are
// the physical rows (h - k + i) mod slots, i = 0 (oldest) .. k-1 (newest).
enum { kStK = 0, kStH = 1, kStPair = 2 };
enum { kGamma = 0, kF0 = 1, kGd0 = 2, kF = 3, kGd = 4, kK = 5, kT = 6 };

// the new pair s = x - x0, y = g - g0 into the spare slot
__global__ void __launch_bounds__(kVecThreads)
    pair_slot(const double* __restrict__ x, const double* __restrict__ x0, const double* __restrict__ g,
              const double* __restrict__ g0, double* __restrict__ S, double* __restrict__ Y, int64_t stride,
              const int* __restrict__ state, int64_t n) {
  if (!state[kStPair]) return;
  const int64_t r = int64_t(state[kStH]) * stride;
  for (int64_t j = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; j < n; j += int64_t(gridDim.x) * blockDim.x) {
    S[r + j] = x[j] - x0[j];
    Y[r + j] = g[j] - g0[j];
  }
}

// out[b] = (b < slots ? S[b] : Y[b - slots]) . v, v = `vec` or (from_slot) the spare Y row;
// one block per dot product, fixed tree
__global__ void __launch_bounds__(kVecThreads)
    ring_dots(const double* __restrict__ S, const double* __restrict__ Y, int64_t stride, int slots,
              const double* __restrict__ vec, const int* __restrict__ state, int from_slot, double* __restrict__ out,
              int64_t n) {
  __shared__ double red[kVecThreads];
  if (from_slot && !state[kStPair]) return;
  const int b = blockIdx.x;
  const double* row = (b < slots ? S : Y) + int64_t(b < slots ? b : b - slots) * stride;
  const double* v = from_slot ? Y + int64_t(state[kStH]) * stride : vec;
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
  if (threadIdx.x == 0) out[b] = red[0];
}

// keep the new pair if it satisfies the curvature condition s.y > 1e-12 y.y: record its
// products with every slot and advance the ring (the oldest pair drops out when full)
__global__ void commit(const double* __restrict__ dots, double* __restrict__ SY, double* __restrict__ YY, int slots,
                       int history, int* __restrict__ state) {
  if (!state[kStPair]) return;
  const int h = state[kStH];
  const double sy = dots[h], yy = dots[slots + h];
  const bool ok = sy > 1e-12 * fmax(yy, 1e-300) && isfinite(sy) && isfinite(yy);
  if (!ok) return;
  for (int r = threadIdx.x; r < slots; r += blockDim.x) {
    SY[r * slots + h] = dots[r];          // s_r . y_new
    YY[r * slots + h] = dots[slots + r];  // y_r . y_new
    YY[h * slots + r] = dots[slots + r];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    state[kStH] = (h + 1) % slots;
    state[kStK] = state[kStK] + 1 < history ? state[kStK] + 1 : history;
  }
}

// Coefficients of the compact representation (Byrd, Nocedal, Schnabel 1994, Thm 2.2) with
// H0 = gamma I:  u = R^-1 p1,  cs = R^-T((D + gamma YY) u - gamma p2),  cy = -gamma u,
// R = upper triangle of S^T Y (oldest first), D its diagonal, p1 = S^T g, p2 = Y^T g.
// One block: R is staged in shared memory ([k][k], dynamic); the two triangular solves
// run on warp 0 (warp-reduced row sums), the matrix-vector product on all threads.
constexpr int kMaxHistory = 128;
constexpr int kCoefThreads = 256;
__global__ void __launch_bounds__(kCoefThreads)
    coefficients(const double* __restrict__ SY, const double* __restrict__ YY, const double* __restrict__ dots,
                 int slots, const int* __restrict__ state, double* __restrict__ coef, int* __restrict__ order,
                 double* __restrict__ scal) {
  extern __shared__ double Rs[];  // [k][k]
  __shared__ int idx[kMaxHistory];
  __shared__ double u[kMaxHistory], w[kMaxHistory], cs[kMaxHistory];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int k = state[kStK], h = state[kStH];
  for (int i = tid; i < k; i += kCoefThreads) {
    idx[i] = ((h - k + i) % slots + slots) % slots;
    order[i] = idx[i];
  }
  if (k == 0) {
    if (tid == 0) { scal[kGamma] = 1.0; scal[kK] = 0.0; }
    return;
  }
  __syncthreads();
  for (int e = tid; e < k * k; e += kCoefThreads) {
    const int i = e / k, j = e % k;
    Rs[e] = j >= i ? SY[idx[i] * slots + idx[j]] : 0.0;
  }
  __syncthreads();
  const int newest = idx[k - 1];
  const double gamma = SY[newest * slots + newest] / YY[newest * slots + newest];
  if (warp == 0) {  // back substitution: R u = p1
    for (int i = k - 1; i >= 0; --i) {
      double part = 0.0;
      for (int j = i + 1 + lane; j < k; j += 32) part += Rs[i * k + j] * u[j];
      for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
      if (lane == 0) u[i] = (dots[idx[i]] - part) / Rs[i * k + i];
      __syncwarp();
    }
  }
  __syncthreads();
  for (int i = tid; i < k; i += kCoefThreads) {  // w = (D + gamma YY) u - gamma p2
    double sum = 0.0;
    for (int j = 0; j < k; ++j) sum += YY[idx[i] * slots + idx[j]] * u[j];
    w[i] = Rs[i * k + i] * u[i] + gamma * sum - gamma * dots[slots + idx[i]];
  }
  __syncthreads();
  if (warp == 0) {  // forward substitution: R^T cs = w
    for (int i = 0; i < k; ++i) {
      double part = 0.0;
      for (int j = lane; j < i; j += 32) part += Rs[j * k + i] * cs[j];
      for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
      if (lane == 0) cs[i] = (w[i] - part) / Rs[i * k + i];
      __syncwarp();
    }
  }
  __syncthreads();
  for (int i = tid; i < k; i += kCoefThreads) {
    coef[i] = cs[i];
    coef[kMaxHistory + i] = -gamma * u[i];
  }
  if (tid == 0) { scal[kGamma] = gamma; scal[kK] = double(k); }
}

// d = -(gamma g + sum_i cs[i] S[order[i]] + cy[i] Y[order[i]]), k and gamma from the device
__global__ void __launch_bounds__(kVecThreads)
    direction(const double* __restrict__ S, const double* __restrict__ Y, int64_t stride, const int* __restrict__ order,
              const int* __restrict__ state, const double* __restrict__ coef, const double* __restrict__ g,
              const double* __restrict__ scal, double* __restrict__ d, int64_t n) {
  const int k = state[kStK];
  const double gamma = scal[kGamma];
  for (int64_t j = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; j < n; j += int64_t(gridDim.x) * blockDim.x) {
    double acc = gamma * g[j];
    for (int i = 0; i < k; ++i) {
      const int64_t r = int64_t(order[i]) * stride;
      acc += coef[i] * S[r + j] + coef[kMaxHistory + i] * Y[r + j];
    }
    d[j] = -acc;
  }
}

// x0 = x, g0 = g, scal[F0] = f
__global__ void __launch_bounds__(kVecThreads)
    save_point(const double* __restrict__ x, const double* __restrict__ g, const double* __restrict__ f,
               double* __restrict__ x0, double* __restrict__ g0, double* __restrict__ scal, int64_t n) {
  for (int64_t j = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; j < n; j += int64_t(gridDim.x) * blockDim.x) {
    x0[j] = x[j];
    g0[j] = g[j];
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) scal[kF0] = *f;
}

// x = x0 + t d with the step t = scal[kT] read on the device (graph-replayable trials)
__global__ void __launch_bounds__(kVecThreads)
    step_point(const double* __restrict__ x0, const double* __restrict__ scal, const double* __restrict__ d,
               double* __restrict__ x, int64_t n) {
  const double t = scal[kT];
  for (int64_t j = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; j < n; j += int64_t(gridDim.x) * blockDim.x)
    x[j] = x0[j] + t * d[j];
}

// Adam (Kingma and Ba 2015) with the bias corrections passed in, eps added to the
// corrected sqrt(v) (as experiments/pinn_solver/backends.py:216-240):
//   m = b1 m + (1-b1) g,  v = b2 v + (1-b2) g^2,  x -= lr (m/c1) / (sqrt(v/c2) + eps)
__global__ void __launch_bounds__(kVecThreads)
    adam_update(double* __restrict__ x, const double* __restrict__ g, double* __restrict__ m, double* __restrict__ v,
                int64_t n, double lr, double b1, double b2, double eps, double c1, double c2) {
  for (int64_t j = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; j < n; j += int64_t(gridDim.x) * blockDim.x) {
    const double gj = g[j];
    const double mj = b1 * m[j] + (1.0 - b1) * gj;
    const double vj = b2 * v[j] + (1.0 - b2) * gj * gj;
    m[j] = mj;
    v[j] = vj;
    x[j] -= lr * (mj / c1) / (sqrt(vj / c2) + eps);
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

int flashns_b200_lbfgs_pair_slot(const double* x, const double* x0, const double* g, const double* g0, double* S,
                                 double* Y, int64_t stride, const int* state, int64_t n, cudaStream_t stream) {
  if (n < 1 || stride < n || !x || !x0 || !g || !g0 || !S || !Y || !state) return int(cudaErrorInvalidValue);
  pair_slot<<<vec_grid(n), kVecThreads, 0, stream>>>(x, x0, g, g0, S, Y, stride, state, n);
  return int(cudaGetLastError());
}

int flashns_b200_lbfgs_ring_dots(const double* S, const double* Y, int64_t stride, int slots, const double* v,
                                 const int* state, int from_slot, double* out, int64_t n, cudaStream_t stream) {
  if (n < 1 || stride < n || slots < 2 || slots > kMaxHistory + 1 || !S || !Y || !state || !out ||
      (!from_slot && !v))
    return int(cudaErrorInvalidValue);
  ring_dots<<<unsigned(2 * slots), kVecThreads, 0, stream>>>(S, Y, stride, slots, v, state, from_slot, out, n);
  return int(cudaGetLastError());
}

int flashns_b200_lbfgs_commit(const double* dots, double* SY, double* YY, int slots, int* state, cudaStream_t stream) {
  if (slots < 2 || slots > kMaxHistory + 1 || !dots || !SY || !YY || !state) return int(cudaErrorInvalidValue);
  commit<<<1, 128, 0, stream>>>(dots, SY, YY, slots, slots - 1, state);
  return int(cudaGetLastError());
}

int flashns_b200_lbfgs_coefficients(const double* SY, const double* YY, const double* dots, int slots,
                                    const int* state, double* coef, int* order, double* scal, cudaStream_t stream) {
  if (slots < 2 || slots > kMaxHistory + 1 || !SY || !YY || !dots || !state || !coef || !order || !scal)
    return int(cudaErrorInvalidValue);
  const size_t smem = sizeof(double) * size_t(slots - 1) * size_t(slots - 1);
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(coefficients, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return int(e);
  }
  coefficients<<<1, kCoefThreads, smem, stream>>>(SY, YY, dots, slots, state, coef, order, scal);
  return int(cudaGetLastError());
}

int flashns_b200_lbfgs_direction(const double* S, const double* Y, int64_t stride, const int* order, const int* state,
                                 const double* coef, const double* g, const double* scal, double* d, int64_t n,
                                 cudaStream_t stream) {
  if (n < 1 || stride < n || !S || !Y || !order || !state || !coef || !g || !scal || !d)
    return int(cudaErrorInvalidValue);
  direction<<<vec_grid(n), kVecThreads, 0, stream>>>(S, Y, stride, order, state, coef, g, scal, d, n);
  return int(cudaGetLastError());
}

int flashns_b200_lbfgs_save(const double* x, const double* g, const double* f, double* x0, double* g0, double* scal,
                            int64_t n, cudaStream_t stream) {
  if (n < 1 || !x || !g || !f || !x0 || !g0 || !scal) return int(cudaErrorInvalidValue);
  save_point<<<vec_grid(n), kVecThreads, 0, stream>>>(x, g, f, x0, g0, scal, n);
  return int(cudaGetLastError());
}

int flashns_b200_lbfgs_step_point(const double* x0, const double* scal, const double* d, double* x, int64_t n,
                                  cudaStream_t stream) {
  if (n < 1 || !x0 || !scal || !d || !x) return int(cudaErrorInvalidValue);
  step_point<<<vec_grid(n), kVecThreads, 0, stream>>>(x0, scal, d, x, n);
  return int(cudaGetLastError());
}

int flashns_b200_adam_step(double* x, const double* g, double* m, double* v, int64_t n, double lr, double beta1,
                           double beta2, double eps, int64_t step, cudaStream_t stream) {
  if (n < 1 || step < 1 || !x || !g || !m || !v || !(lr >= 0) || !(beta1 >= 0 && beta1 < 1) ||
      !(beta2 >= 0 && beta2 < 1) || !(eps > 0))
    return int(cudaErrorInvalidValue);
  const double c1 = 1.0 - pow(beta1, double(step)), c2 = 1.0 - pow(beta2, double(step));
  adam_update<<<vec_grid(n), kVecThreads, 0, stream>>>(x, g, m, v, n, lr, beta1, beta2, eps, c1, c2);
  return int(cudaGetLastError());
}

}  // extern "C"
