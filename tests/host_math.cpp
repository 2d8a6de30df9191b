// Host build of the device arithmetic the kernels use -- the generated stable-tanh jets,
// their VJPs and the residual seeds (flashns_b200/csrc/jets_generated.cuh,
// residual_generated.cuh) -- compiled by g++ so the CPU tests can check the product's own
// formulas against the oracle without a GPU (the pattern of the reference's
// experiments/pinn_v8/coordinate_wgrad_host.py).  Test infrastructure only.
#include <cmath>

#define __device__
#define __forceinline__ inline
using std::copysign;
using std::exp;
using std::fabs;

#include "jets_generated.cuh"
#include "residual_generated.cuh"

using namespace flashns_b200;

namespace {
int coefficients(int dim, int order) {
  if (order == 0) return 1;
  if (order == 1) return dim + 1;
  return dim == 2 ? 10 : 20;
}
}  // namespace

extern "C" {

// h, a1 of n single-channel jets z[n][q]; returns 1 for an unsupported (dim, order)
int host_jet_fwd(int dim, int order, const double* z, double* h, double* a1, long n) {
  const int q = coefficients(dim, order);
  for (long p = 0; p < n; ++p) {
    const double* zp = z + p * q;
    double* hp = h + p * q;
    if (dim == 2 && order == 0) jet_fwd_2d0(zp, hp, a1[p]);
    else if (dim == 2 && order == 1) jet_fwd_2d1(zp, hp, a1[p]);
    else if (dim == 2 && order == 3) jet_fwd_2d3(zp, hp, a1[p]);
    else if (dim == 3 && order == 0) jet_fwd_3d0(zp, hp, a1[p]);
    else if (dim == 3 && order == 1) jet_fwd_3d1(zp, hp, a1[p]);
    else if (dim == 3 && order == 3) jet_fwd_3d3(zp, hp, a1[p]);
    else return 1;
  }
  return 0;
}

int host_jet_vjp(int dim, int order, const double* h, const double* a1, const double* hb, double* zb, long n) {
  const int q = coefficients(dim, order);
  for (long p = 0; p < n; ++p) {
    const double *hp = h + p * q, *bp = hb + p * q;
    double* zp = zb + p * q;
    if (dim == 2 && order == 0) jet_vjp_2d0(hp, a1[p], bp, zp);
    else if (dim == 2 && order == 1) jet_vjp_2d1(hp, a1[p], bp, zp);
    else if (dim == 2 && order == 3) jet_vjp_2d3(hp, a1[p], bp, zp);
    else if (dim == 3 && order == 0) jet_vjp_3d0(hp, a1[p], bp, zp);
    else if (dim == 3 && order == 1) jet_vjp_3d1(hp, a1[p], bp, zp);
    else if (dim == 3 && order == 3) jet_vjp_3d3(hp, a1[p], bp, zp);
    else return 1;
  }
  return 0;
}

// per-point weighted loss and seed of interior jets y[n][q][outputs]; head 0 = (u, v, p)
// in 2-D, 1 = (psi, p) in 2-D or 3-D
int host_seed(int head, int dim, const double* y, const double* w, double nu, double gamma, double* dy,
              double* loss, long n) {
  const int stride = head == 0 ? 30 : (dim == 2 ? 20 : 40);
  for (long p = 0; p < n; ++p) {
    const double* yp = y + p * stride;
    double* dp = dy + p * stride;
    if (head == 0 && dim == 2) loss[p] = seed_uvp_2d(yp, w[p], nu, gamma, dp);
    else if (head == 1 && dim == 2) loss[p] = seed_psi_2d(yp, w[p], nu, gamma, dp);
    else if (head == 1 && dim == 3) loss[p] = seed_psi_3d(yp, w[p], nu, gamma, dp);
    else return 1;
  }
  return 0;
}

// residual values r[n][count] (count: 9 for (u, v, p), 2 for psi)
int host_residuals(int head, int dim, const double* y, double nu, double* r, long n) {
  const int stride = head == 0 ? 30 : (dim == 2 ? 20 : 40), count = head == 0 ? 9 : 2;
  for (long p = 0; p < n; ++p) {
    if (head == 0 && dim == 2) residuals_uvp_2d(y + p * stride, nu, r + p * count);
    else if (head == 1 && dim == 2) residuals_psi_2d(y + p * stride, nu, r + p * count);
    else if (head == 1 && dim == 3) residuals_psi_3d(y + p * stride, nu, r + p * count);
    else return 1;
  }
  return 0;
}

}  // extern "C"
