// In-run FP64 tensor-core peak probe: register-only DMMA m16n8k8 chains.
// Gives the denominator of the FP64 roofline on the same device and clock as the
// measured kernels (no FP64 figure is recorded in the driver's peak file).
#include "common.cuh"
#include "flashns_b200.h"

namespace flashns_b200 {

__global__ void __launch_bounds__(256) dmma_peak(double* sink, int iters) {
  double a[4] = {1e-3 * threadIdx.x, 2e-3, 3e-3, 4e-3};
  const double b0 = 1e-3, b1 = 5e-3;
  double c[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) c[i][j] = 0.0;
  for (int it = 0; it < iters; ++it) {
#pragma unroll
    for (int i = 0; i < 8; ++i) mma_m16n8k8(c[i], a, b0, b1);
  }
  double r = 0.0;
#pragma unroll
  for (int i = 0; i < 8; ++i) r += (c[i][0] + c[i][1]) + (c[i][2] + c[i][3]);
  if (r == 12345.678) sink[0] = r;  // never true; keeps the chains live
}

// ---- the other FP64 instruction shapes, and a shared-memory fed loop in the kernels' tile
// shape, for the peak table (flashns_b200_fp64_probe).  Register-only loops keep 8
// independent accumulator chains per warp; nothing is stored unless a never-true test
// passes.
__device__ __forceinline__ void mma_m8n8k4(double (&c)[2], double a, double b) {
  asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0,%1}, {%2}, {%3}, {%0,%1};\n"
               : "+d"(c[0]), "+d"(c[1])
               : "d"(a), "d"(b));
}
__device__ __forceinline__ void mma_m16n8k4(double (&c)[4], double a0, double a1, double b) {
  asm volatile("mma.sync.aligned.m16n8k4.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};\n"
               : "+d"(c[0]), "+d"(c[1]), "+d"(c[2]), "+d"(c[3])
               : "d"(a0), "d"(a1), "d"(b));
}
__device__ __forceinline__ void mma_m16n8k16(double (&c)[4], const double (&a)[8], const double (&b)[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5,%6,%7,%8,%9,%10,%11}, "
      "{%12,%13,%14,%15}, {%0,%1,%2,%3};\n"
      : "+d"(c[0]), "+d"(c[1]), "+d"(c[2]), "+d"(c[3])
      : "d"(a[0]), "d"(a[1]), "d"(a[2]), "d"(a[3]), "d"(a[4]), "d"(a[5]), "d"(a[6]), "d"(a[7]), "d"(b[0]),
        "d"(b[1]), "d"(b[2]), "d"(b[3]));
}

template <int KIND>
__global__ void register_probe(double* sink, int iters) {
  const double x = 1e-3 * threadIdx.x;
  double r = 0.0;
  if constexpr (KIND == 1) {
    double c[8][2] = {};
    for (int it = 0; it < iters; ++it)
#pragma unroll
      for (int i = 0; i < 8; ++i) mma_m8n8k4(c[i], x, 2e-3);
#pragma unroll
    for (int i = 0; i < 8; ++i) r += c[i][0] + c[i][1];
  } else if constexpr (KIND == 2) {
    double c[8][4] = {};
    for (int it = 0; it < iters; ++it)
#pragma unroll
      for (int i = 0; i < 8; ++i) mma_m16n8k4(c[i], x, 2e-3, 3e-3);
#pragma unroll
    for (int i = 0; i < 8; ++i) r += (c[i][0] + c[i][1]) + (c[i][2] + c[i][3]);
  } else if constexpr (KIND == 3) {
    const double a[8] = {x, 2e-3, 3e-3, 4e-3, 5e-3, 6e-3, 7e-3, 8e-3}, b[4] = {1e-3, 2e-3, 3e-3, 4e-3};
    double c[8][4] = {};
    for (int it = 0; it < iters; ++it)
#pragma unroll
      for (int i = 0; i < 8; ++i) mma_m16n8k16(c[i], a, b);
#pragma unroll
    for (int i = 0; i < 8; ++i) r += (c[i][0] + c[i][1]) + (c[i][2] + c[i][3]);
  } else {  // DFMA: 16 independent chains per thread
    double c[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) c[i] = x + i;
    for (int it = 0; it < iters; ++it)
#pragma unroll
      for (int i = 0; i < 16; ++i) c[i] = fma(c[i], 0.999, 1e-3);
#pragma unroll
    for (int i = 0; i < 16; ++i) r += c[i];
  }
  if (r == 12345.678) sink[0] = r;
}

// Shared-memory fed m16n8k8 in the kernels' tile shape: a warp owns one m16 tile of
// channels and five n8 tiles of rows; every k-step loads its A fragment from a W plane
// (rows padded to 68 doubles) and its B fragments from an activation plane (rows padded
// to 36 doubles), a 32-deep K slice per round, as the dgrad mainloop does.
constexpr int kProbeLdw = 68, kProbeLdc = 36, kProbeRows = 80, kProbeK = 32;
constexpr size_t kProbeSmem = sizeof(double) * (size_t(kProbeK) * kProbeLdw + size_t(kProbeRows) * kProbeLdc);

__global__ void smem_probe(double* sink, int iters) {
  extern __shared__ __align__(16) double sm[];
  double* sA = sm;                        // [32][68]: 64 channels of a 32-deep K slice
  double* sB = sm + kProbeK * kProbeLdw;  // [80][36]: 80 rows of a 32-column plane
  for (int i = threadIdx.x; i < kProbeK * kProbeLdw + kProbeRows * kProbeLdc; i += blockDim.x) sm[i] = 1e-3 * (i & 63);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const double* cA = sA + (warp & 3) * 16;                    // channel tile 0..3
  const double* cB = sB + ((warp >> 2) & 1) * 40 * kProbeLdc;  // rows 0..39 or 40..79
  double acc[5][4] = {};
  for (int it = 0; it < iters; ++it) {
#pragma unroll
    for (int kk = 0; kk < kProbeK; kk += 8) {
      const double a[4] = {cA[(kk + t) * kProbeLdw + g], cA[(kk + t) * kProbeLdw + g + 8],
                           cA[(kk + t + 4) * kProbeLdw + g], cA[(kk + t + 4) * kProbeLdw + g + 8]};
#pragma unroll
      for (int j = 0; j < 5; ++j)
        mma_m16n8k8(acc[j], a, cB[(8 * j + g) * kProbeLdc + kk + t], cB[(8 * j + g) * kProbeLdc + kk + t + 4]);
    }
  }
  double r = 0.0;
#pragma unroll
  for (int j = 0; j < 5; ++j) r += (acc[j][0] + acc[j][1]) + (acc[j][2] + acc[j][3]);
  if (r == 12345.678) sink[0] = r;
}

}  // namespace flashns_b200

extern "C" int flashns_b200_fp64_peak_probe(int blocks, int iters, double* sink, double* flops, cudaStream_t stream) {
  if (blocks < 1 || iters < 1 || !sink || !flops) return int(cudaErrorInvalidValue);
  flashns_b200::dmma_peak<<<blocks, 256, 0, stream>>>(sink, iters);
  *flops = 2.0 * 16 * 8 * 8 * 8.0 * double(iters) * double(blocks) * (256 / 32);
  return int(cudaGetLastError());
}

extern "C" int flashns_b200_fp64_probe(int kind, int blocks, int threads, int iters, double* sink, double* flops,
                                       cudaStream_t stream) {
  using namespace flashns_b200;
  if (kind < 0 || kind > FLASHNS_B200_PROBE_SMEM || blocks < 1 || iters < 1 || !sink || !flops ||
      threads < 32 || threads > 1024 || threads % 32)
    return int(cudaErrorInvalidValue);
  const double warps = double(blocks) * (threads / 32), n = double(iters);
  switch (kind) {
    case FLASHNS_B200_PROBE_M16N8K8:
      if (threads != 256) return int(cudaErrorInvalidValue);  // the in-run probe's launch shape
      return flashns_b200_fp64_peak_probe(blocks, iters, sink, flops, stream);
    case FLASHNS_B200_PROBE_M8N8K4:
      register_probe<1><<<blocks, threads, 0, stream>>>(sink, iters);
      *flops = 2.0 * 8 * 8 * 4 * 8 * n * warps;
      break;
    case FLASHNS_B200_PROBE_M16N8K4:
      register_probe<2><<<blocks, threads, 0, stream>>>(sink, iters);
      *flops = 2.0 * 16 * 8 * 4 * 8 * n * warps;
      break;
    case FLASHNS_B200_PROBE_M16N8K16:
      register_probe<3><<<blocks, threads, 0, stream>>>(sink, iters);
      *flops = 2.0 * 16 * 8 * 16 * 8 * n * warps;
      break;
    case FLASHNS_B200_PROBE_DFMA:
      register_probe<4><<<blocks, threads, 0, stream>>>(sink, iters);
      *flops = 2.0 * 16 * n * warps * 32;
      break;
    default:
      smem_probe<<<blocks, threads, kProbeSmem, stream>>>(sink, iters);
      *flops = 2.0 * 16 * 8 * 8 * 5 * (kProbeK / 8) * n * warps;
      break;
  }
  return int(cudaGetLastError());
}
