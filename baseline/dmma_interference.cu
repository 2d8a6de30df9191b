// What slows the FP64 tensor pipe: the DMMA rate of 8 warps running the evaluation
// kernels' shared-memory-fed m16n8k8 loop (one m16 tile of channels and five n8 tiles of
// rows per warp, fragments from 68- and 36-double padded rows) while the other 8 warps of
// the same 512-thread CTA run one kind of other work.  One CTA per SM on every SM.
//
// Measurement infrastructure beside the baselines (built and run by
// baseline/dmma_interference.py); nothing in the product includes it.  Every wait is
// bounded: the other warps stop when the MMA warps raise a flag, or after 2^22 rounds.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>

namespace {

__device__ __forceinline__ void mma(double (&c)[4], const double (&a)[4], double b0, double b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+d"(c[0]), "+d"(c[1]), "+d"(c[2]), "+d"(c[3])
      : "d"(a[0]), "d"(a[1]), "d"(a[2]), "d"(a[3]), "d"(b0), "d"(b1));
}
__device__ __forceinline__ long long clock_now() {
  long long c;
  asm volatile("mov.u64 %0, %%clock64;" : "=l"(c));
  return c;
}

constexpr int kLdw = 68, kLdc = 36, kRows = 80, kK = 32, kSms = 148, kSlots = 64;
constexpr int kBoxDoubles = 256;  // one warp's bulk-store source: 2 KB
__device__ volatile int g_stop[kSms];

enum Kind {
  kIdle, kDfmaChain, kDfma2, kDfma8, kExp, kLds, kInt, kStg8, kStg8x4, kStg16, kStgStreaming, kBulk, kKinds
};
const char* kNames[kKinds] = {"a loop polling the stop flag (baseline)",
                              "DFMA, one dependent chain",
                              "DFMA, two chains",
                              "DFMA, eight chains",
                              "exp()",
                              "shared-memory loads",
                              "integer multiply-add",
                              "global stores, 8 B, one per round",
                              "global stores, 8 B, four per round",
                              "global stores, 16 B, one per round",
                              "global stores, 8 B, streaming (.cs)",
                              "bulk (TMA) stores, 2 KB per warp every 8 rounds"};
// bytes one thread stores per round
const double kBytes[kKinds] = {0, 0, 0, 0, 0, 0, 0, 8, 32, 16, 8, double(kBoxDoubles * 8) / 32 / 8};

__global__ void __launch_bounds__(512, 1)
    probe(int kind, int iters, double* out, long long* cycles, double* rounds, double* sink) {
  extern __shared__ __align__(16) double sm[];
  double* sA = sm;
  double* sB = sm + kK * kLdw;
  double* sbox = sB + kRows * kLdc;  // [8 warps][kBoxDoubles]
  for (int i = threadIdx.x; i < kK * kLdw + kRows * kLdc + 8 * kBoxDoubles; i += blockDim.x) sm[i] = 1e-3 * (i & 63);
  if (threadIdx.x == 0) g_stop[blockIdx.x] = 0;
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  if (warp < 8) {  // the MMA warps
    const double* cA = sA + (warp & 3) * 16;
    const double* cB = sB + ((warp >> 2) & 1) * 40 * kLdc;
    double acc[5][4] = {};
    const long long t0 = clock_now();
    for (int it = 0; it < iters; ++it) {
#pragma unroll
      for (int kk = 0; kk < kK; kk += 8) {
        const double a[4] = {cA[(kk + t) * kLdw + g], cA[(kk + t) * kLdw + g + 8], cA[(kk + t + 4) * kLdw + g],
                             cA[(kk + t + 4) * kLdw + g + 8]};
#pragma unroll
        for (int j = 0; j < 5; ++j)
          mma(acc[j], a, cB[(8 * j + g) * kLdc + kk + t], cB[(8 * j + g) * kLdc + kk + t + 4]);
      }
    }
    double r = 0.0;
#pragma unroll
    for (int j = 0; j < 5; ++j) r += (acc[j][0] + acc[j][1]) + (acc[j][2] + acc[j][3]);
    const long long t1 = clock_now();
    if (r == 12345.678) sink[0] = r;
    if (lane == 0) cycles[blockIdx.x * 8 + warp] = t1 - t0;
    __syncwarp();
    if (warp == 0 && lane == 0) {
      __threadfence_block();
      g_stop[blockIdx.x] = 1;
    }
    return;
  }
  // the other warps: one kind of work per round until the MMA warps are done
  const int ot = threadIdx.x - 256, w = warp - 8;
  double v0 = 1.0 + 1e-9 * threadIdx.x, v1 = 0.5, v2 = 0.25, v3 = 0.125, v4 = 2.0, v5 = 3.0, v6 = 1.5, v7 = 0.75;
  unsigned u = threadIdx.x;
  const size_t slot = size_t(kSms) * 256;  // doubles per store slot (every CTA's 256 threads)
  double* mine = out + size_t(blockIdx.x) * 256 + ot;
  long n = 0;
  for (long rep = 0; rep < (1L << 22); ++rep) {
    if ((rep & 63) == 0 && g_stop[blockIdx.x]) break;
    const size_t s = size_t(rep) % kSlots;
    switch (kind) {
      case kDfmaChain:
#pragma unroll
        for (int q = 0; q < 16; ++q) v0 = fma(v0, 0.999999, 1e-7);
        break;
      case kDfma2:
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          v0 = fma(v0, 0.999999, 1e-7);
          v1 = fma(v1, 0.999999, 1e-7);
        }
        break;
      case kDfma8:
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          v0 = fma(v0, 0.999999, 1e-7); v1 = fma(v1, 0.999999, 1e-7); v2 = fma(v2, 0.999999, 1e-7);
          v3 = fma(v3, 0.999999, 1e-7); v4 = fma(v4, 0.999999, 1e-7); v5 = fma(v5, 0.999999, 1e-7);
          v6 = fma(v6, 0.999999, 1e-7); v7 = fma(v7, 0.999999, 1e-7);
        }
        break;
      case kExp:
        v0 = exp(-fabs(v0)) + 0.5;
        break;
      case kLds:
        v0 += sm[(u + rep * 7) % (kK * kLdw)];
        break;
      case kInt:
#pragma unroll
        for (int q = 0; q < 16; ++q) u = u * 1664525u + 1013904223u;
        break;
      case kStg8:
        mine[s * slot] = v0;
        break;
      case kStg8x4:  // four slots a round, all inside the buffer of kSlots slots
#pragma unroll
        for (int q = 0; q < 4; ++q) mine[((4 * size_t(rep) + q) % kSlots) * slot] = v0;
        break;
      case kStg16:  // slot pairs: 16 B per thread, half as many slots
        reinterpret_cast<double2*>(out)[size_t(blockIdx.x) * 256 + ot + (s % (kSlots / 2)) * slot] =
            make_double2(v0, v1);
        break;
      case kStgStreaming:
        __stcs(mine + s * slot, v0);
        break;
      case kBulk:
        if ((rep & 7) == 0) {
          if (lane == 0) {
            asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory");
            const unsigned src = unsigned(__cvta_generic_to_shared(sbox + w * kBoxDoubles));
            // 8 bulk slots of [every CTA][8 warps][256 doubles]: inside the buffer
            double* dst = out + (size_t(blockIdx.x) * 8 + w) * kBoxDoubles +
                          (size_t(rep >> 3) % (kSlots / 8)) * (size_t(kSms) * 8 * kBoxDoubles);
            asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;\n" ::"l"(dst), "r"(src),
                         "n"(kBoxDoubles * 8)
                         : "memory");
            asm volatile("cp.async.bulk.commit_group;\n" ::: "memory");
          }
          __syncwarp();
        }
        break;
      default:
        break;
    }
    ++n;
  }
  if (kind == kBulk && lane == 0) asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory");
  const double r = v0 + v1 + v2 + v3 + v4 + v5 + v6 + v7 + double(u & 1);
  if (r == 12345.678) sink[0] = r;
  if (ot == 0) rounds[blockIdx.x] = double(n);
}

}  // namespace

int main(int argc, char** argv) {
  const int iters = argc > 1 ? atoi(argv[1]) : 4096;
  double *out, *sink, *rounds;
  long long* cyc;
  const size_t out_doubles = size_t(kSms) * 256 * kSlots;  // 19.4 MB
  if (cudaMalloc(&out, sizeof(double) * out_doubles) != cudaSuccess || cudaMalloc(&sink, sizeof(double) * 2) ||
      cudaMalloc(&rounds, sizeof(double) * kSms) || cudaMalloc(&cyc, sizeof(long long) * kSms * 8)) {
    fprintf(stderr, "allocation failed\n");
    return 1;
  }
  const size_t smem = sizeof(double) * (kK * kLdw + kRows * kLdc + 8 * kBoxDoubles);
  cudaFuncSetAttribute(probe, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  long long h[kSms * 8];
  double hr[kSms];
  printf("| other 8 warps | DMMA rate of the 8 MMA warps | stored B/clk/SM |\n|---|---|---|\n");
  for (int kind = 0; kind < kKinds; ++kind) {
    for (int rep = 0; rep < 2; ++rep) probe<<<kSms, 512, smem>>>(kind, iters, out, cyc, rounds, sink);
    const cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
      fprintf(stderr, "%s\n", cudaGetErrorString(e));
      return 1;
    }
    cudaMemcpy(h, cyc, sizeof(h), cudaMemcpyDeviceToHost);
    cudaMemcpy(hr, rounds, sizeof(hr), cudaMemcpyDeviceToHost);
    double cycles = 0.0, n = 0.0;
    for (int i = 0; i < kSms * 8; ++i) cycles += double(h[i]);
    for (int i = 0; i < kSms; ++i) n += hr[i];
    cycles /= kSms * 8;
    n /= kSms;
    // per SM sub-partition: 2 MMA warps x 4 k-steps x 5 DMMAs a round, 64 cycles each at the full rate
    const double ideal = 2.0 * 4 * 5 * 64 * iters;
    printf("| %s | %.3f | %.1f |\n", kNames[kind], ideal / cycles, 256.0 * n * kBytes[kind] / cycles);
  }
  return 0;
}
