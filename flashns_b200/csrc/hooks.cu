// Per-stage CUDA hooks with the reference's C ABI, so that the reference bindings
// (experiments/pinn_v8/native.py:26-51 for the packed layout, experiments/cuda_jet_h100/gpu.py
// for the dense [B,Q,C] layout) can load this library in place of theirs.  Each entry point
// keeps the reference's symbol name, argument order and meaning, return convention and
// caller-provided scratch; the kernels are this library's own (generated jet formulas,
// fixed-order reductions).
//
//   flashns_v8_activation                 experiments/pinn_v8/native.cu:47-62
//   flashns_v8_coordinate_affine[_activation]                     :115-129
//   flashns_v8_tail3                                              :174-200
//   flashns_v8_coordinate_[activation_]wgrad                      :275-290
//   flashns_v8_loss_seed                                          :325-337
//   flashns_stable_activation / _tail3    experiments/cuda_jet_h100/stable_kernels.cu:93-131
//   flashns_stable_dgrad_vjp                                      stable_dgrad.cu:150-174
//   flashns_hopper_initialize / _resources / _create / _destroy / _launch
//                                         experiments/cuda_jet_hopper/hopper.cu:287-353
#include <climits>
#include <new>
#include <cstddef>
#include <cstdint>

#include "common.cuh"
#include "flashns_b200.h"
#include "jets_generated.cuh"
#include "residual_generated.cuh"

namespace flashns_b200 {
// eval.cu: the dense dgrad (+ VJP) of a 64 -> 64 layer on the evaluation's backward kernels
// (two-group in 2-D, one-group 160-row tiles in 3-D) without their weight gradient
cudaError_t dense_dgrad_64(int dim, bool fused, const double* d, const double* w, const double* h,
                           const double* aux, double* out, int batch, cudaStream_t stream);
namespace {

constexpr int kHookThreads = 128;

template <int DIM>
struct Q_;
template <>
struct Q_<2> { static constexpr int v = 10; };
template <>
struct Q_<3> { static constexpr int v = 20; };

template <int DIM>
__device__ __forceinline__ void fwd_full(const double* z, double* h, double& a) {
  if constexpr (DIM == 2) jet_fwd_2d3(z, h, a); else jet_fwd_3d3(z, h, a);
}
template <int DIM>
__device__ __forceinline__ void vjp_full(const double* h, double a, const double* hb, double* zb) {
  if constexpr (DIM == 2) jet_vjp_2d3(h, a, hb, zb); else jet_vjp_3d3(h, a, hb, zb);
}
__device__ __forceinline__ void fwd_value(double z, double& h, double& a) {
  double zz[1] = {z}, hh[1];
  jet_fwd_2d0(zz, hh, a);
  h = hh[0];
}

int64_t blocks_for(int64_t n) { return (n + kHookThreads - 1) / kHookThreads; }

bool overlaps(const void* a, size_t na, const void* b, size_t nb) {
  const auto pa = reinterpret_cast<uintptr_t>(a), pb = reinterpret_cast<uintptr_t>(b);
  return a && b && na && nb && (pa <= pb ? pb - pa < na : pa - pb < nb);
}

// ---------------------------------------------------------------- packed activation
template <int DIM, bool BACKWARD>
__global__ void __launch_bounds__(kHookThreads)
    packed_activation(const double* __restrict__ in, const double* __restrict__ aux, const double* __restrict__ seed,
                      double* __restrict__ out, double* __restrict__ out_aux, int64_t full, int64_t value, int channels) {
  constexpr int Q = Q_<DIM>::v;
  const int64_t total = (full + value) * channels;
  for (int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += int64_t(gridDim.x) * blockDim.x) {
    const int64_t p = idx / channels;
    const int c = int(idx % channels);
    if (p < full) {
      const int64_t base = p * Q * channels + c;
      double x[Q], y[Q];
#pragma unroll
      for (int s = 0; s < Q; ++s) x[s] = in[base + int64_t(s) * channels];
      if constexpr (BACKWARD) {
        double hb[Q];
#pragma unroll
        for (int s = 0; s < Q; ++s) hb[s] = seed[base + int64_t(s) * channels];
        vjp_full<DIM>(x, aux[idx], hb, y);
      } else {
        double a;
        fwd_full<DIM>(x, y, a);
        out_aux[idx] = a;
      }
#pragma unroll
      for (int s = 0; s < Q; ++s) out[base + int64_t(s) * channels] = y[s];
    } else {
      const int64_t r = (full * Q + (p - full)) * channels + c;
      if constexpr (BACKWARD) {
        out[r] = seed[r] * aux[idx];
      } else {
        double h, a;
        fwd_value(in[r], h, a);
        out[r] = h;
        out_aux[idx] = a;
      }
    }
  }
}

// ---------------------------------------------------------------- dense activation
template <int DIM, bool BACKWARD>
__global__ void __launch_bounds__(kHookThreads)
    dense_activation(const double* __restrict__ value, const double* __restrict__ adjoint,
                     const double* __restrict__ aux_in, double* __restrict__ out, double* __restrict__ aux_out,
                     int64_t batch, int64_t channels) {
  constexpr int Q = Q_<DIM>::v;
  const int64_t total = batch * channels;
  for (int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += int64_t(gridDim.x) * blockDim.x) {
    const int64_t b = idx / channels, c = idx % channels;
    const int64_t base = b * Q * channels + c;
    double x[Q], y[Q];
#pragma unroll
    for (int s = 0; s < Q; ++s) x[s] = value[base + s * channels];
    if constexpr (BACKWARD) {
      double hb[Q];
#pragma unroll
      for (int s = 0; s < Q; ++s) hb[s] = adjoint[base + s * channels];
      vjp_full<DIM>(x, aux_in[idx], hb, y);
    } else {
      double a;
      fwd_full<DIM>(x, y, a);
      aux_out[idx] = a;
    }
#pragma unroll
    for (int s = 0; s < Q; ++s) out[base + s * channels] = y[s];
  }
}

// ---------------------------------------------------------------- coordinate affine
template <int DIM, bool ACT>
__global__ void __launch_bounds__(kHookThreads)
    coordinate_affine(const double* __restrict__ x, const double* __restrict__ w, const double* __restrict__ b,
                      double* __restrict__ out, double* __restrict__ out_aux, int64_t full, int64_t value,
                      int channels) {
  constexpr int Q = Q_<DIM>::v;
  const int64_t total = (full + value) * channels;
  for (int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += int64_t(gridDim.x) * blockDim.x) {
    const int64_t p = idx / channels;
    const int c = int(idx % channels);
    const double* wr = w + int64_t(c) * DIM;
    const double* xp = x + p * DIM;
    double z0 = xp[0] * wr[0];
#pragma unroll
    for (int a = 1; a < DIM; ++a) z0 += xp[a] * wr[a];
    z0 += b[c];
    if (p < full) {
      double z[Q], h[Q];
#pragma unroll
      for (int s = 0; s < Q; ++s) z[s] = 0.0;
      z[0] = z0;
#pragma unroll
      for (int a = 0; a < DIM; ++a) z[unit_row<DIM>(a)] = wr[a];
      double* dst = out + p * Q * channels + c;
      if constexpr (ACT) {
        double a1;
        fwd_full<DIM>(z, h, a1);
        out_aux[idx] = a1;
#pragma unroll
        for (int s = 0; s < Q; ++s) dst[int64_t(s) * channels] = h[s];
      } else {
#pragma unroll
        for (int s = 0; s < Q; ++s) dst[int64_t(s) * channels] = z[s];
      }
    } else {
      const int64_t r = (full * Q + (p - full)) * channels + c;
      if constexpr (ACT) {
        double h, a1;
        fwd_value(z0, h, a1);
        out[r] = h;
        out_aux[idx] = a1;
      } else {
        out[r] = z0;
      }
    }
  }
}

// ---------------------------------------------------------------- Cout = 3 tail
template <int DIM, bool FUSED>
__global__ void __launch_bounds__(kHookThreads)
    packed_tail3(const double* __restrict__ d, const double* __restrict__ w, const double* __restrict__ hidden,
                 const double* __restrict__ aux, double* __restrict__ out, int64_t full, int64_t value, int channels) {
  constexpr int Q = Q_<DIM>::v;
  const int64_t total = (full + value) * channels;
  for (int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += int64_t(gridDim.x) * blockDim.x) {
    const int64_t p = idx / channels;
    const int c = int(idx % channels);
    const double w0 = w[c], w1 = w[int64_t(channels) + c], w2 = w[int64_t(2) * channels + c];
    if (p < full) {
      const int64_t row = p * Q;
      double bar[Q];
#pragma unroll
      for (int s = 0; s < Q; ++s) {
        const double* dr = d + (row + s) * 3;
        bar[s] = (dr[0] * w0 + dr[1] * w1) + dr[2] * w2;
      }
      double* dst = out + row * channels + c;
      if constexpr (FUSED) {
        double h[Q], zb[Q];
#pragma unroll
        for (int s = 0; s < Q; ++s) h[s] = hidden[(row + s) * channels + c];
        vjp_full<DIM>(h, aux[idx], bar, zb);
#pragma unroll
        for (int s = 0; s < Q; ++s) dst[int64_t(s) * channels] = zb[s];
      } else {
#pragma unroll
        for (int s = 0; s < Q; ++s) dst[int64_t(s) * channels] = bar[s];
      }
    } else {
      const int64_t row = full * Q + (p - full);
      const double* dr = d + row * 3;
      const double bar = (dr[0] * w0 + dr[1] * w1) + dr[2] * w2;
      out[row * channels + c] = FUSED ? bar * aux[idx] : bar;
    }
  }
}

template <int DIM, bool FUSED>
__global__ void __launch_bounds__(kHookThreads)
    dense_tail3(const double* __restrict__ d, const double* __restrict__ w, const double* __restrict__ hidden,
                const double* __restrict__ aux, double* __restrict__ out, int64_t batch, int64_t channels) {
  constexpr int Q = Q_<DIM>::v;
  const int64_t total = batch * channels;
  for (int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += int64_t(gridDim.x) * blockDim.x) {
    const int64_t b = idx / channels, c = idx % channels;
    const double w0 = w[c], w1 = w[channels + c], w2 = w[2 * channels + c];
    double bar[Q];
#pragma unroll
    for (int s = 0; s < Q; ++s) {
      const double* dr = d + (b * Q + s) * 3;
      bar[s] = (dr[0] * w0 + dr[1] * w1) + dr[2] * w2;
    }
    double* dst = out + b * Q * channels + c;
    if constexpr (FUSED) {
      double h[Q], zb[Q];
#pragma unroll
      for (int s = 0; s < Q; ++s) h[s] = hidden[(b * Q + s) * channels + c];
      vjp_full<DIM>(h, aux[idx], bar, zb);
#pragma unroll
      for (int s = 0; s < Q; ++s) dst[s * channels] = zb[s];
    } else {
#pragma unroll
      for (int s = 0; s < Q; ++s) dst[s * channels] = bar[s];
    }
  }
}

// ---------------------------------------------------------------- dense dgrad (+ VJP)
// dH[b, q, i] = sum_o D[b, q, o] W[o, i] on the FP64 tensor pipe (DMMA m16n8k8), then,
// when FUSED, the jet VJP of each (sample, channel) from the accumulators.
//
// The GEMM runs transposed, as in the evaluation kernels: MMA M = input channels i (a CTA
// owns a block of 64), MMA N = rows (b, q), K = output channels o.  A tile is 8 samples
// (TR = 8 Q rows, contiguous in D, in their global order in shared memory); each of the 8
// warps owns 16 channels of 4 samples, and a thread's accumulators hold, for its two
// channels, all Q rows of one sample: the VJP needs no data exchange.  Tiles are (sample
// block, channel block) pairs, grid-strided over a persistent grid of two CTAs per SM in
// 2-D.  K streams through a two-stage ring of 32-column chunks of D that runs on across
// tiles: the first chunk of a CTA's next tile is in flight while it runs the current
// tile's epilogue, and the other CTA on the SM keeps the tensor pipe busy meanwhile.  W
// stays resident in shared memory when one channel block covers cin (cin <= 64) and
// cout <= 128 (the layers of the reference's nets); otherwise its chunks stream beside
// D's.  Copies are 16-byte cp.async when the rows allow it (even cout and cin, 16-byte
// aligned D and W), 8-byte otherwise, zero-filled past the ends, so any cout and cin work.
// The tile's H rows and a1 values (contiguous ranges) are prefetched into L2 when the
// tile starts; the epilogue reads them from there.
constexpr int kDgThreads = 256, kDgKC = 32, kDgLDC = kDgKC + 4, kDgCB = 64, kDgLDW = kDgCB + 4;
constexpr int kDgTC = 8;             // samples per tile
constexpr int kDgResidentRows = 128;  // largest cout (rounded up to KC) kept resident

// W resident: one channel block and cout within the resident rows
inline bool dgrad_resident(int cout, int cin) { return cin <= kDgCB && cout <= kDgResidentRows; }
template <int DIM>
constexpr size_t dgrad_smem_bytes(int w_rows) {
  return sizeof(double) * (2 * size_t(kDgTC) * Q_<DIM>::v * kDgLDC + size_t(w_rows) * kDgLDW);
}
template <int DIM>
size_t dgrad_smem_bytes_for(int cout, int cin) {
  const int nk = (cout + kDgKC - 1) / kDgKC;
  return dgrad_smem_bytes<DIM>(dgrad_resident(cout, cin) ? nk * kDgKC : 2 * kDgKC);
}

__device__ __forceinline__ void cp_async8(void* smem, const void* gmem, bool valid) {
  const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(sa), "l"(gmem), "r"(valid ? 8 : 0));
}

template <int DIM, bool FUSED>
__global__ void __launch_bounds__(kDgThreads, DIM == 2 ? 2 : 1)
    dense_dgrad(const double* __restrict__ d, const double* __restrict__ w, const double* __restrict__ h,
                const double* __restrict__ aux, double* __restrict__ out, int batch, int cout, int cin, bool vec,
                bool resident) {
  constexpr int Q = Q_<DIM>::v, TR = kDgTC * Q, NT = Q / 2, LDC = kDgLDC, LDW = kDgLDW, KC = kDgKC;
  extern __shared__ __align__(16) double dsm[];
  double* sD = dsm;                 // [2][TR][LDC]   D chunk: rows of the tile, 32 output channels
  double* sW = dsm + 2 * TR * LDC;  // W: [nk*KC][LDW] resident, or [2][KC][LDW] chunks
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int wc = warp % 4, wr = warp / 4;  // 16-channel slice, sample group (4 samples)
  const int64_t sample_tiles = (int64_t(batch) + kDgTC - 1) / kDgTC;
  const int channel_blocks = (cin + kDgCB - 1) / kDgCB;
  const int64_t units = sample_tiles * channel_blocks;
  const int64_t mine = int64_t(blockIdx.x) < units ? (units - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int nk = (cout + KC - 1) / KC;
  const int64_t steps = mine * nk;  // (tile, K chunk) pairs of this CTA, in order
  const int brow = (wr * 4 + (g >> 1)) * Q + (g & 1);  // B column g of n8 tile j: row brow + 2j
  auto unit_of = [&](int64_t i) { return int64_t(blockIdx.x) + i * gridDim.x; };
  auto load = [&](int64_t step, int stage) {
    const int64_t u = unit_of(step / nk);
    const int kc = int(step % nk);
    const int64_t b0 = (u / channel_blocks) * kDgTC;
    const int i0 = int(u % channel_blocks) * kDgCB;
    const int64_t rows_left = (int64_t(batch) - b0) * Q;
    double* dD = sD + stage * TR * LDC;
    double* dW = sW + stage * KC * LDW;
    if (vec) {
      for (int e = tid; e < TR * (KC / 2); e += kDgThreads) {
        const int r = e / (KC / 2), c = 2 * (e % (KC / 2)), o = kc * KC + c;
        const bool ok = r < rows_left && o < cout;  // cout even: o < cout covers o + 1
        cp_async16(dD + r * LDC + c, ok ? d + (b0 * Q + r) * cout + o : d, ok);
      }
      if (resident) return;
      for (int e = tid; e < KC * (kDgCB / 2); e += kDgThreads) {
        const int r = e / (kDgCB / 2), c = 2 * (e % (kDgCB / 2)), o = kc * KC + r, i = i0 + c;
        const bool ok = o < cout && i < cin;  // cin even: i < cin covers i + 1
        cp_async16(dW + r * LDW + c, ok ? w + int64_t(o) * cin + i : w, ok);
      }
    } else {
      for (int e = tid; e < TR * KC; e += kDgThreads) {
        const int r = e / KC, c = e % KC, o = kc * KC + c;
        const bool ok = r < rows_left && o < cout;
        cp_async8(dD + r * LDC + c, ok ? d + (b0 * Q + r) * cout + o : d, ok);
      }
      if (resident) return;
      for (int e = tid; e < KC * kDgCB; e += kDgThreads) {
        const int r = e / kDgCB, c = e % kDgCB, o = kc * KC + r, i = i0 + c;
        const bool ok = o < cout && i < cin;
        cp_async8(dW + r * LDW + c, ok ? w + int64_t(o) * cin + i : w, ok);
      }
    }
  };
  double acc[NT][4];
  if (resident && steps > 0) {  // W [nk*KC][64], zero past cout and cin; joins the first chunk's group
    for (int e = tid; e < nk * KC * kDgCB; e += kDgThreads) {
      const int o = e / kDgCB, i = e % kDgCB;
      const bool ok = o < cout && i < cin;
      cp_async8(sW + o * LDW + i, ok ? w + int64_t(o) * cin + i : w, ok);
    }
  }
  if (steps > 0) load(0, 0);
  cp_async_commit();
  for (int64_t step = 0; step < steps; ++step) {
    const int kc = int(step % nk);
    const int64_t u = unit_of(step / nk);
    const int64_t b0 = (u / channel_blocks) * kDgTC;
    const int i0 = int(u % channel_blocks) * kDgCB;
    if (kc == 0) {
#pragma unroll
      for (int j = 0; j < NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[j][e] = 0.0;
      if constexpr (FUSED) {
        if (tid == 0) {  // the epilogue's H rows and a1 values into L2 (whole rows: every channel block)
          const int64_t nb = int64_t(batch) - b0 < kDgTC ? int64_t(batch) - b0 : kDgTC;
          const uint64_t hbytes = uint64_t(nb) * Q * cin * sizeof(double), abytes = uint64_t(nb) * cin * sizeof(double);
          const double* hs = h + b0 * Q * cin;
          const double* as = aux + b0 * cin;
          if (((reinterpret_cast<uintptr_t>(hs) | hbytes) & 15) == 0 && hbytes < (1u << 31)) prefetch_l2(hs, uint32_t(hbytes));
          if (((reinterpret_cast<uintptr_t>(as) | abytes) & 15) == 0 && abytes < (1u << 31)) prefetch_l2(as, uint32_t(abytes));
        }
      }
    }
    if (step + 1 < steps) load(step + 1, int((step + 1) & 1));  // may be the next tile's first chunk
    cp_async_commit();
    cp_async_wait<1>();  // chunk `step` landed (this thread's copies)
    __syncthreads();     // ... and every other thread's
    const double* cB = sD + (step & 1) * TR * LDC + brow * LDC;
    const double* cA = sW + (resident ? kc : int(step & 1)) * KC * LDW + wc * 16;
#pragma unroll
    for (int kk = 0; kk < KC; kk += 8) {
      double a[4];
      a[0] = cA[(kk + t) * LDW + g];
      a[1] = cA[(kk + t) * LDW + g + 8];
      a[2] = cA[(kk + t + 4) * LDW + g];
      a[3] = cA[(kk + t + 4) * LDW + g + 8];
#pragma unroll
      for (int j = 0; j < NT; ++j) mma_m16n8k8(acc[j], a, cB[2 * j * LDC + kk + t], cB[2 * j * LDC + kk + t + 4]);
    }
    __syncthreads();  // stage step & 1 free for chunk step + 2
    if (kc != nk - 1) continue;
    // epilogue of tile u: sample b0 + wr*4 + t, channels i0 + 16 wc + {g, g + 8}
    const int64_t b = b0 + wr * 4 + t;
    if (b >= batch) continue;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int i = i0 + wc * 16 + 8 * hh + g;
      if (i >= cin) continue;
      double dh[Q];
#pragma unroll
      for (int s = 0; s < Q; ++s) dh[s] = acc[s >> 1][2 * hh + (s & 1)];
      double* dst = out + b * Q * cin + i;
      if constexpr (FUSED) {
        double hv[Q], zb[Q];
#pragma unroll
        for (int s = 0; s < Q; ++s) hv[s] = h[(b * Q + s) * cin + i];
        vjp_full<DIM>(hv, aux[b * cin + i], dh, zb);
#pragma unroll
        for (int s = 0; s < Q; ++s) dst[int64_t(s) * cin] = zb[s];
      } else {
#pragma unroll
        for (int s = 0; s < Q; ++s) dst[int64_t(s) * cin] = dh[s];
      }
    }
  }
  cp_async_wait<0>();
}

template <int DIM, bool FUSED>
cudaError_t launch_dense_dgrad(const double* d, const double* w, const double* h, const double* aux, double* out,
                               int batch, int cout, int cin, cudaStream_t stream) {
  const bool resident = dgrad_resident(cout, cin);
  const size_t smem = dgrad_smem_bytes_for<DIM>(cout, cin);
  // a per-device attribute (host-side, not a stream operation): set on every call, so that
  // each device the caller switches to gets it
  cudaError_t e = cudaFuncSetAttribute(dense_dgrad<DIM, FUSED>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(dgrad_smem_bytes<DIM>(kDgResidentRows)));
  if (e != cudaSuccess) return e;
  int device = 0, sms = 0, per_sm = 0;
  e = cudaGetDevice(&device);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, dense_dgrad<DIM, FUSED>, kDgThreads, smem);
  if (e != cudaSuccess) return e;
  const int64_t units = ((int64_t(batch) + kDgTC - 1) / kDgTC) * ((cin + kDgCB - 1) / kDgCB);
  const int64_t slots = int64_t(sms) * (per_sm > 0 ? per_sm : 1);
  const unsigned grid = unsigned(units < slots ? units : slots);
  const bool vec = cout % 2 == 0 && cin % 2 == 0 && (reinterpret_cast<uintptr_t>(d) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(w) & 15) == 0;
  dense_dgrad<DIM, FUSED><<<grid, kDgThreads, smem, stream>>>(d, w, h, aux, out, batch, cout, cin, vec, resident);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- coordinate wgrad
// Stage 1: partials[tile][c][0..DIM-1] = sum over the tile's 8 points of
// D[row0][c] x[a] + D[unit(a)][c] (full points; every other slot enters multiplied by its
// structural zero), partials[tile][c][DIM] = sum D[row0][c].
// ACT first applies the jet VJP (bar_Z from H, a1, bar_H).  Stage 2 reduces the tiles of
// each channel in a fixed order.  Layout of `partials` as the reference's binding
// allocates it: [(points+7)/8][C][DIM+1] (experiments/pinn_v8/native.py:146).
constexpr int kPointTile = 8;

template <int DIM, bool ACT>
__global__ void __launch_bounds__(kHookThreads)
    coordinate_wgrad_partials(const double* __restrict__ dz_or_h, const double* __restrict__ aux,
                              const double* __restrict__ hbar, const double* __restrict__ x,
                              double* __restrict__ partials, int64_t full, int64_t value, int channels,
                              int64_t tiles) {
  constexpr int Q = Q_<DIM>::v;
  const int64_t points = full + value;
  const int64_t total = tiles * channels;
  for (int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += int64_t(gridDim.x) * blockDim.x) {
    const int64_t tile = idx / channels;
    const int c = int(idx % channels);
    double acc[DIM + 1];
#pragma unroll
    for (int a = 0; a <= DIM; ++a) acc[a] = 0.0;
    for (int k = 0; k < kPointTile; ++k) {
      const int64_t p = tile * kPointTile + k;
      if (p >= points) break;
      const double* xp = x + p * DIM;
      if (p < full) {
        const int64_t base = p * Q * channels + c;
        double zb[Q];
        if constexpr (ACT) {
          double hv[Q], hb[Q];
#pragma unroll
          for (int s = 0; s < Q; ++s) {
            hv[s] = dz_or_h[base + int64_t(s) * channels];
            hb[s] = hbar[base + int64_t(s) * channels];
          }
          vjp_full<DIM>(hv, aux[p * channels + c], hb, zb);
        } else {
#pragma unroll
          for (int s = 0; s < Q; ++s) zb[s] = dz_or_h[base + int64_t(s) * channels];
        }
        acc[DIM] += zb[0];
        // the dense contraction bar_Z^T X of the coordinate jets, structural zeros included:
        // a NaN or Inf in any slot reaches dW as it does through 0 * NaN in a GEMM (the
        // reference's experiments/pinn_v8/coordinate_wgrad.cuh:19-31 keeps the same terms)
#pragma unroll
        for (int a = 0; a < DIM; ++a) {
          double v = zb[0] * xp[a];
#pragma unroll
          for (int s = 1; s < Q; ++s) v += zb[s] * (s == unit_row<DIM>(a) ? 1.0 : 0.0);
          acc[a] += v;
        }
      } else {
        const int64_t r = (full * Q + (p - full)) * channels + c;
        const double z0 = ACT ? hbar[r] * aux[p * channels + c] : dz_or_h[r];
        acc[DIM] += z0;
#pragma unroll
        for (int a = 0; a < DIM; ++a) acc[a] += z0 * xp[a];
      }
    }
#pragma unroll
    for (int a = 0; a <= DIM; ++a) partials[idx * (DIM + 1) + a] = acc[a];
  }
}

template <int DIM>
__global__ void __launch_bounds__(kHookThreads)
    coordinate_wgrad_finish(const double* __restrict__ partials, double* __restrict__ dw, double* __restrict__ db,
                            int channels, int64_t tiles) {
  // one block per channel: threads take tiles in a strided fixed order, then a fixed tree
  __shared__ double red[kHookThreads][DIM + 1];
  const int c = blockIdx.x;
  double acc[DIM + 1];
#pragma unroll
  for (int a = 0; a <= DIM; ++a) acc[a] = 0.0;
  for (int64_t t = threadIdx.x; t < tiles; t += blockDim.x) {
    const double* pp = partials + (t * channels + c) * (DIM + 1);
#pragma unroll
    for (int a = 0; a <= DIM; ++a) acc[a] += pp[a];
  }
#pragma unroll
  for (int a = 0; a <= DIM; ++a) red[threadIdx.x][a] = acc[a];
  __syncthreads();
  for (int step = kHookThreads / 2; step > 0; step >>= 1) {
    if (threadIdx.x < step) {
#pragma unroll
      for (int a = 0; a <= DIM; ++a) red[threadIdx.x][a] += red[threadIdx.x + step][a];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
#pragma unroll
    for (int a = 0; a < DIM; ++a) dw[int64_t(c) * DIM + a] = red[0][a];
    db[c] = red[0][DIM];
  }
}

// ---------------------------------------------------------------- residual + loss seed
// One point per thread: interior Q10 (u, v, p) jets -> the nine residuals' loss and
// seed; boundary value rows -> bc * w * err^2 and its seed.  partial_loss[block] is the
// fixed-order tree sum of the block's 128 points (the reference's caller sums it).
__global__ void __launch_bounds__(kHookThreads)
    loss_seed_kernel(const double* __restrict__ jets, const double* __restrict__ boundary,
                     const double* __restrict__ pde_w, const double* __restrict__ bnd_w,
                     const double* __restrict__ target, double* __restrict__ interior_seed,
                     double* __restrict__ boundary_seed, double* __restrict__ partial_loss, int64_t ni, int64_t nb,
                     int64_t stride, double nu, double gamma, double bc) {
  __shared__ double red[kHookThreads];
  const int64_t point = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  double loss = 0.0;
  if (point < ni) {
    double y[30], dy[30];
#pragma unroll
    for (int k = 0; k < 30; ++k) y[k] = jets[point * 30 + k];
    loss = seed_uvp_2d(y, pde_w[point], nu, gamma, dy);
#pragma unroll
    for (int k = 0; k < 30; ++k) interior_seed[point * 30 + k] = dy[k];
  } else if (point < ni + nb) {
    const int64_t b = point - ni;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      const double err = boundary[b * stride + k] - target[b * 3 + k];
      const double wgt = bnd_w[b * 3 + k];
      loss += bc * wgt * err * err;
      boundary_seed[b * 3 + k] = 2.0 * bc * wgt * err;
    }
  }
  red[threadIdx.x] = loss;
  __syncthreads();
  for (int step = kHookThreads / 2; step > 0; step >>= 1) {
    if (threadIdx.x < step) red[threadIdx.x] += red[threadIdx.x + step];
    __syncthreads();
  }
  if (threadIdx.x == 0) partial_loss[blockIdx.x] = red[0];
}

unsigned grid_of(int64_t n) {
  const int64_t b = blocks_for(n);
  return unsigned(b > 65535 * 16 ? 65535 * 16 : b);
}

bool packed_sizes_ok(int dim, int64_t full, int64_t value, int channels, int widest) {
  if ((dim != 2 && dim != 3) || full < 0 || value < 0 || channels < 1) return false;
  const int64_t q = dim == 2 ? 10 : 20;
  if (full > (INT64_MAX - value) / q) return false;
  const int64_t rows = full * q + value;
  return rows <= INT64_MAX / int64_t(sizeof(double)) / (widest > channels ? widest : channels);
}

}  // namespace
}  // namespace flashns_b200

using namespace flashns_b200;

extern "C" {

int flashns_v8_activation(int dimension, int backward, const double* input, const double* auxiliary,
                          const double* seed, double* output, double* output_auxiliary, int64_t full_points,
                          int64_t value_points, int channels, cudaStream_t stream) {
  if (!packed_sizes_ok(dimension, full_points, value_points, channels, channels) || (backward != 0 && backward != 1))
    return int(cudaErrorInvalidValue);
  const int64_t count = (full_points + value_points) * channels;
  if (count == 0) return int(cudaSuccess);
  if (!input || !output || (backward ? (!auxiliary || !seed) : !output_auxiliary)) return int(cudaErrorInvalidValue);
  const unsigned g = grid_of(count);
  if (dimension == 2 && backward) packed_activation<2, true><<<g, kHookThreads, 0, stream>>>(input, auxiliary, seed, output, output_auxiliary, full_points, value_points, channels);
  else if (dimension == 2) packed_activation<2, false><<<g, kHookThreads, 0, stream>>>(input, auxiliary, seed, output, output_auxiliary, full_points, value_points, channels);
  else if (backward) packed_activation<3, true><<<g, kHookThreads, 0, stream>>>(input, auxiliary, seed, output, output_auxiliary, full_points, value_points, channels);
  else packed_activation<3, false><<<g, kHookThreads, 0, stream>>>(input, auxiliary, seed, output, output_auxiliary, full_points, value_points, channels);
  return int(cudaGetLastError());
}

static int coordinate_affine_launch(bool act, int dimension, const double* coordinates, const double* weight,
                                    const double* bias, double* output, double* auxiliary, int64_t full,
                                    int64_t value, int channels, cudaStream_t stream) {
  if (!packed_sizes_ok(dimension, full, value, channels, dimension)) return int(cudaErrorInvalidValue);
  const int64_t count = (full + value) * channels;
  if (count == 0) return int(cudaSuccess);
  if (!coordinates || !weight || !bias || !output || (act && !auxiliary)) return int(cudaErrorInvalidValue);
  const unsigned g = grid_of(count);
  if (dimension == 2 && act) coordinate_affine<2, true><<<g, kHookThreads, 0, stream>>>(coordinates, weight, bias, output, auxiliary, full, value, channels);
  else if (dimension == 2) coordinate_affine<2, false><<<g, kHookThreads, 0, stream>>>(coordinates, weight, bias, output, auxiliary, full, value, channels);
  else if (act) coordinate_affine<3, true><<<g, kHookThreads, 0, stream>>>(coordinates, weight, bias, output, auxiliary, full, value, channels);
  else coordinate_affine<3, false><<<g, kHookThreads, 0, stream>>>(coordinates, weight, bias, output, auxiliary, full, value, channels);
  return int(cudaGetLastError());
}

int flashns_v8_coordinate_affine(int dimension, const double* coordinates, const double* weight, const double* bias,
                                 double* output, int64_t full_points, int64_t value_points, int channels,
                                 cudaStream_t stream) {
  return coordinate_affine_launch(false, dimension, coordinates, weight, bias, output, nullptr, full_points,
                                  value_points, channels, stream);
}

int flashns_v8_coordinate_affine_activation(int dimension, const double* coordinates, const double* weight,
                                            const double* bias, double* hidden, double* auxiliary,
                                            int64_t full_points, int64_t value_points, int channels,
                                            cudaStream_t stream) {
  return coordinate_affine_launch(true, dimension, coordinates, weight, bias, hidden, auxiliary, full_points,
                                  value_points, channels, stream);
}

int flashns_v8_tail3(int dimension, int fused, const double* d, const double* weight, const double* hidden,
                     const double* auxiliary, double* output, int64_t full_points, int64_t value_points, int channels,
                     cudaStream_t stream) {
  if (!packed_sizes_ok(dimension, full_points, value_points, channels, 3) || (fused != 0 && fused != 1))
    return int(cudaErrorInvalidValue);
  const int64_t count = (full_points + value_points) * channels;
  if (count == 0) return int(cudaSuccess);
  if (!d || !weight || !output || (fused && (!hidden || !auxiliary))) return int(cudaErrorInvalidValue);
  const unsigned g = grid_of(count);
  if (dimension == 2 && fused) packed_tail3<2, true><<<g, kHookThreads, 0, stream>>>(d, weight, hidden, auxiliary, output, full_points, value_points, channels);
  else if (dimension == 2) packed_tail3<2, false><<<g, kHookThreads, 0, stream>>>(d, weight, hidden, auxiliary, output, full_points, value_points, channels);
  else if (fused) packed_tail3<3, true><<<g, kHookThreads, 0, stream>>>(d, weight, hidden, auxiliary, output, full_points, value_points, channels);
  else packed_tail3<3, false><<<g, kHookThreads, 0, stream>>>(d, weight, hidden, auxiliary, output, full_points, value_points, channels);
  return int(cudaGetLastError());
}

static int coordinate_wgrad_launch(bool act, int dimension, const double* dz_or_h, const double* aux,
                                   const double* hbar, const double* coordinates, double* partials, double* dw,
                                   double* db, int64_t full, int64_t value, int channels, cudaStream_t stream) {
  if (!packed_sizes_ok(dimension, full, value, channels, dimension)) return int(cudaErrorInvalidValue);
  const int64_t points = full + value;
  const int64_t tiles = (points + kPointTile - 1) / kPointTile;
  if (tiles > INT64_MAX / int64_t(sizeof(double)) / (dimension + 1) / channels) return int(cudaErrorInvalidValue);
  if (!dw || !db || (points && (!dz_or_h || !coordinates || !partials || (act && (!aux || !hbar)))))
    return int(cudaErrorInvalidValue);
  if (tiles) {
    const unsigned g = grid_of(tiles * channels);
    if (dimension == 2 && act) coordinate_wgrad_partials<2, true><<<g, kHookThreads, 0, stream>>>(dz_or_h, aux, hbar, coordinates, partials, full, value, channels, tiles);
    else if (dimension == 2) coordinate_wgrad_partials<2, false><<<g, kHookThreads, 0, stream>>>(dz_or_h, aux, hbar, coordinates, partials, full, value, channels, tiles);
    else if (act) coordinate_wgrad_partials<3, true><<<g, kHookThreads, 0, stream>>>(dz_or_h, aux, hbar, coordinates, partials, full, value, channels, tiles);
    else coordinate_wgrad_partials<3, false><<<g, kHookThreads, 0, stream>>>(dz_or_h, aux, hbar, coordinates, partials, full, value, channels, tiles);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return int(e);
  }
  // even an empty segment owns its parameter gradients: the finish writes zeros then
  if (dimension == 2) coordinate_wgrad_finish<2><<<channels, kHookThreads, 0, stream>>>(partials, dw, db, channels, tiles);
  else coordinate_wgrad_finish<3><<<channels, kHookThreads, 0, stream>>>(partials, dw, db, channels, tiles);
  return int(cudaGetLastError());
}

int flashns_v8_coordinate_wgrad(int dimension, const double* derivative, const double* coordinates, double* partials,
                                double* weight_gradient, double* bias_gradient, int64_t full_points,
                                int64_t value_points, int channels, cudaStream_t stream) {
  return coordinate_wgrad_launch(false, dimension, derivative, nullptr, nullptr, coordinates, partials,
                                 weight_gradient, bias_gradient, full_points, value_points, channels, stream);
}

int flashns_v8_coordinate_activation_wgrad(int dimension, const double* hidden, const double* auxiliary,
                                           const double* seed, const double* coordinates, double* partials,
                                           double* weight_gradient, double* bias_gradient, int64_t full_points,
                                           int64_t value_points, int channels, cudaStream_t stream) {
  return coordinate_wgrad_launch(true, dimension, hidden, auxiliary, seed, coordinates, partials, weight_gradient,
                                 bias_gradient, full_points, value_points, channels, stream);
}

int flashns_v8_loss_seed(const double* jets, const double* boundary, const double* pde_weights,
                         const double* boundary_weights, const double* target, double* interior_seed,
                         double* boundary_seed, double* partial_loss, int64_t ni, int64_t nb, int64_t boundary_stride,
                         double nu, double gamma, double bc_scale, cudaStream_t stream) {
  if (ni < 0 || nb < 0 || boundary_stride < 3) return int(cudaErrorInvalidValue);
  if (ni + nb == 0) return int(cudaSuccess);
  if (!partial_loss || (ni && (!jets || !pde_weights || !interior_seed)) ||
      (nb && (!boundary || !boundary_weights || !target || !boundary_seed)))
    return int(cudaErrorInvalidValue);
  const int64_t blocks = blocks_for(ni + nb);
  if (blocks > 2147483647LL) return int(cudaErrorInvalidConfiguration);
  loss_seed_kernel<<<unsigned(blocks), kHookThreads, 0, stream>>>(jets, boundary, pde_weights, boundary_weights, target,
                                                                 interior_seed, boundary_seed, partial_loss, ni, nb,
                                                                 boundary_stride, nu, gamma, bc_scale);
  return int(cudaGetLastError());
}

int flashns_stable_activation(int dim, bool backward, const double* value, const double* adjoint, const double* aux_in,
                              double* output, double* aux_out, size_t batch, size_t channels, cudaStream_t stream) {
  if ((dim != 2 && dim != 3) || (channels && batch > SIZE_MAX / 20 / sizeof(double) / channels))
    return int(cudaErrorInvalidValue);
  if (batch == 0 || channels == 0) return int(cudaSuccess);
  if (!value || !output || (backward ? (!adjoint || !aux_in) : !aux_out)) return int(cudaErrorInvalidValue);
  const size_t n = batch * channels, bytes = n * (dim == 2 ? 10 : 20) * sizeof(double);
  if (overlaps(output, bytes, value, bytes) ||
      (backward && (overlaps(output, bytes, adjoint, bytes) || overlaps(output, bytes, aux_in, n * sizeof(double)))) ||
      (!backward && (overlaps(aux_out, n * sizeof(double), output, bytes) || overlaps(aux_out, n * sizeof(double), value, bytes))))
    return int(cudaErrorInvalidValue);
  const unsigned g = grid_of(int64_t(n));
  if (dim == 2 && backward) dense_activation<2, true><<<g, kHookThreads, 0, stream>>>(value, adjoint, aux_in, output, aux_out, batch, channels);
  else if (dim == 2) dense_activation<2, false><<<g, kHookThreads, 0, stream>>>(value, adjoint, aux_in, output, aux_out, batch, channels);
  else if (backward) dense_activation<3, true><<<g, kHookThreads, 0, stream>>>(value, adjoint, aux_in, output, aux_out, batch, channels);
  else dense_activation<3, false><<<g, kHookThreads, 0, stream>>>(value, adjoint, aux_in, output, aux_out, batch, channels);
  return int(cudaGetLastError());
}

int flashns_stable_tail3(int dim, bool fused, const double* d, const double* weight, const double* hidden,
                         const double* aux, double* output, size_t batch, size_t channels, cudaStream_t stream) {
  if ((dim != 2 && dim != 3) || (channels && batch > SIZE_MAX / 20 / sizeof(double) / channels) ||
      batch > SIZE_MAX / 20 / 3 / sizeof(double))
    return int(cudaErrorInvalidValue);
  if (batch == 0 || channels == 0) return int(cudaSuccess);
  if (!d || !weight || !output || (fused && (!hidden || !aux))) return int(cudaErrorInvalidValue);
  const size_t n = batch * channels, q = dim == 2 ? 10 : 20, bytes = n * q * sizeof(double);
  if (overlaps(output, bytes, d, batch * q * 3 * sizeof(double)) ||
      overlaps(output, bytes, weight, 3 * channels * sizeof(double)) ||
      (fused && (overlaps(output, bytes, hidden, bytes) || overlaps(output, bytes, aux, n * sizeof(double)))))
    return int(cudaErrorInvalidValue);
  const unsigned g = grid_of(int64_t(n));
  if (dim == 2 && fused) dense_tail3<2, true><<<g, kHookThreads, 0, stream>>>(d, weight, hidden, aux, output, batch, channels);
  else if (dim == 2) dense_tail3<2, false><<<g, kHookThreads, 0, stream>>>(d, weight, hidden, aux, output, batch, channels);
  else if (fused) dense_tail3<3, true><<<g, kHookThreads, 0, stream>>>(d, weight, hidden, aux, output, batch, channels);
  else dense_tail3<3, false><<<g, kHookThreads, 0, stream>>>(d, weight, hidden, aux, output, batch, channels);
  return int(cudaGetLastError());
}

int flashns_stable_dgrad_vjp(int dim, bool fused, const double* d, const double* w, const double* h, const double* aux,
                             double* out, int batch, int cout, int cin, cudaStream_t stream) {
  if ((dim != 2 && dim != 3) || batch < 0 || cin < 0 || cout <= 0 || batch > INT_MAX / 20) return int(cudaErrorInvalidValue);
  if (batch == 0 || cin == 0) return int(cudaSuccess);
  if (!d || !w || !out || (fused && (!h || !aux))) return int(cudaErrorInvalidValue);
  const size_t q = dim == 2 ? 10 : 20, no = size_t(batch) * q * cin;
  if (overlaps(out, no * 8, d, size_t(batch) * q * cout * 8) || overlaps(out, no * 8, w, size_t(cout) * cin * 8) ||
      (fused && (overlaps(out, no * 8, h, no * 8) || overlaps(out, no * 8, aux, size_t(batch) * cin * 8))))
    return int(cudaErrorInvalidValue);
  // 64 -> 64 (the reference's nets): the evaluation's TMA-fed backward kernels without
  // their weight gradient; other shapes: the general kernel above
  const auto aligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  // (TMA reads d, cp.async w; the fused kernels prefetch rows of h and aux into L2 in bulk,
  // which wants 16-byte aligned addresses)
  if (cout == 64 && cin == 64 && aligned(d) && aligned(w) && (!fused || (aligned(h) && aligned(aux))) &&
      int64_t(batch) * (dim == 2 ? 10 : 20) <= INT32_MAX / 2)
    return int(flashns_b200::dense_dgrad_64(dim, fused, d, w, h, aux, out, batch, stream));
  if (dim == 2 && fused) return int(launch_dense_dgrad<2, true>(d, w, h, aux, out, batch, cout, cin, stream));
  if (dim == 2) return int(launch_dense_dgrad<2, false>(d, w, h, aux, out, batch, cout, cin, stream));
  if (fused) return int(launch_dense_dgrad<3, true>(d, w, h, aux, out, batch, cout, cin, stream));
  return int(launch_dense_dgrad<3, false>(d, w, h, aux, out, batch, cout, cin, stream));
}

int flashns_stable_dgrad_shared_bytes() { return int(flashns_b200::dgrad_smem_bytes_for<2>(64, 64)); }

}  // extern "C"

// Residual values of a head at interior points (src/flashns/ns_seed.py:54-64 for the
// (u, v, p) head): out[n][k] for the head's residual polynomials.
namespace flashns_b200 {
namespace {
template <int HEAD, int DIM>
__global__ void __launch_bounds__(kHookThreads)
    residual_values(const double* __restrict__ jets, double nu, double* __restrict__ out, int64_t n) {
  constexpr int Q = Q_<DIM>::v, NF = HEAD == FLASHNS_B200_HEAD_UVP ? 3 : 2, NR = HEAD == FLASHNS_B200_HEAD_UVP ? 9 : 2;
  for (int64_t p = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; p < n; p += int64_t(gridDim.x) * blockDim.x) {
    double y[Q * NF], r[NR];
#pragma unroll
    for (int k = 0; k < Q * NF; ++k) y[k] = jets[p * Q * NF + k];
    if constexpr (HEAD == FLASHNS_B200_HEAD_UVP) residuals_uvp_2d(y, nu, r);
    else if constexpr (DIM == 2) residuals_psi_2d(y, nu, r);
    else residuals_psi_3d(y, nu, r);
#pragma unroll
    for (int k = 0; k < NR; ++k) out[p * NR + k] = r[k];
  }
}
}  // namespace
}  // namespace flashns_b200

extern "C" int flashns_b200_residuals(int head, int dim, const double* jets, double nu, double* out, int64_t n,
                                      cudaStream_t stream) {
  if (n < 0 || (head == FLASHNS_B200_HEAD_UVP && dim != 2) || (dim != 2 && dim != 3) ||
      (head != FLASHNS_B200_HEAD_UVP && head != FLASHNS_B200_HEAD_PSI))
    return int(cudaErrorInvalidValue);
  if (n == 0) return int(cudaSuccess);
  if (!jets || !out) return int(cudaErrorInvalidValue);
  const unsigned g = grid_of(n);
  if (head == FLASHNS_B200_HEAD_UVP) residual_values<FLASHNS_B200_HEAD_UVP, 2><<<g, kHookThreads, 0, stream>>>(jets, nu, out, n);
  else if (dim == 2) residual_values<FLASHNS_B200_HEAD_PSI, 2><<<g, kHookThreads, 0, stream>>>(jets, nu, out, n);
  else residual_values<FLASHNS_B200_HEAD_PSI, 3><<<g, kHookThreads, 0, stream>>>(jets, nu, out, n);
  return int(cudaGetLastError());
}

// ---- plan-based dense dgrad (+ jet VJP) under the reference's Hopper names
// (experiments/cuda_jet_hopper/hopper.cu:287-353): the same argument meaning, limits and
// error codes, so the reference's binding (experiments/cuda_jet_hopper/hopper.py) can load
// this library on B200.  The plan keeps D, W and the sizes; a launch runs the DMMA
// dense_dgrad (+ VJP) above.
namespace flashns_b200 {
namespace {
struct DgradPlan {
  const double* d;
  const double* w;
  int batch, cout, cin, q;
};

template <int DIM, bool FUSED>
int dgrad_resources(long long* values) {
  cudaFuncAttributes attr;
  cudaError_t e = cudaFuncGetAttributes(&attr, dense_dgrad<DIM, FUSED>);
  if (e != cudaSuccess) return int(e);
  const size_t smem = dgrad_smem_bytes_for<DIM>(64, 64);  // the shape of the reference's plans
  e = cudaFuncSetAttribute(dense_dgrad<DIM, FUSED>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           int(dgrad_smem_bytes<DIM>(kDgResidentRows)));
  if (e != cudaSuccess) return int(e);
  int blocks = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, dense_dgrad<DIM, FUSED>, kDgThreads, smem);
  if (e != cudaSuccess) return int(e);
  values[0] = attr.numRegs;
  values[1] = kDgThreads;
  values[2] = int64_t(smem);  // dynamic shared memory per CTA
  values[3] = attr.sharedSizeBytes;
  values[4] = attr.localSizeBytes;
  values[5] = blocks;
  values[6] = attr.maxDynamicSharedSizeBytes;
  values[7] = attr.binaryVersion;
  values[8] = attr.ptxVersion;
  return int(cudaSuccess);
}
}  // namespace
}  // namespace flashns_b200

extern "C" {

int flashns_hopper_initialize(void) { return int(cudaSuccess); }  // no kernel attribute to set

int flashns_hopper_resources(int dim, bool fused, long long* values) {
  using namespace flashns_b200;
  if (!values || (dim != 2 && dim != 3)) return int(cudaErrorInvalidValue);
  if (dim == 2) return fused ? dgrad_resources<2, true>(values) : dgrad_resources<2, false>(values);
  return fused ? dgrad_resources<3, true>(values) : dgrad_resources<3, false>(values);
}

int flashns_hopper_create(int dim, const double* d, const double* w, int batch, int cout, int cin, void** result) {
  using namespace flashns_b200;
  if (!result) return int(cudaErrorInvalidValue);
  *result = nullptr;
  if ((dim != 2 && dim != 3) || !d || !w || batch <= 0 || batch > INT_MAX / 20 || (cout != 32 && cout != 64) ||
      (cin != 32 && cin != 64) || (reinterpret_cast<uintptr_t>(d) & 15) || (reinterpret_cast<uintptr_t>(w) & 15))
    return int(cudaErrorInvalidValue);
  DgradPlan* plan = new (std::nothrow) DgradPlan{d, w, batch, cout, cin, dim == 2 ? 10 : 20};
  if (!plan) return int(cudaErrorMemoryAllocation);
  *result = plan;
  return int(cudaSuccess);
}

void flashns_hopper_destroy(void* plan) { delete static_cast<flashns_b200::DgradPlan*>(plan); }

int flashns_hopper_launch(void* handle, int dim, bool fused, const double* hidden, const double* aux, double* output,
                          cudaStream_t stream) {
  using namespace flashns_b200;
  if (!handle || !output || (dim != 2 && dim != 3) || (fused && (!hidden || !aux))) return int(cudaErrorInvalidValue);
  const DgradPlan& p = *static_cast<const DgradPlan*>(handle);
  if (p.q != (dim == 2 ? 10 : 20)) return int(cudaErrorInvalidValue);
  return flashns_stable_dgrad_vjp(dim, fused, p.d, p.w, hidden, aux, output, p.batch, p.cout, p.cin, stream);
}

}  // extern "C"
