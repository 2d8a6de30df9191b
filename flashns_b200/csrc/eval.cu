// Fused FP64 loss + parameter-gradient evaluation of a packed jet MLP (sm_100a).
//
// Replaces the evaluation behind PackedPINN.__call__ (src/flashns/pinn_packed.py:93-191)
// and its per-stage CUDA hooks (experiments/pinn_v8/native.cu) with one chain of
// persistent kernels per evaluation:
//
//   pack_params   flat [W_0..W_L, b_0..b_L] -> zero-padded per-layer buffers
//   first_layer   coordinates -> layer-0 affine -> stable tanh jet  (H_1, a1_1)
//   fwd_layer     H_l -> DMMA GEMM with W_l -> bias on order-0 rows -> tanh jet epilogue
//   head_layer    output layer + residual seed + output-layer wgrad + dgrad + jet VJP
//   bwd_layer     DMMA dgrad D_{l+1} W_l -> jet VJP epilogue (D_l); the layer-1 instance
//                 contracts D_1 with the coordinate jets instead of storing it
//   wgrad         dW_l = D_{l+1}^T H_l, split over rows, DMMA, deterministic partials
//   reduce        fixed-order sum of all partials -> grad[P] and loss
//
// Layout in HBM: packed rows [interior points x Q ; boundary points x QB] x C,
// FP64 row-major, C padded to 32/64/128 with zero weights (padded channels stay
// exactly zero through the chain).
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <cuda.h>
#include <mutex>
#include <new>
#include <type_traits>
#include <vector>

#include "common.cuh"
#include "jets_generated.cuh"
#include "residual_generated.cuh"
#include "flashns_b200.h"

namespace flashns_b200 {

constexpr int kThreads = 256;
constexpr int kStages = 2;
constexpr int KC = 32;       // k-chunk (doubles) per pipeline stage
constexpr int LDC = KC + 4;  // padded chunk row: conflict-free FP64 fragment loads
constexpr int kMaxAffine = 16;
// set by a kernel whose bounded wait on a bulk copy gave up (read by flashns_b200_device_fault)
__device__ int g_device_fault = 0;
// the dense dgrad (+ VJP) of a 64 -> 64 layer on the evaluation's backward kernels (defined
// with the host launchers below; called by the reference-ABI hook in hooks.cu)
cudaError_t dense_dgrad_64(int dim, bool fused, const double* d, const double* w, const double* h,
                           const double* aux, double* out, int batch, cudaStream_t stream);

// Self-test of the bounded wait: an mbarrier that nothing arrives at.  The wait gives up
// after `spins` polls, raises the fault word and the kernel returns normally.
__global__ void wait_timeout_probe(unsigned spins, int* gave_up) {
  __shared__ uint64_t bar;
  mbar_init(&bar, 1);
  __syncwarp();
  const bool ok = mbar_wait(&bar, 0, spins);
  if (!ok) atomicExch(&g_device_fault, 1);
  *gave_up = ok ? 0 : 1;
  mbar_inval(&bar);
}

struct Geometry {
  int64_t ni, nb;  // interior (full-jet) and boundary points
  int64_t rows;    // ni*Q + nb*QB
};

template <int DIM, int ORDER>
struct Jet;
#define FLASHNS_JET(D, O, N)                                                                  \
  template <>                                                                                 \
  struct Jet<D, O> {                                                                          \
    static constexpr int n = N;                                                               \
    __device__ static void fwd(const double* z, double* h, double& a) { jet_fwd_##D##d##O(z, h, a); } \
    __device__ static void vjp(const double* h, double a, const double* hb, double* zb) {     \
      jet_vjp_##D##d##O(h, a, hb, zb);                                                        \
    }                                                                                         \
  };
FLASHNS_JET(2, 0, 1)
FLASHNS_JET(2, 1, 3)
FLASHNS_JET(2, 3, 10)
FLASHNS_JET(3, 0, 1)
FLASHNS_JET(3, 1, 4)
FLASHNS_JET(3, 3, 20)
#undef FLASHNS_JET

// ----------------------------------------------------------------------------------
// Tiles of the DMMA kernels.  The GEMM is computed transposed: MMA M = channels,
// MMA N = packed rows, so a thread's accumulators hold, for two channels per m16 tile,
// the rows 8j+2t and 8j+2t+1 of every n8 tile j.  Those rows are the S = Q jet
// coefficients of one point ("thread column"): most kernels permute the rows in shared
// memory (tile_slot); the fused backward keeps its TMA-loaded rows in global order and folds
// the permutation into its fragment addresses.  The tanh-jet epilogue and its
// VJP then run entirely in registers.  One m16 tile of channels per warp keeps 20 (2-D) or
// 40 (3-D) accumulators per thread; each kernel picks its warp count (FwdTile, BwdTile,
// FusedTile, HeadTile).
template <int DIM, int CP, int WARPS>
struct MmaTile {
  static constexpr int S = Basis<DIM>::Q;     // slots per thread column
  static constexpr int NT = S / 2;            // n8 tiles per warp
  static constexpr int MT = 1;                // m16 tiles per warp
  static constexpr int WCH = 16 * MT;         // channels per warp
  static constexpr int NWARPS = WARPS;
  static constexpr int THREADS = 32 * WARPS;
  static constexpr int WC = CP / WCH;         // warps along channels
  static constexpr int WR = WARPS / WC;       // warp row groups
  static constexpr int TC = 4 * WR;           // thread columns per tile
  static constexpr int TR = TC * S;           // packed rows per tile
  static_assert(CP % WCH == 0 && WC >= 1 && WARPS % WC == 0, "unsupported padded width");
};

// Forward tiles: the 2-D 64-wide layer runs two 8-warp CTAs per SM (80-row tiles), so one
// CTA's jet epilogue and stores overlap the other's MMAs; 128-wide layers run one 16-warp
// CTA per SM, the rest one 8-warp CTA.  Every shape keeps W_l (up to 128 inputs) resident.
template <int DIM, int CP>
struct FwdTile : MmaTile<DIM, CP, CP >= 128 ? 16 : 8> {
  static constexpr int MINB = (DIM == 2 && CP == 64) ? 2 : 1;  // CTAs per SM
};

// Interior tiles carry TC points (Q rows each); boundary tiles carry TC*PS points of
// QB rows (QB = 1 value rows, QB = DIM+1 first-order rows).
template <int DIM, int BO, int TC>
struct Tiles {
  static constexpr int Q = Basis<DIM>::Q;
  static constexpr int QB = BO ? DIM + 1 : 1;
  static constexpr int PS = Q / QB;
  __host__ __device__ static int64_t interior(int64_t ni) { return (ni + TC - 1) / TC; }
  __host__ __device__ static int64_t boundary(int64_t nb) { return (nb + int64_t(TC) * PS - 1) / (int64_t(TC) * PS); }
  // the tile's points: the first packed point index (interior, then boundary) and the count
  __device__ static void points(const Geometry& g, int64_t nint, int64_t tile, int64_t& p0, int64_t& n) {
    if (tile < nint) {
      p0 = tile * TC;
      n = (g.ni - p0) < TC ? (g.ni - p0) : TC;
    } else {
      const int64_t b0 = (tile - nint) * (int64_t(TC) * PS);
      n = (g.nb - b0) < int64_t(TC) * PS ? (g.nb - b0) : int64_t(TC) * PS;
      p0 = g.ni + b0;
    }
  }
  __device__ static int64_t row(const Geometry& g, int64_t nint, int64_t tile, int tc, int s) {
    if (tile < nint) {
      const int64_t p = tile * TC + tc;
      return p < g.ni ? p * Q + s : -1;
    }
    if (s >= PS * QB) return -1;
    const int64_t b = (tile - nint) * (int64_t(TC) * PS) + int64_t(tc) * PS + s / QB;
    return b < g.nb ? g.ni * Q + b * QB + s % QB : -1;
  }
};

// smem row r -> (thread column, slot) for the permuted tile layout
template <int S>
__device__ __forceinline__ void tile_slot(int r, int& tc, int& s) {
  const int wr = r / (4 * S), within = r % (4 * S);
  const int j = within >> 3, rem = within & 7;
  tc = wr * 4 + (rem >> 1);
  s = 2 * j + (rem & 1);
}

constexpr size_t kMaxSmem = 227 * 1024;  // dynamic shared memory per CTA on sm_100
constexpr int kMaxWidth = 128;            // widest padded layer
// forward: activation ring [stage][TR][LDC] + resident W_l [CP][kin+4] + rowmap[2][TR]
// (int64) + one mbarrier per stage
template <int DIM, int CP>
constexpr size_t fwd_smem_bytes(int kin) {
  using T = FwdTile<DIM, CP>;
  return sizeof(double) * (size_t(kStages) * T::TR * LDC + size_t(CP) * (kin + 4) + 2 * size_t(T::TR) + kStages);
}
// Backward tiles (bwd_layer): the tile's H_l rows stay in shared memory next to the seed and
// weight ring, so 3-D layers use 8-warp (4-warp for 32 channels) CTAs to fit.
template <int DIM, int CP>
struct BwdTile : MmaTile<DIM, CP, DIM == 2 ? (CP >= 64 ? 16 : 8) : (CP >= 64 ? 8 : 4)> {};

template <int DIM, int CP>
constexpr size_t bwd_group_doubles() {
  using T = BwdTile<DIM, CP>;
  return size_t(kStages) * (size_t(T::TR) * LDC + size_t(KC) * (CP + 4)) + size_t(T::TR) * (CP + 4) + 2 * T::TR;
}
template <int DIM, int CP>
constexpr size_t bwd_smem_bytes() {
  using T = BwdTile<DIM, CP>;
  constexpr size_t a = sizeof(double) * bwd_group_doubles<DIM, CP>();
  constexpr size_t red = sizeof(double) * T::WR * CP * (DIM + 1);
  return a > red ? a : red;
}

// number of tiles of this CTA (grid-stride over tiles)
__device__ __forceinline__ int64_t cta_iterations(int64_t ntiles) {
  return int64_t(blockIdx.x) < ntiles ? (ntiles - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
}

// ----------------------------------------------------------------------------------
// forward hidden layer: H_{l+1} = tanh_jet(H_l W_l^T + b_l on order-0 rows).  W_l stays
// resident in shared memory; activation rows stream through a two-stage ring of 32-column
// chunks as bulk copies (TMA engine, one row per copy), each stage completing on its own
// mbarrier.  The next tile's first chunk is requested before this tile's epilogue.
template <int DIM, int CP, int BO>
__global__ void __launch_bounds__(FwdTile<DIM, CP>::THREADS, FwdTile<DIM, CP>::MINB)
    fwd_layer(const double* __restrict__ hin, int kin, const double* __restrict__ w,
              const double* __restrict__ bias, double* __restrict__ hout, double* __restrict__ a1out,
              Geometry geo) {
  using T = FwdTile<DIM, CP>;
  using TL = Tiles<DIM, BO, T::TC>;
  constexpr int S = T::S, TR = T::TR, Q = TL::Q, QB = TL::QB;
  constexpr int NIS = TR < T::THREADS ? TR : T::THREADS;  // threads issuing row copies
  extern __shared__ __align__(128) double smem[];
  const int tid = threadIdx.x;
  const int LDA = kin + 4;
  double* sB = smem;                     // activation chunks [stage][TR][LDC]
  double* sA = sB + kStages * TR * LDC;  // W_l, resident     [CP][kin+4]
  int64_t* rowmap = reinterpret_cast<int64_t*>(sA + CP * LDA);   // [2][TR]
  uint64_t* bars = reinterpret_cast<uint64_t*>(rowmap + 2 * TR);  // [kStages] stage full
  const int warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int wc = warp % T::WC, wr = warp / T::WC;
  const int nk = kin / KC;
  const int64_t nint = TL::interior(geo.ni);
  const int64_t ntiles = nint + TL::boundary(geo.nb);
  auto fill_rowmap = [&](int64_t tile, int64_t* rm) {
    for (int r = tid; r < TR; r += T::THREADS) {
      int tc, s;
      tile_slot<S>(r, tc, s);
      rm[r] = TL::row(geo, nint, tile, tc, s);
    }
  };
  // chunk kc of the tile's rows into `stage`: rows past the end of a segment are zero-filled
  auto load = [&](int kc, int stage, const int64_t* rm) {
    if (tid >= NIS) return;
    double* dB = sB + stage * TR * LDC;
    unsigned bytes = 0;
    for (int r = tid; r < TR; r += T::THREADS) {
      if (rm[r] >= 0) {
        bytes += KC * sizeof(double);
      } else {
        for (int j = 0; j < KC; ++j) dB[r * LDC + j] = 0.0;
      }
    }
    mbar_arrive_expect_tx(&bars[stage], bytes);
    for (int r = tid; r < TR; r += T::THREADS) {
      const int64_t gr = rm[r];
      if (gr >= 0) bulk_g2s(dB + r * LDC, hin + gr * kin + kc * KC, KC * sizeof(double), &bars[stage]);
    }
  };
  // a thread's channels are fixed for the whole kernel: load their biases once
  double bias_r[T::MT][2];
#pragma unroll
  for (int i = 0; i < T::MT; ++i)
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) bias_r[i][hh] = bias[wc * T::WCH + 16 * i + 8 * hh + g];
  for (int i = tid; i < CP * (kin / 2); i += T::THREADS) {  // W_l once per CTA
    const int r = i / (kin / 2), p = i % (kin / 2);
    cp_async16(sA + r * LDA + 2 * p, w + int64_t(r) * kin + 2 * p, true);
  }
  cp_async_commit();
  if (tid == 0)
    for (int st = 0; st < kStages; ++st) mbar_init(&bars[st], NIS);
  if (int64_t(blockIdx.x) < ntiles) fill_rowmap(blockIdx.x, rowmap);
  cp_async_wait<0>();
  __syncthreads();  // W_l, barriers and the first rowmap visible
  pdl_wait();  // H_l is the predecessor's output
  pdl_trigger();
  if (int64_t(blockIdx.x) < ntiles) load(0, 0, rowmap);
  unsigned parity = 0;  // bit st: phase parity of the next completion of stage st
  int buf = 0;
  for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, buf ^= 1) {
    const int64_t* rm = rowmap + buf * TR;
    int64_t* rn = rowmap + (buf ^ 1) * TR;
    const bool has_next = tile + gridDim.x < ntiles;
    if (has_next) fill_rowmap(tile + gridDim.x, rn);  // published by the barriers below
    double acc[T::MT][T::NT][4];
#pragma unroll
    for (int i = 0; i < T::MT; ++i)
#pragma unroll
      for (int j = 0; j < T::NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.0;
    for (int kc = 0; kc < nk; ++kc) {
      const int stage = kc % kStages;
      const bool ok = mbar_wait(&bars[stage], (parity >> stage) & 1u);
      parity ^= 1u << stage;
      // the barrier also retires the reads of the stage refilled next
      if (__syncthreads_or(!ok)) {
        if (tid == 0) atomicExch(&g_device_fault, 1);
        return;
      }
      if (kc + kStages - 1 < nk) load(kc + kStages - 1, (kc + kStages - 1) % kStages, rm);
      const double* cB = sB + stage * TR * LDC + wr * (4 * S) * LDC;
      const double* cA = sA + wc * T::WCH * LDA + kc * KC;
#pragma unroll
      for (int kk = 0; kk < KC; kk += 8) {
        double a[T::MT][4];
#pragma unroll
        for (int i = 0; i < T::MT; ++i) {
          a[i][0] = cA[(16 * i + g) * LDA + kk + t];
          a[i][1] = cA[(16 * i + g + 8) * LDA + kk + t];
          a[i][2] = cA[(16 * i + g) * LDA + kk + t + 4];
          a[i][3] = cA[(16 * i + g + 8) * LDA + kk + t + 4];
        }
#pragma unroll
        for (int j = 0; j < T::NT; ++j) {
          const double b0 = cB[(8 * j + g) * LDC + kk + t];
          const double b1 = cB[(8 * j + g) * LDC + kk + t + 4];
#pragma unroll
          for (int i = 0; i < T::MT; ++i) mma_m16n8k8(acc[i][j], a[i], b0, b1);
        }
      }
    }
    // the ring is free: request the next tile's first chunk, then run this tile's epilogue
    __syncthreads();
    if (has_next) load(0, 0, rn);
    // epilogue: bias on the order-0 coefficient, stable tanh jet, store H and a1
    const int tc = wr * 4 + t;
    const bool interior = tile < nint;
#pragma unroll
    for (int i = 0; i < T::MT; ++i) {
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int ch = wc * T::WCH + 16 * i + 8 * hh + g;
        double z[S];
#pragma unroll
        for (int s = 0; s < S; ++s) z[s] = acc[i][s >> 1][2 * hh + (s & 1)];
        const double bch = bias_r[i][hh];
        if (interior) {
          const int64_t p = tile * T::TC + tc;
          if (p < geo.ni) {
            double hv[Q], a1;
            z[0] += bch;
            Jet<DIM, 3>::fwd(z, hv, a1);
            double* dst = hout + p * Q * CP + ch;
#pragma unroll
            for (int s = 0; s < Q; ++s) dst[int64_t(s) * CP] = hv[s];
            a1out[p * CP + ch] = a1;
          }
        } else {
#pragma unroll
          for (int kq = 0; kq < TL::PS; ++kq) {
            const int64_t b = (tile - nint) * (int64_t(T::TC) * TL::PS) + int64_t(tc) * TL::PS + kq;
            if (b < geo.nb) {
              double zz[QB], hv[QB], a1;
#pragma unroll
              for (int c = 0; c < QB; ++c) zz[c] = z[kq * QB + c];
              zz[0] += bch;
              Jet<DIM, BO ? 1 : 0>::fwd(zz, hv, a1);
              double* dst = hout + (geo.ni * Q + b * QB) * CP + ch;
#pragma unroll
              for (int c = 0; c < QB; ++c) dst[int64_t(c) * CP] = hv[c];
              a1out[(geo.ni + b) * CP + ch] = a1;
            }
          }
        }
      }
    }
  }
  if (tid == 0 && int64_t(blockIdx.x) < ntiles)  // all waits retired before the last ring barrier
    for (int st = 0; st < kStages; ++st) mbar_inval(&bars[st]);
}

// ----------------------------------------------------------------------------------
// backward hidden layer: D_l = jet_vjp(H_l, a1_l, D_{l+1} W_l), and the bias gradient of
// layer l-1 (sum of D_l over order-0 rows) as per-CTA partials [grid][CP].  FIRST: contract
// D_1 with the coordinate jets (dW_0[c][a] += D[row0][c]*x[a] + D[unit(a)][c],
// db_0[c] += D[row0][c]) into per-CTA partials [grid][CP][DIM+1] instead of storing D_1.
// The tile's H_l rows are staged in shared memory (same row permutation) during the
// mainloop and the jet VJP reads them there; the next tile's H_l is requested after the
// epilogue and lands during the next mainloop.
template <int DIM, int CP, int BO, bool FIRST>
__global__ void __launch_bounds__(BwdTile<DIM, CP>::THREADS, 1)
    bwd_layer(const double* __restrict__ dnext, int kout, const double* __restrict__ w,
              const double* __restrict__ hcur, const double* __restrict__ a1cur, double* __restrict__ dcur,
              const double* __restrict__ x, double* __restrict__ partial, Geometry geo) {
  using T = BwdTile<DIM, CP>;
  using TL = Tiles<DIM, BO, T::TC>;
  constexpr int S = T::S, TR = T::TR, Q = TL::Q, QB = TL::QB, LDA = CP + 4, LDH = CP + 4;
  constexpr int NV = FIRST ? DIM + 1 : 1;  // per-channel partial values
  extern __shared__ __align__(128) double smem[];
  const int tid = threadIdx.x;
  double* sB = smem;   // seed chunks   [stage][TR][LDC]
  double* sA = sB + kStages * TR * LDC;                      // weight chunks [stage][KC][CP+4]
  double* sH = sA + kStages * KC * LDA;                      // H_l tile      [TR][CP+4]
  int64_t* rowmap = reinterpret_cast<int64_t*>(sH + TR * LDH);  // [2][TR]
  const int warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int wc = warp % T::WC, wr = warp / T::WC;
  const int nk = kout / KC;
  const int64_t nint = TL::interior(geo.ni);
  const int64_t ntiles = nint + TL::boundary(geo.nb);
  const int64_t iters = cta_iterations(ntiles);
  double cacc[T::MT][2][NV];
#pragma unroll
  for (int i = 0; i < T::MT; ++i)
#pragma unroll
    for (int hh = 0; hh < 2; ++hh)
#pragma unroll
      for (int a = 0; a < NV; ++a) cacc[i][hh][a] = 0.0;
  auto tile_of = [&](int64_t k) { return k * gridDim.x + blockIdx.x; };
  auto fill_rowmap = [&](int64_t tile, int64_t* rm) {
    for (int r = tid; r < TR; r += T::THREADS) {
      int tc, s;
      tile_slot<S>(r, tc, s);
      rm[r] = TL::row(geo, nint, tile, tc, s);
    }
  };
  auto load = [&](int kc, int stage, const int64_t* rm) {
    double* dB = sB + stage * TR * LDC;
    for (int i = tid; i < TR * (KC / 2); i += T::THREADS) {
      const int r = i / (KC / 2), p = i % (KC / 2);
      const int64_t gr = rm[r];
      cp_async16(dB + r * LDC + 2 * p, dnext + (gr >= 0 ? gr : 0) * kout + kc * KC + 2 * p, gr >= 0);
    }
    double* dA = sA + stage * KC * LDA;
    for (int i = tid; i < KC * (CP / 2); i += T::THREADS) {
      const int r = i / (CP / 2), p = i % (CP / 2);
      cp_async16(dA + r * LDA + 2 * p, w + int64_t(kc * KC + r) * CP + 2 * p, true);
    }
  };
  auto prologue = [&](const int64_t* rm) {
#pragma unroll
    for (int s = 0; s < kStages - 1; ++s) {
      if (s < nk) load(s, s, rm);
      cp_async_commit();
    }
  };
  auto load_h = [&](const int64_t* rm) {  // one commit group, after the tile's first chunk
    for (int i = tid; i < TR * (CP / 2); i += T::THREADS) {
      const int r = i / (CP / 2), p = i % (CP / 2);
      const int64_t gr = rm[r];
      cp_async16(sH + r * LDH + 2 * p, hcur + (gr >= 0 ? gr : 0) * CP + 2 * p, gr >= 0);
    }
    cp_async_commit();
  };
  static_assert(kStages == 2, "commit-group accounting: [chunk 0] [H] [chunk 1] ...");
  int buf = 0;
  pdl_wait();  // D_{l+1} is the predecessor's output
  pdl_trigger();
  if (iters > 0 && tile_of(0) < ntiles) {
    fill_rowmap(tile_of(0), rowmap);
    __syncthreads();
    prologue(rowmap);
    load_h(rowmap);
  }
  for (int64_t k = 0; k < iters; ++k, buf ^= 1) {
    const int64_t tile = tile_of(k);
    const bool valid = tile < ntiles;
    const int64_t* rm = rowmap + buf * TR;
    double acc[T::MT][T::NT][4];
#pragma unroll
    for (int i = 0; i < T::MT; ++i)
#pragma unroll
      for (int j = 0; j < T::NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.0;
    if (valid && tid == 0) {
      // the epilogue reads this tile's a1 rows (a contiguous range): bring them into L2
      int64_t pt0, pts;
      TL::points(geo, nint, tile, pt0, pts);
      prefetch_l2(a1cur + pt0 * CP, uint32_t(pts * CP * sizeof(double)));
    }
    if (valid) {
      for (int kc = 0; kc < nk; ++kc) {
        if (kc == 0) cp_async_wait<1>(); else cp_async_wait<0>();  // chunk 0 may overtake H
        __syncthreads();
        if (kc + kStages - 1 < nk) load(kc + kStages - 1, (kc + kStages - 1) % kStages, rm);
        cp_async_commit();
        const double* cB = sB + (kc % kStages) * TR * LDC + wr * (4 * S) * LDC;
        const double* cA = sA + (kc % kStages) * KC * LDA + wc * T::WCH;
#pragma unroll
        for (int kk = 0; kk < KC; kk += 8) {
          double a[T::MT][4];
#pragma unroll
          for (int i = 0; i < T::MT; ++i) {
            a[i][0] = cA[(kk + t) * LDA + 16 * i + g];
            a[i][1] = cA[(kk + t) * LDA + 16 * i + g + 8];
            a[i][2] = cA[(kk + t + 4) * LDA + 16 * i + g];
            a[i][3] = cA[(kk + t + 4) * LDA + 16 * i + g + 8];
          }
#pragma unroll
          for (int j = 0; j < T::NT; ++j) {
            const double b0 = cB[(8 * j + g) * LDC + kk + t];
            const double b1 = cB[(8 * j + g) * LDC + kk + t + 4];
#pragma unroll
            for (int i = 0; i < T::MT; ++i) mma_m16n8k8(acc[i][j], a[i], b0, b1);
          }
        }
      }
    }
    cp_async_wait<0>();  // the H_l tile (a single-chunk tile still has it in flight)
    __syncthreads();
    const bool has_next = k + 1 < iters && tile_of(k + 1) < ntiles;
    int64_t* rn = rowmap + (buf ^ 1) * TR;
    if (has_next) {
      fill_rowmap(tile_of(k + 1), rn);
      __syncthreads();
      prologue(rn);
    }
    if (!valid) continue;
    const int tc = wr * 4 + t;
    const bool interior = tile < nint;
    // H_l of slot s of this thread column from the shared tile (inverse of tile_slot)
    const double* hrow = sH + (wr * (4 * S) + 2 * t) * LDH;
    auto hslot = [&](int s, int ch) { return hrow[(8 * (s >> 1) + (s & 1)) * LDH + ch]; };
#pragma unroll
    for (int i = 0; i < T::MT; ++i) {
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int ch = wc * T::WCH + 16 * i + 8 * hh + g;
        double dh[S];
#pragma unroll
        for (int s = 0; s < S; ++s) dh[s] = acc[i][s >> 1][2 * hh + (s & 1)];
        if (interior) {
          const int64_t p = tile * T::TC + tc;
          if (p < geo.ni) {
            double hv[Q], zb[Q];
#pragma unroll
            for (int s = 0; s < Q; ++s) hv[s] = hslot(s, ch);
            Jet<DIM, 3>::vjp(hv, a1cur[p * CP + ch], dh, zb);
            if constexpr (FIRST) {
              cacc[i][hh][DIM] += zb[0];
#pragma unroll
              for (int a = 0; a < DIM; ++a) cacc[i][hh][a] += zb[0] * x[p * DIM + a] + zb[unit_row<DIM>(a)];
            } else {
              double* dst = dcur + p * Q * CP + ch;
#pragma unroll
              for (int s = 0; s < Q; ++s) dst[int64_t(s) * CP] = zb[s];
              cacc[i][hh][0] += zb[0];
            }
          }
        } else {
#pragma unroll
          for (int kq = 0; kq < TL::PS; ++kq) {
            const int64_t b = (tile - nint) * (int64_t(T::TC) * TL::PS) + int64_t(tc) * TL::PS + kq;
            if (b < geo.nb) {
              double hv[QB], zb[QB];
#pragma unroll
              for (int c = 0; c < QB; ++c) hv[c] = hslot(kq * QB + c, ch);
              Jet<DIM, BO ? 1 : 0>::vjp(hv, a1cur[(geo.ni + b) * CP + ch], dh + kq * QB, zb);
              if constexpr (FIRST) {
                cacc[i][hh][DIM] += zb[0];
#pragma unroll
                for (int a = 0; a < DIM; ++a) {
                  double v = zb[0] * x[(geo.ni + b) * DIM + a];
                  if constexpr (BO) v += zb[unit_row<DIM>(a)];
                  cacc[i][hh][a] += v;
                }
              } else {
                double* dst = dcur + (geo.ni * Q + b * QB) * CP + ch;
#pragma unroll
                for (int c = 0; c < QB; ++c) dst[int64_t(c) * CP] = zb[c];
                cacc[i][hh][0] += zb[0];
              }
            }
          }
        }
      }
    }
    __syncthreads();  // H_l tile free: the next tile's rows stream in during its mainloop
    if (has_next) load_h(rn);
  }
  cp_async_wait<0>();
  // fixed-order reduction: the 4 thread columns of a warp, then the warp row groups
#pragma unroll
  for (int i = 0; i < T::MT; ++i)
#pragma unroll
    for (int hh = 0; hh < 2; ++hh)
#pragma unroll
      for (int a = 0; a < NV; ++a) {
        double v = cacc[i][hh][a];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        cacc[i][hh][a] = v;
      }
  __syncthreads();
  double* red = smem;  // [WR][CP][NV]
  if (t == 0) {
#pragma unroll
    for (int i = 0; i < T::MT; ++i)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int ch = wc * T::WCH + 16 * i + 8 * hh + g;
#pragma unroll
        for (int a = 0; a < NV; ++a) red[(wr * CP + ch) * NV + a] = cacc[i][hh][a];
      }
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < CP * NV; idx += T::THREADS) {
    double s = 0.0;
    for (int r = 0; r < T::WR; ++r) s += red[r * CP * NV + idx];
    partial[int64_t(blockIdx.x) * CP * NV + idx] = s;
  }
}

// ----------------------------------------------------------------------------------
// Fused backward of a square 64-wide hidden layer: the dgrad + jet VJP of bwd_layer and
// the weight gradient dW_l = D_{l+1}^T H_l of the same tile.  The tile's seed D_{l+1} and
// its H_l rows arrive by 2-D TMA loads (two 32-column planes each, rows in global order,
// thread column tc owning rows tc*S..tc*S+S-1; rows past a segment zero-filled by the
// tensor map) and W_l stays resident.  Per tile:
//   dgrad over the two seed planes (DMMA, accumulators in registers)
//   wgrad over the tile's rows: seed planes as A, the H_l planes as B
//   -> the seed planes are free: the next tile's seed is requested
//   jet VJP epilogue, reading H_l from shared memory, storing D_l
//   -> the H_l planes are free: the next tile's H_l is requested
// so the next tile's seed arrives during this epilogue and its H_l during the next dgrad.
// dW_l accumulates in registers across the CTA's tiles and is written once per CTA, so
// D_{l+1} and H_l are read from HBM once per layer instead of twice.
constexpr int kFusedWidth = 64;
// 16 warps in 2-D (160-row tiles); 8 warps in 3-D, where 16 would need 320-row tiles
template <int DIM>
struct FusedTile : MmaTile<DIM, kFusedWidth, DIM == 2 ? 16 : 8> {};

// rows per TMA box of a boundary tile: the whole tile when its points fill every slot of a
// thread column (PS * QB == S); otherwise such tiles stream by cp.async (the value is then
// only the box shape of an unused tensor map)
template <int DIM, int BO>
constexpr int fused_boundary_box_rows() {
  using TL = Tiles<DIM, BO, FusedTile<DIM>::TC>;
  return TL::PS * TL::QB == FusedTile<DIM>::S ? FusedTile<DIM>::TR : TL::PS * TL::QB;
}

template <int DIM>
constexpr size_t fused_smem_bytes() {
  using T = FusedTile<DIM>;
  constexpr size_t planes = size_t(kFusedWidth / KC) * size_t(T::TR) * LDC;  // one tensor's tile
  constexpr size_t wres = size_t(kFusedWidth) * (kFusedWidth + 4);           // resident W_l
  constexpr size_t a = sizeof(double) * (2 * planes + wres + 2);              // + 2 mbarriers
  constexpr size_t red = sizeof(double) * (T::WR * kFusedWidth * (DIM + 1) + 8 * (kFusedWidth / 16) * 4 * 32);
  return a > red ? a : red;
}

// MODE kEvalBackward: the evaluation's layer backward (dgrad, wgrad, VJP, bias and
// coordinate partials).  kHookDgradVjp / kHookDgrad: the dense dgrad (+ jet VJP) of the
// reference-ABI hook (flashns_stable_dgrad_vjp on a 64 -> 64 layer: bwd_pingpong in 2-D, bwd_fused in 3-D): no weight gradient and
// no partials; kHookDgrad also skips H and writes dH itself.
enum { kEvalBackward = 0, kHookDgradVjp = 1, kHookDgrad = 2 };
template <int DIM, int BO, bool FIRST, int MODE = kEvalBackward>
__global__ void __launch_bounds__(FusedTile<DIM>::THREADS, 1)
    bwd_fused(const __grid_constant__ CUtensorMap tm_seed_i, const __grid_constant__ CUtensorMap tm_seed_b,
              const __grid_constant__ CUtensorMap tm_h_i, const __grid_constant__ CUtensorMap tm_h_b,
              const double* __restrict__ dnext, const double* __restrict__ hcur, const double* __restrict__ w,
              const double* __restrict__ a1cur, double* __restrict__ dcur,
              const double* __restrict__ x, double* __restrict__ partial, double* __restrict__ wpart, Geometry geo) {
  constexpr int CP = kFusedWidth;
  using T = FusedTile<DIM>;
  using TL = Tiles<DIM, BO, T::TC>;
  constexpr int S = T::S, TR = T::TR, Q = TL::Q, QB = TL::QB, PS = TL::PS, LDW = CP + 4;
  constexpr int NK = CP / KC;  // 32-column planes per tile
  constexpr int MK = KC / 16;  // m16 tiles of output channels per plane
  constexpr int NM = CP / 16;  // m16 tiles of output channels
  constexpr int NV = FIRST ? DIM + 1 : 1;
  constexpr int BB = fused_boundary_box_rows<DIM, BO>();
  constexpr bool SPLIT = BB != TR;  // boundary tiles: one box per thread column
  // wgrad split: warp -> n8 tile (warp % 8) of dW columns and row share (warp / 8)
  constexpr int RS = T::NWARPS / 8, RROWS = TR / RS;
  static_assert(CP / 8 == 8 && T::NWARPS % 8 == 0 && RROWS % 16 == 0, "wgrad warp split");
  static_assert(NK == 2 && KC == 32 && TR <= 256, "TMA boxes: 36 columns, at most 256 rows");
  constexpr bool EVAL = MODE == kEvalBackward, WITH_H = MODE != kHookDgrad;
  static_assert(EVAL || (!FIRST && BO == 0), "the hook modes cover dense (all full-jet) rows");
  static_assert((size_t(TR) * LDC * sizeof(double)) % 128 == 0, "every TMA destination on a 128-byte boundary");
  extern __shared__ __align__(128) double smem[];
  double* sB = smem;                // seed planes [NK][TR][LDC]
  double* sH = sB + NK * TR * LDC;  // H_l planes  [NK][TR][LDC]
  double* sW = sH + NK * TR * LDC;  // W_l         [CP][LDW] (row = output channel)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sW + CP * LDW);  // [0] seed tile, [1] H_l tile
  if (smem_u32(smem) & 127) {  // TMA destinations need 128-byte alignment: refuse, never fault
    if (threadIdx.x == 0) atomicExch(&g_device_fault, 2);
    return;
  }
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int wc = warp % T::WC, wr = warp / T::WC;
  const int64_t nint = TL::interior(geo.ni);
  const int64_t ntiles = nint + TL::boundary(geo.nb);
  double cacc[T::MT][2][NV];
#pragma unroll
  for (int i = 0; i < T::MT; ++i)
#pragma unroll
    for (int hh = 0; hh < 2; ++hh)
#pragma unroll
      for (int a = 0; a < NV; ++a) cacc[i][hh][a] = 0.0;
  const int wn = warp % 8, wrs = warp / 8;
  double wacc[NM][4];  // dW rows 16m+{g,g+8}, columns 8*wn+{2t,2t+1}, rows of share wrs
#pragma unroll
  for (int m = 0; m < NM; ++m)
#pragma unroll
    for (int e = 0; e < 4; ++e) wacc[m][e] = 0.0;

  // One tensor's tile (seed or H_l) into its planes.  All threads call it.  Interior tiles
  // (and boundary tiles whose points fill every slot) are one TMA box per plane, issued by
  // thread 0 on `bar`; the other boundary tiles (points of fewer rows than a thread column
  // has slots) stream by cp.async, one commit group, rows past the segment zero-filled.
  auto tma_tile = [&](int64_t tile) { return !SPLIT || tile < nint; };
  auto load_tile = [&](int64_t tile, double* dst, const CUtensorMap* mi, const CUtensorMap* mb, uint64_t* bar,
                       const double* src) {
    const bool interior = tile < nint;
    if (SPLIT && !interior) {
      const int64_t b0 = (tile - nint) * (int64_t(T::TC) * PS);
      for (int i = tid; i < NK * TR * (KC / 2); i += T::THREADS) {
        const int kc = i / (TR * (KC / 2)), rem = i % (TR * (KC / 2));
        const int r = rem / (KC / 2), q = rem % (KC / 2);
        const int tc = r / S, sl = r % S;
        const int64_t b = b0 + int64_t(tc) * PS + sl / QB;
        const bool ok = sl < PS * QB && b < geo.nb;
        const int64_t gr = ok ? geo.ni * Q + b * QB + sl % QB : 0;
        cp_async16(dst + kc * TR * LDC + r * LDC + 2 * q, src + gr * CP + kc * KC + 2 * q, ok);
      }
      cp_async_commit();
      return;
    }
    if (tid != 0) return;
    fence_proxy_async();  // the planes' last readers finished before the barrier that led here
    if (interior) {
      mbar_arrive_expect_tx(bar, NK * TR * LDC * sizeof(double));
#pragma unroll
      for (int kc = 0; kc < NK; ++kc) tma_load_2d(dst + kc * TR * LDC, mi, kc * KC, int(tile * T::TC * Q), bar);
      return;
    }
    const int64_t b0 = (tile - nint) * (int64_t(T::TC) * PS);  // first boundary point
    mbar_arrive_expect_tx(bar, NK * TR * LDC * sizeof(double));
#pragma unroll
    for (int kc = 0; kc < NK; ++kc) tma_load_2d(dst + kc * TR * LDC, mb, kc * KC, int(b0 * QB), bar);
  };
  // bounded wait for a tile that arrived by TMA (phase bit of its barrier) or cp.async
  auto wait_tile = [&](int64_t tile, uint64_t* bar, unsigned& ph, bool last_group) {
    bool ok = true;
    if (tma_tile(tile)) {
      ok = mbar_wait(bar, ph);
      ph ^= 1u;
    } else if (last_group) {
      cp_async_wait<0>();
    } else {
      cp_async_wait<1>();  // the seed group; the H_l group may still be in flight
    }
    return ok;
  };
  for (int i = tid; i < CP * (CP / 2); i += T::THREADS) {  // W_l, resident
    const int r = i / (CP / 2), p = i % (CP / 2);
    cp_async16(sW + r * LDW + 2 * p, w + int64_t(r) * CP + 2 * p, true);
  }
  cp_async_commit();
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
  }
  cp_async_wait<0>();
  __syncthreads();  // W_l and the barriers visible
  pdl_wait();  // D_{l+1} is the predecessor's output
  pdl_trigger();
  if (int64_t(blockIdx.x) < ntiles) {
    load_tile(blockIdx.x, sB, &tm_seed_i, &tm_seed_b, &bars[0], dnext);
    if (WITH_H) load_tile(blockIdx.x, sH, &tm_h_i, &tm_h_b, &bars[1], hcur);
  }
  unsigned ph_seed = 0, ph_h = 0;
  // B fragments of the dgrad: column g of an n8 tile is slot 2j + (g & 1) of thread
  // column wr*4 + (g >> 1)
  const int brow = (wr * 4 + (g >> 1)) * S + (g & 1);
  // wgrad B fragments: H_l columns 8*wn + g live in plane wn / 4
  const double* hcol = sH + (wn >> 2) * TR * LDC + ((8 * wn) & (KC - 1)) + g;
  for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const bool has_next = tile + gridDim.x < ntiles;
    if (WITH_H && tid == 0) {  // the epilogue reads this tile's a1 rows (a contiguous range): bring them into L2
      int64_t pt0, pts;
      TL::points(geo, nint, tile, pt0, pts);
      prefetch_l2(a1cur + pt0 * CP, uint32_t(pts * CP * sizeof(double)));
    }
    double acc[T::MT][T::NT][4];
#pragma unroll
    for (int i = 0; i < T::MT; ++i)
#pragma unroll
      for (int j = 0; j < T::NT; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.0;
    if (__syncthreads_or(!wait_tile(tile, &bars[0], ph_seed, false))) {  // seed tile landed (bounded wait)
      if (tid == 0) atomicExch(&g_device_fault, 1);
      return;
    }
    // dgrad: dH[ch][rows] += W_l^T[ch][cout plane] D^T[cout plane][rows]
#pragma unroll
    for (int kc = 0; kc < NK; ++kc) {
      const double* cB = sB + kc * TR * LDC + brow * LDC;
      const double* cA = sW + kc * KC * LDW + wc * T::WCH;
#pragma unroll
      for (int kk = 0; kk < KC; kk += 8) {
        double a[T::MT][4];
#pragma unroll
        for (int i = 0; i < T::MT; ++i) {
          a[i][0] = cA[(kk + t) * LDW + 16 * i + g];
          a[i][1] = cA[(kk + t) * LDW + 16 * i + g + 8];
          a[i][2] = cA[(kk + t + 4) * LDW + 16 * i + g];
          a[i][3] = cA[(kk + t + 4) * LDW + 16 * i + g + 8];
        }
#pragma unroll
        for (int j = 0; j < T::NT; ++j) {
          const double b0 = cB[2 * j * LDC + kk + t];
          const double b1 = cB[2 * j * LDC + kk + t + 4];
#pragma unroll
          for (int i = 0; i < T::MT; ++i) mma_m16n8k8(acc[i][j], a[i], b0, b1);
        }
      }
    }
    if (WITH_H && __syncthreads_or(!wait_tile(tile, &bars[1], ph_h, true))) {  // H_l tile landed
      if (tid == 0) atomicExch(&g_device_fault, 1);
      return;
    }
    // wgrad: dW[cout][8*wn..+8] += D^T[cout][rows] H[rows][cin], rows of share wrs
#pragma unroll
    for (int kc = 0; kc < (EVAL ? NK : 0); ++kc) {
      const double* cD = sB + kc * TR * LDC;
#pragma unroll 4
      for (int r = wrs * RROWS; r < (wrs + 1) * RROWS; r += 8) {
        const double b0 = hcol[(r + t) * LDC];
        const double b1 = hcol[(r + t + 4) * LDC];
#pragma unroll
        for (int mm = 0; mm < MK; ++mm) {
          double a[4];
          a[0] = cD[(r + t) * LDC + 16 * mm + g];
          a[1] = cD[(r + t) * LDC + 16 * mm + g + 8];
          a[2] = cD[(r + t + 4) * LDC + 16 * mm + g];
          a[3] = cD[(r + t + 4) * LDC + 16 * mm + g + 8];
          mma_m16n8k8(wacc[kc * MK + mm], a, b0, b1);
        }
      }
    }
    __syncthreads();  // seed planes free
    if (has_next) load_tile(tile + gridDim.x, sB, &tm_seed_i, &tm_seed_b, &bars[0], dnext);
    // epilogue: jet VJP of this tile; H_l from the shared planes (slot s of thread column
    // wr*4+t is row (wr*4+t)*S + s)
    const int tc = wr * 4 + t;
    const double* hrow = sH + (tc * S) * LDC;
    auto hslot = [&](int s, int ch) { return hrow[(ch >> 5) * TR * LDC + s * LDC + (ch & (KC - 1))]; };
    const bool interior = tile < nint;
    if constexpr (!EVAL) {  // the hook: dense rows, dH (+ VJP) straight to the output
      const int64_t p = tile * T::TC + tc;
      if (p < geo.ni) {
#pragma unroll
        for (int i = 0; i < T::MT; ++i)
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int ch = wc * T::WCH + 16 * i + 8 * hh + g;
            double dh[S], zb[Q];
#pragma unroll
            for (int s = 0; s < S; ++s) dh[s] = acc[i][s >> 1][2 * hh + (s & 1)];
            if constexpr (MODE == kHookDgradVjp) {
              double hv[Q];
#pragma unroll
              for (int s = 0; s < Q; ++s) hv[s] = hslot(s, ch);
              Jet<DIM, 3>::vjp(hv, a1cur[p * CP + ch], dh, zb);
            } else {
#pragma unroll
              for (int s = 0; s < Q; ++s) zb[s] = dh[s];
            }
            double* dst = dcur + p * Q * CP + ch;
#pragma unroll
            for (int s = 0; s < Q; ++s) dst[int64_t(s) * CP] = zb[s];
          }
      }
    }
#pragma unroll
    for (int i = 0; i < (EVAL ? T::MT : 0); ++i) {
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int ch = wc * T::WCH + 16 * i + 8 * hh + g;
        double dh[S];
#pragma unroll
        for (int s = 0; s < S; ++s) dh[s] = acc[i][s >> 1][2 * hh + (s & 1)];
        if (interior) {
          const int64_t p = tile * T::TC + tc;
          if (p < geo.ni) {
            double hv[Q], zb[Q];
#pragma unroll
            for (int s = 0; s < Q; ++s) hv[s] = hslot(s, ch);
            Jet<DIM, 3>::vjp(hv, a1cur[p * CP + ch], dh, zb);
            if constexpr (FIRST) {
              cacc[i][hh][DIM] += zb[0];
#pragma unroll
              for (int a = 0; a < DIM; ++a) cacc[i][hh][a] += zb[0] * x[p * DIM + a] + zb[unit_row<DIM>(a)];
            } else {
              double* dst = dcur + p * Q * CP + ch;
#pragma unroll
              for (int s = 0; s < Q; ++s) dst[int64_t(s) * CP] = zb[s];
              cacc[i][hh][0] += zb[0];
            }
          }
        } else {
#pragma unroll
          for (int kq = 0; kq < TL::PS; ++kq) {
            const int64_t b = (tile - nint) * (int64_t(T::TC) * TL::PS) + int64_t(tc) * TL::PS + kq;
            if (b < geo.nb) {
              double hv[QB], zb[QB];
#pragma unroll
              for (int c = 0; c < QB; ++c) hv[c] = hslot(kq * QB + c, ch);
              Jet<DIM, BO ? 1 : 0>::vjp(hv, a1cur[(geo.ni + b) * CP + ch], dh + kq * QB, zb);
              if constexpr (FIRST) {
                cacc[i][hh][DIM] += zb[0];
#pragma unroll
                for (int a = 0; a < DIM; ++a) {
                  double v = zb[0] * x[(geo.ni + b) * DIM + a];
                  if constexpr (BO) v += zb[unit_row<DIM>(a)];
                  cacc[i][hh][a] += v;
                }
              } else {
                double* dst = dcur + (geo.ni * Q + b * QB) * CP + ch;
#pragma unroll
                for (int c = 0; c < QB; ++c) dst[int64_t(c) * CP] = zb[c];
                cacc[i][hh][0] += zb[0];
              }
            }
          }
        }
      }
    }
    __syncthreads();  // H_l planes free
    if (WITH_H && has_next) load_tile(tile + gridDim.x, sH, &tm_h_i, &tm_h_b, &bars[1], hcur);
  }
  if constexpr (!EVAL) {  // the hook writes no partials
    if (tid == 0) {  // every phase completed before the last barrier
      mbar_inval(&bars[0]);
      mbar_inval(&bars[1]);
    }
    return;
  }
  // weight-gradient partial of this CTA: row shares combined in fixed order through smem
  __syncthreads();
  double* wsh = smem + T::WR * CP * NV;  // [8 warps][NM][4][32 lanes]
  if (RS == 2 && wrs == 1) {
#pragma unroll
    for (int m = 0; m < NM; ++m)
#pragma unroll
      for (int e = 0; e < 4; ++e) wsh[((wn * NM + m) * 4 + e) * 32 + lane] = wacc[m][e];
  }
  __syncthreads();
  if (wrs == 0) {
    double* wp = wpart + int64_t(blockIdx.x) * CP * CP;
#pragma unroll
    for (int m = 0; m < NM; ++m) {
      double v[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) v[e] = wacc[m][e] + (RS == 2 ? wsh[((wn * NM + m) * 4 + e) * 32 + lane] : 0.0);
      const int o = 16 * m + g, c = 8 * wn + 2 * t;
      wp[o * CP + c] = v[0];
      wp[o * CP + c + 1] = v[1];
      wp[(o + 8) * CP + c] = v[2];
      wp[(o + 8) * CP + c + 1] = v[3];
    }
  }
  // bias / coordinate partials: fixed-order reduction as in bwd_layer
#pragma unroll
  for (int i = 0; i < T::MT; ++i)
#pragma unroll
    for (int hh = 0; hh < 2; ++hh)
#pragma unroll
      for (int a = 0; a < NV; ++a) {
        double v = cacc[i][hh][a];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        cacc[i][hh][a] = v;
      }
  __syncthreads();
  double* red = smem;  // [WR][CP][NV]
  if (t == 0) {
#pragma unroll
    for (int i = 0; i < T::MT; ++i)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int ch = wc * T::WCH + 16 * i + 8 * hh + g;
#pragma unroll
        for (int a = 0; a < NV; ++a) red[(wr * CP + ch) * NV + a] = cacc[i][hh][a];
      }
  }
  __syncthreads();
  for (int idx = tid; idx < CP * NV; idx += T::THREADS) {
    double s = 0.0;
    for (int r = 0; r < T::WR; ++r) s += red[r * CP * NV + idx];
    partial[int64_t(blockIdx.x) * CP * NV + idx] = s;
  }
  if (tid == 0) {  // every phase completed before the last barrier
    mbar_inval(&bars[0]);
    mbar_inval(&bars[1]);
  }
}

// Two-group ("ping-pong") form of the fused backward for 2-D 64-wide layers.  The CTA's
// 16 warps form two groups of 8; each group works on its own 80-row half tiles with its
// own seed / H_l planes and barriers, and W_l is shared.  Eight warps keep the FP64 tensor
// pipe full, so the groups take turns on it: a group runs its dgrad + wgrad only while it
// holds the turn, and hands the turn over before its jet-VJP epilogue.  The epilogue (and
// the next tile's copies) of one group then overlaps the other group's MMAs instead of
// leaving the pipe idle.  The turn is a pair of named barriers (one per group, all 512
// threads: the waiting group syncs, the other arrives); every group syncs and arrives a
// fixed number of times, so the counts always match (see the end of the kernel).
//
// The CTA's half tiles are blockIdx.x + k * gridDim.x; group 0 takes even k, group 1 odd
// k, so the groups of a CTA differ by at most one half tile.
struct PPTile : MmaTile<2, kFusedWidth, 8> {};
constexpr int kPPGroups = 2;
constexpr int kPPThreads = kPPGroups * PPTile::THREADS;
enum { kPPBarGroup = 1, kPPBarTurn = 3 };  // named barriers: 1 + group (256), 3 + group (512)

template <int BO>
constexpr int pp_boundary_box_rows() {
  using TL = Tiles<2, BO, PPTile::TC>;
  return TL::PS * TL::QB == PPTile::S ? PPTile::TR : TL::PS * TL::QB;
}

// The turn ring of NG groups of 16 / NG warps (the CTA's 512 threads).  Group g holds the
// tensor pipe after group g - 1 (group 0 after group NG - 1, which opens the ring with one
// arrival); turn barrier g counts group g's threads syncing and group g - 1's arriving.
// A CTA's tiles are blockIdx.x + k * gridDim.x; group g takes k = g, g + NG, ..., so the
// groups' counts differ by at most one, and a group whose predecessor arrived once more
// than it synced closes with one more sync.
template <int NG>
struct Ring {
  using T = MmaTile<2, kFusedWidth, 16 / NG>;
  static constexpr int GT = T::THREADS;
  static_assert(NG * GT == kPPThreads && 2 * NG + 1 <= 16, "512 threads; named barriers 1..2NG");
  __device__ static int group_bar(int g) { return 1 + g; }      // the group's own threads
  __device__ static int turn_bar(int g) { return 1 + NG + g; }  // group g syncs, g - 1 arrives
  __device__ static int64_t count(int64_t mine, int g) { return mine > g ? (mine - 1 - g) / NG + 1 : 0; }
  __device__ static void open(int gp) {
    if (gp == NG - 1) named_arrive(turn_bar(0), 2 * GT);
  }
  __device__ static void take(int gp) { named_sync(turn_bar(gp), 2 * GT); }
  __device__ static void pass(int gp) { named_arrive(turn_bar((gp + 1) % NG), 2 * GT); }
  __device__ static void close(int gp, int64_t mine) {
    const int64_t in = gp == 0 ? count(mine, NG - 1) + 1 : count(mine, gp - 1);
    if (in > count(mine, gp)) named_sync(turn_bar(gp), 2 * GT);
  }
};

template <int BO, int NG>
constexpr int ring_boundary_box_rows() {
  using T = typename Ring<NG>::T;
  using TL = Tiles<2, BO, T::TC>;
  return TL::PS * TL::QB == T::S ? T::TR : TL::PS * TL::QB;
}

constexpr size_t pp_smem_bytes() {
  using T = PPTile;
  constexpr size_t planes = size_t(kFusedWidth / KC) * size_t(T::TR) * LDC;  // one tensor's half tile
  constexpr size_t wres = size_t(kFusedWidth) * (kFusedWidth + 4);           // resident W_l
  constexpr size_t a = sizeof(double) * (kPPGroups * 2 * planes + wres + 2 * kPPGroups);  // + mbarriers
  constexpr size_t red = sizeof(double) * (kPPGroups * T::WR * kFusedWidth * 3 + 8 * (kFusedWidth / 16) * 4 * 32);
  return a > red ? a : red;
}

template <int BO, bool FIRST, int MODE = kEvalBackward>
__global__ void __launch_bounds__(kPPThreads, 1)
    bwd_pingpong(const __grid_constant__ CUtensorMap tm_seed_i, const __grid_constant__ CUtensorMap tm_seed_b,
                 const __grid_constant__ CUtensorMap tm_h_i, const __grid_constant__ CUtensorMap tm_h_b,
                 const double* __restrict__ dnext, const double* __restrict__ hcur, const double* __restrict__ w,
                 const double* __restrict__ a1cur, double* __restrict__ dcur, const double* __restrict__ x,
                 double* __restrict__ partial, double* __restrict__ wpart, Geometry geo) {
  constexpr int DIM = 2, CP = kFusedWidth;
  using T = PPTile;
  using TL = Tiles<DIM, BO, T::TC>;
  constexpr int S = T::S, TR = T::TR, Q = TL::Q, QB = TL::QB, PS = TL::PS, LDW = CP + 4;
  constexpr int NK = CP / KC;  // 32-column planes per tile
  constexpr int MK = KC / 16;  // m16 tiles of output channels per plane
  constexpr int NM = CP / 16;  // m16 tiles of output channels
  constexpr int NV = FIRST ? DIM + 1 : 1;
  constexpr int BB = pp_boundary_box_rows<BO>();
  constexpr bool SPLIT = BB != TR;  // boundary tiles whose points leave slots empty: cp.async
  constexpr int GT = T::THREADS;    // threads per group
  constexpr int PLANES = NK * TR * LDC;
  constexpr bool EVAL = MODE == kEvalBackward, WITH_H = MODE != kHookDgrad;
  static_assert(EVAL || (!FIRST && BO == 0), "the hook modes cover dense (all full-jet) rows");
  static_assert(CP / 8 == T::NWARPS && TR % 16 == 0, "wgrad: warp w of a group owns dW columns 8w..8w+7");
  static_assert(NK == 2 && KC == 32 && TR <= 256, "TMA boxes: 36 columns, at most 256 rows");
  static_assert((size_t(TR) * LDC * sizeof(double)) % 128 == 0, "every TMA destination on a 128-byte boundary");
  extern __shared__ __align__(128) double smem[];
  if (smem_u32(smem) & 127) {  // TMA destinations need 128-byte alignment: refuse, never fault
    if (threadIdx.x == 0) atomicExch(&g_device_fault, 2);
    return;
  }
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int gp = warp / T::NWARPS, lw = warp % T::NWARPS, gtid = tid % GT;
  const int wc = lw % T::WC, wr = lw / T::WC;
  double* sB = smem + gp * 2 * PLANES;  // this group's seed planes [NK][TR][LDC]
  double* sH = sB + PLANES;             // this group's H_l planes  [NK][TR][LDC]
  double* sW = smem + kPPGroups * 2 * PLANES;                    // W_l [CP][LDW], shared
  uint64_t* bars = reinterpret_cast<uint64_t*>(sW + CP * LDW);  // [2 group + 0] seed, [2 group + 1] H_l
  uint64_t* bar_seed = bars + 2 * gp;
  uint64_t* bar_h = bars + 2 * gp + 1;
  const int bar_group = kPPBarGroup + gp;
  const int64_t nint = TL::interior(geo.ni);
  const int64_t nht = nint + TL::boundary(geo.nb);
  const int64_t mine = int64_t(blockIdx.x) < nht ? (nht - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int64_t n0 = (mine + 1) / 2, n1 = mine / 2;  // half tiles of group 0 / group 1
  const int64_t nmy = gp == 0 ? n0 : n1;
  auto tile_of = [&](int64_t k) { return int64_t(blockIdx.x) + (2 * k + gp) * int64_t(gridDim.x); };
  double cacc[2][NV];
#pragma unroll
  for (int hh = 0; hh < 2; ++hh)
#pragma unroll
    for (int a = 0; a < NV; ++a) cacc[hh][a] = 0.0;
  double wacc[NM][4];  // dW rows 16m+{g,g+8}, columns 8*lw+{2t,2t+1}, rows of this group
#pragma unroll
  for (int m = 0; m < NM; ++m)
#pragma unroll
    for (int e = 0; e < 4; ++e) wacc[m][e] = 0.0;

  // One tensor's half tile into this group's planes; every thread of the group calls it.
  auto tma_tile = [&](int64_t tile) { return !SPLIT || tile < nint; };
  auto load_tile = [&](int64_t tile, double* dst, const CUtensorMap* mi, const CUtensorMap* mb, uint64_t* bar,
                       const double* src) {
    const bool interior = tile < nint;
    if (SPLIT && !interior) {
      const int64_t b0 = (tile - nint) * (int64_t(T::TC) * PS);
      for (int i = gtid; i < NK * TR * (KC / 2); i += GT) {
        const int kc = i / (TR * (KC / 2)), rem = i % (TR * (KC / 2));
        const int r = rem / (KC / 2), q = rem % (KC / 2);
        const int tc = r / S, sl = r % S;
        const int64_t b = b0 + int64_t(tc) * PS + sl / QB;
        const bool ok = sl < PS * QB && b < geo.nb;
        const int64_t gr = ok ? geo.ni * Q + b * QB + sl % QB : 0;
        cp_async16(dst + kc * TR * LDC + r * LDC + 2 * q, src + gr * CP + kc * KC + 2 * q, ok);
      }
      cp_async_commit();
      return;
    }
    if (gtid != 0) return;
    fence_proxy_async();  // the planes' last readers finished before the barrier that led here
    const int y = interior ? int(tile * T::TC * Q) : int((tile - nint) * (int64_t(T::TC) * PS) * QB);
    mbar_arrive_expect_tx(bar, NK * TR * LDC * sizeof(double));
#pragma unroll
    for (int kc = 0; kc < NK; ++kc) tma_load_2d(dst + kc * TR * LDC, interior ? mi : mb, kc * KC, y, bar);
  };
  // bounded wait for a half tile that arrived by TMA (phase bit of its barrier) or cp.async
  auto wait_tile = [&](int64_t tile, uint64_t* bar, unsigned& ph, bool last_group) {
    bool ok = true;
    if (tma_tile(tile)) {
      ok = mbar_wait(bar, ph);
      ph ^= 1u;
    } else if (last_group) {
      cp_async_wait<0>();
    } else {
      cp_async_wait<1>();  // the seed group; the H_l group may still be in flight
    }
    return ok;
  };
  for (int i = tid; i < CP * (CP / 2); i += kPPThreads) {  // W_l, resident
    const int r = i / (CP / 2), p = i % (CP / 2);
    cp_async16(sW + r * LDW + 2 * p, w + int64_t(r) * CP + 2 * p, true);
  }
  cp_async_commit();
  if (tid == 0)
    for (int b = 0; b < 2 * kPPGroups; ++b) mbar_init(&bars[b], 1);
  cp_async_wait<0>();
  __syncthreads();  // W_l and the barriers visible
  pdl_wait();  // D_{l+1} is the predecessor's output
  pdl_trigger();
  if (nmy > 0) {
    load_tile(tile_of(0), sB, &tm_seed_i, &tm_seed_b, bar_seed, dnext);
    if (WITH_H) load_tile(tile_of(0), sH, &tm_h_i, &tm_h_b, bar_h, hcur);
  }
  unsigned ph_seed = 0, ph_h = 0;
  bool dead = false;  // a bounded wait ran out: skip the work, keep the turn protocol
  // B fragments of the dgrad: column g of an n8 tile is slot 2j + (g & 1) of thread
  // column wr*4 + (g >> 1)
  const int brow = (wr * 4 + (g >> 1)) * S + (g & 1);
  // wgrad B fragments: H_l columns 8*lw + g live in plane lw / 4
  const double* hcol = sH + (lw >> 2) * TR * LDC + ((8 * lw) & (KC - 1)) + g;
  if (gp == 1) named_arrive(kPPBarTurn + 0, kPPThreads);  // group 0 takes the first turn
  for (int64_t k = 0; k < nmy; ++k) {
    const int64_t tile = tile_of(k);
    const bool has_next = k + 1 < nmy;
    if (WITH_H && gtid == 0 && !dead) {  // the epilogue reads this tile's a1 rows (a contiguous range): into L2
      int64_t pt0, pts;
      TL::points(geo, nint, tile, pt0, pts);
      prefetch_l2(a1cur + pt0 * CP, uint32_t(pts * CP * sizeof(double)));
    }
    double acc[T::NT][4];
#pragma unroll
    for (int j = 0; j < T::NT; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[j][e] = 0.0;
    if (!dead) dead = named_sync_or(bar_group, GT, !wait_tile(tile, bar_seed, ph_seed, false));
    named_sync(kPPBarTurn + gp, kPPThreads);  // this group's turn on the tensor pipe
    if (!dead) {
      // dgrad: dH[ch][rows] += W_l^T[ch][cout plane] D^T[cout plane][rows]
#pragma unroll
      for (int kc = 0; kc < NK; ++kc) {
        const double* cB = sB + kc * TR * LDC + brow * LDC;
        const double* cA = sW + kc * KC * LDW + wc * T::WCH;
#pragma unroll
        for (int kk = 0; kk < KC; kk += 8) {
          double a[4];
          a[0] = cA[(kk + t) * LDW + g];
          a[1] = cA[(kk + t) * LDW + g + 8];
          a[2] = cA[(kk + t + 4) * LDW + g];
          a[3] = cA[(kk + t + 4) * LDW + g + 8];
#pragma unroll
          for (int j = 0; j < T::NT; ++j) mma_m16n8k8(acc[j], a, cB[2 * j * LDC + kk + t], cB[2 * j * LDC + kk + t + 4]);
        }
      }
      if (WITH_H) dead = named_sync_or(bar_group, GT, !wait_tile(tile, bar_h, ph_h, true));  // H_l landed
    }
    if (EVAL && !dead) {
      // wgrad: dW[cout][8*lw..+8] += D^T[cout][rows] H[rows][cin] over the half tile's rows
      // (each row step feeds all NM accumulators from one B fragment: NM MMAs in flight)
#pragma unroll 2
      for (int r = 0; r < TR; r += 8) {
        const double b0 = hcol[(r + t) * LDC];
        const double b1 = hcol[(r + t + 4) * LDC];
#pragma unroll
        for (int m = 0; m < NM; ++m) {  // output channels 16m..: plane m / MK
          const double* cD = sB + (m / MK) * TR * LDC + 16 * (m % MK);
          double a[4];
          a[0] = cD[(r + t) * LDC + g];
          a[1] = cD[(r + t) * LDC + g + 8];
          a[2] = cD[(r + t + 4) * LDC + g];
          a[3] = cD[(r + t + 4) * LDC + g + 8];
          mma_m16n8k8(wacc[m], a, b0, b1);
        }
      }
    }
    named_arrive(kPPBarTurn + (1 - gp), kPPThreads);  // the other group's turn
    named_sync(bar_group, GT);                         // this group's seed planes free
    if (has_next && !dead) load_tile(tile_of(k + 1), sB, &tm_seed_i, &tm_seed_b, bar_seed, dnext);
    if (!dead) {
      // epilogue: jet VJP of this half tile; H_l from the shared planes (slot s of thread
      // column wr*4+t is row (wr*4+t)*S + s)
      const int tc = wr * 4 + t;
      if constexpr (!EVAL) {  // the hook: dense rows, dH (+ VJP) straight to the output
        const int64_t p = tile * T::TC + tc;
        if (p < geo.ni) {
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int ch = wc * T::WCH + 8 * hh + g;
            double dh[S], zb[Q];
#pragma unroll
            for (int s = 0; s < S; ++s) dh[s] = acc[s >> 1][2 * hh + (s & 1)];
            if constexpr (MODE == kHookDgradVjp) {
              double hv[Q];
              const double* hrow = sH + (tc * S) * LDC;
#pragma unroll
              for (int s = 0; s < Q; ++s) hv[s] = hrow[(ch >> 5) * TR * LDC + s * LDC + (ch & (KC - 1))];
              Jet<DIM, 3>::vjp(hv, a1cur[p * CP + ch], dh, zb);
            } else {
#pragma unroll
              for (int s = 0; s < Q; ++s) zb[s] = dh[s];
            }
            double* dst = dcur + p * Q * CP + ch;
#pragma unroll
            for (int s = 0; s < Q; ++s) dst[int64_t(s) * CP] = zb[s];
          }
        }
      } else {
      const double* hrow = sH + (tc * S) * LDC;
      auto hslot = [&](int s, int ch) { return hrow[(ch >> 5) * TR * LDC + s * LDC + (ch & (KC - 1))]; };
      const bool interior = tile < nint;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int ch = wc * T::WCH + 8 * hh + g;
        double dh[S];
#pragma unroll
        for (int s = 0; s < S; ++s) dh[s] = acc[s >> 1][2 * hh + (s & 1)];
        if (interior) {
          const int64_t p = tile * T::TC + tc;
          if (p < geo.ni) {
            double hv[Q], zb[Q];
#pragma unroll
            for (int s = 0; s < Q; ++s) hv[s] = hslot(s, ch);
            Jet<DIM, 3>::vjp(hv, a1cur[p * CP + ch], dh, zb);
            if constexpr (FIRST) {
              cacc[hh][DIM] += zb[0];
#pragma unroll
              for (int a = 0; a < DIM; ++a) cacc[hh][a] += zb[0] * x[p * DIM + a] + zb[unit_row<DIM>(a)];
            } else {
              double* dst = dcur + p * Q * CP + ch;
#pragma unroll
              for (int s = 0; s < Q; ++s) dst[int64_t(s) * CP] = zb[s];
              cacc[hh][0] += zb[0];
            }
          }
        } else {
#pragma unroll
          for (int kq = 0; kq < PS; ++kq) {
            const int64_t b = (tile - nint) * (int64_t(T::TC) * PS) + int64_t(tc) * PS + kq;
            if (b < geo.nb) {
              double hv[QB], zb[QB];
#pragma unroll
              for (int c = 0; c < QB; ++c) hv[c] = hslot(kq * QB + c, ch);
              Jet<DIM, BO ? 1 : 0>::vjp(hv, a1cur[(geo.ni + b) * CP + ch], dh + kq * QB, zb);
              if constexpr (FIRST) {
                cacc[hh][DIM] += zb[0];
#pragma unroll
                for (int a = 0; a < DIM; ++a) {
                  double v = zb[0] * x[(geo.ni + b) * DIM + a];
                  if constexpr (BO) v += zb[unit_row<DIM>(a)];
                  cacc[hh][a] += v;
                }
              } else {
                double* dst = dcur + (geo.ni * Q + b * QB) * CP + ch;
#pragma unroll
                for (int c = 0; c < QB; ++c) dst[int64_t(c) * CP] = zb[c];
                cacc[hh][0] += zb[0];
              }
            }
          }
        }
      }
      }  // EVAL epilogue
    }
    named_sync(bar_group, GT);  // this group's H_l planes free
    if (WITH_H && has_next && !dead) load_tile(tile_of(k + 1), sH, &tm_h_i, &tm_h_b, bar_h, hcur);
  }
  // Turn counts.  Barrier "turn 0" gets n0 syncs from group 0 and 1 + n1 arrivals from
  // group 1; "turn 1" gets n1 syncs from group 1 and n0 arrivals from group 0.  With
  // n0 = n1 + 1 turn 0 is balanced and group 1 owes turn 1 one sync; with n0 = n1 group 0
  // owes turn 0 one sync and turn 1 is balanced.
  if (gp == 0 && n0 == n1) named_sync(kPPBarTurn + 0, kPPThreads);
  if (gp == 1 && n0 == n1 + 1) named_sync(kPPBarTurn + 1, kPPThreads);
  // every tile done: the planes become the reduction scratch.  A group whose wait ran out
  // set `dead`; the whole CTA then leaves together with the fault word set.
  if (__syncthreads_or(dead)) {
    if (tid == 0) atomicExch(&g_device_fault, 1);
    return;
  }
  if constexpr (!EVAL) {  // the hook writes no partials
    if (tid == 0)
      for (int b = 0; b < 2 * kPPGroups; ++b) mbar_inval(&bars[b]);
    return;
  }
  // weight-gradient partial of this CTA: the two groups' row shares combined in fixed order
  double* wsh = smem + kPPGroups * T::WR * CP * NV;  // [8 warps][NM][4][32 lanes]
  if (gp == 1) {
#pragma unroll
    for (int m = 0; m < NM; ++m)
#pragma unroll
      for (int e = 0; e < 4; ++e) wsh[((lw * NM + m) * 4 + e) * 32 + lane] = wacc[m][e];
  }
  __syncthreads();
  if (gp == 0) {
    double* wp = wpart + int64_t(blockIdx.x) * CP * CP;
#pragma unroll
    for (int m = 0; m < NM; ++m) {
      double v[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) v[e] = wacc[m][e] + wsh[((lw * NM + m) * 4 + e) * 32 + lane];
      const int o = 16 * m + g, c = 8 * lw + 2 * t;
      wp[o * CP + c] = v[0];
      wp[o * CP + c + 1] = v[1];
      wp[(o + 8) * CP + c] = v[2];
      wp[(o + 8) * CP + c + 1] = v[3];
    }
  }
  // bias / coordinate partials: quad shuffles, then the 4 row groups in fixed order
#pragma unroll
  for (int hh = 0; hh < 2; ++hh)
#pragma unroll
    for (int a = 0; a < NV; ++a) {
      double v = cacc[hh][a];
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      cacc[hh][a] = v;
    }
  double* red = smem;  // [groups * WR][CP][NV]
  const int rg = gp * T::WR + wr;
  if (t == 0) {
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int ch = wc * T::WCH + 8 * hh + g;
#pragma unroll
      for (int a = 0; a < NV; ++a) red[(rg * CP + ch) * NV + a] = cacc[hh][a];
    }
  }
  __syncthreads();
  for (int idx = tid; idx < CP * NV; idx += kPPThreads) {
    double s = 0.0;
    for (int r = 0; r < kPPGroups * T::WR; ++r) s += red[r * CP * NV + idx];
    partial[int64_t(blockIdx.x) * CP * NV + idx] = s;
  }
  if (tid == 0)  // every phase completed before the barriers above
    for (int b = 0; b < 2 * kPPGroups; ++b) mbar_inval(&bars[b]);
}

// Two-group ("ping-pong") form of the 2-D 64 -> 64 forward layer, on the pattern of
// bwd_pingpong: two 8-warp groups share the resident W_l and take turns on the tensor pipe;
// a group's mainloop runs only while it holds the turn, and its jet epilogue (stable tanh,
// stores of H_{l+1} and a1) overlaps the other group's mainloop.  A group's half tile (80
// rows, 8 thread columns) arrives by 2-D TMA boxes in global row order (split boundary
// tiles by cp.async), the permutation folded into the fragment addresses.
// A warp's store box of an interior half tile: H_{l+1} of its 4 points x Q rows and 16
// channels, 128-byte rows in the TMA 128-byte swizzle (16-byte chunk c of row r at chunk
// c ^ (r & 7)), on a 1024-byte boundary.
constexpr int kFppBox = 4 * 10 * 16;
constexpr size_t fpp_smem_bytes() {
  constexpr size_t planes = size_t(kFusedWidth / KC) * size_t(PPTile::TR) * LDC;  // one half tile
  constexpr size_t boxes = size_t(kPPThreads / 32) * kFppBox + 128;              // + 1024-byte alignment slack
  constexpr size_t wres = size_t(kFusedWidth) * (kFusedWidth + 4);
  return sizeof(double) * (kPPGroups * planes + boxes + wres + kPPGroups);  // + one mbarrier per group
}

template <int BO>
__global__ void __launch_bounds__(kPPThreads, 1)
    fwd_pingpong(const __grid_constant__ CUtensorMap tm_in_i, const __grid_constant__ CUtensorMap tm_in_b,
                 const __grid_constant__ CUtensorMap tm_out, const double* __restrict__ hin, const double* __restrict__ w, const double* __restrict__ bias,
                 double* __restrict__ hout, double* __restrict__ a1out, Geometry geo) {
  constexpr int DIM = 2, CP = kFusedWidth;
  using T = PPTile;
  using TL = Tiles<DIM, BO, T::TC>;
  constexpr int S = T::S, TR = T::TR, Q = TL::Q, QB = TL::QB, PS = TL::PS, LDW = CP + 4;
  constexpr int NK = CP / KC;
  constexpr int BB = pp_boundary_box_rows<BO>();
  constexpr bool SPLIT = BB != TR;
  constexpr int GT = T::THREADS;
  constexpr int PLANES = NK * TR * LDC;
  static_assert(NK == 2 && KC == 32 && TR <= 256, "TMA boxes: 36 columns, at most 256 rows");
  static_assert((size_t(TR) * LDC * sizeof(double)) % 128 == 0, "every TMA destination on a 128-byte boundary");
  extern __shared__ __align__(128) double smem[];
  if (smem_u32(smem) & 127) {  // TMA destinations need 128-byte alignment: refuse, never fault
    if (threadIdx.x == 0) atomicExch(&g_device_fault, 2);
    return;
  }
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int gp = warp / T::NWARPS, lw = warp % T::NWARPS, gtid = tid % GT;
  const int wc = lw % T::WC, wr = lw / T::WC;
  double* sB = smem + gp * PLANES;                               // this group's input planes
  // this warp's store box (1024-byte aligned inside the slack), then W_l [CP][LDW]
  double* boxes = smem + kPPGroups * PLANES;
  boxes += ((1024u - (smem_u32(boxes) & 1023u)) & 1023u) / sizeof(double);
  double* box = boxes + warp * kFppBox;
  double* sW = smem + kPPGroups * PLANES + kPPThreads / 32 * kFppBox + 128;  // row = output channel
  uint64_t* bars = reinterpret_cast<uint64_t*>(sW + CP * LDW);  // one per group
  uint64_t* bar_in = bars + gp;
  const int bar_group = kPPBarGroup + gp;
  const int64_t nint = TL::interior(geo.ni);
  const int64_t nht = nint + TL::boundary(geo.nb);
  const int64_t mine = int64_t(blockIdx.x) < nht ? (nht - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int64_t n0 = (mine + 1) / 2, n1 = mine / 2;
  const int64_t nmy = gp == 0 ? n0 : n1;
  auto tile_of = [&](int64_t k) { return int64_t(blockIdx.x) + (2 * k + gp) * int64_t(gridDim.x); };
  auto load_tile = [&](int64_t tile) {
    const bool interior = tile < nint;
    if (SPLIT && !interior) {
      const int64_t b0 = (tile - nint) * (int64_t(T::TC) * PS);
      for (int i = gtid; i < NK * TR * (KC / 2); i += GT) {
        const int kc = i / (TR * (KC / 2)), rem = i % (TR * (KC / 2));
        const int r = rem / (KC / 2), q = rem % (KC / 2);
        const int tc = r / S, sl = r % S;
        const int64_t b = b0 + int64_t(tc) * PS + sl / QB;
        const bool ok = sl < PS * QB && b < geo.nb;
        const int64_t gr = ok ? geo.ni * Q + b * QB + sl % QB : 0;
        cp_async16(sB + kc * TR * LDC + r * LDC + 2 * q, hin + gr * CP + kc * KC + 2 * q, ok);
      }
      cp_async_commit();
      return;
    }
    if (gtid != 0) return;
    fence_proxy_async();  // the planes' last readers finished before the barrier that led here
    const int y = interior ? int(tile * T::TC * Q) : int((tile - nint) * (int64_t(T::TC) * PS) * QB);
    mbar_arrive_expect_tx(bar_in, NK * TR * LDC * sizeof(double));
#pragma unroll
    for (int kc = 0; kc < NK; ++kc) tma_load_2d(sB + kc * TR * LDC, interior ? &tm_in_i : &tm_in_b, kc * KC, y, bar_in);
  };
  unsigned ph = 0;
  auto wait_tile = [&](int64_t tile) {
    if (SPLIT && tile >= nint) {
      cp_async_wait<0>();
      return true;
    }
    const bool ok = mbar_wait(bar_in, ph);
    ph ^= 1u;
    return ok;
  };
  double bias_r[2];  // a thread's channels are fixed for the whole kernel
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) bias_r[hh] = bias[wc * T::WCH + 8 * hh + g];
  for (int i = tid; i < CP * (CP / 2); i += kPPThreads) {  // W_l, resident
    const int r = i / (CP / 2), p = i % (CP / 2);
    cp_async16(sW + r * LDW + 2 * p, w + int64_t(r) * CP + 2 * p, true);
  }
  cp_async_commit();
  if (tid == 0)
    for (int b = 0; b < kPPGroups; ++b) mbar_init(&bars[b], 1);
  cp_async_wait<0>();
  __syncthreads();  // W_l and the barriers visible
  pdl_wait();  // H_l is the predecessor's output
  pdl_trigger();
  if (nmy > 0) load_tile(tile_of(0));
  bool dead = false;
  // B fragments: column g of an n8 tile is slot 2j + (g & 1) of thread column wr*4 + (g >> 1)
  const int brow = (wr * 4 + (g >> 1)) * S + (g & 1);
  if (gp == 1) named_arrive(kPPBarTurn + 0, kPPThreads);  // group 0 takes the first turn
  for (int64_t k = 0; k < nmy; ++k) {
    const int64_t tile = tile_of(k);
    double acc[T::NT][4];
#pragma unroll
    for (int j = 0; j < T::NT; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[j][e] = 0.0;
    if (!dead) dead = named_sync_or(bar_group, GT, !wait_tile(tile));
    named_sync(kPPBarTurn + gp, kPPThreads);  // this group's turn on the tensor pipe
    if (!dead) {
      // Z^T[ch][rows] = W_l[ch][cin] H_l^T[cin][rows]
#pragma unroll
      for (int kc = 0; kc < NK; ++kc) {
        const double* cB = sB + kc * TR * LDC + brow * LDC;
        const double* cA = sW + wc * T::WCH * LDW + kc * KC;
#pragma unroll
        for (int kk = 0; kk < KC; kk += 8) {
          double a[4];
          a[0] = cA[g * LDW + kk + t];
          a[1] = cA[(g + 8) * LDW + kk + t];
          a[2] = cA[g * LDW + kk + t + 4];
          a[3] = cA[(g + 8) * LDW + kk + t + 4];
#pragma unroll
          for (int j = 0; j < T::NT; ++j) mma_m16n8k8(acc[j], a, cB[2 * j * LDC + kk + t], cB[2 * j * LDC + kk + t + 4]);
        }
      }
    }
    named_arrive(kPPBarTurn + (1 - gp), kPPThreads);  // the other group's turn
    named_sync(bar_group, GT);                         // this group's input planes free
    if (k + 1 < nmy && !dead) load_tile(tile_of(k + 1));
    if (!dead) {
      // epilogue: bias on the order-0 coefficient, stable tanh jet, store H_{l+1} and a1.
      // Interior H_{l+1} goes out through this warp's swizzled box as one TMA store (rows of
      // points past the segment lie beyond the tensor map and are not written): bulk stores
      // take far less from the other group's DMMAs than the same bytes as global stores.
      const int tc = wr * 4 + t;
      const bool interior = tile < nint;
      if (interior) {
        if (lane == 0) bulk_wait_read();  // the box's previous store has read it
        __syncwarp();
      }
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int ch = wc * T::WCH + 8 * hh + g;
        double z[S];
#pragma unroll
        for (int s = 0; s < S; ++s) z[s] = acc[s >> 1][2 * hh + (s & 1)];
        if (interior) {
          const int64_t p = tile * T::TC + tc;
          if (p < geo.ni) {
            double hv[Q], a1;
            z[0] += bias_r[hh];
            Jet<DIM, 3>::fwd(z, hv, a1);
#pragma unroll
            for (int s = 0; s < Q; ++s) {
              const int r = t * Q + s, c = 8 * hh + g;  // box row, column
              box[r * 16 + ((((c >> 1) ^ r) & 7) << 1) + (c & 1)] = hv[s];
            }
            a1out[p * CP + ch] = a1;
          }
        } else {
#pragma unroll
          for (int kq = 0; kq < PS; ++kq) {
            const int64_t b = (tile - nint) * (int64_t(T::TC) * PS) + int64_t(tc) * PS + kq;
            if (b < geo.nb) {
              double zz[QB], hv[QB], a1;
#pragma unroll
              for (int c = 0; c < QB; ++c) zz[c] = z[kq * QB + c];
              zz[0] += bias_r[hh];
              Jet<DIM, BO ? 1 : 0>::fwd(zz, hv, a1);
              double* dst = hout + (geo.ni * Q + b * QB) * CP + ch;
#pragma unroll
              for (int c = 0; c < QB; ++c) dst[int64_t(c) * CP] = hv[c];
              a1out[(geo.ni + b) * CP + ch] = a1;
            }
          }
        }
      }
      if (interior) {
        fence_proxy_async();  // this thread's box writes before the TMA engine reads them
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tm_out, wc * T::WCH, int(tile * T::TC * Q + wr * 4 * Q), box);
          bulk_commit();
        }
      }
    }
  }
  if (lane == 0) bulk_wait();  // this warp's stores complete before the kernel ends
  // turn counts balanced as in bwd_pingpong
  if (gp == 0 && n0 == n1) named_sync(kPPBarTurn + 0, kPPThreads);
  if (gp == 1 && n0 == n1 + 1) named_sync(kPPBarTurn + 1, kPPThreads);
  if (__syncthreads_or(dead)) {
    if (tid == 0) atomicExch(&g_device_fault, 1);
    return;
  }
  if (tid == 0)
    for (int b = 0; b < kPPGroups; ++b) mbar_inval(&bars[b]);
}

// ----------------------------------------------------------------------------------
// wgrad: partial[split][o][i] = sum_{rows in split} D[row][o] H[row][i]
template <int BM, int BN>
__global__ void __launch_bounds__(kThreads, 2)
    wgrad_kernel(const double* __restrict__ d, int kout, const double* __restrict__ h, int kin,
                 Geometry geo, int64_t rows_per_split, double* __restrict__ wpart) {
  constexpr int MT = BM / 32, NT = BN / 32, LDA = BM + 4, LDB = BN + 4;
  extern __shared__ __align__(128) double smem[];
  double* sA = smem;                     // [stage][KC rows][BM+4]
  double* sB = sA + kStages * KC * LDA;  // [stage][KC rows][BN+4]
  const int split = blockIdx.x;
  const int nbn = kin / BN;
  const int bm = blockIdx.y / nbn, bn = blockIdx.y % nbn;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int wm = warp & 1, wn = warp >> 1;  // 2 x 4 warps
  const int64_t r0 = int64_t(split) * rows_per_split;
  const int64_t r1 = (r0 + rows_per_split < geo.rows) ? r0 + rows_per_split : geo.rows;
  const int nk = r1 > r0 ? int((r1 - r0 + KC - 1) / KC) : 0;
  pdl_wait();  // D is the predecessor's output
  pdl_trigger();
  auto load = [&](int kc, int stage) {
    double* dA = sA + stage * KC * LDA;
    for (int i = threadIdx.x; i < KC * (BM / 2); i += kThreads) {
      const int r = i / (BM / 2), p = i % (BM / 2);
      const int64_t gr = r0 + int64_t(kc) * KC + r;
      const bool ok = gr < r1;
      cp_async16(dA + r * LDA + 2 * p, d + (ok ? gr : 0) * kout + bm * BM + 2 * p, ok);
    }
    double* dB = sB + stage * KC * LDB;
    for (int i = threadIdx.x; i < KC * (BN / 2); i += kThreads) {
      const int r = i / (BN / 2), p = i % (BN / 2);
      const int64_t gr = r0 + int64_t(kc) * KC + r;
      const bool ok = gr < r1;
      cp_async16(dB + r * LDB + 2 * p, h + (ok ? gr : 0) * kin + bn * BN + 2 * p, ok);
    }
  };
  double acc[MT][NT][4];
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.0;
#pragma unroll
  for (int s = 0; s < kStages - 1; ++s) {
    if (s < nk) load(s, s);
    cp_async_commit();
  }
  for (int kc = 0; kc < nk; ++kc) {
    cp_async_wait<kStages - 2>();
    __syncthreads();
    if (kc + kStages - 1 < nk) load(kc + kStages - 1, (kc + kStages - 1) % kStages);
    cp_async_commit();
    const double* cA = sA + (kc % kStages) * KC * LDA + wm * (16 * MT);
    const double* cB = sB + (kc % kStages) * KC * LDB + wn * (8 * NT);
#pragma unroll
    for (int kk = 0; kk < KC; kk += 8) {
      double a[MT][4];
#pragma unroll
      for (int i = 0; i < MT; ++i) {
        a[i][0] = cA[(kk + t) * LDA + 16 * i + g];
        a[i][1] = cA[(kk + t) * LDA + 16 * i + g + 8];
        a[i][2] = cA[(kk + t + 4) * LDA + 16 * i + g];
        a[i][3] = cA[(kk + t + 4) * LDA + 16 * i + g + 8];
      }
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        const double b0 = cB[(kk + t) * LDB + 8 * j + g];
        const double b1 = cB[(kk + t + 4) * LDB + 8 * j + g];
#pragma unroll
        for (int i = 0; i < MT; ++i) mma_m16n8k8(acc[i][j], a[i], b0, b1);
      }
    }
  }
  cp_async_wait<0>();
  double* out = wpart + int64_t(split) * kout * kin;
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const int o = bm * BM + wm * (16 * MT) + 16 * i + g;
      const int c = bn * BN + wn * (8 * NT) + 8 * j + 2 * t;
      out[int64_t(o) * kin + c] = acc[i][j][0];
      out[int64_t(o) * kin + c + 1] = acc[i][j][1];
      out[int64_t(o + 8) * kin + c] = acc[i][j][2];
      out[int64_t(o + 8) * kin + c + 1] = acc[i][j][3];
    }
}

// ----------------------------------------------------------------------------------
// output layer + residual seed + output-layer gradients + jet VJP into the last hidden layer
template <int HEAD>
struct HeadTraits;
template <>
struct HeadTraits<FLASHNS_B200_HEAD_UVP> { static constexpr int NF = 3; };
template <>
struct HeadTraits<FLASHNS_B200_HEAD_PSI> { static constexpr int NF = 2; };

template <int DIM, int HEAD>
__device__ __forceinline__ double interior_seed(const double* y, double w, double nu, double gamma, double* dy) {
  if constexpr (HEAD == FLASHNS_B200_HEAD_UVP) {
    return seed_uvp_2d(y, w, nu, gamma, dy);
  } else if constexpr (DIM == 2) {
    return seed_psi_2d(y, w, nu, gamma, dy);
  } else {
    return seed_psi_3d(y, w, nu, gamma, dy);
  }
}

constexpr int kHeadRows = 80;

template <int DIM, int CP, int BO, int HEAD, bool FIRST>
__global__ void __launch_bounds__(kThreads)
    head_layer(const double* __restrict__ hL, const double* __restrict__ a1L, const double* __restrict__ wL,
               const double* __restrict__ bL, const double* __restrict__ pde_w, const double* __restrict__ bnd_w,
               const double* __restrict__ target, double nu, double gamma, double bc, double* __restrict__ dL,
               const double* __restrict__ x, double* __restrict__ coord_partial, double* __restrict__ head_partial,
               Geometry geo) {
  constexpr int NF = HeadTraits<HEAD>::NF;
  constexpr int Q = Basis<DIM>::Q, QB = BO ? DIM + 1 : 1;
  constexpr int NFT = (HEAD == FLASHNS_B200_HEAD_PSI && BO) ? 3 : NF;  // boundary target fields
  constexpr int TPI = kHeadRows / Q, TPB = kHeadRows / QB;
  constexpr int LD = CP + 2;
  constexpr int PARTIAL = NF * CP + NF + 1 + CP;  // dW_L | db_L | loss | db_{L-1}
  static_assert(kThreads % CP == 0, "channel ownership must be fixed per thread");
  extern __shared__ __align__(128) double smem[];
  double* sH = smem;                   // [kHeadRows][LD]
  double* sW = sH + kHeadRows * LD;    // [NF][CP]
  double* sY = sW + NF * CP;           // [kHeadRows][NF]
  double* sD = sY + kHeadRows * NF;    // [kHeadRows][NF]
  double* sRed = sD + kHeadRows * NF;  // [kThreads] reduction scratch
  for (int i = threadIdx.x; i < NF * CP; i += kThreads) sW[i] = wL[i];
  pdl_wait();  // H_L is the predecessor's output
  pdl_trigger();

  const int64_t nint = (geo.ni + TPI - 1) / TPI;
  const int64_t ntiles = nint + (geo.nb + TPB - 1) / TPB;
  constexpr int WPT = (NF * CP + kThreads - 1) / kThreads;
  double wacc[WPT];
#pragma unroll
  for (int k = 0; k < WPT; ++k) wacc[k] = 0.0;
  double bacc = 0.0, lacc = 0.0;
  double cacc[DIM + 1];  // FIRST: coordinate contraction; otherwise cacc[0] = bias of layer L-1
#pragma unroll
  for (int a = 0; a <= DIM; ++a) cacc[a] = 0.0;

  for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const bool interior = tile < nint;
    int64_t p0, row0;
    int npts, nrows;
    if (interior) {
      p0 = tile * TPI;
      npts = int((geo.ni - p0) < TPI ? (geo.ni - p0) : TPI);
      row0 = p0 * Q;
      nrows = npts * Q;
    } else {
      p0 = (tile - nint) * TPB;
      npts = int((geo.nb - p0) < TPB ? (geo.nb - p0) : TPB);
      row0 = geo.ni * Q + p0 * QB;
      nrows = npts * QB;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < nrows * (CP / 2); i += kThreads) {
      const int r = i / (CP / 2), p = i % (CP / 2);
      cp_async16(sH + r * LD + 2 * p, hL + (row0 + r) * CP + 2 * p, true);
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    // outputs Y[r][o] = H[r].W[o] (+ bias on order-0 rows)
    for (int i = threadIdx.x; i < nrows * NF; i += kThreads) {
      const int r = i / NF, o = i % NF;
      const double* hr = sH + r * LD;
      const double* wo = sW + o * CP;
      double s0 = 0.0, s1 = 0.0, s2 = 0.0, s3 = 0.0;
#pragma unroll 4
      for (int c = 0; c < CP; c += 4) {
        s0 += hr[c] * wo[c];
        s1 += hr[c + 1] * wo[c + 1];
        s2 += hr[c + 2] * wo[c + 2];
        s3 += hr[c + 3] * wo[c + 3];
      }
      double y = (s0 + s1) + (s2 + s3);
      const bool zero = interior ? (r % Q == 0) : (r % QB == 0);
      if (zero) y += bL[o];
      sY[r * NF + o] = y;
    }
    __syncthreads();
    // residual seeds, one point per thread
    if (interior) {
      if (threadIdx.x < npts) {
        const int pt = threadIdx.x;
        double y[Q * NF], dy[Q * NF];
#pragma unroll
        for (int k = 0; k < Q * NF; ++k) y[k] = sY[pt * Q * NF + k];
        lacc += interior_seed<DIM, HEAD>(y, pde_w[p0 + pt], nu, gamma, dy);
#pragma unroll
        for (int k = 0; k < Q * NF; ++k) sD[pt * Q * NF + k] = dy[k];
      }
    } else {
      for (int pt = threadIdx.x; pt < npts; pt += kThreads) {
        const int64_t b = p0 + pt;
        const double* yr = sY + pt * QB * NF;
        double* dr = sD + pt * QB * NF;
#pragma unroll
        for (int k = 0; k < QB * NF; ++k) dr[k] = 0.0;
        double f[NFT];
        if constexpr (BO == 0) {
#pragma unroll
          for (int o = 0; o < NF; ++o) f[o] = yr[o];
        } else {
          f[0] = yr[unit_row<DIM>(1) * NF + 0];   // u = psi_y
          f[1] = -yr[unit_row<DIM>(0) * NF + 0];  // v = -psi_x
          f[2] = yr[1];                           // p
        }
        double gsd[NFT];
#pragma unroll
        for (int o = 0; o < NFT; ++o) {
          const double err = f[o] - target[b * NFT + o];
          const double wgt = bnd_w[b * NFT + o];
          lacc += bc * wgt * err * err;
          gsd[o] = 2.0 * bc * wgt * err;
        }
        if constexpr (BO == 0) {
#pragma unroll
          for (int o = 0; o < NF; ++o) dr[o] = gsd[o];
        } else {
          dr[unit_row<DIM>(1) * NF + 0] = gsd[0];
          dr[unit_row<DIM>(0) * NF + 0] = -gsd[1];
          dr[1] = gsd[2];
        }
      }
    }
    __syncthreads();
    // output-layer gradients: dW_L[o][c] += sum_r D[r][o] H[r][c]; db_L[o] over order-0 rows
#pragma unroll
    for (int k = 0; k < WPT; ++k) {
      const int idx = threadIdx.x + k * kThreads;
      if (idx < NF * CP) {
        const int o = idx / CP, c = idx % CP;
        double s = 0.0;
        for (int r = 0; r < nrows; ++r) s += sD[r * NF + o] * sH[r * LD + c];
        wacc[k] += s;
      }
    }
    if (threadIdx.x < NF) {
      const int step = interior ? Q : QB;
      for (int r = 0; r < nrows; r += step) bacc += sD[r * NF + threadIdx.x];
    }
    // dgrad through W_L and the jet VJP of the last hidden layer
    if (interior) {
      for (int idx = threadIdx.x; idx < npts * CP; idx += kThreads) {
        const int pt = idx / CP, c = idx % CP;
        double hv[Q], dh[Q], zb[Q];
#pragma unroll
        for (int s = 0; s < Q; ++s) {
          const int r = pt * Q + s;
          double v = 0.0;
#pragma unroll
          for (int o = 0; o < NF; ++o) v += sD[r * NF + o] * sW[o * CP + c];
          dh[s] = v;
          hv[s] = sH[r * LD + c];
        }
        const int64_t p = p0 + pt;
        Jet<DIM, 3>::vjp(hv, a1L[p * CP + c], dh, zb);
        if constexpr (FIRST) {
          cacc[DIM] += zb[0];
#pragma unroll
          for (int a = 0; a < DIM; ++a) cacc[a] += zb[0] * x[p * DIM + a] + zb[unit_row<DIM>(a)];
        } else {
          double* dst = dL + p * Q * CP + c;
#pragma unroll
          for (int s = 0; s < Q; ++s) dst[int64_t(s) * CP] = zb[s];
          cacc[0] += zb[0];
        }
      }
    } else {
      for (int idx = threadIdx.x; idx < npts * CP; idx += kThreads) {
        const int pt = idx / CP, c = idx % CP;
        double hv[QB], dh[QB], zb[QB];
#pragma unroll
        for (int s = 0; s < QB; ++s) {
          const int r = pt * QB + s;
          double v = 0.0;
#pragma unroll
          for (int o = 0; o < NF; ++o) v += sD[r * NF + o] * sW[o * CP + c];
          dh[s] = v;
          hv[s] = sH[r * LD + c];
        }
        const int64_t b = p0 + pt;
        Jet<DIM, BO ? 1 : 0>::vjp(hv, a1L[(geo.ni + b) * CP + c], dh, zb);
        if constexpr (FIRST) {
          cacc[DIM] += zb[0];
#pragma unroll
          for (int a = 0; a < DIM; ++a) {
            double v = zb[0] * x[(geo.ni + b) * DIM + a];
            if constexpr (BO) v += zb[unit_row<DIM>(a)];
            cacc[a] += v;
          }
        } else {
          double* dst = dL + (geo.ni * Q + b * QB) * CP + c;
#pragma unroll
          for (int s = 0; s < QB; ++s) dst[int64_t(s) * CP] = zb[s];
          cacc[0] += zb[0];
        }
      }
    }
  }
  // per-CTA partials, fixed-order reductions
  double* out = head_partial + int64_t(blockIdx.x) * PARTIAL;
#pragma unroll
  for (int k = 0; k < WPT; ++k) {
    const int idx = threadIdx.x + k * kThreads;
    if (idx < NF * CP) out[idx] = wacc[k];
  }
  if (threadIdx.x < NF) out[NF * CP + threadIdx.x] = bacc;
  __syncthreads();
  sRed[threadIdx.x] = lacc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double s = 0.0;
    for (int i = 0; i < kThreads; ++i) s += sRed[i];
    out[NF * CP + NF] = s;
  }
  // threads with the same channel (tid % CP) combine in fixed order
  for (int a = 0; a < (FIRST ? DIM + 1 : 1); ++a) {
    __syncthreads();
    sRed[threadIdx.x] = cacc[a];
    __syncthreads();
    if (threadIdx.x < CP) {
      double s = 0.0;
      for (int r = threadIdx.x; r < kThreads; r += CP) s += sRed[r];
      if constexpr (FIRST) coord_partial[(int64_t(blockIdx.x) * CP + threadIdx.x) * (DIM + 1) + a] = s;
      else out[NF * CP + NF + 1 + threadIdx.x] = s;
    }
  }
}

template <int DIM, int CP, int NF>
constexpr size_t head_smem_bytes() {
  return sizeof(double) * (size_t(kHeadRows) * (CP + 2) + NF * CP + 2 * kHeadRows * NF + kThreads);
}

// ----------------------------------------------------------------------------------
// Last hidden layer fused with the output layer (64-wide layer L-1 -> L, L the last hidden
// layer): the fwd_layer mainloop gives Z_L in registers; the epilogue forms H_L, stages it
// in shared memory (natural row order, over the free activation ring), and runs the head
// on the tile: Y = H_L W^T + b, the residual seeds, the output-layer gradients and the jet
// VJP into layer L.  Only the seed D_L is stored: H_L and a1_L never reach HBM, and the
// separate head launch goes away.  The head epilogue is long and latency-bound, so in 2-D
// two 8-warp CTAs share an SM and one CTA's epilogue runs under the other's MMAs.
template <int DIM>
struct HeadTile : MmaTile<DIM, kFusedWidth, 8> {
  static constexpr int MINB = DIM == 2 ? 2 : 1;  // 80-row tiles in 2-D, 160-row in 3-D
};

template <int DIM, int NF>
constexpr size_t fwd_head_smem_bytes() {
  using T = HeadTile<DIM>;
  constexpr int CP = kFusedWidth;
  constexpr size_t ring = size_t(kStages) * T::TR * LDC;
  constexpr size_t stage = size_t(T::TR) * (CP + 4);  // H_L tile, aliases the ring
  constexpr size_t main = (ring > stage ? ring : stage) + size_t(CP) * (CP + 4) + 2 * size_t(T::TR);
  constexpr size_t head = size_t(NF) * CP + 2 * size_t(T::TR) * NF;
  return sizeof(double) * (main + head);
}

template <int DIM, int BO, int HEAD>
__global__ void __launch_bounds__(HeadTile<DIM>::THREADS, HeadTile<DIM>::MINB)
    fwd_head(const double* __restrict__ hin, const double* __restrict__ w, const double* __restrict__ bias,
             const double* __restrict__ wL, const double* __restrict__ bL, const double* __restrict__ pde_w,
             const double* __restrict__ bnd_w, const double* __restrict__ target, double nu, double gamma, double bc,
             double* __restrict__ dL, double* __restrict__ head_partial, Geometry geo) {
  constexpr int CP = kFusedWidth, KIN = kFusedWidth;
  using T = HeadTile<DIM>;
  using TL = Tiles<DIM, BO, T::TC>;
  constexpr int S = T::S, TR = T::TR, Q = TL::Q, QB = TL::QB, PS = TL::PS;
  constexpr int NF = HeadTraits<HEAD>::NF;
  constexpr int NFT = (HEAD == FLASHNS_B200_HEAD_PSI && BO) ? 3 : NF;  // boundary target fields
  constexpr int LDA = KIN + 4, LDH = CP + 4;  // LDH = 4 mod 16: conflict-free f64 fragments
  constexpr int PARTIAL = NF * CP + NF + 1 + CP;  // dW_L | db_L | loss | db_{L-1}
  constexpr int NK = KIN / KC;
  static_assert(NK == 2 && kStages == 2, "one chunk of lookahead per tile");
  static_assert(T::NWARPS == CP / 8 && NF <= 8, "warp w owns output-gradient columns 8w..8w+7");
  constexpr int RING = (kStages * TR * LDC > TR * LDH) ? kStages * TR * LDC : TR * LDH;
  extern __shared__ __align__(128) double smem[];
  double* sB = smem;         // activation chunks [stage][TR][LDC] during the mainloop
  double* sH = smem;         // H_L tile [TR][CP+4], natural row order, during the epilogue
  double* sA = sB + RING;    // W_{L-1} resident  [CP][KIN+4]
  int64_t* rowmap = reinterpret_cast<int64_t*>(sA + CP * LDA);  // [2][TR]
  double* sW = reinterpret_cast<double*>(rowmap + 2 * TR);      // W_L [NF][CP]
  double* sY = sW + NF * CP;             // Y  [TR][NF]
  double* sD = sY + TR * NF;             // dY [TR][NF]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int wc = warp % T::WC, wr = warp / T::WC;
  const int64_t nint = TL::interior(geo.ni);
  const int64_t ntiles = nint + TL::boundary(geo.nb);
  for (int i = tid; i < NF * CP; i += T::THREADS) sW[i] = wL[i];
  auto fill_rowmap = [&](int64_t tile, int64_t* rm) {
    for (int r = tid; r < TR; r += T::THREADS) {
      int tc, s;
      tile_slot<S>(r, tc, s);
      rm[r] = TL::row(geo, nint, tile, tc, s);
    }
  };
  auto load = [&](int kc, int stage, const int64_t* rm) {
    double* dB = sB + stage * TR * LDC;
    for (int i = tid; i < TR * (KC / 2); i += T::THREADS) {
      const int r = i / (KC / 2), p = i % (KC / 2);
      const int64_t gr = rm[r];
      cp_async16(dB + r * LDC + 2 * p, hin + (gr >= 0 ? gr : 0) * KIN + kc * KC + 2 * p, gr >= 0);
    }
  };
  double bias_r[2];
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) bias_r[hh] = bias[wc * T::WCH + 8 * hh + g];
  for (int i = tid; i < CP * (KIN / 2); i += T::THREADS) {  // W_{L-1}: its own (oldest) group
    const int r = i / (KIN / 2), p = i % (KIN / 2);
    cp_async16(sA + r * LDA + 2 * p, w + int64_t(r) * KIN + 2 * p, true);
  }
  cp_async_commit();
  double wacc[4] = {0.0, 0.0, 0.0, 0.0};  // dW_L[g][8 warp + 2t (+1)] (rows g < NF)
  double bacc = 0.0, lacc = 0.0, cacc[2] = {0.0, 0.0};
  int buf = 0;
  pdl_wait();  // H_{L-1} is the predecessor's output
  pdl_trigger();
  if (int64_t(blockIdx.x) < ntiles) {
    fill_rowmap(blockIdx.x, rowmap);
    __syncthreads();
    load(0, 0, rowmap);
    cp_async_commit();
  }
  for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, buf ^= 1) {
    const int64_t* rm = rowmap + buf * TR;
    int64_t* rn = rowmap + (buf ^ 1) * TR;
    const bool has_next = tile + gridDim.x < ntiles;
    if (has_next) fill_rowmap(tile + gridDim.x, rn);  // published by the barriers below
    double acc[T::NT][4];
#pragma unroll
    for (int j = 0; j < T::NT; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[j][e] = 0.0;
#pragma unroll
    for (int kc = 0; kc < NK; ++kc) {
      cp_async_wait<0>();
      __syncthreads();
      if (kc + 1 < NK) load(kc + 1, (kc + 1) % kStages, rm);
      cp_async_commit();
      const double* cB = sB + (kc % kStages) * TR * LDC + wr * (4 * S) * LDC;
      const double* cA = sA + wc * T::WCH * LDA + kc * KC;
#pragma unroll
      for (int kk = 0; kk < KC; kk += 8) {
        double a[4];
        a[0] = cA[g * LDA + kk + t];
        a[1] = cA[(g + 8) * LDA + kk + t];
        a[2] = cA[g * LDA + kk + t + 4];
        a[3] = cA[(g + 8) * LDA + kk + t + 4];
#pragma unroll
        for (int j = 0; j < T::NT; ++j) {
          const double b0 = cB[(8 * j + g) * LDC + kk + t];
          const double b1 = cB[(8 * j + g) * LDC + kk + t + 4];
          mma_m16n8k8(acc[j], a, b0, b1);
        }
      }
    }
    __syncthreads();  // ring free: it holds the H_L tile until the end of the epilogue
    const int tc = wr * 4 + t;
    const bool interior = tile < nint;
    const int64_t p0 = interior ? tile * T::TC : (tile - nint) * (int64_t(T::TC) * PS);
    const int64_t left = interior ? geo.ni - p0 : geo.nb - p0;
    const int npts = int(left < (interior ? T::TC : T::TC * PS) ? left : (interior ? T::TC : T::TC * PS));
    const int step = interior ? Q : QB;
    const int nrows = npts * step;
    // 1. bias on the order-0 coefficient, stable tanh jet; H_L into the shared tile
    double a1r[2][PS];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int ch = wc * T::WCH + 8 * hh + g;
      double z[S];
#pragma unroll
      for (int s = 0; s < S; ++s) z[s] = acc[s >> 1][2 * hh + (s & 1)];
      if (interior) {
        if (tc < npts) {
          double hv[Q];
          z[0] += bias_r[hh];
          Jet<DIM, 3>::fwd(z, hv, a1r[hh][0]);
#pragma unroll
          for (int s = 0; s < Q; ++s) sH[(tc * Q + s) * LDH + ch] = hv[s];
        } else {  // rows of points past the segment stay finite for the row contractions
#pragma unroll
          for (int s = 0; s < Q; ++s) sH[(tc * Q + s) * LDH + ch] = 0.0;
        }
      } else {
#pragma unroll
        for (int kq = 0; kq < PS; ++kq) {
          const int lp = tc * PS + kq;
          if (lp < npts) {
            double zz[QB], hv[QB];
#pragma unroll
            for (int c = 0; c < QB; ++c) zz[c] = z[kq * QB + c];
            zz[0] += bias_r[hh];
            Jet<DIM, BO ? 1 : 0>::fwd(zz, hv, a1r[hh][kq]);
#pragma unroll
            for (int c = 0; c < QB; ++c) sH[(lp * QB + c) * LDH + ch] = hv[c];
          } else {
#pragma unroll
            for (int c = 0; c < QB; ++c) sH[(lp * QB + c) * LDH + ch] = 0.0;
          }
        }
      }
    }
    __syncthreads();
    // 2. outputs Y^T[o][r] = W_L[o] . H[r] (+ b_L on order-0 rows) as DMMA tiles:
    //    M = outputs (rows >= NF zero), N = tile rows (n8 tile j per warp), K = channels
    const int kend = (nrows + 7) & ~7;
    for (int j = warp; j < kend / 8; j += T::NWARPS) {
      double c[4] = {0.0, 0.0, 0.0, 0.0};
#pragma unroll
      for (int kk = 0; kk < CP; kk += 8) {
        const double a[4] = {g < NF ? sW[g * CP + kk + t] : 0.0, 0.0, g < NF ? sW[g * CP + kk + t + 4] : 0.0, 0.0};
        mma_m16n8k8(c, a, sH[(8 * j + g) * LDH + kk + t], sH[(8 * j + g) * LDH + kk + t + 4]);
      }
      if (g < NF) {
        const int r0 = 8 * j + 2 * t;
        if (r0 < nrows) sY[r0 * NF + g] = c[0] + (r0 % step == 0 ? bL[g] : 0.0);
        if (r0 + 1 < nrows) sY[(r0 + 1) * NF + g] = c[1] + ((r0 + 1) % step == 0 ? bL[g] : 0.0);
      }
    }
    __syncthreads();
    // 3. residual seeds, one point per thread (dY rows up to the next multiple of 8 zeroed)
    for (int i = tid; i < (kend - nrows) * NF; i += T::THREADS) sD[nrows * NF + i] = 0.0;
    if (interior) {
      if (tid < npts) {
        double y[Q * NF], dy[Q * NF];
#pragma unroll
        for (int k = 0; k < Q * NF; ++k) y[k] = sY[tid * Q * NF + k];
        lacc += interior_seed<DIM, HEAD>(y, pde_w[p0 + tid], nu, gamma, dy);
#pragma unroll
        for (int k = 0; k < Q * NF; ++k) sD[tid * Q * NF + k] = dy[k];
      }
    } else {
      for (int pt = tid; pt < npts; pt += T::THREADS) {
        const int64_t b = p0 + pt;
        const double* yr = sY + pt * QB * NF;
        double* dr = sD + pt * QB * NF;
#pragma unroll
        for (int k = 0; k < QB * NF; ++k) dr[k] = 0.0;
        double f[NFT];
        if constexpr (BO == 0) {
#pragma unroll
          for (int o = 0; o < NF; ++o) f[o] = yr[o];
        } else {
          f[0] = yr[unit_row<DIM>(1) * NF + 0];   // u = psi_y
          f[1] = -yr[unit_row<DIM>(0) * NF + 0];  // v = -psi_x
          f[2] = yr[1];                           // p
        }
        double gsd[NFT];
#pragma unroll
        for (int o = 0; o < NFT; ++o) {
          const double err = f[o] - target[b * NFT + o];
          const double wgt = bnd_w[b * NFT + o];
          lacc += bc * wgt * err * err;
          gsd[o] = 2.0 * bc * wgt * err;
        }
        if constexpr (BO == 0) {
#pragma unroll
          for (int o = 0; o < NF; ++o) dr[o] = gsd[o];
        } else {
          dr[unit_row<DIM>(1) * NF + 0] = gsd[0];
          dr[unit_row<DIM>(0) * NF + 0] = -gsd[1];
          dr[1] = gsd[2];
        }
      }
    }
    __syncthreads();
    // 4. output-layer gradients dW_L[o][c] += sum_r dY[r][o] H[r][c] as DMMA tiles (M =
    //    outputs, N = channels 8 warp.., K = tile rows); db_L over order-0 rows
    for (int k0 = 0; k0 < kend; k0 += 8) {
      const double a[4] = {g < NF ? sD[(k0 + t) * NF + g] : 0.0, 0.0, g < NF ? sD[(k0 + t + 4) * NF + g] : 0.0, 0.0};
      mma_m16n8k8(wacc, a, sH[(k0 + t) * LDH + 8 * warp + g], sH[(k0 + t + 4) * LDH + 8 * warp + g]);
    }
    if (tid < NF)
      for (int r = 0; r < nrows; r += step) bacc += sD[r * NF + tid];
    // 5. dgrad through W_L and the jet VJP of layer L on the owned (point, channel) pairs
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int ch = wc * T::WCH + 8 * hh + g;
      if (interior) {
        if (tc < npts) {
          double hv[Q], dh[Q], zb[Q];
#pragma unroll
          for (int s = 0; s < Q; ++s) {
            const int r = tc * Q + s;
            double v = 0.0;
#pragma unroll
            for (int o = 0; o < NF; ++o) v += sD[r * NF + o] * sW[o * CP + ch];
            dh[s] = v;
            hv[s] = sH[r * LDH + ch];
          }
          Jet<DIM, 3>::vjp(hv, a1r[hh][0], dh, zb);
          double* dst = dL + (p0 + tc) * Q * CP + ch;
#pragma unroll
          for (int s = 0; s < Q; ++s) dst[int64_t(s) * CP] = zb[s];
          cacc[hh] += zb[0];
        }
      } else {
#pragma unroll
        for (int kq = 0; kq < PS; ++kq) {
          const int lp = tc * PS + kq;
          if (lp < npts) {
            double hv[QB], dh[QB], zb[QB];
#pragma unroll
            for (int c = 0; c < QB; ++c) {
              const int r = lp * QB + c;
              double v = 0.0;
#pragma unroll
              for (int o = 0; o < NF; ++o) v += sD[r * NF + o] * sW[o * CP + ch];
              dh[c] = v;
              hv[c] = sH[r * LDH + ch];
            }
            Jet<DIM, BO ? 1 : 0>::vjp(hv, a1r[hh][kq], dh, zb);
            double* dst = dL + (geo.ni * Q + (p0 + lp) * QB) * CP + ch;
#pragma unroll
            for (int c = 0; c < QB; ++c) dst[int64_t(c) * CP] = zb[c];
            cacc[hh] += zb[0];
          }
        }
      }
    }
    __syncthreads();  // staging free: the next tile's first chunk
    if (has_next) {
      load(0, 0, rn);
      cp_async_commit();
    }
  }
  cp_async_wait<0>();
  __syncthreads();
  // per-CTA partials, fixed-order reductions
  double* out = head_partial + int64_t(blockIdx.x) * PARTIAL;
  if (tid < NF) out[NF * CP + tid] = bacc;
  double* red = smem;                 // [THREADS] loss partials
  double* cred = smem + T::THREADS;  // [WR][CP] bias partials of layer L-1
  if (g < NF) {
    out[g * CP + 8 * warp + 2 * t] = wacc[0];
    out[g * CP + 8 * warp + 2 * t + 1] = wacc[1];
  }
  red[tid] = lacc;
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    double v = cacc[hh];
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    if (t == 0) cred[wr * CP + wc * T::WCH + 8 * hh + g] = v;
  }
  __syncthreads();
  if (tid == 0) {
    double sum = 0.0;
    for (int i = 0; i < T::THREADS; ++i) sum += red[i];
    out[NF * CP + NF] = sum;
  }
  for (int c = tid; c < CP; c += T::THREADS) {
    double sum = 0.0;
    for (int r = 0; r < T::WR; ++r) sum += cred[r * CP + c];
    out[NF * CP + NF + 1 + c] = sum;
  }
}

// Turn-taking form of fwd_head for 2-D, staged through shared memory: the last hidden
// layer, the output layer, the residual seeds, the output-layer gradients and the VJP into
// layer L, with the CTA's 16 warps in NG groups (Ring<NG>; kHeadGroups = 4 groups of 4
// warps, 40-row tiles) that take turns on the tensor pipe.  Each group has its own input
// planes (TMA, rows in global order), H_L tile, Y and dY; W_{L-1} and W_L are shared.  A
// group's mainloop runs while it holds the turn; its epilogue (jet, output contraction,
// seeds, output gradients, VJP and the stores of D_L) overlaps the other groups' mainloops.  This form serves the
// (u, v, p) head, whose seed reads 25 outputs (one thread per point forms it from the
// staged outputs), and value boundary rows, where a thread column holds ten points; the
// stream-function head with first-order rows runs head_pingpong below.
template <int NF, int NG>
constexpr size_t hpp_staged_group_doubles() {
  using T = typename Ring<NG>::T;
  return size_t(kFusedWidth / KC) * T::TR * LDC + size_t(T::TR) * (kFusedWidth + 4) + 2 * size_t(T::TR) * NF;
}
template <int NF, int NG>
constexpr size_t hpp_staged_smem_bytes() {
  return sizeof(double) * (NG * hpp_staged_group_doubles<NF, NG>() + size_t(kFusedWidth) * (kFusedWidth + 4) +
                           size_t(NF) * kFusedWidth + NG);
}

template <int BO, int HEAD, int NG>
__global__ void __launch_bounds__(kPPThreads, 1)
    head_pingpong_staged(const __grid_constant__ CUtensorMap tm_in_i, const __grid_constant__ CUtensorMap tm_in_b,
                  const double* __restrict__ hin, const double* __restrict__ w, const double* __restrict__ bias,
                  const double* __restrict__ wL, const double* __restrict__ bL, const double* __restrict__ pde_w,
                  const double* __restrict__ bnd_w, const double* __restrict__ target, double nu, double gamma,
                  double bc, double* __restrict__ dL, double* __restrict__ head_partial, Geometry geo) {
  constexpr int DIM = 2, CP = kFusedWidth;
  using R = Ring<NG>;
  using T = typename R::T;
  using TL = Tiles<DIM, BO, T::TC>;
  constexpr int S = T::S, TR = T::TR, Q = TL::Q, QB = TL::QB, PS = TL::PS;
  constexpr int NF = HeadTraits<HEAD>::NF;
  constexpr int NFT = (HEAD == FLASHNS_B200_HEAD_PSI && BO) ? 3 : NF;  // boundary target fields
  constexpr int LDA = CP + 4, LDH = CP + 4;
  constexpr int PARTIAL = NF * CP + NF + 1 + CP;  // dW_L | db_L | loss | db_{L-1}
  constexpr int NK = CP / KC;
  constexpr int BB = ring_boundary_box_rows<BO, NG>();
  constexpr bool SPLIT = BB != TR;
  constexpr int GT = T::THREADS;
  constexpr int PLANES = NK * TR * LDC;
  constexpr int CB = CP / 8 / T::NWARPS;  // output-gradient column blocks of 8 per warp
  static_assert(CB * T::NWARPS * 8 == CP && NF <= 8, "warp w of a group owns output-gradient columns 8 CB w..");
  static_assert(NK == 2 && KC == 32 && TR <= 256, "TMA boxes: 36 columns, at most 256 rows");
  static_assert((hpp_staged_group_doubles<NF, NG>() * sizeof(double)) % 128 == 0, "group buffers on 128-byte boundaries");
  extern __shared__ __align__(128) double smem[];
  if (smem_u32(smem) & 127) {  // TMA destinations need 128-byte alignment: refuse, never fault
    if (threadIdx.x == 0) atomicExch(&g_device_fault, 2);
    return;
  }
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int gp = warp / T::NWARPS, lw = warp % T::NWARPS, gtid = tid % GT;
  const int wc = lw % T::WC, wr = lw / T::WC;
  double* sB = smem + gp * hpp_staged_group_doubles<NF, NG>();  // this group's input planes [NK][TR][LDC]
  double* sH = sB + PLANES;                          // H_L tile [TR][CP+4], rows in tile order
  double* sY = sH + TR * LDH;                        // Y  [TR][NF]
  double* sD = sY + TR * NF;                         // dY [TR][NF]
  double* sA = smem + NG * hpp_staged_group_doubles<NF, NG>();  // W_{L-1} [CP][CP+4], shared
  double* sW = sA + CP * LDA;                                // W_L [NF][CP], shared
  uint64_t* bars = reinterpret_cast<uint64_t*>(sW + NF * CP);
  uint64_t* bar_in = bars + gp;
  const int bar_group = R::group_bar(gp);
  const int64_t nint = TL::interior(geo.ni);
  const int64_t nht = nint + TL::boundary(geo.nb);
  const int64_t mine = int64_t(blockIdx.x) < nht ? (nht - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int64_t nmy = R::count(mine, gp);
  auto tile_of = [&](int64_t k) { return int64_t(blockIdx.x) + (NG * k + gp) * int64_t(gridDim.x); };
  auto load_tile = [&](int64_t tile) {
    const bool interior = tile < nint;
    if (SPLIT && !interior) {
      const int64_t b0 = (tile - nint) * (int64_t(T::TC) * PS);
      for (int i = gtid; i < NK * TR * (KC / 2); i += GT) {
        const int kc = i / (TR * (KC / 2)), rem = i % (TR * (KC / 2));
        const int r = rem / (KC / 2), q = rem % (KC / 2);
        const int tc = r / S, sl = r % S;
        const int64_t b = b0 + int64_t(tc) * PS + sl / QB;
        const bool ok = sl < PS * QB && b < geo.nb;
        const int64_t gr = ok ? geo.ni * Q + b * QB + sl % QB : 0;
        cp_async16(sB + kc * TR * LDC + r * LDC + 2 * q, hin + gr * CP + kc * KC + 2 * q, ok);
      }
      cp_async_commit();
      return;
    }
    if (gtid != 0) return;
    fence_proxy_async();  // the planes' last readers finished before the barrier that led here
    const int y = interior ? int(tile * T::TC * Q) : int((tile - nint) * (int64_t(T::TC) * PS) * QB);
    mbar_arrive_expect_tx(bar_in, NK * TR * LDC * sizeof(double));
#pragma unroll
    for (int kc = 0; kc < NK; ++kc) tma_load_2d(sB + kc * TR * LDC, interior ? &tm_in_i : &tm_in_b, kc * KC, y, bar_in);
  };
  unsigned ph = 0;
  auto wait_tile = [&](int64_t tile) {
    if (SPLIT && tile >= nint) {
      cp_async_wait<0>();
      return true;
    }
    const bool ok = mbar_wait(bar_in, ph);
    ph ^= 1u;
    return ok;
  };
  double bias_r[2];  // a thread's channels are fixed for the whole kernel
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) bias_r[hh] = bias[wc * T::WCH + 8 * hh + g];
  for (int i = tid; i < CP * (CP / 2); i += kPPThreads) {  // W_{L-1}, resident
    const int r = i / (CP / 2), p = i % (CP / 2);
    cp_async16(sA + r * LDA + 2 * p, w + int64_t(r) * CP + 2 * p, true);
  }
  cp_async_commit();
  for (int i = tid; i < NF * CP; i += kPPThreads) sW[i] = wL[i];
  if (tid == 0)
    for (int b = 0; b < NG; ++b) mbar_init(&bars[b], 1);
  cp_async_wait<0>();
  __syncthreads();  // W_{L-1}, W_L and the barriers visible
  pdl_wait();  // H_{L-1} is the predecessor's output
  pdl_trigger();
  if (nmy > 0) load_tile(tile_of(0));
  double wacc[CB][4];  // dW_L[g][8 (CB lw + cb) + 2t (+1)] (rows g < NF)
#pragma unroll
  for (int cb = 0; cb < CB; ++cb) wacc[cb][0] = wacc[cb][1] = wacc[cb][2] = wacc[cb][3] = 0.0;
  double bacc = 0.0, lacc = 0.0, cacc[2] = {0.0, 0.0};
  bool dead = false;
  // B fragments: column g of an n8 tile is slot 2j + (g & 1) of thread column wr*4 + (g >> 1)
  const int brow = (wr * 4 + (g >> 1)) * S + (g & 1);
  R::open(gp);  // group 0 takes the first turn
  for (int64_t k = 0; k < nmy; ++k) {
    const int64_t tile = tile_of(k);
    double acc[T::NT][4];
#pragma unroll
    for (int j = 0; j < T::NT; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[j][e] = 0.0;
    if (!dead) dead = named_sync_or(bar_group, GT, !wait_tile(tile));
    R::take(gp);  // this group's turn on the tensor pipe
    if (!dead) {
      // Z^T[ch][rows] = W_{L-1}[ch][cin] H_{L-1}^T[cin][rows]
#pragma unroll
      for (int kc = 0; kc < NK; ++kc) {
        const double* cB = sB + kc * TR * LDC + brow * LDC;
        const double* cA = sA + wc * T::WCH * LDA + kc * KC;
#pragma unroll
        for (int kk = 0; kk < KC; kk += 8) {
          double a[4];
          a[0] = cA[g * LDA + kk + t];
          a[1] = cA[(g + 8) * LDA + kk + t];
          a[2] = cA[g * LDA + kk + t + 4];
          a[3] = cA[(g + 8) * LDA + kk + t + 4];
#pragma unroll
          for (int j = 0; j < T::NT; ++j) mma_m16n8k8(acc[j], a, cB[2 * j * LDC + kk + t], cB[2 * j * LDC + kk + t + 4]);
        }
      }
    }
    R::pass(gp);                // the next group's turn
    named_sync(bar_group, GT);                         // this group's input planes free
    if (k + 1 < nmy && !dead) load_tile(tile_of(k + 1));
    if (!dead) {
      const int tc = wr * 4 + t;
      const bool interior = tile < nint;
      const int64_t p0 = interior ? tile * T::TC : (tile - nint) * (int64_t(T::TC) * PS);
      const int64_t left = interior ? geo.ni - p0 : geo.nb - p0;
      const int npts = int(left < (interior ? T::TC : T::TC * PS) ? left : (interior ? T::TC : T::TC * PS));
      const int step = interior ? Q : QB;
      const int nrows = npts * step;
      // 1. bias on the order-0 coefficient, stable tanh jet; H_L into the shared tile
      double a1r[2][PS];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int ch = wc * T::WCH + 8 * hh + g;
        double z[S];
#pragma unroll
        for (int s = 0; s < S; ++s) z[s] = acc[s >> 1][2 * hh + (s & 1)];
        if (interior) {
          if (tc < npts) {
            double hv[Q];
            z[0] += bias_r[hh];
            Jet<DIM, 3>::fwd(z, hv, a1r[hh][0]);
#pragma unroll
            for (int s = 0; s < Q; ++s) sH[(tc * Q + s) * LDH + ch] = hv[s];
          } else {  // rows of points past the segment stay finite for the row contractions
#pragma unroll
            for (int s = 0; s < Q; ++s) sH[(tc * Q + s) * LDH + ch] = 0.0;
          }
        } else {
#pragma unroll
          for (int kq = 0; kq < PS; ++kq) {
            const int lp = tc * PS + kq;
            if (lp < npts) {
              double zz[QB], hv[QB];
#pragma unroll
              for (int c = 0; c < QB; ++c) zz[c] = z[kq * QB + c];
              zz[0] += bias_r[hh];
              Jet<DIM, BO ? 1 : 0>::fwd(zz, hv, a1r[hh][kq]);
#pragma unroll
              for (int c = 0; c < QB; ++c) sH[(lp * QB + c) * LDH + ch] = hv[c];
            } else {
#pragma unroll
              for (int c = 0; c < QB; ++c) sH[(lp * QB + c) * LDH + ch] = 0.0;
            }
          }
        }
      }
      named_sync(bar_group, GT);
      // 2. outputs Y^T[o][r] = W_L[o] . H[r] (+ b_L on order-0 rows) as DMMA tiles:
      //    M = outputs (rows >= NF zero), N = tile rows (n8 tile j per warp), K = channels
      const int kend = (nrows + 7) & ~7;
      for (int j = lw; j < kend / 8; j += T::NWARPS) {
        double c[4] = {0.0, 0.0, 0.0, 0.0};
#pragma unroll
        for (int kk = 0; kk < CP; kk += 8) {
          const double a[4] = {g < NF ? sW[g * CP + kk + t] : 0.0, 0.0, g < NF ? sW[g * CP + kk + t + 4] : 0.0, 0.0};
          mma_m16n8k8(c, a, sH[(8 * j + g) * LDH + kk + t], sH[(8 * j + g) * LDH + kk + t + 4]);
        }
        if (g < NF) {
          const int r0 = 8 * j + 2 * t;
          if (r0 < nrows) sY[r0 * NF + g] = c[0] + (r0 % step == 0 ? bL[g] : 0.0);
          if (r0 + 1 < nrows) sY[(r0 + 1) * NF + g] = c[1] + ((r0 + 1) % step == 0 ? bL[g] : 0.0);
        }
      }
      named_sync(bar_group, GT);
      // 3. residual seeds, one point per thread (dY rows up to the next multiple of 8 zeroed)
      for (int i = gtid; i < (kend - nrows) * NF; i += GT) sD[nrows * NF + i] = 0.0;
      if (interior) {
        if (gtid < npts) {
          double y[Q * NF], dy[Q * NF];
#pragma unroll
          for (int k = 0; k < Q * NF; ++k) y[k] = sY[gtid * Q * NF + k];
          lacc += interior_seed<DIM, HEAD>(y, pde_w[p0 + gtid], nu, gamma, dy);
#pragma unroll
          for (int k = 0; k < Q * NF; ++k) sD[gtid * Q * NF + k] = dy[k];
        }
      } else {
        for (int pt = gtid; pt < npts; pt += GT) {
          const int64_t b = p0 + pt;
          const double* yr = sY + pt * QB * NF;
          double* dr = sD + pt * QB * NF;
#pragma unroll
          for (int k = 0; k < QB * NF; ++k) dr[k] = 0.0;
          double f[NFT];
          if constexpr (BO == 0) {
#pragma unroll
            for (int o = 0; o < NF; ++o) f[o] = yr[o];
          } else {
            f[0] = yr[unit_row<DIM>(1) * NF + 0];   // u = psi_y
            f[1] = -yr[unit_row<DIM>(0) * NF + 0];  // v = -psi_x
            f[2] = yr[1];                           // p
          }
          double gsd[NFT];
#pragma unroll
          for (int o = 0; o < NFT; ++o) {
            const double err = f[o] - target[b * NFT + o];
            const double wgt = bnd_w[b * NFT + o];
            lacc += bc * wgt * err * err;
            gsd[o] = 2.0 * bc * wgt * err;
          }
          if constexpr (BO == 0) {
#pragma unroll
            for (int o = 0; o < NF; ++o) dr[o] = gsd[o];
          } else {
            dr[unit_row<DIM>(1) * NF + 0] = gsd[0];
            dr[unit_row<DIM>(0) * NF + 0] = -gsd[1];
            dr[1] = gsd[2];
          }
        }
      }
      named_sync(bar_group, GT);
      // 4. output-layer gradients dW_L[o][c] += sum_r dY[r][o] H[r][c] as DMMA tiles (M =
      //    outputs, N = channels 8 (CB lw + cb).., K = tile rows); db_L over order-0 rows
      for (int k0 = 0; k0 < kend; k0 += 8) {
        const double a[4] = {g < NF ? sD[(k0 + t) * NF + g] : 0.0, 0.0, g < NF ? sD[(k0 + t + 4) * NF + g] : 0.0, 0.0};
#pragma unroll
        for (int cb = 0; cb < CB; ++cb) {
          const int c8 = 8 * (CB * lw + cb) + g;
          mma_m16n8k8(wacc[cb], a, sH[(k0 + t) * LDH + c8], sH[(k0 + t + 4) * LDH + c8]);
        }
      }
      if (gtid < NF)
        for (int r = 0; r < nrows; r += step) bacc += sD[r * NF + gtid];
      // 5. dgrad through W_L and the jet VJP of layer L on the owned (point, channel) pairs
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int ch = wc * T::WCH + 8 * hh + g;
        if (interior) {
          if (tc < npts) {
            double hv[Q], dh[Q], zb[Q];
#pragma unroll
            for (int s = 0; s < Q; ++s) {
              const int r = tc * Q + s;
              double v = 0.0;
#pragma unroll
              for (int o = 0; o < NF; ++o) v += sD[r * NF + o] * sW[o * CP + ch];
              dh[s] = v;
              hv[s] = sH[r * LDH + ch];
            }
            Jet<DIM, 3>::vjp(hv, a1r[hh][0], dh, zb);
            double* dst = dL + (p0 + tc) * Q * CP + ch;
#pragma unroll
            for (int s = 0; s < Q; ++s) dst[int64_t(s) * CP] = zb[s];
            cacc[hh] += zb[0];
          }
        } else {
#pragma unroll
          for (int kq = 0; kq < PS; ++kq) {
            const int lp = tc * PS + kq;
            if (lp < npts) {
              double hv[QB], dh[QB], zb[QB];
#pragma unroll
              for (int c = 0; c < QB; ++c) {
                const int r = lp * QB + c;
                double v = 0.0;
#pragma unroll
                for (int o = 0; o < NF; ++o) v += sD[r * NF + o] * sW[o * CP + ch];
                dh[c] = v;
                hv[c] = sH[r * LDH + ch];
              }
              Jet<DIM, BO ? 1 : 0>::vjp(hv, a1r[hh][kq], dh, zb);
              double* dst = dL + (geo.ni * Q + (p0 + lp) * QB) * CP + ch;
#pragma unroll
              for (int c = 0; c < QB; ++c) dst[int64_t(c) * CP] = zb[c];
              cacc[hh] += zb[0];
            }
          }
        }
      }
    }
  }
  R::close(gp, mine);  // turn counts balanced
  if (__syncthreads_or(dead)) {
    if (tid == 0) atomicExch(&g_device_fault, 1);
    return;
  }
  // per-CTA partials, fixed-order reductions over the groups
  double* out = head_partial + int64_t(blockIdx.x) * PARTIAL;
  double* red = smem;                      // [512] loss partials
  double* cred = red + kPPThreads;         // [groups * WR][CP] bias partials of layer L-1
  double* wsh = cred + NG * T::WR * CP;    // [groups][warps][CB][32 lanes][2] dW_L
  double* bsh = wsh + NG * T::NWARPS * CB * 32 * 2;  // [groups][NF] db_L
#pragma unroll
  for (int cb = 0; cb < CB; ++cb) {
    wsh[(((gp * T::NWARPS + lw) * CB + cb) * 32 + lane) * 2] = wacc[cb][0];
    wsh[(((gp * T::NWARPS + lw) * CB + cb) * 32 + lane) * 2 + 1] = wacc[cb][1];
  }
  if (gtid < NF) bsh[gp * NF + gtid] = bacc;
  red[tid] = lacc;
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    double v = cacc[hh];
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    if (t == 0) cred[(gp * T::WR + wr) * CP + wc * T::WCH + 8 * hh + g] = v;
  }
  __syncthreads();
  if (gp == 0) {
    if (g < NF) {
#pragma unroll
      for (int cb = 0; cb < CB; ++cb) {
        double v0 = 0.0, v1 = 0.0;
        for (int q = 0; q < NG; ++q) {
          v0 += wsh[(((q * T::NWARPS + lw) * CB + cb) * 32 + lane) * 2];
          v1 += wsh[(((q * T::NWARPS + lw) * CB + cb) * 32 + lane) * 2 + 1];
        }
        out[g * CP + 8 * (CB * lw + cb) + 2 * t] = v0;
        out[g * CP + 8 * (CB * lw + cb) + 2 * t + 1] = v1;
      }
    }
    if (gtid < NF) {
      double v = 0.0;
      for (int q = 0; q < NG; ++q) v += bsh[q * NF + gtid];
      out[NF * CP + gtid] = v;
    }
  }
  if (tid == 0) {
    double sum = 0.0;
    for (int i = 0; i < kPPThreads; ++i) sum += red[i];
    out[NF * CP + NF] = sum;
  }
  for (int c = tid; c < CP; c += kPPThreads) {
    double sum = 0.0;
    for (int r = 0; r < NG * T::WR; ++r) sum += cred[r * CP + c];
    out[NF * CP + NF + 1 + c] = sum;
  }
  if (tid == 0)
    for (int b = 0; b < NG; ++b) mbar_inval(&bars[b]);
}

// Turn-taking form of fwd_head for 2-D: the last hidden layer, the output layer, the
// residual seeds, the output-layer gradients and the VJP into layer L, with the CTA's 16
// warps in NG groups (Ring<NG>; kHeadGroups = 4 groups of 4 warps, 40-row tiles) that take
// turns on the tensor pipe.  Each group has its own input planes (TMA, rows in global
// order); W_{L-1} and W_L are shared.  A group's mainloop runs while it holds the turn; its
// epilogue overlaps the other groups' mainloops.  DMMA issue has priority over the
// epilogue's FP64 instructions, so an epilogue advances mostly between other groups'
// turns: with four groups it has three turns to finish in, which outweighs the lower DMMA
// rate of a 4-warp turn (81 % of the 8-warp rate).
//
// The epilogue keeps everything of a tile in registers.  A thread owns one thread
// column (one interior point, or PS boundary points) and two channels, so after the jet it
// holds H_L of its channels at every slot of its points.  The outputs Y = H_L W_L^T + b_L
// are sums over the 64 channels: each thread forms the partial over its two channels for
// the output values the residual seed reads (HeadOutputs), the 8 lanes of a warp that
// share a thread column reduce them with a three-step shuffle butterfly that leaves each
// lane a disjoint eighth (reduce-scatter), and the 4 channel warps of a row group add
// their eighths through shared memory in fixed order, after one 128-thread barrier.
// Every thread of a point then has its outputs, forms the seed itself (the seed formulas
// are a few dozen flops), accumulates dW_L = dY^T H_L for its channels, contracts
// dH_L = dY W_L and runs the jet VJP.  Per tile that is one row-group barrier and
// about 70 FP64 operations per thread beyond the jet and its VJP, instead of staging
// H_L, Y and dY in shared memory around output-layer MMAs of which 14 of 16 rows are zero.
//
// Output values the stream-function seed reads (and seeds), as flat indices s * NF + f
// (slot s of a point, output f).  Interior points: the inputs of the generated seed formulas
// (seed_psi_2d in residual_generated.cuh; tests/test_codegen.py checks the list against
// that file).  Boundary points (first-order rows): (psi_y, psi_x, p) of each of a thread
// column's PS points, the slots of u = psi_y, v = -psi_x and p.
struct HeadOutputs {
  static constexpr int NF = 2, Q = Basis<2>::Q, QB = 3, PS = Q / QB;
  static constexpr int NI = 11, NB = 3 * PS;
  static constexpr int LDP = 16 + 1;  // both lists padded to 8 lanes x 2; odd: conflict-free reads
  __host__ __device__ static constexpr int interior(int k) {
    constexpr int v[NI] = {2, 3, 4, 5, 6, 8, 10, 12, 14, 16, 18};
    return v[k];
  }
  __host__ __device__ static constexpr int boundary(int k) {
    const int kq = k / 3, j = k % 3;  // j: psi_y, psi_x, p of point kq
    return j == 0 ? (kq * QB + unit_row<2>(1)) * NF : j == 1 ? (kq * QB + unit_row<2>(0)) * NF : kq * QB * NF + 1;
  }
};

constexpr int kHeadGroups = 4;  // groups of the register head's turn ring

template <int NG>
constexpr size_t hpp_smem_bytes() {
  using HO = HeadOutputs;
  using T = typename Ring<NG>::T;
  constexpr size_t planes = size_t(kFusedWidth / KC) * T::TR * LDC;  // one group's input tile
  constexpr size_t parts = size_t(NG) * T::WR * 4 * T::WC * HO::LDP;
  constexpr size_t lead = size_t(NG) * T::WR * 4 * (HO::NF + 1);
  return sizeof(double) * (NG * planes + size_t(kFusedWidth) * (kFusedWidth + 4) +
                           size_t(HO::NF) * (kFusedWidth + 1) + parts + lead + NG);
}

template <int NG>
__global__ void __launch_bounds__(kPPThreads, 1)
    head_pingpong(const __grid_constant__ CUtensorMap tm_in_i, const __grid_constant__ CUtensorMap tm_in_b,
                  const double* __restrict__ hin, const double* __restrict__ w, const double* __restrict__ bias,
                  const double* __restrict__ wL, const double* __restrict__ bL, const double* __restrict__ pde_w,
                  const double* __restrict__ bnd_w, const double* __restrict__ target, double nu, double gamma,
                  double bc, double* __restrict__ dL, double* __restrict__ head_partial, Geometry geo) {
  constexpr int DIM = 2, CP = kFusedWidth;
  using R = Ring<NG>;
  using T = typename R::T;
  constexpr int BO = 1, HEAD = FLASHNS_B200_HEAD_PSI;
  using TL = Tiles<DIM, BO, T::TC>;
  using HO = HeadOutputs;
  constexpr int S = T::S, TR = T::TR, Q = TL::Q, QB = TL::QB, PS = TL::PS;
  constexpr int NF = HO::NF;
  constexpr int NFT = (HEAD == FLASHNS_B200_HEAD_PSI && BO) ? 3 : NF;  // boundary target fields
  constexpr int LDA = CP + 4, LDP = HO::LDP;
  constexpr int PARTIAL = NF * CP + NF + 1 + CP;  // dW_L | db_L | loss | db_{L-1}
  constexpr int NK = CP / KC;
  constexpr int BB = ring_boundary_box_rows<BO, NG>();
  constexpr bool SPLIT = BB != TR;
  constexpr int GT = T::THREADS;
  constexpr int PLANES = NK * TR * LDC;
  static_assert(T::WC == 4 && T::TC == 4 * T::WR, "4 channel warps x row groups of 4 thread columns");
  static_assert(NK == 2 && KC == 32 && TR <= 256, "TMA boxes: 36 columns, at most 256 rows");
  static_assert((size_t(PLANES) * sizeof(double)) % 128 == 0, "group planes on 128-byte boundaries");
  static_assert(PS * QB <= S && HO::NI <= Q * NF, "slots of a thread column");
  extern __shared__ __align__(128) double smem[];
  if (smem_u32(smem) & 127) {  // TMA destinations need 128-byte alignment: refuse, never fault
    if (threadIdx.x == 0) atomicExch(&g_device_fault, 2);
    return;
  }
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int gp = warp / T::NWARPS, lw = warp % T::NWARPS, gtid = tid % GT;
  const int wc = lw % T::WC, wr = lw / T::WC;
  double* sB = smem + gp * PLANES;            // this group's input planes [NK][TR][LDC]
  double* sA = smem + NG * PLANES;            // W_{L-1} [CP][CP+4], shared
  double* sW = sA + CP * LDA;                 // W_L [NF][CP], then b_L [NF]
  double* sP = sW + NF * CP + NF;             // output partials [group][row group][thread column][wc][LDP]
  double* sL = sP + NG * T::WR * 4 * T::WC * LDP;  // per lead thread: loss, db_L [NF]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sL + NG * T::WR * 4 * (NF + 1));
  uint64_t* bar_in = bars + gp;
  const int bar_group = R::group_bar(gp);
  // the 4 channel warps of a row group: the group itself, or barriers 2NG + 1 + ...
  const int bar_rows = T::WR == 1 ? bar_group : 2 * NG + 1 + gp * T::WR + wr;
  double* part = sP + ((gp * T::WR + wr) * 4 + t) * T::WC * LDP;  // this thread column's partials
  const int64_t nint = TL::interior(geo.ni);
  const int64_t nht = nint + TL::boundary(geo.nb);
  const int64_t mine = int64_t(blockIdx.x) < nht ? (nht - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int64_t nmy = R::count(mine, gp);
  auto tile_of = [&](int64_t k) { return int64_t(blockIdx.x) + (NG * k + gp) * int64_t(gridDim.x); };
  auto load_tile = [&](int64_t tile) {
    const bool interior = tile < nint;
    if (SPLIT && !interior) {
      const int64_t b0 = (tile - nint) * (int64_t(T::TC) * PS);
      for (int i = gtid; i < NK * TR * (KC / 2); i += GT) {
        const int kc = i / (TR * (KC / 2)), rem = i % (TR * (KC / 2));
        const int r = rem / (KC / 2), q = rem % (KC / 2);
        const int tc = r / S, sl = r % S;
        const int64_t b = b0 + int64_t(tc) * PS + sl / QB;
        const bool ok = sl < PS * QB && b < geo.nb;
        const int64_t gr = ok ? geo.ni * Q + b * QB + sl % QB : 0;
        cp_async16(sB + kc * TR * LDC + r * LDC + 2 * q, hin + gr * CP + kc * KC + 2 * q, ok);
      }
      cp_async_commit();
      return;
    }
    if (gtid != 0) return;
    fence_proxy_async();  // the planes' last readers finished before the barrier that led here
    const int y = interior ? int(tile * T::TC * Q) : int((tile - nint) * (int64_t(T::TC) * PS) * QB);
    mbar_arrive_expect_tx(bar_in, NK * TR * LDC * sizeof(double));
#pragma unroll
    for (int kc = 0; kc < NK; ++kc) tma_load_2d(sB + kc * TR * LDC, interior ? &tm_in_i : &tm_in_b, kc * KC, y, bar_in);
  };
  unsigned ph = 0;
  auto wait_tile = [&](int64_t tile) {
    if (SPLIT && tile >= nint) {
      cp_async_wait<0>();
      return true;
    }
    const bool ok = mbar_wait(bar_in, ph);
    ph ^= 1u;
    return ok;
  };
  // a thread's channels are fixed for the whole kernel: their W_L columns
  double wl[NF][2];
#pragma unroll
  for (int hh = 0; hh < 2; ++hh)
#pragma unroll
    for (int o = 0; o < NF; ++o) wl[o][hh] = wL[o * CP + wc * T::WCH + 8 * hh + g];
  for (int i = tid; i < CP * (CP / 2); i += kPPThreads) {  // W_{L-1}, resident
    const int r = i / (CP / 2), p = i % (CP / 2);
    cp_async16(sA + r * LDA + 2 * p, w + int64_t(r) * CP + 2 * p, true);
  }
  cp_async_commit();
  for (int i = tid; i < NF * CP; i += kPPThreads) sW[i] = wL[i];
  if (tid < NF) sW[NF * CP + tid] = bL[tid];
  if (tid < NG * T::WR * 4 * (NF + 1)) sL[tid] = 0.0;
  if (tid == 0)
    for (int b = 0; b < NG; ++b) mbar_init(&bars[b], 1);
  cp_async_wait<0>();
  __syncthreads();  // W_{L-1}, W_L, b_L, the loss slots and the barriers visible
  pdl_wait();  // H_{L-1} is the predecessor's output
  pdl_trigger();
  if (nmy > 0) load_tile(tile_of(0));
  double wacc[NF][2], cacc[2] = {0.0, 0.0};
#pragma unroll
  for (int o = 0; o < NF; ++o) wacc[o][0] = wacc[o][1] = 0.0;
  // the one thread of a thread column that books its points' loss and db_L, in its own
  // shared-memory slot (no other thread touches it until the end of the kernel)
  const bool lead = wc == 0 && g == 0;
  double* lslot = sL + ((gp * T::WR + wr) * 4 + t) * (NF + 1);
  bool dead = false;
  // B fragments: column g of an n8 tile is slot 2j + (g & 1) of thread column wr*4 + (g >> 1)
  const int brow = (wr * 4 + (g >> 1)) * S + (g & 1);
  R::open(gp);  // group 0 takes the first turn
  for (int64_t k = 0; k < nmy; ++k) {
    const int64_t tile = tile_of(k);
    double acc[T::NT][4];
#pragma unroll
    for (int j = 0; j < T::NT; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[j][e] = 0.0;
    if (!dead) dead = named_sync_or(bar_group, GT, !wait_tile(tile));
    R::take(gp);  // this group's turn on the tensor pipe
    if (!dead) {
      // Z^T[ch][rows] = W_{L-1}[ch][cin] H_{L-1}^T[cin][rows]
#pragma unroll
      for (int kc = 0; kc < NK; ++kc) {
        const double* cB = sB + kc * TR * LDC + brow * LDC;
        const double* cA = sA + wc * T::WCH * LDA + kc * KC;
#pragma unroll
        for (int kk = 0; kk < KC; kk += 8) {
          double a[4];
          a[0] = cA[g * LDA + kk + t];
          a[1] = cA[(g + 8) * LDA + kk + t];
          a[2] = cA[g * LDA + kk + t + 4];
          a[3] = cA[(g + 8) * LDA + kk + t + 4];
#pragma unroll
          for (int j = 0; j < T::NT; ++j) mma_m16n8k8(acc[j], a, cB[2 * j * LDC + kk + t], cB[2 * j * LDC + kk + t + 4]);
        }
      }
    }
    R::pass(gp);                // the next group's turn
    named_sync(bar_group, GT);                         // this group's input planes free
    if (k + 1 < nmy && !dead) load_tile(tile_of(k + 1));
    if (dead) continue;
    const int tc = wr * 4 + t;
    const bool interior = tile < nint;
    const int64_t p0 = interior ? tile * T::TC : (tile - nint) * (int64_t(T::TC) * PS);
    const int64_t left = interior ? geo.ni - p0 : geo.nb - p0;
    const int cap = interior ? T::TC : T::TC * PS;
    const int npts = int(left < cap ? left : cap);
    // 1. bias on the order-0 coefficient and the stable tanh jet: H_L of this thread's two
    //    channels at every slot of its points, in registers (zero at slots without a point)
    double hv[2][S], a1r[2][PS];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      double z[S];
#pragma unroll
      for (int s = 0; s < S; ++s) {
        z[s] = acc[s >> 1][2 * hh + (s & 1)];
        hv[hh][s] = 0.0;
      }
#pragma unroll
      for (int kq = 0; kq < PS; ++kq) a1r[hh][kq] = 0.0;
      if (interior) {
        if (tc < npts) {
          z[0] += bias[wc * T::WCH + 8 * hh + g];
          Jet<DIM, 3>::fwd(z, hv[hh], a1r[hh][0]);
        }
      } else {
#pragma unroll
        for (int kq = 0; kq < PS; ++kq) {
          if (tc * PS + kq < npts) {
            double zz[QB];
#pragma unroll
            for (int c = 0; c < QB; ++c) zz[c] = z[kq * QB + c];
            zz[0] += bias[wc * T::WCH + 8 * hh + g];
            Jet<DIM, 1>::fwd(zz, hv[hh] + kq * QB, a1r[hh][kq]);
          }
        }
      }
    }
    // 2-4. outputs, seeds, output-layer gradients, dgrad through W_L, VJP: per tile kind
    auto finish = [&](auto kind) {
      constexpr bool INTERIOR = decltype(kind)::value;
      constexpr int NY = INTERIOR ? HO::NI : HO::NB;
      constexpr int NYP = (NY + 7) / 8 * 8, H1 = NYP / 2, H2 = NYP / 4, H3 = NYP / 8;
      constexpr int STEP = INTERIOR ? Q : QB;  // rows per point: b_L on every STEP-th slot
      auto index = [](int k) { return INTERIOR ? HO::interior(k) : HO::boundary(k); };
      // this thread's two channels' share of output value k (zero past NY)
      auto share = [&](int k) {
        if (k >= NY) return 0.0;
        const int s = index(k) / NF, o = index(k) % NF;
        return hv[0][s] * wl[o][0] + hv[1][s] * wl[o][1];
      };
      // reduce-scatter over the 8 lanes of this thread column (g = lane >> 2): after the
      // steps over lane bits 4, 3, 2 lane g holds the sums of values [g*H3, g*H3 + H3)
      double v1[H1], v2[H2], v3[H3];
      const bool u4 = lane & 16, u3 = lane & 8, u2 = lane & 4;
#pragma unroll
      for (int i = 0; i < H1; ++i) {
        const double lo = share(i), hi = share(H1 + i);
        const double keep = u4 ? hi : lo, send = u4 ? lo : hi;
        v1[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
      }
#pragma unroll
      for (int i = 0; i < H2; ++i) {
        const double keep = u3 ? v1[H2 + i] : v1[i], send = u3 ? v1[i] : v1[H2 + i];
        v2[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
      }
#pragma unroll
      for (int i = 0; i < H3; ++i) {
        const double keep = u2 ? v2[H3 + i] : v2[i], send = u2 ? v2[i] : v2[H3 + i];
        v3[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
      }
#pragma unroll
      for (int i = 0; i < H3; ++i) part[wc * LDP + g * H3 + i] = v3[i];
      named_sync(bar_rows, 4 * 32);  // the 4 channel warps of this row group
      double y[NY];
#pragma unroll
      for (int k = 0; k < NY; ++k) {
        y[k] = ((part[k] + part[LDP + k]) + part[2 * LDP + k]) + part[3 * LDP + k];
        if ((index(k) / NF) % STEP == 0) y[k] += sW[NF * CP + index(k) % NF];
      }
      // residual seeds of this thread column's points (every thread of the column forms them)
      double dy[NY];
      if constexpr (INTERIOR) {
        double yv[Q * NF], dyv[Q * NF];
#pragma unroll
        for (int i = 0; i < Q * NF; ++i) yv[i] = 0.0;
#pragma unroll
        for (int kk = 0; kk < NY; ++kk) yv[index(kk)] = y[kk];
        const bool valid = tc < npts;
        const double l = interior_seed<DIM, HEAD>(yv, valid ? pde_w[p0 + tc] : 0.0, nu, gamma, dyv);
        if (valid && lead) lslot[0] += l;
#pragma unroll
        for (int kk = 0; kk < NY; ++kk) dy[kk] = valid ? dyv[index(kk)] : 0.0;
      } else {
        constexpr int PER = NY / PS;  // output values per boundary point
#pragma unroll
        for (int kq = 0; kq < PS; ++kq) {
          const int64_t b = p0 + tc * PS + kq;
          const bool valid = tc * PS + kq < npts;
          double f[NFT];
          f[0] = y[kq * PER + 0];   // u = psi_y
          f[1] = -y[kq * PER + 1];  // v = -psi_x
          f[2] = y[kq * PER + 2];   // p
          double gsd[NFT];
#pragma unroll
          for (int o = 0; o < NFT; ++o) {
            const double err = valid ? f[o] - target[b * NFT + o] : 0.0;
            const double wgt = valid ? bnd_w[b * NFT + o] : 0.0;
            if (valid && lead) lslot[0] += bc * wgt * err * err;
            gsd[o] = 2.0 * bc * wgt * err;
          }
          dy[kq * PER + 0] = gsd[0];
          dy[kq * PER + 1] = -gsd[1];
          dy[kq * PER + 2] = gsd[2];
        }
      }
      // output-layer gradients: dW_L[o][ch] += dY[s][o] H_L[s][ch] over this column's
      // slots; db_L[o] over its points' order-0 rows (once per column)
#pragma unroll
      for (int kk = 0; kk < NY; ++kk) {
        const int s = index(kk) / NF, o = index(kk) % NF;
        wacc[o][0] += dy[kk] * hv[0][s];
        wacc[o][1] += dy[kk] * hv[1][s];
        if (s % STEP == 0 && lead) lslot[1 + o] += dy[kk];
      }
      // dgrad through W_L and the jet VJP of layer L on the owned (point, channel) pairs
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int ch = wc * T::WCH + 8 * hh + g;
        double dh[S];
#pragma unroll
        for (int s = 0; s < S; ++s) dh[s] = 0.0;
#pragma unroll
        for (int kk = 0; kk < NY; ++kk) dh[index(kk) / NF] += dy[kk] * wl[index(kk) % NF][hh];
        if constexpr (INTERIOR) {
          if (tc < npts) {
            double zb[Q];
            Jet<DIM, 3>::vjp(hv[hh], a1r[hh][0], dh, zb);
            double* dst = dL + (p0 + tc) * Q * CP + ch;
#pragma unroll
            for (int s = 0; s < Q; ++s) dst[int64_t(s) * CP] = zb[s];
            cacc[hh] += zb[0];
          }
        } else {
#pragma unroll
          for (int kq = 0; kq < PS; ++kq) {
            const int lp = tc * PS + kq;
            if (lp < npts) {
              double zb[QB];
              Jet<DIM, 1>::vjp(hv[hh] + kq * QB, a1r[hh][kq], dh + kq * QB, zb);
              double* dst = dL + (geo.ni * Q + (p0 + lp) * QB) * CP + ch;
#pragma unroll
              for (int c = 0; c < QB; ++c) dst[int64_t(c) * CP] = zb[c];
              cacc[hh] += zb[0];
            }
          }
        }
      }
    };
    if (interior) finish(std::true_type{});
    else finish(std::false_type{});
  }
  R::close(gp, mine);  // turn counts balanced
  if (__syncthreads_or(dead)) {
    if (tid == 0) atomicExch(&g_device_fault, 1);
    return;
  }
  // per-CTA partials, fixed-order reductions: the 4 thread columns of a warp by shuffles,
  // then the row groups of all groups in order
  constexpr int RG = NG * T::WR;
  double* out = head_partial + int64_t(blockIdx.x) * PARTIAL;
  double* cred = smem;                  // [RG][CP] bias partials of layer L-1
  double* wred = cred + RG * CP;        // [RG][NF][CP] dW_L
  const int rg = gp * T::WR + wr;
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int ch = wc * T::WCH + 8 * hh + g;
    double v = cacc[hh];
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    if (t == 0) cred[rg * CP + ch] = v;
#pragma unroll
    for (int o = 0; o < NF; ++o) {
      double u = wacc[o][hh];
      u += __shfl_xor_sync(0xffffffffu, u, 1);
      u += __shfl_xor_sync(0xffffffffu, u, 2);
      if (t == 0) wred[(rg * NF + o) * CP + ch] = u;
    }
  }
  __syncthreads();
  for (int idx = tid; idx < NF * CP; idx += kPPThreads) {  // dW_L[o][c] at o * CP + c
    double sum = 0.0;
    for (int r = 0; r < RG; ++r) sum += wred[r * NF * CP + idx];
    out[idx] = sum;
  }
  if (tid < NF + 1) {  // db_L (tid < NF), then the loss; the lead slots in fixed order
    const int f = tid < NF ? 1 + tid : 0;
    double sum = 0.0;
    for (int i = 0; i < RG * 4; ++i) sum += sL[i * (NF + 1) + f];
    out[NF * CP + tid] = sum;
  }
  for (int c = tid; c < CP; c += kPPThreads) {
    double sum = 0.0;
    for (int r = 0; r < RG; ++r) sum += cred[r * CP + c];
    out[NF * CP + NF + 1 + c] = sum;
  }
  if (tid == 0)
    for (int b = 0; b < NG; ++b) mbar_inval(&bars[b]);
}


// ----------------------------------------------------------------------------------
// first layer: coordinates -> affine jet -> stable tanh jet
template <int DIM, int BO>
__global__ void __launch_bounds__(kThreads)
    first_layer(const double* __restrict__ x, const double* __restrict__ w0, const double* __restrict__ b0,
                double* __restrict__ h1, double* __restrict__ a1, int cp, Geometry geo) {
  constexpr int Q = Basis<DIM>::Q, QB = BO ? DIM + 1 : 1;
  const int64_t total = (geo.ni + geo.nb) * cp;
  pdl_wait();  // W_0 may be the parameter packing's output
  pdl_trigger();
  for (int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += int64_t(gridDim.x) * blockDim.x) {
    const int64_t p = idx / cp;
    const int c = int(idx % cp);
    const double* wr = w0 + int64_t(c) * DIM;
    const double* xp = x + p * DIM;
    double z0 = xp[0] * wr[0];
#pragma unroll
    for (int a = 1; a < DIM; ++a) z0 += xp[a] * wr[a];
    z0 += b0[c];
    if (p < geo.ni) {
      double z[Q], h[Q], aa;
#pragma unroll
      for (int s = 0; s < Q; ++s) z[s] = 0.0;
      z[0] = z0;
#pragma unroll
      for (int a = 0; a < DIM; ++a) z[unit_row<DIM>(a)] = wr[a];
      Jet<DIM, 3>::fwd(z, h, aa);
      double* dst = h1 + p * Q * cp + c;
#pragma unroll
      for (int s = 0; s < Q; ++s) dst[int64_t(s) * cp] = h[s];
      a1[p * cp + c] = aa;
    } else {
      const int64_t b = p - geo.ni;
      double z[QB], h[QB], aa;
      z[0] = z0;
      if constexpr (BO) {
#pragma unroll
        for (int a = 0; a < DIM; ++a) z[unit_row<DIM>(a)] = wr[a];
      }
      Jet<DIM, BO ? 1 : 0>::fwd(z, h, aa);
      double* dst = h1 + (geo.ni * Q + b * QB) * cp + c;
#pragma unroll
      for (int s = 0; s < QB; ++s) dst[int64_t(s) * cp] = h[s];
      a1[p * cp + c] = aa;
    }
  }
}

// ----------------------------------------------------------------------------------
// parameters: flat [W_0..W_L (row-major, true widths), b_0..b_L] <-> padded buffers
struct LayerDesc {
  int cout, cin;          // true widths
  int coutp, cinp;        // padded widths of the stored buffers
  int64_t w_flat, b_flat; // offsets in the flat parameter vector
  int64_t w_buf, b_buf;   // offsets (doubles) of the padded buffers in the workspace
  // gradient partials: element (k, o, i) at wpart[k*ws + o*wo + i], k < wcount;
  // bias (k, o) at bpart[k*bs + o*bo], k < bcount
  int64_t wpart, bpart, ws, wo, bs, bo;
  int wcount, bcount;
};
struct LayerTable {
  int n;
  int64_t params;
  int64_t loss_part, loss_stride;
  int loss_count;
  LayerDesc l[kMaxAffine];
};

__global__ void pack_params(const double* __restrict__ flat, double* __restrict__ ws, const __grid_constant__ LayerTable tab) {
  int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  for (int k = 0; k < tab.n; ++k) {
    const LayerDesc& L = tab.l[k];
    const int64_t nw = int64_t(L.coutp) * L.cinp;
    if (idx < nw) {
      const int o = int(idx / L.cinp), i = int(idx % L.cinp);
      ws[L.w_buf + idx] = (o < L.cout && i < L.cin) ? flat[L.w_flat + int64_t(o) * L.cin + i] : 0.0;
      return;
    }
    idx -= nw;
    if (idx < L.coutp) {
      ws[L.b_buf + idx] = idx < L.cout ? flat[L.b_flat + idx] : 0.0;
      return;
    }
    idx -= L.coutp;
  }
}

// Fixed-order reduction of the per-CTA / per-split partials.  A block covers 32
// consecutive outputs (coalesced loads along i) and splits the partial index over its 16
// warps.  The partials were written by other SMs and sit in L2 or HBM, so the time is
// load latency: each thread issues a batch of 8 independent loads before it adds any of
// them, and combines them in a fixed tree, so the result is bitwise reproducible for a
// given plan.
constexpr int kReduceCols = 32, kReduceRows = 16, kReduceBatch = 8;

__device__ __forceinline__ double strided_sum(const double* base, int64_t stride, int count, int start, int step) {
  double total = 0.0;
  for (int c = start; c < count; c += kReduceBatch * step) {
    double v[kReduceBatch];
#pragma unroll
    for (int r = 0; r < kReduceBatch; ++r) {
      const int cc = c + r * step;
      v[r] = cc < count ? base[int64_t(cc) * stride] : 0.0;
    }
    total += ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
  }
  return total;
}

__global__ void __launch_bounds__(kReduceCols * kReduceRows)
    reduce_grads(const double* __restrict__ ws, double* __restrict__ out, const __grid_constant__ LayerTable tab) {
  __shared__ double part[kReduceRows][kReduceCols];
  const int64_t f = int64_t(blockIdx.x) * kReduceCols + threadIdx.x;
  const int y = threadIdx.y;
  double v = 0.0;
  pdl_wait();  // the partials of every earlier kernel
  pdl_trigger();
  if (f == tab.params) {
    v = strided_sum(ws + tab.loss_part, tab.loss_stride, tab.loss_count, y, kReduceRows);
  } else if (f < tab.params) {
    for (int k = 0; k < tab.n; ++k) {
      const LayerDesc& L = tab.l[k];
      const int64_t nw = int64_t(L.cout) * L.cin;
      if (f >= L.w_flat && f < L.w_flat + nw) {
        const int64_t e = f - L.w_flat;
        const int o = int(e / L.cin), i = int(e % L.cin);
        v = strided_sum(ws + L.wpart + o * L.wo + i, L.ws, L.wcount, y, kReduceRows);
        break;
      }
      if (f >= L.b_flat && f < L.b_flat + L.cout) {
        const int o = int(f - L.b_flat);
        v = strided_sum(ws + L.bpart + o * L.bo, L.bs, L.bcount, y, kReduceRows);
        break;
      }
    }
  }
  part[y][threadIdx.x] = v;
  __syncthreads();
  if (y == 0 && f <= tab.params) {
    double s = 0.0;
#pragma unroll
    for (int r = 0; r < kReduceRows; ++r) s += part[r][threadIdx.x];
    out[f] = s;
  }
}

}  // namespace flashns_b200

// ======================================================================================
// host side: plan + dispatch
using namespace flashns_b200;

struct flashns_b200_plan {
  int dim, head, bo, n_aff, nf, nft;
  int widths[kMaxAffine + 1];
  int padded[kMaxAffine + 1];
  int64_t ni, nb, rows, points;
  double nu, gamma, bc;
  int device, sms;
  Geometry geo;
  LayerTable tab;
  // workspace offsets in doubles
  int64_t off_h[kMaxAffine + 1], off_a1[kMaxAffine + 1], off_d[2], off_coord, off_head;
  int64_t off_wg[kMaxAffine], off_bb[kMaxAffine];
  int64_t workspace_doubles;
  int grid_fwd[kMaxAffine], grid_bwd[kMaxAffine], grid_head, grid_first, grid_coord;
  int wg_splits[kMaxAffine];
  bool fused[kMaxAffine];  // backward layer l runs bwd_fused (dgrad + VJP + wgrad)
  bool fused_head;         // the last forward layer and the output layer run as fwd_head
  bool direct;             // flat parameters already have the padded layout: no pack launch
  int64_t wg_rows[kMaxAffine];
  int wg_bm[kMaxAffine], wg_bn[kMaxAffine];
};

namespace {

int pad_width(int c) {
  if (c <= 32) return 32;
  if (c <= 64) return 64;
  if (c <= 128) return 128;
  return -1;
}

// Launches of one evaluation after its first kernel may overlap the predecessor's tail
// (programmatic stream serialization); every kernel waits (griddepcontrol.wait) before it
// touches its predecessor's outputs.  Set by run_eval around its launch sequence.
thread_local bool t_programmatic = false;

template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                          Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = t_programmatic ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against libcuda)
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiled tensor_map_encoder() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(p);
  });
  return fn;
}

// [rows][cols] row-major FP64 segment read in boxes of box_rows x box_cols; boxes reaching
// past the segment (rows or columns) read zeros
cudaError_t row_tensor_map(CUtensorMap* m, const double* base, int64_t rows, int cols, int box_cols, int box_rows,
                           CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_NONE) {
  const EncodeTiled enc = tensor_map_encoder();
  if (!enc) return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (cols * sizeof(double)) % 16 || (box_cols * sizeof(double)) % 16)
    return cudaErrorInvalidValue;
  const cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows > 0 ? rows : 1)};
  const cuuint64_t strides[1] = {cuuint64_t(cols) * sizeof(double)};
  const cuuint32_t box[2] = {cuuint32_t(box_cols), cuuint32_t(box_rows)};
  const cuuint32_t elem[2] = {1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT64, 2, const_cast<double*>(base), dims, strides, box, elem,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <typename K>
int occupancy(K kernel, size_t smem, int threads) {
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, smem) != cudaSuccess) return 1;
  return std::max(n, 1);
}

template <typename K>
cudaError_t allow_smem(K kernel, size_t smem) {
  if (smem <= 48 * 1024) return cudaSuccess;
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
}

// ---- dispatch tables: runtime (dim, width, boundary order, head) -> template instance
template <int DIM, int CP, int BO>
struct FwdOps {
  using T = FwdTile<DIM, CP>;
  static_assert(fwd_smem_bytes<DIM, CP>(kMaxWidth) <= kMaxSmem, "resident W_l must fit for every input width");
  // square 64-wide 2-D layers run the two-group kernel over 80-row half tiles
  static constexpr bool kPingPongShape = DIM == 2 && CP == kFusedWidth;
  static bool pingpong(int kin) { return kPingPongShape && kin == kFusedWidth; }
  static cudaError_t setup(int& occ, int kin) {
    if constexpr (kPingPongShape) {
      if (kin == kFusedWidth) {
        static_assert(fpp_smem_bytes() <= kMaxSmem, "two-group forward tile exceeds shared memory");
        cudaError_t e = allow_smem(fwd_pingpong<BO>, fpp_smem_bytes());
        occ = occupancy(fwd_pingpong<BO>, fpp_smem_bytes(), kPPThreads);
        return e;
      }
    }
    // the attribute is per kernel and shared by all plans: allow the largest input width
    cudaError_t e = allow_smem(fwd_layer<DIM, CP, BO>, fwd_smem_bytes<DIM, CP>(kMaxWidth));
    occ = occupancy(fwd_layer<DIM, CP, BO>, fwd_smem_bytes<DIM, CP>(kin), T::THREADS);
    return e;
  }
  static int64_t tiles(const Geometry& g, int kin) {
    if (pingpong(kin)) {
      using TL = Tiles<2, BO, PPTile::TC>;
      return (TL::interior(g.ni) + TL::boundary(g.nb) + 1) / 2;
    }
    using TL = Tiles<DIM, BO, T::TC>;
    return TL::interior(g.ni) + TL::boundary(g.nb);
  }
  static cudaError_t launch(int grid, cudaStream_t st, const double* hin, int kin, const double* w, const double* b,
                            double* hout, double* a1, Geometry g) {
    if constexpr (kPingPongShape) {
      if (kin == kFusedWidth) {
        using TL = Tiles<2, BO, PPTile::TC>;
        constexpr int TR = PPTile::TR, BB = pp_boundary_box_rows<BO>();
        const int64_t ri = g.ni * TL::Q, rb = g.nb * TL::QB;  // interior / boundary segment rows
        if (ri > INT32_MAX - TR || rb > INT32_MAX - TR) return cudaErrorInvalidValue;  // TMA rows are int32
        CUtensorMap m[3];
        cudaError_t e;
        if ((e = row_tensor_map(&m[0], hin, ri, kFusedWidth, LDC, TR)) != cudaSuccess ||
            (e = row_tensor_map(&m[1], hin + ri * kFusedWidth, rb, kFusedWidth, LDC, BB)) != cudaSuccess ||
            (e = row_tensor_map(&m[2], hout, ri, kFusedWidth, 16, 4 * TL::Q, CU_TENSOR_MAP_SWIZZLE_128B)) != cudaSuccess)
          return e;
        return launch_kernel(fwd_pingpong<BO>, grid, kPPThreads, fpp_smem_bytes(), st, m[0], m[1], m[2], hin, w, b,
                             hout, a1, g);
      }
    }
    return launch_kernel(fwd_layer<DIM, CP, BO>, grid, T::THREADS, fwd_smem_bytes<DIM, CP>(kin), st, hin, kin, w, b,
                         hout, a1, g);
  }
};

template <int DIM, int CP, int BO, bool FIRST>
struct BwdOps {
  static_assert(bwd_smem_bytes<DIM, CP>() <= kMaxSmem, "backward tile exceeds shared memory");
  static cudaError_t setup(int& occ) {
    constexpr size_t smem = bwd_smem_bytes<DIM, CP>();
    cudaError_t e = allow_smem(bwd_layer<DIM, CP, BO, FIRST>, smem);
    occ = occupancy(bwd_layer<DIM, CP, BO, FIRST>, smem, BwdTile<DIM, CP>::THREADS);
    return e;
  }
  static int64_t tiles(const Geometry& g) {
    using T = BwdTile<DIM, CP>;
    using TL = Tiles<DIM, BO, T::TC>;
    return TL::interior(g.ni) + TL::boundary(g.nb);
  }
  static void launch(int grid, cudaStream_t st, const double* dn, int kout, const double* w, const double* h,
                     const double* a1, double* dc, const double* x, double* cp, Geometry g) {
    launch_kernel(bwd_layer<DIM, CP, BO, FIRST>, grid, BwdTile<DIM, CP>::THREADS, bwd_smem_bytes<DIM, CP>(), st, dn,
                  kout, w, h, a1, dc, x, cp, g);
  }
};

template <int DIM, int BO, bool FIRST>
struct FusedOps {
  // 2-D: the two-group kernel over 80-row half tiles (a CTA takes about two at a time);
  // 3-D: one 8-warp group over 160-row tiles
  static constexpr bool kPingPong = DIM == 2;
  static cudaError_t setup(int& occ) {
    if constexpr (kPingPong) {
      constexpr size_t smem = pp_smem_bytes();
      static_assert(smem <= kMaxSmem, "two-group backward tile exceeds shared memory");
      cudaError_t e = allow_smem(bwd_pingpong<BO, FIRST>, smem);
      occ = occupancy(bwd_pingpong<BO, FIRST>, smem, kPPThreads);
      return e;
    } else {
      constexpr size_t smem = fused_smem_bytes<DIM>();
      cudaError_t e = allow_smem(bwd_fused<DIM, BO, FIRST>, smem);
      occ = occupancy(bwd_fused<DIM, BO, FIRST>, smem, FusedTile<DIM>::THREADS);
      return e;
    }
  }
  static int64_t tiles(const Geometry& g) {
    if constexpr (kPingPong) {
      using TL = Tiles<2, BO, PPTile::TC>;
      return (TL::interior(g.ni) + TL::boundary(g.nb) + 1) / 2;
    } else {
      using TL = Tiles<DIM, BO, FusedTile<DIM>::TC>;
      return TL::interior(g.ni) + TL::boundary(g.nb);
    }
  }
  static cudaError_t launch(int grid, cudaStream_t st, const double* dn, const double* w, const double* h,
                            const double* a1, double* dc, const double* x, double* part, double* wp, Geometry g) {
    if constexpr (kPingPong) {
      using TL = Tiles<2, BO, PPTile::TC>;
      constexpr int TR = PPTile::TR, BB = pp_boundary_box_rows<BO>();
      const int64_t ri = g.ni * TL::Q, rb = g.nb * TL::QB;  // interior / boundary segment rows
      if (ri > INT32_MAX - TR || rb > INT32_MAX - TR) return cudaErrorInvalidValue;  // TMA rows are int32
      CUtensorMap m[4];
      cudaError_t e;
      if ((e = row_tensor_map(&m[0], dn, ri, kFusedWidth, LDC, TR)) != cudaSuccess ||
          (e = row_tensor_map(&m[1], dn + ri * kFusedWidth, rb, kFusedWidth, LDC, BB)) != cudaSuccess ||
          (e = row_tensor_map(&m[2], h, ri, kFusedWidth, LDC, TR)) != cudaSuccess ||
          (e = row_tensor_map(&m[3], h + ri * kFusedWidth, rb, kFusedWidth, LDC, BB)) != cudaSuccess)
        return e;
      return launch_kernel(bwd_pingpong<BO, FIRST>, grid, kPPThreads, pp_smem_bytes(), st, m[0], m[1], m[2], m[3], dn,
                           h, w, a1, dc, x, part, wp, g);
    }
    using T = FusedTile<DIM>;
    using TL = Tiles<DIM, BO, T::TC>;
    constexpr int BB = fused_boundary_box_rows<DIM, BO>();
    const int64_t ri = g.ni * TL::Q, rb = g.nb * TL::QB;  // interior / boundary segment rows
    if (ri > INT32_MAX - T::TR || rb > INT32_MAX - T::TR) return cudaErrorInvalidValue;  // TMA rows are int32
    CUtensorMap m[4];
    cudaError_t e;
    if ((e = row_tensor_map(&m[0], dn, ri, kFusedWidth, LDC, T::TR)) != cudaSuccess ||
        (e = row_tensor_map(&m[1], dn + ri * kFusedWidth, rb, kFusedWidth, LDC, BB)) != cudaSuccess ||
        (e = row_tensor_map(&m[2], h, ri, kFusedWidth, LDC, T::TR)) != cudaSuccess ||
        (e = row_tensor_map(&m[3], h + ri * kFusedWidth, rb, kFusedWidth, LDC, BB)) != cudaSuccess)
      return e;
    return launch_kernel(bwd_fused<DIM, BO, FIRST>, grid, T::THREADS, fused_smem_bytes<DIM>(), st, m[0], m[1], m[2],
                         m[3], dn, h, w, a1, dc, x, part, wp, g);
  }
};

// Dense dgrad (+ jet VJP) of a 2-D 64 -> 64 layer for the reference-ABI hook
// (flashns_stable_dgrad_vjp, hooks.cu): the two-group backward kernel without its weight
// gradient, over dense rows [batch * Q][64] (all points full jets).  d and h must be 16-byte
// aligned (TMA); rows are counted in int32 by the tensor maps.
template <int MODE>
cudaError_t launch_dense_dgrad_pingpong(const double* d, const double* w, const double* h, const double* aux,
                                        double* out, int batch, cudaStream_t stream) {
  using TL = Tiles<2, 0, PPTile::TC>;
  constexpr int TR = PPTile::TR;
  const int64_t rows = int64_t(batch) * TL::Q;
  if (rows > INT32_MAX - TR) return cudaErrorInvalidValue;
  const Geometry g{batch, 0, rows};
  cudaError_t e = allow_smem(bwd_pingpong<0, false, MODE>, pp_smem_bytes());
  if (e != cudaSuccess) return e;
  int device = 0, sms = 0;
  if ((e = cudaGetDevice(&device)) != cudaSuccess ||
      (e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess)
    return e;
  const int64_t pairs = (TL::interior(batch) + 1) / 2;
  const int grid = int(pairs < sms ? pairs : sms);
  CUtensorMap m[4];
  const double* hm = MODE == kHookDgradVjp ? h : d;  // dgrad only: H is never read
  if ((e = row_tensor_map(&m[0], d, rows, kFusedWidth, LDC, TR)) != cudaSuccess ||
      (e = row_tensor_map(&m[1], d, 0, kFusedWidth, LDC, TR)) != cudaSuccess ||
      (e = row_tensor_map(&m[2], hm, rows, kFusedWidth, LDC, TR)) != cudaSuccess ||
      (e = row_tensor_map(&m[3], hm, 0, kFusedWidth, LDC, TR)) != cudaSuccess)
    return e;
  t_programmatic = false;
  return launch_kernel(bwd_pingpong<0, false, MODE>, grid, kPPThreads, pp_smem_bytes(), stream, m[0], m[1], m[2],
                       m[3], d, hm, w, aux, out, static_cast<const double*>(nullptr), static_cast<double*>(nullptr),
                       static_cast<double*>(nullptr), g);
}

template <bool FIRST, typename F>
bool with_fused(int dim, int bo, F&& f) {
  if (dim == 2 && bo == 0) { f(FusedOps<2, 0, FIRST>{}); return true; }
  if (dim == 2 && bo == 1) { f(FusedOps<2, 1, FIRST>{}); return true; }
  if (dim == 3 && bo == 0) { f(FusedOps<3, 0, FIRST>{}); return true; }
  if (dim == 3 && bo == 1) { f(FusedOps<3, 1, FIRST>{}); return true; }
  return false;
}

template <int DIM, int CP, int BO, int HEAD, bool FIRST>
struct HeadOps {
  static constexpr int NF = HeadTraits<HEAD>::NF;
  static cudaError_t setup(int& occ) {
    constexpr size_t smem = head_smem_bytes<DIM, CP, NF>();
    cudaError_t e = allow_smem(head_layer<DIM, CP, BO, HEAD, FIRST>, smem);
    occ = occupancy(head_layer<DIM, CP, BO, HEAD, FIRST>, smem, kThreads);
    return e;
  }
  static int64_t tiles(const Geometry& g) {
    constexpr int Q = Basis<DIM>::Q, QB = BO ? DIM + 1 : 1;
    constexpr int TPI = kHeadRows / Q, TPB = kHeadRows / QB;
    return (g.ni + TPI - 1) / TPI + (g.nb + TPB - 1) / TPB;
  }
  static void launch(int grid, cudaStream_t st, const double* h, const double* a1, const double* w, const double* b,
                     const double* pw, const double* bw, const double* tg, double nu, double gm, double bc, double* dl,
                     const double* x, double* cpart, double* hpart, Geometry g) {
    launch_kernel(head_layer<DIM, CP, BO, HEAD, FIRST>, grid, kThreads, head_smem_bytes<DIM, CP, NF>(), st, h, a1, w,
                  b, pw, bw, tg, nu, gm, bc, dl, x, cpart, hpart, g);
  }
};

template <int DIM, int BO, int HEAD>
struct FwdHeadOps {
  static constexpr int NF = HeadTraits<HEAD>::NF;
  static constexpr bool kPingPong = DIM == 2;  // 2-D: the turn-taking kernels (four groups, 40-row tiles)
  // the stream-function head with first-order boundary rows keeps its epilogue in registers
  static constexpr bool kRegisters = BO == 1 && HEAD == FLASHNS_B200_HEAD_PSI;
  static constexpr int kGroups = kHeadGroups;  // turn-taking groups of the 2-D kernels
  static cudaError_t setup(int& occ) {
    if constexpr (kPingPong && kRegisters) {
      constexpr size_t smem = hpp_smem_bytes<kHeadGroups>();
      static_assert(smem <= kMaxSmem, "turn-taking head tiles exceed shared memory");
      cudaError_t e = allow_smem(head_pingpong<kHeadGroups>, smem);
      occ = occupancy(head_pingpong<kHeadGroups>, smem, kPPThreads);
      return e;
    } else if constexpr (kPingPong) {
      constexpr size_t smem = hpp_staged_smem_bytes<NF, kHeadGroups>();
      static_assert(smem <= kMaxSmem, "turn-taking head tiles exceed shared memory");
      cudaError_t e = allow_smem(head_pingpong_staged<BO, HEAD, kHeadGroups>, smem);
      occ = occupancy(head_pingpong_staged<BO, HEAD, kHeadGroups>, smem, kPPThreads);
      return e;
    } else {
      constexpr size_t smem = fwd_head_smem_bytes<DIM, NF>();
      static_assert(smem <= kMaxSmem, "fused head tile exceeds shared memory");
      cudaError_t e = allow_smem(fwd_head<DIM, BO, HEAD>, smem);
      occ = occupancy(fwd_head<DIM, BO, HEAD>, smem, HeadTile<DIM>::THREADS);
      return e;
    }
  }
  static int64_t tiles(const Geometry& g) {
    if constexpr (kPingPong) {
      using TL = Tiles<2, BO, Ring<kGroups>::T::TC>;
      return (TL::interior(g.ni) + TL::boundary(g.nb) + kGroups - 1) / kGroups;
    } else {
      using TL = Tiles<DIM, BO, HeadTile<DIM>::TC>;
      return TL::interior(g.ni) + TL::boundary(g.nb);
    }
  }
  static cudaError_t launch(int grid, cudaStream_t st, const double* hin, const double* w, const double* b,
                            const double* wl, const double* bl, const double* pw, const double* bw, const double* tg,
                            double nu, double gm, double bc, double* dl, double* hpart, Geometry g) {
    if constexpr (kPingPong) {
      using TT = typename Ring<kGroups>::T;
      using TL = Tiles<2, BO, TT::TC>;
      constexpr int TR = TT::TR, BB = ring_boundary_box_rows<BO, kGroups>();
      const int64_t ri = g.ni * TL::Q, rb = g.nb * TL::QB;  // interior / boundary segment rows
      if (ri > INT32_MAX - TR || rb > INT32_MAX - TR) return cudaErrorInvalidValue;  // TMA rows are int32
      CUtensorMap m[2];
      cudaError_t e;
      if ((e = row_tensor_map(&m[0], hin, ri, kFusedWidth, LDC, TR)) != cudaSuccess ||
          (e = row_tensor_map(&m[1], hin + ri * kFusedWidth, rb, kFusedWidth, LDC, BB)) != cudaSuccess)
        return e;
      if constexpr (kRegisters)
        return launch_kernel(head_pingpong<kHeadGroups>, grid, kPPThreads, hpp_smem_bytes<kHeadGroups>(), st, m[0],
                             m[1], hin, w, b, wl, bl, pw, bw, tg, nu, gm, bc, dl, hpart, g);
      else
        return launch_kernel(head_pingpong_staged<BO, HEAD, kHeadGroups>, grid, kPPThreads,
                             hpp_staged_smem_bytes<NF, kHeadGroups>(), st, m[0], m[1], hin, w, b, wl, bl, pw, bw, tg,
                             nu, gm, bc, dl, hpart, g);
    } else {
      return launch_kernel(fwd_head<DIM, BO, HEAD>, grid, HeadTile<DIM>::THREADS, fwd_head_smem_bytes<DIM, NF>(), st,
                           hin, w, b, wl, bl, pw, bw, tg, nu, gm, bc, dl, hpart, g);
    }
  }
};

template <typename F>
bool with_fwd_head(int dim, int bo, int head, F&& f) {
#define FLASHNS_CASE(D, B, H) \
  if (dim == D && bo == B && head == H) { f(FwdHeadOps<D, B, H>{}); return true; }
  FLASHNS_CASE(2, 0, 0) FLASHNS_CASE(2, 0, 1) FLASHNS_CASE(2, 1, 1)
  FLASHNS_CASE(3, 0, 1) FLASHNS_CASE(3, 1, 1)
#undef FLASHNS_CASE
  return false;
}

// Generic visitor over the runtime parameters.
template <template <int, int, int> class Ops, typename F>
bool with_fwd(int dim, int cp, int bo, F&& f) {
#define FLASHNS_CASE(D, C, B) \
  if (dim == D && cp == C && bo == B) { f(Ops<D, C, B>{}); return true; }
  FLASHNS_CASE(2, 32, 0) FLASHNS_CASE(2, 64, 0) FLASHNS_CASE(2, 128, 0)
  FLASHNS_CASE(2, 32, 1) FLASHNS_CASE(2, 64, 1) FLASHNS_CASE(2, 128, 1)
  FLASHNS_CASE(3, 32, 0) FLASHNS_CASE(3, 64, 0) FLASHNS_CASE(3, 128, 0)
  FLASHNS_CASE(3, 32, 1) FLASHNS_CASE(3, 64, 1) FLASHNS_CASE(3, 128, 1)
#undef FLASHNS_CASE
  return false;
}

template <bool FIRST, typename F>
bool with_bwd(int dim, int cp, int bo, F&& f) {
#define FLASHNS_CASE(D, C, B) \
  if (dim == D && cp == C && bo == B) { f(BwdOps<D, C, B, FIRST>{}); return true; }
  FLASHNS_CASE(2, 32, 0) FLASHNS_CASE(2, 64, 0) FLASHNS_CASE(2, 128, 0)
  FLASHNS_CASE(2, 32, 1) FLASHNS_CASE(2, 64, 1) FLASHNS_CASE(2, 128, 1)
  FLASHNS_CASE(3, 32, 0) FLASHNS_CASE(3, 64, 0) FLASHNS_CASE(3, 128, 0)
  FLASHNS_CASE(3, 32, 1) FLASHNS_CASE(3, 64, 1) FLASHNS_CASE(3, 128, 1)
#undef FLASHNS_CASE
  return false;
}

template <bool FIRST, typename F>
bool with_head(int dim, int cp, int bo, int head, F&& f) {
#define FLASHNS_CASE(D, C, B, H) \
  if (dim == D && cp == C && bo == B && head == H) { f(HeadOps<D, C, B, H, FIRST>{}); return true; }
  FLASHNS_CASE(2, 32, 0, 0) FLASHNS_CASE(2, 64, 0, 0) FLASHNS_CASE(2, 128, 0, 0)
  FLASHNS_CASE(2, 32, 0, 1) FLASHNS_CASE(2, 64, 0, 1) FLASHNS_CASE(2, 128, 0, 1)
  FLASHNS_CASE(2, 32, 1, 1) FLASHNS_CASE(2, 64, 1, 1) FLASHNS_CASE(2, 128, 1, 1)
  FLASHNS_CASE(3, 32, 0, 1) FLASHNS_CASE(3, 64, 0, 1) FLASHNS_CASE(3, 128, 0, 1)
  FLASHNS_CASE(3, 32, 1, 1) FLASHNS_CASE(3, 64, 1, 1) FLASHNS_CASE(3, 128, 1, 1)
#undef FLASHNS_CASE
  return false;
}

template <int BM, int BN>
struct WgradOps {
  static size_t smem() { return sizeof(double) * kStages * KC * ((BM + 4) + (BN + 4)); }
  static cudaError_t setup() { return allow_smem(wgrad_kernel<BM, BN>, smem()); }
  static void launch(dim3 grid, cudaStream_t st, const double* d, int kout, const double* h, int kin, Geometry g,
                     int64_t rps, double* wp) {
    launch_kernel(wgrad_kernel<BM, BN>, grid, kThreads, smem(), st, d, kout, h, kin, g, rps, wp);
  }
};

template <typename F>
bool with_wgrad(int bm, int bn, F&& f) {
  if (bm == 32 && bn == 32) { f(WgradOps<32, 32>{}); return true; }
  if (bm == 32 && bn == 64) { f(WgradOps<32, 64>{}); return true; }
  if (bm == 64 && bn == 32) { f(WgradOps<64, 32>{}); return true; }
  if (bm == 64 && bn == 64) { f(WgradOps<64, 64>{}); return true; }
  return false;
}

int first_launch(int dim, int bo, int grid, cudaStream_t st, const double* x, const double* w, const double* b,
                 double* h, double* a1, int cp, Geometry g) {
  if (dim == 2 && bo == 0) launch_kernel(first_layer<2, 0>, grid, kThreads, 0, st, x, w, b, h, a1, cp, g);
  else if (dim == 2) launch_kernel(first_layer<2, 1>, grid, kThreads, 0, st, x, w, b, h, a1, cp, g);
  else if (bo == 0) launch_kernel(first_layer<3, 0>, grid, kThreads, 0, st, x, w, b, h, a1, cp, g);
  else launch_kernel(first_layer<3, 1>, grid, kThreads, 0, st, x, w, b, h, a1, cp, g);
  return int(cudaGetLastError());
}

}  // namespace

// The dense 64 -> 64 dgrad (+ VJP) for the reference-ABI hook in hooks.cu: the two-group
// backward kernel in 2-D, the one-group fused backward kernel (160-row tiles) in 3-D
template <int MODE>
cudaError_t launch_dense_dgrad_fused3(const double* d, const double* w, const double* h, const double* aux,
                                      double* out, int batch, cudaStream_t stream) {
  using T = FusedTile<3>;
  using TL = Tiles<3, 0, T::TC>;
  const int64_t rows = int64_t(batch) * TL::Q;
  if (rows > INT32_MAX - T::TR) return cudaErrorInvalidValue;
  const Geometry g{batch, 0, rows};
  cudaError_t e = allow_smem(bwd_fused<3, 0, false, MODE>, fused_smem_bytes<3>());
  if (e != cudaSuccess) return e;
  int device = 0, sms = 0;
  if ((e = cudaGetDevice(&device)) != cudaSuccess ||
      (e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess)
    return e;
  const int64_t tiles = TL::interior(batch);
  const int grid = int(tiles < sms ? tiles : sms);
  CUtensorMap m[4];
  const double* hm = MODE == kHookDgradVjp ? h : d;  // dgrad only: H is never read
  if ((e = row_tensor_map(&m[0], d, rows, kFusedWidth, LDC, T::TR)) != cudaSuccess ||
      (e = row_tensor_map(&m[1], d, 0, kFusedWidth, LDC, T::TR)) != cudaSuccess ||
      (e = row_tensor_map(&m[2], hm, rows, kFusedWidth, LDC, T::TR)) != cudaSuccess ||
      (e = row_tensor_map(&m[3], hm, 0, kFusedWidth, LDC, T::TR)) != cudaSuccess)
    return e;
  t_programmatic = false;
  return launch_kernel(bwd_fused<3, 0, false, MODE>, grid, T::THREADS, fused_smem_bytes<3>(), stream, m[0], m[1],
                       m[2], m[3], d, hm, w, aux, out, static_cast<const double*>(nullptr),
                       static_cast<double*>(nullptr), static_cast<double*>(nullptr), g);
}

cudaError_t flashns_b200::dense_dgrad_64(int dim, bool fused, const double* d, const double* w, const double* h,
                                         const double* aux, double* out, int batch, cudaStream_t stream) {
  if (dim == 3)
    return fused ? launch_dense_dgrad_fused3<kHookDgradVjp>(d, w, h, aux, out, batch, stream)
                 : launch_dense_dgrad_fused3<kHookDgrad>(d, w, h, aux, out, batch, stream);
  return fused ? launch_dense_dgrad_pingpong<kHookDgradVjp>(d, w, h, aux, out, batch, stream)
               : launch_dense_dgrad_pingpong<kHookDgrad>(d, w, h, aux, out, batch, stream);
}

// ======================================================================================
extern "C" {

int flashns_b200_plan_launch_kinds(const flashns_b200_plan* p, int* kinds, int capacity, int* count);

int flashns_b200_plan_create(int dim, int head, int boundary_order, int n_affine, const int* widths,
                             int64_t interior_points, int64_t boundary_points, double viscosity,
                             double gradient_weight, double boundary_weight, flashns_b200_plan** out) {
  if (!out || !widths) return int(cudaErrorInvalidValue);
  *out = nullptr;
  if ((dim != 2 && dim != 3) || (head != FLASHNS_B200_HEAD_UVP && head != FLASHNS_B200_HEAD_PSI) ||
      (boundary_order != 0 && boundary_order != 1) || n_affine < 2 || n_affine > kMaxAffine ||
      interior_points < 0 || boundary_points < 0)
    return int(cudaErrorInvalidValue);
  const int nf = head == FLASHNS_B200_HEAD_UVP ? 3 : 2;
  if (head == FLASHNS_B200_HEAD_UVP && (dim != 2 || boundary_order != 0)) return int(cudaErrorInvalidValue);
  if (widths[0] != dim || widths[n_affine] != nf) return int(cudaErrorInvalidValue);
  if (!(viscosity >= 0) || !(gradient_weight >= 0) || !(boundary_weight >= 0)) return int(cudaErrorInvalidValue);
  flashns_b200_plan* p = new (std::nothrow) flashns_b200_plan();
  if (!p) return int(cudaErrorMemoryAllocation);
  std::memset(p, 0, sizeof(*p));
  p->dim = dim; p->head = head; p->bo = boundary_order; p->n_aff = n_affine; p->nf = nf;
  p->nft = (head == FLASHNS_B200_HEAD_PSI && boundary_order) ? 3 : nf;
  p->nu = viscosity; p->gamma = gradient_weight; p->bc = boundary_weight;
  for (int l = 0; l <= n_affine; ++l) p->widths[l] = widths[l];
  p->padded[0] = dim;
  p->padded[n_affine] = nf;
  for (int l = 1; l < n_affine; ++l) {
    p->padded[l] = widths[l] >= 1 ? pad_width(widths[l]) : -1;
    if (p->padded[l] < 0) { delete p; return int(cudaErrorInvalidValue); }
  }
  const int q = dim == 2 ? 10 : 20, qb = boundary_order ? dim + 1 : 1;
  if (interior_points > (INT64_C(1) << 40) || boundary_points > (INT64_C(1) << 40)) { delete p; return int(cudaErrorInvalidValue); }
  p->ni = interior_points; p->nb = boundary_points;
  p->rows = interior_points * q + boundary_points * qb;
  p->points = interior_points + boundary_points;
  // the kernels address tile rows with 32-bit TMA coordinates; far more rows than a
  // 180 GB device can hold checkpoints for, refused here rather than mis-addressed
  if (p->rows > INT32_MAX) { delete p; return int(cudaErrorInvalidValue); }
  p->geo = Geometry{p->ni, p->nb, p->rows};
  if (cudaGetDevice(&p->device) != cudaSuccess ||
      cudaDeviceGetAttribute(&p->sms, cudaDevAttrMultiProcessorCount, p->device) != cudaSuccess) {
    delete p; return int(cudaErrorInvalidDevice);
  }
  const int nh = n_affine - 1;  // hidden layers
  int maxc = 0;
  for (int l = 1; l <= nh; ++l) maxc = std::max(maxc, p->padded[l]);
  if (p->rows > INT64_MAX / 8 / std::max(maxc, 1) / (nh + 4)) { delete p; return int(cudaErrorInvalidValue); }

  // ---- grids (persistent kernels: one wave of resident CTAs)
  cudaError_t err = cudaSuccess;
  for (int l = 1; l < nh; ++l) {  // forward layer l: H_l (width padded[l]) -> H_{l+1}
    const int cp = p->padded[l + 1];
    with_fwd<FwdOps>(dim, cp, boundary_order, [&](auto ops) {
      int occ = 1;
      cudaError_t e = ops.setup(occ, p->padded[l]);
      if (e != cudaSuccess) err = e;
      const int64_t t = ops.tiles(p->geo, p->padded[l]);
      p->grid_fwd[l] = int(std::max<int64_t>(1, std::min<int64_t>(t, int64_t(occ) * p->sms)));
    });
  }
  for (int l = 1; l < nh; ++l) {  // backward layer l: D_{l+1} -> D_l (width padded[l])
    const int cp = p->padded[l];
    p->fused[l] = cp == kFusedWidth && p->padded[l + 1] == kFusedWidth;
    auto f = [&](auto ops) {
      int occ = 1;
      cudaError_t e = ops.setup(occ);
      if (e != cudaSuccess) err = e;
      const int64_t t = ops.tiles(p->geo);
      p->grid_bwd[l] = int(std::max<int64_t>(1, std::min<int64_t>(t, int64_t(occ) * p->sms)));
    };
    if (p->fused[l]) {
      if (l == 1) with_fused<true>(dim, boundary_order, f);
      else with_fused<false>(dim, boundary_order, f);
    } else if (l == 1) {
      with_bwd<true>(dim, cp, boundary_order, f);
    } else {
      with_bwd<false>(dim, cp, boundary_order, f);
    }
  }
  {
    auto f = [&](auto ops) {
      int occ = 1;
      cudaError_t e = ops.setup(occ);
      if (e != cudaSuccess) err = e;
      const int64_t t = ops.tiles(p->geo);
      p->grid_head = int(std::max<int64_t>(1, std::min<int64_t>(t, int64_t(occ) * p->sms)));
    };
    const bool ok = nh == 1 ? with_head<true>(dim, p->padded[nh], boundary_order, head, f)
                            : with_head<false>(dim, p->padded[nh], boundary_order, head, f);
    if (!ok) { delete p; return int(cudaErrorInvalidValue); }
    // square 64-wide last hidden layer: fuse it with the output layer (one launch, no H_L)
    p->fused_head = nh >= 2 && p->padded[nh] == kFusedWidth && p->padded[nh - 1] == kFusedWidth &&
                    with_fwd_head(dim, boundary_order, head, f);
  }
  if (err != cudaSuccess) { delete p; return int(err); }
  p->grid_first = int(std::max<int64_t>(1, std::min<int64_t>((p->points * p->padded[1] + kThreads - 1) / kThreads,
                                                             int64_t(p->sms) * 8)));
  p->grid_coord = nh == 1 ? p->grid_head : p->grid_bwd[1];

  // ---- workspace layout (doubles)
  int64_t off = 0;
  auto take = [&](int64_t n) { const int64_t o = off; off += (n + 31) / 32 * 32; return o; };
  LayerTable& tab = p->tab;
  tab.n = n_affine;
  int64_t flat = 0;
  for (int l = 0; l < n_affine; ++l) flat += int64_t(widths[l]) * widths[l + 1];
  int64_t fb = flat;
  for (int l = 0; l < n_affine; ++l) fb += widths[l + 1];
  tab.params = fb;
  int64_t fw = 0, fbias = flat;
  for (int l = 0; l < n_affine; ++l) {
    LayerDesc& L = tab.l[l];
    L.cout = widths[l + 1]; L.cin = widths[l];
    L.coutp = p->padded[l + 1]; L.cinp = p->padded[l];
    L.w_flat = fw; L.b_flat = fbias;
    fw += int64_t(L.cout) * L.cin; fbias += L.cout;
    L.w_buf = take(int64_t(L.coutp) * L.cinp);
    L.b_buf = take(L.coutp);
  }
  // widths that need no padding: the kernels read W_l and b_l straight from the flat vector
  // (every block then starts on a 16-byte boundary of a 16-byte aligned parameter vector)
  p->direct = true;
  for (int l = 0; l < n_affine; ++l) {
    const LayerDesc& L = tab.l[l];
    if (L.coutp != L.cout || L.cinp != L.cin || (L.w_flat & 1) || (L.b_flat & 1) || (L.cinp & 1)) p->direct = false;
  }
  for (int l = 1; l <= nh; ++l) {
    p->off_h[l] = take(p->rows * p->padded[l]);
    p->off_a1[l] = take(p->points * p->padded[l]);
  }
  p->off_d[0] = take(p->rows * maxc);
  p->off_d[1] = take(p->rows * maxc);
  // layer 0 partials: [grid_coord][CP1][dim+1]
  p->off_coord = take(int64_t(p->grid_coord) * p->padded[1] * (dim + 1));
  {
    LayerDesc& L = tab.l[0];
    L.wpart = p->off_coord; L.ws = int64_t(p->padded[1]) * (dim + 1); L.wo = dim + 1;
    L.bpart = p->off_coord + dim; L.bs = L.ws; L.bo = dim + 1;
    L.wcount = L.bcount = p->grid_coord;
  }
  // bias partials of layer l-1 written by backward layer l >= 2: [grid_bwd[l]][CP_l]
  for (int l = 2; l < nh; ++l) {
    p->off_bb[l] = take(int64_t(p->grid_bwd[l]) * p->padded[l]);
    LayerDesc& L = tab.l[l - 1];
    L.bpart = p->off_bb[l]; L.bs = p->padded[l]; L.bo = 1; L.bcount = p->grid_bwd[l];
  }
  // hidden-layer wgrad partials
  for (int l = 1; l < nh; ++l) {
    const int kout = p->padded[l + 1], kin = p->padded[l];
    if (p->fused[l]) {  // one [CP][CP] partial per CTA of the fused backward
      p->off_wg[l] = take(int64_t(p->grid_bwd[l]) * kout * kin);
      LayerDesc& L = tab.l[l];
      L.wpart = p->off_wg[l]; L.ws = int64_t(kout) * kin; L.wo = kin;
      L.wcount = p->grid_bwd[l];
      continue;
    }
    const int bm = std::min(kout, 64), bn = std::min(kin, 64);
    const int blocks = (kout / bm) * (kin / bn);
    const int target = 2 * p->sms;
    int64_t splits = std::max<int64_t>(1, target / blocks);
    int64_t rps = (p->rows + splits - 1) / splits;
    rps = std::max<int64_t>(KC, (rps + KC - 1) / KC * KC);
    splits = std::max<int64_t>(1, (p->rows + rps - 1) / rps);
    p->wg_splits[l] = int(splits); p->wg_rows[l] = rps; p->wg_bm[l] = bm; p->wg_bn[l] = bn;
    p->off_wg[l] = take(splits * kout * kin);
    LayerDesc& L = tab.l[l];
    L.wpart = p->off_wg[l]; L.ws = int64_t(kout) * kin; L.wo = kin;
    L.wcount = int(splits);
    with_wgrad(bm, bn, [&](auto ops) {
      cudaError_t e = ops.setup();
      if (e != cudaSuccess) err = e;
    });
  }
  // head partials: [grid_head][NF*CP + NF + 1 + CP]: dW_L, db_L, loss, db_{L-1}
  {
    const int cp = p->padded[nh];
    const int64_t stride = int64_t(nf) * cp + nf + 1 + cp;
    p->off_head = take(int64_t(p->grid_head) * stride);
    LayerDesc& L = tab.l[nh];
    L.wpart = p->off_head; L.ws = stride; L.wo = cp;
    L.bpart = p->off_head + int64_t(nf) * cp; L.bs = stride; L.bo = 1;
    L.wcount = L.bcount = p->grid_head;
    if (nh >= 2) {
      LayerDesc& B = tab.l[nh - 1];
      B.bpart = p->off_head + int64_t(nf) * cp + nf + 1; B.bs = stride; B.bo = 1; B.bcount = p->grid_head;
    }
    tab.loss_part = p->off_head + int64_t(nf) * cp + nf;
    tab.loss_stride = stride;
    tab.loss_count = p->grid_head;
  }
  if (err != cudaSuccess) { delete p; return int(err); }
  if (p->rows == 0) {  // nothing to evaluate: every partial count is zero, outputs are zeros
    for (int l = 0; l < n_affine; ++l) tab.l[l].wcount = tab.l[l].bcount = 0;
    tab.loss_count = 0;
  }
  p->workspace_doubles = off;
  *out = p;
  return int(cudaSuccess);
}

int flashns_b200_plan_destroy(flashns_b200_plan* plan) {
  delete plan;
  return int(cudaSuccess);
}

int flashns_b200_plan_workspace_bytes(const flashns_b200_plan* plan, size_t* bytes) {
  if (!plan || !bytes) return int(cudaErrorInvalidValue);
  *bytes = size_t(plan->workspace_doubles) * sizeof(double);
  return int(cudaSuccess);
}

int flashns_b200_plan_parameter_count(const flashns_b200_plan* plan, int64_t* count) {
  if (!plan || !count) return int(cudaErrorInvalidValue);
  *count = plan->tab.params;
  return int(cudaSuccess);
}

int flashns_b200_device_fault(int* fault, int clear) {
  if (!fault) return int(cudaErrorInvalidValue);
  cudaError_t e = cudaMemcpyFromSymbol(fault, g_device_fault, sizeof(int));
  if (e == cudaSuccess && clear) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_device_fault, &zero, sizeof(int));
  }
  return int(e);
}

int flashns_b200_wait_selftest(unsigned spins, int* gave_up, cudaStream_t stream) {
  if (!gave_up || spins == 0 || spins > (1u << 17)) return int(cudaErrorInvalidValue);
  wait_timeout_probe<<<1, 1, 0, stream>>>(spins, gave_up);
  return int(cudaGetLastError());
}

int flashns_b200_plan_launch_count(const flashns_b200_plan* plan, int* count) {
  return flashns_b200_plan_launch_kinds(plan, nullptr, 0, count);
}

// A plan's grids and buffers belong to the device that was current when it was created;
// launching it with another device current would hand that device foreign pointers.
static bool on_plan_device(const flashns_b200_plan* p) {
  int device = -1;
  return cudaGetDevice(&device) == cudaSuccess && device == p->device;
}

static int run_eval(const flashns_b200_plan* p, const double* coordinates, const double* parameters,
                    const double* pde_weights, const double* boundary_weights, const double* target,
                    double* gradient_and_loss, void* workspace, size_t workspace_bytes, cudaStream_t stream,
                    cudaEvent_t* events, int capacity, int* recorded) {
  if (!p || !parameters || !gradient_and_loss || !workspace) return int(cudaErrorInvalidValue);
  if (workspace_bytes < size_t(p->workspace_doubles) * sizeof(double)) return int(cudaErrorInvalidValue);
  if (!on_plan_device(p)) return int(cudaErrorInvalidDevice);
  if (p->points && !coordinates) return int(cudaErrorInvalidValue);
  if (p->ni && !pde_weights) return int(cudaErrorInvalidValue);
  if (p->nb && (!boundary_weights || !target)) return int(cudaErrorInvalidValue);
  if ((reinterpret_cast<uintptr_t>(workspace) & 15) != 0) return int(cudaErrorInvalidValue);
  if (p->direct && (reinterpret_cast<uintptr_t>(parameters) & 15) != 0) return int(cudaErrorInvalidValue);
  int marks = 0;
  auto mark = [&]() {
    if (events && marks < capacity) cudaEventRecord(events[marks], stream);
    ++marks;
  };
  double* ws = static_cast<double*>(workspace);
  const LayerTable& tab = p->tab;
  cudaError_t e = cudaSuccess;
  // the first kernel of the evaluation follows the caller's work normally; the rest may start
  // under their predecessor's tail (not while per-kernel events are being recorded)
  struct ProgrammaticScope {
    ~ProgrammaticScope() { t_programmatic = false; }
  } programmatic_scope;
  t_programmatic = false;
  const bool overlap = events == nullptr;
  if (!p->direct) {
    int64_t packed = 0;
    for (int l = 0; l < p->n_aff; ++l) packed += int64_t(tab.l[l].coutp) * tab.l[l].cinp + tab.l[l].coutp;
    mark();
    pack_params<<<unsigned((packed + kThreads - 1) / kThreads), kThreads, 0, stream>>>(parameters, ws, tab);
    if ((e = cudaGetLastError()) != cudaSuccess) return int(e);
    t_programmatic = overlap;
  }
  // padded layer buffers, or the flat vector itself when no layer needs padding
  auto Wp = [&](const LayerDesc& L) -> const double* { return p->direct ? parameters + L.w_flat : ws + L.w_buf; };
  auto Bp = [&](const LayerDesc& L) -> const double* { return p->direct ? parameters + L.b_flat : ws + L.b_buf; };
  const int nh = p->n_aff - 1;
  const Geometry g = p->geo;
  if (p->rows > 0) {
    const LayerDesc& L0 = tab.l[0];
    mark();
    int r = first_launch(p->dim, p->bo, p->grid_first, stream, coordinates, Wp(L0), Bp(L0),
                         ws + p->off_h[1], ws + p->off_a1[1], p->padded[1], g);
    if (r) return r;
    t_programmatic = overlap;
    for (int l = 1; l < nh - (p->fused_head ? 1 : 0); ++l) {
      const LayerDesc& L = tab.l[l];
      mark();
      cudaError_t le = cudaSuccess;
      with_fwd<FwdOps>(p->dim, p->padded[l + 1], p->bo, [&](auto ops) {
        le = ops.launch(p->grid_fwd[l], stream, ws + p->off_h[l], p->padded[l], Wp(L), Bp(L),
                        ws + p->off_h[l + 1], ws + p->off_a1[l + 1], g);
      });
      if (le != cudaSuccess) return int(le);
      if ((e = cudaGetLastError()) != cudaSuccess) return int(e);
    }
    if (p->fused_head) {
      const LayerDesc& L = tab.l[nh - 1];
      const LayerDesc& H = tab.l[nh];
      mark();
      cudaError_t le = cudaSuccess;
      with_fwd_head(p->dim, p->bo, p->head, [&](auto ops) {
        le = ops.launch(p->grid_head, stream, ws + p->off_h[nh - 1], Wp(L), Bp(L), Wp(H),
                        Bp(H), pde_weights, boundary_weights, target, p->nu, p->gamma, p->bc,
                        ws + p->off_d[nh % 2], ws + p->off_head, g);
      });
      if (le != cudaSuccess) return int(le);
      if ((e = cudaGetLastError()) != cudaSuccess) return int(e);
    } else {
      const LayerDesc& L = tab.l[nh];
      auto f = [&](auto ops) {
        ops.launch(p->grid_head, stream, ws + p->off_h[nh], ws + p->off_a1[nh], Wp(L), Bp(L),
                   pde_weights, boundary_weights, target, p->nu, p->gamma, p->bc, ws + p->off_d[nh % 2],
                   coordinates, ws + p->off_coord, ws + p->off_head, g);
      };
      mark();
      if (nh == 1) with_head<true>(p->dim, p->padded[nh], p->bo, p->head, f);
      else with_head<false>(p->dim, p->padded[nh], p->bo, p->head, f);
      if ((e = cudaGetLastError()) != cudaSuccess) return int(e);
    }
    for (int l = nh - 1; l >= 1; --l) {
      const LayerDesc& L = tab.l[l];
      const double* dn = ws + p->off_d[(l + 1) % 2];
      auto f = [&](auto ops) {
        ops.launch(p->grid_bwd[l], stream, dn, p->padded[l + 1], Wp(L), ws + p->off_h[l], ws + p->off_a1[l],
                   ws + p->off_d[l % 2], coordinates, ws + (l == 1 ? p->off_coord : p->off_bb[l]), g);
      };
      mark();
      if (p->fused[l]) {
        cudaError_t fe = cudaSuccess;
        auto ff = [&](auto ops) {
          fe = ops.launch(p->grid_bwd[l], stream, dn, Wp(L), ws + p->off_h[l], ws + p->off_a1[l],
                          ws + p->off_d[l % 2], coordinates, ws + (l == 1 ? p->off_coord : p->off_bb[l]),
                          ws + p->off_wg[l], g);
        };
        if (l == 1) with_fused<true>(p->dim, p->bo, ff);
        else with_fused<false>(p->dim, p->bo, ff);
        if (fe != cudaSuccess) return int(fe);
        if ((e = cudaGetLastError()) != cudaSuccess) return int(e);
        continue;
      }
      if (l == 1) with_bwd<true>(p->dim, p->padded[l], p->bo, f);
      else with_bwd<false>(p->dim, p->padded[l], p->bo, f);
      if ((e = cudaGetLastError()) != cudaSuccess) return int(e);
      const int kout = p->padded[l + 1], kin = p->padded[l];
      const dim3 grid(unsigned(p->wg_splits[l]), unsigned((kout / p->wg_bm[l]) * (kin / p->wg_bn[l])));
      mark();
      with_wgrad(p->wg_bm[l], p->wg_bn[l], [&](auto ops) {
        ops.launch(grid, stream, dn, kout, ws + p->off_h[l], kin, g, p->wg_rows[l], ws + p->off_wg[l]);
      });
      if ((e = cudaGetLastError()) != cudaSuccess) return int(e);
    }
  }
  mark();
  launch_kernel(reduce_grads, dim3(unsigned((tab.params + 1 + kReduceCols - 1) / kReduceCols)),
                dim3(kReduceCols, kReduceRows), 0, stream, static_cast<const double*>(ws), gradient_and_loss, tab);
  e = cudaGetLastError();
  mark();
  if (recorded) *recorded = marks;
  return int(e);
}

int flashns_b200_eval(const flashns_b200_plan* p, const double* coordinates, const double* parameters,
                      const double* pde_weights, const double* boundary_weights, const double* target,
                      double* gradient_and_loss, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  return run_eval(p, coordinates, parameters, pde_weights, boundary_weights, target, gradient_and_loss, workspace,
                  workspace_bytes, stream, nullptr, 0, nullptr);
}

int flashns_b200_eval_marked(const flashns_b200_plan* p, const double* coordinates, const double* parameters,
                             const double* pde_weights, const double* boundary_weights, const double* target,
                             double* gradient_and_loss, void* workspace, size_t workspace_bytes, cudaStream_t stream,
                             cudaEvent_t* events, int capacity, int* recorded) {
  if (!events || capacity < 1 || !recorded) return int(cudaErrorInvalidValue);
  return run_eval(p, coordinates, parameters, pde_weights, boundary_weights, target, gradient_and_loss, workspace,
                  workspace_bytes, stream, events, capacity, recorded);
}

int flashns_b200_plan_launch_kinds(const flashns_b200_plan* p, int* kinds, int capacity, int* count) {
  if (!p || !count) return int(cudaErrorInvalidValue);
  std::vector<int> k;
  const int nh = p->n_aff - 1;
  if (!p->direct) k.push_back(FLASHNS_B200_KERNEL_PACK);
  if (p->rows > 0) {
    k.push_back(FLASHNS_B200_KERNEL_FIRST);
    for (int l = 1; l < nh - (p->fused_head ? 1 : 0); ++l) k.push_back(FLASHNS_B200_KERNEL_FORWARD);
    k.push_back(p->fused_head ? FLASHNS_B200_KERNEL_FORWARD_HEAD : FLASHNS_B200_KERNEL_HEAD);
    for (int l = nh - 1; l >= 1; --l) {
      k.push_back(FLASHNS_B200_KERNEL_BACKWARD);
      if (!p->fused[l]) k.push_back(FLASHNS_B200_KERNEL_WGRAD);
    }
  }
  k.push_back(FLASHNS_B200_KERNEL_REDUCE);
  *count = int(k.size());
  if (kinds) for (int i = 0; i < int(k.size()) && i < capacity; ++i) kinds[i] = k[i];
  return int(cudaSuccess);
}

}  // extern "C"

// ======================================================================================
// No-allocation entry point.
//
// Some callers cannot allocate device memory for the workspace: code driven from a host
// runtime with no CUDA allocator of its own (a Go, Java or JavaScript process binding this
// library through its C ABI), or a caller that must not grow device memory after start-up.
// flashns_b200_eval_static runs the same evaluation with its scratch in the file-scope
// array below, so it needs no workspace argument and calls no allocator.
//
// * Capacity: FLASHNS_B200_STATIC_WORKSPACE_BYTES (64 MiB) per GPU.  A plan whose
//   workspace (flashns_b200_plan_workspace_bytes) is larger is rejected with
//   cudaErrorInvalidValue before anything is launched.  The 2-64x4-2 psi net with
//   first-order boundary rows fits about 1,000 interior + 250 boundary points.
// * Every GPU that loads this library holds the array until the process exits.
// * Host code may not use the array's name as a device pointer (it is a host-side
//   stand-in).  The first call on a device, with that device current, looks up the
//   array's device address with cudaGetSymbolAddress and caches it with the device's
//   current context; make that first call before any stream capture.  A later call that
//   finds another context current (after cudaDeviceReset, say) looks the address up again.
// * All calls on a device share the one array and it keeps the last call's contents.
//   Nothing in it has to start at zero: every evaluation writes each scratch value
//   before reading it.  Calls whose executions overlap on the GPU (other streams, or
//   other host threads) race on the array; serialize them.
#include <mutex>

namespace {
__device__ __align__(256) double g_static_workspace[FLASHNS_B200_STATIC_WORKSPACE_BYTES / sizeof(double)];
std::mutex g_static_mutex;
constexpr int kMaxDevices = 64;
struct StaticScratch {
  CUcontext context;  // the context the address belongs to
  void* address;
};
StaticScratch g_static_scratch[kMaxDevices] = {};

// cuCtxGetCurrent through the runtime's driver entry point (no link against libcuda)
using CtxGetCurrent = CUresult (*)(CUcontext*);
CUcontext current_context() {
  static CtxGetCurrent fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrent>(p);
  });
  CUcontext ctx = nullptr;
  if (!fn || fn(&ctx) != CUDA_SUCCESS) return nullptr;
  return ctx;
}
}  // namespace

extern "C" int flashns_b200_eval_static(const flashns_b200_plan* p, const double* coordinates,
                                        const double* parameters, const double* pde_weights,
                                        const double* boundary_weights, const double* target,
                                        double* gradient_and_loss, cudaStream_t stream) {
  if (!p) return int(cudaErrorInvalidValue);
  const size_t need = size_t(p->workspace_doubles) * sizeof(double);
  if (need > size_t(FLASHNS_B200_STATIC_WORKSPACE_BYTES)) return int(cudaErrorInvalidValue);
  int device = -1;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return int(e);
  if (device != p->device || device < 0 || device >= kMaxDevices) return int(cudaErrorInvalidDevice);
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_static_mutex);
    StaticScratch& slot = g_static_scratch[device];
    const CUcontext ctx = current_context();
    if (!slot.address || !ctx || ctx != slot.context) {
      void* address = nullptr;
      e = cudaGetSymbolAddress(&address, g_static_workspace);
      if (e != cudaSuccess) return int(e);
      slot.address = address;
      slot.context = current_context();  // the lookup made the device's context current
    }
    scratch = slot.address;
  }
  return run_eval(p, coordinates, parameters, pde_weights, boundary_weights, target, gradient_and_loss, scratch,
                  size_t(FLASHNS_B200_STATIC_WORKSPACE_BYTES), stream, nullptr, 0, nullptr);
}

// ======================================================================================
// Forward-only fields at points (for acceptance grids and validation): a plan created
// with interior_points = 0 carries every point as a boundary point; the forward kernels
// run as in an evaluation and the output layer writes per point (u, v, p):
// psi head with first-order rows: (psi_y, -psi_x, p); value rows: the raw outputs.
namespace flashns_b200 {
template <int DIM, int BO, int HEAD>
__global__ void __launch_bounds__(kThreads)
    fields_kernel(const double* __restrict__ hL, const double* __restrict__ wL, const double* __restrict__ bL, int cp,
                  double* __restrict__ out, int64_t points) {
  constexpr int NF = HeadTraits<HEAD>::NF, QB = BO ? DIM + 1 : 1;
  constexpr int NFT = (HEAD == FLASHNS_B200_HEAD_PSI && BO) ? 3 : NF;
  for (int64_t p = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; p < points; p += int64_t(gridDim.x) * blockDim.x) {
    double y[QB][NF];
#pragma unroll
    for (int r = 0; r < QB; ++r) {
      const double* h = hL + (p * QB + r) * cp;
#pragma unroll
      for (int o = 0; o < NF; ++o) {
        double s = 0.0;
        for (int c = 0; c < cp; ++c) s += h[c] * wL[o * cp + c];
        y[r][o] = r == 0 ? s + bL[o] : s;
      }
    }
    double* dst = out + p * NFT;
    if constexpr (NFT == 3 && HEAD == FLASHNS_B200_HEAD_PSI) {
      dst[0] = y[unit_row<DIM>(1)][0];   // u = psi_y
      dst[1] = -y[unit_row<DIM>(0)][0];  // v = -psi_x
      dst[2] = y[0][1];                  // p
    } else {
#pragma unroll
      for (int o = 0; o < NF; ++o) dst[o] = y[0][o];
    }
  }
}
}  // namespace flashns_b200

extern "C" int flashns_b200_fields(const flashns_b200_plan* p, const double* coordinates, const double* parameters,
                                   double* fields, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  if (!p || !parameters || !fields || !workspace || p->ni != 0) return int(cudaErrorInvalidValue);
  if (workspace_bytes < size_t(p->workspace_doubles) * sizeof(double)) return int(cudaErrorInvalidValue);
  if (!on_plan_device(p)) return int(cudaErrorInvalidDevice);
  if ((reinterpret_cast<uintptr_t>(workspace) & 15) != 0) return int(cudaErrorInvalidValue);
  if (p->points == 0) return int(cudaSuccess);
  if (!coordinates) return int(cudaErrorInvalidValue);
  double* ws = static_cast<double*>(workspace);
  const LayerTable& tab = p->tab;
  int64_t packed = 0;
  for (int l = 0; l < p->n_aff; ++l) packed += int64_t(tab.l[l].coutp) * tab.l[l].cinp + tab.l[l].coutp;
  pack_params<<<unsigned((packed + kThreads - 1) / kThreads), kThreads, 0, stream>>>(parameters, ws, tab);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return int(e);
  const int nh = p->n_aff - 1;
  const Geometry g = p->geo;
  const LayerDesc& L0 = tab.l[0];
  int r = first_launch(p->dim, p->bo, p->grid_first, stream, coordinates, ws + L0.w_buf, ws + L0.b_buf,
                       ws + p->off_h[1], ws + p->off_a1[1], p->padded[1], g);
  if (r) return r;
  for (int l = 1; l < nh; ++l) {
    const LayerDesc& L = tab.l[l];
    cudaError_t le = cudaSuccess;
    with_fwd<FwdOps>(p->dim, p->padded[l + 1], p->bo, [&](auto ops) {
      le = ops.launch(p->grid_fwd[l], stream, ws + p->off_h[l], p->padded[l], ws + L.w_buf, ws + L.b_buf,
                      ws + p->off_h[l + 1], ws + p->off_a1[l + 1], g);
    });
    if (le != cudaSuccess) return int(le);
    if ((e = cudaGetLastError()) != cudaSuccess) return int(e);
  }
  const LayerDesc& LL = tab.l[nh];
  const unsigned grid = unsigned(std::min<int64_t>((p->points + kThreads - 1) / kThreads, int64_t(p->sms) * 8));
  const double* h = ws + p->off_h[nh];
  const int cp = p->padded[nh];
  if (p->head == FLASHNS_B200_HEAD_UVP) fields_kernel<2, 0, FLASHNS_B200_HEAD_UVP><<<grid, kThreads, 0, stream>>>(h, ws + LL.w_buf, ws + LL.b_buf, cp, fields, p->points);
  else if (p->dim == 2 && p->bo) fields_kernel<2, 1, FLASHNS_B200_HEAD_PSI><<<grid, kThreads, 0, stream>>>(h, ws + LL.w_buf, ws + LL.b_buf, cp, fields, p->points);
  else if (p->dim == 2) fields_kernel<2, 0, FLASHNS_B200_HEAD_PSI><<<grid, kThreads, 0, stream>>>(h, ws + LL.w_buf, ws + LL.b_buf, cp, fields, p->points);
  else if (p->bo) fields_kernel<3, 1, FLASHNS_B200_HEAD_PSI><<<grid, kThreads, 0, stream>>>(h, ws + LL.w_buf, ws + LL.b_buf, cp, fields, p->points);
  else fields_kernel<3, 0, FLASHNS_B200_HEAD_PSI><<<grid, kThreads, 0, stream>>>(h, ws + LL.w_buf, ws + LL.b_buf, cp, fields, p->points);
  return int(cudaGetLastError());
}
