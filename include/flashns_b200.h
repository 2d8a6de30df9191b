/* C ABI of the FlashNS B200 (sm_100a) FP64 PINN loss + parameter-gradient library.
 *
 * Conventions (kept from the reference bindings, experiments/pinn_v8/native.py:53-68 and
 * experiments/pinn_v8/native.cu:47-62,97-107):
 *   - FP64, contiguous, device pointers on the current device; the caller allocates every
 *     output and scratch buffer; no call allocates device memory.
 *   - every call is asynchronous on `stream` and returns a cudaError_t value as int
 *     (0 = success); argument errors return cudaErrorInvalidValue (1).
 *   - sizes are int64_t; empty inputs succeed and write zeros where gradients are owned.
 */
#ifndef FLASHNS_B200_H
#define FLASHNS_B200_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FLASHNS_B200_HEAD_UVP 0 /* outputs (u, v, p): src/flashns/ns_seed.py:26-87 objective */
#define FLASHNS_B200_HEAD_PSI 1 /* outputs (psi, p): u = psi_y, v = -psi_x (no reference counterpart) */

typedef struct flashns_b200_plan flashns_b200_plan;

/* Plan of one packed evaluation.  Replaces the construction of
 * PackedPINN(x, interior_count, ..., layout="compact", loss=NSLoss(...))
 * (src/flashns/pinn_packed.py:16-88) for a fixed geometry.  Host-only; reads the
 * current device's SM count; allocates no device memory.
 *   dim             2 (x, y) or 3 (x, y, t)
 *   head            FLASHNS_B200_HEAD_UVP (dim 2) or FLASHNS_B200_HEAD_PSI
 *   boundary_order  0: boundary points carry value rows (reference layout,
 *                   src/flashns/jet_packed.py:12-41); 1: first-order rows (psi head:
 *                   boundary targets are (u, v, p))
 *   widths          n_affine+1 entries: dim, hidden widths (1..128), outputs (3 uvp / 2 psi)
 *   interior_points, boundary_points: the packed rows (interior x Q + boundary x (1 or dim+1))
 *                   must not exceed 2^31 - 1
 *   viscosity, gradient_weight, boundary_weight: NSLoss (src/flashns/ns_seed.py:13-23) */
int flashns_b200_plan_create(int dim, int head, int boundary_order, int n_affine, const int* widths,
                             int64_t interior_points, int64_t boundary_points, double viscosity,
                             double gradient_weight, double boundary_weight, flashns_b200_plan** plan);
int flashns_b200_plan_destroy(flashns_b200_plan* plan);
/* bytes of caller-allocated device workspace (16-byte aligned) one evaluation needs */
int flashns_b200_plan_workspace_bytes(const flashns_b200_plan* plan, size_t* bytes);
/* P = sum over layers of (in*out + out) */
int flashns_b200_plan_parameter_count(const flashns_b200_plan* plan, int64_t* count);
/* number of kernels one flashns_b200_eval launches */
int flashns_b200_plan_launch_count(const flashns_b200_plan* plan, int* count);

/* kernel kinds of one evaluation, in launch order (for per-kernel timing) */
#define FLASHNS_B200_KERNEL_PACK 0     /* flat parameters -> padded layer buffers */
#define FLASHNS_B200_KERNEL_FIRST 1    /* coordinates -> first affine -> tanh jet */
#define FLASHNS_B200_KERNEL_FORWARD 2  /* DMMA GEMM + bias + tanh-jet epilogue */
#define FLASHNS_B200_KERNEL_HEAD 3     /* output layer + residual seed + output gradients + jet VJP */
#define FLASHNS_B200_KERNEL_BACKWARD 4 /* DMMA dgrad + jet-VJP epilogue (+ coordinate contraction) */
#define FLASHNS_B200_KERNEL_WGRAD 5    /* DMMA weight gradient, split over rows */
#define FLASHNS_B200_KERNEL_REDUCE 6   /* fixed-order partial reduction -> grad, loss */
#define FLASHNS_B200_KERNEL_FORWARD_HEAD 7 /* last 64-wide forward layer fused with the output layer */
int flashns_b200_plan_launch_kinds(const flashns_b200_plan* plan, int* kinds, int capacity, int* count);

/* Device fault word of the current device: nonzero once a kernel gave up a bounded wait on
 * one of its own asynchronous copies (the kernel then returned without finishing, and the
 * outputs of that evaluation are invalid).  Synchronous; clear != 0 resets the word.
 * No reference counterpart (the reference kernels have no in-kernel waits). */
int flashns_b200_device_fault(int* fault, int clear);
/* Launches one thread that waits on an mbarrier nothing arrives at, bounded by `spins`
 * polls (1..131072, each suspending at most 10 us).  It writes 1 to the device int
 * `gave_up` and raises the fault word when the bound ran out, so callers can check that a
 * stuck wait ends with an error instead of a hang.  No reference counterpart. */
int flashns_b200_wait_selftest(unsigned spins, int* gave_up, cudaStream_t stream);

/* One complete loss + parameter-gradient evaluation.  Replaces
 * PackedPINN.__call__(weights, biases) -> (loss, [dW_0..dW_L, db_0..db_L])
 * (src/flashns/pinn_packed.py:93-191) together with the Engine's flattening
 * (experiments/pinn_v8/runtime.py:114-117).  The device current at the call must be the
 * one the plan was created on (cudaErrorInvalidDevice otherwise, nothing launched).
 *   coordinates       [interior + boundary, dim]   interior points first
 *   parameters        [P]  flat [W_0 .. W_L (row-major [out, in]), b_0 .. b_L]
 *   pde_weights       [interior]                   globally normalized
 *   boundary_weights  [boundary, F], target [boundary, F]
 *                     F = 3 for (uvp head) and (psi head, boundary_order 1): (u, v, p);
 *                     F = 2 for (psi head, boundary_order 0): (psi, p)
 *   gradient_and_loss [P + 1]  gradient in the flat order, then the loss
 * The workspace, and the parameter vector, start on 16-byte boundaries (when no layer
 * width needs padding the kernels read W_l and b_l straight from the parameter vector).
 * Deterministic: fixed-order reductions, no floating-point atomics. */
int flashns_b200_eval(const flashns_b200_plan* plan, const double* coordinates, const double* parameters,
                      const double* pde_weights, const double* boundary_weights, const double* target,
                      double* gradient_and_loss, void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* flashns_b200_eval that also records events[i] before the i-th launch and one after the
 * last (count+1 events); *recorded = events written.  Used for per-kernel timing. */
int flashns_b200_eval_marked(const flashns_b200_plan* plan, const double* coordinates, const double* parameters,
                             const double* pde_weights, const double* boundary_weights, const double* target,
                             double* gradient_and_loss, void* workspace, size_t workspace_bytes, cudaStream_t stream,
                             cudaEvent_t* events, int capacity, int* recorded);

/* Forward-only fields at points (acceptance grids, validation).  The plan must have
 * interior_points = 0 (all points ride the boundary-row path).  fields [points, F]:
 * psi head with boundary_order 1 -> (u, v, p) = (psi_y, -psi_x, p); value rows -> raw outputs
 * (F = outputs).  Replaces the reference's forward-only jets(x, W, b) evaluation
 * (experiments/pinn_solver/problem.py:189-196). */
int flashns_b200_fields(const flashns_b200_plan* plan, const double* coordinates, const double* parameters,
                        double* fields, void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* No-allocation variant of flashns_b200_eval (no counterpart in the reference).
 * For callers that cannot allocate device memory -- a host runtime without a CUDA
 * allocator that binds this C ABI (Go, Java, JavaScript FFI), or a process that must not
 * grow device memory after start-up.  The scratch lives in a file-scope device array of
 * FLASHNS_B200_STATIC_WORKSPACE_BYTES (64 MiB) that every GPU loading the library keeps
 * until exit; plans needing more workspace are rejected with cudaErrorInvalidValue.  The
 * first call on a device looks up the array's address and should come before any stream
 * capture; a call that finds another context current (after cudaDeviceReset) looks it up
 * again.  All calls share the array: calls that overlap on the GPU race. */
#define FLASHNS_B200_STATIC_WORKSPACE_BYTES (64u * 1024u * 1024u)
int flashns_b200_eval_static(const flashns_b200_plan* plan, const double* coordinates, const double* parameters,
                             const double* pde_weights, const double* boundary_weights, const double* target,
                             double* gradient_and_loss, cudaStream_t stream);

/* FP64 tensor-core throughput probe: `blocks` CTAs of 256 threads run `iters` rounds of
 * 8 independent DMMA m16n8k8 per warp from registers; *flops = floating-point operations
 * issued.  Time it with events on `stream` for the FP64 roofline denominator. */
int flashns_b200_fp64_peak_probe(int blocks, int iters, double* sink, double* flops, cudaStream_t stream);

/* The FP64 throughput of each instruction shape, for the peak table (no reference
 * counterpart).  `blocks` CTAs of `threads` threads (a multiple of 32, at most 1024) run
 * `iters` rounds; *flops = floating-point operations issued.  Kinds: register-only chains
 * of 8 MMAs per warp for each f64 shape (M16N8K8 is flashns_b200_fp64_peak_probe and needs
 * 256 threads), 16 DFMA chains per thread, or SMEM: m16n8k8 fed from shared memory in the
 * kernels' tile shape (one m16 and five n8 tiles per warp, a 32-deep K slice per round). */
#define FLASHNS_B200_PROBE_M16N8K8 0
#define FLASHNS_B200_PROBE_M8N8K4 1
#define FLASHNS_B200_PROBE_M16N8K4 2
#define FLASHNS_B200_PROBE_M16N8K16 3
#define FLASHNS_B200_PROBE_DFMA 4
#define FLASHNS_B200_PROBE_SMEM 5
int flashns_b200_fp64_probe(int kind, int blocks, int threads, int iters, double* sink, double* flops,
                            cudaStream_t stream);

/* ---------------------------------------------------------------------------------------
 * Per-stage hooks with the reference's C ABI (same names, argument order and meaning,
 * caller-provided scratch), so the reference's ctypes bindings can load this library.
 * Packed layout: rows [full_points x Q ; value_points x 1] x channels, Q = 10 (2-D) / 20 (3-D).
 */

/* experiments/pinn_v8/native.cu:47-62.  backward=0: input = Z -> output = H, output_auxiliary
 * = a1 [points, C]; backward=1: input = H, auxiliary = a1, seed = bar_H -> output = bar_Z. */
int flashns_v8_activation(int dimension, int backward, const double* input, const double* auxiliary,
                          const double* seed, double* output, double* output_auxiliary, int64_t full_points,
                          int64_t value_points, int channels, cudaStream_t stream);
/* experiments/pinn_v8/native.cu:115-121: first affine jet of physical coordinates [points, dim] */
int flashns_v8_coordinate_affine(int dimension, const double* coordinates, const double* weight, const double* bias,
                                 double* output, int64_t full_points, int64_t value_points, int channels,
                                 cudaStream_t stream);
/* experiments/pinn_v8/native.cu:123-129: the same followed by the stable tanh jet */
int flashns_v8_coordinate_affine_activation(int dimension, const double* coordinates, const double* weight,
                                            const double* bias, double* hidden, double* auxiliary,
                                            int64_t full_points, int64_t value_points, int channels,
                                            cudaStream_t stream);
/* experiments/pinn_v8/native.cu:174-200: bar_H = D[rows,3] W[3,C] ((d0 w0 + d1 w1) + d2 w2);
 * fused=1 applies the jet VJP with hidden/auxiliary */
int flashns_v8_tail3(int dimension, int fused, const double* d, const double* weight, const double* hidden,
                     const double* auxiliary, double* output, int64_t full_points, int64_t value_points, int channels,
                     cudaStream_t stream);
/* experiments/pinn_v8/native.cu:275-281: dW0[C,dim], db0[C] from bar_Z; partials scratch
 * [(points+7)/8, C, dim+1]; deterministic (fixed 8-point tiles, fixed-order merge) */
int flashns_v8_coordinate_wgrad(int dimension, const double* derivative, const double* coordinates, double* partials,
                                double* weight_gradient, double* bias_gradient, int64_t full_points,
                                int64_t value_points, int channels, cudaStream_t stream);
/* experiments/pinn_v8/native.cu:283-290: the first activation's VJP followed by the same */
int flashns_v8_coordinate_activation_wgrad(int dimension, const double* hidden, const double* auxiliary,
                                           const double* seed, const double* coordinates, double* partials,
                                           double* weight_gradient, double* bias_gradient, int64_t full_points,
                                           int64_t value_points, int channels, cudaStream_t stream);
/* experiments/pinn_v8/native.cu:325-337: (u, v, p) residual loss + seed; interior jets
 * [ni,10,3], boundary value rows [nb, stride >= 3]; partial_loss[(ni+nb+127)/128] (summed by
 * the caller) */
int flashns_v8_loss_seed(const double* jets, const double* boundary, const double* pde_weights,
                         const double* boundary_weights, const double* target, double* interior_seed,
                         double* boundary_seed, double* partial_loss, int64_t ni, int64_t nb, int64_t boundary_stride,
                         double nu, double gamma, double bc_scale, cudaStream_t stream);

/* Dense [B,Q,C] layout (experiments/cuda_jet_h100/stable_kernels.cu:93-131, stable_dgrad.cu:150-174) */
int flashns_stable_activation(int dim, bool backward, const double* value, const double* adjoint, const double* aux_in,
                              double* output, double* aux_out, size_t batch, size_t channels, cudaStream_t stream);
int flashns_stable_tail3(int dim, bool fused, const double* d, const double* weight, const double* hidden,
                         const double* aux, double* output, size_t batch, size_t channels, cudaStream_t stream);
/* out[B,Q,Cin] = D[B,Q,Cout] W[Cout,Cin] (fused: followed by the jet VJP with h[B,Q,Cin], aux[B,Cin]),
 * on the FP64 tensor pipe (DMMA) with the VJP in the epilogue; any Cout, Cin; pointers 8-byte aligned */
int flashns_stable_dgrad_vjp(int dim, bool fused, const double* d, const double* w, const double* h, const double* aux,
                             double* out, int batch, int cout, int cin, cudaStream_t stream);
/* Residual values at interior points: jets [n, Q, F] coefficient-major -> out [n, R]; head UVP:
 * the nine residuals of src/flashns/ns_seed.py:26-64 (R = 9); head PSI: (r_u, r_v) (R = 2). */
int flashns_b200_residuals(int head, int dim, const double* jets, double nu, double* out, int64_t n,
                           cudaStream_t stream);

/* Vector kernels of the device-resident L-BFGS (no reference counterpart: the reference
 * uses torch.optim.LBFGS, experiments/pinn_solver/solve.py:150-167).
 *   row_dots:      out[r] = rows[r] . v for r < k (rows [k][stride]); fixed-order reductions */
int flashns_b200_row_dots(const double* rows, int64_t stride, int k, const double* v, double* out, int64_t n,
                          cudaStream_t stream);

/* Device-resident L-BFGS state.  The curvature pairs live in a ring of `slots` = history + 1
 * physical rows (one spare) of S and Y ([slots][stride] each); SY[a][b] = s_a . y_b and
 * YY[a][b] = y_a . y_b ([slots][slots], physical rows); state = int32 {k stored pairs,
 * h spare slot, have_pair, 0}; scal = f64 {gamma, f0, g0.d, f, g.d, k, t, 0}; coef = f64[256]
 * (cs at 0.., cy at 128..); order = int32[128] (physical rows of the stored pairs, oldest
 * first).  history <= 128.  Every step reads its counts from the device, so one iteration
 * needs no host round trip before its first line-search trial.  scal[6] holds the trial step.
 *   lbfgs_pair_slot:    if have_pair: S[h] = x - x0, Y[h] = g - g0
 *   lbfgs_ring_dots:    out[b] = (b < slots ? S[b] : Y[b - slots]) . v, b < 2 slots;
 *                       v = `v`, or the spare row Y[h] when from_slot (skipped without a pair)
 *   lbfgs_commit:       keep the spare pair if s.y > 1e-12 y.y (dots from ring_dots with
 *                       from_slot): fill its SY column and YY row/column, advance h, k
 *   lbfgs_coefficients: compact-representation coefficients from dots = [S.g ; Y.g]
 *                       (Byrd, Nocedal, Schnabel 1994, Thm 2.2), gamma = s.y / y.y newest
 *   lbfgs_direction:    d = -(gamma g + sum_i cs[i] S[order[i]] + cy[i] Y[order[i]])
 *   lbfgs_save:         x0 = x, g0 = g, scal[1] = *f
 *   lbfgs_step_point:   x = x0 + scal[6] d (the trial step read on the device, so a CUDA
 *                       graph of a line-search trial replays with a new step) */
int flashns_b200_lbfgs_pair_slot(const double* x, const double* x0, const double* g, const double* g0, double* S,
                                 double* Y, int64_t stride, const int* state, int64_t n, cudaStream_t stream);
int flashns_b200_lbfgs_ring_dots(const double* S, const double* Y, int64_t stride, int slots, const double* v,
                                 const int* state, int from_slot, double* out, int64_t n, cudaStream_t stream);
int flashns_b200_lbfgs_commit(const double* dots, double* SY, double* YY, int slots, int* state, cudaStream_t stream);
int flashns_b200_lbfgs_coefficients(const double* SY, const double* YY, const double* dots, int slots,
                                    const int* state, double* coef, int* order, double* scal, cudaStream_t stream);
int flashns_b200_lbfgs_direction(const double* S, const double* Y, int64_t stride, const int* order, const int* state,
                                 const double* coef, const double* g, const double* scal, double* d, int64_t n,
                                 cudaStream_t stream);
int flashns_b200_lbfgs_save(const double* x, const double* g, const double* f, double* x0, double* g0, double* scal,
                            int64_t n, cudaStream_t stream);
int flashns_b200_lbfgs_step_point(const double* x0, const double* scal, const double* d, double* x, int64_t n,
                                  cudaStream_t stream);

/* One Adam update of the solver's first phase (the reference's captured FP64 Adam,
 * experiments/pinn_solver/backends.py:216-240): m = b1 m + (1-b1) g, v = b2 v + (1-b2) g^2,
 * x -= lr (m / (1 - b1^step)) / (sqrt(v / (1 - b2^step)) + eps); step counts from 1. */
int flashns_b200_adam_step(double* x, const double* g, double* m, double* v, int64_t n, double lr, double beta1,
                           double beta2, double eps, int64_t step, cudaStream_t stream);

/* ---- data preparation on the device (flashns_b200/csrc/sampling.cu) ----
 * Points i = 0 .. n-1 go to out[i * ld + d] (d < dim <= 8) as lo[d] + span[d] * u, the
 * product and the sum rounded separately; lo == NULL drops the sum, span == NULL the
 * product.  `directions`, `shift`, `lo` and `span` are HOST arrays, read at the call. */

/* Scrambled Sobol points first .. first+n-1 (first + n <= 2^30), bit-identical to
 * torch.quasirandom.SobolEngine(dim, scramble=True, seed).draw() after `first` earlier
 * draws, as the reference solver samples (experiments/pinn_solver/problem.py:68-99).
 * directions = the engine's sobolstate [dim][30], shift = its shift [dim]. */
int flashns_b200_sobol_points(const int64_t* directions, const int64_t* shift, int dim, int64_t first, int64_t n,
                              const double* lo, const double* span, double* out, int64_t ld, cudaStream_t stream);

/* Uniform points from Philox4x64-10 keyed by (key0, key1): coordinate d of point i is
 * word (first + i) * dim + d of numpy.random.Generator(numpy.random.Philox(key=key0 +
 * 2^64 key1)).random()'s stream, (word >> 11) * 2^-53. */
int flashns_b200_philox_points(uint64_t key0, uint64_t key1, int dim, int64_t first, int64_t n, const double* lo,
                               const double* span, double* out, int64_t ld, cudaStream_t stream);

/* PackedLayout.coordinates (src/flashns/jet_packed.py:43-53) of x [full_points +
 * value_points][dim]: out [full_points * Q + value_points][dim], Q = C(dim + 3, 3). */
int flashns_b200_pack_coordinates(const double* x, int64_t full_points, int64_t value_points, int dim, double* out,
                                  cudaStream_t stream);

/* dynamic shared memory per CTA of the dense dgrad (its 2-D kernel, 64 -> 64) */
int flashns_stable_dgrad_shared_bytes(void);

/* Plan-based dense dgrad under the reference's Hopper names
 * (experiments/cuda_jet_hopper/hopper.cu:287-353, bound by
 * experiments/cuda_jet_hopper/hopper.py:37-63): create keeps D [batch*Q, cout] and
 * W [cout, cin] (cout, cin in {32, 64}; both 16-byte aligned; 0 < batch <= INT_MAX/20);
 * launch writes out [batch*Q, cin] = D W, followed by the jet VJP with hidden [batch*Q, cin]
 * and aux [batch, cin] when fused.  resources fills 9 values: registers per thread, threads
 * per CTA, dynamic and static shared bytes, local bytes per thread, predicted CTAs per SM,
 * max dynamic shared bytes, binary and PTX versions. */
int flashns_hopper_initialize(void);
int flashns_hopper_resources(int dim, bool fused, long long* values);
int flashns_hopper_create(int dim, const double* d, const double* w, int batch, int cout, int cin, void** plan);
void flashns_hopper_destroy(void* plan);
int flashns_hopper_launch(void* plan, int dim, bool fused, const double* hidden, const double* aux, double* output,
                          cudaStream_t stream);

#ifdef __cplusplus
}
#endif
#endif
