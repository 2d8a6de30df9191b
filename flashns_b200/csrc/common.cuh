// Shared device helpers for the FlashNS B200 kernels (sm_100a, FP64).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace flashns_b200 {

// 16-byte asynchronous global->shared copy; src_size 0 zero-fills the
// destination (rows past the end of a segment).
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  const int size = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(size));
}
// Bulk prefetch of a contiguous global range into L2 (16-byte aligned start and size).
__device__ __forceinline__ void prefetch_l2(const void* gmem, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(gmem), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// D = A*B + D with FP64 tensor-core MMA (DMMA).  Fragment layout (PTX ISA,
// m16n8k8 .f64): g = lane/4, t = lane%4;
//   a0=A[g][t] a1=A[g+8][t] a2=A[g][t+4] a3=A[g+8][t+4]
//   b0=B[t][g] b1=B[t+4][g]
//   c0=C[g][2t] c1=C[g][2t+1] c2=C[g+8][2t] c3=C[g+8][2t+1]
__device__ __forceinline__ void mma_m16n8k8(double (&c)[4], const double (&a)[4], double b0, double b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f64.f64.f64.f64 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+d"(c[0]), "+d"(c[1]), "+d"(c[2]), "+d"(c[3])
      : "d"(a[0]), "d"(a[1]), "d"(a[2]), "d"(a[3]), "d"(b0), "d"(b1));
}

// Row of the first-order coefficient along `axis` in the canonical basis
// (sorted by (|alpha|, alpha)): unit rows appear in reverse axis order.
template <int DIM>
__host__ __device__ constexpr int unit_row(int axis) { return DIM - axis; }

template <int DIM>
struct Basis;
template <>
struct Basis<2> { static constexpr int Q = 10; };
template <>
struct Basis<3> { static constexpr int Q = 20; };

}  // namespace flashns_b200
