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

// ---- mbarrier + bulk (TMA engine) copies, shared::cta barriers, no cluster multicast.
// Waits are bounded: after kMbarSpins polls (each suspends for at most kMbarHintNs) the
// caller gets false and must report a fault instead of waiting forever.
constexpr unsigned kMbarSpins = 1u << 17;
constexpr unsigned kMbarHintNs = 10000u;
__device__ __forceinline__ unsigned smem_u32(const void* p) {
  return static_cast<unsigned>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_inval(uint64_t* bar) {
  asm volatile("mbarrier.inval.shared::cta.b64 [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}
// arrive and add `bytes` to the transaction count of the current phase
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)),
               "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity, unsigned spins = kMbarSpins) {
  const unsigned a = smem_u32(bar);
  for (unsigned i = 0; i < spins; ++i) {
    unsigned done;
    asm volatile(
        "{\n .reg .pred p;\n"
        " mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done) : "r"(a), "r"(parity), "r"(kMbarHintNs) : "memory");
    if (done) return true;
  }
  return false;
}
// contiguous global -> shared copy by the TMA engine (16-byte aligned ends, size % 16 == 0),
// completing `bytes` of the barrier's transaction count
__device__ __forceinline__ void bulk_g2s(void* smem, const void* gmem, unsigned bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
          smem_u32(smem)),
      "l"(gmem), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---- named barriers (ids 1..15) over some of the block's warps: `count` threads, a
// multiple of 32, every warp taking part whole.  bar.arrive counts without waiting.
__device__ __forceinline__ void named_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ void named_arrive(int id, int count) {
  asm volatile("bar.arrive %0, %1;\n" ::"r"(id), "r"(count) : "memory");
}
// named_sync that also tells whether any of the `count` threads passed `v` = true
__device__ __forceinline__ bool named_sync_or(int id, int count, bool v) {
  unsigned r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 q, %1, 0;\n bar.red.or.pred p, %2, %3, q;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(r) : "r"(unsigned(v)), "r"(id), "r"(count) : "memory");
  return r != 0;
}

// orders this thread's earlier generic-proxy shared-memory accesses before its later
// async-proxy (TMA) ones
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }

// 2-D tiled TMA store (no multicast) of the box at `smem` (laid out as the tensor map's
// swizzle mode says) to coordinates (x = column, y = row); rows and columns past the map's
// extent are not written.  x * 8 bytes is a multiple of 16 and x, y >= 0.  Tracked by the
// issuing thread's bulk group (bulk_commit, bulk_wait_read, bulk_wait).
__device__ __forceinline__ void tma_store_2d(const void* tensor_map, int x, int y, const void* smem) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];\n" ::"l"(tensor_map),
               "r"(x), "r"(y), "r"(smem_u32(smem))
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;\n" ::: "memory"); }
// every bulk store this thread issued has finished reading its shared-memory source
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory"); }
// every bulk store this thread issued has completed its writes
__device__ __forceinline__ void bulk_wait() { asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory"); }

// 2-D tiled TMA load (no multicast): box at coordinates (x = column, y = row) of the tensor
// map into shared memory, completing its bytes on `bar`.  x * 8 bytes is a multiple of 16.
__device__ __forceinline__ void tma_load_2d(void* smem, const void* tensor_map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::"r"(
          smem_u32(smem)),
      "l"(tensor_map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Programmatic dependent launch: a kernel launched with programmatic stream serialization
// may start while its predecessor drains; it waits here before touching the predecessor's
// outputs (a no-op without a programmatic predecessor), then lets its own dependents start.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

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
