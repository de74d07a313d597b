// Warp-level bf16 tensor-core helpers (mma.sync m16n8k16 + ldmatrix) for the
// small, latency-bound matrix products inside the GDN chunk recurrence and the
// banded-attention tiles.
//
// Fragment layouts (PTX ISA, mma.m16n8k16 .bf16):
//   A (16x16, row-major)  a[0]: (r, c..c+1)  a[1]: (r+8, c..)  a[2]: (r, c+8..)  a[3]: (r+8, c+8..)
//   B (16x8, k x n)       b[0]: (k=c..c+1, n=r)  b[1]: (k=c+8.., n=r)
//   C (16x8, fp32)        c[0..1]: (r, 2q..2q+1)  c[2..3]: (r+8, 2q..)
// with r = lane / 4, q = lane % 4, c = 2q.
#pragma once

#include "common.cuh"

namespace llmyb {
namespace mma {

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Four 8x8 b16 matrices; lane i supplies the row address for row (i % 8) of
// matrix (i / 8).
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_addr(p)));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_addr(p)));
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// A fragment (16 x 16) from a row-major bf16 tile: rows r0.., cols c0..;
// ld in elements.
__device__ __forceinline__ void load_a(uint32_t (&a)[4], const __nv_bfloat16* base, int ld, int r0,
                                       int c0) {
  const int lane = threadIdx.x & 31;
  const int row = r0 + (lane & 7) + ((lane >> 3) & 1) * 8;
  const int col = c0 + (lane >> 4) * 8;
  ldsm_x4(a, base + row * ld + col);
}

// A fragment from a tile stored TRANSPOSED ([k][m] row-major): A[m][k] = T[k][m].
__device__ __forceinline__ void load_a_t(uint32_t (&a)[4], const __nv_bfloat16* base, int ld, int m0,
                                         int k0) {
  const int lane = threadIdx.x & 31;
  // matrices: (m0..7,k0..7) (m8..15,k0..7) (m0..7,k8..15) (m8..15,k8..15), each read transposed
  const int kk = k0 + (lane & 7) + (lane >> 4) * 8;
  const int mm = m0 + ((lane >> 3) & 1) * 8;
  ldsm_x4_t(a, base + kk * ld + mm);
}

// Two B fragments (k16 x n16 -> n-blocks n0..7 and n8..15) from a tile stored
// as [n][k] row-major (k contiguous).
__device__ __forceinline__ void load_b_nk(uint32_t (&b)[4], const __nv_bfloat16* base, int ld, int n0,
                                          int k0) {
  const int lane = threadIdx.x & 31;
  // matrices: (n0..7,k0..7) (n0..7,k8..15) (n8..15,k0..7) (n8..15,k8..15)
  const int n = n0 + (lane & 7) + (lane >> 4) * 8;
  const int k = k0 + ((lane >> 3) & 1) * 8;
  ldsm_x4(b, base + n * ld + k);
}

// Two B fragments from a tile stored as [k][n] row-major (n contiguous).
__device__ __forceinline__ void load_b_kn(uint32_t (&b)[4], const __nv_bfloat16* base, int ld, int k0,
                                          int n0) {
  const int lane = threadIdx.x & 31;
  // matrices (transposed reads): (k0..7,n0..7) (k8..15,n0..7) (k0..7,n8..15) (k8..15,n8..15)
  const int k = k0 + (lane & 7) + ((lane >> 3) & 1) * 8;
  const int n = n0 + (lane >> 4) * 8;
  ldsm_x4_t(b, base + k * ld + n);
}

// 16-byte asynchronous global -> shared copy; src_bytes = 0 zero-fills.
// fp32 -> tf32 (round to nearest, ties away), kept in a 32-bit register
__device__ __forceinline__ uint32_t to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

// D (16x8 fp32) += A (16x8 tf32, row-major) B (8x8 tf32), mma.m16n8k8 fragments:
//   a[0]: (g, t)  a[1]: (g+8, t)  a[2]: (g, t+4)  a[3]: (g+8, t+4)
//   b[0]: (k=t, n=g)  b[1]: (k=t+4, n=g)
//   d[0..1]: (g, 2t..2t+1)  d[2..3]: (g+8, 2t..)      with g = lane / 4, t = lane % 4.
__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4],
                                         const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

}  // namespace mma
}  // namespace llmyb
