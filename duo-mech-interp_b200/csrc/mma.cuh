// Warp-level 16-bit tensor-core helpers (mma.sync m16n8k16 bf16 / f16, ldmatrix) for the small dependent products of the chunked
// DeltaNet scan.  Fragment layouts follow the PTX ISA "mma.m16n8k16" tables: with g = lane / 4 and q = lane % 4,
//   A (16 x 16, row-major): a0 = (g, 2q..2q+1), a1 = (g + 8, 2q..), a2 = (g, 2q + 8..), a3 = (g + 8, 2q + 8..)
//   B (16 x 8):             b0 = (k = 2q..2q+1, n = g), b1 = (k = 2q + 8.., n = g)
//   C (16 x 8, f32):        c0, c1 = (g, 2q..2q+1), c2, c3 = (g + 8, 2q..2q+1)
#pragma once
#include "common.cuh"

namespace duo {
namespace wm {

__device__ __forceinline__ uint32_t saddr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mma(float* c, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

__device__ __forceinline__ void ldsm4(uint32_t* r, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(saddr(p)));
}
__device__ __forceinline__ void ldsm4t(uint32_t* r, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(saddr(p)));
}

// A fragment of the 16 x 16 tile at (m0, k0) of a row-major [M][K] bf16 matrix with pitch P (elements)
template <typename T16>
__device__ __forceinline__ void lda(uint32_t* a, const T16* A, int P, int m0, int k0) {
  const int l = threadIdx.x & 31;
  ldsm4(a, A + (m0 + (l & 15)) * P + k0 + (l >> 4) * 8);
}
// A fragment of the 16 x 16 tile at (m0, k0) of A = X^T where X is a row-major [K][M] matrix (pitch P)
template <typename T16>
__device__ __forceinline__ void lda_t(uint32_t* a, const T16* X, int P, int m0, int k0) {
  const int l = threadIdx.x & 31;
  ldsm4t(a, X + (k0 + (l & 7) + ((l >> 4) << 3)) * P + m0 + ((l >> 3) & 1) * 8);
}
// B fragments of two n-tiles (n0 .. n0 + 15) x k0 .. k0 + 15, B stored as [N][K] (k contiguous): b[0..1] = tile n0,
// b[2..3] = tile n0 + 8
template <typename T16>
__device__ __forceinline__ void ldb_nk(uint32_t* b, const T16* B, int P, int n0, int k0) {
  const int l = threadIdx.x & 31;
  ldsm4(b, B + (n0 + (l & 7) + ((l >> 4) << 3)) * P + k0 + ((l >> 3) & 1) * 8);
}
// same, B stored as [K][N] (n contiguous)
template <typename T16>
__device__ __forceinline__ void ldb_kn(uint32_t* b, const T16* B, int P, int n0, int k0) {
  const int l = threadIdx.x & 31;
  ldsm4t(b, B + (k0 + (l & 7) + ((l >> 3) & 1) * 8) * P + n0 + (l >> 4) * 8);
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ uint32_t pack_f16(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ void mma_f16(float* c, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// the same for a 16-bit operand type chosen at compile time (__nv_bfloat16 or __half)
template <typename T16> struct Ops;
template <> struct Ops<__nv_bfloat16> {
  static __device__ __forceinline__ void mma(float* c, const uint32_t* a, const uint32_t* b) { wm::mma(c, a, b); }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) { return pack_bf16(lo, hi); }
};
template <> struct Ops<__half> {
  static __device__ __forceinline__ void mma(float* c, const uint32_t* a, const uint32_t* b) { mma_f16(c, a, b); }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) { return pack_f16(lo, hi); }
};

}  // namespace wm
}  // namespace duo
