// Thin inline-PTX wrappers for the Blackwell (sm_100a) tensor-core pipeline: mbarriers, TMA tile loads, tcgen05
// MMA / commit / TMEM allocation and loads.  Descriptor bit layouts follow the PTX ISA (tcgen05 "matrix descriptor"
// and "instruction descriptor" tables); the vendored CuTe sources (cute/arch/mma_sm100_desc.hpp) carry the same
// tables.
#pragma once
#include <cuda.h>

#include "common.cuh"

namespace duo {
namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Device-side fail-fast of a kernel launched without a cluster: true for every thread of the CTA when an earlier
// kernel has recorded a fault.  Call it first thing (every thread); a CTA that skips calls pdl_wait() before it
// returns, so the kernels after it still wait for the ones before it.  Kernels launched as clusters do not use it:
// their CTAs could read different values and the ones that stay would wait at a cluster barrier for the others.
__device__ __forceinline__ bool fault_pending(const unsigned* fault) {
  return __syncthreads_or(threadIdx.x == 0 && *reinterpret_cast<const volatile unsigned*>(fault) != 0u) != 0;
}

// Wait for the phase of `parity` to complete, giving up after `limit_ns` of wall time (the caller records a fault
// and unwinds instead of hanging the GPU).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns = 2000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; i++) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0 && globaltimer_ns() - t0 > limit_ns) return false;
  }
}

// 2D tiled TMA load into shared memory, completion counted on `bar` (no multicast).
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
// 3D tiled TMA load (no multicast): box at (x, y, z) of a [dim2][dim1][dim0] tensor; rows past a dimension's extent
// read as zero.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}
// 4D tiled TMA load (no multicast): box at (x, y, z, w); coordinates past an extent read as zero.
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int x, int y, int z, int w,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
      : "memory");
}
// 2D tiled TMA store of a shared-memory tile (rows and columns past the tensor's extent are not written); the
// writing threads make their generic-proxy stores visible with fence_proxy_async() before the barrier that precedes
// it.  bulk_commit() closes the group; bulk_wait_all() returns once its writes are done.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(smem_u32(src))
               : "memory");
}
// Prefetch a 2D tile of a tensor map into L2 (no shared-memory destination, no completion to wait for).
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* map, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y)
               : "memory");
}
// 1D bulk copy of `bytes` (a multiple of 16; both addresses 16-byte aligned) from global to this CTA's shared
// memory, completing as transactions on `bar` (no multicast).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// returns once the source shared memory of every committed bulk store has been read
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---- TMEM
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor, K-major operand in the 128-byte swizzle layout written by a SWIZZLE_128B TMA
// load: rows of 128 bytes, 8-row (1024-byte) swizzle atoms stacked along M/N.  start >> 4 in bits 0-13, leading
// byte offset (unused for swizzled K-major, 16 bytes) in 16-29, stride byte offset (1024 bytes between 8-row groups)
// in 32-45, descriptor version 1 in 46-47, layout type 2 (SWIZZLE_128B) in 61-63.
__device__ __forceinline__ uint64_t desc_kmajor_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)(16u >> 4) << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

// Shared-memory matrix descriptor of a 128-byte-swizzled operand, either major-ness (PTX ISA tcgen05 matrix
// descriptor; the canonical layouts are those of a SWIZZLE_128B TMA load or of the same pattern written by threads:
// rows of 128 bytes whose 16-byte chunks are XOR-permuted by (row % 8), 1024-byte aligned atoms of 8 rows).
//   K-major  (K contiguous): rows run along M / N; sbo = bytes between 8-row groups (1024 for stacked rows); lbo unused.
//   MN-major (M / N contiguous): each 128-byte row holds 64 consecutive M / N elements of one k; rows run along K;
//            sbo = bytes between 8-row (8-k) groups, lbo = bytes between the 64-element M / N blocks.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

// The descriptor of the same operand layout starting `bytes` (a multiple of 16) further on: the start address is
// the low 14 bits (address >> 4) and shared-memory addresses stay below 2^18, so the add never carries out of the
// field.  One thread issues every MMA of a CTA; building each descriptor from scratch costs it more instructions than
// a small MMA takes to run, so issue loops compute the base once and advance it with this add.
__device__ __forceinline__ uint64_t desc_add(uint64_t d, uint32_t bytes) { return d + (uint64_t)(bytes >> 4); }

// Instruction descriptor for kind::f16 with A and B both f16 (bf16 = false) or both bf16 and an f32 accumulator;
// a_mn / b_mn select the MN-major form of each operand (bits 15 / 16).
__host__ __device__ constexpr uint32_t idesc_16_mn(int m, int n, bool bf16, bool a_mn, bool b_mn) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((a_mn ? 1u : 0u) << 15) |
         ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
__host__ __device__ constexpr uint32_t idesc_f16_f32(int m, int n, bool a_mn, bool b_mn) {
  return idesc_16_mn(m, n, false, a_mn, b_mn);
}

// Instruction descriptor for kind::f16 with A and B both bf16 (f16 = false) or both f16 (both K-major) and an f32
// accumulator.
__host__ __device__ constexpr uint32_t idesc_16_f32(int m, int n, bool f16) {
  return (1u << 4)                      // D format: f32
         | ((f16 ? 0u : 1u) << 7)       // A format: f16 = 0, bf16 = 1
         | ((f16 ? 0u : 1u) << 10)      // B format
         | ((uint32_t)(n >> 3) << 17)   // N / 8
         | ((uint32_t)(m >> 4) << 24);  // M / 16
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
          tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// The same MMA with A read from TMEM (tmem_a: M lanes, K 16-bit values packed two per 32-bit column, K-major) and B
// from shared memory through its descriptor.
__device__ __forceinline__ void mma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(
          tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` once every tcgen05 op issued so far by this thread has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 columns of 32-bit accumulators: register j of lane l <- TMEM (lane_base + l, col + j)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int j = 0; j < 32; j++) v[j] = __uint_as_float(r[j]);
}

// 32 lanes x 32 columns of 32-bit values from registers into TMEM: lane_base + l, columns col .. col + 31; returns
// once the stores are done.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 32 lanes x 16 columns of raw 32-bit words into TMEM (lane_base + l, columns col .. col + 15), without the wait.
__device__ __forceinline__ void tmem_st16_issue(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Named barrier `id` (1..15) over `nthreads` threads (a multiple of 32).
__device__ __forceinline__ void bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// tcgen05.ld of 32 lanes x 32 columns without the wait: the registers are valid only after tmem_ld_wait(r).
__device__ __forceinline__ void tmem_ld32_issue(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// Wait for this thread's outstanding tcgen05.ld, then pin `r` behind the wait (the empty asm statements "modify" each
// register after the wait, so no use of it can be scheduled earlier).
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int j = 0; j < 32; j++) asm volatile("" : "+r"(r[j]));
}

// Two 32-column loads (columns of TMEM addresses ta and tb) in flight together, one wait: a and b receive 32 floats.
__device__ __forceinline__ void tmem_ld2x32(uint32_t ta, uint32_t tb, float* a, float* b) {
  uint32_t ra[32], rb[32];
  tmem_ld32_issue(ta, ra);
  tmem_ld32_issue(tb, rb);
  tmem_ld_wait(ra);
  tmem_ld_wait(rb);
#pragma unroll
  for (int j = 0; j < 32; j++) {
    a[j] = __uint_as_float(ra[j]);
    b[j] = __uint_as_float(rb[j]);
  }
}

}  // namespace tc

// Host: build a 2D 16-bit (DUO_BF16 / DUO_F16) tensor map over a row-major [rows, cols] matrix (leading dim ld
// elements) with a (box_cols x box_rows) box and 128-byte swizzle.  Out-of-range elements of a box read as zero.
int make_tmap_16(CUtensorMap* map, const void* base, int dtype, long rows, long cols, long ld, int box_rows,
                 int box_cols);
// Host: a 3D 16-bit tensor map over [d2][d1][d0] elements (d0 contiguous; byte strides s1 between d1 rows and s2
// between d2 planes, multiples of 16) with a (box0 x box1 x 1) box and 128-byte swizzle; boxes past an extent read as
// zero (used for [rows][tokens][columns] activations, so a chunk that runs past a row's last token reads zeros).
int make_tmap_3d_16(CUtensorMap* map, const void* base, int dtype, long d0, long d1, long d2, long s1, long s2,
                    int box0, int box1);
// Host: an N-d (2..5) 16-bit tensor map with 128-byte swizzle: dims[0] contiguous, byte strides[i] of dims[i + 1]
// (multiples of 16), box[i] elements per dim (box[0] * 2 bytes = 128 at most); boxes past an extent read as zero.
int make_tmap_nd_16(CUtensorMap* map, const void* base, int dtype, int rank, const long* dims, const long* strides,
                    const int* box);
// Host: the same over a 16-bit or f32 (DUO_F32) matrix without swizzle (a dense row-major box), for TMA stores.
int make_tmap_plain(CUtensorMap* map, const void* base, int dtype, long rows, long cols, long ld, int box_rows,
                    int box_cols);

// Device fault word shared by the bounded-wait kernels (fault.cu): a wait that gave up ORs a code into it.
// tc_fault_ptr() is its address on the current device (kernels take it as a parameter).  fault_mirror_init() creates
// the device's host-mapped copy, fault_mirror_dev() is that copy's device address (the engine's last kernel of a
// forward writes it), and fault_gate(where) returns DUO_ECUDA once a fault is visible on the host.
unsigned* tc_fault_ptr();
int fault_mirror_init();
unsigned* fault_mirror_dev();
int fault_gate(const char* where);

}  // namespace duo
