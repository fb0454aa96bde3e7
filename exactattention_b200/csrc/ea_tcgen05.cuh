// Thin wrappers over the sm_100a tensor-core (tcgen05 / TMEM) and mbarrier PTX used by the
// tensor-core kernels. Operand tiles live in shared memory in the canonical K-major layout
// without swizzle: 8-row x 16-byte core matrices, each 128 contiguous bytes,
//   byte (row m, k) of an R-row tile at ((k / 16) * (R / 8) + m / 8) * 128 + (m % 8) * 16 + k % 16,
// so consecutive 8-row groups are 128 bytes apart (SBO) and consecutive 16-byte K chunks are
// R * 16 bytes apart (LBO). Every wait is bounded: it gives up after a fixed number of polls or
// two seconds of %globaltimer and reports failure, so a fault can never hang the device.
#pragma once
#include <stdint.h>

namespace ea {
namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// byte offset of (row m, byte k) in a K-major tile of R rows (R multiple of 8)
__host__ __device__ __forceinline__ uint32_t kmajor_off(uint32_t m, uint32_t k, uint32_t R) {
  return ((k >> 4) * (R >> 3) + (m >> 3)) * 128u + (m & 7u) * 16u + (k & 15u);
}

// shared-memory matrix descriptor, K-major, no swizzle (version 1 for sm_100)
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version
  return d;                // base offset 0, legacy LBO mode, layout type 0 (no swizzle)
}

// byte offset of (row n, byte k) in a K-major tile of `rows` rows (a multiple of 8) with the
// 128-byte swizzle: 1024-byte atoms of 8 rows x 128 bytes, the atoms of one 128-byte K column
// contiguous (8-row groups 1024 bytes apart), K columns (rows / 8) 1024 bytes apart, and 16-byte
// chunk c of row n stored at chunk c ^ (n % 8) of its atom row. The tile starts on a 1024-byte
// boundary.
__host__ __device__ __forceinline__ uint32_t sw128_off(uint32_t n, uint32_t k, uint32_t rows) {
  return ((k >> 7) * (rows >> 3) + (n >> 3)) * 1024u + (n & 7u) * 128u + ((((k >> 4) & 7u) ^ (n & 7u)) << 4) +
         (k & 15u);
}

// shared-memory matrix descriptor of such a tile (version 1, layout SWIZZLE_128B): `saddr` the
// start of the 32-byte K step inside its atom column (the hardware applies the swizzle to the
// address bits), 8-row groups `sbo_bytes` apart; the leading-byte offset is unused by swizzled
// K-major layouts
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// instruction descriptor of kind::i8 with s32 accumulation, both operands K-major
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N, bool a_signed, bool b_signed) {
  return (2u << 4)                           // D format: s32
         | ((a_signed ? 1u : 0u) << 7)       // A: 0 u8, 1 s8
         | ((b_signed ? 1u : 0u) << 10)      // B: 0 u8, 1 s8
         | ((uint32_t)(N >> 3) << 17)        // N / 8
         | ((uint32_t)(M >> 4) << 24);       // M / 16
}

// D[tmem] (+)= A[M x 32 bytes] * B[N x 32 bytes]^T, issued by one thread
__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       bool accumulate) {
  uint32_t acc = accumulate ? 1u : 0u;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n"
      :
      : "r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}

// D[tmem] (+)= A[tmem: M lanes x 32 bytes] * B[N x 32 bytes]^T, issued by one thread. A in tensor
// memory: row m of A in lane m, its 32 K bytes in 8 consecutive 32-bit columns from `tmem_a`
// (byte k % 4 of column k / 4, little-endian).
__device__ __forceinline__ void mma_i8_tmem_a(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                              bool accumulate) {
  uint32_t acc = accumulate ? 1u : 0u;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}\n"
      :
      : "r"(tmem_d), "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}

// arrive on an mbarrier once every tcgen05.mma issued so far by this thread has completed
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// generic-proxy shared-memory writes become visible to the tensor core (async proxy)
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// TMEM allocation by one full warp; the base address is written to shared memory
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_free(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// 8 consecutive 32-bit columns of this thread's TMEM lane (warp w reads lanes 32 (w % 4) ..)
__device__ __forceinline__ void tmem_ld8(uint32_t addr, uint32_t* v) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
      : "r"(addr)
      : "memory");
}
__device__ __forceinline__ void tmem_ld4(uint32_t addr, uint32_t* v) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
               : "r"(addr)
               : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 8 consecutive 32-bit columns of this thread's TMEM lane from registers (same lane rule as the
// loads); tmem_wait_st makes this thread's stores complete
__device__ __forceinline__ void tmem_st8(uint32_t addr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(addr), "r"(v[0]),
      "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld2(uint32_t addr, uint32_t* v) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0, %1}, [%2];" : "=r"(v[0]), "=r"(v[1]) : "r"(addr) : "memory");
}

// ---------------------------------------------------------------------------
// bulk copies global -> shared (the untiled TMA path), completing on an mbarrier
// ---------------------------------------------------------------------------
// The calling thread arrives on `bar` and adds `bytes` to the transaction count of its current
// phase; the phase completes once that many bytes of bulk copies have landed.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
// `bytes` (a multiple of 16) from global `src` to shared `dst`, both 16-byte aligned
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// 2D tiled tensor load (tensor map `tmap`, a kernel parameter; the box at element coordinates
// {x, y}) into shared memory, completing on an mbarrier. x times the element size must be a
// multiple of 16 bytes; rows outside the tensor read as zero.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------------------
// mbarrier with bounded waits
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Waits for the phase with the given parity to complete. Returns false after 2 s (or 2^26
// polls) without completion; callers then record an error, skip the dependent work and drain
// what they still have in flight before the CTA exits.
// debug != 0 (a test hook): the wait still waits for the phase (20 ms at most) but then reports
// expiry, so that the callers' abort and drain path runs with nothing left in flight.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int debug = 0) {
  const uint32_t a = smem_u32(bar);
  const uint64_t t0 = globaltimer();
  const uint64_t limit = debug ? 20000000ull : 2000000000ull;
  for (uint32_t i = 0; i < (1u << 26); ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(a), "r"(parity), "r"(10000u)  // suspend up to 10 us per try (woken by the phase)
        : "memory");
    if (done) return debug == 0;
    if ((i & 255u) == 255u && globaltimer() - t0 > limit) return false;
  }
  return false;
}

}  // namespace tc
}  // namespace ea
