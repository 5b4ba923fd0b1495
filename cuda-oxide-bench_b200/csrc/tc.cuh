// tc.cuh — tcgen05 (5th-generation tensor core) and TMEM helpers for sm_100a:
// shared-memory matrix descriptors for 128-byte-swizzled tiles, the bf16/f16
// instruction descriptor, MMA issue/commit, TMEM allocation and loads, and the
// tensor-map TMA loads that fill the tiles.  Never uses multicast.
#pragma once
#include <cuda.h>

#include <cstdint>

#include "ptx.cuh"

namespace gdn {
namespace tc {

// ---------------------------------------------------------------- smem tiles
// A 128B-swizzled tile stores rows of 128 bytes (64 bf16); 8 consecutive rows
// form a 1024-byte atom in which the 16-byte chunk index is XOR-ed with the
// row index mod 8.  Tile bases are 1024-byte aligned.  The same physical tile
// serves as a K-major operand (rows = M/N index, K along the row) or as an
// MN-major operand (rows = K index, M/N along the row).
__device__ __forceinline__ uint32_t sw128_offset(int row, int chunk) {
  return static_cast<uint32_t>((row >> 3) * 1024 + (row & 7) * 128 + ((chunk ^ (row & 7)) << 4));
}

// Matrix descriptor (tcgen05 shared-memory descriptor, version 1, SWIZZLE_128B).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr, uint32_t lbo_bytes,
                                               uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= 1ull << 46;  // descriptor version (Blackwell)
  d |= 2ull << 61;  // SWIZZLE_128B
  return d;
}

// K-major operand: `kblock_stride` separates the 64-wide K blocks; step s
// covers K elements [16 s, 16 s + 16).
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t tile, uint32_t kblock_stride, int s) {
  return sw128_desc(tile + (s >> 2) * kblock_stride + (s & 3) * 32, 16, 1024);
}

// MN-major operand: rows are the K index; `mnblock_stride` separates the
// 64-wide M/N blocks; step s covers K rows [16 s, 16 s + 16).
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t tile, uint32_t mnblock_stride, int s) {
  return sw128_desc(tile + s * 2048, mnblock_stride, 1024);
}

// Instruction descriptor: 16-bit inputs (bf16 if bf16 else f16), fp32 accumulate.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool a_mn, bool b_mn, bool bf16,
                                                 bool a_neg = false) {
  return (1u << 4)                                   // D format f32
         | ((a_neg ? 1u : 0u) << 13)                 // negate A
         | ((bf16 ? 1u : 0u) << 7)                   // A format
         | ((bf16 ? 1u : 0u) << 10)                  // B format
         | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16)
         | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// ---------------------------------------------------------------- MMA
__device__ __forceinline__ void mma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                    bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(static_cast<uint32_t>(accumulate))
      : "memory");
}

// Arrives on `bar` once every previously issued MMA of this thread completed.
__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Generic-proxy shared-memory writes -> visible to the async proxy (MMA, TMA).
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- TMEM
// Whole-warp allocation; the column base is written to *dst (shared).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t base, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(ncols)
               : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns: thread i of the warp receives
// lane (quarter*32 + i), columns [col, col+16).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&r)[16]) {
  uint32_t u[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15}, [%16];"
      : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]),
        "=r"(u[7]), "=r"(u[8]), "=r"(u[9]), "=r"(u[10]), "=r"(u[11]), "=r"(u[12]), "=r"(u[13]),
        "=r"(u[14]), "=r"(u[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) r[i] = __uint_as_float(u[i]);
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 lanes x 16 consecutive 32-bit columns from registers (thread i -> lane
// quarter*32 + i).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&u)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(u[0]), "r"(u[1]), "r"(u[2]), "r"(u[3]), "r"(u[4]), "r"(u[5]), "r"(u[6]), "r"(u[7]),
      "r"(u[8]), "r"(u[9]), "r"(u[10]), "r"(u[11]), "r"(u[12]), "r"(u[13]), "r"(u[14]), "r"(u[15])
      : "memory");
}
// 32 lanes x 8 consecutive 32-bit columns from registers.
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&u)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
      "r"(u[0]), "r"(u[1]), "r"(u[2]), "r"(u[3]), "r"(u[4]), "r"(u[5]), "r"(u[6]), "r"(u[7])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// MMA with the A operand read from TMEM (M rows = lanes, 16-bit elements
// packed two per 32-bit column, lower element in the low half).
__device__ __forceinline__ void mma_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t b,
                                           uint32_t idesc, bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(static_cast<uint32_t>(accumulate))
      : "memory");
}

// Named barrier over `count` threads (a thread group inside the CTA).
__device__ __forceinline__ void group_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// ---------------------------------------------------------------- TMA
// 4-D tiled load (no multicast) into a 128B-swizzled tile.  c0 * element
// size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int c0, int c1,
                                            int c2, int c3, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, "
      "{%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

// bf16 round-to-nearest-even on the integer pipe: returns the rounded bit
// pattern with the bf16 value in the upper 16 bits (lower 16 bits garbage).
// Finite inputs only (the kernels never feed NaN); overflow rounds to inf.
// Keeps the conversion off the transcendental/conversion (XU) pipe, which
// the prefill epilogues would otherwise saturate.
__device__ __forceinline__ uint32_t bf16_rne_bits(float x) {
  const uint32_t u = __float_as_uint(x);
  return u + 0x7FFFu + ((u >> 16) & 1u);
}
// The float value of x rounded to bf16.
__device__ __forceinline__ float bf16_round(float x) {
  return __uint_as_float(bf16_rne_bits(x) & 0xFFFF0000u);
}

// packs two floats into a bf16x2 / f16x2 word (low half = first)
template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if (BF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}
template <bool BF16>
__device__ __forceinline__ float unpack_lo(uint32_t w) {
  if (BF16) return __uint_as_float(w << 16);
  return __half2float(__ushort_as_half(static_cast<unsigned short>(w & 0xFFFF)));
}
template <bool BF16>
__device__ __forceinline__ float unpack_hi(uint32_t w) {
  if (BF16) return __uint_as_float(w & 0xFFFF0000u);
  return __half2float(__ushort_as_half(static_cast<unsigned short>(w >> 16)));
}

// Four 8x8 b16 matrices from shared memory, transposed (ldmatrix .trans):
// lane L gives the address of row L % 8 of matrix L / 8; afterwards lane t
// holds, for each matrix m, the pair (rows 2 (t % 4), 2 (t % 4) + 1) of
// column t / 4 packed in r[m].
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
// Four 8x8 b16 matrices to shared memory (stmatrix): lane L gives the address
// of row L % 8 of matrix L / 8; r[m] of lane t is stored to row t / 4,
// columns 2 (t % 4) and 2 (t % 4) + 1 of matrix m.
__device__ __forceinline__ void stsm_x4(uint32_t addr, const uint32_t (&r)[4]) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(addr),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3])
               : "memory");
}

__device__ __forceinline__ void sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                       uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

}  // namespace tc
}  // namespace gdn
