// tcgen05 (5th-gen tensor core) helpers for sm_100a: TMEM allocation,
// shared-memory matrix descriptors in the 128-byte-swizzle canonical layouts,
// instruction descriptors, MMA issue / commit and TMEM <-> register moves.
//
// Canonical shared-memory layouts (16-bit elements, 128-byte swizzle):
//  * K-major operand [R rows][KD] (K contiguous): K is cut into blocks of 64
//    elements; block kb lives at kb * R * 128 bytes; inside it row r sits at
//    (r / 8) * 1024 + (r % 8) * 128 and its 16-byte chunk c at chunk
//    position c ^ (r % 8).  Descriptor: LBO = 16 B (unused), SBO = 1024 B.
//    MMA k-step j (16 elements) starts at kb * R * 128 + (j % 4) * 32.
//  * MN-major operand [KD rows][N] (N contiguous): N is cut into groups of
//    64 elements (128 bytes); group g lives at g * KD * 128; inside it K row
//    kk sits at (kk / 8) * 1024 + (kk % 8) * 128, chunk c at c ^ (kk % 8).
//    Descriptor: LBO = KD * 128 (next N group), SBO = 1024 (next 8 K rows).
//    MMA k-step j starts at j * 2048.
// Tiles must start on 1024-byte boundaries.
#pragma once

#include <stdint.h>

#include "ptx.cuh"

namespace gdn2 {
namespace umma {

// byte offset of element (r, k) in a K-major [R][KD] bf16 tile
__device__ __forceinline__ uint32_t kmaj_off(int r, int k, int R) {
  const int kb = k >> 6, kk = k & 63;
  const int c = kk >> 3, e = kk & 7;
  return (uint32_t)(kb * R * 128 + (r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4) + e * 2);
}

// byte offset of element (kk, n) in an MN-major [KD][N] bf16 tile
__device__ __forceinline__ uint32_t mnmaj_off(int kk, int n, int KD) {
  const int g = n >> 6, nn = n & 63;
  const int c = nn >> 3, e = nn & 7;
  return (uint32_t)(g * KD * 128 + (kk >> 3) * 1024 + (kk & 7) * 128 + ((c ^ (kk & 7)) << 4) + e * 2);
}

// byte offset of the 16-byte chunk holding elements (r, 8*c8 .. 8*c8+7) of a K-major tile
__device__ __forceinline__ uint32_t kmaj_chunk(int r, int c8, int R) {
  const int kb = c8 >> 3, c = c8 & 7;
  return (uint32_t)(kb * R * 128 + (r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

// byte offset of the 16-byte chunk holding elements (kk, 8*c8 .. 8*c8+7) of an MN-major tile
__device__ __forceinline__ uint32_t mnmaj_chunk(int kk, int c8, int KD) {
  const int g = c8 >> 3, c = c8 & 7;
  return (uint32_t)(g * KD * 128 + (kk >> 3) * 1024 + (kk & 7) * 128 + ((c ^ (kk & 7)) << 4));
}

__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;  // SWIZZLE_128B
  return d;
}

// K-major A/B tile [R][KD], MMA k-step j (16 elements)
__device__ __forceinline__ uint64_t desc_kmaj(uint32_t tile_saddr, int R, int j) {
  return desc_sw128(tile_saddr + (uint32_t)((j >> 2) * R * 128 + (j & 3) * 32), 16, 1024);
}

// MN-major A/B tile [KD][N], MMA k-step j (16 K rows)
__device__ __forceinline__ uint64_t desc_mnmaj(uint32_t tile_saddr, int KD, int j) {
  return desc_sw128(tile_saddr + (uint32_t)(j * 2048), (uint32_t)(KD * 128), 1024);
}

// The descriptor of the same layout `off_bytes` further on: only the start-address field (address >> 4, the low
// 14 bits) changes, and shared-memory addresses stay below 2^18 bytes, so the sum never carries out of that field.
// One add per MMA instead of rebuilding every field.
__device__ __forceinline__ uint64_t desc_add(uint64_t d, uint32_t off_bytes) {
  return (d & 0xFFFFFFFF00000000ull) | (uint64_t)((uint32_t)d + (off_bytes >> 4));
}
__device__ __forceinline__ uint64_t desc_kmaj_base(uint32_t tile_saddr) { return desc_sw128(tile_saddr, 16, 1024); }
__device__ __forceinline__ uint64_t desc_mnmaj_base(uint32_t tile_saddr, int KD) {
  return desc_sw128(tile_saddr, (uint32_t)(KD * 128), 1024);
}
// k-step j of a K-major [R][KD] tile / an MN-major [KD][N] tile, from its base descriptor
__device__ __forceinline__ uint64_t desc_kmaj_at(uint64_t base, int R, int j) {
  return desc_add(base, (uint32_t)((j >> 2) * R * 128 + (j & 3) * 32));
}
__device__ __forceinline__ uint64_t desc_mnmaj_at(uint64_t base, int j) { return desc_add(base, (uint32_t)(j * 2048)); }

// kind::f16 instruction descriptor: bf16 x bf16 -> f32
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool a_mn_major, bool b_mn_major) {
  return (1u << 4)                       // D format f32
         | (1u << 7)                     // A bf16
         | (1u << 10)                    // B bf16
         | ((a_mn_major ? 1u : 0u) << 15)  //
         | ((b_mn_major ? 1u : 0u) << 16)  //
         | ((uint32_t)(N >> 3) << 17)    //
         | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate ? 1u : 0u)
      : "memory");
}

// arrive on `bar` once all previously issued tcgen05.mma of this thread completed
__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// one full warp: allocate `ncols` TMEM columns (power of two >= 32), base written to *dst
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// warp-collective: 16 consecutive f32 columns of this thread's TMEM lane
__device__ __forceinline__ void ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  #pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15]))
      : "memory");
}
__device__ __forceinline__ void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// TMEM address of (lane, column)
__device__ __forceinline__ uint32_t taddr(uint32_t base, int lane, int col) {
  return base + ((uint32_t)lane << 16) + (uint32_t)col;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

}  // namespace umma
}  // namespace gdn2
