// Split-operand ("x3") tensor-core chunk path: the chunk-intra and
// chunk-inter kernels with f32-grade intermediates, for bf16 or f32 inputs,
// K = 128 key channels, chunk 64, V in {64, 128, 256}.
//
// Every tensor-core operand x that is not exactly a bf16 value is carried as
// a pair of bf16 images, hi = bf16(x) and lo = bf16(x - hi) (x = hi + lo to
// about 2^-17 relative), and every product is issued as three kind::f16 MMAs
// into the same f32 TMEM accumulator: A_hi B_hi + A_lo B_hi + A_hi B_lo (the
// dropped A_lo B_lo term is about 2^-18 of the product).  The path keeps the
// tile-local decay scheme of src/forward.rs:86-274 and holds the reference's
// f32 tolerance (rel 1e-3 / abs 1e-4 against a float64 restatement) for f32
// inputs; with bf16 inputs it computes the same f32-grade intermediates.
//
// Per (b, hv, chunk) record written by the intra kernel (byte offsets):
//   WQ_HI, WQ_LO [128][128] K-major : rows 0..63 W = (I+Akk)^-1 (b k gamma),
//                                     rows 64..127 Qg = scale q gamma
//   AQK_HI, AQK_LO [64][64] K-major : scale * causal(q k^T decay)
//   KD_HI, KD_LO [64][128] MN-major : k exp(G_last - G)
//   U    f32 [V/128 or 1][64][min(V,128)] : (I+Akk)^-1 (w v), slice by slice
//                                     of 128 value columns; within a row,
//                                     16-byte word k is stored at k ^ (row & 7)
//   GL   f32 [128]                  : gamma_last = exp(G_last)
// AQK_HI directly follows WQ_LO and AQK_LO directly follows AQK_HI: the
// inter kernel's [*; Aqk] operand of M = 128 takes its first 64 rows from
// the 8 KB in front of each Aqk image (their products land in accumulator
// rows that are dead by then), so no zero half tile is needed.
#pragma once

#include "chunk_tc.cuh"
#include "umma.cuh"

namespace gdn2 {

struct X3Record {
  size_t wq_hi, wq_lo, aqk_hi, aqk_lo, kd_hi, kd_lo, u, gl, bytes;
};

__host__ __device__ inline X3Record x3_record_layout(int V) {
  X3Record r;
  r.wq_hi = 0;
  r.wq_lo = r.wq_hi + 128 * 128 * 2;
  r.aqk_hi = r.wq_lo + 128 * 128 * 2;
  r.aqk_lo = r.aqk_hi + 64 * 64 * 2;
  r.kd_hi = r.aqk_lo + 64 * 64 * 2;
  r.kd_lo = r.kd_hi + 64 * 128 * 2;
  r.u = r.kd_lo + 64 * 128 * 2;
  r.gl = r.u + (size_t)64 * V * 4;
  r.bytes = (r.gl + TC_K * 4 + 1023) / 1024 * 1024;
  return r;
}

// Per-CTA scratch of the intra kernel, in the workspace after the records: the shared-memory images of the
// second score pass (row tiles 1 and 2), then rhs_k and rhs_v (value columns 0..127, and 128..255 for
// V = 256), written in the chunk's single pass over its rows and brought back by bulk copies.  At most
// X3_SLOTS CTAs (two per SM of a B200) run, so the slots of all of them (40-50 MB) stay resident in L2 while
// they are reused chunk after chunk.
constexpr size_t X3_SLOT_PASSB = 73728;
__host__ __device__ inline size_t x3_slot_bytes(int V) { return X3_SLOT_PASSB + 65536 + (V > 128 ? 32768 : 0); }
constexpr int X3_SLOTS = 2 * 148;
inline size_t x3_scratch_bytes(long long items, int V) {
  return (size_t)(items < X3_SLOTS ? items : X3_SLOTS) * x3_slot_bytes(V);
}

// Chunk-parallel state scan.  Over a segment of chunks the recurrence S' = (diag(gamma_last) - Kd^T W) S +
// Kd^T U is affine in the segment's start state: S_end = M S_start + N, where N is the end state from a zero
// start and M the product of the chunks' transitions (the same recurrence run on K columns with U = 0 from
// the identity).  With few chains (long sequences, few heads per GPU) a chain's chunks are cut into nseg
// segments: phase A computes (N, M) of every segment but the last in parallel, a short sequential pass
// chains the start states (S_{s+1} = M_s S_s + N_s, f32), and phase C runs all segments in parallel from
// their start states, writing the outputs.  Segments for V in {128, 256} when at least three fit (every
// phase-A CTA of a segment, V / 128 state slices + 1 transition slice, on its own SM) with >= 8 chunks each;
// otherwise 1 (no scan).
inline int x3_scan_segments(long long B, long long HV, long long NC, int V, int sms) {
  if (V != 128 && V != 256) return 1;
  const long long slices = V / 128 + 1;
  long long n = sms / (B * HV * slices);
  if (n > NC / 8) n = NC / 8;
  if (n < 3) return 1;
  const long long len = (NC + n - 1) / n;  // chunks per segment; every segment non-empty
  return (int)((NC + len - 1) / len);
}
inline size_t x3_scan_bytes(long long B, long long HV, int V, int nseg) {
  return nseg > 1 ? (size_t)(B * HV) * ((size_t)nseg * TC_K * V + (size_t)(nseg - 1) * TC_K * TC_K) * 4 : 0;
}

bool x3_supported(int K, int V, int C);
int launch_intra_x3(const TcParams& p, int dtype, cudaStream_t st);
int launch_inter_x3(const TcParams& p, int dtype, cudaStream_t st);

// ---- device helpers shared by the two kernels ----

// bf16 pair (lower channel in the low half) -> f32 pair, exact
__device__ __forceinline__ f32x2 bf2f2(uint32_t u) {
  return f2pk(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
}
// f32 pair -> bf16 pair, round to nearest even
__device__ __forceinline__ uint32_t f2bf2(f32x2 r) {
  float lo, hi;
  f2un(r, lo, hi);
  return umma::pack_bf16x2(lo, hi);
}
__device__ __forceinline__ f32x2 f2sub(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
// (x0, x1) -> (hi, lo) bf16 pairs with hi = bf16(x), lo = bf16(x - hi); x - hi is exact in f32.  Plain
// 32-bit operations: two conversions, two masks, two subtractions.
__device__ __forceinline__ void split2f(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(hi) : "f"(x1), "f"(x0));
  const float l0 = x0 - __uint_as_float(hi << 16), l1 = x1 - __uint_as_float(hi & 0xffff0000u);
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(lo) : "f"(l1), "f"(l0));
}
// The same for a packed pair: the two subtractions as one sub.f32x2 (same results: x - hi is exact).
__device__ __forceinline__ void split2(f32x2 x, uint32_t& hi, uint32_t& lo) {
  float x0, x1;
  f2un(x, x0, x1);
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(hi) : "f"(x1), "f"(x0));
  float l0, l1;
  f2un(f2sub(x, f2pk(__uint_as_float(hi << 16), __uint_as_float(hi & 0xffff0000u))), l0, l1);
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(lo) : "f"(l1), "f"(l0));
}
// 8 consecutive f32 -> hi and lo images of 8 bf16 (one 16-byte chunk each)
__device__ __forceinline__ void split8(const float* v, uint4& hi, uint4& lo) {
  split2(f2pk(v[0], v[1]), hi.x, lo.x);
  split2(f2pk(v[2], v[3]), hi.y, lo.y);
  split2(f2pk(v[4], v[5]), hi.z, lo.z);
  split2(f2pk(v[6], v[7]), hi.w, lo.w);
}

// Four consecutive input elements of one row as two f32 pairs, read with a
// non-volatile non-coherent load (the compiler may hoist it above stores
// into the record, which it would otherwise have to assume alias it).
template <typename TIN>
struct Raw4;
template <>
struct Raw4<__nv_bfloat16> {
  uint2 r;
  __device__ __forceinline__ void zero() { r = make_uint2(0u, 0u); }
  __device__ __forceinline__ void load(const void* ptr) {
    asm("ld.global.nc.v2.u32 {%0, %1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(ptr));
  }
  __device__ __forceinline__ void load(const void* ptr, uint64_t pol) {  // with an L2 eviction policy
    asm("ld.global.nc.L1::no_allocate.L2::cache_hint.v2.u32 {%0, %1}, [%2], %3;"
        : "=r"(r.x), "=r"(r.y)
        : "l"(ptr), "l"(pol));
  }
  __device__ __forceinline__ f32x2 pair(int m) const { return bf2f2(m ? r.y : r.x); }
};
template <>
struct Raw4<float> {
  float4 r;
  __device__ __forceinline__ void zero() { r = make_float4(0.f, 0.f, 0.f, 0.f); }
  __device__ __forceinline__ void load(const void* ptr) {
    asm("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w) : "l"(ptr));
  }
  __device__ __forceinline__ void load(const void* ptr, uint64_t pol) {  // with an L2 eviction policy
    asm("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
        : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
        : "l"(ptr), "l"(pol));
  }
  __device__ __forceinline__ f32x2 pair(int m) const { return m ? f2pk(r.z, r.w) : f2pk(r.x, r.y); }
};

template <typename TIN>
__device__ __forceinline__ const void* vptr(const DView& v, int bb, int h, int t, int c) {
  return static_cast<const TIN*>(v.p) + bb * v.s0 + h * v.s1 + (int64_t)t * v.s2 + c;
}

}  // namespace gdn2
