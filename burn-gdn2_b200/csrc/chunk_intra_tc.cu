// Kernel (1) on tensor cores: chunk-intra for bf16 inputs, K = 128, C = 64.
//
// Replaces gdn2_chunk_intra_kernel (src/kernel/chunk_cube.rs:27-295) with the
// numerics of the tensor path src/forward.rs:86-261 (tile-local decay).
// One CTA (8 warps, two per SM) per (chunk, value head, batch):
//
//  1. warps 2p, 2p+1 own the two 8-row halves of the 16-row tile p, lane l
//     owns key channels 4l..4l+3: g sums per half tile -> tile boundaries
//     Gb_p, G_last; the tile-local cumsum gl is rebuilt row by row.
//  2. Score operands in shared memory (bf16, 128-byte swizzle):
//       X_p  = [q e^{gl} ; b k e^{gl}] of tile p          (32 x 128)
//       Ks_p = k e^{Gb_p - G} for rows s < 16(p+1)        (reference point
//              Gb_p for all columns of row tile p, so no factor exceeds
//              16 tokens of decay, forward.rs:131-157)
//  3. Four M=64 N=32 K=128 MMAs: D_p = Ks_p X_p^T = [Aqk^T | Akk^T] columns of
//     row tile p, accumulated in TMEM.
//     Qg = scale q gamma, Kd = k e^{G_last - G}, rhs_k = b k gamma,
//     rhs_v = w v and gamma_last come out of the same pass
//     (forward.rs:189-190, :266-274).
//  5. Aqk (scaled, causal) and Akk (strict) back from TMEM; (I + Akk)^-1 by
//     blocked forward substitution over 16x16 tiles (forward.rs:192-261).
//  6. Two M=64 MMAs: W = (I+Akk)^-1 rhs_k, U = (I+Akk)^-1 rhs_v.
//  7. The record (chunk_tc.cuh) is written as operand-tile images; W and U
//     are staged in shared memory and leave in bulk copies.
#include "chunk_tc.cuh"
#include "umma.cuh"

namespace gdn2 {

namespace intra_smem {
constexpr uint32_t X = 0;               // 4 x 8 KB: K-major [32][128] per row tile
constexpr uint32_t KSV = 32768;         // Ks_p at KSV + 4096 * p(p+1)/2, [16(p+1)][128]
constexpr uint32_t R1_END = 73728;      // 72 KB
// reused after the score MMAs completed
constexpr int SS = 68;                  // row stride (floats) of AKK and TINV: 16-byte rows
constexpr uint32_t AKK = 0;             // f32 [64][SS]
constexpr uint32_t TINV = 17408;        // f32 [64][SS]
constexpr uint32_t AQK_IMG = 36864;     // bf16 K-major [64][64]
constexpr uint32_t TINV_IMG = 45056;    // bf16 K-major [64][64]
constexpr uint32_t SCRATCH = 53248;     // 6 x f32 [16][20] blocks of the inverse
// staging of the record's W and U images (step 7), once the solve's f32 tiles are dead
constexpr uint32_t WST = 0;             // W rows 0..63: K-major [64][128], two 8 KB column blocks
constexpr uint32_t UST = 16384;         // U, first value-column slice: [64][vt] rows (8 or 16 KB)
constexpr uint32_t UST2 = AQK_IMG;      // U, second slice (V = 256), once Aqk and T^-1 images are used
constexpr uint32_t RK = R1_END;         // bf16 MN-major [64][128]
constexpr uint32_t RV = RK + 16384;     // bf16 MN-major [64][128]: rhs_v of (up to) 128 value channels
constexpr uint32_t MISC = RV + 16384;   // half-tile g sums [8][128] f32, sGlast [128] f32, barriers, tmem base
constexpr uint32_t TOTAL = MISC + 4096 + 512 + 64;
}  // namespace intra_smem

// Loads of the kernel's read-only inputs.  Written as non-volatile asm
// without a memory clobber, so the compiler may move them above the stores
// into the record, which it would otherwise have to assume alias them.
__device__ __forceinline__ uint2 ld4_raw(const DView& v, int bb, int h, int t, int c, bool ok) {
  uint2 r = make_uint2(0u, 0u);
  if (ok) {
    const void* ptr = static_cast<const __nv_bfloat16*>(v.p) + bb * v.s0 + h * v.s1 + (int64_t)t * v.s2 + c;
    asm("ld.global.nc.v2.u32 {%0, %1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(ptr));
  }
  return r;
}

__device__ __forceinline__ float4 ld_f4_nc(const float* ptr) {
  float4 r;
  asm("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w) : "l"(ptr));
  return r;
}

__device__ __forceinline__ void l2_prefetch(const void* a) { asm volatile("prefetch.global.L2 [%0];" ::"l"(a)); }

// Line j of token t's inputs: q k b v w (two 128-byte lines each), g (four),
// then for V = 256 the second 256 bytes of v (j = 14, 15) and w (16, 17).
__device__ __forceinline__ void prefetch_line(const TcParams& p, int bb, int kh, int hv, int t, int j) {
  if (j < 10) {
    if (j >= 6 && (j & 1) && p.V <= 64) return;
    const DView& v = j < 2 ? p.q : j < 4 ? p.k : j < 6 ? p.b : j < 8 ? p.v : p.w;
    const int h = j < 6 ? kh : hv;
    l2_prefetch(reinterpret_cast<const char*>(static_cast<const __nv_bfloat16*>(v.p) + bb * v.s0 + h * v.s1 +
                                              (int64_t)t * v.s2) + (j & 1) * 128);
  } else if (j < 14) {
    l2_prefetch(reinterpret_cast<const char*>(static_cast<const float*>(p.g.p) + bb * p.g.s0 + kh * p.g.s1 +
                                              (int64_t)t * p.g.s2) + (j - 10) * 128);
  } else {
    const DView& v = j < 16 ? p.v : p.w;
    l2_prefetch(reinterpret_cast<const char*>(static_cast<const __nv_bfloat16*>(v.p) + bb * v.s0 + hv * v.s1 +
                                              (int64_t)t * v.s2) + 256 + (j & 1) * 128);
  }
}

__device__ __forceinline__ void unpack4(uint2 raw, float (&x)[4]) {
  const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&raw.x);
  const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&raw.y);
  x[0] = __low2float(a); x[1] = __high2float(a); x[2] = __low2float(b); x[3] = __high2float(b);
}

// The operand build of step 2 works on the lane's channels in pairs (c, c + 1), as they arrive in bf16x2
// words, with the packed f32x2 multiply (ptx.cuh).
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

__device__ __forceinline__ uint2 pack4(float a, float b, float c, float d) {
  return make_uint2(umma::pack_bf16x2(a, b), umma::pack_bf16x2(c, d));
}

// VMAX = 128: V in {64, 128}.  VMAX = 256: V = 256 in the same footprint (two
// CTAs per SM, 256 TMEM columns): U's first 128 columns come out of the
// W / U MMA pair as for V = 128; then rhs_v of channels 128..255 is rebuilt
// in the same shared tile from a second read of v and w (prefetched to L2
// with the CTA's other inputs) and a second MMA writes U's upper half into
// W's TMEM columns once W has been read out.
template <int VMAX>
__global__ void __launch_bounds__(256, 2) k_intra_tc(const TcParams p) {
  using namespace intra_smem;
  constexpr uint32_t TCOLS = 256;                     // TMEM columns: W [0, 128), U [128, 256)
  constexpr int NL = VMAX > 128 ? 18 : 14;            // 128-byte input lines per token
  extern __shared__ __align__(1024) unsigned char smraw[];
  unsigned char* sm = smraw + ((1024u - (smem_u32(smraw) & 1023u)) & 1023u);
  float* sHalf = reinterpret_cast<float*>(sm + MISC);  // [8][128] g sums of each 8-row half tile
  float* sGlast = sHalf + 8 * 128;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sGlast + 128);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 2);

  const int c = blockIdx.x, hv = blockIdx.y, bb = blockIdx.z;
  const int kh = hv / p.rep;
  const int t0 = c * TC_C;
  const int cv = min(TC_C, p.T - t0);
  const int V = p.V;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tp = warp >> 1, hh = warp & 1;  // row tile, half of it (rows 16 tp + 8 hh + i)
  const int r0 = tp * 16 + hh * 8;
  const int ch = lane * 4;                  // first of 4 key channels
  unsigned char* rec = p.rec + (((size_t)bb * p.HV + hv) * p.NC + c) * p.rec_bytes;
  const TcRecord L = tc_record_layout(V);

  if (warp == 0) {
    umma::tmem_alloc(tslot, TCOLS);
    umma::tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
  }

  // every input line of this warp's 8 rows on its way to L2 before the first use, in the order of use: g first
  // (step 1 sums it before anything else can start; one line per lane), then q k b v w row by row, then for
  // V = 256 the upper v / w channels of step 8.  Issuing g last, row by row with the rest, left step 1 waiting
  // behind the whole CTA's input (3-4% of the kernel's time).
  for (int idx = lane; idx < 8 * NL; idx += 32) {
    int r, j;
    if (idx < 32) {
      r = idx >> 2; j = 10 + (idx & 3);
    } else if (idx < 112) {
      r = (idx - 32) / 10; j = (idx - 32) % 10;
    } else {
      r = (idx - 112) >> 2; j = 14 + ((idx - 112) & 3);
    }
    r += r0;
    if (r < cv) prefetch_line(p, bb, kh, hv, t0 + r, j);
  }

  // ---- 1. sums of g over each half tile (the per-row cumsum is rebuilt below) ----
  const float* gbase = static_cast<const float*>(p.g.p) + bb * p.g.s0 + kh * p.g.s1 + ch;
  // inputs of row r0 + i, fetched one row ahead of their use in step 2
  uint2 nq, nk, nb, nv = make_uint2(0u, 0u), nw = make_uint2(0u, 0u);
  float4 ng = make_float4(0.f, 0.f, 0.f, 0.f);
  auto fetch = [&](int i) {
    const int r = r0 + i;
    const bool ok = r < cv;
    if (ok) ng = ld_f4_nc(gbase + (int64_t)(t0 + r) * p.g.s2);
    nq = ld4_raw(p.q, bb, kh, t0 + r, ch, ok);
    nk = ld4_raw(p.k, bb, kh, t0 + r, ch, ok);
    nb = ld4_raw(p.b, bb, kh, t0 + r, ch, ok);
    if (ch < V) {
      nv = ld4_raw(p.v, bb, hv, t0 + r, ch, ok);
      nw = ld4_raw(p.w, bb, hv, t0 + r, ch, ok);
    }
  };
  fetch(0);
  float glr[4] = {0.f, 0.f, 0.f, 0.f};  // half-local cumsum at the last valid row, if it is ours
  {
    float run[4] = {0.f, 0.f, 0.f, 0.f};
    #pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = r0 + i;
      float4 gv = make_float4(0.f, 0.f, 0.f, 0.f);
      if (r < cv) gv = ld_f4_nc(gbase + (int64_t)(t0 + r) * p.g.s2);
      run[0] += gv.x; run[1] += gv.y; run[2] += gv.z; run[3] += gv.w;
      if (r == cv - 1) {
        glr[0] = run[0]; glr[1] = run[1]; glr[2] = run[2]; glr[3] = run[3];
      }
    }
    *reinterpret_cast<float4*>(sHalf + warp * 128 + ch) = make_float4(run[0], run[1], run[2], run[3]);
  }
  __syncthreads();
  float Gb[4][4];  // Gb[pp][j]: G at the end of tile pp-1 (0 for pp = 0)
  #pragma unroll
  for (int j = 0; j < 4; ++j) Gb[0][j] = 0.f;
  #pragma unroll
  for (int pp = 1; pp < 4; ++pp) {
    const float4 a = *reinterpret_cast<const float4*>(sHalf + (2 * pp - 2) * 128 + ch);
    const float4 b = *reinterpret_cast<const float4*>(sHalf + (2 * pp - 1) * 128 + ch);
    Gb[pp][0] = Gb[pp - 1][0] + a.x + b.x; Gb[pp][1] = Gb[pp - 1][1] + a.y + b.y;
    Gb[pp][2] = Gb[pp - 1][2] + a.z + b.z; Gb[pp][3] = Gb[pp - 1][3] + a.w + b.w;
  }
  float Gbp[4], off[4];  // Gb of this tile; tile-local cumsum before row r0
  {
    const float4 h0 = *reinterpret_cast<const float4*>(sHalf + (2 * tp) * 128 + ch);
    const float hv0[4] = {h0.x, h0.y, h0.z, h0.w};
    #pragma unroll
    for (int j = 0; j < 4; ++j) {
      Gbp[j] = tp == 0 ? Gb[0][j] : tp == 1 ? Gb[1][j] : tp == 2 ? Gb[2][j] : Gb[3][j];
      off[j] = hh ? hv0[j] : 0.f;
    }
  }
  if (r0 <= cv - 1 && cv - 1 < r0 + 8)
    *reinterpret_cast<float4*>(sGlast + ch) = make_float4(Gbp[0] + off[0] + glr[0], Gbp[1] + off[1] + glr[1],
                                                          Gbp[2] + off[2] + glr[2], Gbp[3] + off[3] + glr[3]);
  __syncthreads();  // sGlast

  // ---- 2. operands (compact loop: the code must stay in the instruction cache) ----
  const float4 glast4 = *reinterpret_cast<const float4*>(sGlast + ch);
  const float glast[4] = {glast4.x, glast4.y, glast4.z, glast4.w};
  // per-channel constants of this row tile (E = e^{gl}, the tile-local decay):
  // gamma = e^{Gb_p} E, Kd = k E^-1 e^{G_last - Gb_p}, Ks_pp = k E^-1 e^{Gb_pp - Gb_p}
  float eGbp[4], eGbpS[4], edk[4], cks[4][4];
  #pragma unroll
  for (int j = 0; j < 4; ++j) {
    eGbp[j] = __expf(Gbp[j]);
    eGbpS[j] = eGbp[j] * p.scale;
    edk[j] = __expf(glast[j] - Gbp[j]);
    #pragma unroll
    for (int pp = 0; pp < 4; ++pp) {
      const float gbpp = pp == 0 ? Gb[0][j] : pp == 1 ? Gb[1][j] : pp == 2 ? Gb[2][j] : Gb[3][j];
      cks[pp][j] = __expf(gbpp - Gbp[j]);
    }
  }
  // the same constants as channel pairs (2m, 2m + 1)
  f32x2 eGbp2[2], eGbpS2[2], edk2[2], cks2[4][2];
  #pragma unroll
  for (int m = 0; m < 2; ++m) {
    eGbp2[m] = f2pk(eGbp[2 * m], eGbp[2 * m + 1]);
    eGbpS2[m] = f2pk(eGbpS[2 * m], eGbpS[2 * m + 1]);
    edk2[m] = f2pk(edk[2 * m], edk[2 * m + 1]);
    #pragma unroll
    for (int pp = 0; pp < 4; ++pp) cks2[pp][m] = f2pk(cks[pp][2 * m], cks[pp][2 * m + 1]);
  }
  {
    // Every store of row r0 + i lands at (lane base of its tile) + i * 128 + ((cx ^ i) << 4): rows r0 .. r0 + 7
    // form one 8-row group of every 128-byte-swizzled tile (r0 is a multiple of 8), and the lane's channel
    // group fixes the rest.
    const int cx = (ch & 63) >> 3, kb = ch >> 6, eb = (ch & 7) * 2, rg = r0 >> 3;
    unsigned char* const xq = sm + X + tp * 8192 + kb * 32 * 128 + hh * 1024 + eb;
    unsigned char* const xb = sm + X + tp * 8192 + kb * 32 * 128 + (2 + hh) * 1024 + eb;
    unsigned char* const wqr = rec + L.wq + kb * 128 * 128 + (8 + rg) * 1024 + eb;
    unsigned char* const kdr = rec + L.kd + kb * 64 * 128 + rg * 1024 + eb;
    unsigned char* const rkr = sm + RK + kb * 64 * 128 + rg * 1024 + eb;
    unsigned char* const rvr = sm + RV + kb * 64 * 128 + rg * 1024 + eb;
    unsigned char* ksr[4];
    #pragma unroll
    for (int pp = 0; pp < 4; ++pp) ksr[pp] = sm + KSV + 4096 * (pp * (pp + 1) / 2) + kb * 16 * (pp + 1) * 128 + rg * 1024 + eb;
    float gl[4] = {off[0], off[1], off[2], off[3]};  // tile-local cumsum of g at row r
    // row i + 1 is loaded while row i is computed and stored
    #pragma unroll 2
    for (int i = 0; i < 8; ++i) {
      const int r = r0 + i;
      const uint2 cq = nq, ck = nk, cb = nb, cvv = nv, cw = nw;
      if (r < cv) {
        gl[0] += ng.x; gl[1] += ng.y; gl[2] += ng.z; gl[3] += ng.w;
      }
      if (i + 1 < 8) fetch(i + 1);
      // bf16 pairs of q e^gl, b k e^gl, Qg, Kd, rhs_k, rhs_v; k e^-gl kept in f32 for the Ks_pp of step 2
      uint32_t oq[2], ob[2], og[2], od[2], ork[2], ov[2];
      f32x2 kinv2s[2];
      #pragma unroll
      for (int m = 0; m < 2; ++m) {
        const f32x2 q2 = bf2f2(m ? cq.y : cq.x), k2 = bf2f2(m ? ck.y : ck.x), b2 = bf2f2(m ? cb.y : cb.x);
        const f32x2 v2 = bf2f2(m ? cvv.y : cvv.x), w2 = bf2f2(m ? cw.y : cw.x);
        const f32x2 e2 = f2pk(__expf(gl[2 * m]), __expf(gl[2 * m + 1]));
        const f32x2 ei2 = f2pk(__expf(-gl[2 * m]), __expf(-gl[2 * m + 1]));
        const f32x2 qs2 = f2mul(q2, e2);
        const f32x2 bks2 = f2mul(f2mul(b2, k2), e2);
        const f32x2 kinv2 = f2mul(k2, ei2);
        oq[m] = f2bf2(qs2);
        ob[m] = f2bf2(bks2);
        og[m] = f2bf2(f2mul(qs2, eGbpS2[m]));
        ork[m] = f2bf2(f2mul(bks2, eGbp2[m]));
        od[m] = f2bf2(f2mul(kinv2, edk2[m]));
        ov[m] = f2bf2(f2mul(w2, v2));
        kinv2s[m] = kinv2;
      }
      const uint32_t ro = i * 128 + ((cx ^ i) << 4);
      *reinterpret_cast<uint2*>(xq + ro) = make_uint2(oq[0], oq[1]);
      *reinterpret_cast<uint2*>(xb + ro) = make_uint2(ob[0], ob[1]);
      *reinterpret_cast<uint2*>(wqr + ro) = make_uint2(og[0], og[1]);
      *reinterpret_cast<uint2*>(kdr + ro) = make_uint2(od[0], od[1]);
      *reinterpret_cast<uint2*>(rkr + ro) = make_uint2(ork[0], ork[1]);
      if (ch < V) *reinterpret_cast<uint2*>(rvr + ro) = make_uint2(ov[0], ov[1]);
      #pragma unroll
      for (int pp = 0; pp < 4; ++pp) {
        if (pp < tp) continue;
        *reinterpret_cast<uint2*>(ksr[pp] + ro) =
            make_uint2(f2bf2(f2mul(kinv2s[0], cks2[pp][0])), f2bf2(f2mul(kinv2s[1], cks2[pp][1])));
      }
    }
  }
  if (warp == 0)
    *reinterpret_cast<float4*>(rec + L.gl + ch * 4) =
        make_float4(expf(glast[0]), expf(glast[1]), expf(glast[2]), expf(glast[3]));
  fence_proxy_async_smem();
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tA = *tslot;

  // ---- 3. score MMAs ----
  if (tid == 0) {
    const uint32_t idesc = umma::idesc_bf16(64, 32, false, false);
    const uint32_t sbase = smem_u32(sm);
    const uint64_t dks = umma::desc_kmaj_base(sbase + KSV), dxs = umma::desc_kmaj_base(sbase + X);
    #pragma unroll
    for (int pp = 0; pp < 4; ++pp) {
      const uint64_t ks = umma::desc_add(dks, 4096 * (pp * (pp + 1) / 2));
      const uint64_t xs = umma::desc_add(dxs, pp * 8192);
      #pragma unroll
      for (int j = 0; j < 8; ++j)
        umma::mma_bf16(tA + 32 * pp, umma::desc_kmaj_at(ks, 16 * (pp + 1), j), umma::desc_kmaj_at(xs, 32, j), idesc,
                       j > 0);
    }
    umma::commit(&bars[0]);
  }

  // ---- 4. scores back from TMEM (warp w: sub-partition w % 4, row tiles 2 (w / 4) .. +1) ----
  mbar_wait_bounded(&bars[0], 0);
  umma::fence_after_sync();
  float* sAkk = reinterpret_cast<float*>(sm + AKK);
  float* sTinv = reinterpret_cast<float*>(sm + TINV);
  {
    const int sp = warp & 3, s = 16 * sp + lane;  // valid for lane < 16 (M = 64 TMEM layout)
    #pragma unroll
    for (int pq = 0; pq < 2; ++pq) {
      const int pp = 2 * (warp >> 2) + pq;
      float vq[16], vk[16];
      umma::ld16(umma::taddr(tA, 32 * sp, 32 * pp), vq);
      umma::ld16(umma::taddr(tA, 32 * sp, 32 * pp + 16), vk);
      umma::wait_ld();
      if (lane < 16) {
        #pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int r = 16 * pp + j;
          const float aq = (s <= r) ? vq[j] * p.scale : 0.f;
          *reinterpret_cast<__nv_bfloat16*>(sm + AQK_IMG + umma::kmaj_off(r, s, 64)) = __float2bfloat16_rn(aq);
          sAkk[r * SS + s] = (s < r) ? vk[j] : 0.f;
        }
      }
    }
  }
  umma::fence_before_sync();
  __syncthreads();

  // ---- 5. T = (I + Akk)^-1 over 16 x 16 blocks ----
  // Diagonal blocks T_ii by forward substitution, then the blocks below
  // them from T_ij = -T_ii sum_{m=j}^{i-1} A_im T_mj, scheduled by doubling
  // so that four rounds of 16 x 16 block products on all warps suffice.
  if (warp < 4 && lane < 16) {  // diagonal block `warp`, column `lane`
    const int o = 16 * warp, j = lane;
    float x[16];
    #pragma unroll
    for (int i = 0; i < 16; ++i) {
      float acc = 0.f;
      #pragma unroll
      for (int m = 0; m < i; ++m) acc += sAkk[(o + i) * SS + o + m] * x[m];
      x[i] = (i == j) ? 1.f : ((i < j) ? 0.f : -acc);
    }
    #pragma unroll
    for (int i = 0; i < 16; ++i) sTinv[(o + i) * SS + o + j] = x[i];
  }
  __syncthreads();
  {
    float* scr = reinterpret_cast<float*>(sm + SCRATCH);  // 6 blocks [16][20]: X10 X32 X20 X30 X21 X31
    const int pair = warp >> 1;
    const int row = (warp & 1) * 8 + (lane >> 2), c0 = (lane & 3) * 4;  // 4 outputs of a 16 x 16 block
    auto AK = [&](int i, int j) { return sAkk + 16 * i * SS + 16 * j; };
    auto TI = [&](int i, int j) { return sTinv + 16 * i * SS + 16 * j; };
    auto XS = [&](int k) { return scr + k * 16 * 20; };
    // acc += a_block[row][:] * b_block[:][c0 .. c0 + 3]
    auto mac = [&](float (&acc)[4], const float* a, int as, const float* b, int bs) {
      f32x2 a01 = f2pk(acc[0], acc[1]), a23 = f2pk(acc[2], acc[3]);
      #pragma unroll
      for (int m = 0; m < 16; ++m) {
        const float x = a[row * as + m];
        const f32x2* y = reinterpret_cast<const f32x2*>(b + m * bs + c0);
        const f32x2 x2 = f2pk(x, x);
        a01 = f2fma(x2, y[0], a01);
        a23 = f2fma(x2, y[1], a23);
      }
      f2un(a01, acc[0], acc[1]);
      f2un(a23, acc[2], acc[3]);
    };
    auto put = [&](float* d, int ds, const float (&acc)[4], float sg) {
      *reinterpret_cast<float4*>(d + row * ds + c0) = make_float4(sg * acc[0], sg * acc[1], sg * acc[2], sg * acc[3]);
    };
    {  // X10 = A10 T00, X32 = A32 T22, X20 = A20 T00 (first term), X30 = A30 T00 (first term)
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      const int ai = pair == 0 ? 1 : pair == 2 ? 2 : 3, aj = pair == 1 ? 2 : 0;
      mac(acc, AK(ai, aj), SS, TI(aj, aj), SS);
      put(XS(pair), 20, acc, 1.f);
    }
    __syncthreads();
    {  // T10 = -T11 X10, T32 = -T33 X32, X21 = A21 T11, X31 = A31 T11
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      if (pair < 2) {
        const int d = pair == 0 ? 1 : 3;
        mac(acc, TI(d, d), SS, XS(pair), 20);
        put(TI(d, d - 1), SS, acc, -1.f);
      } else {
        mac(acc, AK(pair, 1), SS, TI(1, 1), SS);
        put(XS(pair + 2), 20, acc, 1.f);
      }
    }
    __syncthreads();
    {  // X20 += A21 T10, X30 += A31 T10, T21 = -T22 X21, T31 = -(T32 X21 + T33 X31)
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      if (pair < 2) {
        const float4 x0 = *reinterpret_cast<const float4*>(XS(2 + pair) + row * 20 + c0);
        acc[0] = x0.x; acc[1] = x0.y; acc[2] = x0.z; acc[3] = x0.w;
        mac(acc, AK(2 + pair, 1), SS, TI(1, 0), SS);
        put(XS(2 + pair), 20, acc, 1.f);
      } else if (pair == 2) {
        mac(acc, TI(2, 2), SS, XS(4), 20);
        put(TI(2, 1), SS, acc, -1.f);
      } else {
        mac(acc, TI(3, 2), SS, XS(4), 20);
        mac(acc, TI(3, 3), SS, XS(5), 20);
        put(TI(3, 1), SS, acc, -1.f);
      }
    }
    __syncthreads();
    if (pair < 2) {  // T20 = -T22 X20, T30 = -(T32 X20 + T33 X30)
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      if (pair == 0) {
        mac(acc, TI(2, 2), SS, XS(2), 20);
        put(TI(2, 0), SS, acc, -1.f);
      } else {
        mac(acc, TI(3, 2), SS, XS(2), 20);
        mac(acc, TI(3, 3), SS, XS(3), 20);
        put(TI(3, 0), SS, acc, -1.f);
      }
    }
    __syncthreads();
  }
  // bf16 image of T (unit diagonal, zero above), 8 elements per store
  for (int idx = tid; idx < 64 * 8; idx += 256) {
    const int r = idx >> 3, c8 = idx & 7;
    const float4 lo = *reinterpret_cast<const float4*>(sTinv + r * SS + 8 * c8);
    const float4 hi = *reinterpret_cast<const float4*>(sTinv + r * SS + 8 * c8 + 4);
    const float in[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
    float val[8];
    #pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int s2 = 8 * c8 + e;
      val[e] = (s2 == r) ? 1.f : ((s2 < r) ? in[e] : 0.f);
    }
    uint4 o;
    o.x = umma::pack_bf16x2(val[0], val[1]); o.y = umma::pack_bf16x2(val[2], val[3]);
    o.z = umma::pack_bf16x2(val[4], val[5]); o.w = umma::pack_bf16x2(val[6], val[7]);
    *reinterpret_cast<uint4*>(sm + TINV_IMG + umma::kmaj_chunk(r, c8, 64)) = o;
  }
  fence_proxy_async_smem();
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();

  // ---- 6. W = T^-1 rhs_k, U = T^-1 rhs_v ----
  if (tid == 0) {
    const uint32_t sbase = smem_u32(sm);
    const uint32_t iw = umma::idesc_bf16(64, 128, false, true);
    const uint32_t iu = umma::idesc_bf16(64, VMAX > 128 ? 128 : V, false, true);
    const uint64_t dt = umma::desc_kmaj_base(sbase + TINV_IMG);
    const uint64_t drk = umma::desc_mnmaj_base(sbase + RK, 64), drv = umma::desc_mnmaj_base(sbase + RV, 64);
    #pragma unroll
    for (int j = 0; j < 4; ++j)
      umma::mma_bf16(tA, umma::desc_kmaj_at(dt, 64, j), umma::desc_mnmaj_at(drk, j), iw, j > 0);
    #pragma unroll
    for (int j = 0; j < 4; ++j)
      umma::mma_bf16(tA + 128, umma::desc_kmaj_at(dt, 64, j), umma::desc_mnmaj_at(drv, j), iu, j > 0);
    umma::commit(&bars[1]);
  }
  // Aqk image to the record while the MMAs run
  for (int idx = tid; idx < 64 * 64 * 2 / 16; idx += 256)
    reinterpret_cast<uint4*>(rec + L.aqk)[idx] = reinterpret_cast<const uint4*>(sm + AQK_IMG)[idx];
  mbar_wait_bounded(&bars[1], 0);
  umma::fence_after_sync();

  // ---- 7. W and U to the record (warp w: sub-partition w % 4, column half w / 4): TMEM -> bf16 images in
  // shared memory -> bulk copies, so the record is written in 8-16 KB runs (a direct store from the TMEM
  // layout writes 16 bytes into each of 16 rows per instruction) ----
  {
    const int sp = warp & 3, half = warp >> 2;
    const int r = 16 * sp + lane;  // valid for lane < 16
    #pragma unroll
    for (int c16 = 0; c16 < 4; ++c16) {
      const int col = half * 64 + 16 * c16;
      float v[16];
      umma::ld16(umma::taddr(tA, 32 * sp, col), v);
      umma::wait_ld();
      if (lane < 16) {
        uint4 lo, hi;
        lo.x = umma::pack_bf16x2(v[0], v[1]); lo.y = umma::pack_bf16x2(v[2], v[3]);
        lo.z = umma::pack_bf16x2(v[4], v[5]); lo.w = umma::pack_bf16x2(v[6], v[7]);
        hi.x = umma::pack_bf16x2(v[8], v[9]); hi.y = umma::pack_bf16x2(v[10], v[11]);
        hi.z = umma::pack_bf16x2(v[12], v[13]); hi.w = umma::pack_bf16x2(v[14], v[15]);
        *reinterpret_cast<uint4*>(sm + WST + umma::kmaj_chunk(r, col / 8, 64)) = lo;
        *reinterpret_cast<uint4*>(sm + WST + umma::kmaj_chunk(r, col / 8 + 1, 64)) = hi;
      }
    }
    // n columns of one value-column slice from TMEM columns tcol .. tcol + n (this warp's half of them) to
    // the slice image at `ust`: rows of n bf16, 16-byte chunk j of row r at chunk j ^ (r & 7)
    auto stage_u = [&](uint32_t ust, uint32_t tcol, int n) {
      for (int c16 = 0; c16 < n / 32; ++c16) {
        const int lc = half * (n / 2) + 16 * c16;
        float v[16];
        umma::ld16(umma::taddr(tA, 32 * sp, tcol + lc), v);
        umma::wait_ld();
        if (lane < 16) {
          uint4 lo, hi;
          lo.x = umma::pack_bf16x2(v[0], v[1]); lo.y = umma::pack_bf16x2(v[2], v[3]);
          lo.z = umma::pack_bf16x2(v[4], v[5]); lo.w = umma::pack_bf16x2(v[6], v[7]);
          hi.x = umma::pack_bf16x2(v[8], v[9]); hi.y = umma::pack_bf16x2(v[10], v[11]);
          hi.z = umma::pack_bf16x2(v[12], v[13]); hi.w = umma::pack_bf16x2(v[14], v[15]);
          uint4* urow = reinterpret_cast<uint4*>(sm + ust + (size_t)r * n * 2);
          urow[(lc / 8) ^ (r & 7)] = lo;
          urow[(lc / 8 + 1) ^ (r & 7)] = hi;
        }
      }
    };
    constexpr int NU = VMAX > 128 ? 128 : 0;  // first slice width (V for VMAX = 128)
    const int nu = NU ? NU : V;
    stage_u(UST, 128, nu);  // the first U MMA's columns
    fence_proxy_async_smem();
    __syncthreads();
    if (tid == 0) {
      bulk_s2g(rec + L.wq, sm + WST, 8192u);
      bulk_s2g(rec + L.wq + 16384, sm + WST + 8192, 8192u);
      bulk_s2g(rec + L.u, sm + UST, (unsigned)(64 * nu * 2));
      bulk_commit();
    }
    if (VMAX > 128) {
      // ---- 8. U columns 128..255: rhs_v of value channels 128 + ch rebuilt in RV (the first U MMA has read
      // it), then one more MMA into W's TMEM columns, which were read out above ----
      uint2 v8[8], w8[8];
      #pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int rr = r0 + i;
        v8[i] = ld4_raw(p.v, bb, hv, t0 + rr, ch + 128, rr < cv);
        w8[i] = ld4_raw(p.w, bb, hv, t0 + rr, ch + 128, rr < cv);
      }
      const int cx = (ch & 63) >> 3, kb = ch >> 6, eb = (ch & 7) * 2, rg = r0 >> 3;
      unsigned char* const rvr = sm + RV + kb * 64 * 128 + rg * 1024 + eb;  // as in step 2
      #pragma unroll
      for (int i = 0; i < 8; ++i) {
        float vv[4], ww[4];
        unpack4(v8[i], vv);
        unpack4(w8[i], ww);
        *reinterpret_cast<uint2*>(rvr + i * 128 + ((cx ^ i) << 4)) =
            pack4(ww[0] * vv[0], ww[1] * vv[1], ww[2] * vv[2], ww[3] * vv[3]);
      }
      fence_proxy_async_smem();
      umma::fence_before_sync();
      __syncthreads();
      umma::fence_after_sync();
      if (tid == 0) {
        const uint32_t sbase = smem_u32(sm);
        const uint32_t iu = umma::idesc_bf16(64, 128, false, true);
        const uint64_t dt = umma::desc_kmaj_base(sbase + TINV_IMG), drv = umma::desc_mnmaj_base(sbase + RV, 64);
        #pragma unroll
        for (int j = 0; j < 4; ++j)
          umma::mma_bf16(tA, umma::desc_kmaj_at(dt, 64, j), umma::desc_mnmaj_at(drv, j), iu, j > 0);
        umma::commit(&bars[1]);
      }
      mbar_wait_bounded(&bars[1], 1);
      umma::fence_after_sync();
      stage_u(UST2, 0, 128);  // U columns 128..255: the second slice
      fence_proxy_async_smem();
      __syncthreads();
      if (tid == 0) {
        bulk_s2g(rec + L.u + 64 * 128 * 2, sm + UST2, 64u * 128u * 2u);
        bulk_commit();
      }
    }
  }
  umma::fence_before_sync();
  __syncthreads();
  if (tid == 0) bulk_wait_read_all();  // the staged images stay in place until the bulk copies have read them
  __syncwarp();
  if (warp == 0) umma::tmem_dealloc(tA, TCOLS);
}

template <int VMAX>
static int launch_intra_tc_v(const TcParams& p, cudaStream_t st) {
  const size_t smem = intra_smem::TOTAL + 1024;
  cudaError_t e =
      cudaFuncSetAttribute((const void*)k_intra_tc<VMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return check_cuda(e, "chunk intra (tc) smem attribute");
  dim3 grid(p.NC, p.HV, p.B);
  k_intra_tc<VMAX><<<grid, 256, smem, st>>>(p);
  return check_cuda(cudaGetLastError(), "chunk intra (tc) launch");
}

int launch_intra_tc(const TcParams& p, cudaStream_t st) {
  return p.V > 128 ? launch_intra_tc_v<256>(p, st) : launch_intra_tc_v<128>(p, st);
}

GDN2_DEVICE_ERROR_READER(read_device_errors_intra_tc)

}  // namespace gdn2
