// Kernel (1), split-operand form: chunk-intra with f32-grade intermediates
// for bf16 or f32 inputs, K = 128, C = 64, V in {64, 128}.
//
// Replaces gdn2_chunk_intra_kernel (src/kernel/chunk_cube.rs:27-295) with the
// numerics of the tensor path src/forward.rs:86-261 (tile-local decay).  Same
// factorisation as the bf16 kernel (chunk_intra_tc.cu), with every operand
// image doubled into a hi and a lo part (chunk_x3.cuh) and every product
// issued as three MMAs.  One CTA (8 warps, one per SM: 213 KB of shared
// memory) per (chunk, value head, batch):
//
//  1. warps 2p, 2p+1 own the two 8-row halves of the 16-row tile p, lane l
//     owns key channels 4l..4l+3: g sums per half tile -> tile boundaries
//     Gb_p, G_last; the tile-local cumsum gl is rebuilt row by row.
//  2. Operands, hi and lo images: X_p = [q e^{gl}; b k e^{gl}] of tile p,
//     Ks_p = k e^{Gb_p - G} for rows s < 16(p+1) (one reference point per
//     row tile, so no factor exceeds 16 tokens of decay, forward.rs:131-157),
//     rhs_k = b k gamma, rhs_v = w v in shared memory; Qg = scale q gamma and
//     Kd = k e^{G_last - G} straight into the record (forward.rs:189-190,
//     :266-274).
//  3. Score MMAs (M=64 N=32 K=128, three passes per row tile): D_p = Ks_p X_p^T
//     = [Aqk^T | Akk^T] columns of row tile p in TMEM.
//  4. Aqk (scaled, causal) -> record images; Akk (strict) -> f32.
//  5. (I + Akk)^-1 in f32 by blocked forward substitution over 16x16 tiles
//     (forward.rs:192-261) -> hi / lo images.
//  6. W = (I+Akk)^-1 rhs_k, U = (I+Akk)^-1 rhs_v (M=64, three passes each).
//  7. W hi / lo images and U in f32 staged in shared memory, written to the
//     record by bulk copies.
#include "chunk_x3.cuh"

namespace gdn2 {

namespace ix3 {
constexpr uint32_t X_HI = 0;            // 4 x 8 KB: K-major [32][128] per row tile
constexpr uint32_t X_LO = 32768;
constexpr uint32_t KS_HI = 65536;       // Ks_p at + 4096 p(p+1)/2, K-major [16(p+1)][128]: 40 KB
constexpr uint32_t KS_LO = 106496;
constexpr uint32_t R1_END = 147456;
// reused once the score MMAs completed
constexpr int SS = 68;                  // row stride (floats) of AKK and TINV
constexpr uint32_t AKK = 0;             // f32 [64][SS]
constexpr uint32_t TINV = 17408;        // f32 [64][SS]
constexpr uint32_t AQK_HI = 36864;      // bf16 K-major [64][64]
constexpr uint32_t AQK_LO = 45056;
constexpr uint32_t TI_HI = 53248;       // bf16 K-major [64][64]: T = (I + Akk)^-1
constexpr uint32_t TI_LO = 61440;
constexpr uint32_t SCRATCH = 69632;     // 6 x f32 [16][20] blocks of the inverse
constexpr uint32_t WST_HI = 81920;      // W rows: K-major [64][128] (two 8 KB column blocks)
constexpr uint32_t WST_LO = 98304;
constexpr uint32_t UST = 114688;        // U f32 [64][V]
// live from step 2 to step 6
constexpr uint32_t RK_HI = R1_END;      // bf16 MN-major [64][128]
constexpr uint32_t RK_LO = RK_HI + 16384;
constexpr uint32_t RV_HI = RK_LO + 16384;  // bf16 MN-major [64][V]
constexpr uint32_t RV_LO = RV_HI + 16384;
constexpr uint32_t MISC = RV_LO + 16384;   // quarter-tile g sums [16][128] f32, sGlast [128] f32, barriers, tmem slot
constexpr uint32_t TOTAL = MISC + 8192 + 512 + 64;
}  // namespace ix3

__device__ __forceinline__ float4 ld_f4_nc_x3(const float* ptr) {
  float4 r;
  asm("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w) : "l"(ptr));
  return r;
}

// L2 prefetch of the inputs of chunk item `item` (every 128-byte line of q, k, b, v, w and g) for the 8 rows
// r0 .. r0 + 7, issued while the previous chunk computes; the two warps that share those rows (half = 0, 1)
// take alternate lines.
template <typename TIN>
__device__ __forceinline__ void prefetch_rows_x3(const TcParams& p, int item, int r0, int lane, int half) {
  const int c = item % p.NC, hv = (item / p.NC) % p.HV, bb = item / (p.NC * p.HV);
  const int kh = hv / p.rep, t0 = c * TC_C, cv = min(TC_C, p.T - t0);
  constexpr int LQ = 128 * (int)sizeof(TIN) / 128;    // lines of a q / k / b row
  const int lv = max(1, p.V * (int)sizeof(TIN) / 128);  // lines of a v / w row
  const int per_row = 3 * LQ + 2 * lv + 4;             // + four lines of g (f32)
  for (int idx = 2 * lane + half; idx < 8 * per_row; idx += 64) {
    const int r = r0 + idx / per_row;
    int j = idx % per_row;
    if (r >= cv) continue;
    const char* a;
    if (j < 3 * LQ) {
      const DView& v = j < LQ ? p.q : j < 2 * LQ ? p.k : p.b;
      a = reinterpret_cast<const char*>(vptr<TIN>(v, bb, kh, t0 + r, 0)) + (j % LQ) * 128;
    } else if ((j -= 3 * LQ) < 2 * lv) {
      const DView& v = j < lv ? p.v : p.w;
      a = reinterpret_cast<const char*>(vptr<TIN>(v, bb, hv, t0 + r, 0)) + (j % lv) * 128;
    } else {
      a = reinterpret_cast<const char*>(static_cast<const float*>(p.g.p) + bb * p.g.s0 + kh * p.g.s1 +
                                        (int64_t)(t0 + r) * p.g.s2) + (j - 2 * lv) * 128;
    }
    asm volatile("prefetch.global.L2 [%0];" ::"l"(a));
  }
}

// Persistent: one CTA per SM walks the chunk items item = blockIdx.x + i * gridDim.x (item = ((b * HV + hv) *
// NC + chunk)).  16 warps: warp 4p + j owns rows 16p + 4j .. +3 of row tile p, lane l key channels 4l..4l+3.
// TMEM is allocated once; rhs_k / rhs_v are built while the score MMAs run, and the next chunk's input rows
// are pulled into L2 meanwhile; the record's bulk copies of one chunk drain while the next chunk loads its rows.
template <typename TIN>
__global__ void __launch_bounds__(512, 1) k_intra_x3(const TcParams p, int nitems) {
  using namespace ix3;
  constexpr uint32_t TCOLS = 512;   // score D [0, 128), W [128, 256), U [256, 384)
  extern __shared__ __align__(1024) unsigned char smraw[];
  unsigned char* sm = smraw + ((1024u - (smem_u32(smraw) & 1023u)) & 1023u);
  float* sQuart = reinterpret_cast<float*>(sm + MISC);  // [16][128] g sums of each 4-row quarter tile
  float* sGlast = sQuart + 16 * 128;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sGlast + 128);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 2);

  const int V = p.V;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tp = warp >> 2, qq = warp & 3;  // row tile, quarter of it (rows 16 tp + 4 qq + i)
  const int r0 = tp * 16 + qq * 4;
  const int ch = lane * 4;                  // first of 4 key channels
  const X3Record L = x3_record_layout(V);
  // byte offset of row r, 16-byte chunk cx, in a 128-byte-swizzled tile (the block of 8 rows r >> 3)
  auto roff = [](int r, int cx) { return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((cx ^ (r & 7)) << 4)); };
  const int cx = (ch & 63) >> 3, kb = ch >> 6, eb = (ch & 7) * 2;

  if (tid == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    umma::tmem_alloc(tslot, TCOLS);
    umma::tmem_relinquish();
  }
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t tA = *tslot;

  int it = 0;
  for (int item = blockIdx.x; item < nitems; item += gridDim.x, ++it) {
    const unsigned par = (unsigned)(it & 1);  // phase parity of both barriers (each completes once per chunk)
    const int c = item % p.NC, hv = (item / p.NC) % p.HV, bb = item / (p.NC * p.HV);
    const int kh = hv / p.rep;
    const int t0 = c * TC_C;
    const int cv = min(TC_C, p.T - t0);
    unsigned char* rec = p.rec + (size_t)item * p.rec_bytes;

    // ---- 1. this warp's 4 rows of g, q, k, b in registers; sums of g over each quarter tile ----
    const float* gbase = static_cast<const float*>(p.g.p) + bb * p.g.s0 + kh * p.g.s1 + ch;
    float4 rg4[4];
    Raw4<TIN> rq[4], rk[4], rb[4];
    #pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = r0 + i;
      rg4[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      rq[i].zero(); rk[i].zero(); rb[i].zero();
      if (r < cv) {
        rg4[i] = ld_f4_nc_x3(gbase + (int64_t)(t0 + r) * p.g.s2);
        rq[i].load(vptr<TIN>(p.q, bb, kh, t0 + r, ch));
        rk[i].load(vptr<TIN>(p.k, bb, kh, t0 + r, ch));
        rb[i].load(vptr<TIN>(p.b, bb, kh, t0 + r, ch));
      }
    }
    float glr[4] = {0.f, 0.f, 0.f, 0.f};  // quarter-local cumsum at the last valid row, if it is ours
    {
      float run[4] = {0.f, 0.f, 0.f, 0.f};
      #pragma unroll
      for (int i = 0; i < 4; ++i) {
        run[0] += rg4[i].x; run[1] += rg4[i].y; run[2] += rg4[i].z; run[3] += rg4[i].w;
        if (r0 + i == cv - 1) {
          glr[0] = run[0]; glr[1] = run[1]; glr[2] = run[2]; glr[3] = run[3];
        }
      }
      *reinterpret_cast<float4*>(sQuart + warp * 128 + ch) = make_float4(run[0], run[1], run[2], run[3]);
    }
    if (tid == 0) bulk_wait_read_all();  // the previous chunk's record copies have read the staging tiles
    __syncthreads();
    float Gb[4][4];  // Gb[pp][j]: G at the end of tile pp - 1 (0 for pp = 0)
    float off[4] = {0.f, 0.f, 0.f, 0.f};  // tile-local cumsum of g before row r0
    #pragma unroll
    for (int j = 0; j < 4; ++j) Gb[0][j] = 0.f;
    #pragma unroll
    for (int pp = 1; pp < 4; ++pp) {
      float a4[4] = {0.f, 0.f, 0.f, 0.f};
      #pragma unroll
      for (int k4 = 0; k4 < 4; ++k4) {
        const float4 a = *reinterpret_cast<const float4*>(sQuart + (4 * (pp - 1) + k4) * 128 + ch);
        a4[0] += a.x; a4[1] += a.y; a4[2] += a.z; a4[3] += a.w;
      }
      #pragma unroll
      for (int j = 0; j < 4; ++j) Gb[pp][j] = Gb[pp - 1][j] + a4[j];
    }
    for (int k4 = 0; k4 < qq; ++k4) {
      const float4 a = *reinterpret_cast<const float4*>(sQuart + (4 * tp + k4) * 128 + ch);
      off[0] += a.x; off[1] += a.y; off[2] += a.z; off[3] += a.w;
    }
    float Gbp[4];
    #pragma unroll
    for (int j = 0; j < 4; ++j) Gbp[j] = tp == 0 ? Gb[0][j] : tp == 1 ? Gb[1][j] : tp == 2 ? Gb[2][j] : Gb[3][j];
    if (r0 <= cv - 1 && cv - 1 < r0 + 4)
      *reinterpret_cast<float4*>(sGlast + ch) = make_float4(Gbp[0] + off[0] + glr[0], Gbp[1] + off[1] + glr[1],
                                                            Gbp[2] + off[2] + glr[2], Gbp[3] + off[3] + glr[3]);
    __syncthreads();

    // ---- 2. score operands (hi and lo images), Qg and Kd into the record ----
    const float4 glast4 = *reinterpret_cast<const float4*>(sGlast + ch);
    const float glast[4] = {glast4.x, glast4.y, glast4.z, glast4.w};
    f32x2 eGbp2[2], eGbpS2[2], edk2[2], cks2[4][2];
    #pragma unroll
    for (int m = 0; m < 2; ++m) {
      const int j0 = 2 * m, j1 = 2 * m + 1;
      const float e0 = __expf(Gbp[j0]), e1 = __expf(Gbp[j1]);
      eGbp2[m] = f2pk(e0, e1);
      eGbpS2[m] = f2pk(e0 * p.scale, e1 * p.scale);
      edk2[m] = f2pk(__expf(glast[j0] - Gbp[j0]), __expf(glast[j1] - Gbp[j1]));
      #pragma unroll
      for (int pp = 0; pp < 4; ++pp) cks2[pp][m] = f2pk(__expf(Gb[pp][j0] - Gbp[j0]), __expf(Gb[pp][j1] - Gbp[j1]));
    }
    f32x2 bks[4][2];  // b k e^{gl} of each row, for rhs_k in step 2b
    {
      const int rr = r0 - 16 * tp;  // row inside the tile
      unsigned char* const xq = sm + X_HI + tp * 8192 + kb * 32 * 128 + eb;
      unsigned char* const wqr = rec + L.wq_hi + kb * 128 * 128 + eb;
      unsigned char* const kdr = rec + L.kd_hi + kb * 64 * 128 + eb;
      constexpr uint32_t DX = X_LO - X_HI, DKS = KS_LO - KS_HI;
      const size_t DWQ = L.wq_lo - L.wq_hi, DKD = L.kd_lo - L.kd_hi;
      float gl[4] = {off[0], off[1], off[2], off[3]};
      #pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = r0 + i;
        gl[0] += rg4[i].x; gl[1] += rg4[i].y; gl[2] += rg4[i].z; gl[3] += rg4[i].w;
        uint32_t h[4][2], l[4][2];  // q e^gl, b k e^gl, Qg, Kd
        f32x2 kinv2s[2];
        #pragma unroll
        for (int m = 0; m < 2; ++m) {
          const f32x2 q2 = rq[i].pair(m), k2 = rk[i].pair(m), b2 = rb[i].pair(m);
          const f32x2 e2 = f2pk(__expf(gl[2 * m]), __expf(gl[2 * m + 1]));
          const f32x2 ei2 = f2pk(__expf(-gl[2 * m]), __expf(-gl[2 * m + 1]));
          const f32x2 qs2 = f2mul(q2, e2);
          bks[i][m] = f2mul(f2mul(b2, k2), e2);
          kinv2s[m] = f2mul(k2, ei2);
          split2(qs2, h[0][m], l[0][m]);
          split2(bks[i][m], h[1][m], l[1][m]);
          split2(f2mul(qs2, eGbpS2[m]), h[2][m], l[2][m]);
          split2(f2mul(kinv2s[m], edk2[m]), h[3][m], l[3][m]);
        }
        const uint32_t oq = roff(rr + i, cx), ob = roff(16 + rr + i, cx);
        *reinterpret_cast<uint2*>(xq + oq) = make_uint2(h[0][0], h[0][1]);
        *reinterpret_cast<uint2*>(xq + DX + oq) = make_uint2(l[0][0], l[0][1]);
        *reinterpret_cast<uint2*>(xq + ob) = make_uint2(h[1][0], h[1][1]);
        *reinterpret_cast<uint2*>(xq + DX + ob) = make_uint2(l[1][0], l[1][1]);
        const uint32_t og = roff(64 + r, cx), orr = roff(r, cx);
        *reinterpret_cast<uint2*>(wqr + og) = make_uint2(h[2][0], h[2][1]);
        *reinterpret_cast<uint2*>(wqr + DWQ + og) = make_uint2(l[2][0], l[2][1]);
        *reinterpret_cast<uint2*>(kdr + orr) = make_uint2(h[3][0], h[3][1]);
        *reinterpret_cast<uint2*>(kdr + DKD + orr) = make_uint2(l[3][0], l[3][1]);
        #pragma unroll
        for (int pp = 0; pp < 4; ++pp) {
          if (pp < tp) continue;
          unsigned char* const ks = sm + KS_HI + 4096 * (pp * (pp + 1) / 2) + kb * 16 * (pp + 1) * 128 + eb + orr;
          uint32_t kh0, kl0, kh1, kl1;
          split2(f2mul(kinv2s[0], cks2[pp][0]), kh0, kl0);
          split2(f2mul(kinv2s[1], cks2[pp][1]), kh1, kl1);
          *reinterpret_cast<uint2*>(ks) = make_uint2(kh0, kh1);
          *reinterpret_cast<uint2*>(ks + DKS) = make_uint2(kl0, kl1);
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

    // ---- 3. score MMAs: per row tile, Ks_hi X_hi + Ks_lo X_hi + Ks_hi X_lo ----
    if (tid == 0) {
      const uint32_t idesc = umma::idesc_bf16(64, 32, false, false);
      const uint32_t sbase = smem_u32(sm);
      #pragma unroll
      for (int pp = 0; pp < 4; ++pp) {
        const uint32_t ko = 4096 * (pp * (pp + 1) / 2), xo = pp * 8192;
        #pragma unroll 1
        for (int pass = 0; pass < 3; ++pass) {
          const uint64_t ks = umma::desc_kmaj_base(sbase + (pass == 1 ? KS_LO : KS_HI) + ko);
          const uint64_t xs = umma::desc_kmaj_base(sbase + (pass == 2 ? X_LO : X_HI) + xo);
          #pragma unroll
          for (int j = 0; j < 8; ++j)
            umma::mma_bf16(tA + 32 * pp, umma::desc_kmaj_at(ks, 16 * (pp + 1), j), umma::desc_kmaj_at(xs, 32, j),
                           idesc, pass > 0 || j > 0);
        }
      }
      umma::commit(&bars[0]);
    }

    // ---- 2b. while the score MMAs run: rhs_k = b k gamma and rhs_v = w v (hi and lo images), and the next
    // chunk's input rows on their way to L2 ----
    {
      unsigned char* const rkr = sm + RK_HI + kb * 64 * 128 + eb;
      unsigned char* const rvr = sm + RV_HI + kb * 64 * 128 + eb;
      constexpr uint32_t DR = RK_LO - RK_HI, DRV = RV_LO - RV_HI;
      Raw4<TIN> rv4[4], rw4[4];
      #pragma unroll
      for (int i = 0; i < 4; ++i) {
        rv4[i].zero(); rw4[i].zero();
        if (r0 + i < cv && ch < V) {
          rv4[i].load(vptr<TIN>(p.v, bb, hv, t0 + r0 + i, ch));
          rw4[i].load(vptr<TIN>(p.w, bb, hv, t0 + r0 + i, ch));
        }
      }
      #pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t orr = roff(r0 + i, cx);
        uint32_t hk[2], lk[2], hv2[2], lv2[2];
        #pragma unroll
        for (int m = 0; m < 2; ++m) {
          split2(f2mul(bks[i][m], eGbp2[m]), hk[m], lk[m]);
          split2(f2mul(rw4[i].pair(m), rv4[i].pair(m)), hv2[m], lv2[m]);
        }
        *reinterpret_cast<uint2*>(rkr + orr) = make_uint2(hk[0], hk[1]);
        *reinterpret_cast<uint2*>(rkr + DR + orr) = make_uint2(lk[0], lk[1]);
        if (ch < V) {
          *reinterpret_cast<uint2*>(rvr + orr) = make_uint2(hv2[0], hv2[1]);
          *reinterpret_cast<uint2*>(rvr + DRV + orr) = make_uint2(lv2[0], lv2[1]);
        }
      }
      fence_proxy_async_smem();
    }
    if (item + (int)gridDim.x < nitems) prefetch_rows_x3<TIN>(p, item + gridDim.x, r0 & ~7, lane, qq & 1);

    // ---- 4. scores back from TMEM (warp w: sub-partition w % 4, row tile w / 4) ----
    mbar_wait_bounded(&bars[0], par);
    umma::fence_after_sync();
    float* sAkk = reinterpret_cast<float*>(sm + AKK);
    float* sTinv = reinterpret_cast<float*>(sm + TINV);
    {
      const int sp = warp & 3, s = 16 * sp + lane;  // valid for lane < 16 (M = 64 TMEM layout)
      const int pp = warp >> 2;
      float vq[16], vk[16];
      umma::ld16(umma::taddr(tA, 32 * sp, 32 * pp), vq);
      umma::ld16(umma::taddr(tA, 32 * sp, 32 * pp + 16), vk);
      umma::wait_ld();
      if (lane < 16) {
        #pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int r = 16 * pp + j;
          const float aq = (s <= r) ? vq[j] * p.scale : 0.f;
          const __nv_bfloat16 ah = __float2bfloat16_rn(aq);
          const uint32_t o = umma::kmaj_off(r, s, 64);
          *reinterpret_cast<__nv_bfloat16*>(sm + AQK_HI + o) = ah;
          *reinterpret_cast<__nv_bfloat16*>(sm + AQK_LO + o) = __float2bfloat16_rn(aq - __bfloat162float(ah));
          sAkk[r * SS + s] = (s < r) ? vk[j] : 0.f;
        }
      }
    }
    umma::fence_before_sync();
    __syncthreads();

    // ---- 5. T = (I + Akk)^-1 over 16 x 16 blocks (diagonal blocks by forward substitution, the blocks below
    // them by doubling: four rounds of 16 x 16 block products on warps 0..7) ----
    if (warp < 4 && lane < 16) {
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
      const bool act = warp < 8;
      const int pair = (warp >> 1) & 3;
      const int row = (warp & 1) * 8 + (lane >> 2), c0 = (lane & 3) * 4;
      auto AK = [&](int i, int j) { return sAkk + 16 * i * SS + 16 * j; };
      auto TI = [&](int i, int j) { return sTinv + 16 * i * SS + 16 * j; };
      auto XS = [&](int k) { return scr + k * 16 * 20; };
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
      if (act) {  // X10 = A10 T00, X32 = A32 T22, X20 = A20 T00 (first term), X30 = A30 T00 (first term)
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        const int ai = pair == 0 ? 1 : pair == 2 ? 2 : 3, aj = pair == 1 ? 2 : 0;
        mac(acc, AK(ai, aj), SS, TI(aj, aj), SS);
        put(XS(pair), 20, acc, 1.f);
      }
      __syncthreads();
      if (act) {  // T10 = -T11 X10, T32 = -T33 X32, X21 = A21 T11, X31 = A31 T11
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
      if (act) {  // X20 += A21 T10, X30 += A31 T10, T21 = -T22 X21, T31 = -(T32 X21 + T33 X31)
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
      if (act && pair < 2) {  // T20 = -T22 X20, T30 = -(T32 X20 + T33 X30)
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
    // hi / lo images of T (unit diagonal, zero above), 8 elements per thread
    {
      const int r = tid >> 3, c8 = tid & 7;
      const float4 lo = *reinterpret_cast<const float4*>(sTinv + r * SS + 8 * c8);
      const float4 hi = *reinterpret_cast<const float4*>(sTinv + r * SS + 8 * c8 + 4);
      const float in[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
      float val[8];
      #pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int s2 = 8 * c8 + e;
        val[e] = (s2 == r) ? 1.f : ((s2 < r) ? in[e] : 0.f);
      }
      uint4 oh, ol;
      split8(val, oh, ol);
      const uint32_t o = umma::kmaj_chunk(r, c8, 64);
      *reinterpret_cast<uint4*>(sm + TI_HI + o) = oh;
      *reinterpret_cast<uint4*>(sm + TI_LO + o) = ol;
    }
    fence_proxy_async_smem();
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();

    // ---- 6. W = T rhs_k, U = T rhs_v, three passes each ----
    if (tid == 0) {
      const uint32_t sbase = smem_u32(sm);
      const uint32_t iw = umma::idesc_bf16(64, 128, false, true);
      const uint32_t iu = umma::idesc_bf16(64, V, false, true);
      #pragma unroll 1
      for (int pass = 0; pass < 3; ++pass) {
        const uint64_t dt = umma::desc_kmaj_base(sbase + (pass == 1 ? TI_LO : TI_HI));
        const uint64_t drk = umma::desc_mnmaj_base(sbase + (pass == 2 ? RK_LO : RK_HI), 64);
        const uint64_t drv = umma::desc_mnmaj_base(sbase + (pass == 2 ? RV_LO : RV_HI), 64);
        #pragma unroll
        for (int j = 0; j < 4; ++j)
          umma::mma_bf16(tA + 128, umma::desc_kmaj_at(dt, 64, j), umma::desc_mnmaj_at(drk, j), iw, pass > 0 || j > 0);
        #pragma unroll
        for (int j = 0; j < 4; ++j)
          umma::mma_bf16(tA + 256, umma::desc_kmaj_at(dt, 64, j), umma::desc_mnmaj_at(drv, j), iu, pass > 0 || j > 0);
      }
      umma::commit(&bars[1]);
    }
    // Aqk images to the record while the MMAs run (AQK_LO directly follows AQK_HI in both)
    for (int idx = tid; idx < 2 * 64 * 64 * 2 / 16; idx += 512)
      reinterpret_cast<uint4*>(rec + L.aqk_hi)[idx] = reinterpret_cast<const uint4*>(sm + AQK_HI)[idx];
    mbar_wait_bounded(&bars[1], par);
    umma::fence_after_sync();

    // ---- 7. W (hi / lo images) and U (f32) staged in shared memory (warp w: sub-partition w % 4, column
    // quarter w / 4), then bulk copies into the record ----
    {
      const int sp = warp & 3, cq = warp >> 2;
      const int r = 16 * sp + lane;  // valid for lane < 16
      #pragma unroll
      for (int c16 = 0; c16 < 2; ++c16) {
        const int col = cq * 32 + 16 * c16;
        float v[16];
        umma::ld16(umma::taddr(tA, 32 * sp, 128 + col), v);
        umma::wait_ld();
        if (lane < 16) {
          uint4 h0, l0, h1, l1;
          split8(v, h0, l0);
          split8(v + 8, h1, l1);
          const uint32_t o0 = umma::kmaj_chunk(r, col / 8, 64), o1 = umma::kmaj_chunk(r, col / 8 + 1, 64);
          *reinterpret_cast<uint4*>(sm + WST_HI + o0) = h0;
          *reinterpret_cast<uint4*>(sm + WST_HI + o1) = h1;
          *reinterpret_cast<uint4*>(sm + WST_LO + o0) = l0;
          *reinterpret_cast<uint4*>(sm + WST_LO + o1) = l1;
        }
      }
      for (int c16 = 0; c16 < V / 64; ++c16) {
        const int col = cq * (V / 4) + 16 * c16;
        float v[16];
        umma::ld16(umma::taddr(tA, 32 * sp, 256 + col), v);
        umma::wait_ld();
        if (lane < 16) {
          float4* urow = reinterpret_cast<float4*>(sm + UST + (size_t)r * V * 4 + col * 4);
          #pragma unroll
          for (int j = 0; j < 4; ++j) urow[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        }
      }
      fence_proxy_async_smem();
      umma::fence_before_sync();
      __syncthreads();
      if (tid == 0) {
        bulk_s2g(rec + L.wq_hi, sm + WST_HI, 8192u);
        bulk_s2g(rec + L.wq_hi + 16384, sm + WST_HI + 8192, 8192u);
        bulk_s2g(rec + L.wq_lo, sm + WST_LO, 8192u);
        bulk_s2g(rec + L.wq_lo + 16384, sm + WST_LO + 8192, 8192u);
        bulk_s2g(rec + L.u, sm + UST, (unsigned)(64 * V * 4));
        bulk_commit();
      }
    }
    umma::fence_after_sync();
  }  // chunk items
  if (tid == 0) bulk_wait_read_all();
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tA, TCOLS);
}

template <typename TIN>
static int launch_intra_x3_t(const TcParams& p, cudaStream_t st) {
  const size_t smem = ix3::TOTAL + 1024;
  cudaError_t e =
      cudaFuncSetAttribute((const void*)k_intra_x3<TIN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return check_cuda(e, "chunk intra (x3) smem attribute");
  int dev = 0, sms = 0;
  e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return check_cuda(e, "chunk intra (x3) SM count");
  const long long items = (long long)p.NC * p.HV * p.B;
  if (items > 0x7fffffffLL) return set_error(GDN2_EUNSUPPORTED, "chunk intra (x3): %lld chunk items", items);
  const int grid = (int)(items < sms ? items : sms);  // one CTA per SM (213 KB of shared memory each)
  k_intra_x3<TIN><<<grid, 512, smem, st>>>(p, (int)items);
  return check_cuda(cudaGetLastError(), "chunk intra (x3) launch");
}

int launch_intra_x3(const TcParams& p, int dtype, cudaStream_t st) {
  return dtype == GDN2_DTYPE_BF16 ? launch_intra_x3_t<__nv_bfloat16>(p, st) : launch_intra_x3_t<float>(p, st);
}

bool x3_supported(int K, int V, int C) { return K == TC_K && C == TC_C && (V == 64 || V == 128); }

GDN2_DEVICE_ERROR_READER(read_device_errors_intra_x3)

}  // namespace gdn2
