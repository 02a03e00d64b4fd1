// Kernel (1), split-operand form: chunk-intra with f32-grade intermediates
// for bf16 or f32 inputs, K = 128, C = 64, V in {64, 128}.
//
// Replaces gdn2_chunk_intra_kernel (src/kernel/chunk_cube.rs:27-295) with the
// numerics of the tensor path src/forward.rs:86-261 (tile-local decay).  Same
// factorisation as the bf16 kernel (chunk_intra_tc.cu), with every operand
// image doubled into a hi and a lo part (chunk_x3.cuh) and every product
// issued as three MMAs.  Two CTAs per SM (8 warps, 87 KB of shared memory and
// 256 TMEM columns each), persistent over (chunk, value head, batch) items, so
// that one CTA's MMA waits and barriers are filled by the other's work.  Per
// chunk:
//
//  1. warps 2p, 2p+1 own the two 8-row halves of the 16-row tile p, lane l
//     owns key channels 4l..4l+3: g sums per half tile -> tile boundaries
//     Gb_p, G_last; the tile-local cumsum gl is rebuilt row by row.
//  2. One pass over the warp's rows builds every operand of the chunk:
//     X_p = [q e^{gl}; b k e^{gl}] of tile p and Ks_p = k e^{Gb_p - G} for
//     rows s < 16(p+1) (one reference point per row tile, so no factor
//     exceeds 16 tokens of decay, forward.rs:131-157), rhs_k = b k gamma,
//     rhs_v = w v (hi and lo images), Qg = scale q gamma and
//     Kd = k e^{G_last - G} (straight into the record, forward.rs:189-190,
//     :266-274).  The images of row tiles 0 and 3 go to a 72 KB shared
//     buffer, those of tiles 1 and 2 and rhs_k / rhs_v to this CTA's scratch
//     slot in global memory (one per CTA, reused chunk after chunk, so it
//     stays in L2).  Score MMAs (M=64 N=32 K=128, three passes per tile):
//     D_p = Ks_p X_p^T = [Aqk^T | Akk^T] columns of row tile p in TMEM; tiles
//     0 and 3 first, then tiles 1 and 2 after one bulk copy of the slot's
//     image into the same buffer.
//  3. Aqk (scaled, causal) -> record images; Akk (strict) -> f32;
//     (I + Akk)^-1 in f32 by blocked forward substitution over 16x16 tiles
//     (forward.rs:192-261) -> hi / lo images.
//  4. rhs_k / rhs_v back from the slot by one bulk copy;
//     W = (I+Akk)^-1 rhs_k, U = (I+Akk)^-1 rhs_v (M=64, three passes each).
//  5. W hi / lo images and U in f32 staged in shared memory, written to the
//     record by bulk copies that drain while the next chunk starts.
#include "chunk_x3.cuh"

namespace gdn2 {

namespace ix3 {
// step 2, the operands of a pair of row tiles pa < pb (tiles 0, 3 in shared memory; tiles 1, 2 in the scratch
// slot with the same offsets), each a hi image followed by its lo image, so that the pair's scores are one
// M = 64, N = 80 product per k-step:
//   X  K-major [64][128]: rows 0..31 = X_pa (its 16 q rows, then its 16 b k rows), rows 32..63 = X_pb;
//   Ks K-major [80][128]: rows 0 .. 16(pa+1)-1 = Ks_pa (the keys of tiles 0..pa at tile pa's reference
//      point), then the 16(pb+1) rows of Ks_pb;
// D = X Ks^T: row i of X against every key row; the cross blocks (X_pa . Ks_pb, X_pb . Ks_pa) are not read.
constexpr uint32_t XA = 0;               // X hi 16 KB, lo at +16 KB
constexpr uint32_t KSA = 32768;          // Ks hi 20 KB, lo at +20 KB; ends at 73728
constexpr int XS_R = 64, KS_R = 80;      // rows of the two stacked operands
constexpr uint32_t R_END = 81920;
// step 3 (the buffer reused once both score MMA passes completed)
constexpr int SS = 68;                   // row stride (floats) of AKK and TINV
constexpr uint32_t AKK = 0;              // f32 [64][SS]
constexpr uint32_t TINV = 17408;         // f32 [64][SS]
constexpr uint32_t SCRATCH = 34816;      // 6 x f32 [16][20] blocks of the inverse
constexpr uint32_t AQK_HI = 49152;       // bf16 K-major [64][64]
constexpr uint32_t AQK_LO = 57344;
constexpr uint32_t TI_HI = 65536;        // bf16 K-major [64][64]: T = (I + Akk)^-1
constexpr uint32_t TI_LO = 73728;
// step 4 (the f32 tiles of step 3 are dead, the Aqk images copied out): the slot's rhs images, same offsets
// at X3_SLOT_PASSB in the slot.  rhs_k and rhs_v side by side form one MN-major [64][128 + V] operand (hi,
// then lo), so W and U are one MMA per k-step; at V = 256 the second rhs_v half follows at 65536 (hi) and
// 81920 (lo) in the slot
constexpr uint32_t RK_HI = 0;            // bf16 MN-major [64][128]
constexpr uint32_t RV_HI = 16384;        // bf16 MN-major [64][min(V, 128)], N groups 2, 3 of the operand
constexpr uint32_t RK_LO = 32768;
constexpr uint32_t RV_LO = 49152;
// step 5 (after the W / U MMAs completed)
constexpr uint32_t WST_HI = 0;           // W rows: K-major [64][128] (two 8 KB column blocks)
constexpr uint32_t WST_LO = 16384;
constexpr uint32_t UST = 32768;          // U f32 [64][V]
constexpr uint32_t MISC = R_END;         // half-tile g sums [2][8][128] f32 and last-row cumsums [2][128] f32 (by
                                         // chunk parity), sGlast [128] f32, barriers, tmem slot
constexpr uint32_t TOTAL = MISC + 8192 + 1024 + 512 + 64;
}  // namespace ix3

__device__ __forceinline__ float4 ld_f4_nc_plain(const float* ptr) {
  float4 r;
  asm("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w) : "l"(ptr));
  return r;
}
__device__ __forceinline__ float4 ld_f4_nc_x3(const float* ptr, uint64_t pol) {
  float4 r;
  asm("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
      : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
      : "l"(ptr), "l"(pol));
  return r;
}

// L2 prefetch of this warp's 8 rows of the inputs of chunk item `item` (every 128-byte line of q, k, b, v, w
// and g), issued while the previous chunk computes.
template <typename TIN>
__device__ __forceinline__ void prefetch_rows_x3(const TcParams& p, int item, int r0, int lane) {
  const int c = item % p.NC, hv = (item / p.NC) % p.HV, bb = item / (p.NC * p.HV);
  const int kh = hv / p.rep, t0 = c * TC_C, cv = min(TC_C, p.T - t0);
  constexpr int LQ = 128 * (int)sizeof(TIN) / 128;    // lines of a q / k / b row
  const int lv = max(1, p.V * (int)sizeof(TIN) / 128);  // lines of a v / w row
  // lane: row r0 + lane / 4, every fourth line of that row's q, k, b, v, w and g (f32, four lines) from lane % 4
  const int r = r0 + (lane >> 2), q4 = lane & 3;
  if (r >= cv) return;
  const char* rows[6] = {
      reinterpret_cast<const char*>(vptr<TIN>(p.q, bb, kh, t0 + r, 0)),
      reinterpret_cast<const char*>(vptr<TIN>(p.k, bb, kh, t0 + r, 0)),
      reinterpret_cast<const char*>(vptr<TIN>(p.b, bb, kh, t0 + r, 0)),
      reinterpret_cast<const char*>(vptr<TIN>(p.v, bb, hv, t0 + r, 0)),
      reinterpret_cast<const char*>(vptr<TIN>(p.w, bb, hv, t0 + r, 0)),
      reinterpret_cast<const char*>(static_cast<const float*>(p.g.p) + bb * p.g.s0 + kh * p.g.s1 +
                                    (int64_t)(t0 + r) * p.g.s2)};
  #pragma unroll
  for (int s = 0; s < 6; ++s) {
    const int nl = s < 3 ? LQ : s < 5 ? lv : 4;
    for (int j = q4; j < nl; j += 4) asm volatile("prefetch.global.L2 [%0];" ::"l"(rows[s] + j * 128));
  }
}

// f32 pair -> (hi, lo) bf16 pairs as one 8-byte store each, at `hi` and `hi + dlo`
__device__ __forceinline__ void put_split4(unsigned char* hi, size_t dlo, f32x2 a, f32x2 b) {
  uint32_t h0, l0, h1, l1;
  split2(a, h0, l0);
  split2(b, h1, l1);
  *reinterpret_cast<uint2*>(hi) = make_uint2(h0, h1);
  *reinterpret_cast<uint2*>(hi + dlo) = make_uint2(l0, l1);
}
// the same into global memory with an L2 eviction policy (record lines: written once, read by another kernel)
__device__ __forceinline__ void put_split4_g(unsigned char* hi, size_t dlo, f32x2 a, f32x2 b, uint64_t pol) {
  uint32_t h0, l0, h1, l1;
  split2(a, h0, l0);
  split2(b, h1, l1);
  asm volatile("st.global.L2::cache_hint.v2.u32 [%0], {%1, %2}, %3;" ::"l"(hi), "r"(h0), "r"(h1), "l"(pol)
               : "memory");
  asm volatile("st.global.L2::cache_hint.v2.u32 [%0], {%1, %2}, %3;" ::"l"(hi + dlo), "r"(l0), "r"(l1), "l"(pol)
               : "memory");
}

// Persistent: two CTAs per SM walk the chunk items item = blockIdx.x + i * gridDim.x (item = ((b * HV + hv) *
// NC + chunk)).  TMEM is allocated once per CTA; the next chunk's input rows are pulled into L2 while a chunk
// computes; the record's bulk copies of one chunk drain while the next chunk loads its rows.
// V256: V = 256, rhs_v and U in two 128-column halves (a separate instantiation keeps the V <= 128 kernel free
// of the second half's loads and MMAs).
template <typename TIN, bool V256>
__global__ void __launch_bounds__(256, 2) k_intra_x3(const TcParams p, int nitems) {
  using namespace ix3;
  constexpr uint32_t TCOLS = 256;   // score D [0, 128), then W [0, 128) and U [128, 128 + V)
  extern __shared__ __align__(1024) unsigned char smraw[];
  unsigned char* sm = smraw + ((1024u - (smem_u32(smraw) & 1023u)) & 1023u);
  float* sHalfB = reinterpret_cast<float*>(sm + MISC);  // [2][8][128] g sums of each 8-row half tile
  float* sGlrB = sHalfB + 2 * 8 * 128;                  // [2][128] half-local cumsum at the last valid row
  float* sGlast = sGlrB + 2 * 128;
  // score MMAs of tiles 0 / 3, of tiles 1 / 2, W / U MMAs, the slot's score image, the slot's rhs images,
  // (V = 256) the slot's second rhs_v half, the second U MMA
  uint64_t* bars = reinterpret_cast<uint64_t*>(sGlast + 128);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 7);

  const int V = p.V;
  const int VU = V256 ? 128 : V;  // value columns of one rhs_v / U half
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tp = warp >> 1, hh = warp & 1;  // row tile, half of it (rows 16 tp + 8 hh + i)
  const int r0 = tp * 16 + hh * 8;
  const int ch = lane * 4;                  // first of 4 key channels
  const X3Record L = x3_record_layout(V);
  // every store of row r0 + i lands at (lane base) + rg * 1024 + i * 128 + ((cx ^ i) << 4) of its
  // 128-byte-swizzled tile: rows r0 .. r0 + 7 form the 8-row group rg of every tile
  const int cx = (ch & 63) >> 3, kb = ch >> 6, eb = (ch & 7) * 2, rg = r0 >> 3;

  if (tid == 0) {
    for (int i = 0; i < 7; ++i) mbar_init(&bars[i], 1);
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
  // records are read only by the inter kernel, long after: evict-first.  Inputs are read once by this CTA
  // unless value heads share key heads (then by the CTAs of the other value heads too): evict-first
  // unless shared.
  const uint64_t pol_rec = l2_policy_evict_first();
  const uint64_t pol_in = l2_policy_evict_first(), pol_kin = p.rep == 1 ? pol_in : l2_policy_evict_normal();

  // step 1 of chunk item `itm` into buffer bf: the g sums of this warp's 8-row half tile, and the half-local
  // cumsum at the chunk's last valid row (by the thread whose rows hold it).  For every chunk but a CTA's first
  // this runs while the previous chunk's W / U MMAs do, on rows already prefetched to L2.
  auto gsum_item = [&](int itm, int bf) {
    const int c_ = itm % p.NC, hv_ = (itm / p.NC) % p.HV, bb_ = itm / (p.NC * p.HV);
    const int t0_ = c_ * TC_C, cv_ = min(TC_C, p.T - t0_);
    const float* gr = static_cast<const float*>(p.g.p) + bb_ * p.g.s0 + (hv_ / p.rep) * p.g.s1 + ch +
                      (int64_t)(t0_ + r0) * p.g.s2;
    float4 gv[8];
    #pragma unroll
    for (int i = 0; i < 8; ++i)
      gv[i] = r0 + i < cv_ ? ld_f4_nc_plain(gr + (int64_t)i * p.g.s2) : make_float4(0.f, 0.f, 0.f, 0.f);
    float run[4] = {0.f, 0.f, 0.f, 0.f};
    #pragma unroll
    for (int i = 0; i < 8; ++i) {
      run[0] += gv[i].x; run[1] += gv[i].y; run[2] += gv[i].z; run[3] += gv[i].w;
      if (r0 + i == cv_ - 1)
        *reinterpret_cast<float4*>(sGlrB + bf * 128 + ch) = make_float4(run[0], run[1], run[2], run[3]);
    }
    *reinterpret_cast<float4*>(sHalfB + bf * 1024 + warp * 128 + ch) = make_float4(run[0], run[1], run[2], run[3]);
  };

  int it = 0;
  for (int item = blockIdx.x; item < nitems; item += gridDim.x, ++it) {
    const unsigned par = (unsigned)(it & 1);  // phase parity of every barrier (each completes once per chunk)
    const int c = item % p.NC, hv = (item / p.NC) % p.HV, bb = item / (p.NC * p.HV);
    const int kh = hv / p.rep;
    const int t0 = c * TC_C;
    const int cv = min(TC_C, p.T - t0);
    unsigned char* rec = p.rec + (size_t)item * p.rec_bytes;
    const float* gbase = static_cast<const float*>(p.g.p) + bb * p.g.s0 + kh * p.g.s1 + ch;

    // ---- 1. sums of g over each half tile (computed during the previous chunk, except for the first) ----
    if (it == 0) gsum_item(item, 0);
    const float* sHalf = sHalfB + (it & 1) * 1024;
    if (tid == 0) bulk_wait_read_all();  // the previous chunk's record copies have read the staging tiles
    __syncthreads();
    float Gb[4][4];  // Gb[pp][j]: G at the end of tile pp - 1 (0 for pp = 0)
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
    if (r0 <= cv - 1 && cv - 1 < r0 + 8) {
      const float4 gl = *reinterpret_cast<const float4*>(sGlrB + (it & 1) * 128 + ch);
      *reinterpret_cast<float4*>(sGlast + ch) = make_float4(Gbp[0] + off[0] + gl.x, Gbp[1] + off[1] + gl.y,
                                                            Gbp[2] + off[2] + gl.z, Gbp[3] + off[3] + gl.w);
    }
    __syncthreads();
    f32x2 eGbp2[2];
    #pragma unroll
    for (int m = 0; m < 2; ++m) eGbp2[m] = f2pk(__expf(Gbp[2 * m]), __expf(Gbp[2 * m + 1]));

    // ---- 2. one pass over this warp's rows: every operand of the chunk.  Row tiles 0 and 3 (X and Ks images)
    // go to the shared buffer of the first score pass; row tiles 1 and 2 to this CTA's scratch slot, laid out
    // as the buffer of the second pass; rhs_k / rhs_v to the slot too; Qg and Kd into the record. ----
    unsigned char* const slot = p.scratch + (size_t)blockIdx.x * x3_slot_bytes(V);
    {
      f32x2 cks2[4][2], eGbpS2[2], edk2[2];
      {
        const float4 gl4 = *reinterpret_cast<const float4*>(sGlast + ch);
        const float glast[4] = {gl4.x, gl4.y, gl4.z, gl4.w};
        #pragma unroll
        for (int m = 0; m < 2; ++m) {
          const int j0 = 2 * m, j1 = 2 * m + 1;
          eGbpS2[m] = f2mul(eGbp2[m], f2pk(p.scale, p.scale));
          edk2[m] = f2pk(__expf(glast[j0] - Gbp[j0]), __expf(glast[j1] - Gbp[j1]));
          #pragma unroll
          for (int pp = 0; pp < 4; ++pp)
            cks2[pp][m] = f2pk(__expf(Gb[pp][j0] - Gbp[j0]), __expf(Gb[pp][j1] - Gbp[j1]));
        }
      }
      // X rows of this row tile: tiles 0 / 3 in the shared buffer, 1 / 2 in the slot; the pair's first tile at
      // stacked rows 0..31, its second at 32..63
      unsigned char* const xr = (tp == 0 || tp == 3 ? sm : slot) + XA + kb * XS_R * 128 +
                                ((tp == 0 || tp == 1) ? 0 : 4096) + hh * 1024 + eb;
      // Ks_pp rows of this thread's key rows (16 tp + 8 hh + i): Ks_0 / Ks_1 from stacked row 0, Ks_3 from row 16,
      // Ks_2 from row 32
      auto ks_row = [&](int pp) {
        unsigned char* const base = (pp == 0 || pp == 3) ? sm : slot;
        const int row0 = pp == 3 ? 16 : pp == 2 ? 32 : 0;
        return base + KSA + kb * KS_R * 128 + (row0 / 8 + rg) * 1024 + eb;
      };
      unsigned char* const wqr = rec + L.wq_hi + kb * 128 * 128 + (8 + rg) * 1024 + eb;
      unsigned char* const kdr = rec + L.kd_hi + kb * 64 * 128 + rg * 1024 + eb;
      unsigned char* const rkr = slot + X3_SLOT_PASSB + RK_HI + kb * 64 * 128 + rg * 1024 + eb;
      unsigned char* const rvr = slot + X3_SLOT_PASSB + RV_HI + kb * 64 * 128 + rg * 1024 + eb;
      float gl[4] = {off[0], off[1], off[2], off[3]};
      Raw4<TIN> nq, nk, nb, nv, nw, nv2, nw2;  // nv2, nw2: value channels 128 + ch (V = 256)
      float4 ng;
      // this lane's elements of row r0 of each input, advanced by one row per fetch
      const TIN* aq = static_cast<const TIN*>(vptr<TIN>(p.q, bb, kh, t0 + r0, ch));
      const TIN* ak = static_cast<const TIN*>(vptr<TIN>(p.k, bb, kh, t0 + r0, ch));
      const TIN* ab = static_cast<const TIN*>(vptr<TIN>(p.b, bb, kh, t0 + r0, ch));
      const TIN* av = static_cast<const TIN*>(vptr<TIN>(p.v, bb, hv, t0 + r0, ch));
      const TIN* aw = static_cast<const TIN*>(vptr<TIN>(p.w, bb, hv, t0 + r0, ch));
      const float* ag = gbase + (int64_t)(t0 + r0) * p.g.s2;
      auto fetch = [&](int i) {
        const int r = r0 + i;
        nq.zero(); nk.zero(); nb.zero(); nv.zero(); nw.zero();
        ng = make_float4(0.f, 0.f, 0.f, 0.f);
        if (V256) {
          nv2.zero(); nw2.zero();
        }
        if (r < cv) {
          ng = ld_f4_nc_x3(ag, pol_kin);
          nq.load(aq, pol_kin);
          nk.load(ak, pol_kin);
          nb.load(ab, pol_kin);
          if (ch < V) {
            nv.load(av, pol_in);
            nw.load(aw, pol_in);
          }
          if (V256) {
            nv2.load(av + 128, pol_in);
            nw2.load(aw + 128, pol_in);
          }
        }
        aq += p.q.s2; ak += p.k.s2; ab += p.b.s2; av += p.v.s2; aw += p.w.s2; ag += p.g.s2;
      };
      fetch(0);
      #pragma unroll 1
      for (int i = 0; i < 8; ++i) {
        const Raw4<TIN> cq = nq, ck = nk, cb = nb, cvv = nv, cw = nw, cv2 = nv2, cw2 = nw2;
        gl[0] += ng.x; gl[1] += ng.y; gl[2] += ng.z; gl[3] += ng.w;
        if (i + 1 < 8) fetch(i + 1);
        const uint32_t ro = (uint32_t)(i * 128 + ((cx ^ i) << 4));
        f32x2 kinv2[2], qs2[2], bks2[2];
        #pragma unroll
        for (int m = 0; m < 2; ++m) {
          const f32x2 e2 = f2pk(__expf(gl[2 * m]), __expf(gl[2 * m + 1]));
          const f32x2 ei2 = f2pk(__expf(-gl[2 * m]), __expf(-gl[2 * m + 1]));
          const f32x2 k2 = ck.pair(m);
          kinv2[m] = f2mul(k2, ei2);
          qs2[m] = f2mul(cq.pair(m), e2);
          bks2[m] = f2mul(f2mul(cb.pair(m), k2), e2);
        }
        // X rows: q part at row 8 hh + i, b k part at 16 + 8 hh + i of the tile's 32 rows
        put_split4(xr + ro, 16384, qs2[0], qs2[1]);
        put_split4(xr + 2048 + ro, 16384, bks2[0], bks2[1]);
        #pragma unroll
        for (int pp = 0; pp < 4; ++pp) {
          if (pp < tp) continue;
          put_split4(ks_row(pp) + ro, KS_R * 256, f2mul(kinv2[0], cks2[pp][0]), f2mul(kinv2[1], cks2[pp][1]));
        }
        put_split4_g(wqr + ro, L.wq_lo - L.wq_hi, f2mul(qs2[0], eGbpS2[0]), f2mul(qs2[1], eGbpS2[1]), pol_rec);
        put_split4_g(kdr + ro, L.kd_lo - L.kd_hi, f2mul(kinv2[0], edk2[0]), f2mul(kinv2[1], edk2[1]), pol_rec);
        put_split4(rkr + ro, RK_LO - RK_HI, f2mul(bks2[0], eGbp2[0]), f2mul(bks2[1], eGbp2[1]));
        if (ch < V) put_split4(rvr + ro, RV_LO - RV_HI, f2mul(cw.pair(0), cvv.pair(0)), f2mul(cw.pair(1), cvv.pair(1)));
        if (V256)  // the second rhs_v half
          put_split4(rvr + (65536 - RV_HI) + ro, 16384, f2mul(cw2.pair(0), cv2.pair(0)), f2mul(cw2.pair(1), cv2.pair(1)));
      }
    }
    if (warp == 0) {
      const float4 gl4 = *reinterpret_cast<const float4*>(sGlast + ch);
      *reinterpret_cast<float4*>(rec + L.gl + ch * 4) = make_float4(expf(gl4.x), expf(gl4.y), expf(gl4.z),
                                                                    expf(gl4.w));
    }
    fence_proxy_async_smem();     // the operand images in shared memory, for the MMAs
    fence_proxy_async_global();   // the slot, for the bulk copies that bring it back
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();

    // score MMAs of a tile pair, D = X_hi Ks_hi^T + X_hi Ks_lo^T + X_lo Ks_hi^T (M = 64, N = 80): tiles {0, 3}
    // from the buffer into TMEM columns [0, 80); then, once they have read it, tiles {1, 2} after one bulk copy
    // of the slot's images into the same buffer, into columns [128, 208)
    if (tid == 0) {
      const uint32_t idesc = umma::idesc_bf16(64, KS_R, false, false);
      const uint32_t sbase = smem_u32(sm);
      auto pair_mmas = [&](uint32_t dcol) {
        #pragma unroll 1
        for (int ps = 0; ps < 3; ++ps) {
          const uint64_t dxs = umma::desc_kmaj_base(sbase + XA + (ps == 2 ? 16384 : 0));
          const uint64_t dks = umma::desc_kmaj_base(sbase + KSA + (ps == 1 ? KS_R * 256 : 0));
          #pragma unroll
          for (int j = 0; j < 8; ++j)
            umma::mma_bf16(tA + dcol, umma::desc_kmaj_at(dxs, XS_R, j), umma::desc_kmaj_at(dks, KS_R, j), idesc,
                           ps > 0 || j > 0);
        }
      };
      pair_mmas(0);
      umma::commit(&bars[0]);
      mbar_wait_bounded(&bars[0], par);
      umma::fence_after_sync();
      mbar_arrive_expect_tx(&bars[3], (unsigned)X3_SLOT_PASSB);
      bulk_g2s(sm, slot, (unsigned)X3_SLOT_PASSB, &bars[3]);
      mbar_wait_bounded(&bars[3], par);
      pair_mmas(128);
      umma::commit(&bars[1]);
    }
    if (item + (int)gridDim.x < nitems) prefetch_rows_x3<TIN>(p, item + gridDim.x, r0, lane);
    // ---- 3. scores back from TMEM (warp w: sub-partition w % 4, row tiles 2 (w / 4) .. +1), then T ----
    mbar_wait_bounded(&bars[1], par);  // both passes (the second commit covers every earlier MMA)
    umma::fence_after_sync();
    // the slot's score images were read back (the second pass's MMAs, issued after that copy, are done):
    // dropped from L2 instead of written back to HBM
    for (int l = tid; l < (int)(X3_SLOT_PASSB / 128); l += 256) discard_l2_line(slot + (size_t)l * 128);
    float* sAkk = reinterpret_cast<float*>(sm + AKK);
    float* sTinv = reinterpret_cast<float*>(sm + TINV);
    {
      // warp w: pair w / 4 (TMEM columns from 128 (w / 4)), sub-partition w % 4 = D rows 16 (w % 4) + lane
      // (lane < 16, the M = 64 layout): the q rows (even sub-partitions) or b k rows (odd) of the pair's first
      // (sub-partitions 0, 1) or second tile, one query row per lane, against that tile's 16 (t + 1) keys
      const int sp = warp & 3, pr = warp >> 2;
      const int t = pr == 0 ? (sp < 2 ? 0 : 3) : (sp < 2 ? 1 : 2);
      const int kc0 = (sp < 2) ? 0 : (pr == 0 ? 16 : 32);  // first key column of tile t in D
      const int i = 16 * t + lane;                           // query row (lane < 16)
      const bool qrow = (sp & 1) == 0;
      for (int c16 = 0; c16 <= t; ++c16) {
        float v[16];
        umma::ld16(umma::taddr(tA, 32 * sp, 128 * pr + kc0 + 16 * c16), v);
        umma::wait_ld();
        if (lane < 16) {
          const int j0 = 16 * c16;
          if (qrow) {  // Aqk row i, keys j0 .. j0 + 15: scale (q . k decay) for j <= i
            #pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = (j0 + j <= i) ? v[j] * p.scale : 0.f;
            uint4 h0, l0, h1, l1;
            split8(v, h0, l0);
            split8(v + 8, h1, l1);
            const uint32_t o0 = umma::kmaj_chunk(i, j0 / 8, 64), o1 = umma::kmaj_chunk(i, j0 / 8 + 1, 64);
            *reinterpret_cast<uint4*>(sm + AQK_HI + o0) = h0;
            *reinterpret_cast<uint4*>(sm + AQK_HI + o1) = h1;
            *reinterpret_cast<uint4*>(sm + AQK_LO + o0) = l0;
            *reinterpret_cast<uint4*>(sm + AQK_LO + o1) = l1;
          } else {  // Akk row i: (b k . k decay) for j < i
            float4* arow = reinterpret_cast<float4*>(sAkk + i * SS + j0);
            #pragma unroll
            for (int j = 0; j < 16; j += 4)
              arow[j / 4] = make_float4((j0 + j < i) ? v[j] : 0.f, (j0 + j + 1 < i) ? v[j + 1] : 0.f,
                                        (j0 + j + 2 < i) ? v[j + 2] : 0.f, (j0 + j + 3 < i) ? v[j + 3] : 0.f);
          }
        }
      }
      if (lane < 16) {  // the keys after tile t: zero
        for (int j0 = 16 * (t + 1); j0 < 64; j0 += 16) {
          if (qrow) {
            const uint4 z = make_uint4(0u, 0u, 0u, 0u);
            const uint32_t o0 = umma::kmaj_chunk(i, j0 / 8, 64), o1 = umma::kmaj_chunk(i, j0 / 8 + 1, 64);
            *reinterpret_cast<uint4*>(sm + AQK_HI + o0) = z;
            *reinterpret_cast<uint4*>(sm + AQK_HI + o1) = z;
            *reinterpret_cast<uint4*>(sm + AQK_LO + o0) = z;
            *reinterpret_cast<uint4*>(sm + AQK_LO + o1) = z;
          } else {
            float4* arow = reinterpret_cast<float4*>(sAkk + i * SS + j0);
            #pragma unroll
            for (int j = 0; j < 4; ++j) arow[j] = make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
      }
    }
    umma::fence_before_sync();
    __syncthreads();
    // the Aqk images to the record (plain 16-byte copies) while warps 0..3 invert the diagonal blocks
    for (int idx = tid; idx < 2 * 64 * 64 * 2 / 16; idx += 256)
      reinterpret_cast<uint4*>(rec + L.aqk_hi)[idx] = reinterpret_cast<const uint4*>(sm + AQK_HI)[idx];
    if (warp < 4 && lane < 16) {  // diagonal block `warp`, column `lane`, by forward substitution
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
    {  // the blocks below the diagonal by doubling: four rounds of 16 x 16 block products on all warps
      float* scr = reinterpret_cast<float*>(sm + SCRATCH);  // 6 blocks [16][20]: X10 X32 X20 X30 X21 X31
      const int pair = warp >> 1;
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
    // hi / lo images of T (unit diagonal, zero above), 8 elements per store
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
      uint4 oh, ol;
      split8(val, oh, ol);
      const uint32_t o = umma::kmaj_chunk(r, c8, 64);
      *reinterpret_cast<uint4*>(sm + TI_HI + o) = oh;
      *reinterpret_cast<uint4*>(sm + TI_LO + o) = ol;
    }
    fence_proxy_async_smem();  // the f32 tiles and the Aqk images are read: a bulk copy overwrites them
    __syncthreads();

    // ---- 4. rhs_k and rhs_v back from the slot (one bulk copy), then W = T rhs_k, U = T rhs_v ----
    if (tid == 0) {  // W into the score columns [0, 128) (read out above), U into [128, 128 + VU)
      mbar_arrive_expect_tx(&bars[4], 65536u);
      bulk_g2s(sm + RK_HI, slot + X3_SLOT_PASSB, 65536u, &bars[4]);
      mbar_wait_bounded(&bars[4], par);
      const uint32_t sbase = smem_u32(sm);
      const uint32_t iwu = umma::idesc_bf16(64, 128 + VU, false, true);  // [W | U] = T [rhs_k | rhs_v]
      #pragma unroll 1
      for (int ps = 0; ps < 3; ++ps) {
        const uint64_t dt = umma::desc_kmaj_base(sbase + (ps == 1 ? TI_LO : TI_HI));
        const uint64_t drhs = umma::desc_mnmaj_base(sbase + (ps == 2 ? RK_LO : RK_HI), 64);
        #pragma unroll
        for (int j = 0; j < 4; ++j)
          umma::mma_bf16(tA, umma::desc_kmaj_at(dt, 64, j), umma::desc_mnmaj_at(drhs, j), iwu, ps > 0 || j > 0);
      }
      umma::commit(&bars[2]);
    }
    if (item + (int)gridDim.x < nitems) gsum_item(item + (int)gridDim.x, (it + 1) & 1);
    mbar_wait_bounded(&bars[2], par);
    umma::fence_after_sync();
    // the slot's rhs images were read back (the W / U MMAs are done): dropped from L2 likewise (the second rhs_v
    // half of V = 256 is read back later, and dropped then)
    for (int l = tid; l < 65536 / 128; l += 256) discard_l2_line(slot + X3_SLOT_PASSB + (size_t)l * 128);

    // ---- 5. W (hi / lo images) and U (f32, one 128-column slice at a time) staged in shared memory (warp w:
    // sub-partition w % 4, column half w / 4), then bulk copies into the record (they drain while the next
    // chunk starts) ----
    const int sp = warp & 3, half = warp >> 2;
    const int r = 16 * sp + lane;  // valid for lane < 16
    auto stage_u = [&](unsigned char* dst) {  // U columns [128, 128 + VU) of TMEM -> UST -> the record at dst
      for (int c16 = 0; c16 < VU / 32; ++c16) {
        const int col = half * (VU / 2) + 16 * c16;
        float v[16];
        umma::ld16(umma::taddr(tA, 32 * sp, 128 + col), v);
        umma::wait_ld();
        if (lane < 16) {  // 16-byte word k of row r at k ^ (r & 7) (the record's layout; no bank conflicts)
          float4* urow = reinterpret_cast<float4*>(sm + UST + (size_t)r * VU * 4);
          #pragma unroll
          for (int j = 0; j < 4; ++j)
            urow[(col / 4 + j) ^ (r & 7)] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        }
      }
      fence_proxy_async_smem();
      umma::fence_before_sync();
      __syncthreads();
      if (tid == 0) {
        bulk_s2g_hint(dst, sm + UST, (unsigned)(64 * VU * 4), pol_rec);
        bulk_commit();
      }
    };
    {
      #pragma unroll
      for (int c16 = 0; c16 < 4; ++c16) {
        const int col = half * 64 + 16 * c16;
        float v[16];
        umma::ld16(umma::taddr(tA, 32 * sp, col), v);
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
      stage_u(rec + L.u);  // its proxy fence and barrier also cover the W images
      if (tid == 0) {
        bulk_s2g_hint(rec + L.wq_hi, sm + WST_HI, 8192u, pol_rec);
        bulk_s2g_hint(rec + L.wq_hi + 16384, sm + WST_HI + 8192, 8192u, pol_rec);
        bulk_s2g_hint(rec + L.wq_lo, sm + WST_LO, 8192u, pol_rec);
        bulk_s2g_hint(rec + L.wq_lo + 16384, sm + WST_LO + 8192, 8192u, pol_rec);
        bulk_commit();
      }
    }
    if (V256) {
      // the second rhs_v half into the rhs_v tiles (which the U staging shares: wait for its copy to read it),
      // U columns 128..255 into the same TMEM columns, staged and copied as the record's second U slice
      if (tid == 0) {
        umma::fence_after_sync();  // the first U half is read out of TMEM
        bulk_wait_read_all();
        mbar_arrive_expect_tx(&bars[5], 32768u);
        bulk_g2s(sm + RV_HI, slot + X3_SLOT_PASSB + 65536, 16384u, &bars[5]);
        bulk_g2s(sm + RV_LO, slot + X3_SLOT_PASSB + 81920, 16384u, &bars[5]);
        mbar_wait_bounded(&bars[5], par);
        const uint32_t sbase = smem_u32(sm);
        const uint32_t iu = umma::idesc_bf16(64, 128, false, true);
        #pragma unroll 1
        for (int ps = 0; ps < 3; ++ps) {
          const uint64_t dt = umma::desc_kmaj_base(sbase + (ps == 1 ? TI_LO : TI_HI));
          const uint64_t drv = umma::desc_mnmaj_base(sbase + (ps == 2 ? RV_LO : RV_HI), 64);
          #pragma unroll
          for (int j = 0; j < 4; ++j)
            umma::mma_bf16(tA + 128, umma::desc_kmaj_at(dt, 64, j), umma::desc_mnmaj_at(drv, j), iu, ps > 0 || j > 0);
        }
        umma::commit(&bars[6]);
      }
      mbar_wait_bounded(&bars[6], par);
      umma::fence_after_sync();
      // the second rhs_v half was read back (its U MMA is done): dropped from L2 like the rest of the slot
      for (int l = tid; l < 32768 / 128; l += 256) discard_l2_line(slot + X3_SLOT_PASSB + 65536 + (size_t)l * 128);
      stage_u(rec + L.u + 64 * 128 * 4);
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
  void (*fn)(const TcParams, int) = p.V > 128 ? k_intra_x3<TIN, true> : k_intra_x3<TIN, false>;
  cudaError_t e = cudaFuncSetAttribute((const void*)fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return check_cuda(e, "chunk intra (x3) smem attribute");
  const int sms = usable_sms();  // less the SMs the host reserved for its own work
  const long long items = (long long)p.NC * p.HV * p.B;
  if (items > 0x7fffffffLL) return set_error(GDN2_EUNSUPPORTED, "chunk intra (x3): %lld chunk items", items);
  const long long slots = 2LL * sms;  // two CTAs per SM (87 KB of shared memory, 256 TMEM columns each)
  const int grid = (int)(items < slots ? items : slots);
  fn<<<grid, 256, smem, st>>>(p, (int)items);
  return check_cuda(cudaGetLastError(), "chunk intra (x3) launch");
}

int launch_intra_x3(const TcParams& p, int dtype, cudaStream_t st) {
  return dtype == GDN2_DTYPE_BF16 ? launch_intra_x3_t<__nv_bfloat16>(p, st) : launch_intra_x3_t<float>(p, st);
}

bool x3_supported(int K, int V, int C) { return K == TC_K && C == TC_C && (V == 64 || V == 128 || V == 256); }

GDN2_DEVICE_ERROR_READER(read_device_errors_intra_x3)

}  // namespace gdn2
