// Kernel (2) on tensor cores: chunk-inter for bf16 inputs, K = 128, C = 64,
// with the SiLU-gated RMS-norm epilogue fused.
//
// Replaces gdn2_chunk_inter_kernel (src/kernel/chunk_cube.rs:300-610); math
// of src/forward.rs:263-274 with the epilogue of src/module.rs:501-517.
// One CTA (8 warps) per (value-column slice, value head, batch) walks the
// chunks in order; V <= 128 is one slice, V = 256 two slices of 128 columns
// (the value columns of the recurrence are independent: each slice reads the
// shared W, Qg, Kd, Aqk parts of the record and its own U columns).  The
// state S [K][V] slice stays in TMEM in f32 for the whole sequence; a bf16
// image of it in shared memory is the MMA operand.  Per chunk:
//   MMA1  D = [W; Qg] S                    (M=128, N=V, K=128)
//   v_new = U - (W S)                      (rows 0..63 of D, to smem, bf16)
//   MMA2  D += [0; Aqk] v_new              (rows 64..127 become o)
//   MMA3  S = diag(gamma_last) S + Kd^T v_new   (S pre-scaled in TMEM)
//   o -> gated RMS norm -> out; S -> bf16 image for the next chunk.
// With two slices the RMS norm needs both halves of a row: the two CTAs of a
// chain form a cluster, and each epilogue thread writes its slice's row sum
// of squares into the other CTA's shared memory and arrives on that CTA's
// exchange mbarrier (release, cluster scope), then waits on its own (bounded,
// acquire) for the other half.
// The per-chunk record written by the intra kernel (operand-tile images)
// arrives by bulk copies into one of two stages while the previous chunk
// computes.
#include "chunk_tc.cuh"
#include "umma.cuh"

namespace gdn2 {

namespace inter_smem {
constexpr uint32_t ST_WQ = 0;         // K-major [128][128]
constexpr uint32_t ST_TA = 32768;     // K-major [128][64]: rows 0..63 zero, 64..127 Aqk
constexpr uint32_t ST_KD = 49152;     // MN-major [64][128]
constexpr uint32_t ST_U = 65536;      // bf16 [64][V], V <= 128
constexpr uint32_t ST_GL = 81920;     // f32 [128]
constexpr uint32_t STAGE = 82944;     // 81 KB per stage
constexpr uint32_t S_IMG = 2 * STAGE;           // MN-major [128][V]
constexpr uint32_t VN_IMG = S_IMG + 32768;      // MN-major [64][V]
constexpr uint32_t MISC = VN_IMG + 16384;       // rms partials [64][2], o-norm weight [V], barriers, tmem slot
constexpr uint32_t ONW = MISC + 512;
constexpr uint32_t BARS = ONW + 512;
constexpr uint32_t XSUM = BARS + 64;    // f32 [2][64]: the peer slice's row sums, by chunk parity
constexpr uint32_t XBARS = XSUM + 512;  // 2 mbarriers: the peer's 128 epilogue threads arrived, by chunk parity
constexpr uint32_t TOTAL = XBARS + 64;
}  // namespace inter_smem

__device__ __forceinline__ void named_bar(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// XCHG: the two value-column slices of a chain (a 2-CTA cluster) exchange
// the RMS norm's row sums; a separate instantiation keeps the one-slice
// kernel free of that code.
template <bool XCHG>
__global__ void __launch_bounds__(256, 1) k_inter_tc(const TcParams p) {
  using namespace inter_smem;
  extern __shared__ __align__(1024) unsigned char smraw[];
  unsigned char* sm = smraw + ((1024u - (smem_u32(smraw) & 1023u)) & 1023u);
  float* sRms = reinterpret_cast<float*>(sm + MISC);
  float* sOnw = reinterpret_cast<float*>(sm + ONW);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + BARS);  // full[2], mma1, mma2/3, operands ready
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 5);
  float* sXsum = reinterpret_cast<float*>(sm + XSUM);
  uint64_t* xbars = reinterpret_cast<uint64_t*>(sm + XBARS);

  const int hv = blockIdx.y, bb = blockIdx.z;
  const int V = p.vt, HALF = V / 2;                 // columns of this CTA's slice
  const int VF = p.V, cbase = blockIdx.x * p.vt;   // full row width, first column of the slice
  constexpr bool xchg = XCHG;                          // row sums exchanged with the other slice's CTA
  const uint32_t peer = blockIdx.x ^ 1u;               // cluster rank of that CTA (cluster = the vsplit slices)
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int sp = warp & 3, half = warp >> 2;
  const int col0 = half * HALF;
  const TcRecord L = tc_record_layout(VF);
  const unsigned char* recs = p.rec + ((size_t)bb * p.HV + hv) * p.NC * p.rec_bytes;
  float* st = p.state + ((size_t)bb * p.HV + hv) * (size_t)TC_K * VF + cbase;
  const uint32_t sbase = smem_u32(sm);

  if (warp == 0) {
    umma::tmem_alloc(tslot, 512);
    umma::tmem_relinquish();
  }
  if (p.fuse_epilogue)
    for (int i = tid; i < V; i += 256) sOnw[i] = p.onw[cbase + i];
  if (tid == 0) {
    for (int i = 0; i < 4; ++i) mbar_init(&bars[i], 1);
    mbar_init(&bars[4], 256);  // every thread: its v_new rows / S rescale done
    mbar_init(&xbars[0], 128);
    mbar_init(&xbars[1], 128);
    fence_mbar_init();
  }
  // zero halves of the [0; Aqk] tiles (never written by the copies)
  for (int i = tid; i < 2 * 8192 / 16; i += 256) {
    const int s = i / (8192 / 16), o = i % (8192 / 16);
    reinterpret_cast<uint4*>(sm + s * STAGE + ST_TA)[o] = make_uint4(0, 0, 0, 0);
  }
  umma::fence_before_sync();
  __syncthreads();
  if (xchg) cluster_sync_all();  // the peer's exchange barriers are initialised before anyone arrives on them
  umma::fence_after_sync();
  const uint32_t tD0 = *tslot;   // D of even chunks: cols [0, V); odd chunks: [V, 2V)
  const uint32_t tS = tD0 + 2 * V;  // S master: cols [2V, 3V)

  auto issue = [&](int c) {  // thread 0: record of chunk c into stage c & 1
    const int s = c & 1;
    const unsigned char* r = recs + (size_t)c * p.rec_bytes;
    unsigned char* d = sm + s * STAGE;
    const unsigned ub = 64u * V * 2u;
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(&bars[s], 32768u + 8192u + 16384u + ub + 512u);
    bulk_g2s(d + ST_WQ, r + L.wq, 32768u, &bars[s]);
    bulk_g2s(d + ST_TA + 8192, r + L.aqk, 8192u, &bars[s]);
    bulk_g2s(d + ST_KD, r + L.kd, 16384u, &bars[s]);
    bulk_g2s(d + ST_U, r + L.u + (size_t)blockIdx.x * ub, ub, &bars[s]);
    bulk_g2s(d + ST_GL, r + L.gl, 512u, &bars[s]);
  };
  if (tid == 0) issue(0);

  // ---- initial state: f32 master in TMEM, bf16 image in smem ----
  const int kk = 32 * sp + lane;  // key channel = TMEM lane of this thread
  for (int c16 = 0; c16 < HALF / 16; ++c16) {
    const int col = col0 + 16 * c16;
    float v[16];
    const float4* src = reinterpret_cast<const float4*>(st + (size_t)kk * VF + col);
    #pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 f = src[j];
      v[4 * j] = f.x; v[4 * j + 1] = f.y; v[4 * j + 2] = f.z; v[4 * j + 3] = f.w;
    }
    umma::st16(umma::taddr(tS, 32 * sp, col), v);
    uint4 lo, hi;
    lo.x = umma::pack_bf16x2(v[0], v[1]); lo.y = umma::pack_bf16x2(v[2], v[3]);
    lo.z = umma::pack_bf16x2(v[4], v[5]); lo.w = umma::pack_bf16x2(v[6], v[7]);
    hi.x = umma::pack_bf16x2(v[8], v[9]); hi.y = umma::pack_bf16x2(v[10], v[11]);
    hi.z = umma::pack_bf16x2(v[12], v[13]); hi.w = umma::pack_bf16x2(v[14], v[15]);
    *reinterpret_cast<uint4*>(sm + S_IMG + umma::mnmaj_chunk(kk, col / 8, TC_K)) = lo;
    *reinterpret_cast<uint4*>(sm + S_IMG + umma::mnmaj_chunk(kk, col / 8 + 1, TC_K)) = hi;
  }
  umma::wait_st();
  fence_proxy_async_smem();
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();

  const uint32_t i1 = umma::idesc_bf16(128, V, false, true);  // [W;Qg] . S and [0;Aqk] . v_new
  const uint32_t i3 = umma::idesc_bf16(128, V, true, true);   // Kd^T . v_new

  // o rows of chunk c live in rows 64..127 of D[c & 1] (sub-partitions 2, 3);
  // their epilogue runs while the tensor core does MMA1 of chunk c + 1.
  uint4 graw[8];  // gate rows of the chunk whose epilogue runs next (sub-partitions 2, 3)
  const int orow = 32 * (sp - 2) + lane;
  auto load_gate = [&](int c) {
    const int t0 = c * TC_C;
    if (p.fuse_epilogue && orow < min(TC_C, p.T - t0)) {
      const __nv_bfloat16* gp = static_cast<const __nv_bfloat16*>(p.gate.p) + bb * p.gate.s0 + hv * p.gate.s1 +
                                (int64_t)(t0 + orow) * p.gate.s2 + cbase + col0;
      #pragma unroll
      for (int j = 0; j < 8; ++j)
        if (8 * j < HALF) graw[j] = reinterpret_cast<const uint4*>(gp)[j];
    }
  };
  auto epilogue = [&](int c) {
    const int t0 = c * TC_C;
    const int cv = min(TC_C, p.T - t0);
    const uint32_t tD = tD0 + (c & 1) * V;
    float ov[64];  // TMEM loads land straight in ov: registers are valid only after the wait
    #pragma unroll
    for (int c16 = 0; c16 < 4; ++c16)
      if (16 * c16 < HALF)
        umma::ld16(umma::taddr(tD, 32 * sp, col0 + 16 * c16), *reinterpret_cast<float(*)[16]>(ov + 16 * c16));
    umma::wait_ld();
    f32x2 s2[2] = {0ull, 0ull};  // four independent chains, as two pairs
    #pragma unroll
    for (int j = 0; j < 64; j += 2)
      if (j < HALF) {
        const f32x2 o2 = f2pk(ov[j], ov[j + 1]);
        s2[(j >> 1) & 1] = f2fma(o2, o2, s2[(j >> 1) & 1]);
      }
    float s4[4];
    f2un(s2[0], s4[0], s4[1]);
    f2un(s2[1], s4[2], s4[3]);
    const float ss = (s4[0] + s4[1]) + (s4[2] + s4[3]);
    sRms[orow * 2 + half] = ss;
    named_bar(1, 128);
    float tot = sRms[orow * 2] + sRms[orow * 2 + 1];
    if (xchg) {  // add the other slice's sum of this row (both halves of a row send the same value)
      const int par = c & 1;
      st_cluster_f32(cluster_addr(sXsum + par * 64 + orow, peer), tot);
      mbar_arrive_cluster(cluster_addr(&xbars[par], peer));
      mbar_wait_cluster_bounded(&xbars[par], (c >> 1) & 1);
      tot += sXsum[par * 64 + orow];
    }
    const float inv = rsqrtf(tot / (float)VF + p.eps);
    const f32x2 inv2 = f2pk(inv, inv);
    named_bar(1, 128);  // sRms reusable
    if (orow < cv) {
      __nv_bfloat16* op = static_cast<__nv_bfloat16*>(const_cast<void*>(p.out.p)) + bb * p.out.s0 + hv * p.out.s1 +
                          (int64_t)(t0 + orow) * p.out.s2 + cbase + col0;
      #pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (8 * j >= HALF) break;
        float y[8];
        if (p.fuse_epilogue) {
          // SiLU(g) = h + h tanh(h), h = g / 2, on bf16 pairs (the gate is bf16 and the product is rounded to
          // bf16): three packed ops per pair; the norm and the weight stay in f32.
          #pragma unroll
          for (int e2 = 0; e2 < 4; ++e2) {
            uint32_t hh, th, sl;
            const uint32_t g2 = reinterpret_cast<const uint32_t*>(&graw[j])[e2];
            asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(hh) : "r"(g2), "r"(0x3f003f00u));
            asm("tanh.approx.bf16x2 %0, %1;" : "=r"(th) : "r"(hh));
            asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(sl) : "r"(hh), "r"(th), "r"(hh));
            const f32x2 s01 = f2pk(__uint_as_float(sl << 16), __uint_as_float(sl & 0xffff0000u));
            const f32x2 w01 = *reinterpret_cast<const f32x2*>(sOnw + col0 + 8 * j + 2 * e2);
            const f32x2 o01 = f2pk(ov[8 * j + 2 * e2], ov[8 * j + 2 * e2 + 1]);
            f2un(f2mul(f2mul(f2mul(o01, inv2), w01), s01), y[2 * e2], y[2 * e2 + 1]);
          }
        } else {
          #pragma unroll
          for (int e = 0; e < 8; ++e) y[e] = ov[8 * j + e];
        }
        uint4 pk;
        pk.x = umma::pack_bf16x2(y[0], y[1]); pk.y = umma::pack_bf16x2(y[2], y[3]);
        pk.z = umma::pack_bf16x2(y[4], y[5]); pk.w = umma::pack_bf16x2(y[6], y[7]);
        reinterpret_cast<uint4*>(op)[j] = pk;
      }
    }
  };
  if (sp >= 2) load_gate(0);

  for (int c = 0; c < p.NC; ++c) {
    const int s = c & 1;
    const uint32_t tD = tD0 + s * V;
    unsigned char* stg = sm + s * STAGE;
    if (tid == 0 && c + 1 < p.NC) issue(c + 1);
    mbar_wait_bounded(&bars[s], (c >> 1) & 1);
    umma::fence_after_sync();

    // MMA1: D = [W; Qg] S
    if (tid == 0) {
      const uint64_t dwq = umma::desc_kmaj_base(sbase + s * STAGE + ST_WQ);
      const uint64_t dsi = umma::desc_mnmaj_base(sbase + S_IMG, TC_K);
      #pragma unroll
      for (int j = 0; j < 8; ++j)
        umma::mma_bf16(tD, umma::desc_kmaj_at(dwq, 128, j), umma::desc_mnmaj_at(dsi, j), i1, j > 0);
      umma::commit(&bars[2]);
    }
    // meanwhile: S <- diag(gamma_last) S in TMEM (all warps), then the
    // epilogue of the previous chunk (sub-partitions 2, 3)
    {
      const float gam = reinterpret_cast<const float*>(stg + ST_GL)[kk];
      for (int b32 = 0; b32 < HALF; b32 += 32) {
        float v[2][16];
        #pragma unroll
        for (int c16 = 0; c16 < 2; ++c16) umma::ld16(umma::taddr(tS, 32 * sp, col0 + b32 + 16 * c16), v[c16]);
        umma::wait_ld();
        #pragma unroll
        for (int c16 = 0; c16 < 2; ++c16) {
          #pragma unroll
          for (int j = 0; j < 16; ++j) v[c16][j] *= gam;
          umma::st16(umma::taddr(tS, 32 * sp, col0 + b32 + 16 * c16), v[c16]);
        }
      }
      umma::wait_st();
    }
    if (sp >= 2) {
      // rows 64..127 of S rescaled: this thread's part of the MMA3 operands is ready
      umma::fence_before_sync();
      mbar_arrive(&bars[4]);
      if (c > 0) {
        epilogue(c - 1);
        load_gate(c);  // lands while chunk c runs; used by its epilogue in chunk c + 1
      }
    } else {
      mbar_wait_bounded(&bars[2], c & 1);
      umma::fence_after_sync();
    }

    // v_new = U - W S  (rows 0..63 of D: sub-partitions 0, 1)
    if (sp < 2) {
      const int r = 32 * sp + lane;
      const uint4* urow = reinterpret_cast<const uint4*>(stg + ST_U + (size_t)r * V * 2);  // chunks swizzled by r & 7
      for (int b32 = 0; b32 < HALF; b32 += 32) {
        float v[2][16];
        #pragma unroll
        for (int c16 = 0; c16 < 2; ++c16) umma::ld16(umma::taddr(tD, 32 * sp, col0 + b32 + 16 * c16), v[c16]);
        umma::wait_ld();
        #pragma unroll
        for (int c16 = 0; c16 < 2; ++c16) {
          const int col = col0 + b32 + 16 * c16;
          const uint4 u0 = urow[(col / 8) ^ (r & 7)];
          const uint4 u1 = urow[(col / 8 + 1) ^ (r & 7)];
          const __nv_bfloat162* uh0 = reinterpret_cast<const __nv_bfloat162*>(&u0);
          const __nv_bfloat162* uh1 = reinterpret_cast<const __nv_bfloat162*>(&u1);
          float vn[16];
          #pragma unroll
          for (int j = 0; j < 4; ++j) {
            vn[2 * j] = __low2float(uh0[j]) - v[c16][2 * j];
            vn[2 * j + 1] = __high2float(uh0[j]) - v[c16][2 * j + 1];
            vn[8 + 2 * j] = __low2float(uh1[j]) - v[c16][8 + 2 * j];
            vn[8 + 2 * j + 1] = __high2float(uh1[j]) - v[c16][8 + 2 * j + 1];
          }
          uint4 lo, hi;
          lo.x = umma::pack_bf16x2(vn[0], vn[1]); lo.y = umma::pack_bf16x2(vn[2], vn[3]);
          lo.z = umma::pack_bf16x2(vn[4], vn[5]); lo.w = umma::pack_bf16x2(vn[6], vn[7]);
          hi.x = umma::pack_bf16x2(vn[8], vn[9]); hi.y = umma::pack_bf16x2(vn[10], vn[11]);
          hi.z = umma::pack_bf16x2(vn[12], vn[13]); hi.w = umma::pack_bf16x2(vn[14], vn[15]);
          *reinterpret_cast<uint4*>(sm + VN_IMG + umma::mnmaj_chunk(r, col / 8, TC_C)) = lo;
          *reinterpret_cast<uint4*>(sm + VN_IMG + umma::mnmaj_chunk(r, col / 8 + 1, TC_C)) = hi;
        }
      }
    }
    if (sp < 2) {
      fence_proxy_async_smem();
      umma::fence_before_sync();
      mbar_arrive(&bars[4]);
    }

    // MMA2: D += [0; Aqk] v_new ; MMA3: S += Kd^T v_new
    if (tid == 0) {
      mbar_wait_bounded(&bars[4], c & 1);
      umma::fence_after_sync();
      const uint64_t dta = umma::desc_kmaj_base(sbase + s * STAGE + ST_TA);
      const uint64_t dkd = umma::desc_mnmaj_base(sbase + s * STAGE + ST_KD, TC_C);
      const uint64_t dvn = umma::desc_mnmaj_base(sbase + VN_IMG, TC_C);
      #pragma unroll
      for (int j = 0; j < 4; ++j)
        umma::mma_bf16(tD, umma::desc_kmaj_at(dta, 128, j), umma::desc_mnmaj_at(dvn, j), i1, true);
      #pragma unroll
      for (int j = 0; j < 4; ++j)
        umma::mma_bf16(tS, umma::desc_mnmaj_at(dkd, j), umma::desc_mnmaj_at(dvn, j), i3, true);
      umma::commit(&bars[3]);
    }
    mbar_wait_bounded(&bars[3], c & 1);
    umma::fence_after_sync();

    // S (now S_{c+1}) -> bf16 image for the next chunk
    for (int b32 = 0; b32 < HALF; b32 += 32) {
      float v[2][16];
      #pragma unroll
      for (int c16 = 0; c16 < 2; ++c16) umma::ld16(umma::taddr(tS, 32 * sp, col0 + b32 + 16 * c16), v[c16]);
      umma::wait_ld();
      #pragma unroll
      for (int c16 = 0; c16 < 2; ++c16) {
        const int col = col0 + b32 + 16 * c16;
        uint4 lo, hi;
        lo.x = umma::pack_bf16x2(v[c16][0], v[c16][1]); lo.y = umma::pack_bf16x2(v[c16][2], v[c16][3]);
        lo.z = umma::pack_bf16x2(v[c16][4], v[c16][5]); lo.w = umma::pack_bf16x2(v[c16][6], v[c16][7]);
        hi.x = umma::pack_bf16x2(v[c16][8], v[c16][9]); hi.y = umma::pack_bf16x2(v[c16][10], v[c16][11]);
        hi.z = umma::pack_bf16x2(v[c16][12], v[c16][13]); hi.w = umma::pack_bf16x2(v[c16][14], v[c16][15]);
        *reinterpret_cast<uint4*>(sm + S_IMG + umma::mnmaj_chunk(kk, col / 8, TC_K)) = lo;
        *reinterpret_cast<uint4*>(sm + S_IMG + umma::mnmaj_chunk(kk, col / 8 + 1, TC_K)) = hi;
      }
    }
    fence_proxy_async_smem();
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
  }
  if (sp >= 2) epilogue(p.NC - 1);

  // ---- final state back to HBM (f32, in place) ----
  for (int c16 = 0; c16 < HALF / 16; ++c16) {
    const int col = col0 + 16 * c16;
    float v[16];
    umma::ld16(umma::taddr(tS, 32 * sp, col), v);
    umma::wait_ld();
    float4* dst = reinterpret_cast<float4*>(st + (size_t)kk * VF + col);
    #pragma unroll
    for (int j = 0; j < 4; ++j) dst[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  }
  umma::fence_before_sync();
  __syncthreads();
  if (xchg) cluster_sync_all();  // no CTA leaves while its peer may still reach its shared memory
  if (warp == 0) umma::tmem_dealloc(tD0, 512);
}

int launch_inter_tc(const TcParams& p, cudaStream_t st) {
  const size_t smem = inter_smem::TOTAL + 1024;
  const bool xchg = p.vsplit > 1 && p.fuse_epilogue;  // the slices of a chain exchange row sums: one cluster per chain
  void (*fn)(const TcParams) = xchg ? k_inter_tc<true> : k_inter_tc<false>;
  cudaError_t e = cudaFuncSetAttribute((const void*)fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return check_cuda(e, "chunk inter (tc) smem attribute");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.vsplit, p.HV, p.B);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  if (xchg) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = p.vsplit;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return check_cuda(cudaLaunchKernelEx(&cfg, fn, p), "chunk inter (tc) launch");
}

bool tc_supported(int K, int V, int C, int dtype) {
  return dtype == GDN2_DTYPE_BF16 && K == TC_K && C == TC_C && (V == 64 || V == 128 || V == 256);
}

GDN2_DEVICE_ERROR_READER(read_device_errors_inter_tc)

}  // namespace gdn2
