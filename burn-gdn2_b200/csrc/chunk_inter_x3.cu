// Kernel (2), split-operand form: chunk-inter for bf16 or f32 inputs,
// K = 128, C = 64, V in {64, 128, 256}, with the SiLU-gated RMS-norm epilogue
// fused, f32-grade intermediates (chunk_x3.cuh).
//
// Replaces gdn2_chunk_inter_kernel (src/kernel/chunk_cube.rs:300-610); math
// of src/forward.rs:263-274 with the epilogue of src/module.rs:501-517.
// One CTA (8 warps, one per SM) per (value-column slice, value head, batch)
// walks the chunks in order; V <= 128 is one slice, V = 256 two slices of
// 128 columns (the value columns of the recurrence are independent), whose
// CTAs form a 2-CTA cluster that exchanges the RMS norm's row sums through
// distributed shared memory.  The state S [K][V] stays in TMEM in f32 for the whole sequence;
// its hi and lo bf16 images in shared memory are the MMA operands.  Per
// chunk (every product as three MMAs: hi.hi + lo.hi + hi.lo):
//   MMA1  D = [W; Qg] S                      (M=128, N=V, K=128)
//   v_new = U - (W S)                        (rows 0..63 of D; U read from
//                                             the record into registers)
//   MMA2  D += [*; Aqk] v_new                (rows 64..127 become o; rows
//                                             0..63 are dead and take
//                                             whatever the 8 KB in front of
//                                             the Aqk image hold)
//   MMA3  S = diag(gamma_last) S + Kd^T v_new   (S pre-scaled in TMEM)
//   o -> gated RMS norm -> out; S -> hi / lo images for the next chunk.
// The record parts sit in one stage and are refilled as soon as they are
// consumed: [W; Qg] (and gamma_last) once MMA1 completed, Aqk and Kd once
// MMA2 and MMA3 completed, so each copy has the rest of a chunk to land.
// MMA3 (the recurrence) is issued and committed before MMA2 (the o rows),
// and the decay of the next chunk is applied to the TMEM master in the same
// pass that writes the next S images, so the chain from one chunk's MMA1 to
// the next runs MMA1 -> v_new -> MMA3 -> S images only.
#include "chunk_x3.cuh"

namespace gdn2 {

namespace nx3 {
constexpr uint32_t WQ = 0;          // WQ_HI, WQ_LO: K-major [128][128] each (the record's first 64 KB)
constexpr uint32_t AQK = 65536;     // AQK_HI, AQK_LO [64][64], KD_HI, KD_LO MN-major [64][128]: 48 KB
constexpr uint32_t AQK_LO = AQK + 8192;
constexpr uint32_t KD_HI = AQK + 16384;
constexpr uint32_t KD_LO = AQK + 32768;
constexpr uint32_t GL = 114688;     // f32 [2][128], by chunk parity
constexpr uint32_t S_HI = 115712;   // MN-major [128][V]
constexpr uint32_t S_LO = S_HI + 32768;
constexpr uint32_t VN_HI = S_LO + 32768;  // MN-major [64][V]
constexpr uint32_t VN_LO = VN_HI + 16384;
constexpr uint32_t RMS = VN_LO + 16384;   // f32 [64][2]
constexpr uint32_t ONW = RMS + 512;       // f32 [V]
constexpr uint32_t BARS = ONW + 512;
constexpr uint32_t XSUM = BARS + 128;   // f32 [2][64]: the peer slice's row sums, by chunk parity (V = 256)
constexpr uint32_t XBARS = XSUM + 512;  // 2 mbarriers: the peer's 128 epilogue threads arrived, by chunk parity
constexpr uint32_t TOTAL = XBARS + 64;
}  // namespace nx3

__device__ __forceinline__ void named_bar_x3(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// SiLU in f32: g sigma(g) with the MUFU exponential and a fast divide (a few ulp)
__device__ __forceinline__ float silu_acc(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

// XCHG: a chain as two CTAs of V / 2 columns (a 2-CTA cluster: V = 256, or V = 128 with few chains) that
// exchange the RMS norm's row sums; a separate instantiation keeps the one-slice kernel free of that code.
// PHA: scan phase A (segment end states from zero and segment transitions, no output); its own instantiation
// keeps the transition slice's branches out of the output kernels.
template <typename TIN, bool XCHG, bool PHA>
__global__ void __launch_bounds__(256, 1) k_inter_x3(const TcParams p) {
  using namespace nx3;
  extern __shared__ __align__(1024) unsigned char smraw[];
  unsigned char* sm = smraw + ((1024u - (smem_u32(smraw) & 1023u)) & 1023u);
  float* sRms = reinterpret_cast<float*>(sm + RMS);
  float* sOnw = reinterpret_cast<float*>(sm + ONW);
  const float* sGl = reinterpret_cast<const float*>(sm + GL);
  // fullA (W, Qg, gamma_last), fullB (Aqk, Kd), mma1, mma3 (the state update), operands ready, mma2 (o rows)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + BARS);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 6);

  float* sXsum = reinterpret_cast<float*>(sm + XSUM);
  uint64_t* xbars = reinterpret_cast<uint64_t*>(sm + XBARS);

  // blockIdx.z = (batch entry, segment of the chain); blockIdx.x = column slice.  Scan phase A: slices
  // 0 .. VF / V - 1 carry the state's value columns (from a zero start, U from the record), slice VF / V the
  // segment's transition (K columns from the identity, U = 0); no output.
  constexpr bool scanA = PHA;
  const int zseg = scanA ? p.nseg - 1 : p.nseg;  // segments in the grid: phase A skips the last one
  const int hv = blockIdx.y, seg = blockIdx.z % zseg, bb = blockIdx.z / zseg;
  const int V = p.vt, HALF = V / 2;  // columns of this CTA's slice
  const int VF = p.V;                // full row width
  const bool tslice = scanA && (int)blockIdx.x * V >= VF;          // the transition slice (phase A)
  const int cbase = tslice ? (int)blockIdx.x * V - VF : (int)blockIdx.x * V;  // first column of the slice
  const uint32_t peer = blockIdx.x ^ 1u;  // cluster rank of the other slice's CTA (XCHG)
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int sp = warp & 3, half = warp >> 2;
  const int col0 = half * HALF;
  const X3Record L = x3_record_layout(VF);
  const size_t chain = (size_t)bb * p.HV + hv;
  const int c0 = seg * p.seg_len;                  // first chunk of this segment
  const int NCL = min(p.NC, c0 + p.seg_len) - c0;  // its chunks
  const unsigned char* recs = p.rec + (chain * p.NC + c0) * p.rec_bytes;
  // start state (null: zero, or the identity for a transition slice) and where the end state goes (null:
  // nowhere), rows of srow floats
  const float* st_in;
  float* st_out;
  int srow = VF;
  if (scanA) {
    st_in = nullptr;
    if (tslice) {
      srow = TC_K;
      st_out = p.seg_trans + (chain * (p.nseg - 1) + seg) * TC_K * TC_K + cbase;
    } else {
      st_out = p.seg_state + (chain * p.nseg + seg + 1) * TC_K * VF + cbase;  // N_seg, in slot seg + 1
    }
  } else if (p.nseg == 1) {
    st_in = st_out = p.state + chain * TC_K * VF + cbase;
  } else {
    st_in = p.seg_state + (chain * p.nseg + seg) * TC_K * VF + cbase;
    st_out = seg == p.nseg - 1 ? p.state + chain * TC_K * VF + cbase : nullptr;
  }
  const uint32_t sbase = smem_u32(sm);

  if (warp == 0) {
    umma::tmem_alloc(tslot, 512);
    umma::tmem_relinquish();
  }
  if (p.fuse_epilogue && !scanA)
    for (int i = tid; i < V; i += 256) sOnw[i] = p.onw[cbase + i];
  if (tid == 0) {
    for (int i = 0; i < 4; ++i) mbar_init(&bars[i], 1);
    mbar_init(&bars[4], 256);
    mbar_init(&bars[5], 1);
    mbar_init(&xbars[0], 128);
    mbar_init(&xbars[1], 128);
    fence_mbar_init();
  }
  umma::fence_before_sync();
  __syncthreads();
  if (XCHG) cluster_sync_all();  // the peer's exchange barriers are initialised before anyone arrives on them
  umma::fence_after_sync();
  const uint32_t tD0 = *tslot;       // D of even chunks: cols [0, V); odd chunks: [V, 2V)
  const uint32_t tS = tD0 + 2 * V;   // S master: cols [2V, 3V)

  // a record is read once (evict-first), or by both CTAs of a cluster at about the same time
  const uint64_t pol_rec = gridDim.x == 1 ? l2_policy_evict_first() : l2_policy_evict_normal();
  auto issueA = [&](int c) {  // thread 0: [W; Qg] hi / lo and gamma_last of chunk c
    const unsigned char* r = recs + (size_t)c * p.rec_bytes;
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(&bars[0], 65536u + 512u);
    bulk_g2s_hint(sm + WQ, r + L.wq_hi, 65536u, &bars[0], pol_rec);
    bulk_g2s_hint(sm + GL + (c & 1) * 512, r + L.gl, 512u, &bars[0], pol_rec);
  };
  auto issueB = [&](int c) {  // thread 0: Aqk and Kd hi / lo of chunk c
    const unsigned char* r = recs + (size_t)c * p.rec_bytes;
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(&bars[1], 49152u);
    bulk_g2s_hint(sm + AQK, r + L.aqk_hi, 49152u, &bars[1], pol_rec);
  };
  // records two chunks ahead are pulled into L2 (one bulk prefetch per chunk), so the stage refills, issued
  // as soon as a part is consumed, read from L2
  auto prefetch_rec = [&](int c) {
    if (c < NCL) bulk_prefetch_l2(recs + (size_t)c * p.rec_bytes, (unsigned)L.bytes);
  };
  if (tid == 0) {
    issueA(0);
    issueB(0);
    prefetch_rec(1);
  }

  // ---- initial state: hi / lo images of S in smem, f32 master diag(gamma_last) S in TMEM (the decay that
  // MMA3 of chunk 0 accumulates onto; every later rescale rides on the S-image pass of the chunk before) ----
  const int kk = 32 * sp + lane;  // key channel = TMEM lane of this thread
  mbar_wait_bounded(&bars[0], 0);
  const float gam0 = sGl[kk];
  for (int c16 = 0; c16 < HALF / 16; ++c16) {
    const int col = col0 + 16 * c16;
    float v[16];
    if (st_in) {
      const float4* src = reinterpret_cast<const float4*>(st_in + (size_t)kk * srow + col);
      #pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 f = src[j];
        v[4 * j] = f.x; v[4 * j + 1] = f.y; v[4 * j + 2] = f.z; v[4 * j + 3] = f.w;
      }
    } else {  // zero, or the identity (row kk of the transition: 1 in column kk)
      #pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = (tslice && cbase + col + j == kk) ? 1.f : 0.f;
    }
    uint4 h0, l0, h1, l1;
    split8(v, h0, l0);
    split8(v + 8, h1, l1);
    const uint32_t o0 = umma::mnmaj_chunk(kk, col / 8, TC_K), o1 = umma::mnmaj_chunk(kk, col / 8 + 1, TC_K);
    *reinterpret_cast<uint4*>(sm + S_HI + o0) = h0;
    *reinterpret_cast<uint4*>(sm + S_HI + o1) = h1;
    *reinterpret_cast<uint4*>(sm + S_LO + o0) = l0;
    *reinterpret_cast<uint4*>(sm + S_LO + o1) = l1;
    #pragma unroll
    for (int j = 0; j < 16; ++j) v[j] *= gam0;
    umma::st16(umma::taddr(tS, 32 * sp, col), v);
  }
  umma::wait_st();
  fence_proxy_async_smem();
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();

  const uint32_t i1 = umma::idesc_bf16(128, V, false, true);  // [W;Qg] . S and [*;Aqk] . v_new
  const uint32_t i3 = umma::idesc_bf16(128, V, true, true);   // Kd^T . v_new

  // U row of this thread (sub-partitions 0, 1: row 32 sp + lane, this half's columns of this CTA's slice; the
  // record keeps U slice by slice) in the record of chunk c; prefetched to L2 one chunk ahead, read into
  // registers while MMA1 runs
  // U slice of this CTA (cbase / 128; rows of min(VF, 128) floats), first column of this half in it
  const int uc = cbase % 128 + col0;
  const unsigned char* const urow0 =
      recs + L.u + ((size_t)(cbase / 128) * 64 + 32 * sp + lane) * (VF < 128 ? VF : 128) * 4;
  auto u_row = [&](int c) {  // the row's start; word k of the row is at k ^ (row & 7)
    return reinterpret_cast<const float4*>(urow0 + (size_t)c * p.rec_bytes);
  };
  auto prefetch_u = [&](int c) {
    const char* g = reinterpret_cast<const char*>(u_row(c)) + uc * 4;
    for (int b = 0; b < HALF * 4; b += 128) asm volatile("prefetch.global.L2 [%0];" ::"l"(g + b));
  };

  // o rows of chunk c live in rows 64..127 of D[c & 1] (sub-partitions 2, 3); their epilogue runs during
  // chunk c + 1, once MMA2 of chunk c completed.  The gate rows of chunk c are read into registers during
  // chunk c (after the previous epilogue), prefetched to L2 a chunk earlier.
  constexpr int GW = 64 * (int)sizeof(TIN) / 16;  // 16-byte gate words per row half
  const int orow = 32 * (sp - 2) + lane;
  auto gate_row = [&](int c) {
    return reinterpret_cast<const uint4*>(static_cast<const TIN*>(p.gate.p) + bb * p.gate.s0 + hv * p.gate.s1 +
                                          (int64_t)((c0 + c) * TC_C + orow) * p.gate.s2 + cbase + col0);
  };
  auto prefetch_gate = [&](int c) {
    if (p.fuse_epilogue && c < NCL && orow < min(TC_C, p.T - (c0 + c) * TC_C)) {
      const char* g = reinterpret_cast<const char*>(gate_row(c));
      for (int b = 0; b < HALF * (int)sizeof(TIN); b += 128) asm volatile("prefetch.global.L2 [%0];" ::"l"(g + b));
    }
  };
  uint4 graw[GW];
  auto load_gate = [&](int c) {
    if (p.fuse_epilogue && orow < min(TC_C, p.T - (c0 + c) * TC_C)) {
      const uint4* gp = gate_row(c);
      #pragma unroll
      for (int j = 0; j < GW; ++j)
        if (j * 16 < HALF * (int)sizeof(TIN)) graw[j] = gp[j];
    }
  };
  auto gate_at = [&](int j) -> float {  // gate element j of this row half
    if constexpr (sizeof(TIN) == 2) {
      const uint32_t w32 = reinterpret_cast<const uint32_t*>(graw)[j >> 1];
      return __uint_as_float((j & 1) ? (w32 & 0xffff0000u) : (w32 << 16));
    } else {
      return reinterpret_cast<const float*>(graw)[j];
    }
  };
  auto epilogue = [&](int c) {
    const int t0 = (c0 + c) * TC_C;
    const int cv = min(TC_C, p.T - t0);
    const uint32_t tD = tD0 + (c & 1) * V;
    // MMA2 of chunk c has completed: thread 0 waited for it before the barrier that closed chunk c.  The o row
    // is read from TMEM twice, 16 columns at a time (sum of squares, then the scaled output), so that no
    // 64-float copy of it is live next to the gate row.
    float inv = 1.f;
    if (p.fuse_epilogue) {
      f32x2 s2[2] = {0ull, 0ull};
      #pragma unroll
      for (int c16 = 0; c16 < 4; ++c16) {
        if (16 * c16 >= HALF) break;
        float ov[16];
        umma::ld16(umma::taddr(tD, 32 * sp, col0 + 16 * c16), ov);
        umma::wait_ld();
        #pragma unroll
        for (int j = 0; j < 16; j += 2) {
          const f32x2 o2 = f2pk(ov[j], ov[j + 1]);
          s2[(j >> 1) & 1] = f2fma(o2, o2, s2[(j >> 1) & 1]);
        }
      }
      float s4[4];
      f2un(s2[0], s4[0], s4[1]);
      f2un(s2[1], s4[2], s4[3]);
      sRms[orow * 2 + half] = (s4[0] + s4[1]) + (s4[2] + s4[3]);
      named_bar_x3(1, 128);
      float tot = sRms[orow * 2] + sRms[orow * 2 + 1];
      if (XCHG) {  // add the other slice's sum of this row (both halves of a row send the same value)
        const int par = c & 1;
        st_cluster_f32(cluster_addr(sXsum + par * 64 + orow, peer), tot);
        mbar_arrive_cluster(cluster_addr(&xbars[par], peer));
        mbar_wait_cluster_bounded(&xbars[par], (c >> 1) & 1);
        tot += sXsum[par * 64 + orow];
      }
      inv = rsqrtf(tot / (float)VF + p.eps);
      named_bar_x3(1, 128);  // sRms reusable
    }
    TIN* op = static_cast<TIN*>(const_cast<void*>(p.out.p)) + bb * p.out.s0 + hv * p.out.s1 +
              (int64_t)(t0 + orow) * p.out.s2 + cbase + col0;
    #pragma unroll
    for (int c16 = 0; c16 < 4; ++c16) {
      if (16 * c16 >= HALF) break;
      float ov[16];
      umma::ld16(umma::taddr(tD, 32 * sp, col0 + 16 * c16), ov);  // warp-wide: before the row guard
      umma::wait_ld();
      if (orow < cv) {
        #pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int j = 2 * c16 + h;
          float y[8];
          #pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int cc = 8 * j + e;
            y[e] = p.fuse_epilogue ? ov[8 * h + e] * inv * sOnw[col0 + cc] * silu_acc(gate_at(cc)) : ov[8 * h + e];
          }
          if constexpr (sizeof(TIN) == 2) {
            uint4 pk;
            pk.x = umma::pack_bf16x2(y[0], y[1]); pk.y = umma::pack_bf16x2(y[2], y[3]);
            pk.z = umma::pack_bf16x2(y[4], y[5]); pk.w = umma::pack_bf16x2(y[6], y[7]);
            reinterpret_cast<uint4*>(op)[j] = pk;
          } else {
            reinterpret_cast<float4*>(op)[2 * j] = make_float4(y[0], y[1], y[2], y[3]);
            reinterpret_cast<float4*>(op)[2 * j + 1] = make_float4(y[4], y[5], y[6], y[7]);
          }
        }
      }
    }
  };
  if (sp >= 2) {
    if (!scanA) {
      load_gate(0);
      prefetch_gate(1);
    }
  } else if (!tslice) {
    prefetch_u(0);
  }

  // Every mbarrier wait below is on a phase that cannot be overtaken by the next one before the waiting thread
  // passes the barrier closing the chunk (each next phase needs work issued after that barrier), so the
  // parity waits are unambiguous; only thread 0 waits for the [W; Qg] copy of the chunk it starts.
  for (int c = 0; c < NCL; ++c) {
    const uint32_t tD = tD0 + (c & 1) * V;

    // MMA1: D = [W; Qg] S  (the master already holds diag(gamma_last) S for MMA3)
    if (tid == 0) {
      mbar_wait_bounded(&bars[0], c & 1);  // [W; Qg] and gamma_last of chunk c
      umma::fence_after_sync();
      prefetch_rec(c + 2);
      const uint64_t dsh = umma::desc_mnmaj_base(sbase + S_HI, TC_K), dsl = umma::desc_mnmaj_base(sbase + S_LO, TC_K);
      const uint64_t dwh = umma::desc_kmaj_base(sbase + WQ), dwl = umma::desc_kmaj_base(sbase + WQ + 32768);
      #pragma unroll 1
      for (int pass = 0; pass < 3; ++pass) {
        const uint64_t da = pass == 1 ? dwl : dwh, db = pass == 2 ? dsl : dsh;
        #pragma unroll
        for (int j = 0; j < 8; ++j)
          umma::mma_bf16(tD, umma::desc_kmaj_at(da, 128, j), umma::desc_mnmaj_at(db, j), i1, pass > 0 || j > 0);
      }
      umma::commit(&bars[2]);
    }
    if (sp >= 2) {
      // the epilogue of the previous chunk while the tensor core does MMA1, then the next gate rows
      mbar_arrive(&bars[4]);
      if (!scanA) {
        if (c > 0) epilogue(c - 1);
        load_gate(c);
        prefetch_gate(c + 1);
      }
    } else {
      float u[64];  // U rows of this chunk: read while MMA1 runs (zero for a transition slice)
      if (tslice) {
        #pragma unroll
        for (int j = 0; j < 64; ++j) u[j] = 0.f;
      } else {
        const float4* src = u_row(c);
        const int sw = lane & 7;  // = row & 7
        #pragma unroll
        for (int j = 0; j < 16; ++j)
          if (4 * j < HALF) {
            float4 f;
            asm("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];"
                : "=f"(f.x), "=f"(f.y), "=f"(f.z), "=f"(f.w)
                : "l"(src + ((uc / 4 + j) ^ sw)));
            u[4 * j] = f.x; u[4 * j + 1] = f.y; u[4 * j + 2] = f.z; u[4 * j + 3] = f.w;
          }
      }
      mbar_wait_bounded(&bars[2], c & 1);
      umma::fence_after_sync();
      if (tid == 0 && c + 1 < NCL) issueA(c + 1);  // MMA1 has read [W; Qg]; gamma_last goes to the other slot
      // v_new = U - W S (rows 0..63 of D) -> hi / lo images
      const int r = 32 * sp + lane;
      #pragma unroll
      for (int b32 = 0; b32 < 64; b32 += 32) {
        if (b32 >= HALF) break;
        float v[2][16];
        #pragma unroll
        for (int c16 = 0; c16 < 2; ++c16) umma::ld16(umma::taddr(tD, 32 * sp, col0 + b32 + 16 * c16), v[c16]);
        umma::wait_ld();
        #pragma unroll
        for (int c16 = 0; c16 < 2; ++c16) {
          const int col = col0 + b32 + 16 * c16;
          float vn[16];
          #pragma unroll
          for (int j = 0; j < 16; ++j) vn[j] = u[b32 + 16 * c16 + j] - v[c16][j];
          uint4 h0, l0, h1, l1;
          split8(vn, h0, l0);
          split8(vn + 8, h1, l1);
          const uint32_t o0 = umma::mnmaj_chunk(r, col / 8, TC_C), o1 = umma::mnmaj_chunk(r, col / 8 + 1, TC_C);
          *reinterpret_cast<uint4*>(sm + VN_HI + o0) = h0;
          *reinterpret_cast<uint4*>(sm + VN_HI + o1) = h1;
          *reinterpret_cast<uint4*>(sm + VN_LO + o0) = l0;
          *reinterpret_cast<uint4*>(sm + VN_LO + o1) = l1;
        }
      }
      fence_proxy_async_smem();
      umma::fence_before_sync();
      mbar_arrive(&bars[4]);
      if (c + 1 < NCL && !tslice) prefetch_u(c + 1);
    }

    // MMA3: S += Kd^T v_new (the recurrence: committed on its own), then MMA2: D += [*; Aqk] v_new (the o rows)
    if (tid == 0) {
      mbar_wait_bounded(&bars[4], c & 1);
      mbar_wait_bounded(&bars[1], c & 1);
      umma::fence_after_sync();
      const uint64_t dvh = umma::desc_mnmaj_base(sbase + VN_HI, TC_C), dvl = umma::desc_mnmaj_base(sbase + VN_LO, TC_C);
      const uint64_t dth = umma::desc_kmaj_base(sbase + AQK - 8192), dtl = umma::desc_kmaj_base(sbase + AQK_LO - 8192);
      const uint64_t dkh = umma::desc_mnmaj_base(sbase + KD_HI, TC_C), dkl = umma::desc_mnmaj_base(sbase + KD_LO, TC_C);
      #pragma unroll 1
      for (int pass = 0; pass < 3; ++pass) {
        const uint64_t da = pass == 1 ? dkl : dkh, db = pass == 2 ? dvl : dvh;
        #pragma unroll
        for (int j = 0; j < 4; ++j)
          umma::mma_bf16(tS, umma::desc_mnmaj_at(da, j), umma::desc_mnmaj_at(db, j), i3, true);
      }
      umma::commit(&bars[3]);
      if (!scanA) {
        #pragma unroll 1
        for (int pass = 0; pass < 3; ++pass) {
          const uint64_t da = pass == 1 ? dtl : dth, db = pass == 2 ? dvl : dvh;
          #pragma unroll
          for (int j = 0; j < 4; ++j)
            umma::mma_bf16(tD, umma::desc_kmaj_at(da, 128, j), umma::desc_mnmaj_at(db, j), i1, true);
        }
        umma::commit(&bars[5]);
      }
    }
    mbar_wait_bounded(&bars[3], c & 1);
    umma::fence_after_sync();

    // S_{c+1} -> hi / lo images for MMA1 of the next chunk, and the master rescaled by that chunk's gamma_last
    const bool more = c + 1 < NCL;
    float gam = 1.f;
    if (more) {
      mbar_wait_bounded(&bars[0], (c + 1) & 1);  // gamma_last of chunk c + 1 (issued with its [W; Qg])
      gam = sGl[((c + 1) & 1) * 128 + kk];
    }
    for (int b32 = 0; b32 < HALF; b32 += 32) {
      float v[2][16];
      #pragma unroll
      for (int c16 = 0; c16 < 2; ++c16) umma::ld16(umma::taddr(tS, 32 * sp, col0 + b32 + 16 * c16), v[c16]);
      umma::wait_ld();
      #pragma unroll
      for (int c16 = 0; c16 < 2; ++c16) {
        const int col = col0 + b32 + 16 * c16;
        uint4 h0, l0, h1, l1;
        split8(v[c16], h0, l0);
        split8(v[c16] + 8, h1, l1);
        const uint32_t o0 = umma::mnmaj_chunk(kk, col / 8, TC_K), o1 = umma::mnmaj_chunk(kk, col / 8 + 1, TC_K);
        *reinterpret_cast<uint4*>(sm + S_HI + o0) = h0;
        *reinterpret_cast<uint4*>(sm + S_HI + o1) = h1;
        *reinterpret_cast<uint4*>(sm + S_LO + o0) = l0;
        *reinterpret_cast<uint4*>(sm + S_LO + o1) = l1;
        if (more) {
          #pragma unroll
          for (int j = 0; j < 16; ++j) v[c16][j] *= gam;
          umma::st16(umma::taddr(tS, 32 * sp, col0 + b32 + 16 * c16), v[c16]);
        }
      }
    }
    if (more) umma::wait_st();
    if (tid == 0) {
      if (!scanA) mbar_wait_bounded(&bars[5], c & 1);  // MMA2 has read Aqk (MMA3 read Kd before it)
      if (more) issueB(c + 1);
    }
    fence_proxy_async_smem();
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
  }
  if (sp >= 2 && !scanA) epilogue(NCL - 1);

  // ---- end state back to HBM (f32: in place, or the segment's slot) ----
  if (st_out) {
    for (int c16 = 0; c16 < HALF / 16; ++c16) {
      const int col = col0 + 16 * c16;
      float v[16];
      umma::ld16(umma::taddr(tS, 32 * sp, col), v);
      umma::wait_ld();
      float4* dst = reinterpret_cast<float4*>(st_out + (size_t)kk * srow + col);
      #pragma unroll
      for (int j = 0; j < 4; ++j) dst[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    }
  }
  umma::fence_before_sync();
  __syncthreads();
  if (XCHG) cluster_sync_all();  // no CTA leaves while its peer may still reach its shared memory
  if (warp == 0) umma::tmem_dealloc(tD0, 512);
}

// Scan phase B: the start state of every segment, in order, for one 32-column block of one chain:
// slot 0 = the initial state, slot s + 1 = M_s slot s + N_s (N_s is in slot s + 1 already; updated in place).
// f32 on the CUDA cores: M_s (row stride 129: conflict-free column walks) and the column block in shared
// memory; thread t owns row t / 2 and 16 columns.
__global__ void __launch_bounds__(256) k_scan_combine_x3(const TcParams p) {
  extern __shared__ __align__(16) float smf[];
  float* sM = smf;                 // [128][129]
  float* sS = smf + TC_K * 129;    // [128][32]
  const int VF = p.V, cb = blockIdx.x * 32, tid = threadIdx.x;
  const size_t chain = (size_t)blockIdx.z * p.HV + blockIdx.y;
  float* slots = p.seg_state + chain * p.nseg * TC_K * VF + cb;
  const float* st0 = p.state + chain * TC_K * VF + cb;
  for (int i = tid; i < TC_K * 8; i += 256) {  // float4 (row i / 8, columns 4 (i % 8) ..)
    const int r = i >> 3, c4 = (i & 7) * 4;
    const float4 v = *reinterpret_cast<const float4*>(st0 + (size_t)r * VF + c4);
    *reinterpret_cast<float4*>(sS + r * 32 + c4) = v;
    *reinterpret_cast<float4*>(slots + (size_t)r * VF + c4) = v;
  }
  const int r = tid >> 1, cq = (tid & 1) * 16;
  for (int sg = 0; sg + 1 < p.nseg; ++sg) {
    const float* M = p.seg_trans + (chain * (p.nseg - 1) + sg) * TC_K * TC_K;
    for (int i = tid; i < TC_K * TC_K / 4; i += 256) {
      const float4 v = reinterpret_cast<const float4*>(M)[i];
      const int rr = (4 * i) / TC_K, cc = (4 * i) % TC_K;
      float* d = sM + rr * 129 + cc;
      d[0] = v.x; d[1] = v.y; d[2] = v.z; d[3] = v.w;
    }
    float* nxt = slots + (size_t)(sg + 1) * TC_K * VF + (size_t)r * VF + cq;
    float acc[16];
    #pragma unroll
    for (int j = 0; j < 16; j += 4) {
      const float4 v = *reinterpret_cast<const float4*>(nxt + j);
      acc[j] = v.x; acc[j + 1] = v.y; acc[j + 2] = v.z; acc[j + 3] = v.w;
    }
    __syncthreads();  // sM and sS complete
    #pragma unroll 4
    for (int k = 0; k < TC_K; ++k) {
      const float m = sM[r * 129 + k];
      const float4* srow = reinterpret_cast<const float4*>(sS + k * 32 + cq);
      #pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 x = srow[j];
        acc[4 * j] = fmaf(m, x.x, acc[4 * j]);
        acc[4 * j + 1] = fmaf(m, x.y, acc[4 * j + 1]);
        acc[4 * j + 2] = fmaf(m, x.z, acc[4 * j + 2]);
        acc[4 * j + 3] = fmaf(m, x.w, acc[4 * j + 3]);
      }
    }
    __syncthreads();  // every read of sS and sM done
    #pragma unroll
    for (int j = 0; j < 16; j += 4) {
      const float4 v = make_float4(acc[j], acc[j + 1], acc[j + 2], acc[j + 3]);
      *reinterpret_cast<float4*>(sS + r * 32 + cq + j) = v;
      *reinterpret_cast<float4*>(nxt + j) = v;
    }
  }
}

// Fewer chains (times segments) than half the SMs: each chain's 128 value columns are split over two CTAs
// of 64 (a 2-CTA cluster, as for V = 256), which halves the per-chunk work on a chain's critical path.
static TcParams inter_x3_split(const TcParams& p, int sms) {
  TcParams q = p;
  if (p.V == 128 && 2LL * p.B * p.HV * p.nseg <= sms) {
    q.vt = 64;
    q.vsplit = 2;
  }
  return q;
}

template <typename TIN>
static int launch_inter_x3_t(const TcParams& p0, cudaStream_t st) {
  const int sms = usable_sms();  // less the SMs the host reserved for its own work
  const size_t smem = nx3::TOTAL + 1024;
  for (void (*f)(const TcParams) : {k_inter_x3<TIN, true, false>, k_inter_x3<TIN, false, false>,
                                     k_inter_x3<TIN, false, true>}) {
    const cudaError_t e = cudaFuncSetAttribute((const void*)f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return check_cuda(e, "chunk inter (x3) smem attribute");
  }
  auto launch = [&](const TcParams& p, int slices, int zseg, bool xchg, bool pha) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(slices, p.HV, p.B * zseg);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    if (xchg) {
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = slices;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
    }
    void (*fn)(const TcParams) =
        pha ? k_inter_x3<TIN, false, true> : xchg ? k_inter_x3<TIN, true, false> : k_inter_x3<TIN, false, false>;
    return check_cuda(cudaLaunchKernelEx(&cfg, fn, p), "chunk inter (x3) launch");
  };
  if (p0.nseg > 1) {
    // phase A: (N, M) of segments 0 .. nseg - 2, one CTA per 128-column slice of the state and one for the
    // transition (no cluster: no output)
    TcParams a = p0;
    a.vt = 128;
    int rc = launch(a, p0.V / 128 + 1, p0.nseg - 1, false, true);
    if (rc) return rc;
    // phase B
    const size_t bsmem = (TC_K * 129 + TC_K * 32) * sizeof(float);
    cudaError_t e = cudaFuncSetAttribute((const void*)k_scan_combine_x3, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)bsmem);
    if (e != cudaSuccess) return check_cuda(e, "chunk scan (x3) smem attribute");
    k_scan_combine_x3<<<dim3(p0.V / 32, p0.HV, p0.B), 256, bsmem, st>>>(p0);
    rc = check_cuda(cudaGetLastError(), "chunk scan (x3) launch");
    if (rc) return rc;
  }
  // phase C (or the whole chain when nseg = 1)
  const TcParams p = inter_x3_split(p0, sms);
  return launch(p, p.vsplit, p.nseg, p.vsplit > 1 && p.fuse_epilogue, false);
}

int launch_inter_x3(const TcParams& p, int dtype, cudaStream_t st) {
  return dtype == GDN2_DTYPE_BF16 ? launch_inter_x3_t<__nv_bfloat16>(p, st) : launch_inter_x3_t<float>(p, st);
}

GDN2_DEVICE_ERROR_READER(read_device_errors_inter_x3)

}  // namespace gdn2
