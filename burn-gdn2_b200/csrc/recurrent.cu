// Kernel (3): fused-recurrent GDN-2 forward / decode step.
//
// Replaces gdn2_step_kernel + cuda::fused_step
// (src/kernel/fused_recurrent_cube.rs:15-57, :108-172) and the tensor-op
// token loop fused_recurrent_forward (src/kernel/fused_recurrent.rs:11-56).
//
// One CTA owns the state slice S[b, hv, :, col0:col0+VT] for the whole
// call: it is brought from HBM into shared memory once by bulk (TMA) copies
// issued at kernel entry, so the load overlaps the prologue; it stays on
// chip across all T tokens and the last token's update writes it back in
// place with coalesced 128-bit stores.  Small slices (<= 32 KB) let five
// CTAs share an SM, which keeps ~160 KB of state loads in flight per SM.
// Per token (src/kernel/fused_recurrent.rs:36-49):
//     S <- S diag(e^g);  v_new = w v - (b k)^T S;  S <- S + k v_new^T;
//     o = scale q^T S
// is evaluated with one reduction pass and one update pass over the slice:
//     erased = sum_k (b k e^g)_k S[k,:],   qs = sum_k (q e^g)_k S[k,:]
//     v_new  = w v - erased,              o  = scale (qs + (q.k) v_new)
//     S      = e^g S + k v_new^T
// The optional prologue applies the kernel-4 causal short conv + SiLU with
// the [B,3,C] caches (src/short_conv.rs:22-65) and the per-head L2 norm
// (src/l2norm.rs:13-16) to the raw projections; the optional epilogue is the
// SiLU-gated RMS norm (src/module.rs:501-517).
//
// Value columns may be split over `vsplit` CTAs.  When several CTAs share a
// key head's conv cache (GVA, or a V split) and the cache is updated in
// place, or when a split row needs the RMS epilogue, the sharing CTAs form a
// thread-block cluster: cache writes wait behind a cluster barrier and the
// RMS partial sums travel through distributed shared memory.
#include <cooperative_groups.h>

#include "common.cuh"
#include "ptx.cuh"

namespace cg = cooperative_groups;

namespace gdn2 {

constexpr int REC_THREADS = 256;
constexpr int REC_SLICE_BYTES = 32 * 1024;  // target state bytes per CTA

struct RecParams {
  int B, T, Hq, HV, K, V;
  int rep;  // value heads per q/k/g/b head in the views (1 = per value head)
  int vsplit, VT, CPR, RPP, npass;
  int prologue, fuse_epilogue;
  int cluster_x, cluster_y;
  int conv_sync;  // cluster barrier before in-place conv cache writes
  float scale, eps;
  DView q, k, v, g, b, w, gate, out;
  const float *cwq, *cwk, *cwv;
  const float *cq_in, *ck_in, *cv_in;
  float *cq_out, *ck_out, *cv_out;
  const float* onw;
  float* state;
};

// x_pad[j] of src/short_conv.rs:30-55 for one channel: j < 3 comes from the
// cache (or replicates token 0 when there is none), j >= 3 is token j-3.
template <typename T>
__device__ __forceinline__ float conv_pad(const DView& x, const float* cache, int C, int bb, int head, int kk,
                                          int ch, int j) {
  if (j >= 3) return vload<T>(x, bb, head, j - 3, kk);
  if (cache) return cache[((int64_t)bb * 3 + j) * C + ch];
  return vload<T>(x, bb, head, 0, kk);
}

template <typename T>
__device__ __forceinline__ float conv_act(const DView& x, const float* w, const float* cache, int C, int bb, int head,
                                          int kk, int ch, int t) {
  float acc = 0.f;
  #pragma unroll
  for (int i = 0; i < 4; ++i) acc += conv_pad<T>(x, cache, C, bb, head, kk, ch, t + i) * w[(int64_t)ch * 4 + i];
  return silu_f(acc);
}

template <typename T>
__global__ void __launch_bounds__(REC_THREADS, 4) k_recurrent(const RecParams p) {
  extern __shared__ __align__(128) unsigned char smraw[];
  const int K = p.K, VT = p.VT, RPP = p.RPP;
  float* sS = reinterpret_cast<float*>(smraw);  // [K][VT] state slice
  uint64_t* bar = reinterpret_cast<uint64_t*>(sS + K * VT);
  float* sq = reinterpret_cast<float*>(bar + 2);
  float* sk = sq + K;
  float* seg = sk + K;
  float* sbk = seg + K;
  float* sqg = sbk + K;
  float* svv = sqg + K;
  float* svn = svv + VT;
  float* so = svn + VT;
  float* red = so + VT;             // 2 * RPP * VT
  float* misc = red + 2 * RPP * VT;  // 32 (block_sum) + 16 (cluster slots)

  const int vs = blockIdx.x, hv = blockIdx.y, bb = blockIdx.z;
  const int kh = hv / p.rep;
  const int col0 = vs * VT;
  const int tid = threadIdx.x;
  const int cgi = tid % p.CPR, r0 = tid / p.CPR;
  const bool active = r0 < RPP;
  const int Cq = p.Hq * K;   // q/k conv channels
  const int Cv = p.HV * p.V; // v conv channels

  // ---- state slice HBM -> smem with bulk (TMA) copies, overlapped with the prologue ----
  float* st = p.state + ((int64_t)bb * p.HV + hv) * (int64_t)K * p.V + col0;
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (tid < 32) {
    if (tid == 0) mbar_arrive_expect_tx(bar, (unsigned)(K * VT * sizeof(float)));
    __syncwarp();
    if (VT == p.V) {
      if (tid == 0) bulk_g2s(sS, st, (unsigned)(K * VT * sizeof(float)), bar);
    } else {
      for (int kk = tid; kk < K; kk += 32)
        bulk_g2s(sS + kk * VT, st + (int64_t)kk * p.V, (unsigned)(VT * sizeof(float)), bar);
    }
  }
  bool have_state = false;

  for (int t = 0; t < p.T; ++t) {
    // ---- prologue: q, k (conv + SiLU + L2 as requested) ----
    float ssq = 0.f, ssk = 0.f;
    for (int kk = tid; kk < K; kk += REC_THREADS) {
      float qv, kv;
      if (p.prologue == 1) {
        const int ch = kh * K + kk;
        qv = conv_act<T>(p.q, p.cwq, p.cq_in, Cq, bb, kh, kk, ch, t);
        kv = conv_act<T>(p.k, p.cwk, p.ck_in, Cq, bb, kh, kk, ch, t);
      } else {
        qv = vload<T>(p.q, bb, kh, t, kk);
        kv = vload<T>(p.k, bb, kh, t, kk);
        if (p.prologue == 2) {
          qv = silu_f(qv);
          kv = silu_f(kv);
        }
      }
      sq[kk] = qv;
      sk[kk] = kv;
      ssq += qv * qv;
      ssk += kv * kv;
    }
    float nq = 1.f, nk = 1.f;
    if (p.prologue != 0) {
      nq = sqrtf(block_sum<REC_THREADS>(ssq, misc) + 1e-6f);
      nk = sqrtf(block_sum<REC_THREADS>(ssk, misc) + 1e-6f);
    }
    float pqk = 0.f;
    for (int kk = tid; kk < K; kk += REC_THREADS) {
      const float qv = sq[kk] / nq, kv = sk[kk] / nk;
      const float e = expf(vload<float>(p.g, bb, kh, t, kk));
      const float bv = vload<T>(p.b, bb, kh, t, kk);
      sk[kk] = kv;
      seg[kk] = e;
      sbk[kk] = bv * kv * e;
      sqg[kk] = qv * e;
      pqk += qv * kv;
    }
    for (int c = tid; c < VT; c += REC_THREADS) {
      const int col = col0 + c;
      float vv;
      if (p.prologue == 1) {
        vv = conv_act<T>(p.v, p.cwv, p.cv_in, Cv, bb, hv, col, hv * p.V + col, t);
      } else {
        vv = vload<T>(p.v, bb, hv, t, col);
        if (p.prologue == 2) vv = silu_f(vv);
      }
      svv[c] = vload<T>(p.w, bb, hv, t, col) * vv;
    }
    const float qk = block_sum<REC_THREADS>(pqk, misc);  // also publishes seg/sbk/sqg/svv
    if (!have_state) {
      // A wait that gives up has recorded a device error; the CTA still runs
      // every barrier so cluster peers are never left waiting.
      mbar_wait_bounded(bar, 0);
      have_state = true;
    }

    // ---- one pass over the smem-resident state ----
    float4 pe = make_float4(0.f, 0.f, 0.f, 0.f), pq = pe;
    if (active) {
      for (int i = 0; i < p.npass; ++i) {
        const int kk = r0 + i * RPP;
        if (kk < K) {
          const float4 s = *reinterpret_cast<const float4*>(sS + kk * VT + cgi * 4);
          const float a = sbk[kk], c = sqg[kk];
          pe.x += a * s.x; pe.y += a * s.y; pe.z += a * s.z; pe.w += a * s.w;
          pq.x += c * s.x; pq.y += c * s.y; pq.z += c * s.z; pq.w += c * s.w;
        }
      }
      *reinterpret_cast<float4*>(red + r0 * VT + cgi * 4) = pe;
      *reinterpret_cast<float4*>(red + (RPP + r0) * VT + cgi * 4) = pq;
    }
    __syncthreads();
    for (int c = tid; c < VT; c += REC_THREADS) {
      float e = 0.f, qs = 0.f;
      for (int r = 0; r < RPP; ++r) {
        e += red[r * VT + c];
        qs += red[(RPP + r) * VT + c];
      }
      const float vn = svv[c] - e;
      svn[c] = vn;
      so[c] = p.scale * (qs + qk * vn);
    }
    __syncthreads();
    if (active) {
      const float4 vn = *reinterpret_cast<const float4*>(svn + cgi * 4);
      const bool last = t == p.T - 1;
      for (int i = 0; i < p.npass; ++i) {
        const int kk = r0 + i * RPP;
        if (kk < K) {
          float4* sp = reinterpret_cast<float4*>(sS + kk * VT + cgi * 4);
          float4 s = *sp;
          const float e = seg[kk], kv = sk[kk];
          s.x = e * s.x + kv * vn.x;
          s.y = e * s.y + kv * vn.y;
          s.z = e * s.z + kv * vn.z;
          s.w = e * s.w + kv * vn.w;
          if (last)
            *reinterpret_cast<float4*>(st + (int64_t)kk * p.V + cgi * 4) = s;  // in place, coalesced
          else
            *sp = s;
        }
      }
    }

    // ---- epilogue ----
    if (p.fuse_epilogue) {
      float ss = 0.f;
      for (int c = tid; c < VT; c += REC_THREADS) ss += so[c] * so[c];
      float tot = block_sum<REC_THREADS>(ss, misc);
      if (p.cluster_x > 1) {
        cg::cluster_group cl = cg::this_cluster();
        const dim3 ci = cl.block_index();
        float* slot = misc + 32 + (t & 1) * 8;
        if (tid == 0) {
          for (int x = 0; x < p.cluster_x; ++x) {
            const unsigned rank = x + ci.y * p.cluster_x;
            float* peer = cl.map_shared_rank(slot, rank);
            peer[ci.x] = tot;
          }
        }
        cl.sync();
        tot = 0.f;
        for (int x = 0; x < p.cluster_x; ++x) tot += slot[x];
      }
      const float rms = sqrtf(tot / (float)p.V + p.eps);
      for (int c = tid; c < VT; c += REC_THREADS) {
        const int col = col0 + c;
        const float gt = vload<T>(p.gate, bb, hv, t, col);
        vstore<T>(p.out, bb, hv, t, col, so[c] / rms * p.onw[col] * silu_f(gt));
      }
    } else {
      for (int c = tid; c < VT; c += REC_THREADS) vstore<T>(p.out, bb, hv, t, col0 + c, so[c]);
    }
    __syncthreads();  // so / svn / sk / sS reused by the next token
  }

  // ---- new conv caches: rows T..T+2 of the padded sequence ----
  if (p.prologue == 1) {
    if (p.conv_sync) cg::this_cluster().sync();
    if (vs == 0 && hv % p.rep == 0) {
      for (int kk = tid; kk < K; kk += REC_THREADS) {
        const int ch = kh * K + kk;
        float xq[3], xk[3];
        #pragma unroll
        for (int j = 0; j < 3; ++j) {
          xq[j] = conv_pad<T>(p.q, p.cq_in, Cq, bb, kh, kk, ch, p.T + j);
          xk[j] = conv_pad<T>(p.k, p.ck_in, Cq, bb, kh, kk, ch, p.T + j);
        }
        #pragma unroll
        for (int j = 0; j < 3; ++j) {
          p.cq_out[((int64_t)bb * 3 + j) * Cq + ch] = xq[j];
          p.ck_out[((int64_t)bb * 3 + j) * Cq + ch] = xk[j];
        }
      }
    }
    for (int c = tid; c < VT; c += REC_THREADS) {
      const int col = col0 + c, ch = hv * p.V + col;
      float xv[3];
      #pragma unroll
      for (int j = 0; j < 3; ++j) xv[j] = conv_pad<T>(p.v, p.cv_in, Cv, bb, hv, col, ch, p.T + j);
      #pragma unroll
      for (int j = 0; j < 3; ++j) p.cv_out[((int64_t)bb * 3 + j) * Cv + ch] = xv[j];
    }
  }
}

// ---------------------------------------------------------------------------
// Decode step (T == 1): persistent, double-buffered, barrier-free main loop.
//
// A work item is one (batch, key-side head); the CTA handles all `rep` value
// heads of that key head and all 64-column slices of each, so every conv
// cache is read and rewritten by exactly one CTA (in place is safe) and the
// q/k prologue runs once per key head.
//
// Each of the 4 warps owns 16 columns of the current slice over all K rows
// and streams them through two private shared-memory buffers with per-lane
// 16-byte cp.async copies: the copy of step n+1 is issued before step n is
// consumed, and since lane (rg = lane / 4, cg = lane % 4) reads back exactly
// the rows rg, rg+8, ... and columns 4cg..4cg+3 it copied, no barrier is
// needed between copy and use.  A quarter-warp touches two dense 64-byte
// rows, so the 16-float rows need no padding to be bank-conflict free.  The
// K reductions are warp shuffles and updated rows go straight back to HBM
// (64 contiguous bytes per row per warp).  Block barriers remain only in the
// per-item prologue (L2 norms) and the per-value-head RMS epilogue.
// ---------------------------------------------------------------------------
constexpr int DEC_THREADS = 128;
constexpr int DEC_VT = 64;  // columns per slice (4 warps x 16)

constexpr int DEC_VCH = 2;  // value channels per thread (V <= 256)

struct DecTaps {
  float qx[4], kx[4], wq[4], wk[4], g, b;                          // item: thread = key channel
  float vx[DEC_VCH][4], wv[DEC_VCH][4], w[DEC_VCH], gate[DEC_VCH];  // value head: thread = channel(s)
};

template <typename T>
__device__ __forceinline__ void dec_load_qk(const RecParams& p, int item, DecTaps& r) {
  const int tid = threadIdx.x;
  if (tid >= p.K) return;
  const int bb = item / p.Hq, kh = item % p.Hq;
  const int Cq = p.Hq * p.K, ch = kh * p.K + tid;
  if (p.prologue == 1) {
    #pragma unroll
    for (int j = 0; j < 4; ++j) {
      r.qx[j] = conv_pad<T>(p.q, p.cq_in, Cq, bb, kh, tid, ch, j);
      r.kx[j] = conv_pad<T>(p.k, p.ck_in, Cq, bb, kh, tid, ch, j);
      r.wq[j] = p.cwq[(int64_t)ch * 4 + j];
      r.wk[j] = p.cwk[(int64_t)ch * 4 + j];
    }
  } else {
    r.qx[3] = vload<T>(p.q, bb, kh, 0, tid);
    r.kx[3] = vload<T>(p.k, bb, kh, 0, tid);
  }
  r.g = vload<float>(p.g, bb, kh, 0, tid);
  r.b = vload<T>(p.b, bb, kh, 0, tid);
}

template <typename T>
__device__ __forceinline__ void dec_load_v(const RecParams& p, int bb, int hv, DecTaps& r) {
  const int Cv = p.HV * p.V;
  #pragma unroll
  for (int u = 0; u < DEC_VCH; ++u) {
    const int c = threadIdx.x + u * DEC_THREADS;
    if (c >= p.V) break;
    const int ch = hv * p.V + c;
    if (p.prologue == 1) {
      #pragma unroll
      for (int j = 0; j < 4; ++j) {
        r.vx[u][j] = conv_pad<T>(p.v, p.cv_in, Cv, bb, hv, c, ch, j);
        r.wv[u][j] = p.cwv[(int64_t)ch * 4 + j];
      }
    } else {
      r.vx[u][3] = vload<T>(p.v, bb, hv, 0, c);
    }
    r.w[u] = vload<T>(p.w, bb, hv, 0, c);
    r.gate[u] = p.fuse_epilogue ? vload<T>(p.gate, bb, hv, 0, c) : 0.f;
  }
}

// Block sums with one barrier: each warp's partial goes to red, then every
// thread adds the NT / 32 partials itself.  The caller must pass another
// barrier before red is written again.
template <int NT>
__device__ __forceinline__ void block_sum3_1bar(float& a, float& b, float& c, float* red) {
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    b += __shfl_xor_sync(0xffffffffu, b, o);
    c += __shfl_xor_sync(0xffffffffu, c, o);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int NW = NT / 32;
  if (lane == 0) {
    red[warp] = a;
    red[NW + warp] = b;
    red[2 * NW + warp] = c;
  }
  __syncthreads();
  a = b = c = 0.f;
  #pragma unroll
  for (int w = 0; w < NW; ++w) {
    a += red[w];
    b += red[NW + w];
    c += red[2 * NW + w];
  }
}

template <int NT>
__device__ __forceinline__ float block_sum_1bar(float x, float* red) {
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = x;
  __syncthreads();
  float s = 0.f;
  #pragma unroll
  for (int w = 0; w < NT / 32; ++w) s += red[w];
  return s;
}

template <typename T>
__global__ void __launch_bounds__(DEC_THREADS) k_decode(const RecParams p) {
  extern __shared__ __align__(128) unsigned char smraw[];
  const int K = p.K, V = p.V;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rg = lane >> 2, cg = lane & 3;
  float* wbuf = reinterpret_cast<float*>(smraw) + warp * 2 * K * 16;  // this warp's 2 x [K][16]
  float* sk = reinterpret_cast<float*>(smraw) + 4 * 2 * K * 16;
  float* seg = sk + K;
  float* sbk = seg + K;
  float* sqg = sbk + K;
  float* svv = sqg + K;  // [V]
  float* so = svv + V;   // [V]
  float* misc = so + V;  // 32

  const int n_items = p.B * p.Hq;
  const int vsplit = V / DEC_VT;
  const int nsub = p.rep * vsplit;
  const int Cq = p.Hq * K, Cv = p.HV * V;
  const int wc = warp * 16 + cg * 4;  // this lane's column inside a slice
  if ((int)blockIdx.x >= n_items) return;

  // async copy of this lane's part of step (item, sub) into buffer b
  const uint64_t pol_st = l2_policy_evict_first();  // the state lines: read and written once per step
  auto issue = [&](int item, int sub, int b) {
    const int bb = item / p.Hq, kh = item % p.Hq;
    const int hv = kh * p.rep + sub / vsplit, vs = sub % vsplit;
    const float* src = p.state + ((int64_t)bb * p.HV + hv) * (int64_t)K * V + vs * DEC_VT + wc;
    float* dst = wbuf + b * K * 16 + cg * 4;
    for (int kk = rg; kk < K; kk += 8)  // read once per step: evict-first
      asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(smem_u32(dst + kk * 16)),
                   "l"(src + (int64_t)kk * V), "l"(pol_st)
                   : "memory");
    cp_async_commit();
  };

  DecTaps r;
  int buf = 0;
  issue(blockIdx.x, 0, 0);
  dec_load_qk<T>(p, blockIdx.x, r);
  dec_load_v<T>(p, blockIdx.x / p.Hq, (blockIdx.x % p.Hq) * p.rep, r);

  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    const int bb = item / p.Hq, kh = item % p.Hq;
    const int next_item = item + gridDim.x;

    // ---- q/k prologue (once per key head) ----
    float qv = 0.f, kv = 0.f;
    if (tid < K) {
      if (p.prologue == 1) {
        float aq = 0.f, ak = 0.f;
        #pragma unroll
        for (int j = 0; j < 4; ++j) {
          aq += r.qx[j] * r.wq[j];
          ak += r.kx[j] * r.wk[j];
        }
        qv = silu_f(aq);
        kv = silu_f(ak);
        #pragma unroll
        for (int j = 0; j < 3; ++j) {  // new caches = x_pad rows 1..3, in place
          p.cq_out[((int64_t)bb * 3 + j) * Cq + kh * K + tid] = r.qx[j + 1];
          p.ck_out[((int64_t)bb * 3 + j) * Cq + kh * K + tid] = r.kx[j + 1];
        }
      } else {
        qv = r.qx[3];
        kv = r.kx[3];
        if (p.prologue == 2) {
          qv = silu_f(qv);
          kv = silu_f(kv);
        }
      }
    }
    const float gv = r.g, bv = r.b;
    if (next_item < n_items) dec_load_qk<T>(p, next_item, r);  // prefetch, lands during this item
    // |q|^2, |k|^2 and q.k in one reduction; (q / |q|).(k / |k|) = q.k / (|q| |k|)
    float sqq = qv * qv, skk = kv * kv, sqk = qv * kv;
    block_sum3_1bar<DEC_THREADS>(sqq, skk, sqk, misc);
    float nq = 1.f, nk = 1.f;
    if (p.prologue != 0) {
      nq = sqrtf(sqq + 1e-6f);
      nk = sqrtf(skk + 1e-6f);
    }
    const float qk = sqk / (nq * nk);
    if (tid < K) {
      qv /= nq;
      kv /= nk;
      const float e = expf(gv);
      sk[tid] = kv;
      seg[tid] = e;
      sbk[tid] = bv * kv * e;
      sqg[tid] = qv * e;
    }
    __syncthreads();  // publishes sk/seg/sbk/sqg; misc reusable

    for (int j = 0; j < p.rep; ++j) {
      const int hv = kh * p.rep + j;
      // ---- v prologue (once per value head) from the prefetched registers ----
      float gate_reg[DEC_VCH];
      #pragma unroll
      for (int u = 0; u < DEC_VCH; ++u) {
        const int c = tid + u * DEC_THREADS;
        gate_reg[u] = r.gate[u];
        if (c < V) {
          float vv;
          if (p.prologue == 1) {
            float acc = 0.f;
            #pragma unroll
            for (int jj = 0; jj < 4; ++jj) acc += r.vx[u][jj] * r.wv[u][jj];
            vv = silu_f(acc);
            #pragma unroll
            for (int jj = 0; jj < 3; ++jj)  // new v cache = x_pad rows 1..3, in place
              p.cv_out[((int64_t)bb * 3 + jj) * Cv + hv * V + c] = r.vx[u][jj + 1];
          } else {
            vv = r.vx[u][3];
            if (p.prologue == 2) vv = silu_f(vv);
          }
          svv[c] = r.w[u] * vv;
        }
      }
      // prefetch the next value head's inputs
      if (j + 1 < p.rep)
        dec_load_v<T>(p, bb, hv + 1, r);
      else if (next_item < n_items)
        dec_load_v<T>(p, next_item / p.Hq, (next_item % p.Hq) * p.rep, r);
      __syncthreads();

      for (int vs = 0; vs < vsplit; ++vs) {
        const int sub = j * vsplit + vs;
        bool more = true;
        if (sub + 1 < nsub)
          issue(item, sub + 1, buf ^ 1);
        else if (next_item < n_items)
          issue(next_item, 0, buf ^ 1);
        else
          more = false;
        if (more)
          cp_async_wait<1>();
        else
          cp_async_wait<0>();
        const float* sS = wbuf + buf * K * 16 + cg * 4;
        const int col = vs * DEC_VT + wc;

        float4 pe = make_float4(0.f, 0.f, 0.f, 0.f), pq = pe;
        for (int kk = rg; kk < K; kk += 8) {
          const float4 s = *reinterpret_cast<const float4*>(sS + kk * 16);
          const float a = sbk[kk], c = sqg[kk];
          pe.x += a * s.x; pe.y += a * s.y; pe.z += a * s.z; pe.w += a * s.w;
          pq.x += c * s.x; pq.y += c * s.y; pq.z += c * s.z; pq.w += c * s.w;
        }
        #pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          pe.x += __shfl_xor_sync(0xffffffffu, pe.x, o);
          pe.y += __shfl_xor_sync(0xffffffffu, pe.y, o);
          pe.z += __shfl_xor_sync(0xffffffffu, pe.z, o);
          pe.w += __shfl_xor_sync(0xffffffffu, pe.w, o);
          pq.x += __shfl_xor_sync(0xffffffffu, pq.x, o);
          pq.y += __shfl_xor_sync(0xffffffffu, pq.y, o);
          pq.z += __shfl_xor_sync(0xffffffffu, pq.z, o);
          pq.w += __shfl_xor_sync(0xffffffffu, pq.w, o);
        }
        const float4 wv = *reinterpret_cast<const float4*>(svv + col);
        const float4 vn = make_float4(wv.x - pe.x, wv.y - pe.y, wv.z - pe.z, wv.w - pe.w);
        if (rg == 0)
          *reinterpret_cast<float4*>(so + col) =
              make_float4(p.scale * (pq.x + qk * vn.x), p.scale * (pq.y + qk * vn.y), p.scale * (pq.z + qk * vn.z),
                          p.scale * (pq.w + qk * vn.w));
        float* dst = p.state + ((int64_t)bb * p.HV + hv) * (int64_t)K * V + col;
        for (int kk = rg; kk < K; kk += 8) {
          float4 s = *reinterpret_cast<const float4*>(sS + kk * 16);
          const float e = seg[kk], kq = sk[kk];
          s.x = e * s.x + kq * vn.x;
          s.y = e * s.y + kq * vn.y;
          s.z = e * s.z + kq * vn.z;
          s.w = e * s.w + kq * vn.w;
          // written once per step and read again only by the next step, long after: evict-first
          asm volatile("st.global.L1::no_allocate.L2::cache_hint.v4.f32 [%0], {%1, %2, %3, %4}, %5;" ::"l"(
                           dst + (int64_t)kk * V),
                       "f"(s.x), "f"(s.y), "f"(s.z), "f"(s.w), "l"(pol_st)
                       : "memory");
        }
        buf ^= 1;
      }

      // ---- epilogue over the whole value head ----
      __syncthreads();  // so[] complete
      float ss = 0.f;
      for (int c = tid; c < V; c += DEC_THREADS) ss += so[c] * so[c];
      // misc is free: the barrier after the previous reduction's readers ("so[] complete") has passed
      const float rms = p.fuse_epilogue ? sqrtf(block_sum_1bar<DEC_THREADS>(ss, misc) / (float)V + p.eps) : 1.f;
      #pragma unroll
      for (int u = 0; u < DEC_VCH; ++u) {
        const int c = tid + u * DEC_THREADS;
        if (c < V) {
          if (p.fuse_epilogue)
            vstore<T>(p.out, bb, hv, 0, c, so[c] / rms * p.onw[c] * silu_f(gate_reg[u]));
          else
            vstore<T>(p.out, bb, hv, 0, c, so[c]);
        }
      }
      __syncthreads();  // svv / so reused by the next value head
    }
  }
  cp_async_wait<0>();
}

static int launch_decode(const RecParams& p0, int dtype, cudaStream_t stream) {
  RecParams p = p0;
  const int K = p.K, V = p.V;
  const size_t smem = sizeof(float) * (8 * (size_t)K * 16 + 4 * (size_t)K + 2 * (size_t)V + 32);
  void (*fn)(const RecParams) = dtype == GDN2_DTYPE_BF16 ? k_decode<__nv_bfloat16> : k_decode<float>;
  cudaError_t e = cudaFuncSetAttribute((const void*)fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return check_cuda(e, "gdn2_recurrent_fwd: smem attribute");
  int dev = 0, sms = 0, per_sm = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, DEC_THREADS, smem);
  if (e != cudaSuccess) return check_cuda(e, "gdn2_recurrent_fwd: occupancy");
  const int n_items = p.B * p.Hq;
  int grid = sms * (per_sm > 0 ? per_sm : 1);
  if (grid > n_items) grid = n_items;
  fn<<<grid, DEC_THREADS, smem, stream>>>(p);
  return check_cuda(cudaGetLastError(), "gdn2_recurrent_fwd decode launch");
}

GDN2_DEVICE_ERROR_READER(read_device_errors_recurrent)

static bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

int launch_recurrent(const gdn2_recurrent_args* a, cudaStream_t stream) {
  const gdn2_dims& d = a->dims;
  if (d.batch <= 0 || d.seq_len <= 0 || d.num_heads <= 0 || d.num_v_heads <= 0 || d.head_k_dim <= 0 ||
      d.head_v_dim <= 0)
    return set_error(GDN2_EINVAL, "gdn2_recurrent_fwd: all dims must be > 0");
  if (d.num_v_heads % d.num_heads)
    return set_error(GDN2_EINVAL, "gdn2_recurrent_fwd: num_v_heads %d not a multiple of num_heads %d",
                     d.num_v_heads, d.num_heads);
  if (a->dtype != GDN2_DTYPE_F32 && a->dtype != GDN2_DTYPE_BF16)
    return set_error(GDN2_EINVAL, "gdn2_recurrent_fwd: unknown dtype %d", a->dtype);
  if (a->prologue < 0 || a->prologue > 2) return set_error(GDN2_EINVAL, "gdn2_recurrent_fwd: bad prologue");
  if (!a->q.data || !a->k.data || !a->v.data || !a->g.data || !a->b.data || !a->w.data || !a->state ||
      !a->out.data)
    return set_error(GDN2_EINVAL, "gdn2_recurrent_fwd: null tensor pointer");
  if (a->fuse_epilogue && (!a->gate.data || !a->o_norm_weight))
    return set_error(GDN2_EINVAL, "gdn2_recurrent_fwd: epilogue needs gate and o_norm_weight");
  if (a->prologue == 1 && (!a->conv_w_q || !a->conv_w_k || !a->conv_w_v || !a->conv_q_out || !a->conv_k_out ||
                           !a->conv_v_out))
    return set_error(GDN2_EINVAL, "gdn2_recurrent_fwd: conv prologue needs weights and output caches");
  if (!aligned16(a->state)) return set_error(GDN2_EINVAL, "gdn2_recurrent_fwd: state must be 16-byte aligned");

  const int K = d.head_k_dim, V = d.head_v_dim;
  const int rep = a->key_heads_grouped ? d.num_v_heads / d.num_heads : 1;
  if (V % 4) return set_error(GDN2_EUNSUPPORTED, "gdn2_recurrent_fwd: head_v_dim %d not a multiple of 4", V);
  int vsplit = 1;
  while ((int64_t)K * (V / vsplit) * 4 > REC_SLICE_BYTES && (V % (8 * vsplit)) == 0 && V / vsplit > 32) vsplit *= 2;
  const int VT = V / vsplit;
  const int CPR = VT / 4;
  if (CPR > REC_THREADS) return set_error(GDN2_EUNSUPPORTED, "gdn2_recurrent_fwd: head_v_dim %d too large", V);
  const int RPP = REC_THREADS / CPR;
  const int npass = (K + RPP - 1) / RPP;
  RecParams p;
  p.B = d.batch; p.T = d.seq_len; p.HV = d.num_v_heads; p.K = K; p.V = V;
  p.Hq = a->key_heads_grouped ? d.num_heads : d.num_v_heads;
  p.rep = rep;
  p.vsplit = vsplit; p.VT = VT; p.CPR = CPR; p.RPP = RPP; p.npass = npass;
  p.prologue = a->prologue; p.fuse_epilogue = a->fuse_epilogue;
  p.scale = a->scale; p.eps = a->norm_eps;
  p.q = make_dview(a->q); p.k = make_dview(a->k); p.v = make_dview(a->v);
  p.g = make_dview(a->g); p.b = make_dview(a->b); p.w = make_dview(a->w);
  p.gate = make_dview(a->gate); p.out = make_dview(a->out);
  p.cwq = a->conv_w_q; p.cwk = a->conv_w_k; p.cwv = a->conv_w_v;
  p.cq_in = a->conv_q_in; p.ck_in = a->conv_k_in; p.cv_in = a->conv_v_in;
  p.cq_out = a->conv_q_out; p.ck_out = a->conv_k_out; p.cv_out = a->conv_v_out;
  p.onw = a->o_norm_weight;
  p.state = a->state;

  // decode hot path: one token, heads of <= 128 key channels, value heads in 64-column slices
  if (d.seq_len == 1 && K <= DEC_THREADS && V % DEC_VT == 0 && V <= DEC_THREADS * DEC_VCH)
    return launch_decode(p, a->dtype, stream);

  // CTAs that read a key head's conv cache which is overwritten in place
  // must finish reading before the owner writes: put them in one cluster.
  const bool shared_inplace = a->prologue == 1 &&
                              ((a->conv_q_in && a->conv_q_in == a->conv_q_out) ||
                               (a->conv_k_in && a->conv_k_in == a->conv_k_out));
  p.cluster_x = (vsplit > 1 && (a->fuse_epilogue || shared_inplace)) ? vsplit : 1;
  p.cluster_y = (shared_inplace && rep > 1) ? rep : 1;
  p.conv_sync = shared_inplace && p.cluster_x * p.cluster_y > 1;
  if (p.cluster_x * p.cluster_y > 8)
    return set_error(GDN2_EUNSUPPORTED,
                     "gdn2_recurrent_fwd: %d CTAs share one conv cache updated in place (max 8); pass separate "
                     "conv_*_out buffers",
                     p.cluster_x * p.cluster_y);

  const size_t smem = sizeof(float) * ((size_t)K * VT + 4 + 5 * (size_t)K + 3 * (size_t)VT + 2 * (size_t)RPP * VT + 48);
  if (smem > 220 * 1024)
    return set_error(GDN2_EUNSUPPORTED, "gdn2_recurrent_fwd: state slice %dx%d does not fit shared memory", K, VT);
  void (*fn)(const RecParams) = a->dtype == GDN2_DTYPE_BF16 ? k_recurrent<__nv_bfloat16> : k_recurrent<float>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute((const void*)fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return check_cuda(e, "gdn2_recurrent_fwd: smem attribute");
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(vsplit, d.num_v_heads, d.batch);
  cfg.blockDim = dim3(REC_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if (p.cluster_x * p.cluster_y > 1) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = p.cluster_x;
    attr[0].val.clusterDim.y = p.cluster_y;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return check_cuda(cudaLaunchKernelEx(&cfg, fn, p), "gdn2_recurrent_fwd launch");
}

}  // namespace gdn2
