// Kernels (1) + (2), f32 CUDA-core path: chunk-intra and chunk-inter.
//
// This is the exact-f32 path of the chunked forward (src/forward.rs:44-278)
// and the fallback-free general path for every shape the tensor-core path
// does not take (chunk sizes other than 64, head dims that are not a
// multiple of 64).  It follows the reference's tile-local log-space scheme:
// decay factors are taken relative to the start of each 16-row tile, so no
// exp() argument exceeds 16 tokens of decay.
//
// Workspace (f32), per chunk n = (b*HV + hv)*NC + c, rows padded to CP = 64:
//   Aqk [CP][CP]  scale * causal (q E)(k/E)^T e_block     (forward.rs:159-187)
//   W   [CP][K]   (I + Akk)^-1 (b k gamma)                 (forward.rs:189-261)
//   U   [CP][V]   (I + Akk)^-1 (w v)
//   Qg  [CP][K]   scale * q gamma                          (forward.rs:266-267)
//   Kd  [CP][K]   k exp(G_last - G)                        (forward.rs:271-274)
//   gl  [K]       gamma_last
//   O   [B,HV,T,V] raw core output (before the epilogue kernel)
#include "chunk.cuh"

namespace gdn2 {

constexpr int SIMT_THREADS = 256;
// Row stride (floats) of the intra kernel's [KS][CP] operand arrays: a warp
// writes 32 consecutive channels of one row, so a stride of CP = 64 would put
// all 32 stores in one bank; 68 keeps rows 16-byte aligned for the float4
// reads and leaves 4-way conflicts.
constexpr int CPS = CP + 4;

// ---------------------------------------------------------------------------
// chunk-intra: one CTA per (chunk, hv, b)
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(SIMT_THREADS, 2) k_intra_simt(const ChunkParams p) {
  extern __shared__ float sm[];
  float* sQs = sm;                  // [KS][CPS]  q E
  float* sKx = sQs + KS * CPS;      // [KS][CPS]  k / E
  float* sBs = sKx + KS * CPS;      // [KS][CPS]  b k E
  float* seb = sBs + KS * CPS;      // [4][4][KS] exp(min(Gb_p - Gb_q, 0))
  float* sTot = seb + 16 * KS;      // [4][KS] tile sums of g
  float* sGl = sTot + 4 * KS;       // [KS] G at the last valid row
  float* sA = sGl + KS;             // [CP][CP+1] Akk

  const int c = blockIdx.x, hv = blockIdx.y, bb = blockIdx.z;
  const int kh = hv / p.rep;
  const int t0 = c * p.C;
  const int cv = min(p.C, p.T - t0);
  const int K = p.K, V = p.V;
  const int64_t n = ((int64_t)bb * p.HV + hv) * p.NC + c;
  float* gAqk = p.ws_aqk + n * CP * CP;
  float* gW = p.ws_w + n * CP * K;
  float* gU = p.ws_u + n * CP * V;
  float* gQg = p.ws_qg + n * CP * K;
  float* gKd = p.ws_kd + n * CP * K;
  float* gGl = p.ws_gl + n * K;

  const int tid = threadIdx.x;
  const int kk = tid % KS, tp = tid / KS;  // channel within slice, 16-row tile
  const int ti = tid / 16, tj = tid % 16;
  const int r0 = 4 * ti, s0 = 4 * tj;
  const bool blk = s0 <= r0 + 3;
  const int lt = (cv - 1) >> 4, lr = (cv - 1) & 15;  // tile / row of the last valid token

  // the CTA's input rows on their way to L2 before the first use: q, k, b, g (key head), v, w (value head)
  {
    const int es = sizeof(T);
    for (int idx = tid; idx < 6 * CP * 8; idx += SIMT_THREADS) {
      const int j = idx / (CP * 8), rem = idx % (CP * 8), r = rem / 8, seg = rem % 8;
      if (r >= cv) continue;
      const DView& v = j == 0 ? p.q : j == 1 ? p.k : j == 2 ? p.b : j == 3 ? p.g : j == 4 ? p.v : p.w;
      const int h = j < 4 ? kh : hv;
      const int e = j == 3 ? 4 : es;
      const int width = (j < 4 ? K : V) * e;
      if (seg * 128 >= width) continue;
      const char* a0 = static_cast<const char*>(v.p) + ((int64_t)bb * v.s0 + (int64_t)h * v.s1 + (int64_t)(t0 + r) * v.s2) * e;
      asm volatile("prefetch.global.L2 [%0];" ::"l"(a0 + seg * 128));
    }
  }
  float aq[4][4], ak[4][4];
  #pragma unroll
  for (int i = 0; i < 4; ++i)
    #pragma unroll
    for (int j = 0; j < 4; ++j) aq[i][j] = ak[i][j] = 0.f;

  for (int k0 = 0; k0 < K; k0 += KS) {
    const int kc = k0 + kk;
    const bool kval = kc < K;
    float gl[16];
    float run = 0.f, glast_loc = 0.f;
    #pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int r = tp * 16 + i;
      const float gv = (kval && r < cv) ? vload<float>(p.g, bb, kh, t0 + r, kc) : 0.f;
      run += gv;
      gl[i] = run;
      if (i == lr) glast_loc = run;
    }
    sTot[tp * KS + kk] = run;
    __syncthreads();
    float gbp[4];
    gbp[0] = 0.f;
    #pragma unroll
    for (int pp = 1; pp < 4; ++pp) gbp[pp] = gbp[pp - 1] + sTot[(pp - 1) * KS + kk];
    const float gb = gbp[tp];
    if (tp == lt) sGl[kk] = gb + glast_loc;
    #pragma unroll
    for (int qq = 0; qq < 4; ++qq)
      if (qq <= tp) seb[(tp * 4 + qq) * KS + kk] = expf(fminf(gb - gbp[qq], 0.f));
    __syncthreads();
    const float Glast = sGl[kk];
    if (tp == 0 && kval) gGl[kc] = expf(Glast);
    #pragma unroll 4
    for (int i = 0; i < 16; ++i) {
      const int r = tp * 16 + i;
      const bool rv = kval && r < cv;
      const float qv = rv ? vload<T>(p.q, bb, kh, t0 + r, kc) : 0.f;
      const float kv = rv ? vload<T>(p.k, bb, kh, t0 + r, kc) : 0.f;
      const float bv = rv ? vload<T>(p.b, bb, kh, t0 + r, kc) : 0.f;
      const float E = expf(gl[i]);
      const float G = gb + gl[i];
      const float gam = expf(G);
      sQs[kk * CPS + r] = qv * E;
      sKx[kk * CPS + r] = kv / E;
      sBs[kk * CPS + r] = bv * kv * E;
      if (kval) {
        gW[r * K + kc] = bv * kv * gam;
        gQg[r * K + kc] = qv * gam * p.scale;
        gKd[r * K + kc] = kv * expf(Glast - G);
      }
    }
    __syncthreads();
    if (blk) {
      const float* eb = seb + ((r0 >> 4) * 4 + (s0 >> 4)) * KS;
      #pragma unroll 4
      for (int j = 0; j < KS; ++j) {
        const float4 a = *reinterpret_cast<const float4*>(sQs + j * CPS + r0);
        const float4 bq = *reinterpret_cast<const float4*>(sBs + j * CPS + r0);
        const float4 kx = *reinterpret_cast<const float4*>(sKx + j * CPS + s0);
        const float e = eb[j];
        const float av[4] = {a.x * e, a.y * e, a.z * e, a.w * e};
        const float bv[4] = {bq.x * e, bq.y * e, bq.z * e, bq.w * e};
        const float kvv[4] = {kx.x, kx.y, kx.z, kx.w};
        #pragma unroll
        for (int i = 0; i < 4; ++i)
          #pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            aq[i][jj] += av[i] * kvv[jj];
            ak[i][jj] += bv[i] * kvv[jj];
          }
      }
    }
    __syncthreads();
  }

  #pragma unroll
  for (int i = 0; i < 4; ++i)
    #pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int r = r0 + i, s = s0 + j;
      gAqk[r * CP + s] = (blk && s <= r) ? aq[i][j] * p.scale : 0.f;
      sA[r * (CP + 1) + s] = (blk && s < r) ? ak[i][j] : 0.f;
    }
  for (int idx = tid; idx < CP * V; idx += SIMT_THREADS) {
    const int r = idx / V, col = idx % V;
    gU[idx] = r < cv ? vload<T>(p.w, bb, hv, t0 + r, col) * vload<T>(p.v, bb, hv, t0 + r, col) : 0.f;
  }
  __syncthreads();

  // (I + Akk) X = RHS by forward substitution, one column per thread.
  for (int j = tid; j < K + V; j += SIMT_THREADS) {
    float* base = j < K ? gW + j : gU + (j - K);
    const int stride = j < K ? K : V;
    float x[CP];
    #pragma unroll
    for (int r = 0; r < CP; ++r) x[r] = base[r * stride];
    #pragma unroll
    for (int r = 1; r < CP; ++r) {
      float acc = x[r];
      #pragma unroll
      for (int s = 0; s < r; ++s) acc -= sA[r * (CP + 1) + s] * x[s];
      x[r] = acc;
    }
    #pragma unroll
    for (int r = 0; r < CP; ++r) base[r * stride] = x[r];
  }
}

// ---------------------------------------------------------------------------
// chunk-inter: one CTA per (value tile, hv, b), sequential over chunks
// ---------------------------------------------------------------------------
template <int VT>
__global__ void __launch_bounds__(SIMT_THREADS) k_inter_simt(const ChunkParams p) {
  constexpr int CQ = VT / 4;              // float4 column groups
  constexpr int RT = CP * VT / (SIMT_THREADS * 4);  // rows per thread
  extern __shared__ float sm[];
  const int Kp = (p.K + KS - 1) / KS * KS;
  float* sS = sm;                          // [Kp][VT]
  float* sW = sS + Kp * VT;                // [CP][KS+1]
  float* sQ = sW + CP * (KS + 1);          // [CP][KS+1]
  float* sAq = sQ + CP * (KS + 1);         // [CP][CP+1]
  float* svn = sAq + CP * (CP + 1);        // [CP][VT]

  const int vt = blockIdx.x, hv = blockIdx.y, bb = blockIdx.z;
  const int K = p.K, V = p.V;
  const int col0 = vt * VT;
  const int tid = threadIdx.x;
  const int cq = tid % CQ, rb = tid / CQ;
  const int c4 = col0 + cq * 4;
  const bool cval = c4 < V;  // V % 4 == 0, so a float4 group is all-in or all-out
  float* st = p.state + ((int64_t)bb * p.HV + hv) * (int64_t)K * V;

  for (int idx = tid; idx < Kp * CQ; idx += SIMT_THREADS) {
    const int k = idx / CQ, q4 = idx % CQ;
    const int col = col0 + q4 * 4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (k < K && col < V) v = *reinterpret_cast<const float4*>(st + (int64_t)k * V + col);
    *reinterpret_cast<float4*>(sS + k * VT + q4 * 4) = v;
  }
  __syncthreads();

  for (int c = 0; c < p.NC; ++c) {
    const int t0 = c * p.C;
    const int cv = min(p.C, p.T - t0);
    const int64_t n = ((int64_t)bb * p.HV + hv) * p.NC + c;
    const float* gAqk = p.ws_aqk + n * CP * CP;
    const float* gW = p.ws_w + n * CP * K;
    const float* gU = p.ws_u + n * CP * V;
    const float* gQg = p.ws_qg + n * CP * K;
    const float* gKd = p.ws_kd + n * CP * K;
    const float* gGl = p.ws_gl + n * K;

    // the next chunk's blocks on their way to L2 while this one computes: the
    // plain loads below sit between barriers, on the chain's critical path
    if (c + 1 < p.NC) {
      const int64_t n1 = n + 1;
      const int lw = CP * K * 4 / 128, la = CP * CP * 4 / 128, lu = CP * V * 4 / 128;
      for (int l = tid; l < 3 * lw + la + lu; l += SIMT_THREADS) {
        const char* a;
        if (l < lw) a = reinterpret_cast<const char*>(p.ws_w + n1 * CP * K) + 128 * l;
        else if (l < 2 * lw) a = reinterpret_cast<const char*>(p.ws_qg + n1 * CP * K) + 128 * (l - lw);
        else if (l < 3 * lw) a = reinterpret_cast<const char*>(p.ws_kd + n1 * CP * K) + 128 * (l - 2 * lw);
        else if (l < 3 * lw + la) a = reinterpret_cast<const char*>(p.ws_aqk + n1 * CP * CP) + 128 * (l - 3 * lw);
        else a = reinterpret_cast<const char*>(p.ws_u + n1 * CP * V) + 128 * (l - 3 * lw - la);
        asm volatile("prefetch.global.L2 [%0];" ::"l"(a));
      }
    }

    for (int idx = tid; idx < CP * CP / 4; idx += SIMT_THREADS) {
      const float4 a4 = reinterpret_cast<const float4*>(gAqk)[idx];
      float* d = sAq + (4 * idx / CP) * (CP + 1) + (4 * idx) % CP;
      d[0] = a4.x; d[1] = a4.y; d[2] = a4.z; d[3] = a4.w;
    }

    float avn[RT][4], ao[RT][4];
    #pragma unroll
    for (int i = 0; i < RT; ++i)
      #pragma unroll
      for (int j = 0; j < 4; ++j) avn[i][j] = ao[i][j] = 0.f;

    for (int k0 = 0; k0 < K; k0 += KS) {
      if (K % 4 == 0) {  // 16-byte loads (rows of K floats stay 16-byte aligned)
        for (int idx = tid; idx < CP * KS / 4; idx += SIMT_THREADS) {
          const int r = idx / (KS / 4), j = 4 * (idx % (KS / 4));
          float4 w4 = make_float4(0.f, 0.f, 0.f, 0.f), q4 = w4;
          if (k0 + j < K) {
            w4 = *reinterpret_cast<const float4*>(gW + r * K + k0 + j);
            q4 = *reinterpret_cast<const float4*>(gQg + r * K + k0 + j);
          }
          float* dw = sW + r * (KS + 1) + j;
          float* dq = sQ + r * (KS + 1) + j;
          dw[0] = w4.x; dw[1] = w4.y; dw[2] = w4.z; dw[3] = w4.w;
          dq[0] = q4.x; dq[1] = q4.y; dq[2] = q4.z; dq[3] = q4.w;
        }
      } else {
        for (int idx = tid; idx < CP * KS; idx += SIMT_THREADS) {
          const int r = idx / KS, j = idx % KS;
          const bool ok = k0 + j < K;
          sW[r * (KS + 1) + j] = ok ? gW[r * K + k0 + j] : 0.f;
          sQ[r * (KS + 1) + j] = ok ? gQg[r * K + k0 + j] : 0.f;
        }
      }
      __syncthreads();
      #pragma unroll 4
      for (int j = 0; j < KS; ++j) {
        const float4 s4 = *reinterpret_cast<const float4*>(sS + (k0 + j) * VT + cq * 4);
        #pragma unroll
        for (int i = 0; i < RT; ++i) {
          const float wv = sW[(rb * RT + i) * (KS + 1) + j];
          const float qv = sQ[(rb * RT + i) * (KS + 1) + j];
          avn[i][0] += wv * s4.x; avn[i][1] += wv * s4.y; avn[i][2] += wv * s4.z; avn[i][3] += wv * s4.w;
          ao[i][0] += qv * s4.x; ao[i][1] += qv * s4.y; ao[i][2] += qv * s4.z; ao[i][3] += qv * s4.w;
        }
      }
      __syncthreads();
    }
    // v_new = U - W S
    #pragma unroll
    for (int i = 0; i < RT; ++i) {
      const int r = rb * RT + i;
      float4 u = make_float4(0.f, 0.f, 0.f, 0.f);
      if (cval) u = *reinterpret_cast<const float4*>(gU + r * V + c4);
      *reinterpret_cast<float4*>(svn + r * VT + cq * 4) =
          make_float4(u.x - avn[i][0], u.y - avn[i][1], u.z - avn[i][2], u.w - avn[i][3]);
    }
    __syncthreads();
    // o = Aqk v_new + scale q gamma S
    for (int s = 0; s < CP; ++s) {
      const float4 v4 = *reinterpret_cast<const float4*>(svn + s * VT + cq * 4);
      #pragma unroll
      for (int i = 0; i < RT; ++i) {
        const float a = sAq[(rb * RT + i) * (CP + 1) + s];
        ao[i][0] += a * v4.x; ao[i][1] += a * v4.y; ao[i][2] += a * v4.z; ao[i][3] += a * v4.w;
      }
    }
    if (cval) {
      #pragma unroll
      for (int i = 0; i < RT; ++i) {
        const int r = rb * RT + i;
        if (r < cv)
          *reinterpret_cast<float4*>(p.ws_o + (((int64_t)bb * p.HV + hv) * p.T + t0 + r) * V + c4) =
              make_float4(ao[i][0], ao[i][1], ao[i][2], ao[i][3]);
      }
    }
    // S <- diag(gamma_last) S + Kd^T v_new
    for (int k0 = 0; k0 < K; k0 += KS) {
      if (K % 4 == 0) {
        for (int idx = tid; idx < CP * KS / 4; idx += SIMT_THREADS) {
          const int r = idx / (KS / 4), j = 4 * (idx % (KS / 4));
          float4 k4 = make_float4(0.f, 0.f, 0.f, 0.f);
          if (k0 + j < K) k4 = *reinterpret_cast<const float4*>(gKd + r * K + k0 + j);
          float* d = sW + r * (KS + 1) + j;
          d[0] = k4.x; d[1] = k4.y; d[2] = k4.z; d[3] = k4.w;
        }
      } else {
        for (int idx = tid; idx < CP * KS; idx += SIMT_THREADS) {
          const int r = idx / KS, j = idx % KS;
          sW[r * (KS + 1) + j] = (k0 + j < K) ? gKd[r * K + k0 + j] : 0.f;
        }
      }
      __syncthreads();
      float acc[RT][4];
      #pragma unroll
      for (int i = 0; i < RT; ++i)
        #pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
      #pragma unroll 4
      for (int r = 0; r < CP; ++r) {
        const float4 v4 = *reinterpret_cast<const float4*>(svn + r * VT + cq * 4);
        #pragma unroll
        for (int i = 0; i < RT; ++i) {
          const float kd = sW[r * (KS + 1) + rb * RT + i];
          acc[i][0] += kd * v4.x; acc[i][1] += kd * v4.y; acc[i][2] += kd * v4.z; acc[i][3] += kd * v4.w;
        }
      }
      #pragma unroll
      for (int i = 0; i < RT; ++i) {
        const int k = k0 + rb * RT + i;
        if (k < K) {
          const float gk = gGl[k];
          float4* sp = reinterpret_cast<float4*>(sS + k * VT + cq * 4);
          float4 s4 = *sp;
          s4.x = gk * s4.x + acc[i][0]; s4.y = gk * s4.y + acc[i][1];
          s4.z = gk * s4.z + acc[i][2]; s4.w = gk * s4.w + acc[i][3];
          *sp = s4;
        }
      }
      __syncthreads();
    }
  }

  for (int idx = tid; idx < K * CQ; idx += SIMT_THREADS) {
    const int k = idx / CQ, q4 = idx % CQ;
    const int col = col0 + q4 * 4;
    if (col < V) *reinterpret_cast<float4*>(st + (int64_t)k * V + col) = *reinterpret_cast<const float4*>(sS + k * VT + q4 * 4);
  }
}

// ---------------------------------------------------------------------------
// output stage: out = rms_norm_gate(O) or out = O (dtype conversion)
// one warp per (b, hv, t) row
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) k_chunk_out(const ChunkParams p) {
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int64_t nrows = (int64_t)p.B * p.HV * p.T;
  if (row >= nrows) return;
  const int t = (int)(row % p.T);
  const int hv = (int)((row / p.T) % p.HV);
  const int bb = (int)(row / ((int64_t)p.T * p.HV));
  const float* o = p.ws_o + row * p.V;
  float ss = 0.f;
  for (int c = lane; c < p.V; c += 32) ss += o[c] * o[c];
  #pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float rms = sqrtf(ss / (float)p.V + p.eps);
  for (int c = lane; c < p.V; c += 32) {
    float y = o[c];
    if (p.fuse_epilogue) y = y / rms * p.onw[c] * silu_f(vload<T>(p.gate, bb, hv, t, c));
    vstore<T>(p.out, bb, hv, t, c, y);
  }
}

// The same with 4 consecutive columns per lane (16-byte o loads, 8- or 16-byte
// gate / out accesses): taken when the gate and out rows are aligned for it.
__device__ __forceinline__ void ld4(const float* p, float (&x)[4]) {
  const float4 v = *reinterpret_cast<const float4*>(p);
  x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
}
__device__ __forceinline__ void ld4(const __nv_bfloat16* p, float (&x)[4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  x[0] = __uint_as_float(u.x << 16); x[1] = __uint_as_float(u.x & 0xffff0000u);
  x[2] = __uint_as_float(u.y << 16); x[3] = __uint_as_float(u.y & 0xffff0000u);
}
__device__ __forceinline__ void st4(float* p, const float (&y)[4]) {
  *reinterpret_cast<float4*>(p) = make_float4(y[0], y[1], y[2], y[3]);
}
__device__ __forceinline__ void st4(__nv_bfloat16* p, const float (&y)[4]) {
  __nv_bfloat162 a = __floats2bfloat162_rn(y[0], y[1]), b = __floats2bfloat162_rn(y[2], y[3]);
  *reinterpret_cast<uint2*>(p) = make_uint2(*reinterpret_cast<uint32_t*>(&a), *reinterpret_cast<uint32_t*>(&b));
}

template <typename T>
__global__ void __launch_bounds__(256) k_chunk_out4(const ChunkParams p) {
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int64_t nrows = (int64_t)p.B * p.HV * p.T;
  if (row >= nrows) return;
  const int t = (int)(row % p.T);
  const int hv = (int)((row / p.T) % p.HV);
  const int bb = (int)(row / ((int64_t)p.T * p.HV));
  const float* o = p.ws_o + row * p.V;
  float ss = 0.f;
  for (int c = 4 * lane; c < p.V; c += 128) {
    float x[4];
    ld4(o + c, x);
    ss += x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
  }
  #pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float rms = sqrtf(ss / (float)p.V + p.eps);
  const T* gp = static_cast<const T*>(p.gate.p) + bb * p.gate.s0 + hv * p.gate.s1 + (int64_t)t * p.gate.s2;
  T* op = static_cast<T*>(const_cast<void*>(p.out.p)) + bb * p.out.s0 + hv * p.out.s1 + (int64_t)t * p.out.s2;
  for (int c = 4 * lane; c < p.V; c += 128) {
    float x[4], y[4];
    ld4(o + c, x);
    if (p.fuse_epilogue) {
      float g[4];
      ld4(gp + c, g);
      #pragma unroll
      for (int e = 0; e < 4; ++e) y[e] = x[e] / rms * p.onw[c + e] * silu_f(g[e]);
    } else {
      #pragma unroll
      for (int e = 0; e < 4; ++e) y[e] = x[e];
    }
    st4(op + c, y);
  }
}

// ---------------------------------------------------------------------------
// host launchers
// ---------------------------------------------------------------------------
size_t simt_smem_intra() { return sizeof(float) * (3 * KS * CPS + 16 * KS + 4 * KS + KS + CP * (CP + 1)); }

template <int VT>
static size_t smem_inter(int K) {
  const int Kp = (K + KS - 1) / KS * KS;
  return sizeof(float) * ((size_t)Kp * VT + 2 * CP * (KS + 1) + CP * (CP + 1) + CP * VT);
}

static int set_smem(const void* fn, size_t bytes) {
  if (bytes <= 48 * 1024) return GDN2_OK;
  return check_cuda(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes),
                    "smem attribute");
}

int launch_intra_simt(const ChunkParams& p, int dtype, cudaStream_t st) {
  const size_t smem = simt_smem_intra();
  dim3 grid(p.NC, p.HV, p.B);
  if (dtype == GDN2_DTYPE_BF16) {
    int rc = set_smem((const void*)k_intra_simt<__nv_bfloat16>, smem);
    if (rc) return rc;
    k_intra_simt<__nv_bfloat16><<<grid, SIMT_THREADS, smem, st>>>(p);
  } else {
    int rc = set_smem((const void*)k_intra_simt<float>, smem);
    if (rc) return rc;
    k_intra_simt<float><<<grid, SIMT_THREADS, smem, st>>>(p);
  }
  return check_cuda(cudaGetLastError(), "chunk intra launch");
}

template <int VT>
static int launch_inter_vt(const ChunkParams& p, cudaStream_t st) {
  const size_t smem = smem_inter<VT>(p.K);
  int rc = set_smem((const void*)k_inter_simt<VT>, smem);
  if (rc) return rc;
  dim3 grid((p.V + VT - 1) / VT, p.HV, p.B);
  k_inter_simt<VT><<<grid, SIMT_THREADS, smem, st>>>(p);
  return check_cuda(cudaGetLastError(), "chunk inter launch");
}

// Column slice per CTA.  Every CTA walks the whole chunk chain of its (b, hv),
// so the grid must fit in one wave: 64-column slices (256 CTAs for 128
// chains of V = 128, two per SM) beat 32-column ones (512 CTAs, more than
// the 444 that fit) and read each chain's W / Qg / Kd / Aqk half as often.
// With few chains the narrowest slices that still fit two per SM cut the
// per-chunk work on each chain's critical path instead.
int launch_inter_simt(const ChunkParams& p, cudaStream_t st) {
  const long long chains = (long long)p.B * p.HV, fit = 2LL * usable_sms();
  if (p.V % 16 == 0 && chains * (p.V / 16) <= fit) return launch_inter_vt<16>(p, st);
  if (p.V % 32 == 0 && chains * (p.V / 32) <= fit) return launch_inter_vt<32>(p, st);
  if (p.V <= 16) return launch_inter_vt<16>(p, st);
  if (p.V <= 64 && p.V % 32 != 0) return launch_inter_vt<16>(p, st);
  if (p.V % 64 == 0) return launch_inter_vt<64>(p, st);
  return launch_inter_vt<32>(p, st);
}

int launch_chunk_out(const ChunkParams& p, int dtype, cudaStream_t st) {
  const int64_t nrows = (int64_t)p.B * p.HV * p.T;
  dim3 grid((unsigned)((nrows + 7) / 8));
  // 4-column accesses need every gate / out row start aligned to 4 elements (V % 4 == 0 already holds)
  const int es = dtype == GDN2_DTYPE_BF16 ? 2 : 4;
  auto rows4 = [&](const DView& v) {
    return (uintptr_t)v.p % (4 * es) == 0 && v.s0 % 4 == 0 && v.s1 % 4 == 0 && v.s2 % 4 == 0;
  };
  const bool vec = rows4(p.out) && (!p.fuse_epilogue || rows4(p.gate));
  if (dtype == GDN2_DTYPE_BF16) {
    if (vec) k_chunk_out4<__nv_bfloat16><<<grid, 256, 0, st>>>(p);
    else k_chunk_out<__nv_bfloat16><<<grid, 256, 0, st>>>(p);
  } else {
    if (vec) k_chunk_out4<float><<<grid, 256, 0, st>>>(p);
    else k_chunk_out<float><<<grid, 256, 0, st>>>(p);
  }
  return check_cuda(cudaGetLastError(), "chunk output launch");
}

}  // namespace gdn2
