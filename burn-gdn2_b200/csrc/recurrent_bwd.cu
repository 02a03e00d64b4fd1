// Backward of the GDN-2 token recurrence (the core of kernels (1)-(3)),
// exact f32 on the CUDA cores.
//
// The reference has no wired backward: the crate trains through burn's
// autodiff of its tensor path (src/forward.rs:44-278, whose per-token form is
// src/kernel/fused_recurrent.rs:11-56), and its adjoint kernel sketch
// (src/kernel/chunk_adjoint_cube.rs:22-378) is unwired.  This kernel is the
// reverse-mode adjoint of that recurrence.  Per token t, with
// gamma = e^{g_t} (per key channel), bk = b_t k_t:
//     forward:  Sa = gamma S_{t-1};  e = Sa^T bk;  u = w v - e;
//               S_t = Sa + k u^T;    o_t = scale S_t^T q
//     adjoint (dS = dL/dS_t, carried backwards from dL/dS_T):
//               dS  += scale q dO^T;            dq = scale S_t dO
//               du   = dS^T k;                  dk = dS u + (dbk) b
//               dSa  = dS - bk du^T;            dbk = -Sa du,  db = dbk k
//               dg   = rowsum(dSa * Sa);        dv = du w,  dw = du v
//               dS_{t-1} = gamma dSa
//
// Decomposition.  The recurrence is independent per value column; the
// key-side gradients (dq, dk, db, dg) sum over all columns.  A CTA owns VT
// columns of one (batch, value head) chain, a warp owns 2 of them, and lane
// l owns key rows l, l+32, l+64, l+96, so the two K-reductions per token
// on the critical path (e and du) are warp shuffles.  The V-reductions are
// outputs only: each warp stores its per-row partials of a token in its own
// shared slot (plain stores; float atomics on shared memory serialise the
// warps), one barrier later every thread sums two of the 4K values over the
// warps into the sub-chunk buffer, and, every 8 tokens, the CTAs of a chain,
// which form one thread-block cluster, sum each other's buffers through
// distributed shared memory and write dq, dk, db, dg once.
//
// States for the reverse pass.  A forward pass over the sequence (its own
// launch, k_recurrent_bwd_ckpt, at twice the occupancy) stores the state at
// every 8th token boundary in the workspace (each thread its own 2 x RPL
// values, contiguous, so a warp stores one contiguous block).  The reverse
// pass walks the 8-token sub-chunks from the last: it reloads the
// sub-chunk's start state, replays the 8 tokens keeping each token's
// incoming state in registers, then runs the adjoint over them.  Work per
// token is three forward steps and one adjoint step on the slice; the
// workspace is B x HV x ceil(T/8) x K x V floats.
//
// Inputs.  When every view is 16-byte aligned, the raw rows of the next
// sub-chunk (and, in the reverse pass, the thread's next checkpoint) are
// fetched by cp.async into a staging buffer while the current sub-chunk
// computes; one pass then converts them into the packed layout.  Other
// views are read synchronously.
#include <cooperative_groups.h>

#include "common.cuh"
#include "ptx.cuh"

namespace cg = cooperative_groups;

namespace gdn2 {

constexpr int BWD_L = 8;   // tokens per sub-chunk (register history depth)
constexpr int BWD_NC = 2;  // value columns per warp

struct BwdParams {
  int B, T, HV, K, V, rep;
  int NCL, VT, NW, NS;  // CTAs per chain (cluster size), columns per CTA, warps per CTA, sub-chunks
  float scale;
  DView q, k, v, g, b, w, dout;
  DView dq, dk, dv, dg, db, dw;  // f32
  const float* h0;               // [B,HV,K,V] or null
  const float* dht;              // [B,HV,K,V] or null
  float* dh0;                    // [B,HV,K,V] or null
  float* ckpt;                   // workspace
  // trajectory export (k_recurrent_bwd_ckpt with EXPORT): the state entering every chunk of `chunk` tokens,
  // [B,HV,ceil(T/chunk),K,V] f32, and v_new per token (f32 view, p = null: not written)
  int chunk;
  float* states_out;
  DView vnew;
};

__device__ __forceinline__ float warp_sum_bwd(float x) {
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// Shared memory: staged inputs of one sub-chunk, packed so that one 128-bit
// load gives a row's or a column's values for a token, the per-column
// outputs dv / dw, two V-reduction buffers (by sub-chunk parity) and the
// warps' per-token partial slots (by token parity).
struct BwdSmem {
  float4* kr;    // [L][K]: (e^g, b, k, scale q) of key row kk
  float4* vc;    // [L][VT]: (w v, dO, w, v) of value column c
  float *dv, *dw;  // [L][VT]
  float4* red;   // [2][L][K]: (dq, dk through S_t, dbk, dg) of the CTA's columns
  float4* slot;  // [2][NW][K]: the same of one warp's columns, one token
  // cp.async staging (aligned views only): raw q, k, b [L][K], g [L][K] f32, v, w, dO [L][VT]; checkpoints
  unsigned char *rq, *rk, *rb, *rv, *rw, *rdo;
  float* rg;
  float* ck;     // [threads][2 RPL]
};

__host__ __device__ inline size_t bwd_smem_bytes(int K, int VT, int NW, int RPL, int esz) {
  return 16 * ((size_t)BWD_L * K + (size_t)BWD_L * VT + (size_t)2 * BWD_L * K + (size_t)2 * NW * K) +
         8 * (size_t)BWD_L * VT + (size_t)BWD_L * (3 * (size_t)K * esz + 4 * (size_t)K + 3 * (size_t)VT * esz) +
         (size_t)NW * 32 * RPL * 8;
}

// cp.async of sub-chunk tokens t0 .. t0+cv-1 of every input into the staging buffer (one commit group)
template <typename TIN>
__device__ __forceinline__ void bwd_issue(const BwdParams& p, const BwdSmem& s, int bb, int hv, int kh, int col0,
                                          int t0, int cv, bool with_dout) {
  const int nth = blockDim.x, tid = threadIdx.x, K = p.K, VT = p.VT;
  constexpr int ES = (int)sizeof(TIN);
  const int cr = K * ES / 16, cg4 = K * 4 / 16, cvv = VT * ES / 16;  // 16-byte chunks per row
  const int nk = cv * cr;
  for (int i = tid; i < 3 * nk; i += nth) {
    const int which = i / nk, rem = i - which * nk, tt = rem / cr, c = rem - tt * cr;
    const DView& v = which == 0 ? p.q : which == 1 ? p.k : p.b;
    unsigned char* dst = which == 0 ? s.rq : which == 1 ? s.rk : s.rb;
    const char* src = static_cast<const char*>(v.p) + ((int64_t)bb * v.s0 + (int64_t)kh * v.s1 + (int64_t)(t0 + tt) * v.s2) * ES;
    cp_async16(dst + (tt * K) * ES + c * 16, src + c * 16);
  }
  for (int i = tid; i < cv * cg4; i += nth) {
    const int tt = i / cg4, c = i - tt * cg4;
    const char* src = static_cast<const char*>(p.g.p) +
                      ((int64_t)bb * p.g.s0 + (int64_t)kh * p.g.s1 + (int64_t)(t0 + tt) * p.g.s2) * 4;
    cp_async16(reinterpret_cast<unsigned char*>(s.rg) + tt * K * 4 + c * 16, src + c * 16);
  }
  const int nv = cv * cvv, nvt = with_dout ? 3 : 2;
  for (int i = tid; i < nvt * nv; i += nth) {
    const int which = i / nv, rem = i - which * nv, tt = rem / cvv, c = rem - tt * cvv;
    const DView& v = which == 0 ? p.v : which == 1 ? p.w : p.dout;
    unsigned char* dst = which == 0 ? s.rv : which == 1 ? s.rw : s.rdo;
    const char* src = static_cast<const char*>(v.p) +
                      ((int64_t)bb * v.s0 + (int64_t)hv * v.s1 + (int64_t)(t0 + tt) * v.s2 + col0) * ES;
    cp_async16(dst + (tt * VT) * ES + c * 16, src + c * 16);
  }
}

// staged raw rows -> the packed layout (tokens past cv: the identity step's values)
template <typename TIN>
__device__ __forceinline__ void bwd_convert(const BwdParams& p, const BwdSmem& s, int cv, bool with_dout) {
  const int nth = blockDim.x, tid = threadIdx.x, K = p.K, VT = p.VT;
  const TIN *q = reinterpret_cast<const TIN*>(s.rq), *k = reinterpret_cast<const TIN*>(s.rk),
            *b = reinterpret_cast<const TIN*>(s.rb);
  for (int i = tid; i < BWD_L * K; i += nth) {
    float4 r = make_float4(1.f, 0.f, 0.f, 0.f);
    if (i < cv * K) r = make_float4(expf(s.rg[i]), to_f32<TIN>(b[i]), to_f32<TIN>(k[i]), p.scale * to_f32<TIN>(q[i]));
    s.kr[i] = r;
  }
  const TIN *v = reinterpret_cast<const TIN*>(s.rv), *w = reinterpret_cast<const TIN*>(s.rw),
            *d = reinterpret_cast<const TIN*>(s.rdo);
  for (int i = tid; i < BWD_L * VT; i += nth) {
    float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
    if (i < cv * VT) {
      r.z = to_f32<TIN>(w[i]);
      r.w = to_f32<TIN>(v[i]);
      r.x = r.z * r.w;
      if (with_dout) r.y = to_f32<TIN>(d[i]);
    }
    s.vc[i] = r;
  }
}

template <typename TIN>
__device__ __forceinline__ void bwd_stage(const BwdParams& p, const BwdSmem& s, int bb, int hv, int kh, int col0,
                                          int t0, int cv, bool with_dout) {
  const int nth = blockDim.x, tid = threadIdx.x, K = p.K, VT = p.VT;
  for (int i = tid; i < BWD_L * K; i += nth) {
    const int tt = i / K, kk = i - tt * K;
    float4 r = make_float4(1.f, 0.f, 0.f, 0.f);
    if (tt < cv) {
      r.x = expf(vload<float>(p.g, bb, kh, t0 + tt, kk));
      r.y = vload<TIN>(p.b, bb, kh, t0 + tt, kk);
      r.z = vload<TIN>(p.k, bb, kh, t0 + tt, kk);
      r.w = p.scale * vload<TIN>(p.q, bb, kh, t0 + tt, kk);
    }
    s.kr[i] = r;
  }
  for (int i = tid; i < BWD_L * VT; i += nth) {
    const int tt = i / VT, c = i - tt * VT;
    float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
    if (tt < cv) {
      r.z = vload<TIN>(p.w, bb, hv, t0 + tt, col0 + c);
      r.w = vload<TIN>(p.v, bb, hv, t0 + tt, col0 + c);
      r.x = r.z * r.w;
      if (with_dout) r.y = vload<TIN>(p.dout, bb, hv, t0 + tt, col0 + c);
    }
    s.vc[i] = r;
  }
}

// One forward token step on the thread's RPL x NC slice.  Returns u (per column) through `u`.
template <int RPL>
__device__ __forceinline__ void bwd_fwd_step(const BwdSmem& s, int K, int VT, int tt, int lane, int cw,
                                             float (&S)[RPL][BWD_NC], float (&u)[BWD_NC]) {
  float e[BWD_NC], kr[RPL];
  #pragma unroll
  for (int c = 0; c < BWD_NC; ++c) e[c] = 0.f;
  #pragma unroll
  for (int r = 0; r < RPL; ++r) {
    const float4 x = s.kr[tt * K + lane + 32 * r];
    const float bkr = x.y * x.z;
    kr[r] = x.z;
    #pragma unroll
    for (int c = 0; c < BWD_NC; ++c) {
      S[r][c] *= x.x;
      e[c] += bkr * S[r][c];
    }
  }
  #pragma unroll
  for (int c = 0; c < BWD_NC; ++c) u[c] = s.vc[tt * VT + cw + c].x - warp_sum_bwd(e[c]);
  #pragma unroll
  for (int r = 0; r < RPL; ++r)
    #pragma unroll
    for (int c = 0; c < BWD_NC; ++c) S[r][c] += kr[r] * u[c];
}

// this thread's checkpoint of sub-chunk n (RPL float2, contiguous; the same thread of the same CTA position in
// both kernels)
template <int RPL>
__device__ __forceinline__ float2* bwd_ckpt_ptr(const BwdParams& p, int64_t chain, int n, int rank) {
  const int64_t base = ((chain * p.NS + n) * p.NCL + rank) * (int64_t)blockDim.x + threadIdx.x;
  return reinterpret_cast<float2*>(p.ckpt + base * (RPL * BWD_NC));
}

// The forward pass: the state at every sub-chunk start into the workspace.  Its own launch (no register
// history, no cluster), so that more CTAs share an SM than the reverse pass allows.  With EXPORT it is the
// trajectory export instead: every token is stepped, the state entering each chunk goes to p.states_out in
// the public [B,HV,NT,K,V] layout and v_new = w v - (b k)^T (e^g S) of every token to p.vnew.
template <typename TIN, int RPL, bool ASYNC, bool EXPORT>
__global__ void __launch_bounds__(512, 2) k_recurrent_bwd_ckpt(const BwdParams p) {
  extern __shared__ __align__(16) float4 smf4[];
  const int K = p.K, VT = p.VT;
  BwdSmem s;
  s.kr = smf4;
  s.vc = s.kr + BWD_L * K;
  {
    constexpr int ES = (int)sizeof(TIN);
    unsigned char* raw = reinterpret_cast<unsigned char*>(s.vc + BWD_L * VT);
    s.rg = reinterpret_cast<float*>(raw);
    s.rq = raw + BWD_L * K * 4;
    s.rk = s.rq + BWD_L * K * ES;
    s.rb = s.rk + BWD_L * K * ES;
    s.rv = s.rb + BWD_L * K * ES;
    s.rw = s.rv + BWD_L * VT * ES;
    s.rdo = s.rw + BWD_L * VT * ES;
  }
  const int rank = blockIdx.x, hv = blockIdx.y, bb = blockIdx.z, kh = hv / p.rep;
  const int col0 = rank * VT;
  const int lane = threadIdx.x & 31, cw = (threadIdx.x >> 5) * BWD_NC;
  const int64_t chain = (int64_t)bb * p.HV + hv;
  const int64_t KV = (int64_t)K * p.V;

  float S[RPL][BWD_NC];
  #pragma unroll
  for (int r = 0; r < RPL; ++r)
    #pragma unroll
    for (int c = 0; c < BWD_NC; ++c)
      S[r][c] = p.h0 ? p.h0[chain * KV + (int64_t)(lane + 32 * r) * p.V + col0 + cw + c] : 0.f;
  // sub-chunks stepped: all of them for the export, all but the last for the checkpoints (the last is
  // replayed from its start by the reverse pass)
  const int nsteps = EXPORT ? p.NS : p.NS - 1;
  if (ASYNC && nsteps > 0) {
    bwd_issue<TIN>(p, s, bb, hv, kh, col0, 0, min(BWD_L, p.T), false);
    cp_async_commit();
  }
  for (int n = 0; n < p.NS; ++n) {
    const int t0 = n * BWD_L, cv = min(BWD_L, p.T - t0);
    if (EXPORT) {
      if (t0 % p.chunk == 0) {
        float* so = p.states_out + (chain * ((p.T + p.chunk - 1) / p.chunk) + t0 / p.chunk) * KV + col0 + cw;
        #pragma unroll
        for (int r = 0; r < RPL; ++r)
          *reinterpret_cast<float2*>(so + (int64_t)(lane + 32 * r) * p.V) = make_float2(S[r][0], S[r][1]);
      }
    } else {
      float2* ck = bwd_ckpt_ptr<RPL>(p, chain, n, rank);
      #pragma unroll
      for (int r = 0; r < RPL; ++r) ck[r] = make_float2(S[r][0], S[r][1]);
    }
    if (n >= nsteps) break;
    if (ASYNC) {
      cp_async_wait<0>();
      __syncthreads();  // every thread's copies landed; the previous sub-chunk's steps are done
      bwd_convert<TIN>(p, s, cv, false);
      __syncthreads();
      if (n + 1 < nsteps) {
        bwd_issue<TIN>(p, s, bb, hv, kh, col0, t0 + BWD_L, min(BWD_L, p.T - t0 - BWD_L), false);
        cp_async_commit();
      }
    } else {
      bwd_stage<TIN>(p, s, bb, hv, kh, col0, t0, cv, false);
      __syncthreads();
    }
    #pragma unroll
    for (int tt = 0; tt < BWD_L; ++tt) {
      float u[BWD_NC];
      bwd_fwd_step<RPL>(s, K, VT, tt, lane, cw, S, u);  // tokens past the end: identity steps
      if (EXPORT && p.vnew.p && lane < BWD_NC && tt < cv)
        vstore<float>(p.vnew, bb, hv, t0 + tt, col0 + cw + lane, lane == 0 ? u[0] : u[1]);
    }
    if (!ASYNC) __syncthreads();
  }
}

__host__ __device__ inline size_t bwd_ckpt_smem_bytes(int K, int VT, int esz) {
  return 16 * ((size_t)BWD_L * K + (size_t)BWD_L * VT) +
         (size_t)BWD_L * (3 * (size_t)K * esz + 4 * (size_t)K + 3 * (size_t)VT * esz);
}

template <typename TIN, int RPL, bool ASYNC>
__global__ void __launch_bounds__(512, 1) k_recurrent_bwd(const BwdParams p) {
  extern __shared__ __align__(16) float4 smf4[];
  const int K = p.K, VT = p.VT, NCL = p.NCL;
  BwdSmem s;
  s.kr = smf4;
  s.vc = s.kr + BWD_L * K;
  s.red = s.vc + BWD_L * VT;
  s.slot = s.red + 2 * BWD_L * K;
  s.dv = reinterpret_cast<float*>(s.slot + 2 * p.NW * K);
  s.dw = s.dv + BWD_L * VT;
  {
    constexpr int ES = (int)sizeof(TIN);
    unsigned char* raw = reinterpret_cast<unsigned char*>(s.dw + BWD_L * VT);  // 16-byte aligned: L VT = 8 VT floats
    s.rg = reinterpret_cast<float*>(raw);
    s.rq = raw + BWD_L * K * 4;
    s.rk = s.rq + BWD_L * K * ES;
    s.rb = s.rk + BWD_L * K * ES;
    s.rv = s.rb + BWD_L * K * ES;
    s.rw = s.rv + BWD_L * VT * ES;
    s.rdo = s.rw + BWD_L * VT * ES;
    s.ck = reinterpret_cast<float*>(s.rdo + BWD_L * VT * ES);
  }

  cg::cluster_group cl = cg::this_cluster();
  const int rank = (int)cl.block_rank();
  const int hv = blockIdx.y, bb = blockIdx.z, kh = hv / p.rep;
  const int col0 = rank * VT;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nth = blockDim.x;
  const int cw = warp * BWD_NC;  // the warp's first column in the slice
  const int64_t chain = (int64_t)bb * p.HV + hv;
  const int64_t KV = (int64_t)K * p.V;

  // this thread's checkpoint of sub-chunk n, written by k_recurrent_bwd_ckpt
  auto ck = [&](int n) -> float2* { return bwd_ckpt_ptr<RPL>(p, chain, n, rank); };

  float S[RPL][BWD_NC];
  // ---- reverse pass ----
  float dS[RPL][BWD_NC];
  #pragma unroll
  for (int r = 0; r < RPL; ++r)
    #pragma unroll
    for (int c = 0; c < BWD_NC; ++c)
      dS[r][c] = p.dht ? p.dht[chain * KV + (int64_t)(lane + 32 * r) * p.V + col0 + cw + c] : 0.f;

  // this thread's checkpoint and the inputs of sub-chunk n into the staging buffer
  auto issue_rev = [&](int n, bool with_ck) {
    if (with_ck) {
      const float2* src = ck(n);
      #pragma unroll
      for (int r = 0; r < RPL; ++r) cp_async8(s.ck + (tid * RPL + r) * BWD_NC, src + r);
    }
    bwd_issue<TIN>(p, s, bb, hv, kh, col0, n * BWD_L, min(BWD_L, p.T - n * BWD_L), true);
    cp_async_commit();
  };
  if (ASYNC) issue_rev(p.NS - 1, true);
  for (int it = 0; it < p.NS; ++it) {
    const int n = p.NS - 1 - it, par = it & 1;
    const int t0 = n * BWD_L, cv = min(BWD_L, p.T - t0);
    float4* red = s.red + par * BWD_L * K;
    if (ASYNC) {
      cp_async_wait<0>();
      #pragma unroll
      for (int r = 0; r < RPL; ++r) {
        S[r][0] = s.ck[(tid * RPL + r) * BWD_NC];
        S[r][1] = s.ck[(tid * RPL + r) * BWD_NC + 1];
      }
      __syncthreads();  // every thread's copies landed; the previous reduction read the packed rows and dv / dw
      bwd_convert<TIN>(p, s, cv, true);
      __syncthreads();
      if (n > 0) issue_rev(n - 1, true);
    } else {
      #pragma unroll
      for (int r = 0; r < RPL; ++r) {
        const float2 v = ck(n)[r];
        S[r][0] = v.x;
        S[r][1] = v.y;
      }
      __syncthreads();  // the previous reduction read the staged rows and dv / dw
      bwd_stage<TIN>(p, s, bb, hv, kh, col0, t0, cv, true);
      __syncthreads();
    }

    // replay: each token's incoming state and u, in registers
    float H[BWD_L][RPL][BWD_NC], U[BWD_L][BWD_NC];
    #pragma unroll
    for (int tt = 0; tt < BWD_L; ++tt) {
      #pragma unroll
      for (int r = 0; r < RPL; ++r)
        #pragma unroll
        for (int c = 0; c < BWD_NC; ++c) H[tt][r][c] = S[r][c];
      bwd_fwd_step<RPL>(s, K, VT, tt, lane, cw, S, U[tt]);
    }

    // adjoint, last token first (tokens past the end have dO = 0, k = b = 0, gamma = 1: identity steps)
    #pragma unroll
    for (int tt = BWD_L - 1; tt >= 0; --tt) {
      float4 col[BWD_NC];
      float du[BWD_NC];
      #pragma unroll
      for (int c = 0; c < BWD_NC; ++c) {
        col[c] = s.vc[tt * VT + cw + c];
        du[c] = 0.f;
      }
      float4 row[RPL];
      float pq[RPL], pk[RPL];
      #pragma unroll
      for (int r = 0; r < RPL; ++r) {
        row[r] = s.kr[tt * K + lane + 32 * r];
        const float gr = row[r].x, kr = row[r].z, qs = row[r].w;
        pq[r] = 0.f;
        pk[r] = 0.f;
        #pragma unroll
        for (int c = 0; c < BWD_NC; ++c) {
          const float st = gr * H[tt][r][c] + kr * U[tt][c];
          dS[r][c] += qs * col[c].y;
          pq[r] += st * col[c].y;
          du[c] += dS[r][c] * kr;
          pk[r] += dS[r][c] * U[tt][c];
        }
      }
      #pragma unroll
      for (int c = 0; c < BWD_NC; ++c) du[c] = warp_sum_bwd(du[c]);
      #pragma unroll
      for (int r = 0; r < RPL; ++r) {
        const float gr = row[r].x, bkr = row[r].y * row[r].z;
        float pb = 0.f, pg = 0.f;
        #pragma unroll
        for (int c = 0; c < BWD_NC; ++c) {
          const float sa = gr * H[tt][r][c];
          const float dsa = dS[r][c] - bkr * du[c];
          pb -= sa * du[c];
          pg += dsa * sa;
          dS[r][c] = gr * dsa;
        }
        s.slot[((tt & 1) * p.NW + warp) * K + lane + 32 * r] = make_float4(p.scale * pq[r], pk[r], pb, pg);
      }
      if (lane == 0) {
        #pragma unroll
        for (int c = 0; c < BWD_NC; ++c) {
          s.dv[tt * VT + cw + c] = du[c] * col[c].z;
          s.dw[tt * VT + cw + c] = du[c] * col[c].w;
        }
      }
      // the warps' partials of this token summed into the sub-chunk buffer (the slot of this token parity is
      // rewritten two tokens later, after the next token's barrier, by which time every thread has read it)
      __syncthreads();
      const float4* sl = s.slot + (tt & 1) * p.NW * K;
      for (int i = tid; i < K; i += nth) {
        float4 acc = sl[i];
        for (int x = 1; x < p.NW; ++x) {
          const float4 y = sl[x * K + i];
          acc.x += y.x; acc.y += y.y; acc.z += y.z; acc.w += y.w;
        }
        red[tt * K + i] = acc;
      }
    }

    // every CTA of the chain has written its buffer for this sub-chunk (and finished reading the other one,
    // which the next sub-chunk rewrites)
    __syncthreads();
    cl.sync();
    const int per = (cv * K + NCL - 1) / NCL;
    for (int i = rank * per + tid; i < min((rank + 1) * per, cv * K); i += nth) {
      const int tt = i / K, kk = i - tt * K;
      float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
      #pragma unroll
      for (int x = 0; x < 8; ++x) {
        if (x < NCL) {
          const float4 y = cl.map_shared_rank(red, x)[i];
          a.x += y.x; a.y += y.y; a.z += y.z; a.w += y.w;
        }
      }
      const float4 rw = s.kr[i];
      vstore<float>(p.dq, bb, hv, t0 + tt, kk, a.x);
      vstore<float>(p.dk, bb, hv, t0 + tt, kk, a.y + a.z * rw.y);
      vstore<float>(p.db, bb, hv, t0 + tt, kk, a.z * rw.z);
      vstore<float>(p.dg, bb, hv, t0 + tt, kk, a.w);
    }
    for (int i = tid; i < cv * VT; i += nth) {
      const int tt = i / VT, c = i - tt * VT;
      vstore<float>(p.dv, bb, hv, t0 + tt, col0 + c, s.dv[i]);
      vstore<float>(p.dw, bb, hv, t0 + tt, col0 + c, s.dw[i]);
    }
  }
  if (p.dh0) {
    #pragma unroll
    for (int r = 0; r < RPL; ++r)
      #pragma unroll
      for (int c = 0; c < BWD_NC; ++c) p.dh0[chain * KV + (int64_t)(lane + 32 * r) * p.V + col0 + cw + c] = dS[r][c];
  }
  cl.sync();  // no CTA leaves while a peer may still read its buffers
}

// cp.async staging needs every input row (and the slice's first column) on a 16-byte boundary
static bool view_aligned16(const gdn2_view& v, int es) {
  return ((uintptr_t)v.data % 16) == 0 && (v.stride0 * es) % 16 == 0 && (v.stride1 * es) % 16 == 0 &&
         (v.stride2 * es) % 16 == 0;
}
static bool bwd_inputs_aligned(const gdn2_view& q, const gdn2_view& k, const gdn2_view& v, const gdn2_view& g,
                               const gdn2_view& b, const gdn2_view& w, int es, int vt) {
  return view_aligned16(q, es) && view_aligned16(k, es) && view_aligned16(b, es) && view_aligned16(g, 4) &&
         view_aligned16(v, es) && view_aligned16(w, es) && (vt * es) % 16 == 0;
}

static void bwd_shape(int V, int& ncl, int& vt, int& nw) {
  ncl = V / 16 < 8 ? V / 16 : 8;
  vt = V / ncl;
  nw = vt / BWD_NC;
}

size_t recurrent_bwd_workspace_bytes(const gdn2_dims& d) {
  if (d.batch <= 0 || d.seq_len <= 0 || d.num_v_heads <= 0 || d.head_k_dim <= 0 || d.head_v_dim <= 0) return 0;
  const int64_t ns = (d.seq_len + BWD_L - 1) / BWD_L;
  return (size_t)d.batch * d.num_v_heads * ns * d.head_k_dim * d.head_v_dim * sizeof(float);
}

int launch_recurrent_bwd(const gdn2_recurrent_bwd_args* a, void* ws, size_t ws_bytes, cudaStream_t stream) {
  const gdn2_dims& d = a->dims;
  if (d.batch <= 0 || d.seq_len <= 0 || d.num_heads <= 0 || d.num_v_heads <= 0 || d.head_k_dim <= 0 ||
      d.head_v_dim <= 0)
    return set_error(GDN2_EINVAL, "gdn2_recurrent_bwd: all dims must be > 0");
  if (d.num_v_heads % d.num_heads)
    return set_error(GDN2_EINVAL, "gdn2_recurrent_bwd: num_v_heads %d not a multiple of num_heads %d",
                     d.num_v_heads, d.num_heads);
  if (a->dtype != GDN2_DTYPE_F32 && a->dtype != GDN2_DTYPE_BF16)
    return set_error(GDN2_EINVAL, "gdn2_recurrent_bwd: unknown dtype %d", a->dtype);
  if (!a->q.data || !a->k.data || !a->v.data || !a->g.data || !a->b.data || !a->w.data || !a->d_out.data ||
      !a->dq.data || !a->dk.data || !a->dv.data || !a->dg.data || !a->db.data || !a->dw.data)
    return set_error(GDN2_EINVAL, "gdn2_recurrent_bwd: null tensor pointer");
  const int K = d.head_k_dim, V = d.head_v_dim;
  if (K % 32 || K > 128)
    return set_error(GDN2_EUNSUPPORTED, "gdn2_recurrent_bwd: head_k_dim %d (needs a multiple of 32, <= 128)", K);
  if (V % 16 || V > 256)
    return set_error(GDN2_EUNSUPPORTED, "gdn2_recurrent_bwd: head_v_dim %d (needs a multiple of 16, <= 256)", V);
  const size_t need = recurrent_bwd_workspace_bytes(d);
  if (!ws || ws_bytes < need)
    return set_error(GDN2_EWORKSPACE, "gdn2_recurrent_bwd: workspace of %zu bytes needed, %zu given", need,
                     ws ? ws_bytes : (size_t)0);
  if ((uintptr_t)ws & 7) return set_error(GDN2_EINVAL, "gdn2_recurrent_bwd: workspace must be 8-byte aligned");

  BwdParams p = {};
  p.B = d.batch; p.T = d.seq_len; p.HV = d.num_v_heads; p.K = K; p.V = V;
  p.rep = a->key_heads_grouped ? d.num_v_heads / d.num_heads : 1;
  bwd_shape(V, p.NCL, p.VT, p.NW);
  p.NS = (d.seq_len + BWD_L - 1) / BWD_L;
  p.scale = a->scale;
  p.q = make_dview(a->q); p.k = make_dview(a->k); p.v = make_dview(a->v);
  p.g = make_dview(a->g); p.b = make_dview(a->b); p.w = make_dview(a->w);
  p.dout = make_dview(a->d_out);
  p.dq = make_dview(a->dq); p.dk = make_dview(a->dk); p.dv = make_dview(a->dv);
  p.dg = make_dview(a->dg); p.db = make_dview(a->db); p.dw = make_dview(a->dw);
  p.h0 = a->state_in; p.dht = a->d_state_out; p.dh0 = a->d_state_in;
  p.ckpt = static_cast<float*>(ws);

  const bool bf = a->dtype == GDN2_DTYPE_BF16;
  const int esz = bf ? 2 : 4;
  const bool async = bwd_inputs_aligned(a->q, a->k, a->v, a->g, a->b, a->w, esz, p.VT) && view_aligned16(a->d_out, esz);
  void (*fn)(const BwdParams) = nullptr;
  void (*fck)(const BwdParams) = nullptr;
  auto pick = [&](auto tin) {
    using TIN = decltype(tin);
    switch (K / 32) {
      case 1: fn = async ? k_recurrent_bwd<TIN, 1, true> : k_recurrent_bwd<TIN, 1, false>;
              fck = async ? k_recurrent_bwd_ckpt<TIN, 1, true, false> : k_recurrent_bwd_ckpt<TIN, 1, false, false>; break;
      case 2: fn = async ? k_recurrent_bwd<TIN, 2, true> : k_recurrent_bwd<TIN, 2, false>;
              fck = async ? k_recurrent_bwd_ckpt<TIN, 2, true, false> : k_recurrent_bwd_ckpt<TIN, 2, false, false>; break;
      case 3: fn = async ? k_recurrent_bwd<TIN, 3, true> : k_recurrent_bwd<TIN, 3, false>;
              fck = async ? k_recurrent_bwd_ckpt<TIN, 3, true, false> : k_recurrent_bwd_ckpt<TIN, 3, false, false>; break;
      default: fn = async ? k_recurrent_bwd<TIN, 4, true> : k_recurrent_bwd<TIN, 4, false>;
               fck = async ? k_recurrent_bwd_ckpt<TIN, 4, true, false> : k_recurrent_bwd_ckpt<TIN, 4, false, false>; break;
    }
  };
  if (bf)
    pick(__nv_bfloat16());
  else
    pick(0.f);
  const size_t smem_ck = bwd_ckpt_smem_bytes(K, p.VT, esz);
  cudaError_t e = cudaFuncSetAttribute((const void*)fck, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_ck);
  if (e != cudaSuccess) return check_cuda(e, "gdn2_recurrent_bwd: smem attribute");
  fck<<<dim3(p.NCL, d.num_v_heads, d.batch), p.NW * 32, smem_ck, stream>>>(p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return check_cuda(e, "gdn2_recurrent_bwd checkpoint launch");
  const size_t smem = bwd_smem_bytes(K, p.VT, p.NW, K / 32, esz);
  e = cudaFuncSetAttribute((const void*)fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return check_cuda(e, "gdn2_recurrent_bwd: smem attribute");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.NCL, d.num_v_heads, d.batch);
  cfg.blockDim = dim3(p.NW * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.NCL;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return check_cuda(cudaLaunchKernelEx(&cfg, fn, p), "gdn2_recurrent_bwd launch");
}

int launch_chunk_trajectory(const gdn2_recurrent_args* a, int chunk_size, float* states_out, const gdn2_view& vnew,
                            cudaStream_t stream) {
  const gdn2_dims& d = a->dims;
  if (d.batch <= 0 || d.seq_len <= 0 || d.num_heads <= 0 || d.num_v_heads <= 0 || d.head_k_dim <= 0 ||
      d.head_v_dim <= 0)
    return set_error(GDN2_EINVAL, "gdn2_chunk_trajectory: all dims must be > 0");
  if (d.num_v_heads % d.num_heads)
    return set_error(GDN2_EINVAL, "gdn2_chunk_trajectory: num_v_heads %d not a multiple of num_heads %d",
                     d.num_v_heads, d.num_heads);
  if (a->dtype != GDN2_DTYPE_F32 && a->dtype != GDN2_DTYPE_BF16)
    return set_error(GDN2_EINVAL, "gdn2_chunk_trajectory: unknown dtype %d", a->dtype);
  if (a->prologue != 0) return set_error(GDN2_EINVAL, "gdn2_chunk_trajectory: prologue must be 0");
  if (!a->q.data || !a->k.data || !a->v.data || !a->g.data || !a->b.data || !a->w.data || !states_out)
    return set_error(GDN2_EINVAL, "gdn2_chunk_trajectory: null tensor pointer");
  if (chunk_size < BWD_L || chunk_size % BWD_L)
    return set_error(GDN2_EUNSUPPORTED, "gdn2_chunk_trajectory: chunk_size %d (needs a multiple of %d)", chunk_size,
                     BWD_L);
  if ((uintptr_t)states_out % 8) return set_error(GDN2_EINVAL, "gdn2_chunk_trajectory: states_out not 8-byte aligned");
  const int K = d.head_k_dim, V = d.head_v_dim;
  if (K % 32 || K > 128)
    return set_error(GDN2_EUNSUPPORTED, "gdn2_chunk_trajectory: head_k_dim %d (needs a multiple of 32, <= 128)", K);
  if (V % 16 || V > 256)
    return set_error(GDN2_EUNSUPPORTED, "gdn2_chunk_trajectory: head_v_dim %d (needs a multiple of 16, <= 256)", V);
  BwdParams p = {};
  p.B = d.batch; p.T = d.seq_len; p.HV = d.num_v_heads; p.K = K; p.V = V;
  p.rep = a->key_heads_grouped ? d.num_v_heads / d.num_heads : 1;
  bwd_shape(V, p.NCL, p.VT, p.NW);
  p.NS = (d.seq_len + BWD_L - 1) / BWD_L;
  p.q = make_dview(a->q); p.k = make_dview(a->k); p.v = make_dview(a->v);
  p.g = make_dview(a->g); p.b = make_dview(a->b); p.w = make_dview(a->w);
  p.h0 = a->state;
  p.chunk = chunk_size;
  p.states_out = states_out;
  p.vnew = make_dview(vnew);
  const bool bf = a->dtype == GDN2_DTYPE_BF16;
  const int esz = bf ? 2 : 4;
  const bool async = bwd_inputs_aligned(a->q, a->k, a->v, a->g, a->b, a->w, esz, p.VT);
  void (*fn)(const BwdParams) = nullptr;
  auto pick = [&](auto tin) {
    using TIN = decltype(tin);
    switch (K / 32) {
      case 1: fn = async ? k_recurrent_bwd_ckpt<TIN, 1, true, true> : k_recurrent_bwd_ckpt<TIN, 1, false, true>; break;
      case 2: fn = async ? k_recurrent_bwd_ckpt<TIN, 2, true, true> : k_recurrent_bwd_ckpt<TIN, 2, false, true>; break;
      case 3: fn = async ? k_recurrent_bwd_ckpt<TIN, 3, true, true> : k_recurrent_bwd_ckpt<TIN, 3, false, true>; break;
      default: fn = async ? k_recurrent_bwd_ckpt<TIN, 4, true, true> : k_recurrent_bwd_ckpt<TIN, 4, false, true>; break;
    }
  };
  if (bf)
    pick(__nv_bfloat16());
  else
    pick(0.f);
  const size_t smem = bwd_ckpt_smem_bytes(K, p.VT, esz);
  cudaError_t e = cudaFuncSetAttribute((const void*)fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return check_cuda(e, "gdn2_chunk_trajectory: smem attribute");
  fn<<<dim3(p.NCL, d.num_v_heads, d.batch), p.NW * 32, smem, stream>>>(p);
  return check_cuda(cudaGetLastError(), "gdn2_chunk_trajectory launch");
}

}  // namespace gdn2
