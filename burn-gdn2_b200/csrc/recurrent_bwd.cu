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
// outputs only: each warp adds its per-row partials into a shared buffer
// (red.shared) and, every 8 tokens, the CTAs of a chain, which form one
// thread-block cluster, sum each other's buffers through distributed shared
// memory and write dq, dk, db, dg once.
//
// States for the reverse pass.  A forward pass over the sequence stores the
// state at every 8th token boundary in the workspace (each thread its own
// 2 x RPL values, in a private layout that makes every warp store 256
// contiguous bytes).  The reverse pass walks the 8-token sub-chunks from the
// last: it reloads the sub-chunk's start state, replays the 8 tokens keeping
// each token's incoming state in registers, then runs the adjoint over
// them.  Work per token is three forward steps and one adjoint step on the
// slice; the workspace is B x HV x ceil(T/8) x K x V floats.
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
};

__device__ __forceinline__ float warp_sum_bwd(float x) {
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

__device__ __forceinline__ void red_shared_add(float* p, float x) {
  asm volatile("red.shared.add.f32 [%0], %1;" ::"r"((uint32_t)__cvta_generic_to_shared(p)), "f"(x) : "memory");
}

// Shared memory (floats): staged inputs of one sub-chunk, the per-column
// outputs dv / dw, and two V-reduction buffers (by sub-chunk parity).
struct BwdSmem {
  float *q, *k, *b, *gm;  // [L][K]  (gm = e^g)
  float *v, *w, *dO;      // [L][VT]
  float *dv, *dw;         // [L][VT]
  float* red;             // [2][L][4][K]: dq, dk (through S_t), dbk, dg partials
};

__host__ __device__ inline size_t bwd_smem_floats(int K, int VT) {
  return (size_t)4 * BWD_L * K + (size_t)5 * BWD_L * VT + (size_t)2 * BWD_L * 4 * K;
}

template <typename TIN>
__device__ __forceinline__ void bwd_stage(const BwdParams& p, const BwdSmem& s, int bb, int hv, int kh, int col0,
                                          int t0, int cv, bool with_dout) {
  const int nth = blockDim.x, tid = threadIdx.x, K = p.K, VT = p.VT;
  for (int i = tid; i < BWD_L * K; i += nth) {
    const int tt = i / K, kk = i - tt * K;
    float qv = 0.f, kv = 0.f, bv = 0.f, gv = 1.f;
    if (tt < cv) {
      qv = vload<TIN>(p.q, bb, kh, t0 + tt, kk);
      kv = vload<TIN>(p.k, bb, kh, t0 + tt, kk);
      bv = vload<TIN>(p.b, bb, kh, t0 + tt, kk);
      gv = expf(vload<float>(p.g, bb, kh, t0 + tt, kk));
    }
    s.q[i] = qv;
    s.k[i] = kv;
    s.b[i] = bv;
    s.gm[i] = gv;
  }
  for (int i = tid; i < BWD_L * VT; i += nth) {
    const int tt = i / VT, c = i - tt * VT;
    float vv = 0.f, wv = 0.f, dv = 0.f;
    if (tt < cv) {
      vv = vload<TIN>(p.v, bb, hv, t0 + tt, col0 + c);
      wv = vload<TIN>(p.w, bb, hv, t0 + tt, col0 + c);
      if (with_dout) dv = vload<TIN>(p.dout, bb, hv, t0 + tt, col0 + c);
    }
    s.v[i] = vv;
    s.w[i] = wv;
    s.dO[i] = dv;
  }
}

// One forward token step on the thread's RPL x NC slice.  Returns u (per column) through `u`.
template <int RPL>
__device__ __forceinline__ void bwd_fwd_step(const BwdSmem& s, int K, int VT, int tt, int lane, int cw,
                                             float (&S)[RPL][BWD_NC], float (&u)[BWD_NC]) {
  float e[BWD_NC];
  #pragma unroll
  for (int c = 0; c < BWD_NC; ++c) e[c] = 0.f;
  #pragma unroll
  for (int r = 0; r < RPL; ++r) {
    const int kk = lane + 32 * r;
    const float gr = s.gm[tt * K + kk], bkr = s.b[tt * K + kk] * s.k[tt * K + kk];
    #pragma unroll
    for (int c = 0; c < BWD_NC; ++c) {
      S[r][c] *= gr;
      e[c] += bkr * S[r][c];
    }
  }
  #pragma unroll
  for (int c = 0; c < BWD_NC; ++c) u[c] = s.w[tt * VT + cw + c] * s.v[tt * VT + cw + c] - warp_sum_bwd(e[c]);
  #pragma unroll
  for (int r = 0; r < RPL; ++r) {
    const float kr = s.k[tt * K + lane + 32 * r];
    #pragma unroll
    for (int c = 0; c < BWD_NC; ++c) S[r][c] += kr * u[c];
  }
}

template <typename TIN, int RPL>
__global__ void __launch_bounds__(512, 1) k_recurrent_bwd(const BwdParams p) {
  extern __shared__ __align__(16) float smf[];
  const int K = p.K, VT = p.VT, NCL = p.NCL;
  BwdSmem s;
  s.q = smf;
  s.k = s.q + BWD_L * K;
  s.b = s.k + BWD_L * K;
  s.gm = s.b + BWD_L * K;
  s.v = s.gm + BWD_L * K;
  s.w = s.v + BWD_L * VT;
  s.dO = s.w + BWD_L * VT;
  s.dv = s.dO + BWD_L * VT;
  s.dw = s.dv + BWD_L * VT;
  s.red = s.dw + BWD_L * VT;

  cg::cluster_group cl = cg::this_cluster();
  const int rank = (int)cl.block_rank();
  const int hv = blockIdx.y, bb = blockIdx.z, kh = hv / p.rep;
  const int col0 = rank * VT;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nth = blockDim.x;
  const int cw = warp * BWD_NC;  // the warp's first column in the slice
  const int64_t chain = (int64_t)bb * p.HV + hv;
  const int64_t KV = (int64_t)K * p.V;

  // this thread's checkpoint slot of sub-chunk n: 256 contiguous bytes per warp and row group
  auto ck = [&](int n, int r) -> float2* {
    const int64_t base = (((chain * p.NS + n) * NCL + rank) * p.NW + warp) * (int64_t)RPL + r;
    return reinterpret_cast<float2*>(p.ckpt + (base * 32 + lane) * BWD_NC);
  };

  // ---- forward pass: the state at every sub-chunk start into the workspace ----
  float S[RPL][BWD_NC];
  #pragma unroll
  for (int r = 0; r < RPL; ++r)
    #pragma unroll
    for (int c = 0; c < BWD_NC; ++c)
      S[r][c] = p.h0 ? p.h0[chain * KV + (int64_t)(lane + 32 * r) * p.V + col0 + cw + c] : 0.f;
  for (int n = 0; n < p.NS; ++n) {
    const int t0 = n * BWD_L, cv = min(BWD_L, p.T - t0);
    #pragma unroll
    for (int r = 0; r < RPL; ++r) *ck(n, r) = make_float2(S[r][0], S[r][1]);
    if (n == p.NS - 1) break;  // the last sub-chunk is replayed from its checkpoint
    bwd_stage<TIN>(p, s, bb, hv, kh, col0, t0, cv, false);
    __syncthreads();
    #pragma unroll
    for (int tt = 0; tt < BWD_L; ++tt) {
      float u[BWD_NC];
      bwd_fwd_step<RPL>(s, K, VT, tt, lane, cw, S, u);
    }
    __syncthreads();
  }

  // ---- reverse pass ----
  float dS[RPL][BWD_NC];
  #pragma unroll
  for (int r = 0; r < RPL; ++r)
    #pragma unroll
    for (int c = 0; c < BWD_NC; ++c)
      dS[r][c] = p.dht ? p.dht[chain * KV + (int64_t)(lane + 32 * r) * p.V + col0 + cw + c] : 0.f;
  for (int i = tid; i < 2 * BWD_L * 4 * K; i += nth) s.red[i] = 0.f;

  for (int it = 0; it < p.NS; ++it) {
    const int n = p.NS - 1 - it, par = it & 1;
    const int t0 = n * BWD_L, cv = min(BWD_L, p.T - t0);
    float* red = s.red + par * BWD_L * 4 * K;
    #pragma unroll
    for (int r = 0; r < RPL; ++r) {
      const float2 v = *ck(n, r);
      S[r][0] = v.x;
      S[r][1] = v.y;
    }
    __syncthreads();  // the previous reduction read the staged k / b / dv / dw
    bwd_stage<TIN>(p, s, bb, hv, kh, col0, t0, cv, true);
    __syncthreads();

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
      float dO[BWD_NC], du[BWD_NC];
      #pragma unroll
      for (int c = 0; c < BWD_NC; ++c) {
        dO[c] = s.dO[tt * VT + cw + c];
        du[c] = 0.f;
      }
      float pq[RPL], pk[RPL];
      #pragma unroll
      for (int r = 0; r < RPL; ++r) {
        const int kk = lane + 32 * r;
        const float gr = s.gm[tt * K + kk], kr = s.k[tt * K + kk], qs = p.scale * s.q[tt * K + kk];
        pq[r] = 0.f;
        pk[r] = 0.f;
        #pragma unroll
        for (int c = 0; c < BWD_NC; ++c) {
          const float st = gr * H[tt][r][c] + kr * U[tt][c];
          dS[r][c] += qs * dO[c];
          pq[r] += st * dO[c];
          du[c] += dS[r][c] * kr;
          pk[r] += dS[r][c] * U[tt][c];
        }
      }
      #pragma unroll
      for (int c = 0; c < BWD_NC; ++c) du[c] = warp_sum_bwd(du[c]);
      #pragma unroll
      for (int r = 0; r < RPL; ++r) {
        const int kk = lane + 32 * r;
        const float gr = s.gm[tt * K + kk], bkr = s.b[tt * K + kk] * s.k[tt * K + kk];
        float pb = 0.f, pg = 0.f;
        #pragma unroll
        for (int c = 0; c < BWD_NC; ++c) {
          const float sa = gr * H[tt][r][c];
          const float dsa = dS[r][c] - bkr * du[c];
          pb -= sa * du[c];
          pg += dsa * sa;
          dS[r][c] = gr * dsa;
        }
        float* rt = red + tt * 4 * K + kk;
        red_shared_add(rt, p.scale * pq[r]);
        red_shared_add(rt + K, pk[r]);
        red_shared_add(rt + 2 * K, pb);
        red_shared_add(rt + 3 * K, pg);
      }
      if (lane == 0) {
        #pragma unroll
        for (int c = 0; c < BWD_NC; ++c) {
          s.dv[tt * VT + cw + c] = du[c] * s.w[tt * VT + cw + c];
          s.dw[tt * VT + cw + c] = du[c] * s.v[tt * VT + cw + c];
        }
      }
    }

    // every CTA of the chain has added its partials for this sub-chunk (and finished reading the other buffer)
    __syncthreads();
    cl.sync();
    float* other = s.red + (par ^ 1) * BWD_L * 4 * K;
    for (int i = tid; i < BWD_L * 4 * K; i += nth) other[i] = 0.f;
    for (int i = rank * nth + tid; i < BWD_L * K; i += NCL * nth) {
      const int tt = i / K, kk = i - tt * K;
      if (tt >= cv) continue;
      float a[4] = {0.f, 0.f, 0.f, 0.f};
      for (int x = 0; x < NCL; ++x) {
        const float* pr = cl.map_shared_rank(red, x) + tt * 4 * K + kk;
        #pragma unroll
        for (int j = 0; j < 4; ++j) a[j] += pr[j * K];
      }
      const float bv = s.b[tt * K + kk], kv = s.k[tt * K + kk];
      vstore<float>(p.dq, bb, hv, t0 + tt, kk, a[0]);
      vstore<float>(p.dk, bb, hv, t0 + tt, kk, a[1] + a[2] * bv);
      vstore<float>(p.db, bb, hv, t0 + tt, kk, a[2] * kv);
      vstore<float>(p.dg, bb, hv, t0 + tt, kk, a[3]);
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

  BwdParams p;
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

  void (*fn)(const BwdParams) = nullptr;
  const bool bf = a->dtype == GDN2_DTYPE_BF16;
  switch (K / 32) {
    case 1: fn = bf ? k_recurrent_bwd<__nv_bfloat16, 1> : k_recurrent_bwd<float, 1>; break;
    case 2: fn = bf ? k_recurrent_bwd<__nv_bfloat16, 2> : k_recurrent_bwd<float, 2>; break;
    case 3: fn = bf ? k_recurrent_bwd<__nv_bfloat16, 3> : k_recurrent_bwd<float, 3>; break;
    default: fn = bf ? k_recurrent_bwd<__nv_bfloat16, 4> : k_recurrent_bwd<float, 4>; break;
  }
  const size_t smem = bwd_smem_floats(K, p.VT) * sizeof(float);
  cudaError_t e = cudaFuncSetAttribute((const void*)fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
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

}  // namespace gdn2
