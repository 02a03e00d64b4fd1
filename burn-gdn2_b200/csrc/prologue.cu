// Projection activations (gdn2_project_activations): the elementwise part of
// GatedDeltaNet2::project (src/module.rs:381-498) in one memory-bound pass.
//
// Work unit: one warp per (batch, block of PRO_ROWS tokens, stream, head or
// 128-channel slice), walking its tokens in order.  Lane l owns channels
// 4l..4l+3 of each 128-channel group, so a token's row is one coalesced
// 256-byte (bf16) access per group.  q and k tasks cover one key head (one
// or two groups) so that the per-head L2 norm is a warp reduction; v, b, w
// and g are per-channel and run over 128-channel slices.  The causal
// kernel-4 conv keeps its three previous raw rows in registers; a task
// reads three halo rows before its first token (cache / replicated token 0
// at t = 0, src/short_conv.rs:42-54).  Inputs are read with non-coherent
// loads that the compiler may schedule ahead of the output stores.
#include <math.h>

#include "common.cuh"

namespace gdn2 {

int check_cuda(cudaError_t e, const char* where);
int set_error(int code, const char* fmt, ...);

namespace {

constexpr int PRO_ROWS = 64;    // tokens per warp task
constexpr int PRO_WARPS = 8;    // warps per CTA

struct ProParams {
  int B, T, H, K, HV, V;
  int use_conv, negeig;
  float min_decay;  // < 0: none
  const void *qr, *kr, *vr, *br, *wr, *fr;
  int64_t ldq, ldk, ldv, ldb, ldw, ldf;
  const float *cwq, *cwk, *cwv;
  const float *ciq, *cik, *civ;
  float *coq, *cok, *cov;
  const float *a_log, *dt_bias, *decay;
  void *q, *k, *v, *b, *w;
  float* g;
  int ntb;  // token blocks per sequence
};

// 4 consecutive elements of a row
template <typename T>
struct Raw4;
template <>
struct Raw4<__nv_bfloat16> {
  uint2 r;
};
template <>
struct Raw4<float> {
  float4 r;
};

__device__ __forceinline__ Raw4<__nv_bfloat16> ld_raw4(const __nv_bfloat16* p) {
  Raw4<__nv_bfloat16> x;
  asm("ld.global.nc.v2.u32 {%0, %1}, [%2];" : "=r"(x.r.x), "=r"(x.r.y) : "l"(p));
  return x;
}
__device__ __forceinline__ Raw4<float> ld_raw4(const float* p) {
  Raw4<float> x;
  asm("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(x.r.x), "=f"(x.r.y), "=f"(x.r.z), "=f"(x.r.w) : "l"(p));
  return x;
}

__device__ __forceinline__ void unpack(const Raw4<__nv_bfloat16>& x, float (&o)[4]) {
  o[0] = __uint_as_float(x.r.x << 16);
  o[1] = __uint_as_float(x.r.x & 0xffff0000u);
  o[2] = __uint_as_float(x.r.y << 16);
  o[3] = __uint_as_float(x.r.y & 0xffff0000u);
}
__device__ __forceinline__ void unpack(const Raw4<float>& x, float (&o)[4]) {
  o[0] = x.r.x; o[1] = x.r.y; o[2] = x.r.z; o[3] = x.r.w;
}

__device__ __forceinline__ void store4(__nv_bfloat16* p, const float (&x)[4]) {
  __nv_bfloat162 a = __floats2bfloat162_rn(x[0], x[1]);
  __nv_bfloat162 b = __floats2bfloat162_rn(x[2], x[3]);
  uint2 u;
  u.x = *reinterpret_cast<uint32_t*>(&a);
  u.y = *reinterpret_cast<uint32_t*>(&b);
  *reinterpret_cast<uint2*>(p) = u;
}
__device__ __forceinline__ void store4(float* p, const float (&x)[4]) {
  *reinterpret_cast<float4*>(p) = make_float4(x[0], x[1], x[2], x[3]);
}

__device__ __forceinline__ float warp_sum(float x) {
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// Approximate reciprocal division (MUFU) instead of the IEEE sequence: the
// results are rounded to bf16 or checked at f32 tolerance, and for x -> -inf
// the reciprocal of +inf is 0, so both functions still go to 0.
__device__ __forceinline__ float sigmoid_f(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// softplus(x) = log(1 + e^x) (burn's activation::softplus, beta 1), with
// y = e^x:
//  - y < 1/8: the alternating series log(1 + y) = y - y^2/2 + y^3/3 - ...
//    up to y^7/7; the truncation error is below y^8/8, i.e. under 1e-7 of
//    the result;
//  - otherwise ln 2 * log2(1 + y) with the hardware base-2 logarithm
//    (lg2.approx, absolute error ~2^-22 against log2(1 + y) >= 0.17);
//  - above 20 the result is x to f32 precision (and e^x could overflow).
// Relative error about 1e-6 over the whole range (checked against numpy).
__device__ __forceinline__ float softplus_f(float x) {
  const float y = __expf(x);
  float s = fmaf(y, 1.f / 7.f, -1.f / 6.f);
  s = fmaf(y, s, 1.f / 5.f);
  s = fmaf(y, s, -1.f / 4.f);
  s = fmaf(y, s, 1.f / 3.f);
  s = fmaf(y, s, -1.f / 2.f);
  s = fmaf(y, s, 1.f);
  const float small = y * s;
  float l2;
  asm("lg2.approx.f32 %0, %1;" : "=f"(l2) : "f"(1.f + y));
  const float large = l2 * 0.6931471805599453f;  // ln 2
  return x > 20.f ? x : (y < 0.125f ? small : large);
}

// Three halo rows (oldest first) of channels c..c+3 before token t0.
template <typename T>
__device__ __forceinline__ void load_halo(const T* raw, int64_t ld, const float* cin, int C, int b, int T_, int t0,
                                          int c, float (&h)[3][4]) {
  if (t0 > 0) {
    #pragma unroll
    for (int i = 0; i < 3; ++i) unpack(ld_raw4(raw + ((int64_t)b * T_ + t0 - 3 + i) * ld + c), h[i]);
  } else if (cin) {
    #pragma unroll
    for (int i = 0; i < 3; ++i) {
      const float4 x = *reinterpret_cast<const float4*>(cin + ((int64_t)b * 3 + i) * C + c);
      h[i][0] = x.x; h[i][1] = x.y; h[i][2] = x.z; h[i][3] = x.w;
    }
  } else {
    float x0[4];
    unpack(ld_raw4(raw + (int64_t)b * T_ * ld + c), x0);
    #pragma unroll
    for (int i = 0; i < 3; ++i) {
      #pragma unroll
      for (int j = 0; j < 4; ++j) h[i][j] = x0[j];
    }
  }
}

__device__ __forceinline__ void store_cache(float* cout, int C, int b, int c, const float (&h)[3][4]) {
  #pragma unroll
  for (int i = 0; i < 3; ++i)
    *reinterpret_cast<float4*>(cout + ((int64_t)b * 3 + i) * C + c) = make_float4(h[i][0], h[i][1], h[i][2], h[i][3]);
}

// conv4 + SiLU of one 4-channel slice; shifts the window.
template <bool CONV>
__device__ __forceinline__ void conv_silu(const float (&w)[4][4], float (&h)[3][4], const float (&x)[4], float (&y)[4]) {
  #pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float s = CONV ? (w[j][0] * h[0][j] + w[j][1] * h[1][j] + w[j][2] * h[2][j] + w[j][3] * x[j]) : x[j];
    y[j] = silu_fast(s);
    h[0][j] = h[1][j];
    h[1][j] = h[2][j];
    h[2][j] = x[j];
  }
}

__device__ __forceinline__ void load_taps(const float* cw, int c, float (&w)[4][4]) {
  #pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float4 t = *reinterpret_cast<const float4*>(cw + (int64_t)(c + j) * 4);
    w[j][0] = t.x; w[j][1] = t.y; w[j][2] = t.z; w[j][3] = t.w;
  }
}

// Rows of one stream are handled in batches of PRO_BATCH, the next batch
// being fetched while the current one is computed.
constexpr int PRO_BATCH = 4;

// conv4 + SiLU stream over tokens [t0, t1), optionally L2-normalised over
// the NG groups (one key head): q, k (L2 = true) and v (L2 = false).
template <typename T, int NG, bool L2, bool CONV>
__device__ __forceinline__ void conv_task(const ProParams& p, const T* raw, int64_t ld, int C, const float* taps,
                                          const float* cin, float* cout, T* out, int bb, int t0, int t1,
                                          const int (&c)[NG], const bool (&on)[NG]) {
  float w[NG][4][4], h[NG][3][4];
  #pragma unroll
  for (int gi = 0; gi < NG; ++gi) {
    #pragma unroll
    for (int i = 0; i < 4; ++i)
      #pragma unroll
      for (int j = 0; j < 4; ++j) {
        w[gi][i][j] = 0.f;
        if (i < 3) h[gi][i][j] = 0.f;
      }
    if (on[gi] && CONV) {
      load_taps(taps, c[gi], w[gi]);
      load_halo<T>(raw, ld, cin, C, bb, p.T, t0, c[gi], h[gi]);
    }
  }
  const T* src = raw + ((int64_t)bb * p.T + t0) * ld;  // row t0
  T* dst_row = out + ((int64_t)bb * p.T + t0) * C;       // row t0
  Raw4<T> cur[PRO_BATCH][NG], nxt[PRO_BATCH][NG];
  auto fetch = [&](int tb, Raw4<T> (&dst)[PRO_BATCH][NG]) {
    const T* rp = src + (int64_t)(tb - t0) * ld;
    #pragma unroll
    for (int r = 0; r < PRO_BATCH; ++r)
      #pragma unroll
      for (int gi = 0; gi < NG; ++gi)
        if (on[gi] && tb + r < t1) dst[r][gi] = ld_raw4(rp + r * ld + c[gi]);
  };
  fetch(t0, cur);
  #pragma unroll 1
  for (int tb = t0; tb < t1; tb += PRO_BATCH) {
    if (tb + PRO_BATCH < t1) fetch(tb + PRO_BATCH, nxt);
    #pragma unroll
    for (int r = 0; r < PRO_BATCH; ++r) {
      const int t = tb + r;
      if (t >= t1) break;  // uniform over the warp
      float y[NG][4];
      float ss = 0.f;
      #pragma unroll
      for (int gi = 0; gi < NG; ++gi) {
        float x[4] = {0.f, 0.f, 0.f, 0.f};  // lanes past the head: taps, window and x are zero, so y = 0
        if (on[gi]) unpack(cur[r][gi], x);
        conv_silu<CONV>(w[gi], h[gi], x, y[gi]);
        #pragma unroll
        for (int j = 0; j < 4; ++j) ss += y[gi][j] * y[gi][j];
      }
      float inv = 1.f;
      if (L2) inv = rsqrtf(warp_sum(ss) + 1e-6f);
      #pragma unroll
      for (int gi = 0; gi < NG; ++gi) {
        if (!on[gi]) continue;
        float o[4];
        #pragma unroll
        for (int j = 0; j < 4; ++j) o[j] = y[gi][j] * inv;
        store4(dst_row + (int64_t)(t - t0) * C + c[gi], o);
      }
    }
    #pragma unroll
    for (int r = 0; r < PRO_BATCH; ++r)
      #pragma unroll
      for (int gi = 0; gi < NG; ++gi) cur[r][gi] = nxt[r][gi];
  }
  if (CONV && cout && t1 == p.T) {
    #pragma unroll
    for (int gi = 0; gi < NG; ++gi)
      if (on[gi]) store_cache(cout, C, bb, c[gi], h[gi]);
  }
}

// Elementwise gate streams over tokens [t0, t1) of channels c..c+3:
// KIND 3 = b (sigmoid, x 2 with neg-eig), 4 = w (sigmoid), 5 = g (decay, f32 out).
template <typename T, int KIND>
__device__ __forceinline__ void gate_task(const ProParams& p, const T* raw, int64_t ld, int C, void* out, int bb,
                                          int t0, int t1, int c, bool on) {
  float dtb[4] = {0.f, 0.f, 0.f, 0.f}, fac[4] = {0.f, 0.f, 0.f, 0.f}, a = 0.f;
  const bool remap = p.min_decay >= 0.f;
  if (KIND == 5 && on) {
    a = expf(p.a_log[c / p.K]);
    #pragma unroll
    for (int j = 0; j < 4; ++j) {
      dtb[j] = p.dt_bias[c + j];
      if (remap) fac[j] = sigmoid_f(p.decay[c + j]) * (1.0f - p.min_decay);
    }
  }
  const float sc = (KIND == 3 && p.negeig) ? 2.f : 1.f;
  const T* src = raw + ((int64_t)bb * p.T + t0) * ld + c;  // row t0
  const int64_t out0 = ((int64_t)bb * p.T + t0) * C + c;
  Raw4<T> cur[PRO_BATCH], nxt[PRO_BATCH];
  auto fetch = [&](int tb, Raw4<T> (&dst)[PRO_BATCH]) {
    const T* rp = src + (int64_t)(tb - t0) * ld;
    #pragma unroll
    for (int r = 0; r < PRO_BATCH; ++r)
      if (on && tb + r < t1) dst[r] = ld_raw4(rp + r * ld);
  };
  fetch(t0, cur);
  #pragma unroll 1
  for (int tb = t0; tb < t1; tb += PRO_BATCH) {
    if (tb + PRO_BATCH < t1) fetch(tb + PRO_BATCH, nxt);
    #pragma unroll
    for (int r = 0; r < PRO_BATCH; ++r) {
      const int t = tb + r;
      if (!on || t >= t1) break;
      float x[4], o[4];
      unpack(cur[r], x);
      #pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (KIND == 5) {
          float gv = -a * softplus_f(x[j] + dtb[j]);
          if (remap) gv = logf(fac[j] * expf(gv) + p.min_decay);
          o[j] = gv;
        } else {
          o[j] = sigmoid_f(x[j]) * sc;
        }
      }
      const int64_t off = out0 + (int64_t)(t - t0) * C;
      if (KIND == 5) store4(static_cast<float*>(out) + off, o);
      else store4(static_cast<T*>(out) + off, o);
    }
    #pragma unroll
    for (int r = 0; r < PRO_BATCH; ++r) cur[r] = nxt[r];
  }
}

// Conv streams, per (batch, token block): H q heads, H k heads, then the
// 128-channel slices of v.
template <typename T, int NGK, bool CONV>
__global__ void __launch_bounds__(PRO_WARPS * 32, 2) k_prologue_conv(const ProParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t task = (int64_t)blockIdx.x * PRO_WARPS + (threadIdx.x >> 5);
  const int KD = p.H * p.K, VD = p.HV * p.V;
  const int SV = (VD + 127) / 128;
  const int per = 2 * p.H + SV;
  if (task >= (int64_t)p.B * p.ntb * per) return;
  int u = (int)(task % per);
  const int64_t bt = task / per;
  const int tb = (int)(bt % p.ntb), bb = (int)(bt / p.ntb);
  const int t0 = tb * PRO_ROWS, t1 = min(p.T, t0 + PRO_ROWS);
  if (u < 2 * p.H) {  // q or k of one key head
    const bool isk = u >= p.H;
    const int h = isk ? u - p.H : u;
    int c[NGK];
    bool on[NGK];
    #pragma unroll
    for (int gi = 0; gi < NGK; ++gi) {
      const int cc = 128 * gi + 4 * lane;
      on[gi] = cc < p.K;
      c[gi] = h * p.K + (on[gi] ? cc : 0);
    }
    conv_task<T, NGK, true, CONV>(p, static_cast<const T*>(isk ? p.kr : p.qr), isk ? p.ldk : p.ldq, KD,
                            isk ? p.cwk : p.cwq, isk ? p.cik : p.ciq, isk ? p.cok : p.coq,
                            static_cast<T*>(isk ? p.k : p.q), bb, t0, t1, c, on);
    return;
  }
  u -= 2 * p.H;
  const int cc = 128 * u + 4 * lane;
  const int c[1] = {cc < VD ? cc : 0};
  const bool on[1] = {cc < VD};
  conv_task<T, 1, false, CONV>(p, static_cast<const T*>(p.vr), p.ldv, VD, p.cwv, p.civ, p.cov, static_cast<T*>(p.v), bb,
                         t0, t1, c, on);
}

// Gate streams, per (batch, token block): 128-channel slices of b, w, g.
template <typename T>
__global__ void __launch_bounds__(PRO_WARPS * 32, 4) k_prologue_gate(const ProParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t task = (int64_t)blockIdx.x * PRO_WARPS + (threadIdx.x >> 5);
  const int KD = p.H * p.K, VD = p.HV * p.V;
  const int SK = (KD + 127) / 128, SV = (VD + 127) / 128;
  const int per = 2 * SK + SV;
  if (task >= (int64_t)p.B * p.ntb * per) return;
  int u = (int)(task % per);
  const int64_t bt = task / per;
  const int tb = (int)(bt % p.ntb), bb = (int)(bt / p.ntb);
  const int t0 = tb * PRO_ROWS, t1 = min(p.T, t0 + PRO_ROWS);
  if (u < SK) {
    const int cc = 128 * u + 4 * lane;
    gate_task<T, 3>(p, static_cast<const T*>(p.br), p.ldb, KD, p.b, bb, t0, t1, cc < KD ? cc : 0, cc < KD);
    return;
  }
  u -= SK;
  if (u < SV) {
    const int cc = 128 * u + 4 * lane;
    gate_task<T, 4>(p, static_cast<const T*>(p.wr), p.ldw, VD, p.w, bb, t0, t1, cc < VD ? cc : 0, cc < VD);
    return;
  }
  u -= SV;
  const int cc = 128 * u + 4 * lane;
  gate_task<T, 5>(p, static_cast<const T*>(p.fr), p.ldf, KD, p.g, bb, t0, t1, cc < KD ? cc : 0, cc < KD);
}

template <typename T, int NGK>
int launch_t(const ProParams& p, cudaStream_t st) {
  const int KD = p.H * p.K, VD = p.HV * p.V;
  const int SK = (KD + 127) / 128, SV = (VD + 127) / 128;
  const int64_t conv_tasks = (int64_t)p.B * p.ntb * (2 * p.H + SV);
  const int64_t gate_tasks = (int64_t)p.B * p.ntb * (2 * SK + SV);
  const unsigned conv_blocks = (unsigned)((conv_tasks + PRO_WARPS - 1) / PRO_WARPS);
  if (p.use_conv)
    k_prologue_conv<T, NGK, true><<<conv_blocks, PRO_WARPS * 32, 0, st>>>(p);
  else
    k_prologue_conv<T, NGK, false><<<conv_blocks, PRO_WARPS * 32, 0, st>>>(p);
  int rc = check_cuda(cudaGetLastError(), "project activations (conv) launch");
  if (rc) return rc;
  k_prologue_gate<T><<<(unsigned)((gate_tasks + PRO_WARPS - 1) / PRO_WARPS), PRO_WARPS * 32, 0, st>>>(p);
  return check_cuda(cudaGetLastError(), "project activations (gates) launch");
}

template <typename T>
int launch_dt(const ProParams& p, cudaStream_t st) {
  return p.K <= 128 ? launch_t<T, 1>(p, st) : launch_t<T, 2>(p, st);
}

bool aligned(const void* p, int bytes) { return ((uintptr_t)p % bytes) == 0; }

}  // namespace

int launch_project_activations(const gdn2_prologue_args* a, cudaStream_t st) {
  const char* fn = "gdn2_project_activations";
  const gdn2_dims& d = a->dims;
  if (d.batch <= 0 || d.seq_len <= 0 || d.num_heads <= 0 || d.num_v_heads <= 0 || d.head_k_dim <= 0 ||
      d.head_v_dim <= 0)
    return set_error(GDN2_EINVAL, "%s: all dims must be > 0", fn);
  if (a->dtype != GDN2_DTYPE_F32 && a->dtype != GDN2_DTYPE_BF16)
    return set_error(GDN2_EINVAL, "%s: unknown dtype %d", fn, a->dtype);
  if (d.head_k_dim % 4 || d.head_v_dim % 4 || d.head_k_dim > 256)
    return set_error(GDN2_EUNSUPPORTED, "%s: head_k_dim=%d / head_v_dim=%d must be multiples of 4, head_k_dim <= 256",
                     fn, d.head_k_dim, d.head_v_dim);
  const void* raws[6] = {a->q_raw, a->k_raw, a->v_raw, a->b_raw, a->w_raw, a->f_raw};
  const int64_t lds[6] = {a->ld_q, a->ld_k, a->ld_v, a->ld_b, a->ld_w, a->ld_f};
  const int64_t widths[6] = {(int64_t)d.num_heads * d.head_k_dim, (int64_t)d.num_heads * d.head_k_dim,
                             (int64_t)d.num_v_heads * d.head_v_dim, (int64_t)d.num_heads * d.head_k_dim,
                             (int64_t)d.num_v_heads * d.head_v_dim, (int64_t)d.num_heads * d.head_k_dim};
  const int vec = a->dtype == GDN2_DTYPE_BF16 ? 8 : 16;
  for (int i = 0; i < 6; ++i) {
    if (!raws[i]) return set_error(GDN2_EINVAL, "%s: null raw input %d", fn, i);
    if (lds[i] < widths[i] || lds[i] % 4 || !aligned(raws[i], vec))
      return set_error(GDN2_EINVAL, "%s: raw input %d needs ld >= %lld, ld %% 4 == 0 and %d-byte alignment", fn, i,
                       (long long)widths[i], vec);
  }
  const void* outs[6] = {a->q, a->k, a->v, a->b, a->w, a->g};
  for (int i = 0; i < 6; ++i)
    if (!outs[i] || !aligned(outs[i], i == 5 ? 16 : vec))
      return set_error(GDN2_EINVAL, "%s: output %d null or not %d-byte aligned", fn, i, i == 5 ? 16 : vec);
  if (!a->a_log || !a->dt_bias || (a->min_decay >= 0.f && !a->decay_factors))
    return set_error(GDN2_EINVAL, "%s: null a_log / dt_bias / decay_factors", fn);
  if (a->use_short_conv) {
    if (!a->conv_w_q || !a->conv_w_k || !a->conv_w_v)
      return set_error(GDN2_EINVAL, "%s: use_short_conv needs conv_w_q/k/v", fn);
    const float* ins[3] = {a->conv_q_in, a->conv_k_in, a->conv_v_in};
    const float* outs3[3] = {a->conv_q_out, a->conv_k_out, a->conv_v_out};
    for (int i = 0; i < 3; ++i) {
      if ((ins[i] && !aligned(ins[i], 16)) || (outs3[i] && !aligned(outs3[i], 16)) ||
          !aligned(i == 0 ? a->conv_w_q : i == 1 ? a->conv_w_k : a->conv_w_v, 16))
        return set_error(GDN2_EINVAL, "%s: conv weights and caches must be 16-byte aligned", fn);
      if (ins[i] && ins[i] == outs3[i])
        return set_error(GDN2_EINVAL, "%s: conv cache %d: out must not alias in", fn, i);
    }
  }
  ProParams p;
  p.B = d.batch; p.T = d.seq_len; p.H = d.num_heads; p.K = d.head_k_dim; p.HV = d.num_v_heads; p.V = d.head_v_dim;
  p.use_conv = a->use_short_conv ? 1 : 0;
  p.negeig = a->allow_neg_eigval ? 1 : 0;
  p.min_decay = a->min_decay;
  p.qr = a->q_raw; p.kr = a->k_raw; p.vr = a->v_raw; p.br = a->b_raw; p.wr = a->w_raw; p.fr = a->f_raw;
  p.ldq = a->ld_q; p.ldk = a->ld_k; p.ldv = a->ld_v; p.ldb = a->ld_b; p.ldw = a->ld_w; p.ldf = a->ld_f;
  p.cwq = a->conv_w_q; p.cwk = a->conv_w_k; p.cwv = a->conv_w_v;
  p.ciq = a->conv_q_in; p.cik = a->conv_k_in; p.civ = a->conv_v_in;
  p.coq = a->conv_q_out; p.cok = a->conv_k_out; p.cov = a->conv_v_out;
  p.a_log = a->a_log; p.dt_bias = a->dt_bias; p.decay = a->decay_factors;
  p.q = a->q; p.k = a->k; p.v = a->v; p.b = a->b; p.w = a->w; p.g = a->g;
  p.ntb = (d.seq_len + PRO_ROWS - 1) / PRO_ROWS;
  return a->dtype == GDN2_DTYPE_BF16 ? launch_dt<__nv_bfloat16>(p, st) : launch_dt<float>(p, st);
}

}  // namespace gdn2
