// Projection activations (gdn2_project_activations): the elementwise part of
// GatedDeltaNet2::project (src/module.rs:381-498) in one memory-bound pass.
//
// Two paths.  Full 64-token blocks of the common shapes (every stream a
// whole number of 256-channel slices, K a power of two in [32, 256], rows
// 16-byte aligned) go through the wide persistent kernel further down
// (8 channels per lane, cp.async row rings).  Everything else (a ragged last
// block, odd shapes) goes through the generic kernels described here.
//
// Generic work unit: one warp per (batch, block of PRO_ROWS tokens, stream, head or
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
#include "ptx.cuh"

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
  int tb0;  // first token block this launch covers (the generic kernels take the blocks the wide one does not)
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
  const int nblk = p.ntb - p.tb0;
  if (task >= (int64_t)p.B * nblk * per) return;
  int u = (int)(task % per);
  const int64_t bt = task / per;
  const int tb = p.tb0 + (int)(bt % nblk), bb = (int)(bt / nblk);
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
  const int nblk = p.ntb - p.tb0;
  if (task >= (int64_t)p.B * nblk * per) return;
  int u = (int)(task % per);
  const int64_t bt = task / per;
  const int tb = p.tb0 + (int)(bt % nblk), bb = (int)(bt / nblk);
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

// ---------------------------------------------------------------------------
// Wide path: full PRO_ROWS token blocks, every stream a whole number of
// 256-channel slices, K a power of two in [32, 256], rows 16-byte aligned.
// One warp per (batch, token block, stream, 256-channel slice); lane l owns
// channels 8l..8l+7, so a token's slice is one 512-byte (bf16) access per
// warp and the per-row overheads (addresses, loop, reductions) are shared by
// 8 channels.  Conv and gate streams share one persistent launch.  Each lane
// copies its own 16-byte pieces of the next WIDE_DEPTH - 1 rows into a private
// shared-memory ring with cp.async and reads them back itself, so no barrier
// is needed and the bytes in flight hold no registers.  The q/k L2 norm
// reduces four rows at once over the K/8 lanes of a head: two exchange steps
// leave every lane with a partial sum of one of the four rows
// (reduce-scatter), the remaining steps complete it, one rsqrt per lane, and
// four shuffles hand each lane the four factors.

constexpr int WIDE_DEPTH = 8;  // ring slots per lane: rows in flight + the row being read
constexpr int WIDE_WARPS = 8;

__device__ __forceinline__ void cp16(uint32_t sdst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(sdst), "l"(gsrc) : "memory");
}

__device__ __forceinline__ void unpack2(uint32_t u, float& lo, float& hi) {
  lo = __uint_as_float(u << 16);
  hi = __uint_as_float(u & 0xffff0000u);
}

// A lane's 8 consecutive elements of one row: ring copies (16-byte pieces,
// piece i of all 32 lanes adjacent so the read-back is conflict-free), direct
// non-coherent loads (conv halo) and stores.
template <typename T>
struct Wide;
template <>
struct Wide<__nv_bfloat16> {
  static constexpr int PIECES = 1;
  static __device__ __forceinline__ void fetch(uint32_t s, const __nv_bfloat16* g) { cp16(s, g); }
  static __device__ __forceinline__ void read(const unsigned char* s, float (&x)[8]) {
    const uint4 u = *reinterpret_cast<const uint4*>(s);
    unpack2(u.x, x[0], x[1]);
    unpack2(u.y, x[2], x[3]);
    unpack2(u.z, x[4], x[5]);
    unpack2(u.w, x[6], x[7]);
  }
  static __device__ __forceinline__ void ldg(const __nv_bfloat16* g, float (&x)[8]) {
    uint4 u;
    asm("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(u.x), "=r"(u.y), "=r"(u.z), "=r"(u.w) : "l"(g));
    unpack2(u.x, x[0], x[1]);
    unpack2(u.y, x[2], x[3]);
    unpack2(u.z, x[4], x[5]);
    unpack2(u.w, x[6], x[7]);
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* g, const float (&y)[8]) {
    __nv_bfloat162 h[4];
    #pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(y[2 * i], y[2 * i + 1]);
    *reinterpret_cast<uint4*>(g) = *reinterpret_cast<const uint4*>(h);
  }
};
template <>
struct Wide<float> {
  static constexpr int PIECES = 2;
  static __device__ __forceinline__ void fetch(uint32_t s, const float* g) {
    cp16(s, g);
    cp16(s + 512, g + 4);
  }
  static __device__ __forceinline__ void read(const unsigned char* s, float (&x)[8]) {
    const float4 a = *reinterpret_cast<const float4*>(s);
    const float4 b = *reinterpret_cast<const float4*>(s + 512);
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
    x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
  }
  static __device__ __forceinline__ void ldg(const float* g, float (&x)[8]) {
    Raw4<float> a = ld_raw4(g), b = ld_raw4(g + 4);
    x[0] = a.r.x; x[1] = a.r.y; x[2] = a.r.z; x[3] = a.r.w;
    x[4] = b.r.x; x[5] = b.r.y; x[6] = b.r.z; x[7] = b.r.w;
  }
  static __device__ __forceinline__ void store(float* g, const float (&y)[8]) {
    reinterpret_cast<float4*>(g)[0] = make_float4(y[0], y[1], y[2], y[3]);
    reinterpret_cast<float4*>(g)[1] = make_float4(y[4], y[5], y[6], y[7]);
  }
};

__device__ __forceinline__ void store8_f32(float* g, const float (&y)[8]) { Wide<float>::store(g, y); }

// The ring of one lane: slot s starts at sring + s * SLOT (shared-window
// address for cp.async) and at rring + s * SLOT (generic pointer for reads).
template <typename T>
struct Ring {
  static constexpr int SLOT = Wide<T>::PIECES * 512;
  uint32_t s;
  const unsigned char* r;
};

// Starts the ring on rows src, src + ld, ... (WIDE_DEPTH - 1 of them, row i
// in slot i) and returns the pointer of the next row to fetch.
template <typename T>
__device__ __forceinline__ const T* ring_start(const Ring<T>& rg, const T* src, int64_t ld) {
  #pragma unroll
  for (int r = 0; r < WIDE_DEPTH - 1; ++r) {
    Wide<T>::fetch(rg.s + r * Ring<T>::SLOT, src);
    cp_async_commit();
    src += ld;
  }
  return src;
}

// Row t of the block (slot t % WIDE_DEPTH): first refills the slot of row
// t - 1 with row t + WIDE_DEPTH - 1 (an empty group past the block, so the
// wait count stays uniform), then waits for row t and reads it.
template <typename T>
__device__ __forceinline__ void ring_next(const Ring<T>& rg, int t, const T*& fp, int64_t ld, float (&x)[8]) {
  if (t + WIDE_DEPTH - 1 < PRO_ROWS) {
    Wide<T>::fetch(rg.s + ((t + WIDE_DEPTH - 1) % WIDE_DEPTH) * Ring<T>::SLOT, fp);
    fp += ld;
  }
  cp_async_commit();
  cp_async_wait<WIDE_DEPTH - 1>();
  Wide<T>::read(rg.r + (t % WIDE_DEPTH) * Ring<T>::SLOT, x);
}

// conv4 + SiLU of channels c..c+7 over tokens [t0, t0 + PRO_ROWS), with the
// per-head L2 norm when lph (lanes per head, K / 8) is nonzero (q, k).  One
// loop body serves all three streams and handles four rows, the L2 group;
// the ring slots are runtime indices, so the body stays small enough for
// the instruction cache next to the gate bodies.
template <typename T, bool CONV>
__device__ __forceinline__ void wide_conv(const ProParams& p, const Ring<T>& rg, const T* raw, int64_t ld, int C,
                                          const float* taps, const float* cin, float* cout, T* out, int bb, int t0,
                                          int c, int lane, int lph) {
  const T* src = raw + ((int64_t)bb * p.T + t0) * ld + c;
  const T* fp = ring_start<T>(rg, src, ld);
  float w[8][4], h[3][8];
  if (CONV) {
    #pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 tp = *reinterpret_cast<const float4*>(taps + (int64_t)(c + j) * 4);
      w[j][0] = tp.x; w[j][1] = tp.y; w[j][2] = tp.z; w[j][3] = tp.w;
    }
    if (t0 > 0) {
      #pragma unroll
      for (int i = 0; i < 3; ++i) Wide<T>::ldg(src + (int64_t)(i - 3) * ld, h[i]);
    } else if (cin) {
      #pragma unroll
      for (int i = 0; i < 3; ++i) Wide<float>::ldg(cin + ((int64_t)bb * 3 + i) * C + c, h[i]);
    } else {
      Wide<T>::ldg(src, h[0]);
      #pragma unroll
      for (int j = 0; j < 8; ++j) h[1][j] = h[2][j] = h[0][j];
    }
  }
  // L2 lane pattern (uniform per task): after the exchanges at o1 and o2 the
  // lane holds row (hi1 ? 2 : 0) + (hi2 ? 1 : 0) of the group; row r's sum
  // ends on lane hb + (r & 2 ? o1 : 0) + (r & 1 ? o2 : 0).
  const int o1 = lph >> 1, o2 = lph >> 2;
  const bool hi1 = (lane & o1) != 0, hi2 = (lane & o2) != 0;
  const int hb = lane & ~(lph - 1);
  T* dp = out + ((int64_t)bb * p.T + t0) * C + c;
  #pragma unroll 1
  for (int t4 = 0; t4 < PRO_ROWS; t4 += 4) {
    float y[4][8], ss[4];
    #pragma unroll
    for (int r = 0; r < 4; ++r) {
      float x[8];
      ring_next<T>(rg, t4 + r, fp, ld, x);
      ss[r] = 0.f;
      #pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float s = CONV ? (w[j][0] * h[0][j] + w[j][1] * h[1][j] + w[j][2] * h[2][j] + w[j][3] * x[j]) : x[j];
        y[r][j] = silu_fast(s);
        ss[r] += y[r][j] * y[r][j];
        if (CONV) {
          h[0][j] = h[1][j];
          h[1][j] = h[2][j];
          h[2][j] = x[j];
        }
      }
    }
    if (lph) {
      float a0 = hi1 ? ss[2] : ss[0], a1 = hi1 ? ss[3] : ss[1];
      const float s0 = hi1 ? ss[0] : ss[2], s1 = hi1 ? ss[1] : ss[3];
      a0 += __shfl_xor_sync(0xffffffffu, s0, o1);
      a1 += __shfl_xor_sync(0xffffffffu, s1, o1);
      float kp = hi2 ? a1 : a0;
      kp += __shfl_xor_sync(0xffffffffu, hi2 ? a0 : a1, o2);
      for (int o = lph >> 3; o > 0; o >>= 1) kp += __shfl_xor_sync(0xffffffffu, kp, o);
      const float iv = rsqrtf(kp + 1e-6f);
      #pragma unroll
      for (int r = 0; r < 4; ++r) {
        const float f = __shfl_sync(0xffffffffu, iv, hb + ((r & 2) ? o1 : 0) + ((r & 1) ? o2 : 0));
        #pragma unroll
        for (int j = 0; j < 8; ++j) y[r][j] *= f;
      }
    }
    #pragma unroll
    for (int r = 0; r < 4; ++r) {
      Wide<T>::store(dp, y[r]);
      dp += C;
    }
  }
  if (CONV && cout && t0 + PRO_ROWS == p.T) {
    #pragma unroll
    for (int i = 0; i < 3; ++i) store8_f32(cout + ((int64_t)bb * 3 + i) * C + c, h[i]);
  }
}

// Gate stream of channels c..c+7 over tokens [t0, t0 + PRO_ROWS), the same
// formulas as gate_task: G = false: sigmoid x sc (b with sc = 2 under
// neg-eig, w with sc = 1), out T; G = true: the decay g, out f32.
template <typename T, bool G>
__device__ __forceinline__ void wide_gate(const ProParams& p, const Ring<T>& rg, const T* raw, int64_t ld, int C,
                                          void* out, int bb, int t0, int c, float sc) {
  const T* src = raw + ((int64_t)bb * p.T + t0) * ld + c;
  const T* fp = ring_start<T>(rg, src, ld);
  float dtb[8], fac[8], a = 0.f;
  const bool remap = p.min_decay >= 0.f;
  if (G) {
    a = expf(p.a_log[c / p.K]);  // the 8 channels lie in one head (K % 8 == 0)
    #pragma unroll
    for (int j = 0; j < 8; ++j) {
      dtb[j] = p.dt_bias[c + j];
      fac[j] = 0.f;
      if (remap) fac[j] = sigmoid_f(p.decay[c + j]) * (1.0f - p.min_decay);  // decay may be null otherwise
    }
  }
  const int64_t o0 = ((int64_t)bb * p.T + t0) * C + c;
  #pragma unroll 2
  for (int t = 0; t < PRO_ROWS; ++t) {
    float x[8], o[8];
    ring_next<T>(rg, t, fp, ld, x);
    #pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (G) {
        float gv = -a * softplus_f(x[j] + dtb[j]);
        if (remap) gv = logf(fac[j] * expf(gv) + p.min_decay);
        o[j] = gv;
      } else {
        o[j] = sigmoid_f(x[j]) * sc;
      }
    }
    if (G)
      store8_f32(static_cast<float*>(out) + o0 + (int64_t)t * C, o);
    else
      Wide<T>::store(static_cast<T*>(out) + o0 + (int64_t)t * C, o);
  }
}

// Persistent: warps take (batch, full token block, stream slice) tasks in
// order of task id, the slices of one (batch, block) adjacent: q and k
// (KD / 256 each, L2-normalised), v (VD / 256), b (KD / 256), w (VD / 256),
// g (KD / 256).
template <typename T, bool CONV>
__global__ void __launch_bounds__(WIDE_WARPS * 32, 2) k_prologue_wide(const ProParams p, int nfull, int64_t ntask) {
  extern __shared__ __align__(16) unsigned char wring[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int off = (warp * WIDE_DEPTH * Wide<T>::PIECES * 32 + lane) * 16;
  Ring<T> rg;
  rg.s = smem_u32(wring) + off;
  rg.r = wring + off;
  const int KD = p.H * p.K, VD = p.HV * p.V, NQ = KD / 256, NV = VD / 256;
  const int per = 4 * NQ + 2 * NV;
  const int64_t nw = (int64_t)gridDim.x * WIDE_WARPS;
  for (int64_t task = (int64_t)blockIdx.x * WIDE_WARPS + warp; task < ntask; task += nw) {
    const int64_t bt = task / per;
    // the slice order rotated by the block index, so that a warp's successive tasks (task ids nw apart) do
    // not keep landing on the same stream kinds, whose costs differ (L2-normalised conv, conv, sigmoid, softplus)
    int u = (int)((task % per + bt) % per);
    const int t0 = (int)(bt % nfull) * PRO_ROWS, bb = (int)(bt / nfull);
    if (u < 2 * NQ + NV) {  // q, k, v
      const int s = u < NQ ? 0 : u < 2 * NQ ? 1 : 2;
      const int c = 256 * (u - s * NQ) + 8 * lane;
      const T* raw = static_cast<const T*>(s == 0 ? p.qr : s == 1 ? p.kr : p.vr);
      const int64_t ld = s == 0 ? p.ldq : s == 1 ? p.ldk : p.ldv;
      const float* taps = s == 0 ? p.cwq : s == 1 ? p.cwk : p.cwv;
      const float* cin = s == 0 ? p.ciq : s == 1 ? p.cik : p.civ;
      float* cout = s == 0 ? p.coq : s == 1 ? p.cok : p.cov;
      T* out = static_cast<T*>(s == 0 ? p.q : s == 1 ? p.k : p.v);
      wide_conv<T, CONV>(p, rg, raw, ld, s == 2 ? VD : KD, taps, cin, cout, out, bb, t0, c, lane,
                         s == 2 ? 0 : p.K / 8);
      continue;
    }
    u -= 2 * NQ + NV;
    if (u < NQ + NV) {  // b, w
      const bool isw = u >= NQ;
      wide_gate<T, false>(p, rg, static_cast<const T*>(isw ? p.wr : p.br), isw ? p.ldw : p.ldb, isw ? VD : KD,
                          isw ? p.w : p.b, bb, t0, 256 * (isw ? u - NQ : u) + 8 * lane,
                          (!isw && p.negeig) ? 2.f : 1.f);
      continue;
    }
    u -= NQ + NV;
    wide_gate<T, true>(p, rg, static_cast<const T*>(p.fr), p.ldf, KD, p.g, bb, t0, 256 * u + 8 * lane, 1.f);
  }
}

bool aligned16(const void* p) { return ((uintptr_t)p % 16) == 0; }

// Whether the wide kernel can take the full token blocks of this call.
template <typename T>
bool wide_ok(const ProParams& p) {
  const int KD = p.H * p.K, VD = p.HV * p.V;
  if (KD % 256 || VD % 256 || (p.K != 32 && p.K != 64 && p.K != 128 && p.K != 256)) return false;
  const void* raws[6] = {p.qr, p.kr, p.vr, p.br, p.wr, p.fr};
  const int64_t lds[6] = {p.ldq, p.ldk, p.ldv, p.ldb, p.ldw, p.ldf};
  for (int i = 0; i < 6; ++i)
    if (!aligned16(raws[i]) || (lds[i] * (int64_t)sizeof(T)) % 16) return false;
  const void* outs[6] = {p.q, p.k, p.v, p.b, p.w, p.g};
  for (int i = 0; i < 6; ++i)
    if (!aligned16(outs[i])) return false;
  return true;
}

template <typename T, bool CONV>
int launch_wide(const ProParams& p, int nfull, cudaStream_t st) {
  const int KD = p.H * p.K, VD = p.HV * p.V;
  const int64_t ntask = (int64_t)p.B * nfull * (4 * (KD / 256) + 2 * (VD / 256));
  const int smem = WIDE_WARPS * WIDE_DEPTH * Wide<T>::PIECES * 512;
  void (*fn)(const ProParams, int, int64_t) = k_prologue_wide<T, CONV>;
  cudaError_t e = cudaFuncSetAttribute((const void*)fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return check_cuda(e, "project activations (wide): smem attribute");
  int dev = 0, sms = 0, per_sm = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, WIDE_WARPS * 32, smem);
  if (e != cudaSuccess) return check_cuda(e, "project activations (wide): occupancy");
  int64_t grid = (int64_t)sms * (per_sm > 0 ? per_sm : 1);
  const int64_t need = (ntask + WIDE_WARPS - 1) / WIDE_WARPS;
  if (grid > need) grid = need;
  fn<<<(unsigned)grid, WIDE_WARPS * 32, smem, st>>>(p, nfull, ntask);
  return check_cuda(cudaGetLastError(), "project activations (wide) launch");
}

template <typename T, int NGK>
int launch_t(const ProParams& p0, cudaStream_t st) {
  ProParams p = p0;
  // Full token blocks through the wide kernel when the shapes allow; the
  // generic kernels take the rest (a ragged last block, or everything).
  const int nfull = wide_ok<T>(p) ? p.T / PRO_ROWS : 0;
  if (nfull > 0) {
    const int rc = p.use_conv ? launch_wide<T, true>(p, nfull, st) : launch_wide<T, false>(p, nfull, st);
    if (rc) return rc;
  }
  p.tb0 = nfull;
  if (p.tb0 == p.ntb) return 0;
  const int KD = p.H * p.K, VD = p.HV * p.V;
  const int SK = (KD + 127) / 128, SV = (VD + 127) / 128;
  const int64_t conv_tasks = (int64_t)p.B * (p.ntb - p.tb0) * (2 * p.H + SV);
  const int64_t gate_tasks = (int64_t)p.B * (p.ntb - p.tb0) * (2 * SK + SV);
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
  p.tb0 = 0;
  return a->dtype == GDN2_DTYPE_BF16 ? launch_dt<__nv_bfloat16>(p, st) : launch_dt<float>(p, st);
}

}  // namespace gdn2
