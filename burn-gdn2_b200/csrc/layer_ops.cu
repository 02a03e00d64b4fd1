// Standalone layer pieces around the core: short conv + SiLU
// (src/short_conv.rs:22-65) and the SiLU-gated RMS norm
// (src/module.rs:501-517).
#include "common.cuh"

namespace gdn2 {

// y[b,t,c] = silu(sum_i w[c,i] * x_pad[b,t+i,c]); x_pad = cache ++ x (or
// x[:,0] replicated three times when there is no cache).  One thread per
// (b, c) walks the sequence with a 3-deep register window.
template <typename T>
__global__ void k_short_conv(int B, int Tn, int C, const T* __restrict__ x, const float* __restrict__ w,
                             const float* __restrict__ cin, float* __restrict__ cout, T* __restrict__ y) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)B * C) return;
  const int c = (int)(idx % C);
  const int b = (int)(idx / C);
  const T* xb = x + (int64_t)b * Tn * C + c;
  T* yb = y + (int64_t)b * Tn * C + c;
  float w0 = w[(int64_t)c * 4 + 0], w1 = w[(int64_t)c * 4 + 1], w2 = w[(int64_t)c * 4 + 2], w3 = w[(int64_t)c * 4 + 3];
  float p0, p1, p2;
  if (cin) {
    p0 = cin[((int64_t)b * 3 + 0) * C + c];
    p1 = cin[((int64_t)b * 3 + 1) * C + c];
    p2 = cin[((int64_t)b * 3 + 2) * C + c];
  } else {
    p0 = p1 = p2 = to_f32<T>(xb[0]);
  }
  for (int t = 0; t < Tn; ++t) {
    const float xt = to_f32<T>(xb[(int64_t)t * C]);
    float acc = 0.f;
    acc += p0 * w0;
    acc += p1 * w1;
    acc += p2 * w2;
    acc += xt * w3;
    yb[(int64_t)t * C] = from_f32<T>(silu_f(acc));
    p0 = p1;
    p1 = p2;
    p2 = xt;
  }
  if (cout) {
    cout[((int64_t)b * 3 + 0) * C + c] = p0;
    cout[((int64_t)b * 3 + 1) * C + c] = p1;
    cout[((int64_t)b * 3 + 2) * C + c] = p2;
  }
}

int launch_short_conv(int B, int Tn, int C, int dtype, const void* x, const float* w, const float* cin, float* cout,
                      void* y, cudaStream_t st) {
  const int64_t n = (int64_t)B * C;
  const int threads = 256;
  dim3 grid((unsigned)((n + threads - 1) / threads));
  if (dtype == GDN2_DTYPE_BF16)
    k_short_conv<__nv_bfloat16><<<grid, threads, 0, st>>>(B, Tn, C, (const __nv_bfloat16*)x, w, cin, cout,
                                                           (__nv_bfloat16*)y);
  else
    k_short_conv<float><<<grid, threads, 0, st>>>(B, Tn, C, (const float*)x, w, cin, cout, (float*)y);
  return check_cuda(cudaGetLastError(), "short conv launch");
}

// One warp per (b, hv, t) row.
template <typename T>
__global__ void k_rms_norm_gate(int B, int HV, int Tn, int V, DView o, DView gate, const float* __restrict__ w,
                                float eps, DView out) {
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= (int64_t)B * HV * Tn) return;
  const int t = (int)(row % Tn);
  const int hv = (int)((row / Tn) % HV);
  const int b = (int)(row / ((int64_t)Tn * HV));
  float ss = 0.f;
  for (int c = lane; c < V; c += 32) {
    const float x = vload<T>(o, b, hv, t, c);
    ss += x * x;
  }
  #pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float rms = sqrtf(ss / (float)V + eps);
  for (int c = lane; c < V; c += 32) {
    const float x = vload<T>(o, b, hv, t, c);
    vstore<T>(out, b, hv, t, c, x / rms * w[c] * silu_f(vload<T>(gate, b, hv, t, c)));
  }
}

int launch_rms_norm_gate(const gdn2_dims& d, int dtype, const gdn2_view& o, const gdn2_view& gate, const float* w,
                         float eps, const gdn2_view& out, cudaStream_t st) {
  const int64_t rows = (int64_t)d.batch * d.num_v_heads * d.seq_len;
  dim3 grid((unsigned)((rows + 7) / 8));
  if (dtype == GDN2_DTYPE_BF16)
    k_rms_norm_gate<__nv_bfloat16><<<grid, 256, 0, st>>>(d.batch, d.num_v_heads, d.seq_len, d.head_v_dim,
                                                         make_dview(o), make_dview(gate), w, eps, make_dview(out));
  else
    k_rms_norm_gate<float><<<grid, 256, 0, st>>>(d.batch, d.num_v_heads, d.seq_len, d.head_v_dim, make_dview(o),
                                                 make_dview(gate), w, eps, make_dview(out));
  return check_cuda(cudaGetLastError(), "rms norm gate launch");
}

}  // namespace gdn2
