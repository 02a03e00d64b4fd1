// C ABI of libgdn2_b200.so (declared in include/gdn2.h): argument checks,
// error reporting and the launch sequences of the three kernels.
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <mutex>

#include "chunk.cuh"
#include "chunk_tc.cuh"
#include "chunk_x3.cuh"
#include "common.cuh"

namespace gdn2 {

static thread_local char g_err[512] = "";
static thread_local int g_cuda_err = 0;

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int check_cuda(cudaError_t e, const char* where) {
  if (e == cudaSuccess) return GDN2_OK;
  g_cuda_err = (int)e;
  return set_error(GDN2_ECUDA, "%s: %s (%d)", where, cudaGetErrorString(e), (int)e);
}

int launch_recurrent(const gdn2_recurrent_args* a, cudaStream_t stream);
int launch_recurrent_bwd(const gdn2_recurrent_bwd_args* a, void* ws, size_t ws_bytes, cudaStream_t stream);
size_t recurrent_bwd_workspace_bytes(const gdn2_dims& d);
int launch_chunk_trajectory(const gdn2_recurrent_args* a, int chunk_size, float* states_out, const gdn2_view& vnew,
                            cudaStream_t stream);
unsigned read_device_errors_recurrent();
unsigned read_device_errors_selftest();
unsigned read_device_errors_intra_tc();
unsigned read_device_errors_inter_tc();
unsigned read_device_errors_intra_x3();
unsigned read_device_errors_inter_x3();
int selftest_umma(int test, const float* A, const float* B, float* D, cudaStream_t st);
int selftest_wait(unsigned spins, int arrive, int* completed);
int launch_short_conv(int B, int Tn, int C, int dtype, const void* x, const float* w, const float* cin, float* cout,
                      void* y, cudaStream_t st);
int launch_rms_norm_gate(const gdn2_dims& d, int dtype, const gdn2_view& o, const gdn2_view& gate, const float* w,
                         float eps, const gdn2_view& out, cudaStream_t st);
int launch_project_activations(const gdn2_prologue_args* a, cudaStream_t st);

static int check_dims(const gdn2_dims& d, const char* fn) {
  if (d.batch <= 0 || d.seq_len <= 0 || d.num_heads <= 0 || d.num_v_heads <= 0 || d.head_k_dim <= 0 ||
      d.head_v_dim <= 0)
    return set_error(GDN2_EINVAL, "%s: all dims must be > 0 (B=%d T=%d H=%d HV=%d K=%d V=%d)", fn, d.batch,
                     d.seq_len, d.num_heads, d.num_v_heads, d.head_k_dim, d.head_v_dim);
  if (d.num_v_heads % d.num_heads)
    return set_error(GDN2_EINVAL, "%s: num_v_heads=%d must be a multiple of num_heads=%d", fn, d.num_v_heads,
                     d.num_heads);
  return GDN2_OK;
}

static bool mult(int64_t x, int m) { return x % m == 0; }
static bool align_ok(const void* ptr, int bytes) { return ((uintptr_t)ptr % bytes) == 0; }

// Views whose rows allow the tensor-core kernels' vector accesses: four
// q/k/b/v/w elements per load (8 bytes bf16, 16 bytes f32), 16-byte g,
// gate and out pieces.
static bool tc_views_ok(const gdn2_chunk_args* a) {
  auto v_ok = [&](const gdn2_view& v, int elems, int bytes) {
    return align_ok(v.data, bytes) && mult(v.stride0, elems) && mult(v.stride1, elems) && mult(v.stride2, elems);
  };
  const int in_b = a->dtype == GDN2_DTYPE_BF16 ? 8 : 16;   // bytes of four input elements
  const int row_e = a->dtype == GDN2_DTYPE_BF16 ? 8 : 4;   // elements of 16 bytes
  if (!v_ok(a->q, 4, in_b) || !v_ok(a->k, 4, in_b) || !v_ok(a->b, 4, in_b) || !v_ok(a->v, 4, in_b) ||
      !v_ok(a->w, 4, in_b))
    return false;
  if (!v_ok(a->g, 4, 16) || !v_ok(a->out, row_e, 16)) return false;
  if (a->fuse_epilogue && !v_ok(a->gate, row_e, 16)) return false;
  return true;
}

// The bf16-intermediate tensor-core path (GDN2_PRECISION_BF16): bf16 inputs,
// K = 128, V in {64, 128, 256}, 64-token chunks.
static bool use_tc(const gdn2_chunk_args* a) {
  const gdn2_dims& d = a->dims;
  const int C = a->chunk_size < CP ? a->chunk_size : CP;
  if (a->precision != GDN2_PRECISION_BF16) return false;
  if (!tc_supported(d.head_k_dim, d.head_v_dim, C, a->dtype)) return false;
  return tc_views_ok(a);
}

// The split-operand tensor-core path (f32-grade intermediates): bf16 or f32
// inputs, K = 128, V in {64, 128, 256}, 64-token chunks.  Every other shape
// runs on the exact-f32 CUDA-core path.
static bool use_x3(const gdn2_chunk_args* a) {
  const gdn2_dims& d = a->dims;
  const int C = a->chunk_size < CP ? a->chunk_size : CP;
  if (use_tc(a)) return false;
  if (!x3_supported(d.head_k_dim, d.head_v_dim, C)) return false;
  return tc_views_ok(a);
}

// Value columns per inter CTA: V <= 128 in one slice, V = 256 in two.
static int tc_vt(int V) { return V > 128 ? 128 : V; }

static size_t rec_bytes(const gdn2_dims& d, bool x3) {
  return x3 ? x3_record_layout(d.head_v_dim).bytes : tc_record_layout(d.head_v_dim).bytes;
}

static std::atomic<int> g_reserved_sms{0};

int usable_sms() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      sms <= 0) {
    cudaGetLastError();
    sms = 148;
  }
  const int r = g_reserved_sms.load(std::memory_order_relaxed);
  return sms - r >= sms / 2 ? sms - r : sms / 2;
}

static int scan_segments(const gdn2_dims& d, bool x3) {
  return x3 ? x3_scan_segments(d.batch, d.num_v_heads, (d.seq_len + TC_C - 1) / TC_C, d.head_v_dim, usable_sms())
            : 1;
}

static size_t tc_workspace_bytes(const gdn2_dims& d, bool x3) {
  const size_t nch = (size_t)d.batch * d.num_v_heads * ((d.seq_len + TC_C - 1) / TC_C);
  return nch * rec_bytes(d, x3) +
         (x3 ? x3_scratch_bytes((long long)nch, d.head_v_dim) +
                   x3_scan_bytes(d.batch, d.num_v_heads, d.head_v_dim, scan_segments(d, true))
             : 0);
}

static int prep_tc(const gdn2_chunk_args* a, void* ws, size_t wsb, TcParams& p, const char* fn, bool x3) {
  const gdn2_dims& d = a->dims;
  const size_t need = tc_workspace_bytes(d, x3);
  if (wsb < need) return set_error(GDN2_EWORKSPACE, "%s: workspace %zu bytes < required %zu", fn, wsb, need);
  p.B = d.batch; p.T = d.seq_len; p.HV = d.num_v_heads; p.V = d.head_v_dim;
  p.NC = (d.seq_len + TC_C - 1) / TC_C;
  p.rep = a->key_heads_grouped ? d.num_v_heads / d.num_heads : 1;
  p.vt = tc_vt(d.head_v_dim);
  p.vsplit = d.head_v_dim / p.vt;
  p.scale = a->scale; p.eps = a->norm_eps;
  p.fuse_epilogue = a->fuse_epilogue;
  p.q = make_dview(a->q); p.k = make_dview(a->k); p.v = make_dview(a->v);
  p.g = make_dview(a->g); p.b = make_dview(a->b); p.w = make_dview(a->w);
  p.gate = make_dview(a->gate); p.out = make_dview(a->out);
  p.onw = a->o_norm_weight;
  p.state = a->state;
  p.rec = static_cast<unsigned char*>(ws);
  p.rec_bytes = rec_bytes(d, x3);
  p.scratch = p.rec + (size_t)p.B * p.HV * p.NC * p.rec_bytes;
  p.nseg = scan_segments(d, x3);
  p.seg_len = (p.NC + p.nseg - 1) / p.nseg;
  p.seg_state = nullptr;
  p.seg_trans = nullptr;
  if (p.nseg > 1) {
    p.seg_state = reinterpret_cast<float*>(p.scratch + x3_scratch_bytes((long long)p.B * p.HV * p.NC, p.V));
    p.seg_trans = p.seg_state + (size_t)p.B * p.HV * p.nseg * TC_K * p.V;
  }
  return GDN2_OK;
}

static int prep_chunk(const gdn2_chunk_args* a, void* ws, size_t wsb, ChunkParams& p, const char* fn) {
  if (!a) return set_error(GDN2_EINVAL, "%s: null args", fn);
  int rc = check_dims(a->dims, fn);
  if (rc) return rc;
  const gdn2_dims& d = a->dims;
  if (a->dtype != GDN2_DTYPE_F32 && a->dtype != GDN2_DTYPE_BF16)
    return set_error(GDN2_EINVAL, "%s: unknown dtype %d", fn, a->dtype);
  if (a->chunk_size <= 0) return set_error(GDN2_EINVAL, "%s: chunk_size must be > 0, got %d", fn, a->chunk_size);
  if (a->precision != GDN2_PRECISION_F32 && a->precision != GDN2_PRECISION_BF16)
    return set_error(GDN2_EINVAL, "%s: unknown precision %d", fn, a->precision);
  if (!a->q.data || !a->k.data || !a->v.data || !a->g.data || !a->b.data || !a->w.data || !a->state ||
      !a->out.data)
    return set_error(GDN2_EINVAL, "%s: null tensor pointer", fn);
  if (a->fuse_epilogue && (!a->gate.data || !a->o_norm_weight))
    return set_error(GDN2_EINVAL, "%s: fuse_epilogue needs gate and o_norm_weight", fn);
  if (((uintptr_t)a->state & 15u) != 0) return set_error(GDN2_EINVAL, "%s: state must be 16-byte aligned", fn);
  if (d.head_v_dim % 4) return set_error(GDN2_EUNSUPPORTED, "%s: head_v_dim=%d not a multiple of 4", fn, d.head_v_dim);
  const int C = a->chunk_size < CP ? a->chunk_size : CP;
  const ChunkWorkspace L = chunk_workspace_layout(d.batch, d.num_v_heads, d.seq_len, d.head_k_dim, d.head_v_dim, C);
  if (!ws) return set_error(GDN2_EINVAL, "%s: null workspace", fn);
  if (!use_tc(a) && !use_x3(a) && wsb < L.total * sizeof(float))
    return set_error(GDN2_EWORKSPACE, "%s: workspace %zu bytes < required %zu", fn, wsb, L.total * sizeof(float));
  if (((uintptr_t)ws & 255u) != 0) return set_error(GDN2_EINVAL, "%s: workspace must be 256-byte aligned", fn);
  p.B = d.batch; p.T = d.seq_len; p.HV = d.num_v_heads; p.K = d.head_k_dim; p.V = d.head_v_dim;
  p.C = C;
  p.NC = (d.seq_len + C - 1) / C;
  p.rep = a->key_heads_grouped ? d.num_v_heads / d.num_heads : 1;
  p.fuse_epilogue = a->fuse_epilogue;
  p.scale = a->scale; p.eps = a->norm_eps;
  p.q = make_dview(a->q); p.k = make_dview(a->k); p.v = make_dview(a->v);
  p.g = make_dview(a->g); p.b = make_dview(a->b); p.w = make_dview(a->w);
  p.gate = make_dview(a->gate); p.out = make_dview(a->out);
  p.onw = a->o_norm_weight;
  p.state = a->state;
  float* base = static_cast<float*>(ws);
  p.ws_aqk = base + L.aqk; p.ws_w = base + L.w; p.ws_u = base + L.u;
  p.ws_qg = base + L.qg; p.ws_kd = base + L.kd; p.ws_gl = base + L.gl; p.ws_o = base + L.o;
  return GDN2_OK;
}

// Workspace of gdn2_chunk_fwd_noalloc: one copy per device, shared by every
// call on that device.  Host code reaches it only through the address that
// cudaGetSymbolAddress returns.
static __device__ __align__(256) unsigned char g_noalloc_scratch[GDN2_NOALLOC_SCRATCH_BYTES];

constexpr int kNoallocMaxDevices = 64;
static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[kNoallocMaxDevices] = {};

// Address of the current device's scratch copy, looked up on the first call
// for that device and cached.
static int noalloc_scratch(void** out, const char* fn) {
  int dev = -1;
  int rc = check_cuda(cudaGetDevice(&dev), fn);
  if (rc) return rc;
  if (dev < 0 || dev >= kNoallocMaxDevices)
    return set_error(GDN2_EUNSUPPORTED, "%s: device %d beyond the %d devices the scratch table covers", fn, dev,
                     kNoallocMaxDevices);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    rc = check_cuda(cudaGetSymbolAddress(&p, g_noalloc_scratch), fn);
    if (rc) return rc;
    if (!p) return set_error(GDN2_ECUDA, "%s: cudaGetSymbolAddress gave a null scratch address", fn);
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return GDN2_OK;
}

}  // namespace gdn2

using namespace gdn2;

extern "C" {

const char* gdn2_last_error(void) { return g_err; }
int gdn2_last_cuda_error(void) { return g_cuda_err; }
int gdn2_abi_version(void) { return GDN2_ABI_VERSION; }

int gdn2_read_device_errors(uint32_t* flags) {
  if (!flags) return set_error(GDN2_EINVAL, "gdn2_read_device_errors: null flags");
  int rc = check_cuda(cudaDeviceSynchronize(), "gdn2_read_device_errors");
  if (rc) return rc;
  *flags = read_device_errors_recurrent() | read_device_errors_selftest() | read_device_errors_intra_tc() |
           read_device_errors_inter_tc() | read_device_errors_intra_x3() | read_device_errors_inter_x3();
  return GDN2_OK;
}

size_t gdn2_chunk_fwd_workspace_bytes(const gdn2_chunk_args* a) {
  if (!a || a->chunk_size <= 0) return 0;
  const gdn2_dims& d = a->dims;
  if (d.batch <= 0 || d.seq_len <= 0 || d.num_heads <= 0 || d.num_v_heads <= 0 || d.head_k_dim <= 0 ||
      d.head_v_dim <= 0)
    return 0;
  if (a->precision != GDN2_PRECISION_F32 && a->precision != GDN2_PRECISION_BF16) return 0;
  if (use_tc(a)) return tc_workspace_bytes(a->dims, false);
  if (use_x3(a)) return tc_workspace_bytes(a->dims, true);
  const int C = a->chunk_size < CP ? a->chunk_size : CP;
  return chunk_workspace_layout(a->dims.batch, a->dims.num_v_heads, a->dims.seq_len, a->dims.head_k_dim,
                                a->dims.head_v_dim, C)
             .total *
         sizeof(float);
}

int gdn2_chunk_intra(const gdn2_chunk_args* a, void* ws, size_t wsb, void* stream) {
  ChunkParams p;
  int rc = prep_chunk(a, ws, wsb, p, "gdn2_chunk_intra");
  if (rc) return rc;
  const bool x3 = use_x3(a);
  if (x3 || use_tc(a)) {
    TcParams t;
    rc = prep_tc(a, ws, wsb, t, "gdn2_chunk_intra", x3);
    if (rc) return rc;
    return x3 ? launch_intra_x3(t, a->dtype, (cudaStream_t)stream) : launch_intra_tc(t, (cudaStream_t)stream);
  }
  return launch_intra_simt(p, a->dtype, (cudaStream_t)stream);
}

int gdn2_chunk_inter(const gdn2_chunk_args* a, void* ws, size_t wsb, void* stream) {
  ChunkParams p;
  int rc = prep_chunk(a, ws, wsb, p, "gdn2_chunk_inter");
  if (rc) return rc;
  const bool x3 = use_x3(a);
  if (x3 || use_tc(a)) {
    TcParams t;
    rc = prep_tc(a, ws, wsb, t, "gdn2_chunk_inter", x3);
    if (rc) return rc;
    return x3 ? launch_inter_x3(t, a->dtype, (cudaStream_t)stream) : launch_inter_tc(t, (cudaStream_t)stream);
  }
  rc = launch_inter_simt(p, (cudaStream_t)stream);
  if (rc) return rc;
  return launch_chunk_out(p, a->dtype, (cudaStream_t)stream);
}

int gdn2_chunk_fwd(const gdn2_chunk_args* a, void* ws, size_t wsb, void* stream) {
  ChunkParams p;
  int rc = prep_chunk(a, ws, wsb, p, "gdn2_chunk_fwd");
  if (rc) return rc;
  const bool x3 = use_x3(a);
  if (x3 || use_tc(a)) {
    TcParams t;
    rc = prep_tc(a, ws, wsb, t, "gdn2_chunk_fwd", x3);
    if (rc) return rc;
    rc = x3 ? launch_intra_x3(t, a->dtype, (cudaStream_t)stream) : launch_intra_tc(t, (cudaStream_t)stream);
    if (rc) return rc;
    return x3 ? launch_inter_x3(t, a->dtype, (cudaStream_t)stream) : launch_inter_tc(t, (cudaStream_t)stream);
  }
  rc = launch_intra_simt(p, a->dtype, (cudaStream_t)stream);
  if (rc) return rc;
  rc = launch_inter_simt(p, (cudaStream_t)stream);
  if (rc) return rc;
  return launch_chunk_out(p, a->dtype, (cudaStream_t)stream);
}

int gdn2_chunk_fwd_noalloc(const gdn2_chunk_args* a, void* stream) {
  const char* fn = "gdn2_chunk_fwd_noalloc";
  if (!a) return set_error(GDN2_EINVAL, "%s: null args", fn);
  // argument errors are reported as such before the size check (a bad dim
  // must not read as "scratch too small")
  int rc = check_dims(a->dims, fn);
  if (rc) return rc;
  if (a->dtype != GDN2_DTYPE_F32 && a->dtype != GDN2_DTYPE_BF16)
    return set_error(GDN2_EINVAL, "%s: unknown dtype %d", fn, a->dtype);
  if (a->chunk_size <= 0) return set_error(GDN2_EINVAL, "%s: chunk_size must be > 0, got %d", fn, a->chunk_size);
  const size_t need = gdn2_chunk_fwd_workspace_bytes(a);
  if (need > GDN2_NOALLOC_SCRATCH_BYTES)
    return set_error(GDN2_EWORKSPACE,
                     "%s: needs %zu bytes of scratch, more than the %zu of the static array; split the batch or "
                     "call gdn2_chunk_fwd with a workspace",
                     fn, need, (size_t)GDN2_NOALLOC_SCRATCH_BYTES);
  void* ws = nullptr;
  rc = noalloc_scratch(&ws, fn);
  if (rc) return rc;
  return gdn2_chunk_fwd(a, ws, GDN2_NOALLOC_SCRATCH_BYTES, stream);
}

int gdn2_selftest_umma(int32_t test, const float* a, const float* b, float* d, void* stream) {
  if (test < 0 || test > 3) return set_error(GDN2_EINVAL, "gdn2_selftest_umma: test %d not in 0..3", test);
  if (!a || !b || !d) return set_error(GDN2_EINVAL, "gdn2_selftest_umma: null pointer");
  return selftest_umma(test, a, b, d, (cudaStream_t)stream);
}

int gdn2_set_reserved_sms(int32_t n) {
  n = n < 0 ? 0 : n > 64 ? 64 : n;
  return g_reserved_sms.exchange(n);
}

int gdn2_selftest_wait(uint32_t spins, int32_t arrive, int32_t* completed) {
  if (!completed) return set_error(GDN2_EINVAL, "gdn2_selftest_wait: null completed");
  if (spins == 0 || spins > (1u << 24))
    return set_error(GDN2_EINVAL, "gdn2_selftest_wait: spins %u not in 1..2^24", spins);
  return selftest_wait(spins, arrive ? 1 : 0, completed);
}

int gdn2_recurrent_fwd(const gdn2_recurrent_args* a, void* stream) {
  if (!a) return set_error(GDN2_EINVAL, "gdn2_recurrent_fwd: null args");
  return launch_recurrent(a, (cudaStream_t)stream);
}

int gdn2_chunk_trajectory(const gdn2_recurrent_args* a, int32_t chunk_size, float* states_out, gdn2_view v_new_out,
                          void* stream) {
  if (!a) return set_error(GDN2_EINVAL, "gdn2_chunk_trajectory: null args");
  return launch_chunk_trajectory(a, chunk_size, states_out, v_new_out, (cudaStream_t)stream);
}

size_t gdn2_recurrent_bwd_workspace_bytes(const gdn2_dims* d) { return d ? recurrent_bwd_workspace_bytes(*d) : 0; }

int gdn2_recurrent_bwd(const gdn2_recurrent_bwd_args* a, void* workspace, size_t workspace_bytes, void* stream) {
  if (!a) return set_error(GDN2_EINVAL, "gdn2_recurrent_bwd: null args");
  return launch_recurrent_bwd(a, workspace, workspace_bytes, (cudaStream_t)stream);
}

int gdn2_project_activations(const gdn2_prologue_args* a, void* stream) {
  if (!a) return set_error(GDN2_EINVAL, "gdn2_project_activations: null args");
  return launch_project_activations(a, (cudaStream_t)stream);
}

int gdn2_short_conv(int32_t batch, int32_t seq_len, int32_t channels, int32_t dtype, const void* x,
                    const float* weight, const float* cache_in, float* cache_out, void* y, void* stream) {
  if (batch <= 0 || seq_len <= 0 || channels <= 0) return set_error(GDN2_EINVAL, "gdn2_short_conv: dims must be > 0");
  if (dtype != GDN2_DTYPE_F32 && dtype != GDN2_DTYPE_BF16)
    return set_error(GDN2_EINVAL, "gdn2_short_conv: unknown dtype %d", dtype);
  if (!x || !weight || !y) return set_error(GDN2_EINVAL, "gdn2_short_conv: null pointer");
  return launch_short_conv(batch, seq_len, channels, dtype, x, weight, cache_in, cache_out, y, (cudaStream_t)stream);
}

int gdn2_rms_norm_gate(const gdn2_dims* dims, int32_t dtype, gdn2_view o, gdn2_view gate, const float* weight,
                       float eps, gdn2_view out, void* stream) {
  if (!dims) return set_error(GDN2_EINVAL, "gdn2_rms_norm_gate: null dims");
  int rc = check_dims(*dims, "gdn2_rms_norm_gate");
  if (rc) return rc;
  if (dtype != GDN2_DTYPE_F32 && dtype != GDN2_DTYPE_BF16)
    return set_error(GDN2_EINVAL, "gdn2_rms_norm_gate: unknown dtype %d", dtype);
  if (!o.data || !gate.data || !weight || !out.data) return set_error(GDN2_EINVAL, "gdn2_rms_norm_gate: null pointer");
  return launch_rms_norm_gate(*dims, dtype, o, gate, weight, eps, out, (cudaStream_t)stream);
}

int gdn2_config_validate(const gdn2_config* c, char* msg, size_t msg_len) {
  int rc = GDN2_OK;
  if (!c) {
    rc = set_error(GDN2_EINVAL, "null config");
  } else if (c->hidden_size <= 0) {
    rc = set_error(GDN2_EINVAL, "hidden_size must be > 0, got %lld", (long long)c->hidden_size);
  } else if (c->num_heads <= 0) {
    rc = set_error(GDN2_EINVAL, "num_heads must be > 0, got %lld", (long long)c->num_heads);
  } else if (c->head_dim <= 0) {
    rc = set_error(GDN2_EINVAL, "head_dim must be > 0, got %lld", (long long)c->head_dim);
  } else {
    const float prod = (float)c->head_dim * c->expand_v;
    if (!(c->expand_v > 0.0f && prod - floorf(prod) == 0.0f)) {
      rc = set_error(GDN2_EINVAL,
                     "expand_v=%g must produce an integer head_v_dim when multiplied by head_dim=%lld (got %g)",
                     (double)c->expand_v, (long long)c->head_dim, (double)prod);
    } else if (c->num_v_heads == 0) {
      rc = set_error(GDN2_EINVAL, "num_v_heads must be > 0, got %lld", (long long)c->num_v_heads);
    } else if (c->num_v_heads > 0 && c->num_v_heads < c->num_heads) {
      rc = set_error(GDN2_EINVAL,
                     "num_v_heads=%lld < num_heads=%lld is not supported; use num_v_heads >= num_heads (GVA "
                     "repeats key-side heads)",
                     (long long)c->num_v_heads, (long long)c->num_heads);
    } else if (c->num_v_heads > 0 && c->num_v_heads % c->num_heads != 0) {
      rc = set_error(GDN2_EINVAL, "num_v_heads=%lld must be divisible by num_heads=%lld", (long long)c->num_v_heads,
                     (long long)c->num_heads);
    } else if (c->chunk_size <= 0) {
      rc = set_error(GDN2_EINVAL, "chunk_size must be > 0, got %lld", (long long)c->chunk_size);
    } else if (!(c->norm_eps > 0.0)) {
      rc = set_error(GDN2_EINVAL, "norm_eps must be > 0, got %g", c->norm_eps);
    }
  }
  if (msg && msg_len) {
    if (rc)
      snprintf(msg, msg_len, "%s", g_err);
    else
      msg[0] = 0;
  }
  return rc;
}

}  // extern "C"
