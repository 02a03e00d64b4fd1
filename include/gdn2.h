/*
 * gdn2.h — C ABI of the B200 (sm_100a) GDN-2 token-mixer hot path.
 *
 * Drop-in boundary for sehaxe/burn-gdn2 v0.5.1: the crate's host code
 * (Rust) binds these `extern "C"` symbols in place of its cubecl kernels
 * and tensor-op loops.  Plain pointers, sizes and strides only; no CUDA or
 * torch types (a `void* stream` is a `cudaStream_t`).
 *
 * Conventions
 *  - Every entry point returns 0 (GDN2_OK) or a positive gdn2_status.  It
 *    never aborts and never falls back to another implementation; a config
 *    the kernels do not implement returns GDN2_EUNSUPPORTED.  The message
 *    of the last failure on the calling thread is gdn2_last_error().
 *  - Device pointers are caller-owned.  Launches are asynchronous on the
 *    given stream.  Calls on different streams are independent (except
 *    gdn2_chunk_fwd_noalloc, below); the only hidden state is a lazily
 *    built per-device attribute cache and that entry point's scratch.
 *  - Tensors are passed as gdn2_view: a 4-D view [d0][d1][d2][d3] whose
 *    last dim is contiguous and whose first three dims have arbitrary
 *    element strides, so the reference's permuted [B,T,H,K] -> [B,H,T,K]
 *    projections (src/module.rs:395-398) need no copy.
 *  - g (log decay) and the recurrent state are always f32; q k v b w gate
 *    out use `dtype` (f32 or bf16); accumulation is f32.
 */
#ifndef GDN2_H
#define GDN2_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GDN2_ABI_VERSION 2

#if defined(__GNUC__)
#define GDN2_API __attribute__((visibility("default")))
#else
#define GDN2_API
#endif

typedef enum gdn2_status {
  GDN2_OK = 0,
  GDN2_EINVAL = 1,        /* null pointer, bad shape / stride / alignment */
  GDN2_EUNSUPPORTED = 2,  /* valid but not implemented (reported, never downgraded) */
  GDN2_ECUDA = 3,         /* CUDA runtime error, see gdn2_last_cuda_error() */
  GDN2_EWORKSPACE = 4     /* workspace smaller than *_workspace_bytes() */
} gdn2_status;

typedef enum gdn2_dtype { GDN2_DTYPE_F32 = 0, GDN2_DTYPE_BF16 = 1 } gdn2_dtype;

/* Arithmetic of the chunked forward's intermediates (gdn2_chunk_args.precision).
 *  GDN2_PRECISION_F32 (0, the default): every intermediate of the chunk
 *    algorithm is carried at f32 grade (the reference computes in f32,
 *    src/kernel/fused_recurrent_cube.rs:74): on the tensor cores as hi + lo
 *    bf16 operand pairs with f32 accumulation (K = 128, chunk 64,
 *    V in {64, 128}, bf16 or f32 inputs), elsewhere exact f32 on the CUDA
 *    cores.  Meets rel 1e-3 / abs 1e-4 against a float64 restatement.
 *  GDN2_PRECISION_BF16 (1): bf16 inputs only; the per-chunk intermediates
 *    (W, U, Qg, Kd, Aqk, v_new, the state operand) rounded to bf16 once,
 *    on the tensor cores (K = 128, chunk 64, V in {64, 128, 256}): faster,
 *    with a per-head normwise error of about 3e-3.  Other shapes and f32
 *    inputs take the GDN2_PRECISION_F32 path. */
typedef enum gdn2_precision { GDN2_PRECISION_F32 = 0, GDN2_PRECISION_BF16 = 1 } gdn2_precision;

/* 4-D view [d0][d1][d2][d3], d3 contiguous; strides in elements. */
typedef struct gdn2_view {
  void* data;
  int64_t stride0, stride1, stride2;
} gdn2_view;

/* Sizes of one layer call.  H key heads, HV value heads (HV % H == 0). */
typedef struct gdn2_dims {
  int32_t batch;       /* B */
  int32_t seq_len;     /* T */
  int32_t num_heads;   /* H  */
  int32_t num_v_heads; /* HV */
  int32_t head_k_dim;  /* K */
  int32_t head_v_dim;  /* V */
} gdn2_dims;

/* ------------------------------------------------------------------------
 * Chunked forward: kernels (1) chunk-intra and (2) chunk-inter + epilogue.
 * Replaces chunk_wy_forward (src/forward.rs:44-278, called from
 * src/module.rs:269-285 and :354-365) and the unwired cubecl pair
 * cuda::fused_chunk_forward (src/kernel/chunk_cube.rs:781-952).
 *
 *   q, k, b : [B, Hq, T, K] views   (dtype)       Hq = H if key_heads_grouped else HV
 *   g       : [B, Hq, T, K] view    (f32)
 *   v, w    : [B, HV, T, V] views   (dtype)
 *   gate    : [B, HV, T, V] view    (dtype; the module's [B,T,HV,V] storage)
 *   state   : [B, HV, K, V] f32 contiguous, read then overwritten in place
 *   out     : [B, HV, T, V] view    (dtype)
 * key_heads_grouped = 1: value head hv reads key-side head hv / (HV/H)
 * (no materialised GVA repeat).  = 0: the caller passes per-value-head
 * tensors (e.g. the reference's own repeat, src/module.rs:457-468).
 * fuse_epilogue = 1: out = rms_norm_gate_per_head(o, gate, o_norm_weight,
 * norm_eps) (src/module.rs:501-517); = 0: out = o.
 * chunk_size: any value >= 1 (the tuned path is 64).
 * ---------------------------------------------------------------------- */
typedef struct gdn2_chunk_args {
  gdn2_dims dims;
  int32_t chunk_size;
  int32_t dtype;
  int32_t key_heads_grouped;
  int32_t fuse_epilogue;
  float scale;
  float norm_eps;
  gdn2_view q, k, v, g, b, w;
  gdn2_view gate;
  const float* o_norm_weight; /* [V] */
  float* state;
  gdn2_view out;
  int32_t precision; /* gdn2_precision */
} gdn2_chunk_args;

/* Bytes of device workspace gdn2_chunk_fwd / _intra / _inter need. */
GDN2_API size_t gdn2_chunk_fwd_workspace_bytes(const gdn2_chunk_args* args);

/* Full chunked forward (intra, inter, epilogue) on `stream`. */
GDN2_API int gdn2_chunk_fwd(const gdn2_chunk_args* args, void* workspace, size_t workspace_bytes, void* stream);

/* Diagnostics / profiling: the two phases separately.  gdn2_chunk_intra
 * fills the workspace with the per-chunk WY factors; gdn2_chunk_inter
 * consumes them, runs the cross-chunk recurrence and writes out + state.
 * Replaces gdn2_chunk_intra_kernel (src/kernel/chunk_cube.rs:27-295, host
 * :817-887) and gdn2_chunk_inter_kernel (:300-610, host :889-917). */
GDN2_API int gdn2_chunk_intra(const gdn2_chunk_args* args, void* workspace, size_t workspace_bytes, void* stream);
GDN2_API int gdn2_chunk_inter(const gdn2_chunk_args* args, void* workspace, size_t workspace_bytes, void* stream);

/* Size of the scratch array behind gdn2_chunk_fwd_noalloc: 32 MiB per
 * device.  That holds 448 tensor-core chunk records of head_v_dim 128
 * (batch * num_v_heads * ceil(seq_len / 64) <= 448, e.g. 16 value heads
 * over 1792 tokens), or 185 f32 CUDA-core chunks of K = V = 128. */
#define GDN2_NOALLOC_SCRATCH_BYTES ((size_t)32 << 20)

/* The chunked forward of gdn2_chunk_fwd without a caller workspace and
 * without allocating device memory.  No counterpart in the reference: its
 * chunk path allocates its intermediates as tensors on every call.
 *
 * For hosts that cannot allocate device memory at the point of the call: a
 * serving engine that has reserved the device's free memory up front for
 * its own pool, a plugin hook handed only tensor pointers and a stream, or
 * a latency-critical path where cudaMalloc / cudaFree would synchronise
 * the device.
 *
 * The workspace is one file-scope device array of
 * GDN2_NOALLOC_SCRATCH_BYTES, a separate copy on each device.  Like any
 * module-scope device variable it is reserved on a device whenever the
 * library's code is loaded there (at the first launch of any of its
 * kernels with lazy module loading, at context creation with
 * CUDA_MODULE_LOADING=EAGER), whether or not this entry point is ever
 * called, and held until the process exits.  The first call on a device
 * looks up that copy's address (cudaGetSymbolAddress, with the device
 * current) and caches it per device number; make that first call before
 * any stream capture on the device.  The cache assumes the runtime's
 * primary context: after cudaDeviceReset, or when the caller switches to
 * another context of the same device, the cached address is stale.  A
 * call that needs more scratch than the array holds
 * (gdn2_chunk_fwd_workspace_bytes > GDN2_NOALLOC_SCRATCH_BYTES) returns
 * GDN2_EWORKSPACE and launches nothing; argument errors (a dim <= 0, an
 * unknown dtype) return GDN2_EINVAL before that size check.
 *
 * Every call on a device shares the one array, and it keeps the last
 * call's contents: no byte of it needs to start at zero, since each call
 * writes every scratch byte before its kernels read it.  Calls on one
 * stream are ordered and safe; calls whose kernels may overlap on the GPU
 * (different streams without an ordering between them, or host threads
 * using different streams) race on the array and corrupt each other's
 * results. */
GDN2_API int gdn2_chunk_fwd_noalloc(const gdn2_chunk_args* args, void* stream);

/* ------------------------------------------------------------------------
 * Fused recurrent forward: kernel (3).  T >= 1 tokens in one launch with
 * the state held on chip; T == 1 is the decode step.  Replaces
 * fused_recurrent_forward (src/kernel/fused_recurrent.rs:11-56), the decode
 * dispatch fused_recurrent_gdn2 (:65-108) and cuda::fused_step /
 * gdn2_step_kernel (src/kernel/fused_recurrent_cube.rs:15-57, :108-172).
 *
 * prologue = 0: q,k,v are final activations (q,k L2-normalised).
 * prologue = 1: q,k,v are the raw projections ([B,T,C] storage viewed as
 *   [B,Hq,T,K] / [B,HV,T,V]); the kernel applies the kernel-4 causal short
 *   conv + SiLU (src/short_conv.rs:22-65) with the [B,3,C] f32 caches
 *   (conv_*_in NULL = replicate the first token, :42-54) and writes the new
 *   caches to conv_*_out (may alias conv_*_in), then L2-normalises q and k
 *   per head with eps 1e-6 inside the sqrt (src/l2norm.rs:13-16).
 * prologue = 2: SiLU + L2 only (use_short_conv = false, src/module.rs:415).
 * g, b, w are always final (g = log decay, f32).
 * ---------------------------------------------------------------------- */
typedef struct gdn2_recurrent_args {
  gdn2_dims dims;
  int32_t dtype;
  int32_t key_heads_grouped;
  int32_t prologue;
  int32_t fuse_epilogue;
  float scale;
  float norm_eps;
  gdn2_view q, k, v, g, b, w;
  const float* conv_w_q; /* [Hq*K, 4] */
  const float* conv_w_k; /* [Hq*K, 4] */
  const float* conv_w_v; /* [HV*V, 4] */
  const float* conv_q_in;
  const float* conv_k_in;
  const float* conv_v_in;
  float* conv_q_out;
  float* conv_k_out;
  float* conv_v_out;
  gdn2_view gate;
  const float* o_norm_weight;
  float* state; /* [B,HV,K,V] f32, updated in place */
  gdn2_view out;
} gdn2_recurrent_args;

GDN2_API int gdn2_recurrent_fwd(const gdn2_recurrent_args* args, void* stream);

/* ------------------------------------------------------------------------
 * Backward of the core recurrence (exact f32): the reverse-mode adjoint of
 * the per-token scan src/kernel/fused_recurrent.rs:11-56, which is what the
 * crate's burn autodiff differentiates through its tensor path
 * (src/forward.rs:44-278); the crate's own adjoint kernel sketch
 * src/kernel/chunk_adjoint_cube.rs:22-378 is unwired.  For
 *
 *   o_t = scale S_t^T q_t,   S_t = e^{g_t} S_{t-1} + k_t u_t^T,
 *   u_t = w_t v_t - (b_t k_t)^T (e^{g_t} S_{t-1}),   S_0 = state_in
 *
 * given d_out = dL/do and d_state_out = dL/dS_T (NULL = 0), it writes
 * dL/d{q, k, v, g, b, w} and d_state_in = dL/dS_0 (NULL = not written).
 * Inputs as gdn2_recurrent_fwd with prologue = 0 (q, k, g, b are the final,
 * activated values; g is the log decay, f32).  Outputs are f32 views;
 * dq, dk, dg, db are [B, HV, T, K] per VALUE head: with key_heads_grouped =
 * 1 the caller sums each group of HV / H value heads for its key head.
 * K a multiple of 32 up to 128, V a multiple of 16 up to 256.  The
 * workspace (gdn2_recurrent_bwd_workspace_bytes, 8-byte aligned) holds the
 * state at every 8th token: B x HV x ceil(T / 8) x K x V floats.
 * ---------------------------------------------------------------------- */
typedef struct gdn2_recurrent_bwd_args {
  gdn2_dims dims;
  int32_t dtype; /* of q, k, v, b, w and d_out */
  int32_t key_heads_grouped;
  float scale;
  gdn2_view q, k, v, g, b, w;
  const float* state_in;    /* [B,HV,K,V] f32 or NULL (zeros) */
  gdn2_view d_out;          /* [B,HV,T,V] */
  const float* d_state_out; /* [B,HV,K,V] f32 or NULL (zeros) */
  gdn2_view dq, dk, dv, dg, db, dw;
  float* d_state_in; /* [B,HV,K,V] f32 or NULL */
} gdn2_recurrent_bwd_args;

/* Trajectory export for a backward (replaces gdn2_chunk_trajectory_export_kernel,
 * src/kernel/chunk_cube.rs:613-734): from args->state (the initial state,
 * NULL = zeros; not modified) the state entering every chunk of chunk_size
 * tokens, states_out [B, HV, ceil(T / chunk_size), K, V] f32 contiguous,
 * and v_new = w v - (b k)^T (e^g S) of every token into v_new_out
 * ([B, HV, T, V] f32 view; data NULL = not written).  Exact f32.  args as
 * gdn2_recurrent_fwd with prologue = 0 (gate, out, conv and epilogue fields
 * unused); chunk_size a multiple of 8; K and V as gdn2_recurrent_bwd. */
GDN2_API int gdn2_chunk_trajectory(const gdn2_recurrent_args* args, int32_t chunk_size, float* states_out,
                                   gdn2_view v_new_out, void* stream);

GDN2_API size_t gdn2_recurrent_bwd_workspace_bytes(const gdn2_dims* dims);
GDN2_API int gdn2_recurrent_bwd(const gdn2_recurrent_bwd_args* args, void* workspace, size_t workspace_bytes,
                                void* stream);

/* ------------------------------------------------------------------------
 * Projection activations: everything elementwise in GatedDeltaNet2::project
 * (src/module.rs:381-498) between the caller's projection GEMMs and the
 * core, in one launch.  Replaces short_conv_1d (src/short_conv.rs:22-65),
 * the SiLU, l2_normalize_4d (src/l2norm.rs:13-16), the decay
 * g = -exp(A_log) softplus(f + dt_bias) with the min_decay remap
 * (src/module.rs:417-440) and the sigmoid gates (:441-443, b x 2 with
 * allow_neg_eigval :470-472):
 *
 *   q, k = L2(SiLU(conv4(q_raw / k_raw)))   per head of K, eps 1e-6 in the sqrt
 *   v    = SiLU(conv4(v_raw))
 *   b    = sigmoid(b_raw) (x 2 with allow_neg_eigval),   w = sigmoid(w_raw)
 *   g    = -exp(A_log[h]) softplus(f_raw + dt_bias)        (f32)
 *   min_decay >= 0: g = log(sigmoid(decay_factors) (1 - min_decay) e^g + min_decay)
 *
 * use_short_conv = 0 drops conv4 (src/module.rs:415).  Raw inputs are
 * row-major [B*T][ld_*] in `dtype`, channel c at column c (column slices of
 * one concatenated GEMM output work; ld and the base must allow 8-byte bf16
 * / 16-byte f32 vector loads).  Outputs q, k, b: [B*T][H*K], v, w:
 * [B*T][HV*V] contiguous in `dtype`; g: [B*T][H*K] f32.  conv_*_in [B,3,C]
 * f32 or NULL (replicate token 0, src/short_conv.rs:42-54); conv_*_out
 * [B,3,C] f32 or NULL receives the last three raw rows and must not alias
 * conv_*_in.  K <= 256; K and V multiples of 4.
 * ---------------------------------------------------------------------- */
typedef struct gdn2_prologue_args {
  gdn2_dims dims; /* num_heads = key heads H, num_v_heads = HV */
  int32_t dtype;
  int32_t use_short_conv;
  int32_t allow_neg_eigval;
  float min_decay; /* < 0: no remap */
  const void *q_raw, *k_raw, *v_raw, *b_raw, *w_raw, *f_raw;
  int64_t ld_q, ld_k, ld_v, ld_b, ld_w, ld_f;
  const float *conv_w_q, *conv_w_k, *conv_w_v;       /* [C][4] */
  const float *conv_q_in, *conv_k_in, *conv_v_in;    /* [B,3,C] or NULL */
  float *conv_q_out, *conv_k_out, *conv_v_out;       /* [B,3,C] or NULL */
  const float* a_log;         /* [H] */
  const float* dt_bias;       /* [H*K] */
  const float* decay_factors; /* [H*K], read when min_decay >= 0 */
  void *q, *k, *v, *b, *w;
  float* g;
} gdn2_prologue_args;

GDN2_API int gdn2_project_activations(const gdn2_prologue_args* args, void* stream);

/* ------------------------------------------------------------------------
 * Standalone pieces of the layer around the core.
 * ---------------------------------------------------------------------- */
/* short_conv_1d (src/short_conv.rs:22-65): y = silu(causal conv4(x)).
 * x, y: [B,T,C] contiguous (dtype); weight [C,4] f32; cache_in [B,3,C] f32
 * or NULL (replicate first token); cache_out [B,3,C] f32 or NULL. */
GDN2_API int gdn2_short_conv(int32_t batch, int32_t seq_len, int32_t channels, int32_t dtype, const void* x,
                    const float* weight, const float* cache_in, float* cache_out, void* y, void* stream);

/* rms_norm_gate_per_head (src/module.rs:501-517) on [B,HV,T,V] views. */
GDN2_API int gdn2_rms_norm_gate(const gdn2_dims* dims, int32_t dtype, gdn2_view o, gdn2_view gate,
                       const float* weight, float eps, gdn2_view out, void* stream);

/* Mirror of Gdn2Config (src/config.rs:24-58) and its validate()
 * (src/config.rs:71-111).  num_v_heads < 0 means None; min_decay < 0
 * means None; mode 0 = FusedRecurrent, 1 = Chunk. */
typedef struct gdn2_config {
  int64_t hidden_size;
  int64_t num_heads;
  int64_t head_dim;
  float expand_v;
  int64_t num_v_heads;
  int32_t use_short_conv;
  int32_t allow_neg_eigval;
  double norm_eps;
  int32_t mode;
  int64_t chunk_size;
  double min_decay;
} gdn2_config;

/* Returns GDN2_OK or GDN2_EINVAL with the reference's panic message in
 * msg (and in gdn2_last_error()). */
GDN2_API int gdn2_config_validate(const gdn2_config* cfg, char* msg, size_t msg_len);

/* Device-side error bits accumulated since the last call (and cleared):
 * bit 0 = a bounded wait inside a kernel gave up (a bulk copy that never
 * completed); the kernel finished without hanging but its results are
 * invalid.  Synchronises the current device. */
GDN2_API int gdn2_read_device_errors(uint32_t* flags);

/* Diagnostic (no counterpart in the reference): one tcgen05 MMA tile,
 * D[M][N] = A[M][K] . B[K][N] with bf16-rounded operands and f32
 * accumulation, in the shared-memory layout of case `test`:
 *   0: M=128 N=64  K=128, A K-major, B MN-major
 *   1: M=64  N=32  K=128, A K-major, B K-major
 *   2: M=128 N=64  K=64,  A MN-major, B MN-major
 *   3: M=128 N=128 K=64,  A K-major, B MN-major (two N groups)
 * a, b, d: row-major f32 device arrays. */
GDN2_API int gdn2_selftest_umma(int32_t test, const float* a, const float* b, float* d, void* stream);

/* Diagnostic (no counterpart in the reference) of the failure path that
 * every wait inside the kernels shares: one block whose thread 0 waits on
 * an mbarrier with a bounded wait of `spins` try_wait rounds (1..2^24).
 * arrive = 0: nothing arrives, so the wait gives up, sets bit 0 of the
 * device error bits (gdn2_read_device_errors) and the kernel returns
 * normally; *completed = 0.  arrive = 1: the phase completes; *completed
 * = 1.  No trap and no fault either way: the context stays usable.
 * Synchronises the current device. */
GDN2_API int gdn2_selftest_wait(uint32_t spins, int32_t arrive, int32_t* completed);

/* SMs that the split-operand chunk kernels leave free (no counterpart in
 * the reference; default 0).  Those kernels otherwise fill every SM for
 * their duration (two CTAs per SM holding all registers, or one CTA per SM
 * holding most of the shared memory), so a host that runs its own work
 * beside a chunked forward on another stream -- for example the NCCL
 * all-reduce of a head-sharded layer's previous token range -- reserves SMs
 * for it here.  Process-wide, for every device; clamped to [0, 64]; returns
 * the previous value.  The workspace size of a chunk call can depend on it
 * (the chunk-parallel scan sizes its segments by the usable SMs): query the
 * size after changing it. */
GDN2_API int gdn2_set_reserved_sms(int32_t n);

/* Error / version queries. */
GDN2_API const char* gdn2_last_error(void);
GDN2_API int gdn2_last_cuda_error(void);
GDN2_API int gdn2_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* GDN2_H */
