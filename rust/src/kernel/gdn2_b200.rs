//! FFI binding of `libgdn2_b200.so`, the B200 (sm_100a) GDN-2 hot path, declared in `include/gdn2.h`.
//!
//! Every structure is `#[repr(C)]` with the header's field order; every entry point returns a `gdn2_status`
//! (0 = ok) and never falls back to another implementation.  Not compiled here (no Rust toolchain in this
//! image); `tests/test_rust_shim.py` checks the layouts against the header.
#![allow(non_camel_case_types)]

use std::ffi::{c_char, c_void, CStr};

pub const GDN2_ABI_VERSION: i32 = 2;

pub const GDN2_OK: i32 = 0;
pub const GDN2_EINVAL: i32 = 1;
pub const GDN2_EUNSUPPORTED: i32 = 2;
pub const GDN2_ECUDA: i32 = 3;
pub const GDN2_EWORKSPACE: i32 = 4;

pub const GDN2_DTYPE_F32: i32 = 0;
pub const GDN2_DTYPE_BF16: i32 = 1;

pub const GDN2_PRECISION_F32: i32 = 0;
pub const GDN2_PRECISION_BF16: i32 = 1;

pub const GDN2_NOALLOC_SCRATCH_BYTES: usize = 32 << 20;

/// 4-D view `[d0][d1][d2][d3]`, `d3` contiguous, strides in elements.
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct Gdn2View {
    pub data: *mut c_void,
    pub stride0: i64,
    pub stride1: i64,
    pub stride2: i64,
}

impl Default for Gdn2View {
    fn default() -> Self {
        Gdn2View { data: std::ptr::null_mut(), stride0: 0, stride1: 0, stride2: 0 }
    }
}

#[repr(C)]
#[derive(Clone, Copy, Debug, Default)]
pub struct Gdn2Dims {
    pub batch: i32,
    pub seq_len: i32,
    pub num_heads: i32,
    pub num_v_heads: i32,
    pub head_k_dim: i32,
    pub head_v_dim: i32,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct Gdn2ChunkArgs {
    pub dims: Gdn2Dims,
    pub chunk_size: i32,
    pub dtype: i32,
    pub key_heads_grouped: i32,
    pub fuse_epilogue: i32,
    pub scale: f32,
    pub norm_eps: f32,
    pub q: Gdn2View,
    pub k: Gdn2View,
    pub v: Gdn2View,
    pub g: Gdn2View,
    pub b: Gdn2View,
    pub w: Gdn2View,
    pub gate: Gdn2View,
    pub o_norm_weight: *const f32,
    pub state: *mut f32,
    pub out: Gdn2View,
    pub precision: i32,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct Gdn2RecurrentArgs {
    pub dims: Gdn2Dims,
    pub dtype: i32,
    pub key_heads_grouped: i32,
    pub prologue: i32,
    pub fuse_epilogue: i32,
    pub scale: f32,
    pub norm_eps: f32,
    pub q: Gdn2View,
    pub k: Gdn2View,
    pub v: Gdn2View,
    pub g: Gdn2View,
    pub b: Gdn2View,
    pub w: Gdn2View,
    pub conv_w_q: *const f32,
    pub conv_w_k: *const f32,
    pub conv_w_v: *const f32,
    pub conv_q_in: *const f32,
    pub conv_k_in: *const f32,
    pub conv_v_in: *const f32,
    pub conv_q_out: *mut f32,
    pub conv_k_out: *mut f32,
    pub conv_v_out: *mut f32,
    pub gate: Gdn2View,
    pub o_norm_weight: *const f32,
    pub state: *mut f32,
    pub out: Gdn2View,
}

/// Backward of the core recurrence (`gdn2_recurrent_bwd`): dq, dk, dg, db are
/// per value head; with `key_heads_grouped` the caller sums each group.
#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct Gdn2RecurrentBwdArgs {
    pub dims: Gdn2Dims,
    pub dtype: i32,
    pub key_heads_grouped: i32,
    pub scale: f32,
    pub q: Gdn2View,
    pub k: Gdn2View,
    pub v: Gdn2View,
    pub g: Gdn2View,
    pub b: Gdn2View,
    pub w: Gdn2View,
    pub state_in: *const f32,
    pub d_out: Gdn2View,
    pub d_state_out: *const f32,
    pub dq: Gdn2View,
    pub dk: Gdn2View,
    pub dv: Gdn2View,
    pub dg: Gdn2View,
    pub db: Gdn2View,
    pub dw: Gdn2View,
    pub d_state_in: *mut f32,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct Gdn2PrologueArgs {
    pub dims: Gdn2Dims,
    pub dtype: i32,
    pub use_short_conv: i32,
    pub allow_neg_eigval: i32,
    pub min_decay: f32,
    pub q_raw: *const c_void,
    pub k_raw: *const c_void,
    pub v_raw: *const c_void,
    pub b_raw: *const c_void,
    pub w_raw: *const c_void,
    pub f_raw: *const c_void,
    pub ld_q: i64,
    pub ld_k: i64,
    pub ld_v: i64,
    pub ld_b: i64,
    pub ld_w: i64,
    pub ld_f: i64,
    pub conv_w_q: *const f32,
    pub conv_w_k: *const f32,
    pub conv_w_v: *const f32,
    pub conv_q_in: *const f32,
    pub conv_k_in: *const f32,
    pub conv_v_in: *const f32,
    pub conv_q_out: *mut f32,
    pub conv_k_out: *mut f32,
    pub conv_v_out: *mut f32,
    pub a_log: *const f32,
    pub dt_bias: *const f32,
    pub decay_factors: *const f32,
    pub q: *mut c_void,
    pub k: *mut c_void,
    pub v: *mut c_void,
    pub b: *mut c_void,
    pub w: *mut c_void,
    pub g: *mut f32,
}

#[repr(C)]
#[derive(Clone, Copy, Debug)]
pub struct Gdn2Config {
    pub hidden_size: i64,
    pub num_heads: i64,
    pub head_dim: i64,
    pub expand_v: f32,
    pub num_v_heads: i64,
    pub use_short_conv: i32,
    pub allow_neg_eigval: i32,
    pub norm_eps: f64,
    pub mode: i32,
    pub chunk_size: i64,
    pub min_decay: f64,
}

#[link(name = "gdn2_b200")]
extern "C" {
    pub fn gdn2_chunk_fwd_workspace_bytes(args: *const Gdn2ChunkArgs) -> usize;
    pub fn gdn2_chunk_fwd(args: *const Gdn2ChunkArgs, ws: *mut c_void, ws_bytes: usize, stream: *mut c_void) -> i32;
    pub fn gdn2_chunk_intra(args: *const Gdn2ChunkArgs, ws: *mut c_void, ws_bytes: usize, stream: *mut c_void)
        -> i32;
    pub fn gdn2_chunk_inter(args: *const Gdn2ChunkArgs, ws: *mut c_void, ws_bytes: usize, stream: *mut c_void)
        -> i32;
    pub fn gdn2_chunk_fwd_noalloc(args: *const Gdn2ChunkArgs, stream: *mut c_void) -> i32;
    pub fn gdn2_recurrent_fwd(args: *const Gdn2RecurrentArgs, stream: *mut c_void) -> i32;
    pub fn gdn2_chunk_trajectory(args: *const Gdn2RecurrentArgs, chunk_size: i32, states_out: *mut f32,
                                 v_new_out: Gdn2View, stream: *mut c_void) -> i32;
    pub fn gdn2_recurrent_bwd_workspace_bytes(dims: *const Gdn2Dims) -> usize;
    pub fn gdn2_recurrent_bwd(args: *const Gdn2RecurrentBwdArgs, workspace: *mut c_void, workspace_bytes: usize,
                              stream: *mut c_void) -> i32;
    pub fn gdn2_project_activations(args: *const Gdn2PrologueArgs, stream: *mut c_void) -> i32;
    pub fn gdn2_short_conv(batch: i32, seq_len: i32, channels: i32, dtype: i32, x: *const c_void,
                           weight: *const f32, cache_in: *const f32, cache_out: *mut f32, y: *mut c_void,
                           stream: *mut c_void) -> i32;
    pub fn gdn2_rms_norm_gate(dims: *const Gdn2Dims, dtype: i32, o: Gdn2View, gate: Gdn2View, weight: *const f32,
                              eps: f32, out: Gdn2View, stream: *mut c_void) -> i32;
    pub fn gdn2_config_validate(cfg: *const Gdn2Config, msg: *mut c_char, msg_len: usize) -> i32;
    pub fn gdn2_read_device_errors(flags: *mut u32) -> i32;
    pub fn gdn2_selftest_umma(test: i32, a: *const f32, b: *const f32, d: *mut f32, stream: *mut c_void) -> i32;
    pub fn gdn2_selftest_wait(spins: u32, arrive: i32, completed: *mut i32) -> i32;
    pub fn gdn2_set_reserved_sms(n: i32) -> i32;
    pub fn gdn2_last_error() -> *const c_char;
    pub fn gdn2_last_cuda_error() -> i32;
    pub fn gdn2_abi_version() -> i32;
}

/// A non-zero `gdn2_status` with the library's message for it.
#[derive(Debug, Clone)]
pub struct Gdn2Error {
    pub status: i32,
    pub message: String,
}

impl std::fmt::Display for Gdn2Error {
    fn fmt(&self, f: &mut std::fmt::Formatter<'_>) -> std::fmt::Result {
        write!(f, "gdn2 status {}: {}", self.status, self.message)
    }
}

impl std::error::Error for Gdn2Error {}

/// `Ok(())` for `GDN2_OK`, else the status with `gdn2_last_error()` of this thread.
pub fn check(status: i32) -> Result<(), Gdn2Error> {
    if status == GDN2_OK {
        return Ok(());
    }
    // SAFETY: gdn2_last_error returns a NUL-terminated thread-local buffer that lives until the next call.
    let message = unsafe { CStr::from_ptr(gdn2_last_error()) }.to_string_lossy().into_owned();
    Err(Gdn2Error { status, message })
}

/// Chunked forward (intra + inter + fused gated RMS norm) on `stream` with a caller workspace of
/// `gdn2_chunk_fwd_workspace_bytes(args)` bytes.
///
/// # Safety
/// Every pointer in `args`, `ws` and `stream` must be valid device memory / a live CUDA stream of the current
/// device for the duration of the launch.
pub unsafe fn chunk_fwd(args: &Gdn2ChunkArgs, ws: *mut c_void, ws_bytes: usize, stream: *mut c_void)
    -> Result<(), Gdn2Error> {
    check(gdn2_chunk_fwd(args, ws, ws_bytes, stream))
}

/// Fused recurrent forward / decode step (kernel 3), state updated in place.
///
/// # Safety
/// As for [`chunk_fwd`].
pub unsafe fn recurrent_fwd(args: &Gdn2RecurrentArgs, stream: *mut c_void) -> Result<(), Gdn2Error> {
    check(gdn2_recurrent_fwd(args, stream))
}
