//! Crate-side dispatch of sehaxe/burn-gdn2 onto `libgdn2_b200.so` (behind the crate's `cuda` feature).
//!
//! * `fused_recurrent_b200` replaces the `cuda::fused_step` branch of `fused_recurrent_gdn2`
//!   (`src/kernel/fused_recurrent.rs:83-97`): any T (T = 1 is the decode step), one launch of kernel (3), the
//!   state updated in place.
//! * `chunk_forward_b200` replaces `chunk_wy_forward` at its two call sites (`src/module.rs:269-285` and
//!   `:354-365`): kernels (1) + (2) with f32-grade intermediates.
//! * Both update the recurrent state tensor in place and return that same tensor, so the assignment
//!   `st.recurrent = new_rec` of `src/module.rs:288-295` hands `Gdn2State` back its own buffer: the state is
//!   carried across calls without a copy.
//!
//! On any backend other than the bare CUDA `CubeBackend` both return `None` and the crate keeps its tensor path
//! (exactly as `cube_of` gates the cubecl kernel today).  On the CUDA backend an error from the library panics
//! with its message (the crate's convention for invalid configurations) instead of falling back.
//!
//! Not compiled here: no Rust toolchain in this image, burn 0.21 / cubecl 0.10 not vendored.  `raw_ptr` is the
//! one place that depends on the cubecl release's accessor of a handle's device address.
use std::any::{Any, TypeId};
use std::ffi::c_void;

use burn::tensor::{backend::Backend, Tensor};
use burn_cubecl::tensor::CubeTensor;

use super::gdn2_b200::*;

type CudaBare = burn_cubecl::CubeBackend<cubecl::cuda::CudaRuntime, f32, i32, u8>;

/// The CubeTensor of `t` when `B` is the bare CUDA backend.
fn cube<B: Backend>(t: &Tensor<B, 4>) -> Option<CubeTensor<cubecl::cuda::CudaRuntime>> {
    if TypeId::of::<B>() != TypeId::of::<CudaBare>() {
        return None;
    }
    let prim = t.clone().into_primitive().tensor();
    (&prim as &dyn Any).downcast_ref::<CubeTensor<cubecl::cuda::CudaRuntime>>().cloned()
}

/// Device address of the tensor's first element (the handle's buffer plus its byte offset).
fn raw_ptr(t: &CubeTensor<cubecl::cuda::CudaRuntime>) -> *mut c_void {
    let res = t.client.get_resource(t.handle.clone().binding());
    (res.resource().ptr as usize + res.resource().offset() as usize) as *mut c_void
}

/// gdn2_view of a 4-D tensor: its own element strides, so the permuted `[B,T,H,K] -> [B,H,T,K]` views of
/// `project` (`src/module.rs:395-398`) reach the kernels without the copy `mul_scalar(1.0)` makes.
fn view(t: &CubeTensor<cubecl::cuda::CudaRuntime>) -> Gdn2View {
    let s = t.meta.strides();
    Gdn2View { data: raw_ptr(t), stride0: s[0] as i64, stride1: s[1] as i64, stride2: s[2] as i64 }
}

/// cubecl launches on its own stream: finish its queued work, run the library on the default stream, and wait
/// for it before cubecl continues.
fn run_on_device(client_sync: impl Fn(), launch: impl FnOnce(*mut c_void) -> i32) {
    client_sync();
    let status = launch(std::ptr::null_mut());
    if let Err(e) = check(status) {
        panic!("libgdn2_b200: {e}");
    }
    let mut flags = 0u32;
    // synchronises the device and reports a bounded wait that gave up inside a kernel
    if let Err(e) = check(unsafe { gdn2_read_device_errors(&mut flags) }) {
        panic!("libgdn2_b200: {e}");
    }
    assert!(flags == 0, "libgdn2_b200: device error bits {flags:#x}");
}

/// `fused_recurrent_gdn2` with `update_state = true` on kernel (3): q,k,g,b `[B,HV,T,K]`, v,w `[B,HV,T,V]`,
/// state `[B,HV,K,V]` (f32, contiguous, updated in place).  Returns (out `[B,HV,T,V]`, state).
#[allow(clippy::too_many_arguments)]
pub fn fused_recurrent_b200<B: Backend>(q: &Tensor<B, 4>, k: &Tensor<B, 4>, v: &Tensor<B, 4>, g: &Tensor<B, 4>,
                                        b: &Tensor<B, 4>, w: &Tensor<B, 4>, state: Tensor<B, 4>, scale: f64)
                                        -> Option<(Tensor<B, 4>, Tensor<B, 4>)> {
    let (cq, ck, cv, cg, cb, cw, cs) = (cube(q)?, cube(k)?, cube(v)?, cube(g)?, cube(b)?, cube(w)?, cube(&state)?);
    let [batch, hv, t, kd] = q.shape().dims::<4>();
    let vd = v.shape().dims::<4>()[3];
    let out = Tensor::<B, 4>::empty([batch, hv, t, vd], &q.device());
    let co = cube(&out)?;
    let a = Gdn2RecurrentArgs {
        dims: Gdn2Dims { batch: batch as i32, seq_len: t as i32, num_heads: hv as i32, num_v_heads: hv as i32,
                         head_k_dim: kd as i32, head_v_dim: vd as i32 },
        dtype: GDN2_DTYPE_F32, key_heads_grouped: 0, prologue: 0, fuse_epilogue: 0, scale: scale as f32,
        norm_eps: 0.0, q: view(&cq), k: view(&ck), v: view(&cv), g: view(&cg), b: view(&cb), w: view(&cw),
        conv_w_q: std::ptr::null(), conv_w_k: std::ptr::null(), conv_w_v: std::ptr::null(),
        conv_q_in: std::ptr::null(), conv_k_in: std::ptr::null(), conv_v_in: std::ptr::null(),
        conv_q_out: std::ptr::null_mut(), conv_k_out: std::ptr::null_mut(), conv_v_out: std::ptr::null_mut(),
        gate: Gdn2View::default(), o_norm_weight: std::ptr::null(), state: raw_ptr(&cs) as *mut f32,
        out: view(&co),
    };
    run_on_device(|| cs.client.sync(), |stream| unsafe { gdn2_recurrent_fwd(&a, stream) });
    Some((out, state))
}

/// `chunk_wy_forward` (src/forward.rs:44-278) on kernels (1) + (2): same arguments, state updated in place.
/// Returns (out `[B,HV,T,V]`, state).
#[allow(clippy::too_many_arguments)]
pub fn chunk_forward_b200<B: Backend>(q: &Tensor<B, 4>, k: &Tensor<B, 4>, v: &Tensor<B, 4>, g: &Tensor<B, 4>,
                                      b: &Tensor<B, 4>, w: &Tensor<B, 4>, state: Tensor<B, 4>, scale: f64,
                                      chunk_size: usize) -> Option<(Tensor<B, 4>, Tensor<B, 4>)> {
    let (cq, ck, cv, cg, cb, cw, cs) = (cube(q)?, cube(k)?, cube(v)?, cube(g)?, cube(b)?, cube(w)?, cube(&state)?);
    let [batch, hv, t, kd] = q.shape().dims::<4>();
    let vd = v.shape().dims::<4>()[3];
    let out = Tensor::<B, 4>::empty([batch, hv, t, vd], &q.device());
    let co = cube(&out)?;
    let mut a = Gdn2ChunkArgs {
        dims: Gdn2Dims { batch: batch as i32, seq_len: t as i32, num_heads: hv as i32, num_v_heads: hv as i32,
                         head_k_dim: kd as i32, head_v_dim: vd as i32 },
        chunk_size: chunk_size as i32, dtype: GDN2_DTYPE_F32, key_heads_grouped: 0, fuse_epilogue: 0,
        scale: scale as f32, norm_eps: 0.0, q: view(&cq), k: view(&ck), v: view(&cv), g: view(&cg), b: view(&cb),
        w: view(&cw), gate: Gdn2View::default(), o_norm_weight: std::ptr::null(),
        state: raw_ptr(&cs) as *mut f32, out: view(&co), precision: GDN2_PRECISION_F32,
    };
    let bytes = unsafe { gdn2_chunk_fwd_workspace_bytes(&a) }.max(256);
    let ws = Tensor::<B, 1>::empty([bytes.div_ceil(4)], &q.device());
    let cws = cube1(&ws)?;
    let wsp = raw_ptr(&cws);
    a.precision = GDN2_PRECISION_F32;
    run_on_device(|| cs.client.sync(), |stream| unsafe { gdn2_chunk_fwd(&a, wsp, bytes, stream) });
    Some((out, state))
}

fn cube1<B: Backend>(t: &Tensor<B, 1>) -> Option<CubeTensor<cubecl::cuda::CudaRuntime>> {
    if TypeId::of::<B>() != TypeId::of::<CudaBare>() {
        return None;
    }
    let prim = t.clone().into_primitive().tensor();
    (&prim as &dyn Any).downcast_ref::<CubeTensor<cubecl::cuda::CudaRuntime>>().cloned()
}
