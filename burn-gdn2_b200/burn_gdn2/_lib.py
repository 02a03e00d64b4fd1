"""ctypes binding of libgdn2_b200.so — the C ABI declared in include/gdn2.h.

The structures below mirror the header field by field.  Loading the library
needs no GPU (it links the CUDA runtime statically); every compute entry
point needs one.  There is no fallback: if the library is missing the
import of ``burn_gdn2`` fails with the build command to run.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libgdn2_b200.so")

GDN2_OK, GDN2_EINVAL, GDN2_EUNSUPPORTED, GDN2_ECUDA, GDN2_EWORKSPACE = range(5)
GDN2_DTYPE_F32, GDN2_DTYPE_BF16 = 0, 1
GDN2_PRECISION_F32, GDN2_PRECISION_BF16 = 0, 1

_STATUS = {1: "EINVAL", 2: "EUNSUPPORTED", 3: "ECUDA", 4: "EWORKSPACE"}


class Gdn2Error(RuntimeError):
    """Non-zero status of a gdn2_* entry point."""

    def __init__(self, status, msg):
        super().__init__(f"{_STATUS.get(status, status)}: {msg}")
        self.status = status


class View(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("stride0", ctypes.c_int64), ("stride1", ctypes.c_int64),
                ("stride2", ctypes.c_int64)]


class Dims(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int32), ("seq_len", ctypes.c_int32), ("num_heads", ctypes.c_int32),
                ("num_v_heads", ctypes.c_int32), ("head_k_dim", ctypes.c_int32), ("head_v_dim", ctypes.c_int32)]


class ChunkArgs(ctypes.Structure):
    _fields_ = [("dims", Dims), ("chunk_size", ctypes.c_int32), ("dtype", ctypes.c_int32),
                ("key_heads_grouped", ctypes.c_int32), ("fuse_epilogue", ctypes.c_int32),
                ("scale", ctypes.c_float), ("norm_eps", ctypes.c_float),
                ("q", View), ("k", View), ("v", View), ("g", View), ("b", View), ("w", View),
                ("gate", View), ("o_norm_weight", ctypes.c_void_p), ("state", ctypes.c_void_p), ("out", View),
                ("precision", ctypes.c_int32)]


class RecurrentArgs(ctypes.Structure):
    _fields_ = [("dims", Dims), ("dtype", ctypes.c_int32), ("key_heads_grouped", ctypes.c_int32),
                ("prologue", ctypes.c_int32), ("fuse_epilogue", ctypes.c_int32),
                ("scale", ctypes.c_float), ("norm_eps", ctypes.c_float),
                ("q", View), ("k", View), ("v", View), ("g", View), ("b", View), ("w", View),
                ("conv_w_q", ctypes.c_void_p), ("conv_w_k", ctypes.c_void_p), ("conv_w_v", ctypes.c_void_p),
                ("conv_q_in", ctypes.c_void_p), ("conv_k_in", ctypes.c_void_p), ("conv_v_in", ctypes.c_void_p),
                ("conv_q_out", ctypes.c_void_p), ("conv_k_out", ctypes.c_void_p), ("conv_v_out", ctypes.c_void_p),
                ("gate", View), ("o_norm_weight", ctypes.c_void_p), ("state", ctypes.c_void_p), ("out", View)]


class RecurrentBwdArgs(ctypes.Structure):
    _fields_ = [("dims", Dims), ("dtype", ctypes.c_int32), ("key_heads_grouped", ctypes.c_int32),
                ("scale", ctypes.c_float),
                ("q", View), ("k", View), ("v", View), ("g", View), ("b", View), ("w", View),
                ("state_in", ctypes.c_void_p), ("d_out", View), ("d_state_out", ctypes.c_void_p),
                ("dq", View), ("dk", View), ("dv", View), ("dg", View), ("db", View), ("dw", View),
                ("d_state_in", ctypes.c_void_p)]


class PrologueArgs(ctypes.Structure):
    _fields_ = [("dims", Dims), ("dtype", ctypes.c_int32), ("use_short_conv", ctypes.c_int32),
                ("allow_neg_eigval", ctypes.c_int32), ("min_decay", ctypes.c_float),
                ("q_raw", ctypes.c_void_p), ("k_raw", ctypes.c_void_p), ("v_raw", ctypes.c_void_p),
                ("b_raw", ctypes.c_void_p), ("w_raw", ctypes.c_void_p), ("f_raw", ctypes.c_void_p),
                ("ld_q", ctypes.c_int64), ("ld_k", ctypes.c_int64), ("ld_v", ctypes.c_int64),
                ("ld_b", ctypes.c_int64), ("ld_w", ctypes.c_int64), ("ld_f", ctypes.c_int64),
                ("conv_w_q", ctypes.c_void_p), ("conv_w_k", ctypes.c_void_p), ("conv_w_v", ctypes.c_void_p),
                ("conv_q_in", ctypes.c_void_p), ("conv_k_in", ctypes.c_void_p), ("conv_v_in", ctypes.c_void_p),
                ("conv_q_out", ctypes.c_void_p), ("conv_k_out", ctypes.c_void_p), ("conv_v_out", ctypes.c_void_p),
                ("a_log", ctypes.c_void_p), ("dt_bias", ctypes.c_void_p), ("decay_factors", ctypes.c_void_p),
                ("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p), ("b", ctypes.c_void_p),
                ("w", ctypes.c_void_p), ("g", ctypes.c_void_p)]


class Config(ctypes.Structure):
    _fields_ = [("hidden_size", ctypes.c_int64), ("num_heads", ctypes.c_int64), ("head_dim", ctypes.c_int64),
                ("expand_v", ctypes.c_float), ("num_v_heads", ctypes.c_int64), ("use_short_conv", ctypes.c_int32),
                ("allow_neg_eigval", ctypes.c_int32), ("norm_eps", ctypes.c_double), ("mode", ctypes.c_int32),
                ("chunk_size", ctypes.c_int64), ("min_decay", ctypes.c_double)]


# every symbol declared in include/gdn2.h
EXPORTS = (
    "gdn2_chunk_fwd_workspace_bytes", "gdn2_chunk_fwd", "gdn2_chunk_intra", "gdn2_chunk_inter",
    "gdn2_recurrent_fwd", "gdn2_short_conv", "gdn2_rms_norm_gate", "gdn2_config_validate",
    "gdn2_last_error", "gdn2_last_cuda_error", "gdn2_abi_version", "gdn2_read_device_errors",
    "gdn2_selftest_umma", "gdn2_chunk_fwd_noalloc", "gdn2_project_activations", "gdn2_selftest_wait",
    "gdn2_set_reserved_sms", "gdn2_recurrent_bwd_workspace_bytes", "gdn2_recurrent_bwd",
    "gdn2_chunk_trajectory",
)


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} not built: run `python burn-gdn2_b200/build.py` (nvcc, sm_100a)")
    lib = ctypes.CDLL(LIB_PATH)
    P = ctypes.POINTER
    vp, i32, f32, sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_float, ctypes.c_size_t
    lib.gdn2_chunk_fwd_workspace_bytes.argtypes = [P(ChunkArgs)]
    lib.gdn2_chunk_fwd_workspace_bytes.restype = sz
    for fn in ("gdn2_chunk_fwd", "gdn2_chunk_intra", "gdn2_chunk_inter"):
        getattr(lib, fn).argtypes = [P(ChunkArgs), vp, sz, vp]
        getattr(lib, fn).restype = ctypes.c_int
    lib.gdn2_project_activations.argtypes = [P(PrologueArgs), vp]
    lib.gdn2_project_activations.restype = ctypes.c_int
    lib.gdn2_chunk_fwd_noalloc.argtypes = [P(ChunkArgs), vp]
    lib.gdn2_chunk_fwd_noalloc.restype = ctypes.c_int
    lib.gdn2_recurrent_fwd.argtypes = [P(RecurrentArgs), vp]
    lib.gdn2_recurrent_fwd.restype = ctypes.c_int
    lib.gdn2_recurrent_bwd_workspace_bytes.argtypes = [P(Dims)]
    lib.gdn2_recurrent_bwd_workspace_bytes.restype = sz
    lib.gdn2_recurrent_bwd.argtypes = [P(RecurrentBwdArgs), vp, sz, vp]
    lib.gdn2_recurrent_bwd.restype = ctypes.c_int
    lib.gdn2_chunk_trajectory.argtypes = [P(RecurrentArgs), i32, vp, View, vp]
    lib.gdn2_chunk_trajectory.restype = ctypes.c_int
    lib.gdn2_short_conv.argtypes = [i32, i32, i32, i32, vp, vp, vp, vp, vp, vp]
    lib.gdn2_short_conv.restype = ctypes.c_int
    lib.gdn2_rms_norm_gate.argtypes = [P(Dims), i32, View, View, vp, f32, View, vp]
    lib.gdn2_rms_norm_gate.restype = ctypes.c_int
    lib.gdn2_config_validate.argtypes = [P(Config), ctypes.c_char_p, sz]
    lib.gdn2_config_validate.restype = ctypes.c_int
    lib.gdn2_last_error.argtypes = []
    lib.gdn2_last_error.restype = ctypes.c_char_p
    lib.gdn2_last_cuda_error.restype = ctypes.c_int
    lib.gdn2_abi_version.restype = ctypes.c_int
    lib.gdn2_read_device_errors.argtypes = [ctypes.POINTER(ctypes.c_uint32)]
    lib.gdn2_read_device_errors.restype = ctypes.c_int
    lib.gdn2_selftest_umma.argtypes = [i32, vp, vp, vp, vp]
    lib.gdn2_selftest_umma.restype = ctypes.c_int
    lib.gdn2_selftest_wait.argtypes = [ctypes.c_uint32, i32, ctypes.POINTER(ctypes.c_int32)]
    lib.gdn2_selftest_wait.restype = ctypes.c_int
    lib.gdn2_set_reserved_sms.argtypes = [i32]
    lib.gdn2_set_reserved_sms.restype = ctypes.c_int
    return lib


LIB = _load()


def read_device_errors() -> int:
    """Device error bits since the last call (bit 0: a bounded wait gave up)."""
    v = ctypes.c_uint32(0)
    check(LIB.gdn2_read_device_errors(ctypes.byref(v)))
    return int(v.value)


def check(status):
    """Raise Gdn2Error for a non-zero status (message from gdn2_last_error)."""
    if status != GDN2_OK:
        raise Gdn2Error(status, LIB.gdn2_last_error().decode())
    return status
