"""CPU: the C ABI library loads without a GPU, exports every symbol that
include/gdn2.h declares, its structs agree with the ctypes mirror (checked
against a gcc-compiled probe of the header), and argument errors come back
as status codes before any CUDA call (no GPU needed)."""
import ctypes
import os
import re
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "gdn2.h")


def test_library_exports_every_header_symbol():
    import burn_gdn2
    from burn_gdn2 import _lib

    decls = set(re.findall(r"GDN2_API\s+[\w\s\*]+?\b(gdn2_\w+)\s*\(", open(HEADER).read()))
    assert decls, "no declarations parsed"
    assert decls == set(_lib.EXPORTS)
    out = subprocess.run(["nm", "-D", "--defined-only", burn_gdn2.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (gdn2_\w+)", out))
    missing = decls - exported
    assert not missing, missing
    for name in decls:
        assert hasattr(burn_gdn2.LIB, name)
    assert burn_gdn2.LIB.gdn2_abi_version() == 2


def test_struct_layout_matches_header():
    from burn_gdn2 import _lib

    probe = r"""
#include <stdio.h>
#include <stddef.h>
#include "gdn2.h"
#define P(T, F) printf(#T "." #F " %zu\n", offsetof(T, F));
int main() {
  printf("view %zu\ndims %zu\nchunk %zu\nrec %zu\ncfg %zu\npro %zu\nbwd %zu\n", sizeof(gdn2_view),
         sizeof(gdn2_dims), sizeof(gdn2_chunk_args), sizeof(gdn2_recurrent_args), sizeof(gdn2_config),
         sizeof(gdn2_prologue_args), sizeof(gdn2_recurrent_bwd_args));
  P(gdn2_recurrent_bwd_args, scale) P(gdn2_recurrent_bwd_args, q) P(gdn2_recurrent_bwd_args, state_in)
  P(gdn2_recurrent_bwd_args, d_out) P(gdn2_recurrent_bwd_args, d_state_out) P(gdn2_recurrent_bwd_args, dq)
  P(gdn2_recurrent_bwd_args, dw) P(gdn2_recurrent_bwd_args, d_state_in)
  P(gdn2_prologue_args, min_decay) P(gdn2_prologue_args, q_raw) P(gdn2_prologue_args, ld_q)
  P(gdn2_prologue_args, ld_f) P(gdn2_prologue_args, conv_w_q) P(gdn2_prologue_args, conv_v_out)
  P(gdn2_prologue_args, a_log) P(gdn2_prologue_args, decay_factors) P(gdn2_prologue_args, q)
  P(gdn2_prologue_args, g)
  P(gdn2_chunk_args, scale) P(gdn2_chunk_args, q) P(gdn2_chunk_args, gate) P(gdn2_chunk_args, o_norm_weight)
  P(gdn2_chunk_args, state) P(gdn2_chunk_args, out) P(gdn2_chunk_args, precision)
  P(gdn2_recurrent_args, q) P(gdn2_recurrent_args, conv_w_q) P(gdn2_recurrent_args, conv_v_out)
  P(gdn2_recurrent_args, gate) P(gdn2_recurrent_args, state) P(gdn2_recurrent_args, out)
  P(gdn2_config, expand_v) P(gdn2_config, num_v_heads) P(gdn2_config, norm_eps) P(gdn2_config, chunk_size)
  P(gdn2_config, min_decay)
  return 0;
}
"""
    with tempfile.TemporaryDirectory() as d:
        src, exe = os.path.join(d, "p.c"), os.path.join(d, "p")
        open(src, "w").write(probe)
        subprocess.run(["gcc", "-I", os.path.dirname(HEADER), src, "-o", exe], check=True)
        lines = dict(l.rsplit(" ", 1) for l in subprocess.run([exe], capture_output=True, text=True,
                                                              check=True).stdout.split("\n") if l)
    got = {k: int(v) for k, v in lines.items()}
    assert got["view"] == ctypes.sizeof(_lib.View)
    assert got["dims"] == ctypes.sizeof(_lib.Dims)
    assert got["chunk"] == ctypes.sizeof(_lib.ChunkArgs)
    assert got["rec"] == ctypes.sizeof(_lib.RecurrentArgs)
    assert got["cfg"] == ctypes.sizeof(_lib.Config)
    assert got["pro"] == ctypes.sizeof(_lib.PrologueArgs)
    assert got["bwd"] == ctypes.sizeof(_lib.RecurrentBwdArgs)
    names = {"gdn2_chunk_args": _lib.ChunkArgs, "gdn2_recurrent_args": _lib.RecurrentArgs,
             "gdn2_recurrent_bwd_args": _lib.RecurrentBwdArgs,
             "gdn2_config": _lib.Config, "gdn2_prologue_args": _lib.PrologueArgs}
    for key, off in got.items():
        if "." in key:
            t, f = key.split(".")
            assert getattr(names[t], f).offset == off, key


def _chunk_args(**over):
    from burn_gdn2 import _lib

    a = _lib.ChunkArgs()
    a.dims = _lib.Dims(1, 64, 1, 1, 16, 16)
    a.chunk_size, a.dtype, a.scale, a.norm_eps = 64, 0, 0.25, 1e-5
    fake = 1 << 20  # never dereferenced: validation fails first
    for n in ("q", "k", "v", "g", "b", "w", "out"):
        setattr(a, n, _lib.View(fake, 0, 0, 0))
    a.state = fake
    for k, v in over.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("over,status", [
    (dict(chunk_size=0), 1),
    (dict(dtype=7), 1),
    (dict(state=None), 1),
    (dict(state=(1 << 20) + 4), 1),  # misaligned state
    (dict(fuse_epilogue=1), 1),      # epilogue without gate
])
def test_chunk_fwd_argument_errors(over, status):
    from burn_gdn2 import LIB, _lib

    a = _chunk_args(**over)
    ws = ctypes.create_string_buffer(256)
    rc = LIB.gdn2_chunk_fwd(ctypes.byref(a), ctypes.addressof(ws), 256, None)
    assert rc == status, LIB.gdn2_last_error()
    assert LIB.gdn2_last_error().decode().startswith("gdn2_chunk_fwd")


def test_chunk_fwd_dims_and_workspace_errors():
    from burn_gdn2 import LIB, _lib

    a = _chunk_args()
    a.dims = _lib.Dims(1, 64, 2, 3, 16, 16)  # HV % H != 0
    assert LIB.gdn2_chunk_fwd(ctypes.byref(a), None, 0, None) == _lib.GDN2_EINVAL
    a = _chunk_args()
    need = LIB.gdn2_chunk_fwd_workspace_bytes(ctypes.byref(a))
    assert need > 0
    rc = LIB.gdn2_chunk_fwd(ctypes.byref(a), ctypes.c_void_p(1 << 20), need - 1, None)
    assert rc == _lib.GDN2_EWORKSPACE
    a = _chunk_args()
    a.dims = _lib.Dims(1, 64, 1, 1, 16, 18)  # V % 4 != 0
    assert LIB.gdn2_chunk_fwd(ctypes.byref(a), ctypes.c_void_p(1 << 20), 1 << 30, None) == _lib.GDN2_EUNSUPPORTED


def test_chunk_fwd_noalloc_size_limit():
    """Calls that need more than the 32 MiB static scratch are refused before
    any CUDA call, so this runs without a GPU."""
    from burn_gdn2 import LIB, _lib

    assert LIB.gdn2_chunk_fwd_noalloc(None, None) == _lib.GDN2_EINVAL
    a = _chunk_args()
    a.dims = _lib.Dims(1, 1 << 16, 1, 16, 16, 16)
    assert LIB.gdn2_chunk_fwd_workspace_bytes(ctypes.byref(a)) > 32 << 20
    assert LIB.gdn2_chunk_fwd_noalloc(ctypes.byref(a), None) == _lib.GDN2_EWORKSPACE
    msg = LIB.gdn2_last_error().decode()
    assert msg.startswith("gdn2_chunk_fwd_noalloc") and str(32 << 20) in msg
    # a negative dim is an argument error, not a scratch-size one
    a.dims = _lib.Dims(1, 64, 1, -16, 16, 16)
    assert LIB.gdn2_chunk_fwd_workspace_bytes(ctypes.byref(a)) == 0
    assert LIB.gdn2_chunk_fwd_noalloc(ctypes.byref(a), None) == _lib.GDN2_EINVAL
    a.dims = _lib.Dims(1, 64, 1, 1, -128, 16)
    assert LIB.gdn2_chunk_fwd_noalloc(ctypes.byref(a), None) == _lib.GDN2_EINVAL


def test_selftest_wait_argument_errors():
    from burn_gdn2 import LIB, _lib

    done = ctypes.c_int32(-1)
    assert LIB.gdn2_selftest_wait(0, 0, ctypes.byref(done)) == _lib.GDN2_EINVAL
    assert LIB.gdn2_selftest_wait((1 << 24) + 1, 0, ctypes.byref(done)) == _lib.GDN2_EINVAL
    assert LIB.gdn2_selftest_wait(10, 0, None) == _lib.GDN2_EINVAL
    assert done.value == -1


def test_chunk_precision_argument():
    from burn_gdn2 import LIB, _lib

    a = _chunk_args(precision=5)
    ws = ctypes.create_string_buffer(256)
    assert LIB.gdn2_chunk_fwd(ctypes.byref(a), ctypes.addressof(ws), 256, None) == _lib.GDN2_EINVAL
    assert "precision" in LIB.gdn2_last_error().decode()
    assert LIB.gdn2_chunk_fwd_workspace_bytes(ctypes.byref(a)) == 0
    # K = V = 128, chunk 64: the split-operand records (f32 precision) are larger than the bf16-intermediate ones
    sizes = {}
    for prec in (_lib.GDN2_PRECISION_F32, _lib.GDN2_PRECISION_BF16):
        a = _chunk_args(precision=prec, dtype=_lib.GDN2_DTYPE_BF16)
        a.dims = _lib.Dims(1, 128, 1, 1, 128, 128)
        for n in ("q", "k", "v", "g", "b", "w", "out"):
            setattr(a, n, _lib.View(1 << 20, 128 * 128, 128 * 128, 128))
        sizes[prec] = LIB.gdn2_chunk_fwd_workspace_bytes(ctypes.byref(a))
    assert sizes[_lib.GDN2_PRECISION_F32] == 2 * 148480 + 2 * 139264  # two records + two per-CTA scratch slots
    assert sizes[_lib.GDN2_PRECISION_BF16] == 2 * 74752


def test_recurrent_argument_errors():
    from burn_gdn2 import LIB, _lib

    a = _lib.RecurrentArgs()
    a.dims = _lib.Dims(1, 1, 1, 1, 16, 16)
    assert LIB.gdn2_recurrent_fwd(ctypes.byref(a), None) == _lib.GDN2_EINVAL  # null tensors
    assert LIB.gdn2_recurrent_fwd(None, None) == _lib.GDN2_EINVAL
    fake = 1 << 20
    for n in ("q", "k", "v", "g", "b", "w", "out"):
        setattr(a, n, _lib.View(fake, 0, 0, 0))
    a.state = fake
    a.prologue = 3
    assert LIB.gdn2_recurrent_fwd(ctypes.byref(a), None) == _lib.GDN2_EINVAL
    a.prologue = 1  # conv prologue without weights / caches
    assert LIB.gdn2_recurrent_fwd(ctypes.byref(a), None) == _lib.GDN2_EINVAL


def test_ops_refuse_cpu_tensors():
    """No CPU fallback: ops and the module raise on CPU tensors."""
    import torch
    import burn_gdn2 as bg

    q = torch.zeros(1, 1, 4, 16)
    v = torch.zeros(1, 1, 4, 16)
    with pytest.raises(RuntimeError):
        bg.fused_recurrent_forward(q, q, v, q, q, v, torch.zeros(1, 1, 16, 16), 0.25)
    with pytest.raises(RuntimeError):
        bg.chunk_wy_forward(q, q, v, q, q, v, torch.zeros(1, 1, 16, 16), 0.25, 64)
    cfg = bg.Gdn2Config(hidden_size=32, num_heads=2, head_dim=16)
    import gdn2_oracle as O
    m = bg.GatedDeltaNet2(cfg, O.init_weights(O.Gdn2Config(hidden_size=32, num_heads=2, head_dim=16)), device="cpu")
    with pytest.raises(RuntimeError):
        m.forward_train(torch.zeros(1, 4, 32))


def test_config_mirror_validate():
    import burn_gdn2 as bg

    bg.Gdn2Config().validate()
    with pytest.raises(ValueError, match="num_v_heads=24 must be divisible"):
        bg.Gdn2Config(num_v_heads=24).validate()
    with pytest.raises(ValueError, match="chunk_size must be > 0"):
        bg.Gdn2Config(chunk_size=0).validate()


def test_set_reserved_sms_clamps_and_returns_previous():
    """Host-only setting: the previous value comes back, the value is
    clamped to [0, 64]; no device is touched."""
    from burn_gdn2 import _lib

    lib = _lib.LIB
    prev = lib.gdn2_set_reserved_sms(16)
    try:
        assert lib.gdn2_set_reserved_sms(-5) == 16
        assert lib.gdn2_set_reserved_sms(1000) == 0
        assert lib.gdn2_set_reserved_sms(0) == 64
    finally:
        lib.gdn2_set_reserved_sms(prev)


def test_recurrent_bwd_argument_errors():
    from burn_gdn2 import LIB, _lib

    a = _lib.RecurrentBwdArgs()
    a.dims = _lib.Dims(1, 20, 1, 1, 128, 128)
    assert LIB.gdn2_recurrent_bwd(None, None, 0, None) == _lib.GDN2_EINVAL
    assert LIB.gdn2_recurrent_bwd(ctypes.byref(a), None, 0, None) == _lib.GDN2_EINVAL  # null tensors
    # workspace: the state at every 8th token, ceil(20 / 8) = 3 of them
    assert LIB.gdn2_recurrent_bwd_workspace_bytes(ctypes.byref(a.dims)) == 3 * 128 * 128 * 4
    bad = _lib.Dims(1, 20, 1, -1, 128, 128)
    assert LIB.gdn2_recurrent_bwd_workspace_bytes(ctypes.byref(bad)) == 0
    fake = 1 << 20  # never dereferenced: validation fails first
    for n in ("q", "k", "v", "g", "b", "w", "d_out", "dq", "dk", "dv", "dg", "db", "dw"):
        setattr(a, n, _lib.View(fake, 0, 0, 0))
    assert LIB.gdn2_recurrent_bwd(ctypes.byref(a), None, 0, None) == _lib.GDN2_EWORKSPACE
    assert LIB.gdn2_recurrent_bwd(ctypes.byref(a), ctypes.c_void_p(fake), 1024, None) == _lib.GDN2_EWORKSPACE
    for dims in [(1, 20, 1, 1, 100, 128), (1, 20, 1, 1, 256, 128), (1, 20, 1, 1, 128, 24), (1, 20, 1, 1, 128, 512)]:
        a.dims = _lib.Dims(*dims)
        assert LIB.gdn2_recurrent_bwd(ctypes.byref(a), ctypes.c_void_p(fake), 1 << 30, None) == \
            _lib.GDN2_EUNSUPPORTED, dims
    a.dims = _lib.Dims(1, 20, 2, 3, 128, 128)
    assert LIB.gdn2_recurrent_bwd(ctypes.byref(a), ctypes.c_void_p(fake), 1 << 30, None) == _lib.GDN2_EINVAL
    a.dims = _lib.Dims(1, 20, 1, 1, 128, 128)
    a.dtype = 5
    assert LIB.gdn2_recurrent_bwd(ctypes.byref(a), ctypes.c_void_p(fake), 1 << 30, None) == _lib.GDN2_EINVAL


def test_chunk_trajectory_argument_errors():
    from burn_gdn2 import LIB, _lib

    a = _lib.RecurrentArgs()
    a.dims = _lib.Dims(1, 20, 1, 1, 128, 128)
    fake = ctypes.c_void_p(1 << 20)
    assert LIB.gdn2_chunk_trajectory(None, 64, fake, _lib.View(), None) == _lib.GDN2_EINVAL
    assert LIB.gdn2_chunk_trajectory(ctypes.byref(a), 64, fake, _lib.View(), None) == _lib.GDN2_EINVAL  # nulls
    for n in ("q", "k", "v", "g", "b", "w"):
        setattr(a, n, _lib.View(1 << 20, 0, 0, 0))
    assert LIB.gdn2_chunk_trajectory(ctypes.byref(a), 64, None, _lib.View(), None) == _lib.GDN2_EINVAL
    assert LIB.gdn2_chunk_trajectory(ctypes.byref(a), 12, fake, _lib.View(), None) == _lib.GDN2_EUNSUPPORTED
    a.prologue = 1
    assert LIB.gdn2_chunk_trajectory(ctypes.byref(a), 64, fake, _lib.View(), None) == _lib.GDN2_EINVAL
    a.prologue = 0
    a.dims = _lib.Dims(1, 20, 1, 1, 128, 40)
    assert LIB.gdn2_chunk_trajectory(ctypes.byref(a), 64, fake, _lib.View(), None) == _lib.GDN2_EUNSUPPORTED
