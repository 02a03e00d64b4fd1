"""burn_gdn2 — B200-native (sm_100a) GDN-2 token mixer.

Host-side mirror of the reference crate's public API (sehaxe/burn-gdn2
v0.5.1, src/lib.rs:58-63) over the C ABI of ``libgdn2_b200.so``
(include/gdn2.h).  Tensors are torch CUDA tensors; all recurrent math runs
in the library's hand-written kernels.
"""
from ._lib import EXPORTS, LIB, LIB_PATH, Gdn2Error
from .config import Gdn2Config, Gdn2Mode
from .graphs import GraphedCall
from .module import FUSED_RECURRENT_MAX_SEQ, GatedDeltaNet2, Gdn2State, Linear, ProjectedInputs
from .ops import (SHORT_CONV_CACHE, SHORT_CONV_KERNEL, GatedDeltaCore, chunk_trajectory, chunk_wy_forward, fused_recurrent_forward,
                  fused_recurrent_gdn2, l2_normalize_4d, project_activations, recurrent_backward,
                  rms_norm_gate_per_head, short_conv_1d)

__all__ = [
    "Gdn2Config", "Gdn2Mode", "GatedDeltaNet2", "Gdn2State", "ProjectedInputs", "Linear", "Gdn2Error",
    "chunk_wy_forward", "fused_recurrent_forward", "fused_recurrent_gdn2", "short_conv_1d", "l2_normalize_4d",
    "rms_norm_gate_per_head", "project_activations", "SHORT_CONV_CACHE", "SHORT_CONV_KERNEL", "FUSED_RECURRENT_MAX_SEQ",
    "LIB", "LIB_PATH", "EXPORTS", "GraphedCall", "recurrent_backward", "GatedDeltaCore", "chunk_trajectory",
]
