"""Gdn2Config / Gdn2Mode — mirror of src/config.rs (sehaxe/burn-gdn2 v0.5.1).

``validate()`` runs the C-ABI check ``gdn2_config_validate`` (the reference's
panics at src/config.rs:71-111, raised here as ``ValueError`` with the same
messages).
"""
from __future__ import annotations

import ctypes
import dataclasses
import enum
from typing import Optional

import numpy as np

from . import _lib


class Gdn2Mode(enum.Enum):
    """src/config.rs:2-12."""

    FusedRecurrent = 0
    Chunk = 1


@dataclasses.dataclass
class Gdn2Config:
    """Layer hyperparameters (src/config.rs:24-58, defaults :114-129)."""

    hidden_size: int = 2048
    num_heads: int = 16
    head_dim: int = 128
    expand_v: float = 1.0
    num_v_heads: Optional[int] = None
    use_short_conv: bool = True
    allow_neg_eigval: bool = False
    norm_eps: float = 1e-5
    mode: Gdn2Mode = Gdn2Mode.FusedRecurrent
    chunk_size: int = 64
    min_decay: Optional[float] = None

    def to_c(self) -> _lib.Config:
        return _lib.Config(
            hidden_size=int(self.hidden_size), num_heads=int(self.num_heads), head_dim=int(self.head_dim),
            expand_v=float(self.expand_v),
            num_v_heads=-1 if self.num_v_heads is None else int(self.num_v_heads),
            use_short_conv=int(bool(self.use_short_conv)), allow_neg_eigval=int(bool(self.allow_neg_eigval)),
            norm_eps=float(self.norm_eps), mode=Gdn2Mode(self.mode).value, chunk_size=int(self.chunk_size),
            min_decay=-1.0 if self.min_decay is None else float(self.min_decay))

    def validate(self) -> None:
        """Raise ValueError on the configurations src/config.rs:71-111 rejects."""
        msg = ctypes.create_string_buffer(512)
        c = self.to_c()
        if _lib.LIB.gdn2_config_validate(ctypes.byref(c), msg, len(msg)) != _lib.GDN2_OK:
            raise ValueError(msg.value.decode())

    @property
    def hv(self) -> int:
        return self.num_heads if self.num_v_heads is None else self.num_v_heads

    @property
    def v_head(self) -> int:
        # (hk as f32 * expand_v) as usize  (src/module.rs:117)
        return int(np.float32(self.head_dim) * np.float32(self.expand_v))
