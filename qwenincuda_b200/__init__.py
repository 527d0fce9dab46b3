"""QweninCuda decode-time KV-cache hot path on B200 (sm_100a).

Python mirror of the reference's kernel-layer interface (include/kernels.cuh and
the full-attention / linear-attention block bodies of src/model.cpp in the
QweninCuda project), bound through ctypes to the C-ABI library libqic.so
(include/qic.h). PyTorch tensors are used only as device buffers and for the
current CUDA stream; all arithmetic runs in the library's sm_100a kernels.

The library must have been built (``python -m qwenincuda_b200.build`` or
``__graft_entry__.build()``); importing the package without it raises.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

from .abi import (  # noqa: F401
    QIC_DTYPE_BF16,
    QIC_DTYPE_F16,
    QIC_FUSE_APPEND,
    QIC_FUSE_Q_PROLOGUE,
    DecodeArgs,
    GdnArgs,
    QicError,
    lib,
    lib_path,
)
from .ops import (  # noqa: F401
    BatchPlan,
    Workspace,
    batch_decode_attention,
    decode_attention,
    gated_delta_decode,
    gemv,
    kv_append,
    launch_flash_attention,
    launch_head_rmsnorm,
    launch_paged_attention,
    launch_rope_inplace,
    launch_sigmoid_mul_inplace,
)

__all__ = [
    "QIC_DTYPE_BF16",
    "QIC_DTYPE_F16",
    "QIC_FUSE_APPEND",
    "QIC_FUSE_Q_PROLOGUE",
    "BatchPlan",
    "DecodeArgs",
    "batch_decode_attention",
    "GdnArgs",
    "QicError",
    "Workspace",
    "decode_attention",
    "gated_delta_decode",
    "gemv",
    "kv_append",
    "launch_flash_attention",
    "launch_head_rmsnorm",
    "launch_paged_attention",
    "launch_rope_inplace",
    "launch_sigmoid_mul_inplace",
    "lib",
    "lib_path",
]
