"""ctypes declarations of include/qic.h (the C-ABI of libqic.so)."""
from __future__ import annotations

import ctypes
from pathlib import Path

QIC_DTYPE_F16 = 0
QIC_DTYPE_BF16 = 1
QIC_FUSE_Q_PROLOGUE = 1
QIC_FUSE_APPEND = 2

QIC_DEV_TIMEOUT = 1
QIC_DEV_BAD_PAGE = 2
QIC_DEV_PEER_TIMEOUT = 4
QIC_DEV_BAD_PLAN = 8
QIC_DEV_BAD_LENGTH = 16
QIC_PDL = 4
QIC_PARTIAL_OUT = 8
QIC_EXPLICIT_POSITION = 16
QIC_DETERMINISTIC = 32
QIC_Q_GATE_INTERLEAVED = 64
QIC_DEVICE_SEQ_LEN = 128
QIC_GDN_STATES_READY = 256
QIC_MAX_RANKS = 8
QIC_MAX_SEQ_LEN = 1 << 30
QIC_IPC_HANDLE_BYTES = 64

STATUS_NAMES = {
    0: "QIC_SUCCESS",
    1: "QIC_ERROR_INVALID_VALUE",
    2: "QIC_ERROR_NOT_SUPPORTED",
    3: "QIC_ERROR_MISALIGNED",
    4: "QIC_ERROR_WORKSPACE",
    5: "QIC_ERROR_CUDA",
    6: "QIC_ERROR_DEVICE_TIMEOUT",
    7: "QIC_ERROR_BAD_PAGE",
    8: "QIC_ERROR_PEER",
}

_PKG = Path(__file__).resolve().parent


def lib_path() -> Path:
    return _PKG / "libqic.so"


class QicError(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        self.status = status
        name = STATUS_NAMES.get(status, str(status))
        msg = f"{what}: {name}" if what else name
        if status == 5 and _LIB is not None:
            msg += f" (cudaError {_LIB.qic_last_cuda_error()})"
        super().__init__(msg)


class DecodeArgs(ctypes.Structure):
    """Mirror of qic_decode_args."""

    _fields_ = [
        ("dtype", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("seq_len", ctypes.c_int32),
        ("page_size", ctypes.c_int32),
        ("cache_tokens", ctypes.c_int64),
        ("q", ctypes.c_void_p),
        ("k_cache", ctypes.c_void_p),
        ("v_cache", ctypes.c_void_p),
        ("page_table", ctypes.c_void_p),
        ("gate", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("flags", ctypes.c_uint32),
        ("eps", ctypes.c_float),
        ("rope_theta", ctypes.c_float),
        ("q_norm_w", ctypes.c_void_p),
        ("k_norm_w", ctypes.c_void_p),
        ("k_new", ctypes.c_void_p),
        ("v_new", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
        ("num_splits", ctypes.c_int32),
        ("cluster_size", ctypes.c_int32),
        ("position", ctypes.c_int64),
        ("seq_len_dev", ctypes.c_void_p),
    ]


class CpArgs(ctypes.Structure):
    """Mirror of qic_cp_args."""

    _fields_ = [
        ("rank", ctypes.c_int32),
        ("world", ctypes.c_int32),
        ("exchange", ctypes.c_void_p),
        ("exchange_bytes", ctypes.c_size_t),
        ("peer_exchange", ctypes.c_void_p * QIC_MAX_RANKS),
        ("timeout_ms", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


class BatchDecodeArgs(ctypes.Structure):
    """Mirror of qic_batch_decode_args."""

    _fields_ = [
        ("dtype", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("batch", ctypes.c_int32),
        ("page_size", ctypes.c_int32),
        ("cache_tokens", ctypes.c_int64),
        ("max_pages_per_seq", ctypes.c_int32),
        ("flags", ctypes.c_uint32),
        ("q", ctypes.c_void_p),
        ("k_cache", ctypes.c_void_p),
        ("v_cache", ctypes.c_void_p),
        ("block_tables", ctypes.c_void_p),
        ("gate", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("eps", ctypes.c_float),
        ("rope_theta", ctypes.c_float),
        ("q_norm_w", ctypes.c_void_p),
        ("k_norm_w", ctypes.c_void_p),
        ("k_new", ctypes.c_void_p),
        ("v_new", ctypes.c_void_p),
        ("plan", ctypes.c_void_p),
        ("plan_items", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
    ]


QIC_PLAN_ITEM_BYTES = 32


class GdnArgs(ctypes.Structure):
    """Mirror of qic_gdn_args."""

    _fields_ = [
        ("dtype", ctypes.c_int32),
        ("num_k_heads", ctypes.c_int32),
        ("num_v_heads", ctypes.c_int32),
        ("k_head_dim", ctypes.c_int32),
        ("v_head_dim", ctypes.c_int32),
        ("conv_kernel", ctypes.c_int32),
        ("eps", ctypes.c_float),
        ("flags", ctypes.c_uint32),
        ("qkv", ctypes.c_void_p),
        ("z", ctypes.c_void_p),
        ("b", ctypes.c_void_p),
        ("a", ctypes.c_void_p),
        ("conv_w", ctypes.c_void_p),
        ("dt_bias", ctypes.c_void_p),
        ("a_log", ctypes.c_void_p),
        ("norm_w", ctypes.c_void_p),
        ("conv_state", ctypes.c_void_p),
        ("recurrent_state", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("status", ctypes.c_void_p),
    ]


QIC_GEMV_MAX_SEGMENTS = 4
QIC_GEMV_RMSNORM = 1
QIC_GEMV_SWIGLU = 2
QIC_GEMV_RESIDUAL = 8


class GemvSegment(ctypes.Structure):
    """Mirror of qic_gemv_segment."""

    _fields_ = [
        ("w", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("residual", ctypes.c_void_p),
        ("out_dim", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


class GemvArgs(ctypes.Structure):
    """Mirror of qic_gemv_args."""

    _fields_ = [
        ("dtype", ctypes.c_int32),
        ("in_dim", ctypes.c_int32),
        ("num_segments", ctypes.c_int32),
        ("flags", ctypes.c_uint32),
        ("x", ctypes.c_void_p),
        ("norm_w", ctypes.c_void_p),
        ("eps", ctypes.c_float),
        ("splits", ctypes.c_int32),
        ("seg", GemvSegment * QIC_GEMV_MAX_SEGMENTS),
        ("status", ctypes.c_void_p),
    ]


class ModelConfig(ctypes.Structure):
    """Mirror of qic_model_config."""

    _fields_ = [(n, ctypes.c_int32) for n in (
        "vocab_size", "hidden_size", "intermediate_size", "num_layers", "num_heads", "num_kv_heads", "head_dim",
        "linear_num_key_heads", "linear_num_value_heads", "linear_key_head_dim", "linear_value_head_dim",
        "linear_conv_kernel_dim", "max_seq_len")] + [
        ("rms_norm_eps", ctypes.c_float), ("rope_theta", ctypes.c_float),
        ("layer_types", ctypes.POINTER(ctypes.c_int32))]


LAYER_WEIGHT_NAMES = ("attn_norm", "wq", "wk", "wv", "q_norm", "k_norm", "wo", "linear_in_qkv", "linear_in_z",
                      "linear_in_b", "linear_in_a", "linear_conv1d_w", "linear_dt_bias", "linear_a_log",
                      "linear_norm_w", "linear_out_proj", "ffn_norm", "w_gate", "w_up", "w_down")


class LayerWeights(ctypes.Structure):
    """Mirror of qic_layer_weights."""

    _fields_ = [("is_linear", ctypes.c_int32)] + [(n, ctypes.c_void_p) for n in LAYER_WEIGHT_NAMES]


class ModelWeights(ctypes.Structure):
    """Mirror of qic_model_weights."""

    _fields_ = [("tok_embeddings", ctypes.c_void_p), ("final_norm", ctypes.c_void_p), ("lm_head", ctypes.c_void_p),
                ("layers", ctypes.POINTER(LayerWeights))]


_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_f32 = ctypes.c_float

# name -> (restype, argtypes); every function declared in include/qic.h
SIGNATURES = {
    "qic_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "qic_last_cuda_error": (ctypes.c_int, []),
    "qic_version": (ctypes.c_int, []),
    "qic_head_rmsnorm": (ctypes.c_int, [ctypes.c_int, _vp, _vp, ctypes.c_int, ctypes.c_int, _f32, _vp, _vp]),
    "qic_rope_inplace": (ctypes.c_int, [ctypes.c_int, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, _f32, _vp]),
    "qic_sigmoid_mul_inplace": (ctypes.c_int, [ctypes.c_int, _vp, _vp, ctypes.c_int, _vp]),
    "qic_kv_append": (
        ctypes.c_int,
        [ctypes.c_int, _vp, _vp, _vp, _f32, _f32, ctypes.c_int, _vp, _vp, _vp, ctypes.c_int, _i64, ctypes.c_int,
         ctypes.c_int, _vp],
    ),
    "qic_decode_workspace_bytes": (ctypes.c_size_t, [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    "qic_workspace_init": (ctypes.c_int, [_vp, ctypes.c_size_t, _vp]),
    "qic_workspace_status": (ctypes.c_int, [_vp, _vp, ctypes.POINTER(ctypes.c_int)]),
    "qic_decode_attention": (ctypes.c_int, [ctypes.POINTER(DecodeArgs), _vp]),
    "qic_decode_launch_shape": (ctypes.c_int, [ctypes.POINTER(DecodeArgs), ctypes.POINTER(ctypes.c_int),
                                               ctypes.POINTER(ctypes.c_int)]),
    "qic_gated_delta_decode": (ctypes.c_int, [ctypes.POINTER(GdnArgs), _vp]),
    "qic_gemv": (ctypes.c_int, [ctypes.POINTER(GemvArgs), _vp]),
    "qic_model_create": (ctypes.c_int, [ctypes.POINTER(ModelConfig), ctypes.c_int, ctypes.POINTER(ModelWeights),
                                        ctypes.POINTER(ctypes.c_void_p)]),
    "qic_model_load": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(ctypes.c_void_p)]),
    "qic_model_info": (ctypes.c_int, [_vp, ctypes.POINTER(ModelConfig), ctypes.POINTER(ctypes.c_size_t)]),
    "qic_model_reset": (ctypes.c_int, [_vp]),
    "qic_model_decode": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _vp, ctypes.POINTER(ctypes.c_int), _vp]),
    "qic_model_set_position": (ctypes.c_int, [_vp, ctypes.c_int, ctypes.c_int, _vp]),
    "qic_model_step_graph": (ctypes.c_int, [_vp, _vp]),
    "qic_model_free": (ctypes.c_int, [_vp]),
    "qic_gemv_launch_shape": (ctypes.c_int, [ctypes.POINTER(GemvArgs), ctypes.POINTER(ctypes.c_int),
                                             ctypes.POINTER(ctypes.c_int)]),
    "qic_batch_plan": (
        ctypes.c_int,
        [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp, ctypes.c_int,
         ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_size_t)],
    ),
    "qic_batch_decode_attention": (ctypes.c_int, [ctypes.POINTER(BatchDecodeArgs), _vp]),
    "qic_decode_attention_noalloc": (ctypes.c_int, [ctypes.POINTER(DecodeArgs), _vp]),
    "qic_noalloc_scratch_bytes": (ctypes.c_size_t, []),
    "qic_noalloc_status": (ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_int)]),
    "qic_partial_floats": (ctypes.c_size_t, [ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    "qic_attention_merge": (
        ctypes.c_int, [ctypes.c_int, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp, _vp, _vp]),
    "qic_cp_exchange_bytes": (ctypes.c_size_t, [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]),
    "qic_cp_decode_attention": (ctypes.c_int, [ctypes.POINTER(DecodeArgs), ctypes.POINTER(CpArgs), _vp]),
    "qic_device_alloc": (ctypes.c_int, [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p)]),
    "qic_device_free": (ctypes.c_int, [_vp]),
    "qic_ipc_get_handle": (ctypes.c_int, [_vp, _vp]),
    "qic_ipc_open_handle": (ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_void_p)]),
    "qic_ipc_close_handle": (ctypes.c_int, [_vp]),
}

_LIB: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """Loads libqic.so once. Raises if it has not been built: there is no fallback."""
    global _LIB
    if _LIB is None:
        path = lib_path()
        if not path.exists():
            raise ImportError(f"{path} is missing; build it with `python -m qwenincuda_b200.build`")
        handle = ctypes.CDLL(str(path), mode=ctypes.RTLD_LOCAL)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = handle
    return _LIB


def check(status: int, what: str) -> None:
    if status != 0:
        raise QicError(status, what)
