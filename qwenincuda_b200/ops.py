"""Tensor-level wrappers over the C-ABI, mirroring the reference's call surface.

Names and argument order follow include/kernels.cuh of the QweninCuda project
(launch_head_rmsnorm, launch_rope_inplace, launch_sigmoid_mul_inplace,
launch_flash_attention, launch_paged_attention) with torch tensors in place of raw
device pointers, plus the fused entry points this library adds (kv_append,
decode_attention, gated_delta_decode). Every call runs on the current torch CUDA
stream unless a stream is given, and raises QicError on a non-success status.
"""
from __future__ import annotations

import ctypes

import torch

from .abi import (
    QIC_DTYPE_BF16,
    QIC_DTYPE_F16,
    QIC_DETERMINISTIC,
    QIC_DEVICE_SEQ_LEN,
    QIC_GDN_STATES_READY,
    QIC_EXPLICIT_POSITION,
    QIC_FUSE_APPEND,
    QIC_FUSE_Q_PROLOGUE,
    QIC_PARTIAL_OUT,
    QIC_PDL,
    QIC_PLAN_ITEM_BYTES,
    QIC_Q_GATE_INTERLEAVED,
    BatchDecodeArgs,
    DecodeArgs,
    GdnArgs,
    check,
    lib,
)


def dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return QIC_DTYPE_BF16
    if t.dtype == torch.float16:
        return QIC_DTYPE_F16
    raise TypeError(f"unsupported dtype {t.dtype}; expected bfloat16 or float16")


def _ptr(t):
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("expected a CUDA tensor")
    return t.data_ptr()


def _stream(stream) -> int | None:
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, torch.cuda.Stream):
        return stream.cuda_stream
    return int(stream)


class Workspace:
    """Caller-owned split-KV scratch (partials, merge counters, device status word)."""

    def __init__(self, num_heads: int, num_kv_heads: int, head_dim: int, max_seq_len: int, device=None,
                 stream=None):
        nbytes = lib().qic_decode_workspace_bytes(num_heads, num_kv_heads, head_dim, max_seq_len)
        if nbytes == 0:
            raise ValueError("invalid workspace shape")
        self.nbytes = int(nbytes)
        self.buf = torch.empty(self.nbytes, dtype=torch.uint8, device=device or "cuda")
        check(lib().qic_workspace_init(self.buf.data_ptr(), self.nbytes, _stream(stream)), "qic_workspace_init")

    @property
    def ptr(self) -> int:
        return self.buf.data_ptr()

    def status(self, stream=None) -> int:
        """Reads and clears the device status word (QIC_DEV_* bits)."""
        v = ctypes.c_int(0)
        check(lib().qic_workspace_status(self.ptr, _stream(stream), ctypes.byref(v)), "qic_workspace_status")
        return v.value


def launch_head_rmsnorm(x, weight, num_heads, head_dim, eps, out, stream=None):
    check(lib().qic_head_rmsnorm(dtype_code(x), _ptr(x), _ptr(weight), num_heads, head_dim, eps, _ptr(out),
                                 _stream(stream)), "launch_head_rmsnorm")


def launch_rope_inplace(q_or_k, num_heads, head_dim, position, rope_theta, stream=None):
    check(lib().qic_rope_inplace(dtype_code(q_or_k), _ptr(q_or_k), num_heads, head_dim, position, rope_theta,
                                 _stream(stream)), "launch_rope_inplace")


def launch_sigmoid_mul_inplace(x, gate, n, stream=None):
    check(lib().qic_sigmoid_mul_inplace(dtype_code(x), _ptr(x), _ptr(gate), n, _stream(stream)),
          "launch_sigmoid_mul_inplace")


def kv_append(k_new, v_new, k_norm_w, eps, rope_theta, position, k_cache, v_cache, num_kv_heads, head_dim,
              page_table=None, page_size=16, cache_tokens=None, stream=None):
    """Fused head-RMSNorm(k) + RoPE(k) + write of k and v into the slot of `position`."""
    if cache_tokens is None:
        cache_tokens = k_cache.numel() // (num_kv_heads * head_dim)
    check(lib().qic_kv_append(dtype_code(k_cache), _ptr(k_new), _ptr(v_new), _ptr(k_norm_w), eps, rope_theta,
                              position, _ptr(k_cache), _ptr(v_cache), _ptr(page_table), page_size, cache_tokens,
                              num_kv_heads, head_dim, _stream(stream)), "kv_append")


def decode_args(*, q, k_cache, v_cache, out, num_heads, num_kv_heads, head_dim, seq_len, page_table=None,
                page_size=16, gate=None, q_norm_w=None, k_norm_w=None, k_new=None, v_new=None, eps=1e-6,
                rope_theta=1.0e6, fuse_q=False, fuse_append=False, workspace=None, num_splits=0,
                cache_tokens=None, pdl=False, cluster_size=0, position=None, partial_out=False,
                deterministic=False, q_gate_interleaved=False, seq_len_dev=None) -> DecodeArgs:
    """qic_decode_args for one call. position: RoPE position of q and the appended k
    (default seq_len - 1). partial_out: `out` is an fp32 tensor of
    num_kv_heads * partial_floats(...) elements receiving the (o, lse) partial.
    deterministic: bitwise-reproducible outputs (no dynamic stage pool).
    q_gate_interleaved: q is the [H, 2d] q/gate projection and out is gated by its
    second halves (gate must be None). seq_len_dev: a device int32 tensor holding the
    current length, read when the kernel starts (seq_len is then its upper bound)."""
    a = DecodeArgs()
    a.dtype = dtype_code(k_cache)
    a.num_heads = num_heads
    a.num_kv_heads = num_kv_heads
    a.head_dim = head_dim
    a.seq_len = seq_len
    a.page_size = page_size if page_table is not None else 0
    a.cache_tokens = cache_tokens if cache_tokens is not None else k_cache.numel() // (num_kv_heads * head_dim)
    a.q = _ptr(q)
    a.k_cache = _ptr(k_cache)
    a.v_cache = _ptr(v_cache)
    a.page_table = _ptr(page_table)
    a.gate = _ptr(gate)
    a.out = _ptr(out)
    a.flags = _flags(fuse_q, fuse_append, pdl, q_gate_interleaved)
    if position is not None:
        a.flags |= QIC_EXPLICIT_POSITION
        a.position = int(position)
    if deterministic:
        a.flags |= QIC_DETERMINISTIC
    if seq_len_dev is not None:
        if seq_len_dev.dtype != torch.int32 or not seq_len_dev.is_cuda:
            raise TypeError("seq_len_dev is a CUDA int32 tensor")
        a.flags |= QIC_DEVICE_SEQ_LEN
        a.seq_len_dev = seq_len_dev.data_ptr()
    if partial_out:
        if out.dtype != torch.float32:
            raise TypeError("a partial output is float32")
        a.flags |= QIC_PARTIAL_OUT
    a.eps = eps
    a.rope_theta = rope_theta
    a.q_norm_w = _ptr(q_norm_w)
    a.k_norm_w = _ptr(k_norm_w)
    a.k_new = _ptr(k_new)
    a.v_new = _ptr(v_new)
    if workspace is not None:
        a.workspace = workspace.ptr
        a.workspace_bytes = workspace.nbytes
    a.num_splits = num_splits
    a.cluster_size = cluster_size
    return a


def _flags(fuse_q, fuse_append, pdl, q_gate_interleaved=False):
    return ((QIC_FUSE_Q_PROLOGUE if fuse_q else 0) | (QIC_FUSE_APPEND if fuse_append else 0) |
            (QIC_PDL if pdl else 0) | (QIC_Q_GATE_INTERLEAVED if q_gate_interleaved else 0))


def decode_launch_shape(*, num_heads, num_kv_heads, head_dim, seq_len, dtype=torch.bfloat16, pdl=False,
                        workspace=True, num_splits=0, cluster_size=0, fuse_append=False):
    """(splits per kv head, CTAs per cluster) that qic_decode_attention uses for this
    shape. workspace: whether the call passes one (without it the splits are merged
    on chip only, at most 16). fuse_append: QIC_FUSE_APPEND (an appended token alone
    in the last stage is not copied, so that stage does not count)."""
    a = DecodeArgs()
    a.dtype = QIC_DTYPE_BF16 if dtype == torch.bfloat16 else QIC_DTYPE_F16
    a.num_heads, a.num_kv_heads, a.head_dim, a.seq_len = num_heads, num_kv_heads, head_dim, seq_len
    a.flags = (QIC_PDL if pdl else 0) | (QIC_FUSE_APPEND if fuse_append else 0)
    a.workspace = 16 if workspace else None  # only its presence is read
    a.num_splits, a.cluster_size = num_splits, cluster_size
    n, c = ctypes.c_int(0), ctypes.c_int(0)
    check(lib().qic_decode_launch_shape(ctypes.byref(a), ctypes.byref(n), ctypes.byref(c)), "qic_decode_launch_shape")
    return n.value, c.value


def decode_attention(stream=None, **kw):
    """Split-KV decode attention; see qic_decode_attention in include/qic.h."""
    a = decode_args(**kw)
    check(lib().qic_decode_attention(ctypes.byref(a), _stream(stream)), "qic_decode_attention")


def partial_floats(num_heads: int, num_kv_heads: int, head_dim: int) -> int:
    """fp32 elements per kv head of a partial: G*d outputs, G log-sum-exp values, padding."""
    return int(lib().qic_partial_floats(num_heads, num_kv_heads, head_dim))


def attention_merge(partials, num_heads, num_kv_heads, head_dim, out, gate=None, stream=None):
    """out = log-sum-exp merge of stacked partials [n, Hkv, partial_floats] (+ gate)."""
    if partials.dtype != torch.float32:
        raise TypeError("partials are float32")
    n = partials.numel() // (num_kv_heads * partial_floats(num_heads, num_kv_heads, head_dim))
    check(lib().qic_attention_merge(dtype_code(out), _ptr(partials), n, num_heads, num_kv_heads, head_dim, _ptr(gate),
                                    _ptr(out), _stream(stream)), "qic_attention_merge")


def launch_flash_attention(q, k_cache, v_cache, num_heads, num_kv_heads, head_dim, seq_len, context,
                           workspace=None, stream=None):
    decode_attention(q=q, k_cache=k_cache, v_cache=v_cache, out=context, num_heads=num_heads,
                     num_kv_heads=num_kv_heads, head_dim=head_dim, seq_len=seq_len, workspace=workspace,
                     stream=stream)


def launch_paged_attention(q, k_cache, v_cache, page_table, page_size, num_heads, num_kv_heads, head_dim, seq_len,
                           context, workspace=None, stream=None):
    decode_attention(q=q, k_cache=k_cache, v_cache=v_cache, out=context, num_heads=num_heads,
                     num_kv_heads=num_kv_heads, head_dim=head_dim, seq_len=seq_len, page_table=page_table,
                     page_size=page_size, workspace=workspace, stream=stream)


def gated_delta_decode(*, qkv, z, b, a, conv_w, dt_bias, a_log, norm_w, conv_state, recurrent_state, out,
                       num_k_heads, num_v_heads, k_head_dim=128, v_head_dim=128, conv_kernel=4, eps=1e-6,
                       pdl=False, states_ready=False, status=None, stream=None):
    """One GatedDeltaNet decode step; conv_state and recurrent_state (fp32) are updated in place.
    states_ready (with pdl): QIC_GDN_STATES_READY, the caller guarantees that the kernels
    which last wrote the states have completed before this launch starts.
    status: an optional CUDA int32 tensor whose first word collects QIC_DEV_TIMEOUT."""
    g = GdnArgs()
    g.flags = (QIC_PDL if pdl else 0) | (QIC_GDN_STATES_READY if states_ready else 0)
    g.dtype = dtype_code(qkv)
    g.num_k_heads = num_k_heads
    g.num_v_heads = num_v_heads
    g.k_head_dim = k_head_dim
    g.v_head_dim = v_head_dim
    g.conv_kernel = conv_kernel
    g.eps = eps
    g.qkv, g.z, g.b, g.a = _ptr(qkv), _ptr(z), _ptr(b), _ptr(a)
    g.conv_w, g.dt_bias, g.a_log, g.norm_w = _ptr(conv_w), _ptr(dt_bias), _ptr(a_log), _ptr(norm_w)
    g.conv_state, g.recurrent_state, g.out = _ptr(conv_state), _ptr(recurrent_state), _ptr(out)
    g.status = _ptr(status)
    check(lib().qic_gated_delta_decode(ctypes.byref(g), _stream(stream)), "qic_gated_delta_decode")


class BatchPlan:
    """Work plan of a batched paged decode (qic_batch_plan), with its device copy and
    the workspace it needs. seq_lens are host integers: tokens attended per sequence."""

    def __init__(self, seq_lens, num_heads, num_kv_heads, head_dim, target_ctas=0, device=None, stream=None):
        L = lib()
        lens = (ctypes.c_int32 * len(seq_lens))(*[int(x) for x in seq_lens])
        items = ctypes.c_int(0)
        wsb = ctypes.c_size_t(0)
        check(L.qic_batch_plan(ctypes.cast(lens, ctypes.c_void_p), len(seq_lens), num_heads, num_kv_heads, head_dim,
                               target_ctas, None, 0, ctypes.byref(items), ctypes.byref(wsb)), "qic_batch_plan")
        host = torch.empty(items.value * QIC_PLAN_ITEM_BYTES, dtype=torch.uint8)
        check(L.qic_batch_plan(ctypes.cast(lens, ctypes.c_void_p), len(seq_lens), num_heads, num_kv_heads, head_dim,
                               target_ctas, host.data_ptr(), items.value, ctypes.byref(items), ctypes.byref(wsb)),
              "qic_batch_plan")
        self.items = items.value
        self.host = host
        self.device_plan = host.to(device or "cuda")
        self.workspace_bytes = int(wsb.value)
        self.workspace = torch.zeros(self.workspace_bytes, dtype=torch.uint8, device=device or "cuda")
        self.seq_lens = [int(x) for x in seq_lens]

    def status(self, stream=None) -> int:
        v = ctypes.c_int(0)
        check(lib().qic_workspace_status(self.workspace.data_ptr(), _stream(stream), ctypes.byref(v)),
              "qic_workspace_status")
        return v.value


def batch_decode_args(*, plan: BatchPlan, q, k_cache, v_cache, block_tables, out, num_heads, num_kv_heads, head_dim,
                      page_size=16, gate=None, q_norm_w=None, k_norm_w=None, k_new=None, v_new=None, eps=1e-6,
                      rope_theta=1.0e6, fuse_q=False, fuse_append=False, pdl=False, cache_tokens=None,
                      q_gate_interleaved=False):
    a = BatchDecodeArgs()
    a.dtype = dtype_code(k_cache)
    a.num_heads, a.num_kv_heads, a.head_dim = num_heads, num_kv_heads, head_dim
    a.batch = len(plan.seq_lens)
    a.page_size = page_size
    a.cache_tokens = cache_tokens if cache_tokens is not None else k_cache.numel() // (num_kv_heads * head_dim)
    a.max_pages_per_seq = block_tables.shape[1]
    a.flags = _flags(fuse_q, fuse_append, pdl, q_gate_interleaved)
    a.q, a.k_cache, a.v_cache = _ptr(q), _ptr(k_cache), _ptr(v_cache)
    a.block_tables, a.gate, a.out = _ptr(block_tables), _ptr(gate), _ptr(out)
    a.eps, a.rope_theta = eps, rope_theta
    a.q_norm_w, a.k_norm_w, a.k_new, a.v_new = _ptr(q_norm_w), _ptr(k_norm_w), _ptr(k_new), _ptr(v_new)
    a.plan = plan.device_plan.data_ptr()
    a.plan_items = plan.items
    a.workspace = plan.workspace.data_ptr()
    a.workspace_bytes = plan.workspace_bytes
    return a


def batch_decode_attention(stream=None, **kw):
    """Batched paged decode over a shared page pool; see qic_batch_decode_attention."""
    a = batch_decode_args(**kw)
    check(lib().qic_batch_decode_attention(ctypes.byref(a), _stream(stream)), "qic_batch_decode_attention")


def gemv_args(*, x, weights, outs, residuals=None, norm_w=None, eps=1e-6, swiglu=False, pdl=False,
              splits=0, status=None) -> "GemvArgs":
    """qic_gemv_args for one launch: x [K]; weights: list of [K, N_k] tensors (N_k
    contiguous, the reference's column-major layout); outs: list of [N_k] outputs (with
    swiglu, weights = [w_gate, w_up] and outs = [out], silu(gate)*up); residuals: list
    of [N_k] tensors added to the products (may be the outs themselves); norm_w: fuse
    the RMSNorm of x with this weight."""
    from .abi import QIC_GEMV_MAX_SEGMENTS, QIC_GEMV_RESIDUAL, QIC_GEMV_RMSNORM, QIC_GEMV_SWIGLU, GemvArgs

    if not 1 <= len(weights) <= QIC_GEMV_MAX_SEGMENTS:
        raise ValueError(f"1..{QIC_GEMV_MAX_SEGMENTS} weight segments")
    outs = list(outs) + [None] * (len(weights) - len(outs))
    a = GemvArgs()
    a.dtype = dtype_code(x)
    a.in_dim = x.numel()
    a.num_segments = len(weights)
    a.x = _ptr(x)
    a.eps = eps
    a.splits = splits
    flags = QIC_PDL if pdl else 0
    if norm_w is not None:
        flags |= QIC_GEMV_RMSNORM
        a.norm_w = _ptr(norm_w)
    if swiglu:
        flags |= QIC_GEMV_SWIGLU
    if residuals is not None:
        flags |= QIC_GEMV_RESIDUAL
    for k, w in enumerate(weights):
        if w.dim() != 2 or w.shape[0] != a.in_dim or not w.is_contiguous():
            raise ValueError(f"weight {k}: a contiguous [{a.in_dim}, N] tensor")
        a.seg[k].w = _ptr(w)
        a.seg[k].out_dim = w.shape[1]
        a.seg[k].out = _ptr(outs[k])
        if residuals is not None:
            a.seg[k].residual = _ptr(residuals[k])
    if status is not None:
        if status.dtype != torch.int32 or not status.is_cuda:
            raise TypeError("status is a CUDA int32 tensor")
        a.status = status.data_ptr()
    a.flags = flags
    return a


def gemv(stream=None, **kw) -> None:
    """Weight-streaming GEMV projections of one token; see qic_gemv in include/qic.h."""
    a = gemv_args(**kw)
    check(lib().qic_gemv(ctypes.byref(a), _stream(stream)), "qic_gemv")


def gemv_launch_shape(**kw) -> tuple[int, int]:
    """(splits, column tiles) qic_gemv uses for these arguments."""
    a = gemv_args(**kw)
    s, t = ctypes.c_int(0), ctypes.c_int(0)
    check(lib().qic_gemv_launch_shape(ctypes.byref(a), ctypes.byref(s), ctypes.byref(t)), "qic_gemv_launch_shape")
    return s.value, t.value


class Model:
    """A decode-step runner (qic_model_*): load(path) for a qmini v4 file, or
    from_weights(config, dtype, weights) over device tensors the caller keeps alive.
    decode(token, position) replays the captured step and returns the greedy token
    (and the logits when asked), like the reference's QwenMiniModel::decode_next."""

    def __init__(self, handle: int, keep=None):
        self.handle = ctypes.c_void_p(handle)
        self._keep = keep
        cfg = __import__("qwenincuda_b200.abi", fromlist=["ModelConfig"]).ModelConfig()
        wb = ctypes.c_size_t(0)
        check(lib().qic_model_info(self.handle, ctypes.byref(cfg), ctypes.byref(wb)), "qic_model_info")
        self.config = cfg
        self.weight_bytes = wb.value

    @classmethod
    def load(cls, path, max_seq_len: int = 0) -> "Model":
        h = ctypes.c_void_p(0)
        check(lib().qic_model_load(str(path).encode(), max_seq_len, ctypes.byref(h)), "qic_model_load")
        return cls(h.value)

    @classmethod
    def from_weights(cls, config, dtype: int, tok_embeddings, final_norm, lm_head, layers) -> "Model":
        """layers: list of dicts of tensors keyed by qic_layer_weights field names (plus is_linear)."""
        from .abi import LayerWeights, ModelConfig, ModelWeights

        arr = (LayerWeights * len(layers))()
        for i, lw in enumerate(layers):
            arr[i].is_linear = int(lw.get("is_linear", 0))
            for k, t in lw.items():
                if k != "is_linear" and t is not None:
                    setattr(arr[i], k, t.data_ptr())
        types = (ctypes.c_int32 * len(layers))(*[int(lw.get("is_linear", 0)) for lw in layers])
        cfg = ModelConfig(**{k: v for k, v in config.items() if k != "layer_types"})
        cfg.layer_types = ctypes.cast(types, ctypes.POINTER(ctypes.c_int32))
        w = ModelWeights(tok_embeddings=tok_embeddings.data_ptr(), final_norm=final_norm.data_ptr(),
                         lm_head=lm_head.data_ptr(), layers=ctypes.cast(arr, ctypes.POINTER(LayerWeights)))
        h = ctypes.c_void_p(0)
        check(lib().qic_model_create(ctypes.byref(cfg), dtype, ctypes.byref(w), ctypes.byref(h)), "qic_model_create")
        return cls(h.value, keep=(tok_embeddings, final_norm, lm_head, layers))

    def reset(self) -> None:
        check(lib().qic_model_reset(self.handle), "qic_model_reset")

    def decode(self, token: int, position: int, logits=None, stream=None) -> int:
        """Greedy next token; `logits`: optional CPU 16-bit tensor of vocab_size elements."""
        nxt = ctypes.c_int(-1)
        ptr = None if logits is None else ctypes.c_void_p(logits.data_ptr())
        check(lib().qic_model_decode(self.handle, int(token), int(position), ptr, ctypes.byref(nxt), _stream(stream)),
              "qic_model_decode")
        return nxt.value

    def set_position(self, token: int, position: int, stream=None) -> None:
        check(lib().qic_model_set_position(self.handle, int(token), int(position), _stream(stream)),
              "qic_model_set_position")

    def step_graph(self, stream=None) -> None:
        check(lib().qic_model_step_graph(self.handle, _stream(stream)), "qic_model_step_graph")

    def close(self) -> None:
        if self.handle:
            check(lib().qic_model_free(self.handle), "qic_model_free")
            self.handle = ctypes.c_void_p(0)
