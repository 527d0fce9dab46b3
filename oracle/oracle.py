"""TEST INFRASTRUCTURE ONLY — Python bindings of the oracle.

* ``Oracle``: ctypes binding of oracle/libqic_oracle.so, the CPU restatement of the
  reference path (oracle/qic_oracle.c). Takes and returns CPU torch tensors
  (bfloat16 / float16 / float32 / int32).
* ``RefKernels``: ctypes binding of oracle/_ref/libqicref_{f16,bf16}.so, the
  reference's own src/kernels.cu compiled unchanged for sm_100a (oracle/Makefile).
  Takes CUDA torch tensors; launches on the legacy default stream like the
  reference and synchronises.
* ``RefModel``: the reference model's gemv and FFN block members from the same
  libraries as ``RefGatedDelta`` (CUDA tensors in).
* ``RefGatedDelta``: ctypes binding of oracle/_ref/libqicref_gdn{,_bf16}.so, the
  reference's own GatedDeltaNet decode step (src/model.cpp:656-795, compiled unchanged
  inside oracle/ref_gdn_harness.cpp; fp16, or the bfloat16 instance). Takes and returns
  CPU tensors (16-bit inputs, fp32 states); needs a CUDA device, through which the
  reference copies its inputs.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference legs
use this module; the product library never does.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "libqic_oracle.so"
REF_DIR = HERE / "_ref"

_vp = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64
_f = ctypes.c_float


def _code(dtype: torch.dtype) -> int:
    if dtype == torch.bfloat16:
        return 1
    if dtype == torch.float16:
        return 0
    raise TypeError(dtype)


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _cpu(t):
    if t is None:
        return None
    t = t.detach()
    if t.is_cuda:
        t = t.cpu()
    return t.contiguous()


class Oracle:
    """CPU restatement of the reference hot path (see qic_oracle.c for the citations)."""

    def __init__(self, path: Path = ORACLE_SO):
        if not path.exists():
            raise FileNotFoundError(f"{path} not built (make -C oracle)")
        lib = ctypes.CDLL(str(path))
        lib.qico_head_rmsnorm.argtypes = [_i, _vp, _vp, _i, _i, _f, _vp]
        lib.qico_rope_inplace.argtypes = [_i, _vp, _i, _i, _i, _f]
        lib.qico_sigmoid_mul_inplace.argtypes = [_i, _vp, _vp, _i64]
        lib.qico_kv_append.argtypes = [_i, _vp, _vp, _vp, _f, _f, _i, _vp, _vp, _vp, _i, _i, _i]
        lib.qico_attention.argtypes = [_i, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp]
        lib.qico_batched_attention.argtypes = [_i, _vp, _vp, _vp, _vp, _i, _vp, _i, _i, _i, _i, _i, _vp]
        lib.qico_gated_delta_decode.argtypes = [_i, _i, _i, _i, _i, _i, _f] + [_vp] * 11
        lib.qico_num_threads.restype = _i
        lib.qico_set_num_threads.argtypes = [_i]
        self.lib = lib

    def num_threads(self) -> int:
        return self.lib.qico_num_threads()

    def set_num_threads(self, n: int) -> None:
        self.lib.qico_set_num_threads(n)

    def head_rmsnorm(self, x, w, num_heads, head_dim, eps):
        x, w = _cpu(x), _cpu(w)
        out = torch.empty_like(x)
        self.lib.qico_head_rmsnorm(_code(x.dtype), _p(x), _p(w), num_heads, head_dim, eps, _p(out))
        return out

    def rope(self, x, num_heads, head_dim, position, theta):
        x = _cpu(x).clone()
        self.lib.qico_rope_inplace(_code(x.dtype), _p(x), num_heads, head_dim, position, theta)
        return x

    def sigmoid_mul(self, x, gate):
        x, gate = _cpu(x).clone(), _cpu(gate)
        self.lib.qico_sigmoid_mul_inplace(_code(x.dtype), _p(x), _p(gate), x.numel())
        return x

    def kv_append(self, k_new, v_new, k_norm_w, eps, theta, position, k_cache, v_cache, num_kv_heads, head_dim,
                  page_table=None, page_size=16):
        """Returns updated copies of (k_cache, v_cache)."""
        kc, vc = _cpu(k_cache).clone(), _cpu(v_cache).clone()
        k_new, v_new, w = _cpu(k_new), _cpu(v_new), _cpu(k_norm_w)
        pt = _cpu(page_table)
        if pt is not None:
            pt = pt.to(torch.int32)
        self.lib.qico_kv_append(_code(kc.dtype), _p(k_new), _p(v_new), _p(w), eps, theta, position, _p(kc), _p(vc),
                                _p(pt), page_size, num_kv_heads, head_dim)
        return kc, vc

    def attention(self, q, k_cache, v_cache, num_heads, num_kv_heads, head_dim, seq_len, page_table=None,
                  page_size=16):
        q, kc, vc = _cpu(q), _cpu(k_cache), _cpu(v_cache)
        pt = _cpu(page_table)
        if pt is not None:
            pt = pt.to(torch.int32)
        out = torch.empty(num_heads * head_dim, dtype=q.dtype)
        self.lib.qico_attention(_code(q.dtype), _p(q), _p(kc), _p(vc), _p(pt), page_size, num_heads, num_kv_heads,
                                head_dim, seq_len, _p(out))
        return out

    def batched_attention(self, q, k_cache, v_cache, block_tables, seq_lens, page_size, num_heads, num_kv_heads,
                          head_dim):
        q, kc, vc = _cpu(q), _cpu(k_cache), _cpu(v_cache)
        bt = _cpu(block_tables).to(torch.int32)
        sl = _cpu(seq_lens).to(torch.int32)
        batch, max_pages = bt.shape
        out = torch.empty(batch, num_heads * head_dim, dtype=q.dtype)
        self.lib.qico_batched_attention(_code(q.dtype), _p(q), _p(kc), _p(vc), _p(bt), max_pages, _p(sl), batch,
                                        page_size, num_heads, num_kv_heads, head_dim, _p(out))
        return out

    def gated_delta(self, *, qkv, z, b, a, conv_w, dt_bias, a_log, norm_w, conv_state, recurrent_state,
                    num_k_heads, num_v_heads, k_head_dim=128, v_head_dim=128, conv_kernel=4, eps=1e-6):
        """Returns (out, new conv_state, new recurrent_state); inputs are not modified."""
        ins = [_cpu(t) for t in (qkv, z, b, a, conv_w, dt_bias, a_log, norm_w)]
        cs = _cpu(conv_state).float().clone()
        rs = _cpu(recurrent_state).float().clone()
        out = torch.empty(num_v_heads * v_head_dim, dtype=ins[0].dtype)
        self.lib.qico_gated_delta_decode(_code(ins[0].dtype), num_k_heads, num_v_heads, k_head_dim, v_head_dim,
                                         conv_kernel, eps, *[_p(t) for t in ins], _p(cs), _p(rs), _p(out))
        return out, cs, rs


class RefKernels:
    """The reference's own kernels (src/kernels.cu) built for sm_100a; CUDA tensors in, legacy default stream."""

    def __init__(self, dtype: torch.dtype):
        name = "libqicref_bf16.so" if dtype == torch.bfloat16 else "libqicref_f16.so"
        path = REF_DIR / name
        if not path.exists():
            raise FileNotFoundError(f"{path} not built (make -C oracle ref REF=<reference project root>)")
        lib = ctypes.CDLL(str(path), mode=ctypes.RTLD_LOCAL)
        lib.qicref_head_rmsnorm.argtypes = [_vp, _vp, _i, _i, _f, _vp]
        lib.qicref_rope_inplace.argtypes = [_vp, _i, _i, _i, _f]
        lib.qicref_sigmoid_mul_inplace.argtypes = [_vp, _vp, _i]
        lib.qicref_split_q_gate.argtypes = [_vp, _i, _i, _vp, _vp]
        lib.qicref_flash_attention.argtypes = [_vp, _vp, _vp, _i, _i, _i, _i, _vp]
        lib.qicref_paged_attention.argtypes = [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp]
        lib.qicref_copy_row.argtypes = [_vp, _vp, ctypes.c_longlong, _i]
        lib.qicref_rmsnorm.argtypes = [_vp, _vp, _i, _f, _vp]
        lib.qicref_add_inplace.argtypes = [_vp, _vp, _i]
        lib.qicref_swiglu.argtypes = [_vp, _vp, _i, _vp]
        self.lib = lib
        self.dtype = dtype

    @staticmethod
    def available(dtype: torch.dtype) -> bool:
        name = "libqicref_bf16.so" if dtype == torch.bfloat16 else "libqicref_f16.so"
        return (REF_DIR / name).exists()

    def _chk(self, rc, what):
        if rc != 0:
            raise RuntimeError(f"reference {what} failed: cudaError {rc}")

    def sync(self):
        self._chk(self.lib.qicref_synchronize(), "synchronize")

    def head_rmsnorm(self, x, w, num_heads, head_dim, eps, out):
        torch.cuda.synchronize()
        self._chk(self.lib.qicref_head_rmsnorm(_p(x), _p(w), num_heads, head_dim, eps, _p(out)), "head_rmsnorm")
        self.sync()

    def rope_inplace(self, x, num_heads, head_dim, position, theta):
        torch.cuda.synchronize()
        self._chk(self.lib.qicref_rope_inplace(_p(x), num_heads, head_dim, position, theta), "rope")
        self.sync()

    def sigmoid_mul_inplace(self, x, gate, n):
        torch.cuda.synchronize()
        self._chk(self.lib.qicref_sigmoid_mul_inplace(_p(x), _p(gate), n), "sigmoid_mul")
        self.sync()

    def split_q_gate(self, packed, num_heads, head_dim, q, gate):
        torch.cuda.synchronize()
        self._chk(self.lib.qicref_split_q_gate(_p(packed), num_heads, head_dim, _p(q), _p(gate)), "split_q_gate")
        self.sync()

    def flash_attention(self, q, k_cache, v_cache, num_heads, num_kv_heads, head_dim, seq_len, ctx, sync=True):
        if sync:
            torch.cuda.synchronize()
        self._chk(self.lib.qicref_flash_attention(_p(q), _p(k_cache), _p(v_cache), num_heads, num_kv_heads, head_dim,
                                                  seq_len, _p(ctx)), "flash_attention")
        if sync:
            self.sync()

    def paged_attention(self, q, k_cache, v_cache, page_table, page_size, num_heads, num_kv_heads, head_dim,
                        seq_len, ctx, sync=True):
        if sync:
            torch.cuda.synchronize()
        self._chk(self.lib.qicref_paged_attention(_p(q), _p(k_cache), _p(v_cache), _p(page_table), page_size,
                                                  num_heads, num_kv_heads, head_dim, seq_len, _p(ctx)),
                  "paged_attention")
        if sync:
            self.sync()

    def rmsnorm(self, x, w, n, eps, out):
        torch.cuda.synchronize()
        self._chk(self.lib.qicref_rmsnorm(_p(x), _p(w), n, eps, _p(out)), "rmsnorm")
        self.sync()

    def add_inplace(self, x, y, n):
        torch.cuda.synchronize()
        self._chk(self.lib.qicref_add_inplace(_p(x), _p(y), n), "add_inplace")
        self.sync()

    def swiglu(self, gate, up, n, out):
        torch.cuda.synchronize()
        self._chk(self.lib.qicref_swiglu(_p(gate), _p(up), n, _p(out)), "swiglu")
        self.sync()

    def append_chain(self, k_new, v_new, k_norm_w, eps, theta, position, k_cache, v_cache, num_kv_heads, head_dim,
                     slot):
        """The reference's append sequence (src/model.cpp:634,637,639-641) on copies of k/v,
        written at row `slot` of the caches."""
        k = k_new.clone()
        self.head_rmsnorm(k, k_norm_w, num_kv_heads, head_dim, eps, k)
        self.rope_inplace(k, num_kv_heads, head_dim, position, theta)
        kv_dim = num_kv_heads * head_dim
        self._chk(self.lib.qicref_copy_row(_p(k_cache), _p(k), slot, kv_dim), "copy k")
        self._chk(self.lib.qicref_copy_row(_p(v_cache), _p(v_new), slot, kv_dim), "copy v")
        self.sync()
        return k


class RefGatedDelta:
    """The reference's own GatedDeltaNet decode step (run_linear_attention_block,
    src/model.cpp:656-795): fp16 as the reference ships it, or its bfloat16 instance."""

    def __init__(self, dtype: torch.dtype = torch.float16):
        self.dtype = dtype
        path = REF_DIR / ("libqicref_gdn.so" if dtype == torch.float16 else "libqicref_gdn_bf16.so")
        if not path.exists():
            raise FileNotFoundError(f"{path} not built (make -C oracle ref REF=<reference project root>)")
        lib = ctypes.CDLL(str(path), mode=ctypes.RTLD_LOCAL)
        lib.qicref_gdn_step.argtypes = [_i, _i, _i, _i, _i, _f] + [_vp] * 11
        lib.qicref_gdn_step.restype = _i
        lib.qicref_gdn_create.argtypes = [_i, _i, _i, _i, _i, _f] + [_vp] * 6
        lib.qicref_gdn_create.restype = _vp
        lib.qicref_gdn_run.argtypes = [_vp] * 6
        lib.qicref_gdn_run.restype = _i
        lib.qicref_gdn_states.argtypes = [_vp] * 3
        lib.qicref_gdn_destroy.argtypes = [_vp]
        self.lib = lib

    @staticmethod
    def available(dtype: torch.dtype = torch.float16) -> bool:
        return (REF_DIR / ("libqicref_gdn.so" if dtype == torch.float16 else "libqicref_gdn_bf16.so")).exists()

    def step(self, *, qkv, z, b, a, conv_w, dt_bias, a_log, norm_w, conv_state, recurrent_state, num_k_heads,
             num_v_heads, k_head_dim=128, v_head_dim=128, conv_kernel=4, eps=1e-6):
        """Returns (out, new conv_state, new recurrent_state); inputs are not modified."""
        ins = [_cpu(t) for t in (qkv, z, b, a, conv_w, dt_bias, a_log, norm_w)]
        if any(t.dtype != self.dtype for t in ins):
            raise TypeError(f"this instance of the reference's step takes {self.dtype}")
        cs = _cpu(conv_state).float().clone()
        rs = _cpu(recurrent_state).float().clone()
        out = torch.empty(num_v_heads * v_head_dim, dtype=self.dtype)
        rc = self.lib.qicref_gdn_step(num_k_heads, num_v_heads, k_head_dim, v_head_dim, conv_kernel, eps,
                                      *[_p(t) for t in ins], _p(cs), _p(rs), _p(out))
        if rc != 0:
            raise RuntimeError("reference GatedDeltaNet step failed")
        return out, cs, rs

    def layer(self, *, conv_w, dt_bias, a_log, norm_w, conv_state, recurrent_state, num_k_heads, num_v_heads,
              k_head_dim=128, v_head_dim=128, conv_kernel=4, eps=1e-6):
        """One linear-attention layer of the reference model, set up once (weights on the
        device, cuBLAS handle), for repeated steps; close() releases it."""
        return _RefGatedDeltaLayer(self.lib, self.dtype, conv_w, dt_bias, a_log, norm_w, conv_state,
                                   recurrent_state, num_k_heads, num_v_heads, k_head_dim, v_head_dim, conv_kernel, eps)


class RefModel:
    """The reference model's projection members run on CUDA tensors: QwenMiniModel::gemv
    (src/model.cpp:603-617, cuBLAS with the reference's arguments) and run_ffn_block
    (src/model.cpp:797-807), compiled unchanged into oracle/_ref/libqicref_gdn{,_bf16}.so."""

    def __init__(self, dtype: torch.dtype = torch.float16):
        self.dtype = dtype
        path = REF_DIR / ("libqicref_gdn.so" if dtype == torch.float16 else "libqicref_gdn_bf16.so")
        if not path.exists():
            raise FileNotFoundError(f"{path} not built (make -C oracle ref REF=<reference project root>)")
        lib = ctypes.CDLL(str(path), mode=ctypes.RTLD_LOCAL)
        lib.qicref_gemv.argtypes = [_vp, _vp, _i, _i, _vp]
        lib.qicref_gemv.restype = _i
        lib.qicref_ffn_block.argtypes = [_vp, _vp, _vp, _vp, _vp, _i, _i, _f]
        lib.qicref_ffn_block.restype = _i
        self.lib = lib

    def gemv(self, x, w, in_dim, out_dim, out):
        """out = the reference's gemv of x with w [in_dim, out_dim] (out_dim contiguous)."""
        torch.cuda.synchronize()
        if self.lib.qicref_gemv(_p(x), _p(w), in_dim, out_dim, _p(out)) != 0:
            raise RuntimeError("reference gemv failed")

    def ffn_block(self, x, ffn_norm, w_gate, w_up, w_down, hidden, inter, eps):
        """x (in place) = the reference's FFN block of x."""
        torch.cuda.synchronize()
        if self.lib.qicref_ffn_block(_p(x), _p(ffn_norm), _p(w_gate), _p(w_up), _p(w_down), hidden, inter, eps) != 0:
            raise RuntimeError("reference FFN block failed")


class RefQwenModel:
    """The reference model end to end: QwenMiniModel::load of a qmini v4 file and
    decode_next (src/model.cpp:319-428, 823-845), compiled unchanged into
    oracle/_ref/libqicref_gdn.so (fp16, as the format stores)."""

    def __init__(self, path):
        lib_path = REF_DIR / "libqicref_gdn.so"
        if not lib_path.exists():
            raise FileNotFoundError(f"{lib_path} not built (make -C oracle ref REF=<reference project root>)")
        lib = ctypes.CDLL(str(lib_path), mode=ctypes.RTLD_LOCAL)
        lib.qicref_model_load.argtypes = [ctypes.c_char_p]
        lib.qicref_model_load.restype = _vp
        lib.qicref_model_decode.argtypes = [_vp, _i, _i, _vp]
        lib.qicref_model_decode.restype = _i
        lib.qicref_model_free.argtypes = [_vp]
        self.lib = lib
        self.h = lib.qicref_model_load(str(path).encode())
        if not self.h:
            raise RuntimeError(f"reference load of {path} failed")

    def decode(self, token, position, logits=None):
        """decode_next(token, position): the greedy token; `logits` (CPU fp16, vocab) receives the logits."""
        nxt = self.lib.qicref_model_decode(self.h, int(token), int(position), _p(logits))
        if nxt < 0:
            raise RuntimeError("reference decode_next failed")
        return nxt

    def close(self):
        if self.h:
            self.lib.qicref_model_free(self.h)
            self.h = None


class _RefGatedDeltaLayer:
    def __init__(self, lib, dtype, conv_w, dt_bias, a_log, norm_w, conv_state, recurrent_state, Hk, Hv, dk, dv, K,
                 eps):
        self.lib = lib
        self.shapes = (Hk, Hv, dk, dv, K)
        ws = [_cpu(t) for t in (conv_w, dt_bias, a_log, norm_w)]
        if any(t.dtype != dtype for t in ws):
            raise TypeError(f"this instance of the reference's step takes {dtype}")
        cs = _cpu(conv_state).float().contiguous()
        rs = _cpu(recurrent_state).float().contiguous()
        self.h = lib.qicref_gdn_create(Hk, Hv, dk, dv, K, eps, *[_p(t) for t in ws], _p(cs), _p(rs))
        if not self.h:
            raise RuntimeError("reference GatedDeltaNet set-up failed")

    def run(self, qkv=None, z=None, b=None, a=None, out=None):
        """One step; qkv/z/b/a (CPU fp16) replace the previous step's projections when given."""
        ins = [None if t is None else _cpu(t) for t in (qkv, z, b, a)]
        if self.lib.qicref_gdn_run(self.h, *[_p(t) for t in ins], _p(out)) != 0:
            raise RuntimeError("reference GatedDeltaNet step failed")

    def states(self):
        Hk, Hv, dk, dv, K = self.shapes
        cs = torch.empty((2 * Hk * dk + Hv * dv) * K, dtype=torch.float32)
        rs = torch.empty(Hv * dk * dv, dtype=torch.float32)
        self.lib.qicref_gdn_states(self.h, _p(cs), _p(rs))
        return cs, rs

    def close(self):
        if self.h:
            self.lib.qicref_gdn_destroy(self.h)
            self.h = None
