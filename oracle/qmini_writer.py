"""TEST INFRASTRUCTURE ONLY — writes synthetic model files in the reference's qmini v4
format, so that the reference's own loader and decode loop (QwenMiniModel::load and
decode_next, src/model.cpp:319-428 and 823-845 of the QweninCuda project) and this
repository's runner (qic_model_load) run the same weights.

Format (the order QwenMiniModel::load reads, src/model.cpp:328-421): the 8 bytes
"QWENMINI", int32 version 4; int32 vocab_size, hidden_size, intermediate_size,
num_layers, num_heads, num_kv_heads, head_dim, linear_num_key_heads,
linear_num_value_heads, linear_key_head_dim, linear_value_head_dim,
linear_conv_kernel_dim, max_seq_len; float32 rms_norm_eps, rope_theta; int32 layer
kind per layer (0 full attention, 1 linear attention); then tensors, each a uint64
element count and that many fp16 values: tok_embeddings [vocab, hidden]; per layer
attn_norm [hidden], then for a linear layer in_qkv [hidden, conv_dim], in_z
[hidden, val_dim], in_b and in_a [hidden, Hv], conv1d_w [conv_dim, K], dt_bias [Hv],
a_log [Hv], norm_w [dv], out_proj [val_dim, hidden], or for a full-attention layer wq
[hidden, 2*q_dim], wk and wv [hidden, kv_dim], q_norm and k_norm [head_dim], wo
[q_dim, hidden]; then ffn_norm [hidden], w_gate and w_up [hidden, inter], w_down
[inter, hidden]; finally final_norm [hidden] and lm_head [hidden, vocab]. Projection
weights are column-major [in][out] (out contiguous), as the reference's gemv reads them.

Values are seeded: projections N(0, 1/in), norm weights 1 + N(0, 0.1^2), embeddings
N(0, 1), conv weights N(0, 0.5^2), dt_bias N(0, 0.1^2), A_log log U[1, 16].
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field

import numpy as np


@dataclass
class QminiConfig:
    vocab_size: int = 2048
    hidden_size: int = 512
    intermediate_size: int = 1536
    num_heads: int = 4
    num_kv_heads: int = 2
    head_dim: int = 128
    linear_num_key_heads: int = 4
    linear_num_value_heads: int = 8
    linear_key_head_dim: int = 128
    linear_value_head_dim: int = 128
    linear_conv_kernel_dim: int = 4
    max_seq_len: int = 512
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1.0e7
    layer_types: list = field(default_factory=lambda: [1, 1, 1, 0])  # Qwen3.5: three linear, one full

    @property
    def num_layers(self) -> int:
        return len(self.layer_types)


def write_qmini(path, cfg: QminiConfig, seed: int = 0) -> dict:
    """Writes the file and returns its tensors as fp16 numpy arrays: tok_embeddings,
    final_norm, lm_head and `layers` (one dict per layer, keyed like the reference's
    LayerWeights members)."""
    rng = np.random.default_rng(seed)
    out = {"layers": []}
    H, Hkv, d = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
    hid, inter, vocab = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size
    q_dim, kv_dim = H * d, Hkv * d
    key_dim = cfg.linear_num_key_heads * cfg.linear_key_head_dim
    val_dim = cfg.linear_num_value_heads * cfg.linear_value_head_dim
    conv_dim = 2 * key_dim + val_dim
    Hv = cfg.linear_num_value_heads

    with open(path, "wb") as f:
        def tensor(a, name=None, layer=None):
            a = np.ascontiguousarray(a, dtype=np.float16)
            flat = a.ravel()
            f.write(struct.pack("<Q", flat.size))
            f.write(flat.tobytes())
            if name is not None:
                (out if layer is None else layer)[name] = a

        def proj(n_in, n_out):
            return rng.standard_normal((n_in, n_out), dtype=np.float32) / np.sqrt(n_in)

        def norm(n):
            return 1.0 + 0.1 * rng.standard_normal(n, dtype=np.float32)

        f.write(b"QWENMINI")
        f.write(struct.pack("<i", 4))
        f.write(struct.pack("<13i", vocab, hid, inter, cfg.num_layers, H, Hkv, d, cfg.linear_num_key_heads,
                            cfg.linear_num_value_heads, cfg.linear_key_head_dim, cfg.linear_value_head_dim,
                            cfg.linear_conv_kernel_dim, cfg.max_seq_len))
        f.write(struct.pack("<2f", cfg.rms_norm_eps, cfg.rope_theta))
        f.write(struct.pack(f"<{cfg.num_layers}i", *cfg.layer_types))
        tensor(rng.standard_normal((vocab, hid), dtype=np.float32), "tok_embeddings")
        for kind in cfg.layer_types:
            lw = {"is_linear": kind}
            out["layers"].append(lw)
            tensor(norm(hid), "attn_norm", lw)
            if kind == 1:
                tensor(proj(hid, conv_dim), "linear_in_qkv", lw)
                tensor(proj(hid, val_dim), "linear_in_z", lw)
                tensor(proj(hid, Hv), "linear_in_b", lw)
                tensor(proj(hid, Hv), "linear_in_a", lw)
                tensor(0.5 * rng.standard_normal((conv_dim, cfg.linear_conv_kernel_dim), dtype=np.float32),
                       "linear_conv1d_w", lw)
                tensor(0.1 * rng.standard_normal(Hv, dtype=np.float32), "linear_dt_bias", lw)
                tensor(np.log(rng.uniform(1.0, 16.0, Hv)).astype(np.float32), "linear_a_log", lw)
                tensor(norm(cfg.linear_value_head_dim), "linear_norm_w", lw)
                tensor(proj(val_dim, hid), "linear_out_proj", lw)
            else:
                tensor(proj(hid, 2 * q_dim), "wq", lw)
                tensor(proj(hid, kv_dim), "wk", lw)
                tensor(proj(hid, kv_dim), "wv", lw)
                tensor(norm(d), "q_norm", lw)
                tensor(norm(d), "k_norm", lw)
                tensor(proj(q_dim, hid), "wo", lw)
            tensor(norm(hid), "ffn_norm", lw)
            tensor(proj(hid, inter), "w_gate", lw)
            tensor(proj(hid, inter), "w_up", lw)
            tensor(proj(inter, hid), "w_down", lw)
        tensor(norm(hid), "final_norm")
        tensor(proj(hid, vocab), "lm_head")
    return out
