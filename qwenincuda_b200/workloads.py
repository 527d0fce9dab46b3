"""Seeded synthetic decode workloads with the shapes of the path's benchmark configs.

There is no model checkpoint here: K/V caches, projections and norm weights are
random tensors drawn from fixed seeds (torch generators), with the shapes and value
distributions of the configurations below.

  qwen3_0p6b_s1025   16 q heads, 8 kv heads, d=128, 1024 cached + append at 1024
                     (S=1025); K/V ~ N(0,1)*0.5; q/k head-RMSNormed (weight 1) then
                     RoPE theta=1e6; page 16, table = seeded permutation of 65 pages;
                     32 layers, each with its own cache (the model has 28; 32 make a
                     step's 134 MB of K/V larger than L2)
  qwen3_8b_s8192     36 layers, 32 q heads, 8 kv heads, d=128; stacked cache
                     [36, 8192, 8*128] ~ N(0, 0.5^2); append at 8191, S=8192;
                     contiguous and paged (page 16, shuffled table per layer)
  qwen35_gdn         GatedDeltaNet Hk=16, Hv=32, dk=dv=128, conv_dim=8192, K=4;
                     state ~ N(0, 0.02^2), a,b ~ N(0,1), A_log = log U[1,16],
                     dt_bias ~ N(0, 0.1^2)
  qwen35_gated_s32769  16 q heads, 4 kv heads, d=256, 32768 cached + append at
                     32768 (S=32769), q_gate ~ N(0,1); 8 layers, each with its own
                     cache: the gated-attention layers of a 32-layer hybrid stack
                     with one full-attention layer in four (the reference takes the
                     layer kinds from the model config, src/model.cpp:368-389)
  qwen3_8b_s131073   32/8 heads, d=128, 131072 cached + append (S=131073), page 16,
                     shuffled table
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch


@dataclass
class AttnConfig:
    name: str
    num_heads: int
    num_kv_heads: int
    head_dim: int
    seq_len: int              # S = position + 1 (the appended token is the last one)
    layers: int = 1
    page_size: int = 16
    gate: bool = False
    kv_std: float = 0.5
    rope_theta: float = 1.0e6
    eps: float = 1e-6
    seed: int = 0

    @property
    def position(self) -> int:
        return self.seq_len - 1

    @property
    def kv_dim(self) -> int:
        return self.num_kv_heads * self.head_dim

    @property
    def group(self) -> int:
        return self.num_heads // self.num_kv_heads

    def kv_read_bytes(self) -> int:
        """Algorithmic K+V bytes one layer reads (S tokens, 16-bit)."""
        return 2 * self.seq_len * self.kv_dim * 2

    def append_bytes(self) -> int:
        return 2 * self.kv_dim * 2


CONFIGS = {
    "qwen3_0p6b_s1025": AttnConfig("qwen3_0p6b_s1025", 16, 8, 128, 1025, layers=32, kv_std=0.5, seed=1),
    "qwen3_8b_s8192": AttnConfig("qwen3_8b_s8192", 32, 8, 128, 8192, layers=36, seed=2),
    "qwen35_gated_s32769": AttnConfig("qwen35_gated_s32769", 16, 4, 256, 32769, layers=8, gate=True, seed=3),
    "qwen3_8b_s131073": AttnConfig("qwen3_8b_s131073", 32, 8, 128, 131073, seed=4),
}


@dataclass
class AttnInputs:
    cfg: AttnConfig
    paged: bool
    q: torch.Tensor            # [L, H, d] raw q projections (normed + roped in the fused prologue)
    k_new: torch.Tensor        # [L, Hkv, d] raw k projections of the new token
    v_new: torch.Tensor        # [L, Hkv, d]
    q_norm_w: torch.Tensor     # [d]
    k_norm_w: torch.Tensor     # [d]
    k_cache: torch.Tensor      # [L, cache_tokens, Hkv, d]
    v_cache: torch.Tensor
    page_table: torch.Tensor | None  # [L, pages] int32
    gate: torch.Tensor | None  # [L, H, d]
    out: torch.Tensor          # [L, H, d]
    cache_tokens: int = 0
    extra: dict = field(default_factory=dict)


def make_attention_inputs(cfg: AttnConfig, *, paged: bool, device="cuda", dtype=torch.bfloat16,
                          layers: int | None = None) -> AttnInputs:
    L = cfg.layers if layers is None else layers
    g = torch.Generator(device=device)
    g.manual_seed(cfg.seed * 1000 + (1 if paged else 0))
    P = cfg.page_size
    npages = (cfg.seq_len + P - 1) // P
    cache_tokens = npages * P if paged else cfg.seq_len
    H, Hkv, d = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim

    def randn(*shape, std=1.0):
        return (torch.randn(*shape, generator=g, device=device, dtype=torch.float32) * std).to(dtype)

    k_cache = randn(L, cache_tokens, Hkv, d, std=cfg.kv_std)
    v_cache = randn(L, cache_tokens, Hkv, d, std=cfg.kv_std)
    q = randn(L, H, d)
    k_new = randn(L, Hkv, d)
    v_new = randn(L, Hkv, d, std=cfg.kv_std)
    ones = torch.ones(d, device=device, dtype=dtype)
    page_table = None
    if paged:
        perms = [torch.randperm(npages, generator=g, device=device) for _ in range(L)]
        page_table = torch.stack(perms).to(torch.int32).contiguous()
    gate = randn(L, H, d) if cfg.gate else None
    out = torch.zeros(L, H, d, device=device, dtype=dtype)
    return AttnInputs(cfg, paged, q, k_new, v_new, ones, ones.clone(), k_cache, v_cache, page_table, gate, out,
                      cache_tokens)


@dataclass
class GdnConfig:
    name: str = "qwen35_gdn"
    num_k_heads: int = 16
    num_v_heads: int = 32
    k_head_dim: int = 128
    v_head_dim: int = 128
    conv_kernel: int = 4
    eps: float = 1e-6
    seed: int = 5

    @property
    def conv_dim(self) -> int:
        return 2 * self.num_k_heads * self.k_head_dim + self.num_v_heads * self.v_head_dim

    def state_bytes(self) -> int:
        """Algorithmic bytes of one step: fp32 recurrent + conv state read and written, plus inputs/output."""
        rs = self.num_v_heads * self.k_head_dim * self.v_head_dim * 4 * 2
        cs = self.conv_dim * self.conv_kernel * 4 * 2
        ins = (self.conv_dim + 2 * self.num_v_heads * self.v_head_dim + self.conv_dim * self.conv_kernel
               + 4 * self.num_v_heads + self.v_head_dim) * 2
        return rs + cs + ins


def make_gdn_inputs(cfg: GdnConfig, device="cuda", dtype=torch.bfloat16) -> dict:
    g = torch.Generator(device=device)
    g.manual_seed(cfg.seed)
    Hv, dk, dv = cfg.num_v_heads, cfg.k_head_dim, cfg.v_head_dim

    def randn(*shape, std=1.0, dt=dtype):
        return (torch.randn(*shape, generator=g, device=device, dtype=torch.float32) * std).to(dt)

    a_log = torch.log(torch.rand(Hv, generator=g, device=device) * 15.0 + 1.0).to(dtype)
    return dict(
        qkv=randn(cfg.conv_dim),
        z=randn(Hv * dv),
        b=randn(Hv),
        a=randn(Hv),
        conv_w=randn(cfg.conv_dim, cfg.conv_kernel, std=0.5),
        dt_bias=randn(Hv, std=0.1),
        a_log=a_log,
        norm_w=(1.0 + randn(dv, std=0.1, dt=torch.float32)).to(dtype),
        conv_state=randn(cfg.conv_dim, cfg.conv_kernel, dt=torch.float32),
        recurrent_state=randn(Hv, dk, dv, std=0.02, dt=torch.float32),
        out=torch.zeros(Hv * dv, device=device, dtype=dtype),
    )


@dataclass
class BatchConfig:
    """Batched paged decode: `batch` sequences with seeded cached lengths in
    [min_len, max_len], one token appended per sequence (S_b = cached_b + 1), pages of
    `page_size` tokens drawn from one shuffled pool of about `pool_tokens` tokens."""

    name: str = "qwen3_8b_batch64"
    batch: int = 64
    num_heads: int = 32
    num_kv_heads: int = 8
    head_dim: int = 128
    min_len: int = 512
    max_len: int = 32768
    page_size: int = 16
    pool_tokens: int = 1_100_000
    kv_std: float = 0.5
    rope_theta: float = 1.0e6
    eps: float = 1e-6
    seed: int = 6

    def seq_lens(self) -> list[int]:
        g = torch.Generator().manual_seed(self.seed)
        cached = torch.randint(self.min_len, self.max_len + 1, (self.batch,), generator=g)
        return [int(c) + 1 for c in cached]

    @property
    def kv_dim(self) -> int:
        return self.num_kv_heads * self.head_dim


def batched_bytes(seq_lens, kv_dim: int) -> int:
    """Algorithmic bytes of one batched step: K+V read for every attended token plus the appends."""
    return sum(2 * s * kv_dim * 2 for s in seq_lens) + len(seq_lens) * 2 * kv_dim * 2


def make_batched_inputs(cfg: BatchConfig, *, device="cuda", dtype=torch.bfloat16, seq_lens=None) -> dict:
    lens = seq_lens if seq_lens is not None else cfg.seq_lens()
    P = cfg.page_size
    pages_per = [(s + P - 1) // P for s in lens]
    need = sum(pages_per)
    pool_pages = max((cfg.pool_tokens + P - 1) // P, need)
    gen = torch.Generator().manual_seed(cfg.seed + 1)
    perm = torch.randperm(pool_pages, generator=gen)
    max_pages = max(pages_per)
    tables = torch.zeros(len(lens), max_pages, dtype=torch.int32)
    at = 0
    for b, n in enumerate(pages_per):
        tables[b, :n] = perm[at:at + n].to(torch.int32)
        at += n
    g = torch.Generator(device=device)
    g.manual_seed(cfg.seed)
    H, Hkv, d = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim

    def randn(*shape, std=1.0):
        return (torch.randn(*shape, generator=g, device=device, dtype=torch.float32) * std).to(dtype)

    cache_tokens = pool_pages * P
    B = len(lens)
    return dict(
        seq_lens=lens,
        block_tables=tables.to(device),
        k_cache=randn(cache_tokens, Hkv, d, std=cfg.kv_std),
        v_cache=randn(cache_tokens, Hkv, d, std=cfg.kv_std),
        q=randn(B, H, d),
        k_new=randn(B, Hkv, d),
        v_new=randn(B, Hkv, d, std=cfg.kv_std),
        q_norm_w=torch.ones(d, device=device, dtype=dtype),
        k_norm_w=torch.ones(d, device=device, dtype=dtype),
        out=torch.zeros(B, H, d, device=device, dtype=dtype),
        cache_tokens=cache_tokens,
    )
