"""GPU: the two partitioned benchmark configurations at their full size, against the
reference's own kernels (src/kernels.cu built for sm_100a, oracle/_ref).

* One 131,073-token sequence (Qwen3-8B attention shape: 32 q heads, 8 kv heads,
  d=128; page 16, shuffled table; 131,072 cached + the fused append at position
  131,072): qic_decode_attention with the fused q prologue and append against the
  reference chain head-norm q/k -> RoPE q/k -> two row copies -> paged_attention
  (src/model.cpp:633-649, src/kernels.cu:292-374); then the context-parallel kernel
  with one rank on the same cache.
* 64 sequences with seeded lengths U[512, 32768] + 1 drawn from one shuffled page
  pool of about 1.1M tokens (4.5 GB of K/V, so row offsets in bytes pass 2^31): one
  batched launch with the fused prologue and append, every sequence against its own
  reference launch_paged_attention call, and every cache row byte for byte.

Outputs within max-abs 2e-3 / rel 1e-2; appended V rows and every other row
byte-identical; the appended K rows inside the reference's own run-to-run envelope.
"""
import pytest
import torch

import qwenincuda_b200 as q
from conftest import allclose_report, assert_in_reference_envelope
from oracle.oracle import RefKernels
from qwenincuda_b200 import context_parallel as cpm
from qwenincuda_b200.workloads import CONFIGS, BatchConfig, make_attention_inputs, make_batched_inputs

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-3, 1e-2


def _reference_q(ref, qraw, w, H, d, eps, pos, theta):
    qq = qraw.flatten().clone()
    ref.head_rmsnorm(qq, w, H, d, eps, qq)
    ref.rope_inplace(qq, H, d, pos, theta)
    return qq


def test_long_sequence_131073_vs_reference():
    cfg = CONFIGS["qwen3_8b_s131073"]
    H, Hkv, d, S, P, pos = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, cfg.seq_len, cfg.page_size, cfg.position
    mine = make_attention_inputs(cfg, paged=True, layers=1)
    theirs = make_attention_inputs(cfg, paged=True, layers=1)
    table = mine.page_table[0]
    ws = q.Workspace(H, Hkv, d, S)
    out = torch.full((H * d,), float("nan"), device="cuda", dtype=torch.bfloat16)
    q.decode_attention(q=mine.q[0], k_cache=mine.k_cache[0], v_cache=mine.v_cache[0], out=out, num_heads=H,
                       num_kv_heads=Hkv, head_dim=d, seq_len=S, page_table=table, page_size=P,
                       q_norm_w=mine.q_norm_w, k_norm_w=mine.k_norm_w, k_new=mine.k_new[0], v_new=mine.v_new[0],
                       eps=cfg.eps, rope_theta=cfg.rope_theta, fuse_q=True, fuse_append=True, workspace=ws)
    torch.cuda.synchronize()
    assert ws.status() == 0

    ref = RefKernels(torch.bfloat16)
    kc = theirs.k_cache[0].view(-1, Hkv * d)
    vc = theirs.v_cache[0].view(-1, Hkv * d)
    mk = mine.k_cache[0].view(-1, Hkv * d)
    slot = int(table[pos // P]) * P + pos % P
    rows = []
    for _ in range(16):  # the reference's appended k row over several runs
        ref.append_chain(theirs.k_new[0].flatten(), theirs.v_new[0].flatten(), theirs.k_norm_w, cfg.eps,
                         cfg.rope_theta, pos, kc, vc, Hkv, d, slot)
        rows.append(kc[slot].clone())
    assert_in_reference_envelope(mk[slot], rows)
    mk[slot] = kc[slot]  # from here both caches hold the same bytes
    assert torch.equal(mine.k_cache.view(torch.int16), theirs.k_cache.view(torch.int16))
    assert torch.equal(mine.v_cache.view(torch.int16), theirs.v_cache.view(torch.int16))
    qq = _reference_q(ref, theirs.q[0], theirs.q_norm_w, H, d, cfg.eps, pos, cfg.rope_theta)
    want = torch.empty(H * d, device="cuda", dtype=torch.bfloat16)
    ref.paged_attention(qq, kc, vc, table, P, H, Hkv, d, S, want)
    ok, err, idx = allclose_report(out, want, ATOL, RTOL)
    assert ok, f"single-GPU call: max abs err {err} at {idx}"

    # the context-parallel kernel, one rank, on the same (appended) cache
    group = cpm.ExchangeGroup(H, Hkv, d, rank=0, world=1, gather=lambda b, r, n: [b])
    try:
        out_cp = torch.full_like(out, float("nan"))
        cpm.cp_decode_attention(group, q=mine.q[0], k_cache=mine.k_cache[0], v_cache=mine.v_cache[0], out=out_cp,
                                num_heads=H, num_kv_heads=Hkv, head_dim=d, seq_len=S, page_table=table, page_size=P,
                                q_norm_w=mine.q_norm_w, eps=cfg.eps, rope_theta=cfg.rope_theta, fuse_q=True,
                                workspace=ws, position=pos)
        torch.cuda.synchronize()
        assert ws.status() == 0
        ok, err, idx = allclose_report(out_cp, want, ATOL, RTOL)
        assert ok, f"context-parallel call: max abs err {err} at {idx}"
    finally:
        torch.cuda.synchronize()
        group.close()


def test_batch64_pool_1p1m_vs_reference():
    cfg = BatchConfig()
    lens = cfg.seq_lens()
    assert len(lens) == 64 and min(lens) >= 513 and max(lens) <= 32769
    H, Hkv, d, P = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, cfg.page_size
    mine = make_batched_inputs(cfg, seq_lens=lens)
    assert mine["cache_tokens"] >= 1_100_000
    assert mine["cache_tokens"] * Hkv * d * 2 > 2 ** 31  # byte offsets beyond 32 bits
    plan = q.BatchPlan(lens, H, Hkv, d)
    q.batch_decode_attention(plan=plan, q=mine["q"], k_cache=mine["k_cache"], v_cache=mine["v_cache"],
                             block_tables=mine["block_tables"], out=mine["out"], num_heads=H, num_kv_heads=Hkv,
                             head_dim=d, page_size=P, q_norm_w=mine["q_norm_w"], k_norm_w=mine["k_norm_w"],
                             k_new=mine["k_new"], v_new=mine["v_new"], fuse_q=True, fuse_append=True)
    torch.cuda.synchronize()
    assert plan.status() == 0
    # the sequences' pages are the highest rows of the pool in some tables
    assert int(mine["block_tables"].max()) * P + P > 2 ** 20

    theirs = make_batched_inputs(cfg, seq_lens=lens)
    ref = RefKernels(torch.bfloat16)
    kc = theirs["k_cache"].view(-1, Hkv * d)
    vc = theirs["v_cache"].view(-1, Hkv * d)
    mk = mine["k_cache"].view(-1, Hkv * d)
    for b, S in enumerate(lens):
        pos = S - 1
        slot = int(theirs["block_tables"][b][pos // P]) * P + pos % P
        rows = []
        for _ in range(8):
            ref.append_chain(theirs["k_new"][b].flatten(), theirs["v_new"][b].flatten(), theirs["k_norm_w"], cfg.eps,
                             cfg.rope_theta, pos, kc, vc, Hkv, d, slot)
            rows.append(kc[slot].clone())
        assert_in_reference_envelope(mk[slot], rows)
        mk[slot] = kc[slot]
    assert torch.equal(mine["k_cache"].view(torch.int16), theirs["k_cache"].view(torch.int16))
    assert torch.equal(mine["v_cache"].view(torch.int16), theirs["v_cache"].view(torch.int16))
    want = torch.empty(H * d, device="cuda", dtype=torch.bfloat16)
    for b, S in enumerate(lens):
        qq = _reference_q(ref, theirs["q"][b], theirs["q_norm_w"], H, d, cfg.eps, S - 1, cfg.rope_theta)
        ref.paged_attention(qq, kc, vc, theirs["block_tables"][b], P, H, Hkv, d, S, want)
        ok, err, idx = allclose_report(mine["out"][b], want, ATOL, RTOL)
        assert ok, f"sequence {b} (S={S}): max abs err {err} at {idx}"
