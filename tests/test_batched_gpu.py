"""GPU: batched paged decode over one shared page pool, checked per sequence against
the reference's own paged_attention kernel (one launch per sequence with its own
block-table row) and the CPU oracle; the fused append writes every sequence's slot
byte-identically to the reference chain."""
import pytest
import torch

import qwenincuda_b200 as q
from conftest import allclose_report, assert_in_reference_envelope
from oracle.oracle import RefKernels
from qwenincuda_b200.workloads import BatchConfig, make_batched_inputs

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-3, 1e-2


def _small_cfg(**kw):
    base = dict(batch=6, min_len=1, max_len=3000, pool_tokens=40_000, seed=11)
    base.update(kw)
    return BatchConfig(**base)


@pytest.mark.parametrize("target_ctas", [0, 7, 64])
def test_batched_vs_reference_per_sequence(target_ctas):
    cfg = _small_cfg()
    lens = [1, 2, 33, 777, 2049, 3001]
    inp = make_batched_inputs(cfg, seq_lens=lens)
    plan = q.BatchPlan(lens, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, target_ctas=target_ctas)
    q.batch_decode_attention(plan=plan, q=inp["q"], k_cache=inp["k_cache"], v_cache=inp["v_cache"],
                             block_tables=inp["block_tables"], out=inp["out"], num_heads=cfg.num_heads,
                             num_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim, page_size=cfg.page_size)
    torch.cuda.synchronize()
    assert plan.status() == 0
    ref = RefKernels(torch.bfloat16)
    kc = inp["k_cache"].view(-1, cfg.kv_dim)
    vc = inp["v_cache"].view(-1, cfg.kv_dim)
    for b, S in enumerate(lens):
        want = torch.empty(cfg.num_heads * cfg.head_dim, device="cuda", dtype=torch.bfloat16)
        ref.paged_attention(inp["q"][b].flatten(), kc, vc, inp["block_tables"][b], cfg.page_size, cfg.num_heads,
                            cfg.num_kv_heads, cfg.head_dim, S, want)
        ok, err, idx = allclose_report(inp["out"][b], want, ATOL, RTOL)
        assert ok, f"sequence {b} (S={S}): max err {err} at {idx}"


def test_batched_fused_append_and_oracle(oracle):
    cfg = _small_cfg(seed=12)
    lens = [5, 400, 1500, 16, 17, 2500]
    mine = make_batched_inputs(cfg, seq_lens=lens)
    theirs = make_batched_inputs(cfg, seq_lens=lens)
    plan = q.BatchPlan(lens, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim)
    q.batch_decode_attention(plan=plan, q=mine["q"], k_cache=mine["k_cache"], v_cache=mine["v_cache"],
                             block_tables=mine["block_tables"], out=mine["out"], num_heads=cfg.num_heads,
                             num_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim, page_size=cfg.page_size,
                             q_norm_w=mine["q_norm_w"], k_norm_w=mine["k_norm_w"], k_new=mine["k_new"],
                             v_new=mine["v_new"], fuse_q=True, fuse_append=True, pdl=True)
    torch.cuda.synchronize()
    assert plan.status() == 0
    ref = RefKernels(torch.bfloat16)
    H, Hkv, d, P = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, cfg.page_size
    kc = theirs["k_cache"].view(-1, Hkv * d)
    vc = theirs["v_cache"].view(-1, Hkv * d)
    mk = mine["k_cache"].view(-1, Hkv * d)
    qs = []
    for b, S in enumerate(lens):
        pos = S - 1
        slot = int(theirs["block_tables"][b][pos // P]) * P + pos % P
        rows = []
        for _ in range(16):  # the reference's appended k row over several runs
            ref.append_chain(theirs["k_new"][b].flatten(), theirs["v_new"][b].flatten(), theirs["k_norm_w"], cfg.eps,
                             cfg.rope_theta, pos, kc, vc, Hkv, d, slot)
            rows.append(kc[slot].clone())
        assert_in_reference_envelope(mk[slot], rows)
        mk[slot] = kc[slot]
        qq = theirs["q"][b].flatten().clone()
        ref.head_rmsnorm(qq, theirs["q_norm_w"], H, d, cfg.eps, qq)
        ref.rope_inplace(qq, H, d, pos, cfg.rope_theta)
        qs.append(qq)
    assert torch.equal(mine["k_cache"].view(torch.int16), theirs["k_cache"].view(torch.int16))
    assert torch.equal(mine["v_cache"].view(torch.int16), theirs["v_cache"].view(torch.int16))
    want = oracle.batched_attention(torch.stack(qs), kc, vc, theirs["block_tables"],
                                    torch.tensor(lens, dtype=torch.int32), P, H, Hkv, d)
    ok, err, idx = allclose_report(mine["out"].view(len(lens), -1), want, ATOL, RTOL)
    assert ok, f"max err {err} at {idx}"


def test_pdl_chain_matches_plain_launches():
    """Back-to-back calls with programmatic dependent launch give the same bytes as
    plain launches (the second call reads the first call's output as its q). Both use
    the same split shape: by default chained launches leave a sixth of the resident
    slots free and so split differently."""
    from qwenincuda_b200.workloads import AttnConfig, make_attention_inputs

    cfg = AttnConfig("pdl", 32, 8, 128, 3000, layers=4, seed=9)
    outs = []
    for pdl in (False, True):
        inp = make_attention_inputs(cfg, paged=True)
        ws = q.Workspace(32, 8, 128, cfg.seq_len)
        for layer in range(cfg.layers):
            # chain: layer l's q is layer l-1's output, written by the previous kernel
            qin = inp.q[layer] if layer == 0 else inp.out[layer - 1]
            q.decode_attention(q=qin, k_cache=inp.k_cache[layer], v_cache=inp.v_cache[layer], out=inp.out[layer],
                               num_heads=32, num_kv_heads=8, head_dim=128, seq_len=cfg.seq_len,
                               page_table=inp.page_table[layer], page_size=16, q_norm_w=inp.q_norm_w,
                               k_norm_w=inp.k_norm_w, k_new=inp.k_new[layer], v_new=inp.v_new[layer], fuse_q=True,
                               fuse_append=True, workspace=ws, pdl=pdl, num_splits=40, cluster_size=8)
        torch.cuda.synchronize()
        assert ws.status() == 0
        outs.append((inp.out.clone(), inp.k_cache.clone()))
    assert torch.equal(outs[0][1].view(torch.int16), outs[1][1].view(torch.int16))
    assert torch.equal(outs[0][0].view(torch.int16), outs[1][0].view(torch.int16))


def test_batched_interleaved_q_gate_matches_split():
    """Batched calls with the [B, H, 2d] interleaved q/gate projection give the same
    bytes as calls on the split q [B, H, d] and gate [B, H, d]."""
    cfg = _small_cfg(seed=13)
    lens = [3, 900, 2100, 64]
    H, d = cfg.num_heads, cfg.head_dim
    outs = []
    for interleaved in (True, False):
        inp = make_batched_inputs(cfg, seq_lens=lens)
        g = torch.Generator(device="cuda").manual_seed(14)
        gate = torch.randn(len(lens), H, d, generator=g, device="cuda").to(inp["q"].dtype)
        qraw = inp["q"].view(len(lens), H, d)
        packed = torch.cat([qraw, gate], dim=2).contiguous()
        plan = q.BatchPlan(lens, H, cfg.num_kv_heads, d)
        q.batch_decode_attention(plan=plan, q=packed if interleaved else qraw, gate=None if interleaved else gate,
                                 k_cache=inp["k_cache"], v_cache=inp["v_cache"], block_tables=inp["block_tables"],
                                 out=inp["out"], num_heads=H, num_kv_heads=cfg.num_kv_heads, head_dim=d,
                                 page_size=cfg.page_size, q_norm_w=inp["q_norm_w"], k_norm_w=inp["k_norm_w"],
                                 k_new=inp["k_new"], v_new=inp["v_new"], fuse_q=True, fuse_append=True,
                                 q_gate_interleaved=interleaved)
        torch.cuda.synchronize()
        assert plan.status() == 0
        outs.append((inp["out"].clone(), inp["k_cache"].clone()))
    assert torch.equal(outs[0][1].view(torch.int16), outs[1][1].view(torch.int16))
    assert torch.equal(outs[0][0].view(torch.int16), outs[1][0].view(torch.int16))


def test_batched_odd_group_vs_reference():
    """Group 3 at head_dim 64: every sequence against the reference's paged kernel."""
    cfg = _small_cfg(num_heads=24, num_kv_heads=8, head_dim=64, seed=15)
    lens = [5, 300, 1000, 64]
    inp = make_batched_inputs(cfg, seq_lens=lens)
    plan = q.BatchPlan(lens, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim)
    q.batch_decode_attention(plan=plan, q=inp["q"], k_cache=inp["k_cache"], v_cache=inp["v_cache"],
                             block_tables=inp["block_tables"], out=inp["out"], num_heads=cfg.num_heads,
                             num_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim, page_size=cfg.page_size)
    torch.cuda.synchronize()
    assert plan.status() == 0
    ref = RefKernels(torch.bfloat16)
    kc = inp["k_cache"].view(-1, cfg.kv_dim)
    vc = inp["v_cache"].view(-1, cfg.kv_dim)
    for b, S in enumerate(lens):
        want = torch.empty(cfg.num_heads * cfg.head_dim, device="cuda", dtype=torch.bfloat16)
        ref.paged_attention(inp["q"][b].flatten(), kc, vc, inp["block_tables"][b], cfg.page_size, cfg.num_heads,
                            cfg.num_kv_heads, cfg.head_dim, S, want)
        ok, err, idx = allclose_report(inp["out"][b], want, ATOL, RTOL)
        assert ok, f"sequence {b} (S={S}): max err {err} at {idx}"
