"""GPU: split-KV decode attention (contiguous and paged) against the reference's own
flash/paged kernels (oracle/_ref) and the CPU oracle, within max-abs 2e-3 / rel 1e-2,
over the benchmark shapes and the edge cases (short, ragged and empty sequences,
page sizes, split counts, GQA groups, head dims, bad page entries)."""
import pytest
import torch

import qwenincuda_b200 as q
from conftest import allclose_report, assert_in_reference_envelope
from oracle.oracle import RefKernels

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-3, 1e-2


def _gen(seed):
    return torch.Generator(device="cuda").manual_seed(seed)


def _inputs(H, Hkv, d, S, P, dtype, seed, extra_pages=0):
    g = _gen(seed)
    npages = max(1, (S + P - 1) // P) + extra_pages
    tokens = npages * P
    qv = torch.randn(H * d, generator=g, device="cuda").to(dtype)
    kc = (torch.randn(tokens, Hkv * d, generator=g, device="cuda") * 0.5).to(dtype)
    vc = (torch.randn(tokens, Hkv * d, generator=g, device="cuda") * 0.5).to(dtype)
    table = torch.randperm(npages, generator=g, device="cuda").to(torch.int32)
    return qv, kc, vc, table


def _ours(qv, kc, vc, H, Hkv, d, S, table=None, P=16, splits=0, ws=True, gate=None):
    out = torch.full((H * d,), float("nan"), device="cuda", dtype=qv.dtype)
    w = q.Workspace(H, Hkv, d, max(S, 1)) if ws else None
    q.decode_attention(q=qv, k_cache=kc, v_cache=vc, out=out, num_heads=H, num_kv_heads=Hkv, head_dim=d, seq_len=S,
                       page_table=table, page_size=P, gate=gate, workspace=w, num_splits=splits)
    torch.cuda.synchronize()
    if w is not None:
        assert w.status() == 0
    return out


def _ref(qv, kc, vc, H, Hkv, d, S, table=None, P=16):
    ref = RefKernels(qv.dtype)
    out = torch.empty(H * d, device="cuda", dtype=qv.dtype)
    if table is None:
        ref.flash_attention(qv, kc, vc, H, Hkv, d, S, out)
    else:
        ref.paged_attention(qv, kc, vc, table, P, H, Hkv, d, S, out)
    return out


CASES = [
    # H, Hkv, d, S, P
    (16, 8, 128, 1025, 16),     # Qwen3-0.6B shape, S = 1024 cached + 1
    (32, 8, 128, 8192, 16),     # Qwen3-8B shape
    (16, 4, 256, 4097, 16),     # Qwen3.5 gated-attention shape (shorter S)
    (8, 8, 64, 100, 8),
    (64, 8, 128, 777, 32),      # group 8
    (8, 8, 128, 1, 16),
    (8, 8, 128, 2, 16),
    (16, 8, 128, 31, 16),
    (16, 8, 128, 32, 16),
    (16, 8, 128, 33, 16),
    (16, 8, 128, 129, 48),      # page size not a power of two (box height 16)
    (16, 8, 128, 300, 64),      # pages larger than a stage
    (4, 2, 256, 95, 24),        # box height 8
    (24, 8, 128, 1000, 16),     # group 3
    (40, 8, 128, 2000, 16),     # group 5
    (48, 8, 64, 700, 32),       # group 6, head_dim 64
    (28, 4, 256, 900, 16),      # group 7, head_dim 256
    (8, 1, 128, 3000, 16),      # one kv head, group 8
    (8, 1, 128, 40000, 16),     # one kv head, long: 208 splits, 26 clusters merged across
    (2, 2, 256, 17, 8),         # group 1, head_dim 256
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("H,Hkv,d,S,P", CASES)
@pytest.mark.parametrize("paged", [True, False])
def test_attention_vs_reference(dtype, H, Hkv, d, S, P, paged):
    qv, kc, vc, table = _inputs(H, Hkv, d, S, P, dtype, seed=S * 3 + d + H)
    tbl = table if paged else None
    want = _ref(qv, kc, vc, H, Hkv, d, S, tbl, P)
    got = _ours(qv, kc, vc, H, Hkv, d, S, tbl, P)
    ok, err, idx = allclose_report(got, want, ATOL, RTOL)
    if not ok:
        bad = (torch.isnan(got.float()) | ((got.float() - want.float()).abs() > ATOL + RTOL * want.float().abs()))
        where = bad.nonzero().flatten().tolist()
        again = _ours(qv, kc, vc, H, Hkv, d, S, tbl, P)
        ok2, err2, _ = allclose_report(again, want, ATOL, RTOL)
        pytest.fail(f"max abs err {err} at {idx}; {len(where)} bad, first {where[:6]} last {where[-6:]}; "
                    f"nan {int(torch.isnan(got.float()).sum())}; repeat ok={ok2} err={err2}")


@pytest.mark.parametrize("S", [1025, 5000])
def test_attention_vs_cpu_oracle(oracle, S):
    H, Hkv, d, P = 32, 8, 128, 16
    qv, kc, vc, table = _inputs(H, Hkv, d, S, P, torch.bfloat16, seed=S)
    got = _ours(qv, kc, vc, H, Hkv, d, S, table, P)
    want = oracle.attention(qv, kc, vc, H, Hkv, d, S, page_table=table, page_size=P)
    ok, err, idx = allclose_report(got, want, ATOL, RTOL)
    assert ok, f"max abs err {err} at {idx}"


@pytest.mark.parametrize("splits", [1, 2, 3, 7, 64, 0])
def test_split_counts_agree(splits):
    H, Hkv, d, S, P = 32, 8, 128, 2049, 16
    qv, kc, vc, table = _inputs(H, Hkv, d, S, P, torch.bfloat16, seed=17)
    want = _ref(qv, kc, vc, H, Hkv, d, S, table, P)
    got = _ours(qv, kc, vc, H, Hkv, d, S, table, P, splits=splits)
    ok, err, _ = allclose_report(got, want, ATOL, RTOL)
    assert ok, err


def test_no_workspace_runs_one_split():
    H, Hkv, d, S, P = 16, 8, 128, 600, 16
    qv, kc, vc, table = _inputs(H, Hkv, d, S, P, torch.bfloat16, seed=23)
    want = _ref(qv, kc, vc, H, Hkv, d, S, table, P)
    got = _ours(qv, kc, vc, H, Hkv, d, S, table, P, ws=False)
    ok, err, _ = allclose_report(got, want, ATOL, RTOL)
    assert ok, err


def test_empty_sequence_writes_zeros():
    H, Hkv, d = 16, 8, 128
    qv, kc, vc, _ = _inputs(H, Hkv, d, 16, 16, torch.bfloat16, seed=1)
    got = _ours(qv, kc, vc, H, Hkv, d, 0)
    assert torch.count_nonzero(got) == 0


def test_gate_epilogue():
    H, Hkv, d, S, P = 16, 4, 256, 3000, 16
    dtype = torch.bfloat16
    qv, kc, vc, table = _inputs(H, Hkv, d, S, P, dtype, seed=31)
    gate = torch.randn(H * d, generator=_gen(32), device="cuda").to(dtype)
    ref = RefKernels(dtype)
    want = _ref(qv, kc, vc, H, Hkv, d, S, table, P)
    ref.sigmoid_mul_inplace(want, gate, H * d)
    got = _ours(qv, kc, vc, H, Hkv, d, S, table, P, gate=gate)
    ok, err, _ = allclose_report(got, want, ATOL, RTOL)
    assert ok, err


def test_workspace_too_small_is_rejected():
    """Several clusters per kv head need global partial slots; a workspace sized for a
    short sequence is rejected before launch."""
    H, Hkv, d, S = 32, 8, 128, 4096
    qv, kc, vc, _ = _inputs(H, Hkv, d, S, 16, torch.bfloat16, seed=2)
    small = q.Workspace(H, Hkv, d, 64)
    out = torch.empty(H * d, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(q.QicError) as e:
        q.decode_attention(q=qv, k_cache=kc, v_cache=vc, out=out, num_heads=H, num_kv_heads=Hkv, head_dim=d,
                           seq_len=S, workspace=small, num_splits=64, cluster_size=16)
    assert e.value.status == 4


@pytest.mark.parametrize("splits,cluster", [(16, 16), (16, 8), (24, 12), (32, 8), (36, 12), (64, 16), (12, 1), (3, 3)])
def test_cluster_shapes_agree(splits, cluster):
    """Every split/cluster shape gives the reference result: DSMEM merge inside a
    cluster, release/acquire merge across clusters."""
    H, Hkv, d, S, P = 32, 8, 128, 4100, 16
    for dtype in (torch.bfloat16, torch.float16):
        qv, kc, vc, table = _inputs(H, Hkv, d, S, P, dtype, seed=splits * 7 + cluster)
        want = _ref(qv, kc, vc, H, Hkv, d, S, table, P)
        out = torch.full((H * d,), float("nan"), device="cuda", dtype=dtype)
        w = q.Workspace(H, Hkv, d, S)
        for _ in range(3):
            q.decode_attention(q=qv, k_cache=kc, v_cache=vc, out=out, num_heads=H, num_kv_heads=Hkv, head_dim=d,
                               seq_len=S, page_table=table, page_size=P, workspace=w, num_splits=splits,
                               cluster_size=cluster)
            torch.cuda.synchronize()
            assert w.status() == 0
            ok, err, idx = allclose_report(out, want, ATOL, RTOL)
            assert ok, f"{dtype}: max abs err {err} at {idx}"


def test_bad_page_entry_is_reported_not_faulted():
    """An out-of-range page-table entry is caught by the kernel's bounds check,
    clamped to page 0 and reported in the device status word."""
    H, Hkv, d, S, P = 16, 8, 128, 256, 16
    qv, kc, vc, table = _inputs(H, Hkv, d, S, P, torch.bfloat16, seed=3)
    table = table.clone()
    table[3] = 10 ** 6
    out = torch.empty(H * d, device="cuda", dtype=torch.bfloat16)
    w = q.Workspace(H, Hkv, d, S)
    q.decode_attention(q=qv, k_cache=kc, v_cache=vc, out=out, num_heads=H, num_kv_heads=Hkv, head_dim=d, seq_len=S,
                       page_table=table, page_size=P, workspace=w)
    torch.cuda.synchronize()
    assert w.status() & q.abi.QIC_DEV_BAD_PAGE
    assert w.status() == 0  # cleared by the read


def _reference_step(ref, inp, layer, paged):
    """The reference full-attention block body src/model.cpp:633-652 (without the
    projections): head-norm q and k, RoPE q and k, append, attention, gate."""
    cfg = inp.cfg
    H, Hkv, d, pos, P = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, cfg.position, cfg.page_size
    qv = inp.q[layer].flatten().clone()
    ref.head_rmsnorm(qv, inp.q_norm_w, H, d, cfg.eps, qv)
    ref.rope_inplace(qv, H, d, pos, cfg.rope_theta)
    kc = inp.k_cache[layer].view(-1, Hkv * d)
    vc = inp.v_cache[layer].view(-1, Hkv * d)
    table = inp.page_table[layer] if paged else None
    slot = int(table[pos // P]) * P + pos % P if paged else pos
    ref.append_chain(inp.k_new[layer].flatten(), inp.v_new[layer].flatten(), inp.k_norm_w, cfg.eps, cfg.rope_theta,
                     pos, kc, vc, Hkv, d, slot)
    out = torch.empty(H * d, device="cuda", dtype=qv.dtype)
    if paged:
        ref.paged_attention(qv, kc, vc, table, P, H, Hkv, d, cfg.seq_len, out)
    else:
        ref.flash_attention(qv, kc, vc, H, Hkv, d, cfg.seq_len, out)
    if inp.gate is not None:
        ref.sigmoid_mul_inplace(out, inp.gate[layer].flatten(), H * d)
    return out


# (H, Hkv, d, S, gate): the appended token alone in the last stage (S - 1 a multiple of
# 32 tokens, 16 at d=256), whose contribution comes from registers, and beside it
_FUSED_EXTRA = {"d64_s65": (8, 2, 64, 65, False), "d64_s70": (8, 2, 64, 70, False),
                "d128_s33": (16, 8, 128, 33, False), "d128_s2049": (32, 8, 128, 2049, False),
                "d256_s17": (16, 4, 256, 17, True), "d256_s18": (16, 4, 256, 18, True)}


@pytest.mark.parametrize("name", ["qwen3_0p6b_s1025", "qwen35_gated_s32769", "qwen3_8b_s8192", *_FUSED_EXTRA])
@pytest.mark.parametrize("paged", [True, False])
def test_fused_decode_step_matches_reference_chain(name, paged):
    from qwenincuda_b200.workloads import CONFIGS, AttnConfig, make_attention_inputs

    if name in _FUSED_EXTRA:
        H, Hkv, d, S, gate = _FUSED_EXTRA[name]
        cfg = AttnConfig(name, H, Hkv, d, S, gate=gate, seed=S)
    else:
        cfg = CONFIGS[name]
    dtype = torch.bfloat16
    mine = make_attention_inputs(cfg, paged=paged, layers=1, dtype=dtype)
    theirs = make_attention_inputs(cfg, paged=paged, layers=1, dtype=dtype)
    ref = RefKernels(dtype)
    P, pos, Hkv, d = cfg.page_size, cfg.position, cfg.num_kv_heads, cfg.head_dim
    slot = int(theirs.page_table[0][pos // P]) * P + pos % P if paged else pos
    k_rows = []
    for _ in range(16):  # the reference's appended k row over several runs
        extra = make_attention_inputs(cfg, paged=paged, layers=1, dtype=dtype)
        _reference_step(ref, extra, 0, paged)
        k_rows.append(extra.k_cache[0].view(-1, Hkv * d)[slot].clone())
        del extra
    want = _reference_step(ref, theirs, 0, paged)
    k_rows.append(theirs.k_cache[0].view(-1, Hkv * d)[slot].clone())
    w = q.Workspace(cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, cfg.seq_len)
    out = mine.out[0].flatten()
    q.decode_attention(q=mine.q[0], k_cache=mine.k_cache[0], v_cache=mine.v_cache[0], out=out,
                       num_heads=cfg.num_heads, num_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim,
                       seq_len=cfg.seq_len, page_table=mine.page_table[0] if paged else None,
                       page_size=cfg.page_size, gate=None if mine.gate is None else mine.gate[0],
                       q_norm_w=mine.q_norm_w, k_norm_w=mine.k_norm_w, k_new=mine.k_new[0], v_new=mine.v_new[0],
                       eps=cfg.eps, rope_theta=cfg.rope_theta, fuse_q=True, fuse_append=True, workspace=w)
    torch.cuda.synchronize()
    assert w.status() == 0
    # appended cache contents: the k row within the reference's envelope, everything else identical
    mk = mine.k_cache[0].view(-1, Hkv * d)
    assert_in_reference_envelope(mk[slot], k_rows)
    mk[slot] = theirs.k_cache[0].view(-1, Hkv * d)[slot]
    assert torch.equal(mine.k_cache.view(torch.int16), theirs.k_cache.view(torch.int16))
    assert torch.equal(mine.v_cache.view(torch.int16), theirs.v_cache.view(torch.int16))
    ok, err, idx = allclose_report(out, want, ATOL, RTOL)
    assert ok, f"max abs err {err} at {idx}"


def test_stage_pool_counters_reset_between_calls():
    """Long sequences take part of their stages from a per-kv-head ticket counter in
    the workspace; the last merger resets it. Calls of two shapes alternating on one
    workspace (several clusters per kv head, and one CTA per kv head) stay correct."""
    w = q.Workspace(32, 8, 128, 16385)
    shapes = [(32, 8, 128, 16385, 16, 0), (16, 4, 128, 5000, 16, 1), (32, 8, 128, 9001, 32, 16)]
    inputs = {}
    for H, Hkv, d, S, P, splits in shapes:
        qv, kc, vc, table = _inputs(H, Hkv, d, S, P, torch.bfloat16, seed=S)
        inputs[S] = (qv, kc, vc, table, _ref(qv, kc, vc, H, Hkv, d, S, table, P))
    for rep in range(3):
        for H, Hkv, d, S, P, splits in shapes:
            qv, kc, vc, table, want = inputs[S]
            out = torch.full((H * d,), float("nan"), device="cuda", dtype=torch.bfloat16)
            q.decode_attention(q=qv, k_cache=kc, v_cache=vc, out=out, num_heads=H, num_kv_heads=Hkv, head_dim=d,
                               seq_len=S, page_table=table, page_size=P, workspace=w, num_splits=splits)
            torch.cuda.synchronize()
            assert w.status() == 0
            ok, err, idx = allclose_report(out, want, ATOL, RTOL)
            assert ok, f"call {rep} S={S}: max abs err {err} at {idx}"
    # the ticket counters (the last 64 counters) are back at zero
    top = w.buf[256 + (8192 - 64) * 4: 256 + 8192 * 4].view(torch.int32)
    assert int(top.abs().sum()) == 0


def test_deterministic_flag_reproduces_bits():
    """With QIC_DETERMINISTIC two calls give the same bits; without it (stage pool on,
    33 stages per split here) every call stays within tolerance of the reference."""
    H, Hkv, d, S, P = 32, 8, 128, 40001, 16
    qv, kc, vc, table = _inputs(H, Hkv, d, S, P, torch.bfloat16, seed=51)
    want = _ref(qv, kc, vc, H, Hkv, d, S, table, P)
    w = q.Workspace(H, Hkv, d, S)
    outs = {}
    for det in (True, False):
        runs = []
        for _ in range(3):
            out = torch.empty(H * d, device="cuda", dtype=torch.bfloat16)
            q.decode_attention(q=qv, k_cache=kc, v_cache=vc, out=out, num_heads=H, num_kv_heads=Hkv, head_dim=d,
                               seq_len=S, page_table=table, page_size=P, workspace=w, deterministic=det)
            torch.cuda.synchronize()
            assert w.status() == 0
            ok, err, idx = allclose_report(out, want, ATOL, RTOL)
            assert ok, f"deterministic={det}: max abs err {err} at {idx}"
            runs.append(out)
        outs[det] = runs
    assert all(torch.equal(r.view(torch.int16), outs[True][0].view(torch.int16)) for r in outs[True])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("paged", [True, False])
def test_interleaved_q_gate_matches_reference_split(dtype, paged):
    """QIC_Q_GATE_INTERLEAVED reads q and the output gate straight from the packed
    [H, 2d] q/gate projection. The reference splits it with
    launch_split_q_gate_interleaved (src/kernels.cu:113-127), then head-norms and
    ropes q, attends and gates (src/model.cpp:628,633,636,644-650). The result is
    also bit-identical to this library's call on the split q and gate."""
    H, Hkv, d, S, P = 16, 4, 256, 4097, 16
    eps, theta = 1e-6, 1.0e7
    _, kc, vc, table = _inputs(H, Hkv, d, S, P, dtype, seed=61)
    table = table if paged else None
    g = _gen(62)
    packed = torch.randn(H * 2 * d, generator=g, device="cuda").to(dtype)
    qnw = (1.0 + 0.1 * torch.randn(d, generator=g, device="cuda")).to(dtype)
    ref = RefKernels(dtype)
    qq = torch.empty(H * d, device="cuda", dtype=dtype)
    gg = torch.empty(H * d, device="cuda", dtype=dtype)
    ref.split_q_gate(packed, H, d, qq, gg)
    assert torch.equal(qq.view(H, d), packed.view(H, 2, d)[:, 0])
    assert torch.equal(gg.view(H, d), packed.view(H, 2, d)[:, 1])
    q_raw = qq.clone()
    ref.head_rmsnorm(qq, qnw, H, d, eps, qq)
    ref.rope_inplace(qq, H, d, S - 1, theta)
    want = _ref(qq, kc, vc, H, Hkv, d, S, table, P)
    ref.sigmoid_mul_inplace(want, gg, H * d)
    w = q.Workspace(H, Hkv, d, S)
    outs = []
    for interleaved in (True, False):
        out = torch.full((H * d,), float("nan"), device="cuda", dtype=dtype)
        q.decode_attention(q=packed if interleaved else q_raw, gate=None if interleaved else gg, k_cache=kc,
                           v_cache=vc, out=out, num_heads=H, num_kv_heads=Hkv, head_dim=d, seq_len=S,
                           page_table=table, page_size=P, q_norm_w=qnw, eps=eps, rope_theta=theta, fuse_q=True,
                           workspace=w, deterministic=True, q_gate_interleaved=interleaved)
        torch.cuda.synchronize()
        assert w.status() == 0
        outs.append(out)
    ok, err, idx = allclose_report(outs[0], want, ATOL, RTOL)
    assert ok, f"max abs err {err} at {idx}"
    assert torch.equal(outs[0].view(torch.int16), outs[1].view(torch.int16))


def test_interleaved_q_gate_rejects_a_second_gate():
    H, Hkv, d, S = 8, 8, 128, 64
    qv, kc, vc, _ = _inputs(H, Hkv, d, S, 16, torch.bfloat16, seed=63)
    packed = torch.cat([qv.view(H, d), qv.view(H, d)], dim=1).flatten()
    out = torch.empty(H * d, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="INVALID_VALUE"):
        q.decode_attention(q=packed, gate=qv, k_cache=kc, v_cache=vc, out=out, num_heads=H, num_kv_heads=Hkv,
                           head_dim=d, seq_len=S, q_gate_interleaved=True)


def _dev_len_case(S_max, seed, dtype=torch.bfloat16):
    """Paged K/V for S_max tokens, raw q / k_new / v_new and norm weights."""
    H, Hkv, d, P = 32, 8, 128, 16
    qv, kc, vc, table = _inputs(H, Hkv, d, S_max, P, dtype, seed)
    g = _gen(seed + 1)
    kn = torch.randn(Hkv * d, generator=g, device="cuda").to(dtype)
    vn = (torch.randn(Hkv * d, generator=g, device="cuda") * 0.5).to(dtype)
    w = (1.0 + 0.1 * torch.randn(d, generator=g, device="cuda")).to(dtype)
    return (H, Hkv, d, P), dict(q=qv, k_cache=kc, v_cache=vc, page_table=table, page_size=P, q_norm_w=w, k_norm_w=w,
                                k_new=kn, v_new=vn, num_heads=H, num_kv_heads=Hkv, head_dim=d, fuse_q=True,
                                fuse_append=True, num_splits=16, cluster_size=8, deterministic=True)


@pytest.mark.parametrize("S", [1, 33, 1025, 4097])
def test_device_seq_len_matches_host_length(S):
    """QIC_DEVICE_SEQ_LEN: the length read from device memory by a launch sized for
    6000 tokens gives the same bytes (outputs and the appended rows) as the same
    launch shape with the length passed by value."""
    S_max = 6000
    (H, Hkv, d, P), kw = _dev_len_case(S_max, seed=71)
    kc0, vc0 = kw["k_cache"].clone(), kw["v_cache"].clone()
    outs, caches = [], []
    for dev in (False, True):
        kk = dict(kw, k_cache=kc0.clone(), v_cache=vc0.clone())
        out = torch.full((H * d,), float("nan"), device="cuda", dtype=torch.bfloat16)
        ws = q.Workspace(H, Hkv, d, S_max)
        if dev:
            q.decode_attention(out=out, seq_len=S_max, seq_len_dev=torch.tensor([S], dtype=torch.int32, device="cuda"),
                               workspace=ws, **kk)
        else:
            q.decode_attention(out=out, seq_len=S, workspace=ws, **kk)
        torch.cuda.synchronize()
        assert ws.status() == 0
        outs.append(out)
        caches.append((kk["k_cache"], kk["v_cache"]))
    assert torch.equal(outs[0].view(torch.int16), outs[1].view(torch.int16))
    for a, b in zip(caches[0], caches[1]):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    want = _ref(*_reference_q(kw, S), caches[0][0], caches[0][1], H, Hkv, d, S, kw["page_table"], P)
    ok, err, idx = allclose_report(outs[1], want, ATOL, RTOL)
    assert ok, f"max abs err {err} at {idx}"


def _reference_q(kw, S):
    """q after the reference's head-RMSNorm and RoPE at position S-1."""
    ref = RefKernels(kw["q"].dtype)
    qq = kw["q"].clone()
    ref.head_rmsnorm(qq, kw["q_norm_w"], kw["num_heads"], kw["head_dim"], 1e-6, qq)
    ref.rope_inplace(qq, kw["num_heads"], kw["head_dim"], S - 1, 1.0e6)
    return (qq,)


def test_device_seq_len_graph_replays_a_decode_loop():
    """One fused decode call captured once in a CUDA graph and replayed for four
    successive tokens (the length advanced in device memory and the token's q, k_new,
    v_new copied in before each replay) gives the same outputs and cache bytes as four
    calls with the length passed by value."""
    S0, S_max, steps = 1000, 1100, 4
    (H, Hkv, d, P), kw = _dev_len_case(S_max, seed=73)
    g = _gen(74)
    toks = [(torch.randn(H * d, generator=g, device="cuda").to(torch.bfloat16),
             torch.randn(Hkv * d, generator=g, device="cuda").to(torch.bfloat16),
             (torch.randn(Hkv * d, generator=g, device="cuda") * 0.5).to(torch.bfloat16)) for _ in range(steps)]
    kc0, vc0 = kw["k_cache"].clone(), kw["v_cache"].clone()
    # by value
    kc, vc = kc0.clone(), vc0.clone()
    ws = q.Workspace(H, Hkv, d, S_max)
    want = []
    for t, (qt, kt, vt) in enumerate(toks):
        out = torch.empty(H * d, device="cuda", dtype=torch.bfloat16)
        q.decode_attention(out=out, seq_len=S0 + t, workspace=ws, **dict(kw, q=qt, k_new=kt, v_new=vt, k_cache=kc,
                                                                          v_cache=vc))
        want.append(out)
    torch.cuda.synchronize()
    assert ws.status() == 0
    # one graph, replayed
    kg, vg = kc0.clone(), vc0.clone()
    qb, kb, vb = (torch.empty_like(x) for x in toks[0])
    length = torch.tensor([S0], dtype=torch.int32, device="cuda")
    out_g = torch.empty(H * d, device="cuda", dtype=torch.bfloat16)
    wsg = q.Workspace(H, Hkv, d, S_max)
    args = dict(kw, q=qb, k_new=kb, v_new=vb, k_cache=kg, v_cache=vg)
    # the first call on a device does per-device set-up: make it outside the capture,
    # on copies of the caches
    q.decode_attention(out=out_g, seq_len=S_max, seq_len_dev=length, workspace=wsg,
                       **dict(args, k_cache=kc0.clone(), v_cache=vc0.clone()))
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        q.decode_attention(out=out_g, seq_len=S_max, seq_len_dev=length, workspace=wsg, **args)
    got = []
    for t, (qt, kt, vt) in enumerate(toks):
        length.fill_(S0 + t)
        qb.copy_(qt)
        kb.copy_(kt)
        vb.copy_(vt)
        graph.replay()
        got.append(out_g.clone())
    torch.cuda.synchronize()
    assert wsg.status() == 0
    for t in range(steps):
        assert torch.equal(got[t].view(torch.int16), want[t].view(torch.int16)), f"token {t}"
    assert torch.equal(kg.view(torch.int16), kc.view(torch.int16))
    assert torch.equal(vg.view(torch.int16), vc.view(torch.int16))


def test_device_seq_len_out_of_range_is_clamped_and_reported():
    """A device length outside [1, seq_len] is clamped into it (every access stays
    inside the launch's bounds) and reported in the status word."""
    S_max = 300
    (H, Hkv, d, P), kw = _dev_len_case(S_max, seed=75)
    kw = dict(kw, fuse_append=False)
    ws = q.Workspace(H, Hkv, d, S_max)
    for bad in (0, -5, S_max + 7):
        out = torch.full((H * d,), float("nan"), device="cuda", dtype=torch.bfloat16)
        q.decode_attention(out=out, seq_len=S_max, seq_len_dev=torch.tensor([bad], dtype=torch.int32, device="cuda"),
                           workspace=ws, **kw)
        torch.cuda.synchronize()
        assert ws.status() & q.abi.QIC_DEV_BAD_LENGTH, bad
        assert torch.isfinite(out.float()).all(), bad
    assert ws.status() == 0
