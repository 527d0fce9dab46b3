"""GPU (one device): context parallelism pieces that need no second GPU.

* Shard partials (QIC_PARTIAL_OUT with QIC_EXPLICIT_POSITION) of 2-4 token ranges of
  one sequence, merged by qic_attention_merge, equal the whole-sequence call (q
  prologue at the global position, append on the shard holding the last token)
  within max-abs 2e-3 / rel 1e-2, and the appended rows are byte-identical.
* The fused exchange with one rank equals the plain call bit for bit, call after call
  (epoch and parity bookkeeping).
* Failure detection: a peer that never publishes (no exchange word ever carries the
  call's tag) makes the bounded wait give up; the kernel records QIC_DEV_PEER_TIMEOUT, leaves the output
  untouched and the context stays usable.
"""
import ctypes

import pytest
import torch

import qwenincuda_b200 as q
from conftest import allclose_report
from qwenincuda_b200 import context_parallel as cpm

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-3, 1e-2
H, HKV, D, P = 32, 8, 128, 16


def _sequence(S, seed, dtype=torch.bfloat16):
    """Logical K/V rows of one sequence (token order), raw q / k_new / v_new, weights."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    k = (torch.randn(S, HKV * D, generator=g, device="cuda") * 0.5).to(dtype)
    v = (torch.randn(S, HKV * D, generator=g, device="cuda") * 0.5).to(dtype)
    qv = torch.randn(H * D, generator=g, device="cuda").to(dtype)
    kn = torch.randn(HKV * D, generator=g, device="cuda").to(dtype)
    vn = (torch.randn(HKV * D, generator=g, device="cuda") * 0.5).to(dtype)
    w = (1.0 + 0.1 * torch.randn(D, generator=g, device="cuda")).to(dtype)
    return k, v, qv, kn, vn, w


def _paged(rows, seed):
    """Rows scattered into a shuffled page pool; returns (k_pool, table)."""
    n = rows.shape[0]
    pages = (n + P - 1) // P
    g = torch.Generator(device="cuda").manual_seed(seed)
    perm = torch.randperm(pages, generator=g, device="cuda")
    pool = torch.zeros(pages * P, rows.shape[1], device="cuda", dtype=rows.dtype)
    for lp in range(pages):
        t0, t1 = lp * P, min((lp + 1) * P, n)
        pp = int(perm[lp])
        pool[pp * P:pp * P + (t1 - t0)] = rows[t0:t1]
    return pool, perm.to(torch.int32)


def _kw(S, qv, kc, vc, table, w, kn, vn, append, ws, **extra):
    return dict(q=qv, k_cache=kc, v_cache=vc, num_heads=H, num_kv_heads=HKV, head_dim=D, seq_len=S,
                page_table=table, page_size=P, q_norm_w=w, k_norm_w=w, k_new=kn, v_new=vn, fuse_q=True,
                fuse_append=append, workspace=ws, **extra)


@pytest.mark.parametrize("world", [2, 3, 4])
def test_shard_partials_merge_to_whole_sequence(world):
    S = 4099  # the appended token is position 4098, on the last (partial) page
    k, v, qv, kn, vn, w = _sequence(S, seed=100 + world)
    # whole sequence, one call
    kc_full, tab_full = _paged(k, seed=1)
    vc_full, _ = _paged(v, seed=1)
    out_full = torch.empty(H * D, device="cuda", dtype=qv.dtype)
    ws = q.Workspace(H, HKV, D, S)
    q.decode_attention(out=out_full, **_kw(S, qv, kc_full, vc_full, tab_full, w, kn, vn, True, ws))
    torch.cuda.synchronize()
    assert ws.status() == 0
    # shards: partials, then the merge
    pf = q.ops.partial_floats(H, HKV, D)
    parts = torch.full((world, HKV * pf), float("nan"), device="cuda", dtype=torch.float32)
    shards = cpm.shard_tokens(S, P, world)
    owner_row = None
    for r, (t0, t1) in enumerate(shards):
        n = t1 - t0
        kc, tab = _paged(k[t0:t1], seed=10 + r)
        vc, _ = _paged(v[t0:t1], seed=10 + r)
        last = r == world - 1
        wsr = q.Workspace(H, HKV, D, n)
        q.decode_attention(out=parts[r], **_kw(n, qv, kc, vc, tab, w, kn, vn, last, wsr, position=S - 1,
                                               partial_out=True))
        torch.cuda.synchronize()
        assert wsr.status() == 0
        if last:
            lp = (n - 1) // P
            owner_row = (kc[int(tab[lp]) * P + (n - 1) % P].clone(), vc[int(tab[lp]) * P + (n - 1) % P].clone())
    assert not torch.isnan(parts).any()
    out = torch.empty(H * D, device="cuda", dtype=qv.dtype)
    q.ops.attention_merge(parts, H, HKV, D, out)
    torch.cuda.synchronize()
    ok, err, idx = allclose_report(out, out_full, ATOL, RTOL)
    assert ok, f"max abs err {err} at {idx}"
    # the append on the owner shard wrote the same bytes as the whole-sequence call
    lp = (S - 1) // P
    full_k = kc_full[int(tab_full[lp]) * P + (S - 1) % P]
    full_v = vc_full[int(tab_full[lp]) * P + (S - 1) % P]
    assert torch.equal(owner_row[0].view(torch.int16), full_k.view(torch.int16))
    assert torch.equal(owner_row[1].view(torch.int16), full_v.view(torch.int16))


def test_partial_out_single_split_and_gate():
    """A short sequence (one split, no cluster) in partial form, merged with a gate."""
    S = 40
    k, v, qv, kn, vn, w = _sequence(S, seed=7)
    g = torch.randn(H * D, device="cuda").to(qv.dtype)
    kc, tab = _paged(k, seed=3)
    vc, _ = _paged(v, seed=3)
    ref = torch.empty(H * D, device="cuda", dtype=qv.dtype)
    ws = q.Workspace(H, HKV, D, S)
    q.decode_attention(out=ref, gate=g, **_kw(S, qv, kc.clone(), vc.clone(), tab, w, kn, vn, True, ws,
                                               num_splits=1))
    pf = q.ops.partial_floats(H, HKV, D)
    part = torch.empty(HKV * pf, device="cuda", dtype=torch.float32)
    q.decode_attention(out=part, **_kw(S, qv, kc, vc, tab, w, kn, vn, True, ws, num_splits=1, partial_out=True))
    out = torch.empty(H * D, device="cuda", dtype=qv.dtype)
    q.ops.attention_merge(part, H, HKV, D, out, gate=g)
    torch.cuda.synchronize()
    assert ws.status() == 0
    ok, err, idx = allclose_report(out, ref, ATOL, RTOL)
    assert ok, f"max abs err {err} at {idx}"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_fused_exchange_world1_equals_plain_call(dtype):
    S = 8192
    k, v, qv, kn, vn, w = _sequence(S, seed=21, dtype=dtype)
    kc, tab = _paged(k, seed=5)
    vc, _ = _paged(v, seed=5)
    group = cpm.ExchangeGroup(H, HKV, D, rank=0, world=1, gather=lambda b, r, n: [b])
    try:
        ws_cp = q.Workspace(H, HKV, D, S)
        ws = q.Workspace(H, HKV, D, S)
        for call in range(3):  # epochs 1..3: both parities of the exchange buffer
            out_cp = torch.full((H * D,), float("nan"), device="cuda", dtype=qv.dtype)
            out = torch.empty(H * D, device="cuda", dtype=qv.dtype)
            cpm.cp_decode_attention(group, out=out_cp, **_kw(S, qv, kc, vc, tab, w, kn, vn, False, ws_cp,
                                                             position=S - 1, cluster_size=8))
            q.decode_attention(out=out, **_kw(S, qv, kc, vc, tab, w, kn, vn, False, ws, cluster_size=8))
            torch.cuda.synchronize()
            assert ws_cp.status() == 0, f"call {call}"
            assert torch.equal(out_cp.view(torch.int16), out.view(torch.int16)), f"call {call}"
        epoch = torch.empty(1, dtype=torch.int32)
        epoch.copy_(ws_cp.buf[64:68].view(torch.int32).cpu())
        assert int(epoch) == 3
    finally:
        torch.cuda.synchronize()
        group.close()


def test_peer_that_never_publishes_times_out():
    """World 2 on one GPU with only rank 0 running: rank 1's words in rank 0's exchange
    buffer never carry the call's tag, so the bounded wait (50 ms) gives up."""
    S = 2048
    k, v, qv, kn, vn, w = _sequence(S, seed=33)
    kc, tab = _paged(k, seed=6)
    vc, _ = _paged(v, seed=6)
    ipc = cpm.CudaIpc()
    nbytes = int(q.lib().qic_cp_exchange_bytes(H, HKV, D, 2))
    mine, other = ipc.alloc(nbytes), ipc.alloc(nbytes)
    try:
        args = q.abi.CpArgs()
        args.rank, args.world = 0, 2
        args.exchange, args.exchange_bytes = mine, nbytes
        args.peer_exchange[0], args.peer_exchange[1] = mine, other
        args.timeout_ms = 50
        ws = q.Workspace(H, HKV, D, S)
        out = torch.full((H * D,), float("nan"), device="cuda", dtype=qv.dtype)
        a = q.ops.decode_args(out=out, **_kw(S, qv, kc, vc, tab, w, kn, vn, False, ws, position=S - 1))
        rc = q.lib().qic_cp_decode_attention(ctypes.byref(a), ctypes.byref(args),
                                             torch.cuda.current_stream().cuda_stream)
        assert rc == 0
        torch.cuda.synchronize()
        assert ws.status() & q.abi.QIC_DEV_PEER_TIMEOUT
        assert torch.isnan(out.float()).all(), "no output is written after a peer timeout"
        # the context is still usable
        ref = torch.empty(H * D, device="cuda", dtype=qv.dtype)
        q.decode_attention(out=ref, **_kw(S, qv, kc, vc, tab, w, kn, vn, False, ws))
        torch.cuda.synchronize()
        assert ws.status() == 0
        assert not torch.isnan(ref.float()).any()
    finally:
        torch.cuda.synchronize()
        ipc.free(mine)
        ipc.free(other)


def test_cp_rejects_bad_arguments():
    S = 2048
    k, v, qv, kn, vn, w = _sequence(S, seed=2)
    kc, tab = _paged(k, seed=2)
    vc, _ = _paged(v, seed=2)
    ws = q.Workspace(H, HKV, D, S)
    out = torch.empty(H * D, device="cuda", dtype=qv.dtype)
    a = q.ops.decode_args(out=out, **_kw(S, qv, kc, vc, tab, w, kn, vn, False, ws))
    args = q.abi.CpArgs()
    args.rank, args.world = 0, 2
    args.exchange = ws.ptr  # any aligned device pointer
    args.exchange_bytes = 16  # too small
    args.peer_exchange[0] = ws.ptr
    args.peer_exchange[1] = ws.ptr
    stream = torch.cuda.current_stream().cuda_stream
    assert q.lib().qic_cp_decode_attention(ctypes.byref(a), ctypes.byref(args), stream) == 4  # QIC_ERROR_WORKSPACE
    args.exchange_bytes = 1 << 30
    args.peer_exchange[0] = 0
    assert q.lib().qic_cp_decode_attention(ctypes.byref(a), ctypes.byref(args), stream) == 1
    args.peer_exchange[0] = ws.ptr
    args.world = 9
    assert q.lib().qic_cp_decode_attention(ctypes.byref(a), ctypes.byref(args), stream) == 1
    args.world = 2
    a.cluster_size = 4
    assert q.lib().qic_cp_decode_attention(ctypes.byref(a), ctypes.byref(args), stream) == 2
    a.cluster_size = 0
    a.workspace = None
    assert q.lib().qic_cp_decode_attention(ctypes.byref(a), ctypes.byref(args), stream) == 1


def _gated_case(S, seed, dtype=torch.bfloat16):
    """Qwen3.5 gated-attention shape (16 q heads, 4 kv heads, d=256): paged cache,
    raw q / k_new / v_new, norm weights and the output gate."""
    Hg, Hkvg, Dg = 16, 4, 256
    g = torch.Generator(device="cuda").manual_seed(seed)
    pages = (S + P - 1) // P
    kc = (torch.randn(pages * P, Hkvg * Dg, generator=g, device="cuda") * 0.5).to(dtype)
    vc = (torch.randn(pages * P, Hkvg * Dg, generator=g, device="cuda") * 0.5).to(dtype)
    tab = torch.randperm(pages, generator=g, device="cuda").to(torch.int32)
    qv = torch.randn(Hg * Dg, generator=g, device="cuda").to(dtype)
    kn = torch.randn(Hkvg * Dg, generator=g, device="cuda").to(dtype)
    vn = (torch.randn(Hkvg * Dg, generator=g, device="cuda") * 0.5).to(dtype)
    gate = torch.randn(Hg * Dg, generator=g, device="cuda").to(dtype)
    w = (1.0 + 0.1 * torch.randn(Dg, generator=g, device="cuda")).to(dtype)
    kw = dict(q=qv, k_cache=kc, v_cache=vc, num_heads=Hg, num_kv_heads=Hkvg, head_dim=Dg, seq_len=S,
              page_table=tab, page_size=P, q_norm_w=w, k_norm_w=w, k_new=kn, v_new=vn, fuse_q=True, gate=gate)
    return (Hg, Hkvg, Dg), kw


@pytest.mark.parametrize("interleaved", [False, True])
def test_fused_exchange_world1_gated_d256(interleaved):
    """Gated d=256 shape through the fused exchange at world 1: bit-identical to the
    plain call (gate applied once, after the merge), two calls in a row; with
    `interleaved` the exchange call reads q and the gate from the packed [H, 2d]
    projection. Both run with QIC_DETERMINISTIC: at this length the stage pool would
    otherwise change the order of the split sums from call to call."""
    S = 16385
    (Hg, Hkvg, Dg), kw = _gated_case(S, seed=41)
    kw_cp = dict(kw)
    if interleaved:
        packed = torch.cat([kw["q"].view(Hg, Dg), kw["gate"].view(Hg, Dg)], dim=1).flatten()
        kw_cp.update(q=packed, gate=None, q_gate_interleaved=True)
    group = cpm.ExchangeGroup(Hg, Hkvg, Dg, rank=0, world=1, gather=lambda b, r, n: [b])
    try:
        ws_cp = q.Workspace(Hg, Hkvg, Dg, S)
        ws = q.Workspace(Hg, Hkvg, Dg, S)
        for call in range(2):
            out_cp = torch.full((Hg * Dg,), float("nan"), device="cuda", dtype=torch.bfloat16)
            out = torch.empty(Hg * Dg, device="cuda", dtype=torch.bfloat16)
            cpm.cp_decode_attention(group, out=out_cp, workspace=ws_cp, position=S - 1, cluster_size=8,
                                    deterministic=True, **kw_cp)
            q.decode_attention(out=out, workspace=ws, cluster_size=8, deterministic=True, **kw)
            torch.cuda.synchronize()
            assert ws_cp.status() == 0 and ws.status() == 0
            assert torch.equal(out_cp.view(torch.int16), out.view(torch.int16)), f"call {call}"
    finally:
        torch.cuda.synchronize()
        group.close()


def test_gated_d256_partials_merge_with_gate():
    """Gated d=256 shape: two token ranges as partials (q prologue at the global
    position), merged with the gate by qic_attention_merge, equal the whole call."""
    S = 6001
    (Hg, Hkvg, Dg), kw = _gated_case(S, seed=43)
    gate = kw.pop("gate")
    ref = torch.empty(Hg * Dg, device="cuda", dtype=torch.bfloat16)
    q.decode_attention(out=ref, gate=gate, workspace=q.Workspace(Hg, Hkvg, Dg, S), **kw)
    pf = q.ops.partial_floats(Hg, Hkvg, Dg)
    parts = torch.empty((2, Hkvg * pf), device="cuda", dtype=torch.float32)
    tab = kw["page_table"]
    cut = 200 * P  # tokens [0, cut) and [cut, S): the second range's table is the tail of the first
    for r, (t0, t1) in enumerate([(0, cut), (cut, S)]):
        kr = dict(kw, seq_len=t1 - t0, page_table=tab[t0 // P:].contiguous())
        q.decode_attention(out=parts[r], workspace=q.Workspace(Hg, Hkvg, Dg, t1 - t0), position=S - 1,
                           partial_out=True, **kr)
    out = torch.empty(Hg * Dg, device="cuda", dtype=torch.bfloat16)
    q.ops.attention_merge(parts, Hg, Hkvg, Dg, out, gate=gate)
    torch.cuda.synchronize()
    ok, err, idx = allclose_report(out, ref, ATOL, RTOL)
    assert ok, f"max abs err {err} at {idx}"
