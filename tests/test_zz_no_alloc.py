"""GPU: qic_decode_attention_noalloc, the entry point for callers that cannot allocate
device memory (code written against the reference's kernels.cuh interface has no
workspace to pass, and a per-token decode loop must not stop for a synchronising
cudaMalloc). Its scratch is a fixed array inside the library; this checks, through
the C-ABI, that two calls in a row give the same results as qic_decode_attention
with a caller-allocated workspace, that repeated calls take no device memory, and
that the array's device status word reports a bad page-table entry to
qic_noalloc_status instead of being cleared by the next call. Collected last so a
failure here comes after every other test has run; it also passes alone in a fresh
process."""
import ctypes

import pytest
import torch

import qwenincuda_b200 as q
from conftest import allclose_report
from qwenincuda_b200.workloads import AttnConfig, make_attention_inputs

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-3, 1e-2


def _args(inp, layer, out, cfg, workspace=None, page_table=None):
    return q.ops.decode_args(
        q=inp.q[layer], k_cache=inp.k_cache[layer], v_cache=inp.v_cache[layer], out=out, num_heads=cfg.num_heads,
        num_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim, seq_len=cfg.seq_len,
        page_table=inp.page_table[layer] if page_table is None else page_table, page_size=cfg.page_size,
        workspace=workspace, cache_tokens=inp.cache_tokens)


def _noalloc_status(L, stream):
    v = ctypes.c_int(-1)
    assert L.qic_noalloc_status(stream, ctypes.byref(v)) == 0
    return v.value


def test_noalloc_two_calls_match_workspace_entry_point():
    L = q.lib()
    assert L.qic_noalloc_scratch_bytes() == 2 << 20
    # long enough that several thread-block clusters merge through the scratch partials
    cfg = AttnConfig("noalloc", 32, 8, 128, 12000, layers=2, seed=21)
    inp = make_attention_inputs(cfg, paged=True)
    ws = q.Workspace(cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, cfg.seq_len)
    stream = torch.cuda.current_stream().cuda_stream
    for layer in range(2):
        want = torch.empty(cfg.num_heads * cfg.head_dim, device="cuda", dtype=torch.bfloat16)
        a = _args(inp, layer, want, cfg, workspace=ws)
        assert L.qic_decode_attention(ctypes.byref(a), stream) == 0
        got = torch.full_like(want, float("nan"))
        b = _args(inp, layer, got, cfg)
        assert L.qic_decode_attention_noalloc(ctypes.byref(b), stream) == 0
        torch.cuda.synchronize()
        assert ws.status() == 0
        assert _noalloc_status(L, stream) == 0
        ok, err, idx = allclose_report(got, want, ATOL, RTOL)
        assert ok, f"call {layer}: max abs err {err} at {idx}"


def test_noalloc_takes_no_device_memory():
    """After the first call, repeated calls leave the device's free memory unchanged."""
    L = q.lib()
    cfg = AttnConfig("noalloc_mem", 32, 8, 128, 9000, layers=1, seed=23)
    inp = make_attention_inputs(cfg, paged=True)
    out = torch.empty(cfg.num_heads * cfg.head_dim, device="cuda", dtype=torch.bfloat16)
    stream = torch.cuda.current_stream().cuda_stream
    a = _args(inp, 0, out, cfg)
    assert L.qic_decode_attention_noalloc(ctypes.byref(a), stream) == 0
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(20):
        assert L.qic_decode_attention_noalloc(ctypes.byref(a), stream) == 0
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    assert _noalloc_status(L, stream) == 0


def test_noalloc_graph_replays_a_chained_decode_loop():
    """Two noalloc calls (two layers, chained with QIC_PDL, the length read from device
    memory) captured once in a CUDA graph and replayed at three lengths give the bytes
    of the workspace entry point called with each length by value, at the same launch
    shape; the scratch status word stays clear."""
    L = q.lib()
    S_max = 5000
    cfg = AttnConfig("noalloc_graph", 32, 8, 128, S_max, layers=2, seed=25)
    inp = make_attention_inputs(cfg, paged=True)
    stream = torch.cuda.current_stream().cuda_stream
    shape = dict(num_splits=16, cluster_size=8, deterministic=True)

    def call(layer, out, seq_len, entry, **kw):
        a = q.ops.decode_args(
            q=inp.q[layer], k_cache=inp.k_cache[layer], v_cache=inp.v_cache[layer], out=out,
            num_heads=cfg.num_heads, num_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim, seq_len=seq_len,
            page_table=inp.page_table[layer], page_size=cfg.page_size, cache_tokens=inp.cache_tokens, **shape, **kw)
        assert entry(ctypes.byref(a), torch.cuda.current_stream().cuda_stream) == 0

    lengths = (4999, 3001, 17)
    ws = q.Workspace(cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, S_max)
    want = []
    for S in lengths:
        outs = [torch.empty(cfg.num_heads * cfg.head_dim, device="cuda", dtype=torch.bfloat16) for _ in range(2)]
        for layer in range(2):
            call(layer, outs[layer], S, L.qic_decode_attention, workspace=ws)
        want.append(outs)
    torch.cuda.synchronize()
    assert ws.status() == 0

    length = torch.tensor([S_max], dtype=torch.int32, device="cuda")
    outs = [torch.empty(cfg.num_heads * cfg.head_dim, device="cuda", dtype=torch.bfloat16) for _ in range(2)]
    for layer in range(2):  # the first call on a device looks up the scratch: outside the capture
        call(layer, outs[layer], S_max, L.qic_decode_attention_noalloc, pdl=True, seq_len_dev=length)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for layer in range(2):
            call(layer, outs[layer], S_max, L.qic_decode_attention_noalloc, pdl=True, seq_len_dev=length)
    for t, S in enumerate(lengths):
        length.fill_(S)
        graph.replay()
        torch.cuda.synchronize()
        for layer in range(2):
            assert torch.equal(outs[layer].view(torch.int16), want[t][layer].view(torch.int16)), f"S={S} layer {layer}"
    assert _noalloc_status(L, stream) == 0
    del graph


def test_noalloc_reports_a_bad_page_entry():
    """A page-table entry outside the cache is clamped by the kernel's bounds check and
    its bit stays in the array's status word, through a later clean call, until
    qic_noalloc_status reads (and clears) it."""
    L = q.lib()
    cfg = AttnConfig("noalloc_bad", 16, 8, 128, 256, layers=1, seed=24)
    inp = make_attention_inputs(cfg, paged=True)
    stream = torch.cuda.current_stream().cuda_stream
    bad = inp.page_table[0].clone()
    bad[3] = 10 ** 6
    out = torch.empty(cfg.num_heads * cfg.head_dim, device="cuda", dtype=torch.bfloat16)
    assert _noalloc_status(L, stream) == 0
    a = _args(inp, 0, out, cfg, page_table=bad)
    assert L.qic_decode_attention_noalloc(ctypes.byref(a), stream) == 0
    b = _args(inp, 0, out, cfg)  # a clean call after it keeps the bit
    assert L.qic_decode_attention_noalloc(ctypes.byref(b), stream) == 0
    assert _noalloc_status(L, stream) & q.abi.QIC_DEV_BAD_PAGE
    assert _noalloc_status(L, stream) == 0  # cleared by the read


def test_noalloc_rejects_shapes_beyond_its_scratch():
    """A split count whose partials exceed the fixed array is refused before launch."""
    L = q.lib()
    cfg = AttnConfig("noalloc_big", 64, 8, 256, 40000, seed=22)
    inp = make_attention_inputs(cfg, paged=True)
    out = torch.empty(cfg.num_heads * cfg.head_dim, device="cuda", dtype=torch.bfloat16)
    a = _args(inp, 0, out, cfg)
    a.num_splits, a.cluster_size = 256, 1  # 8 kv heads x 256 partial slots of 8 KB each
    assert L.qic_decode_attention_noalloc(ctypes.byref(a), torch.cuda.current_stream().cuda_stream) == 4
