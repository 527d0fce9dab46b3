"""GPU, two or more devices: the fused context-parallel exchange across real GPUs.

Each rank is a spawned process on its own GPU. All ranks build the same seeded
sequence, keep their own shard (shard_tokens) in their own shuffled page pool, map
each other's exchange buffers with CUDA IPC (handles exchanged over a gloo process
group) and call qic_cp_decode_attention three times. Every rank checks its output
against the whole-sequence call made on its own GPU (also over four calls chained with
programmatic dependent launch) and against the reference's own chain on the whole
sequence (head-norm + RoPE of q and k, row copies, paged_attention
of src/kernels.cu built for sm_100a), both within max-abs 2e-3 / rel 1e-2, and the
owner of the last token checks the appended rows byte for byte. Skipped with fewer
than two GPUs.
"""
import os
import socket
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, S, results):
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "tests"))
    import datetime

    import torch.distributed as dist

    try:
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        import qwenincuda_b200 as q
        from conftest import allclose_report
        from qwenincuda_b200 import context_parallel as cpm
        from test_context_parallel_gpu import D, H, HKV, P, _kw, _paged, _sequence

        k, v, qv, kn, vn, w = _sequence(S, seed=77)
        kc_full, tab_full = _paged(k, seed=1)
        vc_full, _ = _paged(v, seed=1)
        ws_full = q.Workspace(H, HKV, D, S)
        want = torch.empty(H * D, device="cuda", dtype=qv.dtype)
        q.decode_attention(out=want, **_kw(S, qv, kc_full, vc_full, tab_full, w, kn, vn, True, ws_full))
        torch.cuda.synchronize()
        # the reference's chain on the whole sequence, on copies of the caches
        from oracle.oracle import RefKernels

        ref = RefKernels(qv.dtype)
        kr, vr = kc_full.clone(), vc_full.clone()
        lf = (S - 1) // P
        ref.append_chain(kn, vn, w, 1e-6, 1.0e6, S - 1, kr, vr, HKV, D, int(tab_full[lf]) * P + (S - 1) % P)
        qr = qv.clone()
        ref.head_rmsnorm(qr, w, H, D, 1e-6, qr)
        ref.rope_inplace(qr, H, D, S - 1, 1.0e6)
        want_ref = torch.empty(H * D, device="cuda", dtype=qv.dtype)
        ref.paged_attention(qr, kr, vr, tab_full, P, H, HKV, D, S, want_ref)
        del kr, vr
        t0, t1 = cpm.shard_tokens(S, P, world)[rank]
        n = t1 - t0
        kc, tab = _paged(k[t0:t1], seed=10 + rank)
        vc, _ = _paged(v[t0:t1], seed=10 + rank)
        last = rank == world - 1
        group = cpm.ExchangeGroup(H, HKV, D, rank, world, timeout_ms=5000)
        ws = q.Workspace(H, HKV, D, n)
        errs = []
        for call in range(3):
            out = torch.full((H * D,), float("nan"), device="cuda", dtype=qv.dtype)
            # the append happens once; later calls attend over the appended row again
            cpm.cp_decode_attention(group, out=out, **_kw(n, qv, kc, vc, tab, w, kn, vn, last and call == 0, ws,
                                                          position=S - 1))
            torch.cuda.synchronize()
            st = ws.status()
            ok, err, idx = allclose_report(out, want, 2e-3, 1e-2)
            ok_r, err_r, _ = allclose_report(out, want_ref, 2e-3, 1e-2)
            errs.append((call, st, ok and ok_r, max(err, err_r)))
        # four more calls chained with programmatic dependent launch, not synchronised in
        # between: each call's K/V copies start while the previous call exchanges
        outs = [torch.full((H * D,), float("nan"), device="cuda", dtype=qv.dtype) for _ in range(4)]
        for o in outs:
            cpm.cp_decode_attention(group, out=o, pdl=True, **_kw(n, qv, kc, vc, tab, w, kn, vn, False, ws,
                                                                  position=S - 1))
        torch.cuda.synchronize()
        st = ws.status()
        for i, o in enumerate(outs):
            ok, err, idx = allclose_report(o, want, 2e-3, 1e-2)
            errs.append((3 + i, st, ok, err))
        row_ok = True
        if last:
            lp, lf = (n - 1) // P, (S - 1) // P
            row_ok = (torch.equal(kc[int(tab[lp]) * P + (n - 1) % P].view(torch.int16),
                                  kc_full[int(tab_full[lf]) * P + (S - 1) % P].view(torch.int16)) and
                      torch.equal(vc[int(tab[lp]) * P + (n - 1) % P].view(torch.int16),
                                  vc_full[int(tab_full[lf]) * P + (S - 1) % P].view(torch.int16)))
        dist.barrier()  # no rank unmaps a buffer another rank may still write
        torch.cuda.synchronize()
        group.close()
        dist.destroy_process_group()
        results.put((rank, errs, row_ok, None))
    except Exception as exc:  # reported to the parent
        import traceback

        results.put((rank, None, False, traceback.format_exc()))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_fused_exchange_across_gpus(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = _free_port()
    S = 8192 + 5
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, S, results)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(world):
            rank, errs, row_ok, tb = results.get(timeout=240)
            got[rank] = (errs, row_ok, tb)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank in range(world):
        errs, row_ok, tb = got[rank]
        assert tb is None, f"rank {rank}:\n{tb}"
        for call, st, ok, err in errs:
            assert st == 0, f"rank {rank} call {call}: device status {st}"
            assert ok, f"rank {rank} call {call}: max abs err {err}"
        assert row_ok, f"rank {rank}: appended rows differ"
