"""CPU: the host side of the multi-GPU paths.

* shard_tokens: contiguous whole-page token ranges covering the sequence, the last
  token on the last rank, pages balanced within one.
* partition_sequences: every sequence on exactly one rank, loads balanced (longest
  processing time first).
* ExchangeGroup over a real 2-rank gloo process group (spawned processes), with a
  fake IPC backend: every rank maps every other rank's handle, in rank order, and
  keeps its own buffer in its own slot.
* The (o, lse) partial format: partials of disjoint token ranges merged by
  log-sum-exp give the attention over the whole range (numpy, float64).
* The exchange-buffer size formula agrees with the library's.
"""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

from qwenincuda_b200 import context_parallel as cpm  # noqa: E402


@pytest.mark.parametrize("S,P,world", [(131073, 16, 8), (131073, 16, 3), (8197, 16, 2), (1025, 16, 4), (64, 16, 4),
                                       (100, 32, 2)])
def test_shard_tokens(S, P, world):
    shards = cpm.shard_tokens(S, P, world)
    assert len(shards) == world
    assert shards[0][0] == 0 and shards[-1][1] == S
    for (a0, a1), (b0, b1) in zip(shards, shards[1:]):
        assert a1 == b0
    for t0, t1 in shards:
        assert t0 % P == 0 and t1 > t0
    pages = [(t1 - t0 + P - 1) // P for t0, t1 in shards]
    assert max(pages) - min(pages) <= 1
    assert shards[-1][0] <= S - 1 < shards[-1][1]


def test_shard_tokens_rejects_too_many_ranks():
    with pytest.raises(ValueError):
        cpm.shard_tokens(16, 16, 2)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_partition_sequences(world):
    rng = np.random.default_rng(6)
    lens = [int(x) + 1 for x in rng.integers(512, 32769, size=64)]
    parts = cpm.partition_sequences(lens, world)
    flat = sorted(i for p in parts for i in p)
    assert flat == list(range(64))
    loads = [sum(lens[i] for i in p) for p in parts]
    assert max(loads) - min(loads) <= max(lens)
    assert max(loads) <= sum(lens) / world * 4 / 3 + max(lens)
    assert parts == cpm.partition_sequences(lens, world)  # deterministic


def test_partial_merge_equals_whole_range():
    rng = np.random.default_rng(1)
    G, D, S = 4, 16, 300
    q = rng.standard_normal((G, D))
    k = rng.standard_normal((S, D))
    v = rng.standard_normal((S, D))
    scale = np.log2(np.e) / np.sqrt(D)
    s = q @ k.T * scale  # log2-domain scores

    def partial(lo, hi):
        m = s[:, lo:hi].max(1, keepdims=True)
        p = np.exp2(s[:, lo:hi] - m)
        l = p.sum(1, keepdims=True)
        return (p @ v[lo:hi]) / l, (m + np.log2(l))[:, 0]

    whole, _ = partial(0, S)
    cuts = [0, 17, 160, 161, S]
    parts = [partial(a, b) for a, b in zip(cuts, cuts[1:])]
    lse = np.stack([p[1] for p in parts])  # [n, G]
    mx = lse.max(0)
    wts = np.exp2(lse - mx)
    merged = sum(wts[i][:, None] * parts[i][0] for i in range(len(parts))) / wts.sum(0)[:, None]
    np.testing.assert_allclose(merged, whole, rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("H,Hkv,D,world", [(32, 8, 128, 8), (16, 4, 256, 2), (8, 8, 64, 1)])
def test_exchange_bytes_formula(H, Hkv, D, world):
    from qwenincuda_b200.abi import lib

    assert cpm.exchange_bytes_host(H, Hkv, D, world) == lib().qic_cp_exchange_bytes(H, Hkv, D, world)


class FakeIpc:
    """Stands in for CUDA IPC: buffers are integers, a handle names its owner."""

    def __init__(self, rank):
        self.rank = rank
        self.opened, self.closed, self.freed = [], [], []

    def alloc(self, nbytes):
        return 0x1000 * (self.rank + 1)

    def free(self, ptr):
        self.freed.append(ptr)

    def handle(self, ptr):
        return f"rank{self.rank}:{ptr}".encode()

    def open(self, handle):
        owner, ptr = handle.decode().split(":")
        mapped = 0x100000 + int(ptr)
        self.opened.append((owner, mapped))
        return mapped

    def close(self, ptr):
        self.closed.append(ptr)


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    import datetime

    import torch.distributed as dist

    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "tests"))
    from test_partition_cpu import FakeIpc as Fake

    from qwenincuda_b200 import context_parallel as cp

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    try:
        ipc = Fake(rank)
        g = cp.ExchangeGroup(32, 8, 128, rank, world, ipc=ipc, timeout_ms=7)
        plan = (cp.shard_tokens(131073, 16, world), cp.partition_sequences([5, 9, 2, 7, 3], world))
        plans = [None] * world
        dist.all_gather_object(plans, plan)
        g.close()
        out.put((rank, list(g.peers), g.args.rank, g.args.world, g.args.timeout_ms,
                 [g.args.peer_exchange[r] for r in range(world)], ipc.opened, ipc.closed, ipc.freed,
                 all(p == plans[0] for p in plans), None))
    except Exception:
        import traceback

        out.put((rank,) + (None,) * 9 + (traceback.format_exc(),))
    finally:
        dist.destroy_process_group()


def test_exchange_group_over_gloo_two_ranks():
    import torch.multiprocessing as mp

    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    world, port = 2, _port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r = out.get(timeout=120)
            res[r[0]] = r
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    for rank in range(world):
        _, peers, arank, aworld, tmo, pex, opened, closed, freed, same_plan, tb = res[rank]
        assert tb is None, tb
        own = 0x1000 * (rank + 1)
        assert peers[rank] == own and pex[rank] == own
        for r in range(world):
            if r != rank:
                assert peers[r] == 0x100000 + 0x1000 * (r + 1)
        assert [o for o, _ in opened] == [f"rank{r}" for r in range(world) if r != rank]
        assert sorted(closed) == sorted(p for i, p in enumerate(peers) if i != rank)
        assert freed == [own]
        assert (arank, aworld, tmo) == (rank, world, 7)
        assert same_plan
