"""Work split across GPUs, one process per GPU.

Long single sequences (context parallelism): the sequence's pages are cut into
contiguous ranges, one per rank (shard_tokens). Every rank keeps the K/V pages and
block table of its own range and calls qic_cp_decode_attention with the same q;
inside the kernel the rank's (o, lse) partial of each (kv head, slice), merged over
the rank's clusters, is stored into every rank's exchange buffer over NVLink as
tagged 8-byte words, and the CTA that produced that slice polls the words of every
rank's contribution (bounded wait) and merges them by log-sum-exp, so every rank
ends with the full output. The rank that holds the last token performs the append. ExchangeGroup allocates this rank's
exchange buffer and maps every other rank's buffer into this process with CUDA IPC;
the IPC handles travel over torch.distributed (any backend, gloo included).

Batched requests: sequences are assigned to ranks by K/V bytes, longest first
(partition_sequences); each rank decodes its own sequences from its own page pool and
nothing is exchanged.

The reference runs on one GPU and has neither; the math each rank runs is the
reference's attention (src/kernels.cu:292-374) over its token range.
"""
from __future__ import annotations

import ctypes
import heapq

from .abi import QIC_IPC_HANDLE_BYTES, QIC_MAX_RANKS, CpArgs, check, lib
from .ops import _stream, decode_args


def shard_tokens(seq_len: int, page_size: int, world: int) -> list[tuple[int, int]]:
    """Token range [lo, hi) of every rank: whole pages, contiguous, as even as the page
    count allows; rank world-1 holds the last (possibly partial) page, hence the token
    at position seq_len-1."""
    if world < 1 or seq_len < 1 or page_size < 1:
        raise ValueError("world, seq_len and page_size must be positive")
    pages = (seq_len + page_size - 1) // page_size
    if pages < world:
        raise ValueError(f"{pages} pages cannot be shared by {world} ranks")
    out = []
    for r in range(world):
        p_lo, p_hi = r * pages // world, (r + 1) * pages // world
        out.append((p_lo * page_size, min(p_hi * page_size, seq_len)))
    return out


def partition_sequences(seq_lens, world: int) -> list[list[int]]:
    """Sequence indices of every rank, balanced by tokens (K/V bytes are proportional):
    longest first, each to the rank with the fewest tokens so far (lowest rank on ties)."""
    if world < 1:
        raise ValueError("world must be positive")
    order = sorted(range(len(seq_lens)), key=lambda i: (-int(seq_lens[i]), i))
    heap = [(0, r) for r in range(world)]
    parts: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        parts[r].append(i)
        heapq.heappush(heap, (load + int(seq_lens[i]), r))
    return [sorted(p) for p in parts]


class CudaIpc:
    """Exchange-buffer memory and CUDA IPC through libqic (qic_device_alloc, qic_ipc_*)."""

    def alloc(self, nbytes: int) -> int:
        p = ctypes.c_void_p(0)
        check(lib().qic_device_alloc(nbytes, ctypes.byref(p)), "qic_device_alloc")
        return int(p.value)

    def free(self, ptr: int) -> None:
        check(lib().qic_device_free(ptr), "qic_device_free")

    def handle(self, ptr: int) -> bytes:
        buf = (ctypes.c_ubyte * QIC_IPC_HANDLE_BYTES)()
        check(lib().qic_ipc_get_handle(ptr, ctypes.cast(buf, ctypes.c_void_p)), "qic_ipc_get_handle")
        return bytes(buf)

    def open(self, handle: bytes) -> int:
        buf = (ctypes.c_ubyte * QIC_IPC_HANDLE_BYTES).from_buffer_copy(handle)
        p = ctypes.c_void_p(0)
        check(lib().qic_ipc_open_handle(ctypes.cast(buf, ctypes.c_void_p), ctypes.byref(p)), "qic_ipc_open_handle")
        return int(p.value)

    def close(self, ptr: int) -> None:
        check(lib().qic_ipc_close_handle(ptr), "qic_ipc_close_handle")


def _all_gather_bytes(payload: bytes, rank: int, world: int, group=None) -> list[bytes]:
    import torch.distributed as dist

    out: list = [None] * world
    dist.all_gather_object(out, payload, group=group)
    return out


class ExchangeGroup:
    """This rank's exchange buffer plus every other rank's, mapped into this process.

    Collective: every rank of the group constructs it at the same point, with the same
    shapes. `gather` (payload, rank, world) -> list of every rank's payload defaults to
    torch.distributed.all_gather_object; `ipc` defaults to CUDA IPC through libqic.
    """

    def __init__(self, num_heads: int, num_kv_heads: int, head_dim: int, rank: int, world: int, *,
                 timeout_ms: int = 0, group=None, gather=None, ipc=None):
        if not 1 <= world <= QIC_MAX_RANKS or not 0 <= rank < world:
            raise ValueError(f"rank {rank} of world {world} (at most {QIC_MAX_RANKS} ranks)")
        self.rank, self.world = rank, world
        self.ipc = ipc if ipc is not None else CudaIpc()
        self.nbytes = int(lib().qic_cp_exchange_bytes(num_heads, num_kv_heads, head_dim, world))
        if self.nbytes == 0:
            raise ValueError("invalid exchange shape")
        self.local = self.ipc.alloc(self.nbytes)
        gather = gather if gather is not None else (lambda b, r, w: _all_gather_bytes(b, r, w, group))
        handles = gather(self.ipc.handle(self.local), rank, world)
        if len(handles) != world:
            raise RuntimeError(f"expected {world} handles, got {len(handles)}")
        self.peers: list[int] = []
        self._opened: list[int] = []
        for r, h in enumerate(handles):
            if r == rank:
                self.peers.append(self.local)
            else:
                ptr = self.ipc.open(h)
                self._opened.append(ptr)
                self.peers.append(ptr)
        self.args = CpArgs()
        self.args.rank, self.args.world = rank, world
        self.args.exchange = self.local
        self.args.exchange_bytes = self.nbytes
        for r, ptr in enumerate(self.peers):
            self.args.peer_exchange[r] = ptr
        self.args.timeout_ms = timeout_ms

    def close(self) -> None:
        """Unmaps the peers' buffers and frees this rank's (after the device is idle)."""
        for ptr in self._opened:
            self.ipc.close(ptr)
        self._opened = []
        if self.local:
            self.ipc.free(self.local)
            self.local = 0


def exchange_bytes_host(num_heads: int, num_kv_heads: int, head_dim: int, world: int) -> int:
    """Size of one rank's exchange buffer, computed on the host (the layout of
    qic_cp_exchange_bytes): [2 parities][world][Hkv][8 slices] contributions of
    ceil(G*d/8) + 2 eight-byte words (outputs, then two log-sum-exp words)."""
    g = num_heads // num_kv_heads
    words = (g * head_dim + 7) // 8 + 2
    return 2 * world * num_kv_heads * 8 * words * 8


def cp_decode_attention(group: ExchangeGroup, stream=None, **kw) -> None:
    """One rank's call of qic_cp_decode_attention (decode_args keywords; the workspace is
    required, and `position` is the global position of the new token)."""
    if kw.get("workspace") is None:
        raise ValueError("context-parallel attention needs a workspace (it keeps the exchange epoch)")
    a = decode_args(**kw)
    check(lib().qic_cp_decode_attention(ctypes.byref(a), ctypes.byref(group.args), _stream(stream)),
          "qic_cp_decode_attention")


def cp_args_pointer(group: ExchangeGroup):
    """ctypes pointer to the group's qic_cp_args (for callers that build their own calls)."""
    return ctypes.byref(group.args)


__all__ = ["shard_tokens", "partition_sequences", "ExchangeGroup", "CudaIpc", "cp_decode_attention",
           "exchange_bytes_host", "cp_args_pointer"]
