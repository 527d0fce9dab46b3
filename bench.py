"""Benchmark of the decode-time KV-cache hot path (one JSON line on rank 0).

Default workload (the benchmark configuration the metric is quoted on): Qwen3-8B
full-attention decode, 36 layers, 32 query heads, 8 kv heads, head_dim 128, bf16,
8191 cached tokens + 1 appended per layer (S = 8192), paged layout (page 16, seeded
shuffled block table per layer). One step = for every layer, one fused launch: q
head-RMSNorm + RoPE, k head-RMSNorm + RoPE + page write of the new token (append),
split-KV attention over all 8192 positions; layers chained with programmatic
dependent launch inside a CUDA graph. Synthetic seeded data; the step's K/V (1.2 GB)
is larger than L2. The contiguous (flash) layout is timed as well.

metric: decode-attn KV-read GB/s = (K+V bytes read for S tokens + append bytes) per
layer x layers / step time; also reported as us per layer. N > 1 GPUs (torchrun, one
process per GPU): the default workload runs one independent replica per GPU (a
single-sequence layer does not shard; weak scaling, value = N x bytes / the slowest
rank's step time). At every N (N = 1 included) the same JSON line carries the
partitioned configurations: `context_parallel_qwen3_8b_s131073` (the 131073-token
sequence split across the ranks with the fused in-kernel NVLink exchange; the NCCL
all-gather path timed beside it) and `partitioned_qwen3_8b_batch64` (the 64-sequence
batch partitioned by K/V bytes), each with whole-job GB/s (total bytes / the slowest
rank's time), the whole job timed on one GPU in the same run (rank 0 alone), the
speed-up over it and the efficiency (speed-up / N). At N = 1 the line also carries
`qwen35_gated_s32769`, `qwen3_0p6b_s1025` and `qwen35_gdn` (each with its roofline
fraction) and `e2e_eager` (the end-to-end step without a CUDA graph: one C-ABI call
per layer, with the host's time per call). --workload qwen3_8b_s131073 or
qwen3_8b_batch64 with N > 1 makes a partitioned configuration the line's value.
`config` is the same in this line and the reference arm's; run-dependent details
are under `details`.

Other workloads (--workload): qwen3_0p6b_s1025 (32 chained layers of S=1025, each with
its own cache: 134 MB per step), qwen35_gated_s32769 (d=256;
q is the interleaved q/gate projection and the output is gated; 8 layers chained like
the full-attention layers of a hybrid stack, each with its own 32K cache),
qwen3_8b_s131073 (single 128K sequence), qwen35_gdn (32 chained GatedDeltaNet layers,
each with its own state; state bytes),
qwen35_pair (GatedDeltaNet + gated attention layer), qwen3_8b_batch64 (64 sequences,
lengths 512..32768, one shared page pool, one batched launch). Profiling runs with
--no-extra: gemv_qwen3_8b (the projections alone) and qwen35_4b_decode_step (the
decode-step runner alone, one line of its figures). Tuning runs: --splits, --seq-len.

--impl reference (rank 0 only): the reference's implementation of the same workload
on the host cores, as the line's value, on a bounded sample. Attention: the oracle's C
restatement of src/kernels.cu's paged attention, OpenMP over heads (the reference has
no CPU attention), and the reference's own kernels built for sm_100a timed on the GPU
as extra information. GatedDeltaNet: the reference's own step, whose loop runs on the
host (run_linear_attention_block, src/model.cpp:656-795, built unchanged into
oracle/_ref), or the oracle's restatement of it when that library is absent.
"""
from __future__ import annotations

import argparse
import ctypes
import dataclasses
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
ATTN_WORKLOADS = ("qwen3_0p6b_s1025", "qwen3_8b_s8192", "qwen35_gated_s32769", "qwen3_8b_s131073")
GDN_STACK_LAYERS = 32  # GatedDeltaNet layers per qwen35_gdn step: 146 MB, more than L2


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "source": "measured"}
    return dict(PEAKS_FALLBACK, source="fallback")


def measured_traffic(workload: str):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary of
    this workload (profiles/<kernel>_<workload>.md or profiles/<workload>.md, line
    'traffic_bytes_per_launch: N')."""
    paths = list((ROOT / "profiles").glob(f"*_{workload}.md")) + list((ROOT / "profiles").glob(f"{workload}.md"))
    for p in paths:
        for line in p.read_text().splitlines():
            if line.startswith("traffic_bytes_per_launch:"):
                try:
                    return int(line.split(":", 1)[1].strip())
                except ValueError:
                    return None
    return None


class ClockSampler:
    """Samples SM clock and throttle reasons with NVML while the timed region runs."""

    NAMES = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown", 0x4: "sw_power_cap",
             0x80: "hw_power_brake_slowdown"}

    def __init__(self, device_index: int, period_s: float = 0.002):
        self.period = period_s
        self.samples: list[int] = []
        self.reasons: set[str] = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nvml = pynvml
            self.handle = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
        except Exception:  # NVML unavailable: report no samples
            self.nvml = None

    def _run(self):
        n = self.nvml
        while not self._stop.is_set():
            try:
                self.samples.append(n.nvmlDeviceGetClockInfo(self.handle, n.NVML_CLOCK_SM))
                mask = n.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                for bit, name in self.NAMES.items():
                    if mask & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def capture(fn):
    """CUDA graph of fn (after one eager run that performs per-device set-up)."""
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    with torch.cuda.graph(g):
        fn()
    torch.cuda.synchronize()
    return g


def time_graph(g, steps, warmup, world, sampler=None):
    """ms per replay: W untimed replays, then exactly `steps` replays between CUDA
    events, bracketed by barrier + synchronize; max over ranks."""
    for _ in range(warmup):
        g.replay()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if sampler is not None:
        sampler.__enter__()
    start.record()
    for _ in range(steps):
        g.replay()
    end.record()
    torch.cuda.synchronize()
    if sampler is not None:
        sampler.__exit__()
    barrier(world)
    return max_over_ranks(start.elapsed_time(end) / steps, world)


def _call(fn, args_struct):
    def run():
        rc = fn(ctypes.byref(args_struct), torch.cuda.current_stream().cuda_stream)
        if rc != 0:
            import qwenincuda_b200 as q

            raise q.QicError(rc, fn.__name__)

    return run


# ---------------------------------------------------------------------------
# workloads: each returns dict(step=callable, bytes=int, launches=int per step,
# e2e=(callable, h2d, d2h), kernel=name, status=callable, config=dict)
# ---------------------------------------------------------------------------
def attention_workload(name, layout, layers=None, splits=0, seq_len=None):
    import dataclasses

    import qwenincuda_b200 as q
    from qwenincuda_b200.workloads import CONFIGS, make_attention_inputs

    cfg = CONFIGS[name]
    if seq_len:
        cfg = dataclasses.replace(cfg, seq_len=seq_len)
    inp = make_attention_inputs(cfg, paged=(layout == "paged"), layers=layers)
    L_ = inp.q.shape[0]
    # the step's per-layer inputs (q, k_new, v_new of every layer) live in one device
    # buffer, so the end-to-end step moves them with one host-to-device copy. Gated
    # layers take q as the interleaved [H, 2d] q/gate projection (the output of the
    # reference's wq GEMV, src/model.cpp:627), so the gate moves with it.
    gated = inp.gate is not None
    qin = torch.cat([inp.q, inp.gate], dim=2) if gated else inp.q
    packed, views = _pack([qin, inp.k_new, inp.v_new])
    qin, inp.k_new, inp.v_new = views
    ws = q.Workspace(cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, cfg.seq_len)
    fns = []
    for layer in range(L_):
        a = q.ops.decode_args(
            q=qin[layer], k_cache=inp.k_cache[layer], v_cache=inp.v_cache[layer], out=inp.out[layer],
            num_heads=cfg.num_heads, num_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim, seq_len=cfg.seq_len,
            page_table=inp.page_table[layer] if inp.paged else None, page_size=cfg.page_size,
            q_norm_w=inp.q_norm_w, k_norm_w=inp.k_norm_w, k_new=inp.k_new[layer], v_new=inp.v_new[layer],
            eps=cfg.eps, rope_theta=cfg.rope_theta, fuse_q=True, fuse_append=True, workspace=ws,
            cache_tokens=inp.cache_tokens, pdl=True, q_gate_interleaved=gated, num_splits=splits)
        fns.append(_call(q.lib().qic_decode_attention, a))

    def step():
        for f in fns:
            f()

    hin = packed.cpu().pin_memory()
    ho = torch.empty_like(inp.out, device="cpu").pin_memory()

    def e2e():
        packed.copy_(hin, non_blocking=True)
        step()
        ho.copy_(inp.out, non_blocking=True)

    per_layer = cfg.kv_read_bytes() + cfg.append_bytes()
    return dict(step=step, bytes=per_layer * L_, launches=L_, bytes_per_launch=per_layer,
                e2e=(e2e, hin.numel() * hin.element_size(), ho.numel() * ho.element_size()),
                kernel="decode_attn_kernel", status=ws.status, keep=(inp, ws, packed),
                config={"layout": layout, "page_size": cfg.page_size, "layers": L_, "seq_len": cfg.seq_len,
                        "num_heads": cfg.num_heads, "num_kv_heads": cfg.num_kv_heads, "head_dim": cfg.head_dim,
                        "gate": "interleaved q/gate projection" if gated else False})


def _pack(tensors):
    """One device buffer holding `tensors` (same dtype) back to back, and views of it
    with their shapes (filled with their values)."""
    total = sum(t.numel() for t in tensors)
    buf = torch.empty(total, device=tensors[0].device, dtype=tensors[0].dtype)
    views, at = [], 0
    for t in tensors:
        v = buf[at:at + t.numel()].view(t.shape)
        v.copy_(t)
        views.append(v)
        at += t.numel()
    return buf, views


def gdn_workload(layers=GDN_STACK_LAYERS):
    """`layers` GatedDeltaNet layers of a hybrid stack, each with its own state and
    weights, chained with programmatic dependent launch: 32 layers move 146 MB of
    state and inputs per step, more than L2 holds."""
    import dataclasses

    import qwenincuda_b200 as q
    from qwenincuda_b200.workloads import GdnConfig, make_gdn_inputs

    cfg = GdnConfig()
    stack = [make_gdn_inputs(dataclasses.replace(cfg, seed=cfg.seed + 1000 * l)) for l in range(layers)]
    # every layer's step inputs in one buffer (one host-to-device copy per step), every
    # layer's output in another (one device-to-host copy)
    packed, views = _pack([t[k] for t in stack for k in ("qkv", "z", "b", "a")])
    outs, out_views = _pack([t["out"] for t in stack])
    for i, t in enumerate(stack):
        t["qkv"], t["z"], t["b"], t["a"] = views[4 * i:4 * i + 4]
        t["out"] = out_views[i]
    fns, args = [], []
    for t in stack:
        g = q.GdnArgs()
        g.dtype = 1
        g.num_k_heads, g.num_v_heads, g.k_head_dim, g.v_head_dim = cfg.num_k_heads, cfg.num_v_heads, 128, 128
        g.conv_kernel, g.eps = cfg.conv_kernel, cfg.eps
        # the next layer may start its weight and state loads while this one runs: each
        # layer's states are written once per step, and every step is its own graph
        # launch, so their writer has completed before the launch starts
        g.flags = q.abi.QIC_PDL | q.abi.QIC_GDN_STATES_READY
        for k in ("qkv", "z", "b", "a", "conv_w", "dt_bias", "a_log", "norm_w", "conv_state", "recurrent_state",
                  "out"):
            setattr(g, k, t[k].data_ptr())
        args.append(g)
        fns.append(_call(q.lib().qic_gated_delta_decode, g))

    def step():
        for f in fns:
            f()

    hin = packed.cpu().pin_memory()
    hout = torch.empty_like(outs, device="cpu").pin_memory()

    def e2e():
        packed.copy_(hin, non_blocking=True)
        step()
        hout.copy_(outs, non_blocking=True)

    h2d = hin.numel() * hin.element_size()
    return dict(step=step, bytes=cfg.state_bytes() * layers, launches=layers, bytes_per_launch=cfg.state_bytes(),
                e2e=(e2e, h2d, hout.numel() * hout.element_size()), kernel="gated_delta_kernel", status=lambda: 0,
                keep=(stack, args, packed, outs),
                config={"layers": layers, "num_k_heads": cfg.num_k_heads, "num_v_heads": cfg.num_v_heads,
                        "k_head_dim": 128, "v_head_dim": 128, "conv_dim": cfg.conv_dim,
                        "conv_kernel": cfg.conv_kernel, "state": "fp32, resident on the device, one per layer"})


def pair_workload():
    gdn = gdn_workload(layers=1)
    att = attention_workload("qwen35_gated_s32769", "paged", layers=1)

    def step():
        gdn["step"]()
        att["step"]()

    def e2e():
        gdn["e2e"][0]()
        att["e2e"][0]()

    # the roofline line is the attention kernel's, timed on its own (the step's two
    # launches differ too much in length to split the step time between them)
    return dict(step=step, bytes=gdn["bytes"] + att["bytes"], launches=2, bytes_per_launch=att["bytes_per_launch"],
                kernel_step=att["step"],
                e2e=(e2e, gdn["e2e"][1] + att["e2e"][1], gdn["e2e"][2] + att["e2e"][2]), kernel="decode_attn_kernel",
                status=att["status"], keep=(gdn, att),
                config={"layers": "GatedDeltaNet + gated attention (16/4 heads, d=256, S=32769, paged)",
                        "gdn_bytes": gdn["bytes"], "attention_bytes": att["bytes"]})


def batched_workload(world, rank):
    """64 sequences; with N ranks each decodes its share (partition_sequences: balanced
    by K/V bytes) from its own page pool of about 1.1M/N tokens; no exchange."""
    import dataclasses

    import qwenincuda_b200 as q
    from qwenincuda_b200.context_parallel import partition_sequences
    from qwenincuda_b200.workloads import BatchConfig, batched_bytes, make_batched_inputs

    cfg = BatchConfig()
    all_lens = cfg.seq_lens()
    mine = partition_sequences(all_lens, world)[rank]
    lens = [all_lens[i] for i in mine]
    cfg = dataclasses.replace(cfg, pool_tokens=(cfg.pool_tokens + world - 1) // world, seed=cfg.seed + 101 * rank)
    inp = make_batched_inputs(cfg, seq_lens=lens)
    packed, (inp["q"], inp["k_new"], inp["v_new"]) = _pack([inp["q"], inp["k_new"], inp["v_new"]])
    plan = q.BatchPlan(lens, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim)
    a = q.ops.batch_decode_args(plan=plan, q=inp["q"], k_cache=inp["k_cache"], v_cache=inp["v_cache"],
                                block_tables=inp["block_tables"], out=inp["out"], num_heads=cfg.num_heads,
                                num_kv_heads=cfg.num_kv_heads, head_dim=cfg.head_dim, page_size=cfg.page_size,
                                q_norm_w=inp["q_norm_w"], k_norm_w=inp["k_norm_w"], k_new=inp["k_new"],
                                v_new=inp["v_new"], fuse_q=True, fuse_append=True, cache_tokens=inp["cache_tokens"])
    step = _call(q.lib().qic_batch_decode_attention, a)
    hin = packed.cpu().pin_memory()
    ho = torch.empty_like(inp["out"], device="cpu").pin_memory()

    def e2e():
        packed.copy_(hin, non_blocking=True)
        step()
        ho.copy_(inp["out"], non_blocking=True)

    nbytes = batched_bytes(lens, cfg.kv_dim)
    return dict(step=step, bytes=nbytes, launches=1, bytes_per_launch=nbytes, partitioned=world > 1,
                e2e=(e2e, hin.numel() * 2, ho.numel() * 2), kernel="decode_attn_kernel",
                status=plan.status, keep=(inp, plan, a, packed),
                config={"batch": cfg.batch, "seq_lens": f"U[{cfg.min_len},{cfg.max_len}]+1, seed {BatchConfig().seed}",
                        "sequences_on_rank0": len(lens) if rank == 0 else None, "ranks": world,
                        "tokens_total": sum(all_lens), "page_size": cfg.page_size, "pool_tokens_per_rank": inp["cache_tokens"],
                        "plan_items": plan.items, "num_heads": cfg.num_heads, "num_kv_heads": cfg.num_kv_heads,
                        "head_dim": cfg.head_dim})


def cp_workload(world, rank, with_allgather=True, layers=2):
    """One 131073-token sequence (Qwen3-8B attention shape, page 16, shuffled tables)
    in each of `layers` layers, split into N contiguous page ranges, one per rank
    (shard_tokens). A step is one fused qic_cp_decode_attention per rank and layer: q
    prologue at the global position, the append on the rank that holds the last token,
    attention over the rank's shard, and the in-kernel NVLink exchange + log-sum-exp
    merge of the ranks' partials; the layers are chained with programmatic dependent
    launch. Two layers keep a rank's K/V per step (134 MB at 8
    ranks) larger than L2. Each rank's shards are seeded independently; q, k_new and
    v_new are the same on every rank."""
    import qwenincuda_b200 as q
    from qwenincuda_b200 import context_parallel as cpm
    from qwenincuda_b200.workloads import CONFIGS

    cfg = CONFIGS["qwen3_8b_s131073"]
    H, Hkv, d, S, P = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, cfg.seq_len, cfg.page_size
    t0, t1 = cpm.shard_tokens(S, P, world)[rank]
    n = t1 - t0
    pages = (n + P - 1) // P
    dtype = torch.bfloat16
    g = torch.Generator(device="cuda").manual_seed(cfg.seed * 1000 + 17 * rank + 1)
    kcs = [(torch.randn(pages * P, Hkv * d, generator=g, device="cuda") * cfg.kv_std).to(dtype) for _ in range(layers)]
    vcs = [(torch.randn(pages * P, Hkv * d, generator=g, device="cuda") * cfg.kv_std).to(dtype) for _ in range(layers)]
    tables = [torch.randperm(pages, generator=g, device="cuda").to(torch.int32) for _ in range(layers)]
    gs = torch.Generator(device="cuda").manual_seed(cfg.seed * 1000 + 999)
    ins = []
    for _ in range(layers):
        ins += [torch.randn(H * d, generator=gs, device="cuda").to(dtype),
                torch.randn(Hkv * d, generator=gs, device="cuda").to(dtype),
                (torch.randn(Hkv * d, generator=gs, device="cuda") * cfg.kv_std).to(dtype)]
    packed, ins = _pack(ins)  # one host-to-device copy per step
    ones = torch.ones(d, device="cuda", dtype=dtype)
    outs, out_views = _pack([torch.zeros(H * d, device="cuda", dtype=dtype) for _ in range(layers)])
    ws = q.Workspace(H, Hkv, d, n)  # the layers' calls are in stream order: one workspace, one exchange group
    owner = rank == world - 1
    group = cpm.ExchangeGroup(H, Hkv, d, rank, world, gather=(lambda b, r, n: [b]) if world == 1 else None)
    kws = [dict(q=ins[3 * l], k_cache=kcs[l], v_cache=vcs[l], num_heads=H, num_kv_heads=Hkv, head_dim=d, seq_len=n,
                page_table=tables[l], page_size=P, q_norm_w=ones, k_norm_w=ones, k_new=ins[3 * l + 1],
                v_new=ins[3 * l + 2], eps=cfg.eps, rope_theta=cfg.rope_theta, fuse_q=True, fuse_append=owner,
                workspace=ws, cache_tokens=pages * P, position=S - 1) for l in range(layers)]
    # chained with programmatic dependent launch: a layer's K/V copies start while the
    # previous layer exchanges (its exchange words are touched only after the wait)
    args = [q.ops.decode_args(out=out_views[l], pdl=True, **kws[l]) for l in range(layers)]
    lib = q.lib()
    cp_ptr = ctypes.byref(group.args)

    def step():
        for a in args:
            rc = lib.qic_cp_decode_attention(ctypes.byref(a), cp_ptr, torch.cuda.current_stream().cuda_stream)
            if rc != 0:
                raise q.QicError(rc, "qic_cp_decode_attention")

    hin = packed.cpu().pin_memory()
    ho = torch.empty_like(outs, device="cpu").pin_memory()

    def e2e():
        packed.copy_(hin, non_blocking=True)
        step()
        ho.copy_(outs, non_blocking=True)

    per_layer = 2 * n * Hkv * d * 2 + (2 * Hkv * d * 2 if owner else 0)
    allgather = None
    if with_allgather and world > 1:
        import torch.distributed as dist

        pf = q.ops.partial_floats(H, Hkv, d)
        part = torch.empty(Hkv * pf, device="cuda", dtype=torch.float32)
        gathered = torch.empty(world * Hkv * pf, device="cuda", dtype=torch.float32)
        outs2 = [torch.zeros(H * d, device="cuda", dtype=dtype) for _ in range(layers)]
        ws2 = q.Workspace(H, Hkv, d, n)
        args2 = [q.ops.decode_args(out=part, partial_out=True, **dict(kws[l], workspace=ws2, fuse_append=False))
                 for l in range(layers)]

        def ag_step():
            for l in range(layers):
                rc = lib.qic_decode_attention(ctypes.byref(args2[l]), torch.cuda.current_stream().cuda_stream)
                if rc != 0:
                    raise q.QicError(rc, "qic_decode_attention")
                dist.all_gather_into_tensor(gathered, part)
                q.ops.attention_merge(gathered, H, Hkv, d, outs2[l])

        allgather = ag_step
    return dict(step=step, bytes=per_layer * layers, launches=layers, bytes_per_launch=per_layer, partitioned=True,
                e2e=(e2e, hin.numel() * 2, ho.numel() * 2),
                kernel="decode_attn_kernel (fused NVLink exchange)", status=ws.status, allgather=allgather,
                keep=(kcs, vcs, tables, ins, outs, ws, group, args, packed),
                config={"seq_len": S, "layers": layers, "page_size": P, "num_heads": H, "num_kv_heads": Hkv,
                        "head_dim": d, "ranks": world, "shard_tokens_rank0": cpm.shard_tokens(S, P, world)[0][1],
                        "exchange": "in-kernel NVLink stores of tagged words, log-sum-exp merge"})


def gemv_workload(layers=4, hidden=4096, inter=12288, q_out=4096, kv_out=1024, seed=7):
    """The weight-streaming projections of `layers` Qwen3-8B layers (hidden 4096, 32 q
    heads and 8 kv heads of 128, FFN 12288), four launches per layer chained with
    programmatic dependent launch: RMSNorm + q/k/v (one launch over three weight
    buffers), o + residual, RMSNorm + gate/up + SwiGLU, down + residual. Every layer has
    its own weights (386 MB per layer, more than L2). Bytes = weight bytes + the
    16-bit inputs, outputs and residuals."""
    import qwenincuda_b200 as q

    dtype = torch.bfloat16
    g = torch.Generator(device="cuda").manual_seed(seed)

    def w(k, n):
        return (torch.randn(k, n, generator=g, device="cuda") * 0.02).to(dtype)

    x = torch.randn(hidden, generator=g, device="cuda").to(dtype)
    ctx = torch.randn(q_out, generator=g, device="cuda").to(dtype)  # attention output of every layer
    qb = torch.empty(q_out, device="cuda", dtype=dtype)
    kb = torch.empty(kv_out, device="cuda", dtype=dtype)
    vb = torch.empty(kv_out, device="cuda", dtype=dtype)
    hb = torch.empty(inter, device="cuda", dtype=dtype)
    ones = torch.ones(hidden, device="cuda", dtype=dtype)
    lib = q.lib()
    args, keep = [], []
    for _ in range(layers):
        wq, wk, wv, wo = w(hidden, q_out), w(hidden, kv_out), w(hidden, kv_out), w(q_out, hidden)
        wg, wu, wd = w(hidden, inter), w(hidden, inter), w(inter, hidden)
        keep += [wq, wk, wv, wo, wg, wu, wd]
        args += [q.ops.gemv_args(x=x, weights=[wq, wk, wv], outs=[qb, kb, vb], norm_w=ones, pdl=True),
                 q.ops.gemv_args(x=ctx, weights=[wo], outs=[x], residuals=[x], pdl=True),
                 q.ops.gemv_args(x=x, weights=[wg, wu], outs=[hb], norm_w=ones, swiglu=True, pdl=True),
                 q.ops.gemv_args(x=hb, weights=[wd], outs=[x], residuals=[x], pdl=True)]
    fns = [_call(lib.qic_gemv, a) for a in args]

    def step():
        for f in fns:
            f()

    W = [keep[7 * i:7 * i + 7] for i in range(layers)]

    def cublas_step():
        # the same products through torch's cuBLAS calls, unfused (norms omitted)
        for wq, wk, wv, wo, wg, wu, wd in W:
            xr = x.view(1, -1)
            torch.matmul(xr, wq, out=qb.view(1, -1))
            torch.matmul(xr, wk, out=kb.view(1, -1))
            torch.matmul(xr, wv, out=vb.view(1, -1))
            x.add_(torch.matmul(ctx.view(1, -1), wo).view(-1))
            hb.copy_((torch.nn.functional.silu(torch.matmul(xr, wg)) * torch.matmul(xr, wu)).view(-1))
            x.add_(torch.matmul(hb.view(1, -1), wd).view(-1))

    hin = x.cpu().pin_memory()
    hout = torch.empty_like(x, device="cpu").pin_memory()

    def e2e():
        x.copy_(hin, non_blocking=True)
        step()
        hout.copy_(x, non_blocking=True)

    wbytes = 2 * (hidden * (q_out + 2 * kv_out) + q_out * hidden + 2 * hidden * inter + inter * hidden)
    vec = 2 * (hidden + (q_out + 2 * kv_out) + q_out + 2 * hidden + hidden + inter + inter + 2 * hidden)
    per_layer = wbytes + vec
    splits = [q.ops.gemv_launch_shape(x=x, weights=[wq, wk, wv], outs=[qb, kb, vb], norm_w=ones)[0],
              q.ops.gemv_launch_shape(x=ctx, weights=[wo], outs=[x], residuals=[x])[0],
              q.ops.gemv_launch_shape(x=x, weights=[wg, wu], outs=[hb], norm_w=ones, swiglu=True)[0],
              q.ops.gemv_launch_shape(x=hb, weights=[wd], outs=[x], residuals=[x])[0]]
    return dict(step=step, bytes=per_layer * layers, launches=4 * layers, bytes_per_launch=per_layer / 4,
                e2e=(e2e, 2 * hidden, 2 * hidden), kernel="gemv_kernel", status=lambda: 0, keep=(keep, args),
                library_step=cublas_step,
                config={"layers": layers, "hidden": hidden, "intermediate": inter, "q_out": q_out, "kv_out": kv_out,
                        "weight_bytes_per_layer": wbytes, "launches_per_layer": 4, "splits": splits,
                        "what": "RMSNorm+q/k/v, o+residual, RMSNorm+gate/up+SwiGLU, down+residual"})


QWEN35_4B = dict(vocab_size=151936, hidden_size=2560, intermediate_size=9216, num_heads=16, num_kv_heads=4,
                 head_dim=256, linear_num_key_heads=16, linear_num_value_heads=32, linear_key_head_dim=128,
                 linear_value_head_dim=128, linear_conv_kernel_dim=4, rms_norm_eps=1e-6, rope_theta=1.0e7)


def decode_step_workload(context=4096, layer_types=(1, 1, 1, 0) * 8, seed=9):
    """One whole decode step of a Qwen3.5-4B-shaped hybrid model (32 layers: 24
    GatedDeltaNet, 8 gated full attention with 16/4 heads of 256; hidden 2560, FFN 9216,
    vocab 151936) with random bf16 weights, through the decode-step runner
    (qic_model_create + the captured step graph) at position `context` (the caches hold
    `context` tokens). Bytes = weights + the K/V read by the attention layers + the
    GatedDeltaNet states read and written."""
    import qwenincuda_b200 as q
    from qwenincuda_b200.abi import QIC_DTYPE_BF16
    from qwenincuda_b200.workloads import GdnConfig

    c = dict(QWEN35_4B, max_seq_len=context + 1, num_layers=len(layer_types))
    dt = torch.bfloat16
    g = torch.Generator(device="cuda").manual_seed(seed)
    hid, inter, V = c["hidden_size"], c["intermediate_size"], c["vocab_size"]
    qd, kvd = c["num_heads"] * c["head_dim"], c["num_kv_heads"] * c["head_dim"]
    kd, vd = c["linear_num_key_heads"] * 128, c["linear_num_value_heads"] * 128
    conv, Hv = 2 * kd + vd, c["linear_num_value_heads"]

    def w(*shape, std=None):
        std = std if std is not None else 1.0 / shape[0] ** 0.5
        return (torch.randn(*shape, generator=g, device="cuda") * std).to(dt)

    def ones(n):
        return torch.ones(n, device="cuda", dtype=dt)

    layers, nbytes = [], 0
    for kind in layer_types:
        lw = dict(is_linear=kind, attn_norm=ones(hid), ffn_norm=ones(hid), w_gate=w(hid, inter), w_up=w(hid, inter),
                  w_down=w(inter, hid))
        if kind == 1:
            lw.update(linear_in_qkv=w(hid, conv), linear_in_z=w(hid, vd), linear_in_b=w(hid, Hv),
                      linear_in_a=w(hid, Hv), linear_conv1d_w=w(conv, 4, std=0.5), linear_dt_bias=w(Hv, std=0.1),
                      linear_a_log=torch.log(torch.rand(Hv, generator=g, device="cuda") * 15 + 1).to(dt),
                      linear_norm_w=ones(128), linear_out_proj=w(vd, hid))
        else:
            lw.update(wq=w(hid, 2 * qd), wk=w(hid, kvd), wv=w(hid, kvd), q_norm=ones(c["head_dim"]),
                      k_norm=ones(c["head_dim"]), wo=w(qd, hid))
        nbytes += sum(t.numel() * 2 for k, t in lw.items() if k != "is_linear")
        layers.append(lw)
    emb, fnorm, head = w(V, hid, std=1.0), ones(hid), w(hid, V)
    weight_bytes = nbytes + (emb[0].numel() + fnorm.numel() + head.numel()) * 2  # one embedding row is read
    model = q.ops.Model.from_weights(dict(c, layer_types=None), QIC_DTYPE_BF16, emb, fnorm, head, layers)
    n_full = sum(1 for k in layer_types if k == 0)
    kv_bytes = n_full * 2 * (context + 1) * kvd * 2
    state_bytes = (len(layer_types) - n_full) * GdnConfig(num_k_heads=16, num_v_heads=32).state_bytes()
    # the caches up to `context` hold whatever the first steps wrote; the timed step
    # appends at `context` and attends over context + 1 tokens
    model.set_position(1, context)
    torch.cuda.synchronize()
    logits = torch.empty(V, dtype=dt).pin_memory()

    def e2e():
        return model.decode(1, context, logits)

    return dict(model=model, bytes=weight_bytes + kv_bytes + state_bytes, weight_bytes=weight_bytes,
                kv_bytes=kv_bytes, state_bytes=state_bytes, e2e=e2e, keep=(layers, emb, fnorm, head),
                config={"model": "Qwen3.5-4B-shaped hybrid, random bf16 weights", "layers": len(layer_types),
                        "full_attention_layers": n_full, "context": context, "hidden": hid, "intermediate": inter,
                        "vocab": V, "heads": f"{c['num_heads']}/{c['num_kv_heads']} x {c['head_dim']}",
                        "launches_per_step": 2 + 5 * len(layer_types) + 1})


def measure_decode_step(wl, steps, warmup, peaks):
    """Device time of the captured step (CUDA events around `steps` replays) and the
    end-to-end qic_model_decode (token copy, replay, greedy token and logits back,
    synchronised), per token."""
    m = wl["model"]
    for _ in range(warmup):
        m.step_graph()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        m.step_graph()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / steps
    for _ in range(warmup):
        wl["e2e"]()
    t0 = time.perf_counter()
    for _ in range(steps):
        wl["e2e"]()
    ms_e2e = (time.perf_counter() - t0) * 1000 / steps
    gbs = wl["bytes"] / (ms * 1e-3) / 1e9
    return {"tokens_per_s": round(1000.0 / ms, 1), "ms_per_token": round(ms, 4), "value": round(gbs, 1),
            "unit": "GB/s", "frac_of_hbm": round(gbs / peaks["hbm_gbs"], 4), "bytes_per_token": int(wl["bytes"]),
            "weight_bytes": int(wl["weight_bytes"]), "kv_bytes": int(wl["kv_bytes"]),
            "state_bytes": int(wl["state_bytes"]),
            "e2e": {"tokens_per_s": round(1000.0 / ms_e2e, 1), "ms_per_token": round(ms_e2e, 4),
                    "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 8 + 2 * wl["config"]["vocab"],
                    "what": "qic_model_decode: token and position copied in, the step's graph, greedy token and "
                            "logits copied out, synchronised (host wall clock)"},
            "config": wl["config"]}


def decode_step_vs_reference(steps=20, warmup=3, context=512):
    """The reference's own decode loop against this library's runner on the same
    synthetic qmini v4 file (Qwen3.5-4B widths, 8 layers: 6 GatedDeltaNet and 2 gated
    full attention; vocab 32768; fp16, the format's type): QwenMiniModel::decode_next
    (src/model.cpp:823-845, built unmodified into oracle/_ref) and qic_model_decode,
    each timed end to end per token (host wall clock, synchronised) at position
    `context` after a prefill of `context` tokens."""
    import tempfile

    import qwenincuda_b200 as q
    from oracle.oracle import RefQwenModel
    from oracle.qmini_writer import QminiConfig, write_qmini

    cfg = QminiConfig(vocab_size=32768, hidden_size=2560, intermediate_size=9216, num_heads=16, num_kv_heads=4,
                      head_dim=256, linear_num_key_heads=16, linear_num_value_heads=32, max_seq_len=context + steps
                      + warmup + 8, layer_types=[1, 1, 1, 0, 1, 1, 1, 0])
    with tempfile.TemporaryDirectory() as d:
        path = Path(d) / "synth_qwen35_8l.qmini"
        write_qmini(path, cfg, seed=3)
        res = {}
        for name, make in (("reference_decode_next", lambda: RefQwenModel(path)),
                           ("qic_model_decode", lambda: q.ops.Model.load(path))):
            m = make()
            try:
                for pos in range(context):  # prefill, token by token as the reference's generate does
                    m.decode(pos % cfg.vocab_size, pos)
                pos = context
                for _ in range(warmup):
                    m.decode(1, pos)
                    pos += 1
                torch.cuda.synchronize()
                t0 = time.perf_counter()
                for _ in range(steps):
                    m.decode(1, pos)
                    pos += 1
                ms = (time.perf_counter() - t0) * 1000 / steps
            finally:
                m.close()
            res[name] = {"ms_per_token": round(ms, 3), "tokens_per_s": round(1000 / ms, 1)}
    res["speedup"] = round(res["reference_decode_next"]["ms_per_token"] / res["qic_model_decode"]["ms_per_token"], 1)
    res["what"] = ("same synthetic qmini v4 file (Qwen3.5-4B widths, 8 layers, vocab 32768, fp16), position "
                   f"{context}; end to end per token, host wall clock")
    return res


def time_eager(fn, steps, warmup, world):
    """ms per call of fn (no graph): used for the NCCL all-gather path."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        fn()
    e.record()
    torch.cuda.synchronize()
    barrier(world)
    return max_over_ranks(s.elapsed_time(e) / steps, world)


def sum_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def partitioned_summary(wl, args, world, local, peaks):
    """Measures a partitioned workload (every rank its own share) and returns the
    whole-job numbers: total algorithmic bytes of all ranks / the slowest rank's time."""
    ms, ms_e2e, clocks = measure(wl, args, world, local)
    total = sum_over_ranks(float(wl["bytes"]), world)
    per_rank_gbs = wl["bytes"] / (ms * 1e-3) / 1e9
    res = {"value": round(total / (ms * 1e-3) / 1e9, 2), "unit": "GB/s", "ms_per_step": round(ms, 4),
           "us_per_step": round(ms * 1000, 2), "us_per_layer": round(ms * 1000 / wl["launches"], 2),
           "bytes_total": int(total),
           "e2e": {"value": round(total / (ms_e2e * 1e-3) / 1e9, 2), "unit": "GB/s",
                   "h2d_bytes_per_step": wl["e2e"][1], "d2h_bytes_per_step": wl["e2e"][2]},
           "rank0_frac_of_hbm": round(per_rank_gbs / peaks["hbm_gbs"], 4), "scaling": "strong",
           "config": wl["config"]}
    if wl.get("allgather") is not None:
        ms_ag = time_eager(wl["allgather"], args.steps, args.warmup, world)
        res["allgather_nccl_path"] = {"value": round(total / (ms_ag * 1e-3) / 1e9, 2), "unit": "GB/s",
                                      "us_per_step": round(ms_ag * 1000, 2),
                                      "us_per_layer": round(ms_ag * 1000 / wl["launches"], 2),
                                      "what": "partial kernel + NCCL all_gather_into_tensor + merge kernel"}
    return res, ms, ms_e2e, clocks


def measure(wl, args, world, local):
    g = capture(wl["step"])
    sampler = ClockSampler(local)
    ms = time_graph(g, args.steps, args.warmup, world, sampler)
    status = wl["status"]()
    if status != 0:
        raise RuntimeError(f"device status {status} after the timed steps")
    del g
    ge = capture(wl["e2e"][0])
    ms_e2e = time_graph(ge, args.steps, args.warmup, world)
    del ge
    torch.cuda.synchronize()
    return ms, ms_e2e, sampler.summary()


# ---------------------------------------------------------------------------
# CPU baseline and the reference arm
# ---------------------------------------------------------------------------
def _timed_loop(fn, budget_s):
    """Runs fn until budget_s seconds have passed; returns (calls, seconds)."""
    n = 0
    t0 = time.perf_counter()
    while True:
        fn()
        n += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            return n, el


def cpu_baseline(workload, budget_s=6.0):
    """The oracle (C restatement of the reference's path, OpenMP over heads) on a
    bounded sample of `workload` on this host's cores, in the workload's metric.
    Attention: whole layers at the workload's S. GatedDeltaNet: whole steps (the
    reference runs this block as a host loop, src/model.cpp:692-793). Pair: both.
    Batch: whole steps over the first sequences of the seeded length list."""
    from oracle.oracle import Oracle
    from qwenincuda_b200.workloads import (CONFIGS, BatchConfig, GdnConfig, batched_bytes, make_attention_inputs,
                                           make_batched_inputs, make_gdn_inputs)

    orc = Oracle()
    # every host thread this process may run on (torchrun sets OMP_NUM_THREADS=1)
    orc.set_num_threads(len(os.sched_getaffinity(0)))
    threads = orc.num_threads()

    def attention_layer(cfg):
        inp = make_attention_inputs(cfg, paged=True, layers=1, device="cpu")
        H, Hkv, d, S = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, cfg.seq_len
        kc = inp.k_cache[0].view(-1, Hkv * d)
        vc = inp.v_cache[0].view(-1, Hkv * d)
        gate = inp.gate[0].flatten() if inp.gate is not None else None

        def run():
            o = orc.attention(inp.q[0].flatten(), kc, vc, H, Hkv, d, S, page_table=inp.page_table[0],
                              page_size=cfg.page_size)
            if gate is not None:
                orc.sigmoid_mul(o, gate)

        return run, cfg.kv_read_bytes() + cfg.append_bytes(), f"paged attention at S={S} (H={H}, Hkv={Hkv}, d={d})"

    def gdn_step():
        """The reference's own step (its host loop with its device copies, fp16 as it
        ships, one host thread) when oracle/_ref holds it and a GPU is present, else
        the oracle's restatement (OpenMP)."""
        from oracle.oracle import RefGatedDelta

        cfg = GdnConfig()
        what = f"GatedDeltaNet decode (Hk={cfg.num_k_heads}, Hv={cfg.num_v_heads}, d=128)"
        if RefGatedDelta.available() and torch.cuda.is_available():
            t = make_gdn_inputs(cfg, device="cpu", dtype=torch.float16)
            layer = RefGatedDelta().layer(conv_w=t["conv_w"], dt_bias=t["dt_bias"], a_log=t["a_log"],
                                          norm_w=t["norm_w"], conv_state=t["conv_state"],
                                          recurrent_state=t["recurrent_state"], num_k_heads=cfg.num_k_heads,
                                          num_v_heads=cfg.num_v_heads, conv_kernel=cfg.conv_kernel, eps=cfg.eps)
            layer.run(qkv=t["qkv"], z=t["z"], b=t["b"], a=t["a"])  # the step's projections, uploaded once
            keep.append(layer)
            return (layer.run, cfg.state_bytes(), "reference", 1,
                    what + " through the reference's run_linear_attention_block (src/model.cpp:656-795: cuBLAS "
                    "projections, 8 device-to-host copies, host loop, 1 copy back), fp16, one host thread")
        t = make_gdn_inputs(cfg, device="cpu")
        kw = {k: t[k] for k in ("qkv", "z", "b", "a", "conv_w", "dt_bias", "a_log", "norm_w", "conv_state",
                                "recurrent_state")}

        def run():
            orc.gated_delta(num_k_heads=cfg.num_k_heads, num_v_heads=cfg.num_v_heads, conv_kernel=cfg.conv_kernel,
                            eps=cfg.eps, **kw)

        return run, cfg.state_bytes(), "port", threads, what + " (oracle restatement)"

    keep = []  # reference layers held open while timed
    kind, cores = "port", threads
    if workload in ATTN_WORKLOADS:
        run, nbytes, what = attention_layer(CONFIGS[workload])
        unit_name = "layers"
    elif workload == "qwen35_gdn":
        run, nbytes, kind, cores, what = gdn_step()
        unit_name = "steps"
    elif workload == "qwen35_pair":
        g_run, g_bytes, g_kind, _, g_what = gdn_step()
        a_run, a_bytes, a_what = attention_layer(CONFIGS["qwen35_gated_s32769"])

        def run():
            g_run()
            a_run()

        nbytes, what, unit_name = g_bytes + a_bytes, f"{g_what}, then gated {a_what} (oracle)", "steps"
        kind = "reference + port" if g_kind == "reference" else "port"
    elif workload == "qwen3_8b_batch64":
        cfg = BatchConfig()
        lens = cfg.seq_lens()[:4]
        # a pool just large enough for the sample (the full pool is 4.5 GB)
        cfg = dataclasses.replace(cfg, pool_tokens=sum(lens) + len(lens) * cfg.page_size)
        inp = make_batched_inputs(cfg, device="cpu", seq_lens=lens)
        qs = inp["q"].view(len(lens), -1)
        kc = inp["k_cache"].view(-1, cfg.kv_dim)
        vc = inp["v_cache"].view(-1, cfg.kv_dim)
        sl = torch.tensor(lens, dtype=torch.int32)

        def run():
            orc.batched_attention(qs, kc, vc, inp["block_tables"], sl, cfg.page_size, cfg.num_heads,
                                  cfg.num_kv_heads, cfg.head_dim)

        nbytes = batched_bytes(lens, cfg.kv_dim)
        what, unit_name = f"batched paged attention over the first {len(lens)} of the 64 sequences ({sum(lens)} tokens)", "steps"
    else:
        raise SystemExit(f"unknown workload {workload}")
    n, el = _timed_loop(run, budget_s)
    for layer in keep:
        layer.close()
    per = el / n
    return {"value": round(nbytes / per / 1e9, 3), "unit": "GB/s", f"us_per_{unit_name[:-1]}": round(per * 1e6, 1),
            "cores": cores, "kind": kind, "sample": f"{n} {unit_name} of {what} in {el:.1f} s"}


def reference_gpu(cfg, layers, steps, warmup):
    """The reference's own kernels (src/kernels.cu built for sm_100a with
    --use_fast_math, bf16 instance) driving the per-layer sequence of
    src/model.cpp:628-650: (gated layers) split of the q/gate projection, head-norm
    q and k, RoPE q and k, two row copies, paged attention, (gated layers) the
    sigmoid gate."""
    from oracle.oracle import RefKernels, _p
    from qwenincuda_b200.workloads import make_attention_inputs

    dtype = torch.bfloat16
    ref = RefKernels(dtype)
    inp = make_attention_inputs(cfg, paged=True, layers=layers)
    H, Hkv, d, S, P, pos = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, cfg.seq_len, cfg.page_size, cfg.position
    lib = ref.lib
    qbuf = torch.empty(H * d, device="cuda", dtype=dtype)
    gbuf = torch.empty(H * d, device="cuda", dtype=dtype)
    kbuf = torch.empty(Hkv * d, device="cuda", dtype=dtype)
    slots = [int(inp.page_table[i][pos // P]) * P + pos % P for i in range(layers)]
    qg = torch.cat([inp.q, inp.gate], dim=2).contiguous() if inp.gate is not None else None

    def step():
        for i in range(layers):
            if qg is not None:
                lib.qicref_split_q_gate(_p(qg[i]), H, d, _p(qbuf), _p(gbuf))
            else:
                qbuf.copy_(inp.q[i].flatten())
            kbuf.copy_(inp.k_new[i].flatten())
            lib.qicref_head_rmsnorm(_p(qbuf), _p(inp.q_norm_w), H, d, cfg.eps, _p(qbuf))
            lib.qicref_head_rmsnorm(_p(kbuf), _p(inp.k_norm_w), Hkv, d, cfg.eps, _p(kbuf))
            lib.qicref_rope_inplace(_p(qbuf), H, d, pos, cfg.rope_theta)
            lib.qicref_rope_inplace(_p(kbuf), Hkv, d, pos, cfg.rope_theta)
            kc = inp.k_cache[i].view(-1, Hkv * d)
            vc = inp.v_cache[i].view(-1, Hkv * d)
            lib.qicref_copy_row(_p(kc), _p(kbuf), slots[i], Hkv * d)
            lib.qicref_copy_row(_p(vc), _p(inp.v_new[i].flatten()), slots[i], Hkv * d)
            lib.qicref_paged_attention(_p(qbuf), _p(kc), _p(vc), _p(inp.page_table[i]), P, H, Hkv, d, S,
                                       _p(inp.out[i]))
            if qg is not None:
                lib.qicref_sigmoid_mul_inplace(_p(inp.out[i]), _p(gbuf), H * d)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(steps):
        step()
    e.record()
    torch.cuda.synchronize()
    per_layer_us = s.elapsed_time(e) / steps * 1000 / layers
    lb = cfg.kv_read_bytes() + cfg.append_bytes()
    return {"value": round(lb / (per_layer_us * 1e-6) / 1e9, 3), "unit": "GB/s", "us_per_layer": round(per_layer_us, 1),
            "layers_timed": layers,
            "build": "src/kernels.cu unmodified, nvcc -gencode arch=compute_100a,code=sm_100a --use_fast_math, bf16"}


def line_config(workload, world):
    """The JSON line's `config`: what the workload is, identical in both arms (this
    library's and the reference's) for the same workload and N. Details that depend on
    the run (plan items, per-rank shares) go under the line's `details` key instead."""
    from qwenincuda_b200.workloads import CONFIGS, BatchConfig, GdnConfig, batched_bytes

    if workload in ATTN_WORKLOADS:
        cfg = CONFIGS[workload]
        cp = workload == "qwen3_8b_s131073" and world > 1
        layers = 2 if cp else cfg.layers
        c = {"layout": "paged", "page_size": cfg.page_size, "layers": layers, "seq_len": cfg.seq_len,
             "num_heads": cfg.num_heads, "num_kv_heads": cfg.num_kv_heads, "head_dim": cfg.head_dim,
             "gate": "interleaved q/gate projection" if cfg.gate else False}
        rank_bytes = (cfg.kv_read_bytes() + cfg.append_bytes()) * layers // (world if cp else 1)
        par = f"context-parallel{world}" if cp else (f"replicas{world}" if world > 1 else "single")
    elif workload == "qwen35_gdn":
        g = GdnConfig()
        c = {"layers": GDN_STACK_LAYERS, "num_k_heads": g.num_k_heads, "num_v_heads": g.num_v_heads,
             "k_head_dim": g.k_head_dim, "v_head_dim": g.v_head_dim, "conv_dim": g.conv_dim,
             "conv_kernel": g.conv_kernel, "state": "fp32, resident on the device, one per layer"}
        rank_bytes = g.state_bytes() * GDN_STACK_LAYERS
        par = f"replicas{world}" if world > 1 else "single"
    elif workload == "qwen35_pair":
        att = CONFIGS["qwen35_gated_s32769"]
        c = {"layers": "GatedDeltaNet + gated attention (16/4 heads, d=256, S=32769, paged)"}
        rank_bytes = GdnConfig().state_bytes() + att.kv_read_bytes() + att.append_bytes()
        par = f"replicas{world}" if world > 1 else "single"
    elif workload == "gemv_qwen3_8b":
        c = {"layers": 4, "hidden": 4096, "intermediate": 12288, "q_out": 4096, "kv_out": 1024,
             "launches_per_layer": 4}
        rank_bytes = 4 * 386 << 20
        par = f"replicas{world}" if world > 1 else "single"
    elif workload == "qwen3_8b_batch64":
        b = BatchConfig()
        c = {"batch": b.batch, "seq_lens": f"U[{b.min_len},{b.max_len}]+1, seed {b.seed}", "page_size": b.page_size,
             "pool_tokens": b.pool_tokens, "num_heads": b.num_heads, "num_kv_heads": b.num_kv_heads,
             "head_dim": b.head_dim}
        rank_bytes = batched_bytes(b.seq_lens(), b.kv_dim) // world
        par = f"partitioned{world}" if world > 1 else "single"
    else:
        raise SystemExit(f"unknown workload {workload}")
    l2 = ("step inputs larger than the 126 MB L2" if rank_bytes > (126 << 20)
          else "step smaller than L2; consecutive steps re-read it")
    return {"workload": workload, "parallelism": par, "l2": l2, **c}


def run_reference_arm(args, world, rank):
    """The reference's own implementation of the path on this host's cores, on the
    same workload, metric and unit as this library's line (rank 0 only). For the
    attention workloads the reference's kernels built for sm_100a are also timed on
    the GPU, as extra information."""
    from qwenincuda_b200.workloads import CONFIGS, BatchConfig, GdnConfig, batched_bytes

    if rank != 0:
        return
    name = args.workload
    config = line_config(name, world)
    cb = cpu_baseline(name, budget_s=max(2.0, min(20.0, 0.5 * args.steps)))
    layers = 1
    if name in ATTN_WORKLOADS:
        cfg = CONFIGS[name]
        layers = config["layers"]
        step_bytes = (cfg.kv_read_bytes() + cfg.append_bytes()) * layers
    elif name == "qwen35_gdn":
        layers = GDN_STACK_LAYERS
        step_bytes = GdnConfig().state_bytes() * layers
    elif name == "qwen35_pair":
        att = CONFIGS["qwen35_gated_s32769"]
        step_bytes = GdnConfig().state_bytes() + att.kv_read_bytes() + att.append_bytes()
    else:
        b = BatchConfig()
        step_bytes = batched_bytes(b.seq_lens(), b.kv_dim)
    # the whole step of the workload at the sample's rate
    ms_step = step_bytes / (cb["value"] * 1e9) * 1e3
    line = {
        "impl": "reference",
        "metric": "GatedDeltaNet state GB/s" if name == "qwen35_gdn" else "decode-attn KV-read GB/s",
        "value": cb["value"], "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms_step, 3), "us_per_layer": round(ms_step * 1000 / layers, 1),
        "higher_is_better": True, "scaling": "strong" if world > 1 and name in ("qwen3_8b_s131073", "qwen3_8b_batch64") else "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": config,
        "cpu_baseline": cb,
        "e2e": {"value": cb["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if name in ATTN_WORKLOADS:
        try:
            line["reference_kernels_sm100a"] = reference_gpu(CONFIGS[name], layers=min(2, layers),
                                                             steps=max(1, min(5, args.steps // 20)), warmup=1)
        except Exception as exc:  # extra information only
            line["reference_kernels_sm100a"] = {"unavailable": str(exc)[:200]}
    print(json.dumps(line), flush=True)


def summarize(wl, ms, ms_e2e, peaks, kernel_ms=None, workload=None):
    """One workload's figures on one GPU: GB/s, us per layer, the roofline fraction of
    its dominant kernel, and the end-to-end figure."""
    per_launch_ms = ms / wl["launches"]
    achieved = wl["bytes_per_launch"] / ((kernel_ms if kernel_ms is not None else per_launch_ms) * 1e-3) / 1e9
    return {"value": round(wl["bytes"] / (ms * 1e-3) / 1e9, 2), "unit": "GB/s", "ms_per_step": round(ms, 4),
            "us_per_layer": round(per_launch_ms * 1000, 3),
            "roofline": {"bound": "hbm", "kernel": wl["kernel"], "achieved": round(achieved, 1),
                         "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                         "frac_of_8tbs": round(achieved / 8000.0, 4), "bytes_per_launch": wl["bytes_per_launch"],
                         "traffic": measured_traffic(workload) if workload else None},
            "e2e": {"value": round(wl["bytes"] / (ms_e2e * 1e-3) / 1e9, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": wl["e2e"][1], "d2h_bytes_per_step": wl["e2e"][2]},
            "config": wl["config"]}


def eager_e2e(wl, args):
    """The workload's end-to-end step without a CUDA graph: the host-to-device copy of
    the step's inputs from pinned memory, one C-ABI call per layer as a caller's decode
    loop makes them (argument checks, TMA descriptors and the launch on the host, every
    call), and the device-to-host copy of the outputs; timed with CUDA events. Also the
    host time to issue one call (the loop runs ahead of the GPU)."""
    fn = wl["e2e"][0]
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.steps):
        fn()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / args.steps
    # host time to issue a call, from a burst short enough not to fill the launch queue
    # (a longer loop waits for the GPU and measures it instead)
    burst = max(1, 256 // wl["launches"])
    t0 = time.perf_counter()
    for _ in range(burst):
        fn()
    host_s = time.perf_counter() - t0
    torch.cuda.synchronize()
    return {"value": round(wl["bytes"] / (ms * 1e-3) / 1e9, 2), "unit": "GB/s", "ms_per_step": round(ms, 4),
            "h2d_bytes_per_step": wl["e2e"][1], "d2h_bytes_per_step": wl["e2e"][2],
            "host_us_per_call": round(host_s * 1e6 / (burst * wl["launches"]), 2),
            "what": "eager: pinned H2D copy, one qic_decode_attention call per layer, D2H copy; no CUDA graph"}


def strong_scaling_key(make, args, world, rank, local, peaks):
    """A partitioned configuration at this N (every rank its share, whole-job bytes /
    the slowest rank's time) and, measured in the same run with rank 0 alone, the whole
    job on one GPU: the speed-up over one GPU and the efficiency (speed-up / N)."""
    ms1 = None
    if world > 1:
        if rank == 0:
            wl1 = make(1, 0, False)
            ms1, _, _ = measure(wl1, args, 1, local)
            del wl1
            torch.cuda.empty_cache()
        barrier(world)
    wl = make(world, rank, True)
    res, ms, _, _ = partitioned_summary(wl, args, world, local, peaks)
    del wl
    torch.cuda.empty_cache()
    if ms1 is None:
        ms1 = ms
    res["n1_us_per_step"] = round(ms1 * 1000, 2)
    res["speedup_vs_n1"] = round(ms1 / ms, 3)
    res["efficiency"] = round(ms1 / ms / world, 3)
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="qwen3_8b_s8192")
    ap.add_argument("--layers", type=int, default=None, help="override the layer count (profiling runs only)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="only the requested workload (profiling runs)")
    ap.add_argument("--splits", type=int, default=0, help="attention splits per kv head (tuning runs; 0 = chosen)")
    ap.add_argument("--seq-len", type=int, default=0, help="attended tokens of an attention workload (tuning runs)")
    args = ap.parse_args()
    world, rank, local = dist_setup()
    if args.impl == "reference":
        run_reference_arm(args, world, rank)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return

    peaks = load_peaks()
    if args.workload == "qwen35_4b_decode_step" and args.no_extra and world == 1:
        # profiling runs of the decode-step runner alone: one line of its figures
        w3 = decode_step_workload()
        r = measure_decode_step(w3, max(10, args.steps // 4), args.warmup, peaks)
        w3["model"].close()
        print(json.dumps({"workload": args.workload, **r}), flush=True)
        return
    extra = {}
    partitioned_mode = world > 1 and args.workload in ("qwen3_8b_s131073", "qwen3_8b_batch64")
    if args.workload == "qwen3_8b_s131073" and world > 1:
        # the long sequence split across the ranks, partials exchanged in-kernel
        wl = cp_workload(world, rank)
        res, ms, ms_e2e, clocks = partitioned_summary(wl, args, world, local, peaks)
        if "allgather_nccl_path" in res:
            extra["allgather_nccl_path"] = res["allgather_nccl_path"]
    elif args.workload in ATTN_WORKLOADS:
        wl = attention_workload(args.workload, "paged", args.layers, args.splits, args.seq_len)
        ms, ms_e2e, clocks = measure(wl, args, world, local)
        if world == 1 and not args.no_extra:
            extra["e2e_eager"] = eager_e2e(wl, args)
        if not args.no_extra:
            wl_c = attention_workload(args.workload, "contiguous", args.layers)
            ms_c, _, _ = measure(wl_c, args, world, local)
            extra["contiguous"] = {"value": round(world * wl_c["bytes"] / (ms_c * 1e-3) / 1e9, 2), "unit": "GB/s",
                                   "us_per_layer": round(ms_c / wl_c["launches"] * 1000, 3)}
            del wl_c
    elif args.workload == "qwen35_gdn":
        wl = gdn_workload()
        ms, ms_e2e, clocks = measure(wl, args, world, local)
    elif args.workload == "qwen35_pair":
        wl = pair_workload()
        ms, ms_e2e, clocks = measure(wl, args, world, local)
    elif args.workload == "qwen3_8b_batch64":
        wl = batched_workload(world, rank)
        ms, ms_e2e, clocks = measure(wl, args, world, local)
    elif args.workload == "gemv_qwen3_8b" and args.no_extra:
        wl = gemv_workload(args.layers or 4)  # profiling runs of the projections alone
        ms, ms_e2e, clocks = measure(wl, args, world, local)
    else:
        raise SystemExit(f"unknown workload {args.workload}")

    kernel_ms = None
    if wl.get("kernel_step") is not None:
        gk = capture(wl["kernel_step"])
        kernel_ms = time_graph(gk, args.steps, args.warmup, world)
        del gk
    step_bytes = wl["bytes"]
    if partitioned_mode:
        # every rank processed its own share: whole-job bytes / the slowest rank's time
        total_bytes = sum_over_ranks(float(step_bytes), world)
        scaling = "strong"
    else:
        total_bytes = float(world * step_bytes)
        scaling = "weak"
    value = total_bytes / (ms * 1e-3) / 1e9
    per_launch_ms = ms / wl["launches"]
    achieved = wl["bytes_per_launch"] / ((kernel_ms if kernel_ms is not None else per_launch_ms) * 1e-3) / 1e9
    traffic = measured_traffic(args.workload) if world == 1 else None
    details = wl["config"]
    h2d, d2h, kernel_name, launches, bpl = wl["e2e"][1], wl["e2e"][2], wl["kernel"], wl["launches"], wl["bytes_per_launch"]
    del wl
    torch.cuda.empty_cache()
    if args.workload == "qwen3_8b_s8192" and not args.no_extra:
        # the partitioned configurations at this N (N = 1 included), each with its own
        # one-GPU baseline, speed-up and efficiency
        extra["context_parallel_qwen3_8b_s131073"] = strong_scaling_key(
            lambda w, r, ag: cp_workload(w, r, with_allgather=ag), args, world, rank, local, peaks)
        extra["partitioned_qwen3_8b_batch64"] = strong_scaling_key(
            lambda w, r, ag: batched_workload(w, r), args, world, rank, local, peaks)
        if world == 1:
            # the other single-GPU configurations: the 32K gated layer (the 70%-of-HBM
            # target), the short Qwen3-0.6B layer and the GatedDeltaNet step
            for name in ("qwen35_gated_s32769", "qwen3_0p6b_s1025"):
                w2 = attention_workload(name, "paged")
                m2, e2, _ = measure(w2, args, 1, local)
                extra[name] = summarize(w2, m2, e2, peaks, workload=name)
                del w2
                torch.cuda.empty_cache()
            w2 = gdn_workload()
            m2, e2, _ = measure(w2, args, 1, local)
            extra["qwen35_gdn"] = summarize(w2, m2, e2, peaks, workload="qwen35_gdn")
            del w2
            torch.cuda.empty_cache()
            # the projections around the attention of the same model (weight bytes)
            w2 = gemv_workload()
            m2, e2, _ = measure(w2, args, 1, local)
            extra["gemv_qwen3_8b"] = summarize(w2, m2, e2, peaks, workload="gemv_qwen3_8b")
            extra["gemv_qwen3_8b"]["us_per_model_layer"] = round(m2 * 1000 / w2["config"]["layers"], 2)
            gl = capture(w2["library_step"])
            ml = time_graph(gl, args.steps, args.warmup, 1)
            del gl
            # a whole decode step of a hybrid model through the decode-step runner
            w3 = decode_step_workload()
            extra["decode_step_qwen35_4b"] = measure_decode_step(w3, max(10, args.steps // 4), args.warmup, peaks)
            w3["model"].close()
            del w3
            torch.cuda.empty_cache()
            try:  # the reference's own decode loop on the same file (its build lives in oracle/_ref)
                extra["decode_step_qwen35_4b"]["vs_reference_decode_next"] = decode_step_vs_reference()
            except Exception as exc:  # extra information only
                extra["decode_step_qwen35_4b"]["vs_reference_decode_next"] = {"unavailable": str(exc)[:200]}
            extra["gemv_qwen3_8b"]["torch_cublas_unfused"] = {
                "value": round(w2["bytes"] / (ml * 1e-3) / 1e9, 2), "unit": "GB/s",
                "us_per_model_layer": round(ml * 1000 / w2["config"]["layers"], 2),
                "what": "the same products as torch.matmul (cuBLAS) calls with separate SiLU, multiply and adds"}
            del w2
            torch.cuda.empty_cache()
    line = {
        "metric": "decode-attn KV-read GB/s" if args.workload != "qwen35_gdn" else "GatedDeltaNet state GB/s",
        "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 4), "us_per_layer": round(per_launch_ms * 1000, 3), "higher_is_better": True,
        "scaling": scaling, "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": line_config(args.workload, world),
        "details": details,
        **extra,
        "e2e": {"value": round(total_bytes / (ms_e2e * 1e-3) / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(ms_e2e, 4)},
        "roofline": {"bound": "hbm", "kernel": kernel_name, "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4), "peak_source": peaks["source"],
                     "frac_of_8tbs": round(achieved / 8000.0, 4), "bytes_per_launch": bpl,
                     "launch_time": ("the kernel's launches timed on their own" if kernel_ms is not None
                                     else "step time / launches per step (includes launch gaps)")
                     + ("; rank 0's bytes over the slowest rank's time" if partitioned_mode else ""),
                     "traffic": traffic},
        "gpu_launches": launches * args.steps,
        "clocks": clocks,
    }
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args.workload)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        torch.cuda.synchronize()
        dist.barrier()  # no rank unmaps an exchange buffer a peer may still write
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
