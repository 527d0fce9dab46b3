"""CPU checks of the host-side launch planning.

* The batched-decode planner (qic_batch_plan): with an explicit CTA target it queries
  no device. Every (sequence, kv head) has its pipeline stages covered exactly once by
  items with consistent split indices; partial slots do not collide; items are ordered
  longest first; the workspace covers every slot; targets are respected where they can
  be.
* The single-sequence launch shape (qic_decode_launch_shape): the split rule, checked
  against the shapes a B200 runs (exact values with the no-device occupancy fallback)."""
import ctypes

import pytest

from qwenincuda_b200 import abi

ITEM_FIELDS = ("b", "kvh", "split", "nsplit", "st_lo", "st_hi", "seq_len", "part_base")


def _plan(lens, H, Hkv, d, target):
    L = abi.lib()
    arr = (ctypes.c_int32 * len(lens))(*lens)
    items = ctypes.c_int(0)
    wsb = ctypes.c_size_t(0)
    rc = L.qic_batch_plan(ctypes.cast(arr, ctypes.c_void_p), len(lens), H, Hkv, d, target, None, 0,
                          ctypes.byref(items), ctypes.byref(wsb))
    assert rc == 0
    buf = (ctypes.c_int32 * (8 * items.value))()
    n = items.value
    rc = L.qic_batch_plan(ctypes.cast(arr, ctypes.c_void_p), len(lens), H, Hkv, d, target,
                          ctypes.cast(buf, ctypes.c_void_p), n, ctypes.byref(items), ctypes.byref(wsb))
    assert rc == 0 and items.value == n
    plan = [dict(zip(ITEM_FIELDS, buf[8 * i:8 * i + 8])) for i in range(n)]
    return plan, int(wsb.value)


def _tok(d):
    return 16 if d > 128 else 32


@pytest.mark.parametrize("lens,H,Hkv,d", [
    ([1, 2, 33, 777, 2049, 3001], 32, 8, 128),
    ([32769, 1025, 17, 4096, 4097], 16, 4, 256),
    ([100] * 40, 16, 8, 64),
    ([131073], 32, 8, 128),
])
@pytest.mark.parametrize("target", [1, 7, 64, 444, 5000])
def test_plan_covers_every_stage_once(lens, H, Hkv, d, target):
    plan, ws_bytes = _plan(lens, H, Hkv, d, target)
    tok = _tok(d)
    G = H // Hkv
    pf = ((G * (d + 1)) + 3) & ~3
    cover = {}
    for it in plan:
        key = (it["b"], it["kvh"])
        assert 0 <= it["b"] < len(lens) and 0 <= it["kvh"] < Hkv
        assert it["seq_len"] == lens[it["b"]]
        assert 0 <= it["split"] < it["nsplit"]
        assert 0 <= it["st_lo"] < it["st_hi"]
        cover.setdefault(key, []).append(it)
    assert len(cover) == len(lens) * Hkv
    slots = set()
    for (b, kvh), its in cover.items():
        n_st = (lens[b] + tok - 1) // tok
        its.sort(key=lambda x: x["split"])
        assert [x["split"] for x in its] == list(range(len(its)))
        assert all(x["nsplit"] == len(its) for x in its)
        # contiguous ranges that partition [0, n_st)
        assert its[0]["st_lo"] == 0 and its[-1]["st_hi"] == n_st
        for a, c in zip(its, its[1:]):
            assert a["st_hi"] == c["st_lo"]
        if len(its) > 1:
            for x in its:
                slot = x["part_base"] + x["split"]
                assert slot not in slots
                slots.add(slot)
    # the workspace holds the header, the counters and every partial slot
    if slots:
        assert ws_bytes >= 256 + 8192 * 4 + (max(slots) + 1) * pf * 4
    # longest items first
    lengths = [it["st_hi"] - it["st_lo"] for it in plan]
    assert lengths == sorted(lengths, reverse=True)
    # the target is met unless one item per (sequence, kv head) already exceeds it
    assert len(plan) <= max(target, len(lens) * Hkv)


def test_plan_rejects_bad_arguments():
    L = abi.lib()
    items = ctypes.c_int(0)
    wsb = ctypes.c_size_t(0)
    arr = (ctypes.c_int32 * 2)(5, 0)
    assert L.qic_batch_plan(ctypes.cast(arr, ctypes.c_void_p), 2, 32, 8, 128, 8, None, 0, ctypes.byref(items),
                            ctypes.byref(wsb)) == 1  # an empty sequence
    arr = (ctypes.c_int32 * 1)(5)
    assert L.qic_batch_plan(ctypes.cast(arr, ctypes.c_void_p), 1, 32, 8, 96, 8, None, 0, ctypes.byref(items),
                            ctypes.byref(wsb)) == 2  # head_dim 96
    assert L.qic_batch_plan(ctypes.cast(arr, ctypes.c_void_p), 1, 32, 6, 128, 8, None, 0, ctypes.byref(items),
                            ctypes.byref(wsb)) == 1  # 32 % 6


# (head_dim, H, Hkv, S, pdl) -> (splits per kv head, CTAs per cluster), for a GPU
# holding three 128-thread CTAs per SM on 148 SMs (the host fallback when no device
# answers the occupancy query; a B200 reports the same: grid (40, 8) at S=8192)
SHAPES = {
    (128, 32, 8, 1025, True): (16, 16), (128, 32, 8, 2049, True): (16, 16), (128, 32, 8, 3073, True): (16, 16),
    (128, 32, 8, 4097, True): (16, 16), (128, 32, 8, 6145, True): (32, 8), (128, 32, 8, 8192, True): (40, 8),
    (128, 32, 8, 8192, False): (40, 8), (128, 32, 8, 131073, True): (40, 8), (128, 32, 8, 131073, False): (48, 8),
    (256, 16, 4, 2049, True): (16, 16), (256, 16, 4, 8193, True): (64, 8), (256, 16, 4, 32769, True): (88, 8),
    (128, 32, 8, 100, False): (4, 4), (128, 16, 8, 1, False): (1, 1),
    # one kv head: the wave (55 clusters of 8) exceeds the 256 splits a kv head may have
    (128, 8, 1, 131073, False): (256, 8), (128, 8, 1, 131073, True): (256, 8), (128, 8, 1, 40000, False): (208, 8),
}


@pytest.mark.parametrize("key", list(SHAPES), ids=lambda k: "d{}_h{}_kv{}_s{}_{}".format(*k))
def test_decode_launch_shape(key):
    """qic_decode_launch_shape: one wave of resident 8-CTA clusters (five sixths with
    QIC_PDL), about 6 (d=128) or 8 (d=256) stages per CTA below that but 16 CTAs once
    the stages exceed 8 CTAs' rings, one cluster per kv head up to 16 CTAs; never more
    splits than stages."""
    import torch

    import qwenincuda_b200 as q

    d, H, Hkv, S, pdl = key
    n, c = q.ops.decode_launch_shape(num_heads=H, num_kv_heads=Hkv, head_dim=d, seq_len=S, pdl=pdl)
    tok = _tok(d)
    assert 1 <= c <= 16 and n % c == 0 and n <= max(1, (S + tok - 1) // tok)
    if not torch.cuda.is_available():
        assert (n, c) == SHAPES[key]


def test_decode_launch_shape_fused_append_tail():
    """With a fused append whose token is alone in the last stage (S - 1 a multiple of
    the stage size) that stage is not copied: S=1025 at d=128 is 32 stages, which 8 CTAs'
    rings hold; S=1024 keeps all 32 stages either way."""
    import torch

    import qwenincuda_b200 as q

    shape = lambda **kw: q.ops.decode_launch_shape(num_heads=32, num_kv_heads=8, head_dim=128, pdl=True, **kw)
    if not torch.cuda.is_available():
        assert shape(seq_len=1025, fuse_append=True) == (8, 8)
        assert shape(seq_len=1025) == (16, 16)
        assert shape(seq_len=1024, fuse_append=True) == shape(seq_len=1024) == (8, 8)
        assert shape(seq_len=2049, fuse_append=True) == (16, 16)
    assert shape(seq_len=2, fuse_append=True) == (1, 1)


def test_decode_launch_shape_explicit_and_without_workspace():
    import qwenincuda_b200 as q

    shape = lambda **kw: q.ops.decode_launch_shape(num_heads=32, num_kv_heads=8, head_dim=128, **kw)
    assert shape(seq_len=8192, num_splits=24, cluster_size=8) == (24, 8)
    assert shape(seq_len=8192, num_splits=24, cluster_size=0) == (24, 12)  # largest cluster <= 16 dividing 24
    n, c = shape(seq_len=8192, workspace=False)
    assert n == c and n <= 16  # merged on chip only
    assert shape(seq_len=0) == (0, 0)
    with pytest.raises(q.QicError):
        shape(seq_len=100, cluster_size=17)
