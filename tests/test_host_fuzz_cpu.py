"""CPU fuzz (hypothesis) of the host-only entry points of libqic: the launch-shape
query, the batched-decode planner and the size helpers. On any arguments, lengths up
to 2^31-1 included, they return a documented status and never crash; on success their
results satisfy the launch invariants the kernels rely on."""
import ctypes

from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

from qwenincuda_b200 import abi

STATUSES = {0, 1, 2}  # QIC_SUCCESS, QIC_ERROR_INVALID_VALUE, QIC_ERROR_NOT_SUPPORTED
lengths = st.one_of(st.integers(-5, 70000), st.integers(abi.QIC_MAX_SEQ_LEN - 40, 2**31 - 1))
SETTINGS = dict(max_examples=300, deadline=None, suppress_health_check=[HealthCheck.too_slow])


@settings(**SETTINGS)
@given(H=st.integers(-4, 80), Hkv=st.integers(-2, 20), d=st.sampled_from([0, 32, 64, 96, 128, 256, 512]),
       S=lengths, pdl=st.booleans(), ws=st.booleans(), splits=st.integers(-3, 300), cluster=st.integers(-2, 20),
       dtype=st.sampled_from([0, 1, 2]))
def test_launch_shape_fuzz(H, Hkv, d, S, pdl, ws, splits, cluster, dtype):
    a = abi.DecodeArgs()
    a.dtype, a.num_heads, a.num_kv_heads, a.head_dim, a.seq_len = dtype, H, Hkv, d, S
    a.flags = abi.QIC_PDL if pdl else 0
    a.workspace = 16 if ws else None
    a.num_splits, a.cluster_size = splits, cluster
    n, c = ctypes.c_int(-1), ctypes.c_int(-1)
    rc = abi.lib().qic_decode_launch_shape(ctypes.byref(a), ctypes.byref(n), ctypes.byref(c))
    assert rc in STATUSES
    if rc == 0:
        assert 0 < S <= abi.QIC_MAX_SEQ_LEN or (S == 0 and (n.value, c.value) == (0, 0))
        if S > 0:
            assert 1 <= c.value <= 16 and n.value % c.value == 0 and 1 <= n.value <= 256
            if not ws:
                assert n.value == c.value


@settings(**SETTINGS)
@given(lens=st.lists(lengths, min_size=0, max_size=40), H=st.integers(-2, 64), Hkv=st.integers(-1, 16),
       d=st.sampled_from([0, 64, 96, 128, 256]), target=st.integers(-5, 100000))
def test_batch_plan_fuzz(lens, H, Hkv, d, target):
    L = abi.lib()
    arr = (ctypes.c_int32 * max(1, len(lens)))(*lens)
    items = ctypes.c_int(-1)
    wsb = ctypes.c_size_t(0)
    rc = L.qic_batch_plan(ctypes.cast(arr, ctypes.c_void_p), len(lens), H, Hkv, d, target, None, 0,
                          ctypes.byref(items), ctypes.byref(wsb))
    assert rc in STATUSES
    if rc == 0:
        assert all(1 <= x <= abi.QIC_MAX_SEQ_LEN for x in lens) and len(lens) > 0
        assert items.value >= len(lens) * Hkv
        assert items.value <= len(lens) * Hkv * 256  # at most 256 items per (sequence, kv head)
        assert 256 + 8192 * 4 <= wsb.value < 1 << 50


@settings(**SETTINGS)
@given(H=st.integers(-4, 80), Hkv=st.integers(-2, 20), d=st.integers(-1, 600), S=lengths,
       world=st.integers(-1, 10))
def test_size_helpers_fuzz(H, Hkv, d, S, world):
    L = abi.lib()
    ws = L.qic_decode_workspace_bytes(H, Hkv, d, S)
    assert ws == 0 or ws >= 256 + 8192 * 4
    if ws:
        assert H > 0 and Hkv > 0 and 0 <= S <= abi.QIC_MAX_SEQ_LEN
    L.qic_partial_floats(H, Hkv, d)
    L.qic_cp_exchange_bytes(H, Hkv, d, world)
