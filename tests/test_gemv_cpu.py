"""CPU: qic_gemv refuses invalid arguments before touching a device (status codes of
include/qic.h), and the ctypes mirror of qic_gemv_args matches the C layout."""
import ctypes

import pytest
import qwenincuda_b200 as q
from qwenincuda_b200.abi import QIC_GEMV_RESIDUAL, QIC_GEMV_SWIGLU, GemvArgs


def _args(K=64, Ns=(64,), swiglu=False):
    """Arguments with made-up, well-aligned, non-overlapping addresses: every call
    below is refused before any address is used."""
    a = GemvArgs()
    a.dtype, a.in_dim, a.num_segments = 1, K, len(Ns)
    a.x = 0x100000
    a.flags = QIC_GEMV_SWIGLU if swiglu else 0
    for k, n in enumerate(Ns):
        a.seg[k].w = 0x1000000 * (k + 1)
        a.seg[k].out = 0x200000 + 0x10000 * k
        a.seg[k].out_dim = n
    return a, None


def _call(a):
    return q.lib().qic_gemv(ctypes.byref(a), None)


def test_layout():
    # 4 int32 + 2 pointers + float + int32 + 4 segments of (3 pointers + 2 int32) + status pointer
    assert ctypes.sizeof(GemvArgs) == 16 + 16 + 8 + 4 * 32 + 8


@pytest.mark.parametrize("mutate,status", [
    (lambda a: setattr(a, "x", None), 1),
    (lambda a: setattr(a, "in_dim", 0), 1),
    (lambda a: setattr(a, "num_segments", 0), 1),
    (lambda a: setattr(a, "num_segments", 5), 1),
    (lambda a: setattr(a, "flags", 1 << 10), 1),
    (lambda a: setattr(a, "splits", 17), 1),
    (lambda a: setattr(a, "dtype", 7), 1),
    (lambda a: setattr(a.seg[0], "out_dim", 12), 1),
    (lambda a: setattr(a.seg[0], "w", None), 1),
    (lambda a: setattr(a.seg[0], "w", a.seg[0].w + 2), 3),
    (lambda a: setattr(a, "flags", QIC_GEMV_SWIGLU), 1),          # SwiGLU needs two segments
    (lambda a: setattr(a, "flags", QIC_GEMV_RESIDUAL), 1),        # residual missing
    (lambda a: setattr(a, "flags", 1), 1),                         # RMSNorm without its weight
    (lambda a: setattr(a, "in_dim", 16 * 8192 + 1), 2),
])
def test_invalid_arguments(mutate, status):
    a, keep = _args()
    mutate(a)
    assert _call(a) == status


def test_input_overlapping_an_output_is_refused():
    a, _ = _args()
    a.seg[0].out = a.x  # every CTA reads x while others write out
    assert _call(a) == 1


def test_swiglu_pair_needs_equal_widths():
    a, keep = _args(Ns=(64, 128), swiglu=True)
    assert _call(a) == 1
