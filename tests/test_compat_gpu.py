"""GPU: the kernels.cuh C++ surface exported by libqic.so (the drop-in for
src/model.cpp) against the reference's own fp16 kernels, through the exact mangled
symbols, including calls of different shapes that share the library-owned workspace."""
import ctypes

import pytest
import torch

import qwenincuda_b200 as q
from conftest import allclose_report, assert_in_reference_envelope
from oracle.oracle import RefKernels

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-3, 1e-2

SYMS = {
    "flash": "_Z22launch_flash_attentionPK6__halfS1_S1_iiiiPS_",
    "paged": "_Z22launch_paged_attentionPK6__halfS1_S1_PKiiiiiiPS_",
    "norm": "_Z19launch_head_rmsnormPK6__halfS1_iifPS_",
    "rope": "_Z19launch_rope_inplaceP6__halfiiif",
    "gate": "_Z26launch_sigmoid_mul_inplaceP6__halfPKS_i",
}


def _compat():
    L = q.lib()
    vp, i, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    fns = {k: getattr(L, v) for k, v in SYMS.items()}
    fns["flash"].argtypes = [vp, vp, vp, i, i, i, i, vp]
    fns["paged"].argtypes = [vp, vp, vp, vp, i, i, i, i, i, vp]
    fns["norm"].argtypes = [vp, vp, i, i, f, vp]
    fns["rope"].argtypes = [vp, i, i, i, f]
    fns["gate"].argtypes = [vp, vp, i]
    for fn in fns.values():
        fn.restype = None
    L.qic_compat_last_status.restype = ctypes.c_int
    return fns, L


def test_compat_attention_shapes_share_workspace():
    fns, L = _compat()
    ref = RefKernels(torch.float16)
    g = torch.Generator(device="cuda").manual_seed(3)
    shapes = [(16, 4, 256, 3000, True), (32, 8, 128, 8192, True), (16, 8, 128, 1025, False), (8, 8, 64, 33, True),
              (64, 8, 128, 777, False), (32, 8, 128, 4100, True)]
    for H, Hkv, d, S, paged in shapes:
        P = 16
        npages = (S + P - 1) // P
        qv = torch.randn(H * d, generator=g, device="cuda").half()
        kc = (torch.randn(npages * P, Hkv * d, generator=g, device="cuda") * 0.5).half()
        vc = (torch.randn(npages * P, Hkv * d, generator=g, device="cuda") * 0.5).half()
        table = torch.randperm(npages, generator=g, device="cuda").to(torch.int32)
        want = torch.empty(H * d, device="cuda", dtype=torch.float16)
        got = torch.full((H * d,), float("nan"), device="cuda", dtype=torch.float16)
        if paged:
            ref.paged_attention(qv, kc, vc, table, P, H, Hkv, d, S, want)
            torch.cuda.synchronize()
            fns["paged"](qv.data_ptr(), kc.data_ptr(), vc.data_ptr(), table.data_ptr(), P, H, Hkv, d, S, got.data_ptr())
        else:
            ref.flash_attention(qv, kc, vc, H, Hkv, d, S, want)
            torch.cuda.synchronize()
            fns["flash"](qv.data_ptr(), kc.data_ptr(), vc.data_ptr(), H, Hkv, d, S, got.data_ptr())
        torch.cuda.synchronize()
        assert L.qic_compat_last_status() == 0
        ok, err, idx = allclose_report(got, want, ATOL, RTOL)
        assert ok, f"{(H, Hkv, d, S, paged)}: max err {err} at {idx}"


def test_compat_norm_rope_gate_match_reference():
    fns, L = _compat()
    ref = RefKernels(torch.float16)
    g = torch.Generator(device="cuda").manual_seed(4)
    H, d = 32, 128
    x = torch.randn(H * d, generator=g, device="cuda").half()
    w = (1 + 0.1 * torch.randn(d, generator=g, device="cuda")).half()
    runs = []
    for _ in range(32):
        r = torch.empty_like(x)
        ref.head_rmsnorm(x, w, H, d, 1e-6, r)
        runs.append(r)
    got = torch.empty_like(x)
    fns["norm"](x.data_ptr(), w.data_ptr(), H, d, 1e-6, got.data_ptr())
    torch.cuda.synchronize()
    assert_in_reference_envelope(got, runs)
    want = got.clone()
    ref.rope_inplace(want, H, d, 5000, 1.0e6)
    fns["rope"](got.data_ptr(), H, d, 5000, 1.0e6)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    gate = torch.randn(H * d, generator=g, device="cuda").half()
    ref.sigmoid_mul_inplace(want, gate, H * d)
    fns["gate"](got.data_ptr(), gate.data_ptr(), H * d)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    assert L.qic_compat_last_status() == 0


def test_compat_decode_loop_allocates_once():
    """A decode loop through launch_paged_attention whose length grows from 1 to 8192
    tokens (the reference's decode_next, src/model.cpp:643-650) takes the shim's
    workspace on its first call and no device memory after it; the last call matches
    the reference's paged kernel."""
    fns, L = _compat()
    H, Hkv, d, P, S_max = 32, 8, 128, 16, 8192
    g = torch.Generator(device="cuda").manual_seed(5)
    npages = S_max // P
    qv = torch.randn(H * d, generator=g, device="cuda").half()
    kc = (torch.randn(npages * P, Hkv * d, generator=g, device="cuda") * 0.5).half()
    vc = (torch.randn(npages * P, Hkv * d, generator=g, device="cuda") * 0.5).half()
    table = torch.randperm(npages, generator=g, device="cuda").to(torch.int32)
    got = torch.empty(H * d, device="cuda", dtype=torch.float16)

    def call(S):
        fns["paged"](qv.data_ptr(), kc.data_ptr(), vc.data_ptr(), table.data_ptr(), P, H, Hkv, d, S, got.data_ptr())

    call(1)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for S in list(range(2, 300)) + list(range(300, S_max, 61)) + [S_max]:
        call(S)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    assert L.qic_compat_last_status() == 0
    want = torch.empty_like(got)
    RefKernels(torch.float16).paged_attention(qv, kc, vc, table, P, H, Hkv, d, S_max, want)
    ok, err, idx = allclose_report(got, want, ATOL, RTOL)
    assert ok, f"max err {err} at {idx}"
