"""GPU: weight-streaming GEMV projections (qic_gemv) against the reference's own
projection code, compiled unchanged into oracle/_ref: QwenMiniModel::gemv (cuBLAS with
the reference's arguments, src/model.cpp:603-617), its run_ffn_block (src/model.cpp:
797-807) and its rmsnorm / swiglu / add kernels (src/kernels.cu); and against a plain
PyTorch fp32 product. Outputs within max-abs 2e-3 / rel 1e-2 (the 16-bit results of
two fp32 accumulations in different orders differ by a rounding step at most); the
kernel's own results are bit-identical call after call and with or without
programmatic dependent launch."""
import pytest
import torch

import qwenincuda_b200 as q
from conftest import allclose_report
from oracle.oracle import RefKernels, RefModel

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-3, 1e-2
DTYPES = [torch.bfloat16, torch.float16]


def _gen(seed):
    return torch.Generator(device="cuda").manual_seed(seed)


def _x(K, g, dtype):
    return torch.randn(K, generator=g, device="cuda").to(dtype)


def _w(K, N, g, dtype, std=0.02):
    return (torch.randn(K, N, generator=g, device="cuda") * std).to(dtype)


def _nan(N, dtype):
    return torch.full((N,), float("nan"), device="cuda", dtype=dtype)


SHAPES = [
    (4096, 4096),    # Qwen3-8B q / o projection
    (4096, 1024),    # k / v
    (12288, 4096),   # FFN down
    (4096, 12288),   # FFN gate / up
    (1024, 2048),    # Qwen3-0.6B q
    (1, 8),
    (7, 264),        # ragged last tile
    (100, 1000),
    (2560, 9728),
    (5000, 136),
]


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("K,N", SHAPES)
def test_gemv_vs_reference_gemv(dtype, K, N):
    g = _gen(K * 7 + N)
    x, W = _x(K, g, dtype), _w(K, N, g, dtype)
    got = _nan(N, dtype)
    q.gemv(x=x, weights=[W], outs=[got])
    want = torch.empty(N, device="cuda", dtype=dtype)
    RefModel(dtype).gemv(x, W, K, N, want)
    ok, err, idx = allclose_report(got, want, ATOL, RTOL)
    assert ok, f"vs reference gemv: max abs err {err} at {idx}"
    fp32 = (x.float() @ W.float()).to(dtype)
    ok, err, idx = allclose_report(got, fp32, ATOL, RTOL)
    assert ok, f"vs fp32 product: max abs err {err} at {idx}"


@pytest.mark.parametrize("dtype", DTYPES)
def test_fused_norm_qkv_one_launch(dtype):
    """RMSNorm of x then the q, k and v projections, one launch over three weight
    buffers, against the reference's launch_rmsnorm and three reference gemv calls
    (src/model.cpp:832, 627-631)."""
    K, eps = 4096, 1e-6
    g = _gen(31)
    x = _x(K, g, dtype)
    nw = (1.0 + 0.1 * torch.randn(K, generator=g, device="cuda")).to(dtype)
    Ws = [_w(K, n, g, dtype) for n in (8192, 1024, 1024)]  # gated q (q and gate interleaved), k, v
    outs = [_nan(w.shape[1], dtype) for w in Ws]
    q.gemv(x=x, weights=Ws, outs=outs, norm_w=nw, eps=eps)
    ref, rm = RefKernels(dtype), RefModel(dtype)
    xn = torch.empty_like(x)
    ref.rmsnorm(x, nw, K, eps, xn)
    for k, (w, got) in enumerate(zip(Ws, outs)):
        want = torch.empty(w.shape[1], device="cuda", dtype=dtype)
        rm.gemv(xn, w, K, w.shape[1], want)
        ok, err, idx = allclose_report(got, want, ATOL, RTOL)
        assert ok, f"segment {k}: max abs err {err} at {idx}"


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("hidden,inter", [(1024, 3072), (4096, 12288)])
def test_ffn_two_launches_vs_reference_ffn_block(dtype, hidden, inter):
    """The FFN block as two launches (norm + gate/up + SwiGLU; down + residual into x)
    against the reference's own run_ffn_block on the same x and weights. The block
    rounds to 16 bits four times (gate and up, SwiGLU, the down product, the residual
    sum), and the down product can be larger than the block's output (the residual
    cancels part of it): besides max-abs 2e-3 / rel 1e-2 of the output, an element may
    differ by two units in the last place of the larger of |output| and
    |output - x| (the down product)."""
    eps = 1e-6
    g = _gen(hidden + inter)
    x = _x(hidden, g, dtype)
    nw = (1.0 + 0.1 * torch.randn(hidden, generator=g, device="cuda")).to(dtype)
    wg, wu = _w(hidden, inter, g, dtype), _w(hidden, inter, g, dtype)
    wd = _w(inter, hidden, g, dtype)
    want = x.clone()
    RefModel(dtype).ffn_block(want, nw, wg, wu, wd, hidden, inter, eps)
    torch.cuda.synchronize()
    got = x.clone()
    h = _nan(inter, dtype)
    q.gemv(x=got, weights=[wg, wu], outs=[h], norm_w=nw, eps=eps, swiglu=True)
    q.gemv(x=h, weights=[wd], outs=[got], residuals=[got])
    torch.cuda.synchronize()
    w32, g32, x32 = want.float(), got.float(), x.float()
    mag = torch.maximum(w32.abs(), (w32 - x32).abs())
    mant = 7 if dtype == torch.bfloat16 else 10
    ulp = torch.exp2(torch.floor(torch.log2(mag.clamp_min(1e-30))) - mant)
    bound = ATOL + RTOL * w32.abs() + 2 * ulp
    diff = (g32 - w32).abs()
    assert not torch.isnan(g32).any()
    assert bool((diff <= bound).all()), f"max abs err {float(diff.max())} at {int(diff.argmax())}"
    # and most elements within the plain tolerance
    assert float(((diff > ATOL + RTOL * w32.abs()).float().mean())) < 0.01


@pytest.mark.parametrize("dtype", DTYPES)
def test_swiglu_and_residual_match_reference_kernels(dtype):
    """The fused epilogues against the reference kernels: SwiGLU of the 16-bit gate and
    up products (launch_swiglu) within tolerance (the pair's products are summed over
    four warps instead of eight, so a product can differ by a rounding step), and the
    residual add (launch_add_inplace) byte for byte from the same product."""
    K, N = 2048, 4096
    g = _gen(41)
    x = _x(K, g, dtype)
    wg, wu = _w(K, N, g, dtype), _w(K, N, g, dtype)
    gate, up, h = _nan(N, dtype), _nan(N, dtype), _nan(N, dtype)
    q.gemv(x=x, weights=[wg, wu], outs=[gate, up])  # plain products, two segments in one launch
    q.gemv(x=x, weights=[wg, wu], outs=[h], swiglu=True)
    ref = RefKernels(dtype)
    want = torch.empty_like(h)
    ref.swiglu(gate, up, N, want)
    ok, err, idx = allclose_report(h, want, ATOL, RTOL)
    assert ok, f"SwiGLU: max abs err {err} at {idx}"
    res = _x(N, g, dtype)
    y = res.clone()
    q.gemv(x=x, weights=[wg], outs=[y], residuals=[y], splits=1)
    p = _nan(N, dtype)
    q.gemv(x=x, weights=[wg], outs=[p], splits=1)
    ref.add_inplace(p, res, N)
    assert torch.equal(y.view(torch.int16), p.view(torch.int16))


@pytest.mark.parametrize("splits", [1, 2, 3, 5, 8, 16, 0])
def test_split_counts_agree(splits):
    K, N, dtype = 4096, 3072, torch.bfloat16
    g = _gen(51)
    x, W = _x(K, g, dtype), _w(K, N, g, dtype)
    got = _nan(N, dtype)
    q.gemv(x=x, weights=[W], outs=[got], splits=splits)
    want = (x.float() @ W.float()).to(dtype)
    ok, err, idx = allclose_report(got, want, ATOL, RTOL)
    assert ok, f"splits {splits}: max abs err {err} at {idx}"


def test_deterministic_and_pdl_chain():
    """A chain of GEMV launches (each one's input is the previous one's output) with
    programmatic dependent launch gives the bits of plain launches, twice."""
    K, dtype = 2048, torch.bfloat16
    g = _gen(61)
    Ws = [(torch.randn(K, K, generator=g, device="cuda") * (1.0 / K ** 0.5)).to(dtype) for _ in range(6)]
    x0 = _x(K, g, dtype)
    runs = []
    for pdl in (False, True, True):
        bufs = [x0.clone()] + [_nan(K, dtype) for _ in Ws]
        for i, w in enumerate(Ws):
            q.gemv(x=bufs[i], weights=[w], outs=[bufs[i + 1]], pdl=pdl)
        torch.cuda.synchronize()
        runs.append(torch.stack(bufs[1:]))
    for r in runs[1:]:
        assert torch.equal(r.view(torch.int16), runs[0].view(torch.int16))


def test_launch_shape_fills_the_gpu():
    """The chosen split count puts every tile's cluster on the GPU at once for the
    Qwen3-8B projections (at least one CTA per SM for the q/k/v, o, gate/up and down
    launches)."""
    dtype = torch.bfloat16
    x = torch.zeros(4096, device="cuda", dtype=dtype)
    x2 = torch.zeros(12288, device="cuda", dtype=dtype)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    for xx, Ns in ((x, (4096, 1024, 1024)), (x, (4096,)), (x, (12288, 12288)), (x2, (4096,))):
        Ws = [torch.empty(xx.numel(), n, device="cuda", dtype=dtype) for n in Ns]
        swiglu = len(Ns) == 2
        outs = [torch.empty(Ns[0], device="cuda", dtype=dtype)] if swiglu else [torch.empty(n, device="cuda", dtype=dtype) for n in Ns]
        s, t = q.ops.gemv_launch_shape(x=xx, weights=Ws, outs=outs, swiglu=swiglu)
        assert 1 <= s <= 16 and s * t >= sms * 0.8, (Ns, s, t)
