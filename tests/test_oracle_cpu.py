"""CPU checks of the oracle (oracle/qic_oracle.c): its 16-bit rounding, and its
restatements of the reference math against independent float64 formulas and
against the golden vectors produced by the reference kernels (tests/golden)."""
import math
from pathlib import Path

import pytest
import torch

from conftest import allclose_report

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_rounding_matches_torch(oracle, dtype):
    g = torch.Generator().manual_seed(0)
    x = torch.cat([
        torch.randn(20000, generator=g) * 3,
        torch.randn(5000, generator=g) * 1e-5,        # f16 subnormals
        torch.randn(5000, generator=g) * 70000,       # f16 overflow region
        torch.tensor([0.0, -0.0, float("inf"), -float("inf"), 65504.0, 65519.0, 65520.0, 2 ** -24, 2 ** -25,
                      3 * 2 ** -25, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -9]),
    ]).float()
    # round through the oracle's sigmoid_mul with gate=+inf (sigmoid=1): x -> dtype(x)
    want = x.to(dtype)
    gate = torch.full_like(want, float("inf"))
    got = oracle.sigmoid_mul(want, gate)
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))


def _ref_attention_f64(q, k, v, H, Hkv, d, S, table=None, P=16):
    q = q.double().view(H, d)
    kv = k.double().view(-1, Hkv, d)
    vv = v.double().view(-1, Hkv, d)
    t = torch.arange(S)
    rows = t if table is None else table.long()[t // P] * P + t % P
    out = torch.empty(H, d, dtype=torch.float64)
    g = H // Hkv
    for h in range(H):
        K = kv[rows, h // g]
        V = vv[rows, h // g]
        s = (K @ q[h]) / math.sqrt(d)
        p = torch.softmax(s, 0)
        out[h] = p @ V
    return out


@pytest.mark.parametrize("H,Hkv,d,S", [(4, 2, 64, 1), (4, 2, 64, 37), (8, 2, 128, 100), (4, 4, 256, 65)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_attention_oracle_vs_float64(oracle, H, Hkv, d, S, dtype):
    g = torch.Generator().manual_seed(S * 7 + d)
    P = 16
    npages = (S + P - 1) // P
    q = torch.randn(H * d, generator=g).to(dtype)
    k = (torch.randn(npages * P, Hkv * d, generator=g) * 0.5).to(dtype)
    v = (torch.randn(npages * P, Hkv * d, generator=g) * 0.5).to(dtype)
    want = _ref_attention_f64(q, k, v, H, Hkv, d, S)
    got = oracle.attention(q, k, v, H, Hkv, d, S)
    ok, err, _ = allclose_report(got, want.flatten(), atol=1e-3, rtol=8e-3)
    assert ok, err
    # paged view of a permuted copy gives the same result
    perm = torch.randperm(npages, generator=g).to(torch.int32)
    kp = torch.empty_like(k)
    vp = torch.empty_like(v)
    for lp in range(npages):
        kp[perm[lp] * P:(perm[lp] + 1) * P] = k[lp * P:(lp + 1) * P]
        vp[perm[lp] * P:(perm[lp] + 1) * P] = v[lp * P:(lp + 1) * P]
    got_p = oracle.attention(q, kp, vp, H, Hkv, d, S, page_table=perm, page_size=P)
    assert torch.equal(got_p.view(torch.int16), got.view(torch.int16))


def test_attention_oracle_empty_sequence(oracle):
    q = torch.randn(4 * 64).to(torch.bfloat16)
    k = torch.randn(16, 2 * 64).to(torch.bfloat16)
    out = oracle.attention(q, k, k, 4, 2, 64, 0)
    assert torch.count_nonzero(out.float()) == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_norm_rope_oracle_vs_float64(oracle, dtype):
    g = torch.Generator().manual_seed(3)
    H, d = 8, 128
    x = torch.randn(H * d, generator=g).to(dtype)
    w = (1 + 0.1 * torch.randn(d, generator=g)).to(dtype)
    got = oracle.head_rmsnorm(x, w, H, d, 1e-6)
    xd = x.double().view(H, d)
    want = xd / torch.sqrt((xd ** 2).mean(1, keepdim=True) + 1e-6) * w.double()
    assert torch.allclose(got.double().view(H, d), want, rtol=2 ** -7, atol=0)
    for pos in (0, 5, 1024):
        r = oracle.rope(got, H, d, pos, 1.0e6)
        gd = got.double().view(H, d)
        i = torch.arange(d // 2, dtype=torch.float64)
        ang = pos * (1.0e6 ** (-2 * i / d))
        c, s = torch.cos(ang), torch.sin(ang)
        x0, x1 = gd[:, : d // 2], gd[:, d // 2:]
        want_r = torch.cat([x0 * c - x1 * s, x1 * c + x0 * s], 1)
        assert torch.allclose(r.double().view(H, d), want_r, rtol=2 ** -6, atol=2 ** -7 * 4)


def test_append_oracle_slot(oracle):
    Hkv, d, P = 2, 64, 16
    g = torch.Generator().manual_seed(9)
    npages = 4
    kc = torch.randn(npages * P, Hkv * d, generator=g).to(torch.bfloat16)
    vc = torch.randn(npages * P, Hkv * d, generator=g).to(torch.bfloat16)
    kn = torch.randn(Hkv * d, generator=g).to(torch.bfloat16)
    vn = torch.randn(Hkv * d, generator=g).to(torch.bfloat16)
    w = torch.ones(d, dtype=torch.bfloat16)
    table = torch.tensor([2, 0, 3, 1], dtype=torch.int32)
    pos = 37  # logical page 2, offset 5 -> physical row 3*16+5
    k2, v2 = oracle.kv_append(kn, vn, w, 1e-6, 1e6, pos, kc, vc, Hkv, d, page_table=table, page_size=P)
    row = 3 * P + 5
    changed = (k2.view(torch.int16) != kc.view(torch.int16)).any(1).nonzero().flatten().tolist()
    assert changed == [row]
    assert torch.equal(v2[row], vn)
    kk = oracle.rope(oracle.head_rmsnorm(kn, w, Hkv, d, 1e-6), Hkv, d, pos, 1e6)
    assert torch.equal(k2[row].view(torch.int16), kk.view(torch.int16))


def _gdn_f64(inp, Hk, Hv, dk, dv, K, eps):
    f = {k: v.double() for k, v in inp.items()}
    cs = f["conv_state"].clone()
    rs = f["recurrent_state"].clone()
    cs = torch.cat([cs[:, 1:], f["qkv"][:, None]], 1)
    acc = (f["conv_w"] * cs).sum(1)
    mixed = acc / (1 + torch.exp(-acc))
    q = mixed[: Hk * dk].view(Hk, dk)
    k = mixed[Hk * dk: 2 * Hk * dk].view(Hk, dk)
    v = mixed[2 * Hk * dk:].view(Hv, dv)
    q = q / torch.sqrt((q ** 2).sum(1, keepdim=True) + 1e-6)
    k = k / torch.sqrt((k ** 2).sum(1, keepdim=True) + 1e-6)
    rep = Hv // Hk
    out = torch.empty(Hv, dv, dtype=torch.float64)
    for h in range(Hv):
        qh = q[h // rep] / math.sqrt(dk)
        kh = k[h // rep]
        beta = 1 / (1 + torch.exp(-f["b"][h]))
        g = torch.exp(-torch.exp(f["a_log"][h]) * torch.log1p(torch.exp(f["a"][h] + f["dt_bias"][h])))
        S = rs[h] * g
        kv_mem = kh @ S
        S = S + torch.outer(kh, (v[h] - kv_mem) * beta)
        rs[h] = S
        o = qh @ S
        inv = 1 / torch.sqrt((o ** 2).mean() + eps)
        z = f["z"].view(Hv, dv)[h]
        out[h] = o * inv * f["norm_w"] * (z / (1 + torch.exp(-z)))
    return out.flatten(), cs, rs


@pytest.mark.parametrize("Hk,Hv", [(4, 8), (2, 2), (2, 8)])
def test_gdn_oracle_vs_float64(oracle, Hk, Hv):
    from qwenincuda_b200.workloads import GdnConfig, make_gdn_inputs

    cfg = GdnConfig(num_k_heads=Hk, num_v_heads=Hv)
    inp = make_gdn_inputs(cfg, device="cpu")
    inp.pop("out")
    got, cs, rs = oracle.gated_delta(**inp, num_k_heads=Hk, num_v_heads=Hv)
    want, cs_w, rs_w = _gdn_f64(inp, Hk, Hv, 128, 128, 4, 1e-6)
    assert torch.allclose(cs.double(), cs_w, atol=1e-6)
    assert torch.allclose(rs.double(), rs_w, atol=1e-5, rtol=1e-4)
    ok, err, _ = allclose_report(got, want)
    assert ok, err


def _golden_files():
    return sorted(GOLDEN.glob("*.pt"))


@pytest.mark.skipif(not _golden_files(), reason="no golden vectors committed")
@pytest.mark.parametrize("path", _golden_files(), ids=lambda p: p.stem)
def test_oracle_against_reference_golden(oracle, path):
    """The reference kernels' outputs on seeded inputs (tests/golden/make_golden.py)
    pin the restatement: attention within the bf16 tolerance; norm/RoPE within the
    fast-math error of the reference build."""
    case = torch.load(path)
    kind = case["kind"]
    if kind == "attention":
        got = oracle.attention(case["q"], case["k"], case["v"], case["H"], case["Hkv"], case["d"], case["S"],
                               page_table=case.get("table"), page_size=case.get("P", 16))
        ok, err, _ = allclose_report(got, case["out"])
        assert ok, err
    elif kind == "head_rmsnorm":
        got = oracle.head_rmsnorm(case["x"], case["w"], case["H"], case["d"], case["eps"])
        ok, err, _ = allclose_report(got, case["out"], atol=0, rtol=2 ** -7)
        assert ok, err
    elif kind == "rope":
        got = oracle.rope(case["x"], case["H"], case["d"], case["pos"], case["theta"])
        ok, err, _ = allclose_report(got, case["out"], atol=case["atol"], rtol=2 ** -7)
        assert ok, err
    elif kind == "sigmoid_mul":
        got = oracle.sigmoid_mul(case["x"], case["gate"])
        ok, err, _ = allclose_report(got, case["out"], atol=0, rtol=2 ** -7)
        assert ok, err
    elif kind == "gated_delta":
        # the reference's own host loop (tests/golden/make_gdn_golden.py): the
        # restatement follows it operation for operation in IEEE fp32, so every step's
        # output and both final states are bit-identical
        Hk, Hv, dk, dv, K, _ = case["case"]
        inp = case["inputs"]
        cs, rs = inp["conv_state"], inp["recurrent_state"]
        for t, st in enumerate(inp["steps"]):
            got, cs, rs = oracle.gated_delta(**st, conv_w=inp["conv_w"], dt_bias=inp["dt_bias"], a_log=inp["a_log"],
                                             norm_w=inp["norm_w"], conv_state=cs, recurrent_state=rs, num_k_heads=Hk,
                                             num_v_heads=Hv, k_head_dim=dk, v_head_dim=dv, conv_kernel=K,
                                             eps=case["eps"])
            assert torch.equal(got.view(torch.int16), case["outs"][t].view(torch.int16)), f"output, step {t}"
        assert torch.equal(cs, case["conv_state"])
        assert torch.equal(rs, case["recurrent_state"])
    else:
        pytest.fail(f"unknown golden kind {kind}")


def test_gdn_golden_inputs_regenerate_from_their_seeds():
    """tests/golden/make_gdn_golden.py still produces the inputs stored in the
    committed GatedDeltaNet fixtures (same cases, same seeds, same draws)."""
    import sys

    sys.path.insert(0, str(GOLDEN))
    import make_gdn_golden as gen

    files = sorted(GOLDEN.glob("gdn_ref_*.pt"))
    for _, tag in gen.DTYPES:
        assert len(list(GOLDEN.glob(f"gdn_ref_{tag}_*.pt"))) == len(gen.CASES), tag
    for path in files:
        case = torch.load(path)
        assert tuple(case["case"]) in [tuple(c) for c in gen.CASES]
        want = gen.case_inputs(*case["case"], dtype=case["inputs"]["conv_w"].dtype)
        got = case["inputs"]
        for k in ("conv_w", "dt_bias", "a_log", "norm_w", "conv_state", "recurrent_state"):
            assert torch.equal(got[k], want[k]), (path.name, k)
        for t, (a, b) in enumerate(zip(got["steps"], want["steps"])):
            for k in a:
                assert torch.equal(a[k], b[k]), (path.name, t, k)
