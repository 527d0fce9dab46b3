"""GPU: the GatedDeltaNet decode kernel against the oracle's restatement of the
reference's host loop (src/model.cpp:692-791): output within max-abs 2e-3 /
rel 1e-2, conv state exact, recurrent state within fp32 rounding, over several
consecutive steps with the state carried on the device."""
import pytest
import torch

import qwenincuda_b200 as q
from conftest import allclose_report
from qwenincuda_b200.workloads import GdnConfig, make_gdn_inputs

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("Hk,Hv", [(16, 32), (8, 8), (4, 16)])
def test_gdn_steps_vs_oracle(oracle, dtype, Hk, Hv):
    cfg = GdnConfig(num_k_heads=Hk, num_v_heads=Hv)
    dev = make_gdn_inputs(cfg, device="cuda", dtype=dtype)
    host = {k: v.cpu().clone() for k, v in dev.items()}
    g = torch.Generator(device="cuda").manual_seed(77)
    for step in range(3):
        if step:
            new_qkv = torch.randn(cfg.conv_dim, generator=g, device="cuda").to(dtype)
            new_z = torch.randn(Hv * 128, generator=g, device="cuda").to(dtype)
            dev["qkv"].copy_(new_qkv)
            dev["z"].copy_(new_z)
            host["qkv"] = new_qkv.cpu()
            host["z"] = new_z.cpu()
        q.gated_delta_decode(**{k: dev[k] for k in dev}, num_k_heads=Hk, num_v_heads=Hv)
        torch.cuda.synchronize()
        want_out, want_cs, want_rs = oracle.gated_delta(
            **{k: host[k] for k in host if k != "out"}, num_k_heads=Hk, num_v_heads=Hv)
        host["conv_state"], host["recurrent_state"] = want_cs, want_rs
        assert torch.equal(dev["conv_state"].cpu(), want_cs), f"conv state step {step}"
        ok, err, _ = allclose_report(dev["recurrent_state"], want_rs, atol=1e-5, rtol=1e-4)
        assert ok, f"state step {step}: {err}"
        ok, err, idx = allclose_report(dev["out"], want_out)
        assert ok, f"out step {step}: {err} at {idx}"


@pytest.mark.parametrize("layers", [1, 4])
def test_gdn_pdl_chain_matches_plain_launches(layers):
    """GatedDeltaNet layers, each with its own state, stepped three times back to back
    with programmatic dependent launch give the same bytes as plain launches. With one
    layer every launch reads the state the launch before it wrote; with several, layer
    l's output-gate input z is layer l-1's output. The kernel loads only weights and
    L2 prefetches before griddepcontrol.wait, so both hazards are ordered."""
    import dataclasses

    results = []
    for pdl in (False, True):
        stack = [make_gdn_inputs(dataclasses.replace(GdnConfig(), seed=100 + l)) for l in range(layers)]
        for _ in range(3):
            for l, t in enumerate(stack):
                z = t["z"] if l == 0 else stack[l - 1]["out"]
                q.gated_delta_decode(qkv=t["qkv"], z=z, b=t["b"], a=t["a"], conv_w=t["conv_w"], dt_bias=t["dt_bias"],
                                     a_log=t["a_log"], norm_w=t["norm_w"], conv_state=t["conv_state"],
                                     recurrent_state=t["recurrent_state"], out=t["out"], num_k_heads=16,
                                     num_v_heads=32, pdl=pdl)
        torch.cuda.synchronize()
        results.append([(t["out"].clone(), t["conv_state"].clone(), t["recurrent_state"].clone()) for t in stack])
    for l, (plain, chained) in enumerate(zip(*results)):
        for name, x, y in zip(("out", "conv_state", "recurrent_state"), plain, chained):
            assert torch.equal(x, y), f"layer {l} {name}"


def test_gdn_states_ready_graph_matches_plain_launches():
    """A stack of four GatedDeltaNet layers captured once as a CUDA graph with
    QIC_PDL | QIC_GDN_STATES_READY (the states read before griddepcontrol.wait: each
    layer's states are written once per replay, and replays are whole graph launches)
    and replayed three times gives the bytes of three rounds of plain launches."""
    import dataclasses

    def stack():
        return [make_gdn_inputs(dataclasses.replace(GdnConfig(), seed=200 + l)) for l in range(4)]

    def step(st, **kw):
        for l, t in enumerate(st):
            z = t["z"] if l == 0 else st[l - 1]["out"]
            q.gated_delta_decode(qkv=t["qkv"], z=z, b=t["b"], a=t["a"], conv_w=t["conv_w"], dt_bias=t["dt_bias"],
                                 a_log=t["a_log"], norm_w=t["norm_w"], conv_state=t["conv_state"],
                                 recurrent_state=t["recurrent_state"], out=t["out"], num_k_heads=16, num_v_heads=32,
                                 **kw)

    plain = stack()
    for _ in range(3):
        step(plain)
    torch.cuda.synchronize()
    fast = stack()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        step(fast, pdl=True, states_ready=True, status=status)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    for l, (x, y) in enumerate(zip(plain, fast)):
        for name in ("out", "conv_state", "recurrent_state"):
            assert torch.equal(x[name], y[name]), f"layer {l} {name}"
    del graph


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_gdn_kernel_vs_reference_step(dtype):
    """The CUDA kernel against the reference's own decode step (run_linear_attention_block,
    src/model.cpp:656-795, run unchanged through oracle/_ref: fp16 as shipped and its
    bfloat16 instance) over three steps carrying the states: output within max-abs
    2e-3 / rel 1e-2, conv state exact, recurrent state within fp32 rounding."""
    from oracle.oracle import RefGatedDelta

    ref = RefGatedDelta(dtype)
    Hk, Hv = 4, 8
    cfg = GdnConfig(num_k_heads=Hk, num_v_heads=Hv)
    dev = make_gdn_inputs(cfg, device="cuda", dtype=dtype)
    host = {k: v.cpu().clone() for k, v in dev.items()}
    g = torch.Generator(device="cuda").manual_seed(78)
    for step in range(3):
        if step:
            for k, n in (("qkv", cfg.conv_dim), ("z", Hv * 128), ("b", Hv), ("a", Hv)):
                new = torch.randn(n, generator=g, device="cuda").to(dtype)
                dev[k].copy_(new)
                host[k] = new.cpu()
        q.gated_delta_decode(**dev, num_k_heads=Hk, num_v_heads=Hv)
        torch.cuda.synchronize()
        want_out, want_cs, want_rs = ref.step(**{k: host[k] for k in host if k != "out"}, num_k_heads=Hk,
                                              num_v_heads=Hv, eps=cfg.eps)
        host["conv_state"], host["recurrent_state"] = want_cs.view_as(host["conv_state"]), \
            want_rs.view_as(host["recurrent_state"])
        assert torch.equal(dev["conv_state"].cpu(), host["conv_state"]), f"conv state step {step}"
        ok, err, _ = allclose_report(dev["recurrent_state"], host["recurrent_state"], atol=1e-5, rtol=1e-4)
        assert ok, f"state step {step}: {err}"
        ok, err, idx = allclose_report(dev["out"], want_out)
        assert ok, f"out step {step}: {err} at {idx}"
