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
