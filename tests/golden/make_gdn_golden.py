"""Generates the GatedDeltaNet golden vectors in tests/golden/ from the reference's
own decode step.

Runs run_linear_attention_block (src/model.cpp:656-795, compiled unchanged by
oracle/Makefile into oracle/_ref/libqicref_gdn.so, and its bfloat16 instance
libqicref_gdn_bf16.so) for three consecutive decode steps on small seeded inputs, carrying the conv and recurrent states, on a CUDA device
(the reference copies its inputs through the device). Saves inputs, per-step outputs
and final states; tests/test_oracle_cpu.py checks the CPU oracle's restatement of the
same loop against them.

    python tests/golden/make_gdn_golden.py [output_dir]
"""
from __future__ import annotations

import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from oracle.oracle import RefGatedDelta  # noqa: E402

# (Hk, Hv, dk, dv, conv kernel, seed): value heads per key head 2, 1 and 2; head dims
# 32, 64 and 128; conv kernels 4 and 3
CASES = [(2, 4, 32, 32, 4, 11), (2, 2, 64, 64, 3, 12), (1, 2, 128, 128, 4, 13)]
STEPS = 3
EPS = 1e-6


def case_inputs(Hk, Hv, dk, dv, K, seed, dtype=torch.float16):
    """Seeded inputs of one case (CPU generator): weights, initial states and the
    per-step projections."""
    g = torch.Generator().manual_seed(seed)
    conv_dim = 2 * Hk * dk + Hv * dv

    def randn(n, std=1.0):
        return (torch.randn(n, generator=g) * std).to(dtype)

    return dict(
        conv_w=randn(conv_dim * K, 0.5),
        dt_bias=randn(Hv, 0.1),
        a_log=torch.log(torch.rand(Hv, generator=g) * 15.0 + 1.0).to(dtype),
        norm_w=(1.0 + torch.randn(dv, generator=g) * 0.1).to(dtype),
        conv_state=torch.randn(conv_dim * K, generator=g),
        recurrent_state=torch.randn(Hv * dk * dv, generator=g) * 0.02,
        steps=[dict(qkv=randn(conv_dim), z=randn(Hv * dv), b=randn(Hv), a=randn(Hv)) for _ in range(STEPS)],
    )


DTYPES = ((torch.float16, "f16"), (torch.bfloat16, "bf16"))  # as shipped; the bfloat16 instance


def main(out_dir: Path = HERE) -> None:
    out_dir.mkdir(parents=True, exist_ok=True)
    for dtype, tag in DTYPES:
        ref = RefGatedDelta(dtype)
        for Hk, Hv, dk, dv, K, seed in CASES:
            _one_case(ref, out_dir, tag, dtype, Hk, Hv, dk, dv, K, seed)


def _one_case(ref, out_dir, tag, dtype, Hk, Hv, dk, dv, K, seed):
    """Three steps of one case through the reference, saved with their inputs."""
    inp = case_inputs(Hk, Hv, dk, dv, K, seed, dtype)
    cs, rs = inp["conv_state"], inp["recurrent_state"]
    outs = []
    for st in inp["steps"]:
        out, cs, rs = ref.step(**st, conv_w=inp["conv_w"], dt_bias=inp["dt_bias"], a_log=inp["a_log"],
                               norm_w=inp["norm_w"], conv_state=cs, recurrent_state=rs, num_k_heads=Hk,
                               num_v_heads=Hv, k_head_dim=dk, v_head_dim=dv, conv_kernel=K, eps=EPS)
        outs.append(out)
    name = f"gdn_ref_{tag}_hk{Hk}_hv{Hv}_d{dk}_k{K}.pt"
    torch.save(dict(kind="gated_delta", case=(Hk, Hv, dk, dv, K, seed), eps=EPS, inputs=inp, outs=torch.stack(outs),
                    conv_state=cs, recurrent_state=rs), out_dir / name)
    print("wrote", name)


if __name__ == "__main__":
    main(Path(sys.argv[1]) if len(sys.argv) > 1 else HERE)
