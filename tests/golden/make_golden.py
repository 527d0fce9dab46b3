"""Generates the golden vectors in tests/golden/ from the reference's own kernels.

Runs the reference's src/kernels.cu (compiled unchanged for sm_100a by
oracle/Makefile into oracle/_ref/) on small seeded inputs on a CUDA device and saves
inputs and outputs as torch files. tests/test_oracle_cpu.py checks the CPU oracle
against them, which pins the oracle to the reference's behaviour.

    python tests/golden/make_golden.py [output_dir]
"""
from __future__ import annotations

import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from oracle.oracle import RefKernels  # noqa: E402


def main(out_dir: Path = HERE) -> None:
    out_dir.mkdir(parents=True, exist_ok=True)
    g = torch.Generator(device="cuda").manual_seed(2024)
    n = 0
    for dtype, tag in ((torch.bfloat16, "bf16"), (torch.float16, "f16")):
        ref = RefKernels(dtype)
        # attention: contiguous and paged, GQA groups 1/2/4, head dims 64/128/256
        for (H, Hkv, d, S, P, paged) in [(4, 2, 64, 33, 16, False), (8, 4, 128, 200, 16, True),
                                         (16, 4, 256, 130, 16, True), (4, 4, 128, 1, 16, True),
                                         (16, 8, 128, 1025, 16, True)]:
            npages = (S + P - 1) // P
            qv = torch.randn(H * d, generator=g, device="cuda").to(dtype)
            kc = (torch.randn(npages * P, Hkv * d, generator=g, device="cuda") * 0.5).to(dtype)
            vc = (torch.randn(npages * P, Hkv * d, generator=g, device="cuda") * 0.5).to(dtype)
            table = torch.randperm(npages, generator=g, device="cuda").to(torch.int32)
            out = torch.empty(H * d, device="cuda", dtype=dtype)
            if paged:
                ref.paged_attention(qv, kc, vc, table, P, H, Hkv, d, S, out)
            else:
                ref.flash_attention(qv, kc, vc, H, Hkv, d, S, out)
            case = dict(kind="attention", H=H, Hkv=Hkv, d=d, S=S, P=P, q=qv.cpu(), k=kc.cpu(), v=vc.cpu(),
                        out=out.cpu())
            if paged:
                case["table"] = table.cpu()
            torch.save(case, out_dir / f"attention_{tag}_h{H}_kv{Hkv}_d{d}_s{S}_{'paged' if paged else 'flat'}.pt")
            n += 1
        # head RMSNorm
        H, d = 16, 128
        x = (torch.randn(H * d, generator=g, device="cuda") * 2).to(dtype)
        w = (1 + 0.1 * torch.randn(d, generator=g, device="cuda")).to(dtype)
        out = torch.empty_like(x)
        ref.head_rmsnorm(x, w, H, d, 1e-6, out)
        torch.save(dict(kind="head_rmsnorm", H=H, d=d, eps=1e-6, x=x.cpu(), w=w.cpu(), out=out.cpu()),
                   out_dir / f"head_rmsnorm_{tag}.pt")
        n += 1
        # RoPE at small and large positions
        for pos in (0, 3, 1024, 131072):
            x = torch.randn(8 * 128, generator=g, device="cuda").to(dtype)
            out = x.clone()
            ref.rope_inplace(out, 8, 128, pos, 1.0e6)
            torch.save(dict(kind="rope", H=8, d=128, pos=pos, theta=1.0e6, x=x.cpu(), out=out.cpu(),
                            atol=2.0 ** -7 if pos <= 1024 else 0.05), out_dir / f"rope_{tag}_pos{pos}.pt")
            n += 1
        x = torch.randn(1024, generator=g, device="cuda").to(dtype)
        gate = torch.randn(1024, generator=g, device="cuda").to(dtype)
        out = x.clone()
        ref.sigmoid_mul_inplace(out, gate, 1024)
        torch.save(dict(kind="sigmoid_mul", x=x.cpu(), gate=gate.cpu(), out=out.cpu()), out_dir / f"sigmoid_mul_{tag}.pt")
        n += 1
    print(f"wrote {n} golden cases to {out_dir}")


if __name__ == "__main__":
    main(Path(sys.argv[1]) if len(sys.argv) > 1 else HERE)
