"""CPU checks of bench.py's host-side legs: the CPU baseline and the reference arm
time the same workload as this library's line (GatedDeltaNet, batched, pair and
attention samples), in the same metric and unit, and say what they sampled."""
import argparse
import json

import pytest

import bench


@pytest.mark.parametrize("workload", ["qwen35_gdn", "qwen3_0p6b_s1025"])
def test_cpu_baseline_per_workload(workload):
    cb = bench.cpu_baseline(workload, budget_s=0.2)
    assert cb["kind"] == "port" and cb["unit"] == "GB/s"
    assert cb["value"] > 0 and cb["cores"] >= 1
    assert workload != "qwen35_gdn" or "GatedDeltaNet" in cb["sample"]


def test_cpu_baseline_rejects_unknown_workload():
    with pytest.raises(SystemExit):
        bench.cpu_baseline("no_such_workload", budget_s=0.1)


@pytest.mark.parametrize("workload,metric", [("qwen35_gdn", "GatedDeltaNet state GB/s"),
                                             ("qwen3_0p6b_s1025", "decode-attn KV-read GB/s")])
def test_reference_arm_line(workload, metric, capsys, monkeypatch):
    # the reference kernels on the GPU are extra information; without a GPU they are skipped
    monkeypatch.setattr(bench, "reference_gpu", lambda *a, **k: {"unavailable": "no GPU"})
    monkeypatch.setattr(bench, "cpu_baseline", lambda w, budget_s: {
        "value": 2.0, "unit": "GB/s", "kind": "port", "cores": 1, "sample": w,
        "us_per_step": 1.0, "us_per_layer": 1.0})
    args = argparse.Namespace(workload=workload, steps=4, warmup=1, gpus=1)
    bench.run_reference_arm(args, 1, 0)
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["metric"] == metric
    assert line["config"]["workload"] == workload
    assert line["value"] == line["cpu_baseline"]["value"] == line["e2e"]["value"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    assert line["ms_per_step"] > 0


def test_reference_arm_silent_on_other_ranks(capsys):
    args = argparse.Namespace(workload="qwen35_gdn", steps=4, warmup=1, gpus=2)
    bench.run_reference_arm(args, 2, 1)
    assert capsys.readouterr().out == ""


@pytest.mark.parametrize("workload", ["qwen3_8b_s8192", "qwen3_0p6b_s1025", "qwen35_gated_s32769", "qwen3_8b_s131073",
                                      "qwen35_gdn", "qwen35_pair", "qwen3_8b_batch64"])
@pytest.mark.parametrize("world", [1, 2, 8])
def test_reference_arm_config_is_this_library_config(workload, world, capsys, monkeypatch):
    """Both arms print the same `config` for the same workload and N (the reference
    arm's line is built from line_config too, and nothing run-dependent is in it)."""
    monkeypatch.setattr(bench, "reference_gpu", lambda *a, **k: {"unavailable": "no GPU"})
    monkeypatch.setattr(bench, "cpu_baseline", lambda w, budget_s: {
        "value": 2.0, "unit": "GB/s", "kind": "port", "cores": 1, "sample": w})
    args = argparse.Namespace(workload=workload, steps=4, warmup=1, gpus=world)
    bench.run_reference_arm(args, world, 0)
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert line["config"] == bench.line_config(workload, world)
    assert line["config"]["workload"] == workload
    partitioned = world > 1 and workload in ("qwen3_8b_s131073", "qwen3_8b_batch64")
    assert line["scaling"] == ("strong" if partitioned else "weak")
    if world == 1:
        assert line["config"]["parallelism"] == "single"
