"""CPU tests of bench.py's vLLM comparison driver: one engine process per run,
arms interleaved with the order rotated each repeat, and per batch size the
mean / min / max of each arm and its ratio to the reference Triton arm.  The
engine processes are faked; nothing runs vLLM."""
import json
import subprocess
import types

import bench


def _fake_run_factory(calls, tok_s):
    def fake_run(cmd, capture_output, text, env, timeout):
        arm = cmd[cmd.index("--vllm-arm") + 1]
        calls.append(arm)
        rep = sum(1 for c in calls if c == arm) - 1
        res = {"batch": {str(bs): {"output_tok_s": tok_s[arm][rep] * bs}
                         for bs in (1, 16, 64, 256)},
               "hook_calls_during_compile_and_capture": 7, "quantized_layers": 128}
        return types.SimpleNamespace(returncode=0, stdout="noise\nVLLM_ARM_RESULT " +
                                     json.dumps(res) + "\n", stderr="")
    return fake_run


def test_arms_interleaved_rotated_and_summarised(monkeypatch, capsys):
    calls = []
    tok_s = {"cutlass": [10.0, 12.0, 11.0], "reference_triton": [5.0, 5.0, 8.0],
             "scalesweep_mse": [9.0, 9.0, 9.0]}
    monkeypatch.setattr(subprocess, "run", _fake_run_factory(calls, tok_s))
    args = types.SimpleNamespace(vllm_workload="decode", vllm_repeats=3,
                                 vllm_arms=["cutlass", "reference_triton", "scalesweep_mse"])
    bench.run_vllm_e2e(args)
    out = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    # one process per run, the arm order rotated each repeat
    assert calls == ["cutlass", "reference_triton", "scalesweep_mse",
                     "reference_triton", "scalesweep_mse", "cutlass",
                     "scalesweep_mse", "cutlass", "reference_triton"]
    row = out["batch"]["16"]
    assert row["cutlass"]["runs"] == [160.0, 192.0, 176.0]
    assert row["cutlass"]["min"] == 160.0 and row["cutlass"]["max"] == 192.0
    assert row["reference_triton"]["mean"] == 96.0
    assert row["reference_triton"]["over_reference_triton"] == 1.0
    assert row["scalesweep_mse"]["over_reference_triton"] == 1.5
    assert out["failures"] == [] and out["repeats"] == 3
    assert out["per_run"]["cutlass"][0] == {"hook_calls_during_compile_and_capture": 7,
                                            "quantized_layers": 128,
                                            "process_seconds": out["per_run"]["cutlass"][0][
                                                "process_seconds"]}


def test_a_failed_run_is_reported_not_averaged(monkeypatch, capsys):
    def fake_run(cmd, capture_output, text, env, timeout):
        return types.SimpleNamespace(returncode=1, stdout="", stderr="engine died")
    monkeypatch.setattr(subprocess, "run", fake_run)
    args = types.SimpleNamespace(vllm_workload="reference", vllm_repeats=1,
                                 vllm_arms=["reference_triton"])
    bench.run_vllm_e2e(args)
    out = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert out["batch"]["256"] == {}
    assert out["failures"][0]["arm"] == "reference_triton"
    assert "engine died" in out["failures"][0]["tail"]
