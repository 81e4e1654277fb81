"""bench.py's host-side logic (no GPU): the op sweep's median over full
passes and its spread figure, the clock summary's throttle reasons, the NCCL
log that reports the exchange's algorithm, the reference arm's line and the
CPU path it times, the peaks file and the rank environment."""

from __future__ import annotations

import os

import pytest

import bench


def test_op_sweep_reports_the_median_pass_and_its_spread(monkeypatch):
    passes = iter([
        {"row_a": (1.0, 1e9), "row_b": (2.0, 1e9)},
        {"row_a": (3.0, 1e9), "row_b": (2.2, 1e9)},   # a disturbed pass of row_a
        {"row_a": (1.1, 1e9), "row_b": (2.1, 1e9)},
    ])
    monkeypatch.setattr(bench, "_op_sweep_pass", lambda ops, iters: next(passes))
    res = bench.op_sweep(None, hbm_peak=1000.0, iters=20, passes=3)
    assert res["row_a"]["ms"] == 1.1 and res["row_a"]["spread"] == 3.0
    assert res["row_a"]["gb_s"] == round(1e9 / 1.1e-3 / 1e9, 1)
    assert res["row_a"]["frac"] == round(1e9 / 1.1e-3 / 1e9 / 1000.0, 3)
    assert res["row_b"]["ms"] == 2.1 and res["row_b"]["spread"] == 1.1


def test_clock_summary_lists_active_throttle_reasons():
    s = bench.ClockSampler(0)
    s.source = "nvidia-smi"
    s.add_smi_lines([
        "0, 1965, 1965, 700.0, 0x0, Not Active, Not Active, Not Active, Not Active",
        "0, 1410, 1965, 1000.0, 0x4, Not Active, Not Active, Not Active, Active",
        "0, 1380, 1965, 1000.0, 0x4, Not Active, Not Active, Not Active, Active",
        "garbage",
    ])
    out = s.summary()
    assert out["sm_mhz"] == 1410 and out["sm_max_mhz"] == 1965 and out["sm_mhz_min"] == 1380
    assert out["reasons"] == ["sw_power_cap"] and out["samples"] == 3
    assert bench.ClockSampler(0).summary()["reasons"] == ["unsampled"]


def test_clock_summary_from_nvml_flags():
    s = bench.ClockSampler(0)
    s.source = "nvml"
    s.rows = [(1965.0, 1965.0, [False, False, False, False]), (1900.0, 1965.0, [True, False, False, False])]
    assert s.summary()["reasons"] == ["hw_slowdown"]


def test_nccl_choices_from_tuning_lines():
    # Lines as NCCL 2.28 writes them with NCCL_DEBUG=INFO, NCCL_DEBUG_SUBSYS=INIT,TUNING.
    lines = [
        "vm:774:823 [0] NCCL INFO NVLS multicast support is available on dev 0 (NVLS_NCHANNELS 16)",
        "vm:774:857 [0] NCCL INFO AllReduce: 67141632 Bytes -> Algo NVLS proto SIMPLE channel{Lo..Hi}={0..15}",
        "vm:774:875 [0] NCCL INFO AllReduce: 67108864 Bytes -> Algo NVLS proto SIMPLE channel{Lo..Hi}={0..15}",
        "vm:774:879 [0] NCCL INFO AllReduce: 134225920 Bytes -> Algo NVLS proto SIMPLE channel{Lo..Hi}={0..15}",
        "vm:774:880 [0] NCCL INFO AllReduce: 134225920 Bytes -> Algo NVLS proto SIMPLE channel{Lo..Hi}={0..15}",
        "vm:774:881 [0] NCCL INFO AllReduce: 4 Bytes -> Algo RING proto LL channel{Lo..Hi}={0..0}",
    ]
    got = bench.nccl_choices(lines, {134225920, 67141632, 67108864})
    assert got["nvls_available"]
    assert got["allreduce"]["134225920"] == {"algo": "NVLS", "proto": "SIMPLE", "channels": 16, "calls": 2}
    assert got["allreduce"]["67108864"]["calls"] == 1 and "4" not in got["allreduce"]
    mixed = bench.nccl_choices(lines + ["x AllReduce: 67108864 Bytes -> Algo RING proto LL channel{Lo..Hi}={0..7}"],
                               {67108864})
    assert mixed["allreduce"]["67108864"]["algo"] == "mixed"


@pytest.mark.parametrize("env,takes_over", [
    ({}, True),
    ({"NCCL_DEBUG": "VERSION"}, True),   # a quiet level set by the environment
    ({"NCCL_DEBUG": "warn"}, True),
    ({"NCCL_DEBUG": "INFO"}, False),     # the user reads NCCL's log themselves
    ({"NCCL_DEBUG": "TRACE"}, False),
    ({"NCCL_DEBUG": "VERSION", "NCCL_DEBUG_FILE": "/tmp/mine.%h.%p"}, False),
])
def test_nccl_log_setup_respects_a_user_log(monkeypatch, env, takes_over):
    for key in ("NCCL_DEBUG", "NCCL_DEBUG_FILE", "NCCL_DEBUG_SUBSYS"):
        monkeypatch.delenv(key, raising=False)
    for key, value in env.items():
        monkeypatch.setenv(key, value)
    path = bench.nccl_log_setup(3)
    if takes_over:
        assert path is not None and "rank3" in path
        assert os.environ["NCCL_DEBUG"] == "INFO" and os.environ["NCCL_DEBUG_FILE"] == path
        assert "TUNING" in os.environ["NCCL_DEBUG_SUBSYS"]
    else:
        assert path is None
        assert os.environ["NCCL_DEBUG"] == env["NCCL_DEBUG"]


def test_reference_arm_prints_one_line_on_rank_zero_only(monkeypatch, capsys):
    # The reference arm's line carries the same metric, unit and config as
    # our arm's, a cpu_baseline describing the run and an e2e with no copies.
    import json
    import types

    monkeypatch.setattr(bench, "cpu_mlp_throughput", lambda steps, warmup: (2950.0, 16, 5.5, 1980.0))
    args = types.SimpleNamespace(gpus=2, steps=2, warmup=3)
    bench.run_reference(args, rank=1, world=2)
    assert capsys.readouterr().out == ""
    bench.run_reference(args, rank=0, world=2)
    line = json.loads(capsys.readouterr().out)
    assert line["impl"] == "reference" and line["metric"] == bench.METRIC and line["unit"] == bench.UNIT
    assert line["config"] == bench.workload_config(2) and line["config"]["global_batch"] == 2 * bench.PER_RANK_BATCH
    assert line["value"] == 2950.0 and line["ms_per_step"] == 2750.0 and line["higher_is_better"] is True
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] == 16
    assert line["e2e"] == {"value": 2950.0, "unit": bench.UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_cpu_path_of_the_step_runs_on_every_host_core():
    # The CPU port of the step (full-size weights, a few rows here) on all
    # the cores this process may use, whatever OMP_NUM_THREADS says.
    value, threads, elapsed, gflops = bench.cpu_mlp_throughput(1, 0, rows=64)
    assert value > 0 and elapsed > 0 and gflops > 0
    # every core the process may use, unless the OpenMP runtime caps it (or
    # the port was built without OpenMP: one thread)
    limit = int(os.environ.get("OMP_THREAD_LIMIT", "0")) or bench.host_threads()
    assert threads == min(bench.host_threads(), limit) or threads == 1


def test_nccl_summary_reads_the_steps_exchange_sizes(tmp_path):
    import types

    import torch

    from tensorplay_mlu_b200.train import bucket_b_slices

    model = types.SimpleNamespace(bucket_a=torch.empty(4096 * 16384 + 4096, dtype=torch.bfloat16),
                                  _bucket_b_slices=bucket_b_slices(4096, 16384, 2))
    log = tmp_path / "nccl.log"
    log.write_text("\n".join([
        "h:1:2 [0] NCCL INFO NVLS multicast support is available on dev 0 (NVLS_NCHANNELS 16)",
        "h:1:3 [0] NCCL INFO AllReduce: 134225920 Bytes -> Algo NVLS proto SIMPLE channel{Lo..Hi}={0..15}",
        "h:1:4 [0] NCCL INFO AllReduce: 67141632 Bytes -> Algo RING proto SIMPLE channel{Lo..Hi}={0..23}",
        "h:1:5 [0] NCCL INFO AllReduce: 67108864 Bytes -> Algo RING proto SIMPLE channel{Lo..Hi}={0..23}",
        "h:1:6 [0] NCCL INFO AllReduce: 1073741824 Bytes -> Algo NVLS proto SIMPLE channel{Lo..Hi}={0..15}",
    ]) + "\n")
    got = bench.nccl_summary(str(log), model)
    assert got["nvls_available"]
    assert set(got["allreduce"]) == {"134225920", "67141632", "67108864"}  # the sweep's 1 GiB is not the step's
    assert got["allreduce"]["67141632"] == {"algo": "RING", "proto": "SIMPLE", "channels": 24, "calls": 1}
    assert bench.nccl_summary(None, model) is None
    assert bench.nccl_summary(str(tmp_path / "missing.log"), model) is None


def test_peaks_fall_back_when_the_measured_file_is_absent(monkeypatch, tmp_path):
    monkeypatch.setattr(bench, "ROOT", str(tmp_path))
    assert bench.peaks() == (6650.0, 1590.0, 1400.0, "fallback")
    (tmp_path / "MEASURED_PEAKS.json").write_text(
        '{"hbm_gbs": 6455.3, "bf16_tflops": 1659.6, "bf16_tflops_sustained": 1405.5}')
    assert bench.peaks() == (6455.3, 1659.6, 1405.5, "measured")


def test_rank_environment(monkeypatch):
    for key in ("RANK", "WORLD_SIZE", "LOCAL_RANK"):
        monkeypatch.delenv(key, raising=False)
    assert bench.dist_env() == (0, 1, 0)
    monkeypatch.setenv("RANK", "5")
    monkeypatch.setenv("WORLD_SIZE", "8")
    assert bench.dist_env() == (5, 8, 5)
    monkeypatch.setenv("LOCAL_RANK", "1")
    assert bench.dist_env() == (5, 8, 1)
