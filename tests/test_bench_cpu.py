"""bench.py's host-side logic: the op sweep's median over full passes and
its spread figure, the clock summary's throttle reasons, and the NCCL log
that reports the exchange's algorithm (no GPU)."""

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
