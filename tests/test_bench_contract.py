"""bench.py defaults and helpers that the benchmark contract relies on, checked
without a GPU."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_defaults_are_one_gpu_and_enough_warmup(monkeypatch):
    monkeypatch.setattr(sys, "argv", ["bench.py"])
    a = bench.parse()
    assert a.gpus == 1 and a.impl == "ours" and a.store == "device"
    assert a.warmup >= 3 and a.steps >= 1
    assert a.tokens == 512 and a.cache == 16 and a.chunks == 3 and a.codec == "LZ4HC" and a.level == 9


def test_clock_sampler_is_inert_without_a_device():
    # ranks other than 0 pass None: no driver query, no probe, no summary
    with bench.ClockSampler(None) as clk:
        for i in range(10):
            clk.probe(i, 10)
    assert clk.summary() is None
    assert clk.edges == [] and clk.probes == []


def test_metric_and_unit():
    assert bench.METRIC == "MoE-layer tokens/s" and bench.UNIT == "tokens/s"
