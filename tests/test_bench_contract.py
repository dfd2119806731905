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


def test_reference_arm_loads_no_product_library():
    """The reference arm encodes and runs through the oracle (liblz4 + torch
    CPU) only: nothing in its process may load libzmoe.so."""
    import inspect
    import subprocess
    src = inspect.getsource(bench.run_reference) + inspect.getsource(bench.cpu_reference_layer)
    for banned in ("zmoe import codec", "zmoe.codec", "zmoe.layer", "zmoe._lib", "zmoe import ops", "build_workload"):
        assert banned not in src, banned
    code = ("import sys; sys.path[:0] = [%r, %r]; import bench; from oracle import codec, reference_cpu; "
            "from zmoe import synthetic; import torch; "
            "t = synthetic.expert_weights(synthetic.LayerShape(256, 2, 64, 1), 1)[0][0]; "
            "codec.encode_tensors(t, 3, 'LZ4HC', 9, 2); "
            "maps = open('/proc/self/maps').read(); print('libzmoe' in maps)") % (ROOT, os.path.join(ROOT, "zipmoe-icml26_b200"))
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr
    assert out.stdout.strip().splitlines()[-1] == "False"


def test_both_arms_print_the_same_config(monkeypatch):
    from zmoe import synthetic as syn
    monkeypatch.setattr(sys, "argv", ["bench.py"])
    a = bench.parse()
    c1 = bench.bench_config(a, syn.QWEN, 1)
    assert c1 == bench.bench_config(a, syn.QWEN, 1)
    assert c1["workload"] == "qwen1.5-moe-layer" and c1["parallelism"] == "single"
    assert bench.bench_config(a, syn.QWEN, 8)["parallelism"] == "ep8"
