"""The cache-pool planner (zmoe.cache_planning) against the outputs of the
reference's own runtime/cache_planning.py on the same inputs
(tests/golden/cache_planning_cases.json, made by tests/golden/make_golden.py).
The port keeps the reference's arithmetic order, so results must be equal,
not just close."""
import json
import os
import tempfile

import numpy as np
import pytest
import torch

from zmoe import cache_planning as cp

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def cases():
    with open(os.path.join(HERE, "golden", "cache_planning_cases.json")) as f:
        return json.load(f)


def test_calculate_prob_matches_reference(cases):
    for c in cases["calculate_prob"]:
        got = cp.calculate_prob(c["probs"])
        assert got == c["out"]
        assert abs(sum(got) - 1.0) < 1e-12


def test_delay_simu_matches_reference(cases):
    for c in cases["delay_simu"]:
        assert cp.delay_simu(*c["args"]) == c["out"]


def test_scale_to_k_matches_reference(cases):
    for c in cases["scale_to_k"]:
        got = cp.scale_to_k(c["probs"], c["k"])
        assert got.tolist() == c["out"]
        assert np.all(got < 1.0)


def test_coverage_to_weight_matches_reference(cases):
    for c in cases["coverage_to_weight"]:
        w = cp.coverage_to_weight(c["target"], c["k"])
        assert w == c["out"]
        assert all(0.0 < v < 1.0 for v in cp.weight_to_prob(w))


def test_plan_cache_matches_reference(cases):
    for c in cases["plan"]:
        a = c["args"]
        assert cp.obtain_dist_from_trace(a["batch_size"], c["trace"]) == c["dist"]
        ratio, feasible = cp.plan_cache(c["trace"], total_memory=c["total_memory"], **a)
        assert (ratio, feasible) == (c["ratio"], c["feasible"])
        # the reference's own call (runtime/model_offload.py:102-116) passes keywords and a file
        with tempfile.NamedTemporaryFile(suffix=".pt") as f:
            torch.save(c["trace"], f.name)
            assert cp.PlanCache(trace_path=f.name, total_memory=c["total_memory"], **a) == (ratio, feasible)


def test_coverage_to_weight_rejects_wrong_sum():
    with pytest.raises(ValueError):
        cp.coverage_to_weight([0.5, 0.5, 0.5], 2)


def test_decoded_slots_follow_the_pool():
    # the module's sizing: pool bytes per layer / decoded expert bytes, capped at E
    n = cp.decoded_slots(0.5, 183 * 2**30, 0.2, 24, 3, 2048 * 1408, 60)
    assert n == int(0.5 * (0.2 * 183 * 2**30 / 24) / (2 * 3 * 2048 * 1408)) < 60
    assert cp.decoded_slots(1.0, 10**15, 1.0, 1, 3, 10, 60) == 60
    assert cp.decoded_slots(0.0, 10**9, 0.5, 4, 3, 10, 60) == 0


def test_sm_slots_split_the_budget_with_decoded_slots():
    from zmoe import cache_planning as cp
    kw = dict(total_memory=180 * 2 ** 30, device_memory_ratio=0.5, num_sparse_layers=240, tensors_per_expert=3,
              num_elements_per_tensor=2048 * 1408, num_experts=60)
    full = cp.decoded_slots(0.5, **kw)
    sm = cp.sm_slots(0.5, **kw)
    budget = 0.5 * 180 * 2 ** 30 / 240
    assert full == int(0.5 * budget / (2 * 3 * 2048 * 1408))
    assert sm == min(60 - full, int(0.5 * budget / (3 * 2048 * 1408)))
    assert cp.sm_slots(1.0, **kw) == 0
