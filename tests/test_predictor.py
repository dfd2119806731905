"""zmoe.predictor.ExpertPredictor against predictions recorded from the
reference's own experts/expert_predictor.py (tests/golden/predictor_cases.json)."""
import json
import os

from zmoe.predictor import ExpertPredictor

GOLD = os.path.join(os.path.dirname(__file__), "golden", "predictor_cases.json")


def test_predictions_match_reference_replay():
    cases = json.load(open(GOLD))
    assert cases
    for case in cases:
        p = ExpertPredictor(case["layers"], case["topk"], window_size=case["window"])
        for st in case["steps"]:
            p.update(st["layer"], st["experts"])
            nl, got = p.predict_next_layer(st["layer"])
            assert nl == st["next"] and got == st["predicted"], (case["layers"], st)


def test_empty_and_topk_zero():
    p = ExpertPredictor(2, 0)
    assert p.predict_next_layer(0) == (1, [])
    p.update(1, [3, 1])
    assert p.predict_next_layer(0) == (1, [])
    q = ExpertPredictor(2, 5)
    assert q.predict_next_layer(1) == (0, [])
