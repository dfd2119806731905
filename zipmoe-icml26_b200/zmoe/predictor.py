"""Next-layer expert prediction for prefetching.

Restates ``ExpertPredictor`` (``experts/expert_predictor.py:11-45``): per
sparse layer, a running count of how often each expert was activated, plus a
bounded history of (layer, activated experts).  The prediction for the layer
after ``current`` ranks that layer's experts by

    0.8 * (activations so far) + 0.2 * (activations in its last 5 visits)

and keeps the ``prefetcher_topk`` best; experts with equal scores keep the
order in which the layer first saw them.  The dispatcher's ``submit_prefetch``
(``zmoe_layer_prefetch``) decodes the predicted experts into the HBM cache
ahead of the layer.
"""
from __future__ import annotations

from collections import deque
from typing import Dict, Iterable, List, Tuple


class ExpertPredictor:
    def __init__(self, n_sparse_layers: int, prefetcher_topk: int, window_size: int = 26 * 6 * 10):
        if n_sparse_layers < 1:
            raise ValueError("n_sparse_layers must be >= 1")
        self.num_sparse_layers = n_sparse_layers
        self.prefetcher_topk = prefetcher_topk
        # per layer: expert -> activation count, in first-seen order
        self.counts: List[Dict[int, int]] = [dict() for _ in range(n_sparse_layers)]
        self.history: deque = deque(maxlen=window_size)

    def update(self, layer_id: int, expert_ids: Iterable[int]) -> None:
        ids = list(expert_ids)
        table = self.counts[layer_id]
        for e in ids:
            table[e] = table.get(e, 0) + 1
        self.history.append((layer_id, ids))

    def predict_next_layer(self, current_layer: int) -> Tuple[int, List[int]]:
        nxt = (current_layer + 1) % self.num_sparse_layers
        recent: Dict[int, int] = {}
        visits = 0
        for layer, ids in reversed(self.history):
            if layer != nxt:
                continue
            for e in ids:
                recent[e] = recent.get(e, 0) + 1
            visits += 1
            if visits == 5:
                break
        table = self.counts[nxt]
        order = {e: i for i, e in enumerate(table)}
        scored = [(0.8 * n + 0.2 * recent.get(e, 0), e) for e, n in table.items()]
        scored.sort(key=lambda se: (-se[0], order[se[1]]))
        return nxt, [e for _, e in scored[: max(self.prefetcher_topk, 0)]]
