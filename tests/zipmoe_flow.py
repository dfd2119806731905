"""Test helper: drives the `ZipMoE` module the way the reference's Python does
(runtime/model_offload.py offload + experts/expert_executor.py dispatch_local)."""
from __future__ import annotations

import numpy as np
import torch

from oracle import codec as oc


def split_exp_chunks(t: torch.Tensor, num_file_chunks: int):
    """split_and_extract_from_tensor (runtime/model_offload.py:706-726): exponent
    plane cut into ceil(n/c)-element chunks, and the sign+mantissa plane."""
    bits = oc.bf16_bits(t)
    exp, sm = oc.split_planes(bits)
    per = -(-exp.size // num_file_chunks)
    return [np.ascontiguousarray(exp[i * per:(i + 1) * per]) for i in range(num_file_chunks)], sm


def make_handle(ZipMoE, folder, E, layers, per_expert, numel, topk, cache_ratio=0.0, code="LZ4HC",
                policy="LFU", chunks=3):
    return ZipMoE.zipmoe_prefetch_handle(
        folder, "zipmoe_param", code, policy, 0.5, cache_ratio, 0.01, 0.01, 4, chunks, 0, topk, numel,
        per_expert, layers, E, 5, 9, 3, 0.1, False)


def dispatch_local(dispatcher, hidden, router_mask, layer_id):
    """experts/expert_executor.py:40-84 without the predictor."""
    num_expert = router_mask.shape[-1]
    expert_count = torch.sum(router_mask.view((-1, num_expert)), dim=0).cpu().numpy().flatten()
    expert_list = np.arange(num_expert).astype(int)[expert_count > 0].tolist()
    dispatcher.set_inputs(hidden, router_mask)
    dispatcher.set_expected_queue(len(expert_list))
    counts = expert_count[expert_count > 0].tolist()
    for i, e in enumerate(expert_list):
        dispatcher.enqueue_expert(layer_id, e, int(counts[i]))
    dispatcher.ops_schedule()
    return dispatcher.wait_expert()
