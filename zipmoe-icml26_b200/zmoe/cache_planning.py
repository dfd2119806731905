"""Cache-pool planning: which share of a layer's device-memory budget holds
fully decoded experts (the rest holds sign+mantissa planes only).

Restates the reference's ``runtime/cache_planning.py`` (called from
``runtime/model_offload.py:102-116`` when the caching algorithm is "ZipMoE").
The planned ``gpu_pool_ratio`` is what the ``ZipMoE`` module's
``zipmoe_prefetch_handle`` turns into decoded cache slots per layer:
``device memory * device_memory_ratio * gpu_pool_ratio / expert bytes / layers``.

The model:

* A routing trace gives, per batch and layer, expert invocation counts sorted
  in decreasing order; their average is the popularity curve.
* The curve is scaled so its entries sum to k (no entry above 1), turned into
  conditional-Poisson sampling weights (Chen, Dempster and Liu, Biometrika
  1994) and from there into independent inclusion probabilities.
* For each split of the budget, the most popular experts fill the full pool,
  the next ones the sign+mantissa pool.  The number of hits in each pool is a
  Poisson-binomial variable; conditioned on k experts being selected, the
  expected delay of a step is averaged over the (full, sign+mantissa) hit
  counts with a max(compute, IO) delay model.
* The split with the lowest delay on a 5-point centred moving average wins.

Every function keeps the reference's arithmetic order, so its results match
the reference's to the last bit on the same inputs (tests/golden).
The device's memory is a parameter (``total_memory``) instead of a query of
GPU 0, so the planner runs without a GPU.
"""
from __future__ import annotations

import os
from collections import Counter
from typing import List, Optional, Sequence, Tuple

import numpy as np


def calculate_prob(probs: Sequence[float]) -> List[float]:
    """Poisson-binomial distribution: entry j is the probability that exactly j
    of the independent events (probabilities ``probs``) happen.
    CalculateProb (runtime/cache_planning.py:18-31)."""
    out = np.zeros(len(probs) + 1)
    out[0] = 1.0
    for p in probs:
        # every entry from the previous distribution: j events before and this
        # one missing, or j - 1 before and this one happening
        out[1:] = out[1:] * (1 - p) + out[:-1] * p
        out[0] = out[0] * (1 - p)
    return out.tolist()


def delay_simu(k, num_full_cached, num_sm_cached, decompression_delay, SM_IO_delay, compression_ratio,
               num_file_chunks, tensors_per_expert, compute_pool_size) -> float:
    """Delay of one step with k experts, num_full_cached of them decoded in
    the pool and num_sm_cached with only their sign+mantissa plane there: the
    larger of the decompression work (exponent chunks of every non-decoded
    expert over the compute pool, each chunk also read) and the reads
    (whole planes of uncached experts, exponent planes of sign+mantissa-cached
    ones).  DelaySimu (runtime/cache_planning.py:34-51)."""
    chunks = num_file_chunks * (k - num_full_cached) * tensors_per_expert
    chunk_read = SM_IO_delay * compression_ratio / num_file_chunks
    compute = (chunks / compute_pool_size) * (decompression_delay + chunk_read)
    io = (tensors_per_expert * SM_IO_delay * (k - num_full_cached - num_sm_cached)
          + num_sm_cached * tensors_per_expert * SM_IO_delay * compression_ratio)
    return max(compute, io)


def _multiset_minus(a: Sequence[float], b: Sequence[float]) -> List[float]:
    """a minus b as multisets, in the order values first appear in a (with
    their remaining multiplicity), as collections.Counter subtraction gives."""
    left = Counter(a)
    left.subtract(Counter(b))
    out: List[float] = []
    for v in dict.fromkeys(a):
        out.extend([v] * max(left[v], 0))
    return out


def _centred_mean5(v: Sequence[float]) -> np.ndarray:
    """5-point centred moving average, shorter windows at the ends
    (pandas rolling(window=5, center=True, min_periods=1).mean())."""
    import pandas as pd
    return pd.Series(list(v)).rolling(window=5, center=True, min_periods=1).mean().to_numpy()


def cache_pool_planning_simu(k, num_experts, num_sparse_layers, tensors_per_expert, num_elements_per_tensor,
                             compression_ratio, num_file_chunks, compute_pool_size, device_memory_ratio,
                             decompression_delay, SM_IO_delay, all_probs, step_size=0.01,
                             total_memory: Optional[int] = None, trace: Optional[list] = None
                             ) -> Tuple[float, bool]:
    """Best share of the per-layer budget for fully decoded experts, and
    whether any split was feasible.  all_probs: inclusion probabilities in
    decreasing popularity.  total_memory: device bytes (default: the current
    CUDA device's).  trace, when a list, receives (ratio, expected delay) per
    split considered.  CachePoolPlanningSimu (runtime/cache_planning.py:54-139)."""
    if total_memory is None:
        import torch
        total_memory = torch.cuda.get_device_properties(torch.cuda.current_device()).total_memory
    budget = device_memory_ratio * total_memory / num_sparse_layers
    sm_slot = tensors_per_expert * num_elements_per_tensor
    full_slot = sm_slot * 2
    probs = list(all_probs)
    ratios, delays = [], []
    best_delay, best_ratio = float("inf"), 0
    feasible = False
    for ratio_full in [i * step_size for i in range(1, int(1 / step_size))]:
        n_full = int((ratio_full * budget) / full_slot)
        n_sm = int(((1 - ratio_full) * budget) / sm_slot)
        if n_full + n_sm > num_experts:
            continue
        if n_full * num_sparse_layers < num_experts or n_sm * num_sparse_layers < num_experts:
            continue
        feasible = True
        p_full = probs[:n_full]
        p_sm = probs[n_full:n_full + n_sm]
        d_full = calculate_prob(p_full)
        d_sm = calculate_prob(p_sm)
        d_rest = calculate_prob(_multiset_minus(probs, p_full + p_sm))
        total = np.convolve(np.convolve(d_full, d_sm), d_rest)
        p_k = total[k] if k < len(total) else 0
        if p_k <= 0:
            continue
        expected = 0
        for full_hit in range(len(d_full)):
            for sm_hit in range(len(d_sm)):
                if full_hit + sm_hit > k:
                    continue
                r = k - (full_hit + sm_hit)
                if r >= len(d_rest):
                    continue
                prob = (d_full[full_hit] * d_sm[sm_hit] * d_rest[r]) / p_k
                expected += prob * delay_simu(k, full_hit, sm_hit, decompression_delay, SM_IO_delay,
                                              compression_ratio, num_file_chunks, tensors_per_expert,
                                              compute_pool_size)
        ratios.append(ratio_full)
        delays.append(expected)
        if trace is not None:
            trace.append((ratio_full, expected))
        if expected < best_delay and ratio_full >= 0.3:
            best_delay, best_ratio = expected, ratio_full
    if best_delay == float("inf"):
        return 1.0 - step_size, feasible
    smooth = _centred_mean5(delays)
    return ratios[int(np.argmin(smooth))], feasible


def obtain_dist_from_trace(batch_size: int, trace_path) -> List[float]:
    """Popularity curve from a routing trace: trace_path is a file torch.load
    reads, or the trace itself, trace[prompt][layer][expert] = invocation count.  Per batch of
    prompts and per layer the summed counts are sorted in decreasing order;
    the curves of all layers and batches are summed and normalised to 1
    (a trailing partial batch is dropped); sums run in the reference's order.
    ObtainDistFromTrace (runtime/cache_planning.py:142-162)."""
    trace = trace_path
    if isinstance(trace, (str, bytes, os.PathLike)):
        import torch
        trace = torch.load(trace, map_location="cpu")
    t = np.asarray(trace)
    if t.ndim != 3:
        raise ValueError(f"trace must be [prompts][layers][experts], got shape {t.shape}")
    n_batches = t.shape[0] // batch_size
    curve = np.zeros(t.shape[2], dtype=t.dtype)
    for b in range(n_batches):
        batch = np.zeros(t.shape[2], dtype=t.dtype)
        for layer in range(t.shape[1]):
            inv = np.zeros(t.shape[2], dtype=t.dtype)
            for i in range(batch_size):
                inv = inv + t[b * batch_size + i, layer]
            batch = batch + -np.sort(-inv, kind="stable")
        curve = curve + batch
    total = sum(curve.tolist())
    return [p / total for p in curve.tolist()]


def scale_to_k(probs: Sequence[float], k: int, tol: float = 1e-9) -> np.ndarray:
    """Scales probs to sum to k with no entry above 1 - tol: entries that would
    pass it are pinned there and the rest rescaled to the remaining sum.
    scale_to_k (runtime/cache_planning.py:231-257)."""
    pi = np.array(probs, dtype=float)
    if np.sum(pi) == 0:
        return pi
    pi = pi * (k / np.sum(pi))
    rest = np.arange(len(pi))
    left = float(k)
    while len(rest) > 0:
        s = np.sum(pi[rest])
        if s < tol:
            break
        scaled = pi[rest] * (left / s)
        over = rest[scaled >= 1.0 - tol]
        if len(over) == 0:
            pi[rest] = scaled
            break
        pi[over] = 1.0 - tol
        left -= len(over)
        rest = rest[~np.isin(rest, over)]
        if left <= 0:
            pi[rest] = 0.0
            break
    return pi


def coverage_to_weight(target_probs: Sequence[float], k: int, max_iter: int = 50, tol: float = 1e-8) -> List[float]:
    """Conditional-Poisson sampling weights w whose inclusion probabilities in
    a sample of k are target_probs (which must sum to k), by the fixed-point
    update w <- w * target / current of Chen, Dempster and Liu (1994).  The
    inclusion probability of item i is w_i * E_{-i}(k - 1) / E(k), with E the
    elementary symmetric sums of the weights, from a forward and a backward
    recursion.  CoverageToWeight (runtime/cache_planning.py:167-220)."""
    pi = np.array(target_probs)
    n = len(pi)
    if not np.isclose(np.sum(pi), k):
        raise ValueError(f"target probabilities sum to {np.sum(pi)}, not k = {k}")
    w = pi / (1.0 - pi + 1e-12)
    for _ in range(max_iter):
        fwd = np.zeros((n + 1, k + 1))                 # fwd[j][m]: sum over m-subsets of the first j items
        fwd[:, 0] = 1.0
        for j in range(1, n + 1):
            fwd[j, 1:] = fwd[j - 1, 1:] + w[j - 1] * fwd[j - 1, :-1]
        bwd = np.zeros((n + 2, k + 1))                 # bwd[j][m]: ... of items j .. n (1-based)
        bwd[:, 0] = 1.0
        for j in range(n, 0, -1):
            bwd[j, 1:] = bwd[j + 1, 1:] + w[j - 1] * bwd[j + 1, :-1]
        without = np.zeros(n)                          # E_{-i}(k - 1), summed over the split point m in order
        for m in range(k):
            without = without + fwd[:n, m] * bwd[2:n + 2, k - 1 - m]
        current = w * without / fwd[n][k]
        if np.linalg.norm(current - pi) < tol:
            return w.tolist()
        w = w * (pi / (current + 1e-12))
        w /= np.mean(w)
    return w.tolist()


def weight_to_prob(weight: Sequence[float]) -> List[float]:
    """Inclusion probability w / (1 + w) of each weight (WeightToProb,
    runtime/cache_planning.py:260-261)."""
    return [w / (1 + w) for w in weight]


def plan_cache(trace_path, batch_size, k, num_experts, num_sparse_layers, tensors_per_expert, num_elements_per_tensor,
               compression_ratio, num_file_chunks, compute_pool_size, device_memory_ratio, decompression_delay,
               SM_IO_delay, step_size=0.05, synthetic=False, total_memory: Optional[int] = None
               ) -> Tuple[float, bool]:
    """gpu_pool_ratio for zipmoe_prefetch_handle from a routing trace
    (trace_path: a file, or the [prompts][layers][experts] count array itself), and whether the budget
    allows a split at all (0.99 when it does not).  PlanCache
    (runtime/cache_planning.py:264-303)."""
    curve = obtain_dist_from_trace(batch_size, trace_path)
    target = scale_to_k(curve, k)
    probs = weight_to_prob(coverage_to_weight(target, k))
    avg_k = int(np.sum(probs))
    best, feasible = cache_pool_planning_simu(avg_k, num_experts, num_sparse_layers, tensors_per_expert,
                                              num_elements_per_tensor, compression_ratio, num_file_chunks,
                                              compute_pool_size, device_memory_ratio, decompression_delay,
                                              SM_IO_delay, probs, step_size, total_memory=total_memory)
    return (best if feasible else 0.99), feasible


def decoded_slots(gpu_pool_ratio: float, total_memory: int, device_memory_ratio: float, num_sparse_layers: int,
                  tensors_per_expert: int, num_elements_per_tensor: int, num_experts: int) -> int:
    """Decoded experts per layer that a gpu_pool_ratio gives: the same sizing
    the ZipMoE module's handle applies (BF16 experts, all layers sharing the
    budget).  The reference's full pool
    (runtime/cache_planning.py:71-74, 88)."""
    budget = device_memory_ratio * total_memory / num_sparse_layers
    return max(0, min(num_experts, int(gpu_pool_ratio * budget / (2 * tensors_per_expert * num_elements_per_tensor))))


def sm_slots(gpu_pool_ratio: float, total_memory: int, device_memory_ratio: float, num_sparse_layers: int,
             tensors_per_expert: int, num_elements_per_tensor: int, num_experts: int) -> int:
    """Experts per layer whose sign+mantissa planes (1 byte per element) the
    rest of the budget holds: the reference's SM pool,
    int((1 - ratio_full) * total_mem / sm_slot_size) (runtime/cache_planning.py:71-88).
    MoELayer(store="host", sm_slots=...) keeps that many planes in HBM."""
    budget = device_memory_ratio * total_memory / num_sparse_layers
    full = decoded_slots(gpu_pool_ratio, total_memory, device_memory_ratio, num_sparse_layers, tensors_per_expert,
                         num_elements_per_tensor, num_experts)
    n = int((1.0 - gpu_pool_ratio) * budget / (tensors_per_expert * num_elements_per_tensor))
    return max(0, min(num_experts - full, n))


# the reference's names
CalculateProb = calculate_prob
DelaySimu = delay_simu
CachePoolPlanningSimu = cache_pool_planning_simu
ObtainDistFromTrace = obtain_dist_from_trace
CoverageToWeight = coverage_to_weight
WeightToProb = weight_to_prob
PlanCache = plan_cache
