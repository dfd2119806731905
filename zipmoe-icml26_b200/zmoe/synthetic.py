"""Seeded synthetic MoE workloads (no checkpoints or datasets are used).

All tensors are drawn on the CPU with ``torch.Generator().manual_seed(seed)``
in float32 and rounded to BF16 (round to nearest even), so every machine
produces the same bytes.  Seeds: expert weights 0 (order layer -> expert ->
tensor), activations 1, router weights 2, the Zipf permutation of layer l is
seed 3 + l.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import torch


@dataclass(frozen=True)
class LayerShape:
    """Shapes of one MoE layer.  ``kind`` 0 = SwiGLU experts (Qwen/DeepSeek),
    1 = ReLU experts (Switch)."""
    hidden: int
    num_experts: int
    inter: int
    topk: int
    kind: int = 0
    shared_inter: int = 0           # 0 = no shared expert
    shared_gate: bool = False       # Qwen sigmoid gate on the shared expert
    scaling: float = 1.0            # DeepSeek routed_scaling_factor
    capacity: int = 0               # Switch expert capacity (per sequence)
    seq_len: int = 0                # Switch sequence length for the capacity count
    zipf_s: float = 0.0             # router logit bias -s*ln(rank)

    @property
    def tensors_per_expert(self) -> int:
        return 3 if self.kind == 0 else 2

    @property
    def elements_per_tensor(self) -> int:
        return self.hidden * self.inter


QWEN = LayerShape(2048, 60, 1408, 4, 0, 5632, True, 1.0, 0, 0, 1.0)
DEEPSEEK = LayerShape(2048, 64, 1408, 6, 0, 2816, False, 1.0, 0, 0, 1.2)
SWITCH = LayerShape(1024, 128, 2816, 1, 1, 0, False, 1.0, 40, 4096, 0.0)


def normal_bf16(shape, std: float, gen: torch.Generator) -> torch.Tensor:
    return (torch.randn(*shape, generator=gen, dtype=torch.float32) * std).to(torch.bfloat16)


def expert_shapes(s: LayerShape) -> List[Tuple[int, int]]:
    if s.kind == 0:
        return [(s.inter, s.hidden), (s.inter, s.hidden), (s.hidden, s.inter)]
    return [(s.inter, s.hidden), (s.hidden, s.inter)]


def expert_weights(s: LayerShape, num_layers: int = 1, std: float = 0.02, seed: int = 0,
                   experts: Optional[Sequence[int]] = None) -> List[List[List[torch.Tensor]]]:
    """weights[layer][expert] = [gate, up, down] or [wi, wo] (BF16, row-major)."""
    gen = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(num_layers):
        layer = []
        for e in range(s.num_experts):
            ts = [normal_bf16(shp, std, gen) for shp in expert_shapes(s)]
            layer.append(ts)
        out.append(layer)
    return out


def shared_weights(s: LayerShape, std: float = 0.02, seed: int = 4) -> Optional[List[torch.Tensor]]:
    if not s.shared_inter:
        return None
    gen = torch.Generator().manual_seed(seed)
    return [normal_bf16((s.shared_inter, s.hidden), std, gen),
            normal_bf16((s.shared_inter, s.hidden), std, gen),
            normal_bf16((s.hidden, s.shared_inter), std, gen)]


def router_weights(s: LayerShape, std: float = 0.02, seed: int = 2) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """(router [E, H], shared-expert gate [1, H] or None), BF16."""
    gen = torch.Generator().manual_seed(seed)
    wr = normal_bf16((s.num_experts, s.hidden), std, gen)
    sg = normal_bf16((1, s.hidden), std, gen) if s.shared_gate else None
    return wr, sg


def zipf_bias(s: LayerShape, layer: int = 0) -> Optional[torch.Tensor]:
    """Per-expert fp32 logit bias b_e = -s * ln(rank_e), rank from a seeded
    permutation, so expert popularity follows Zipf(s)."""
    if s.zipf_s <= 0:
        return None
    gen = torch.Generator().manual_seed(3 + layer)
    perm = torch.randperm(s.num_experts, generator=gen)
    rank = torch.empty(s.num_experts, dtype=torch.float32)
    rank[perm] = torch.arange(1, s.num_experts + 1, dtype=torch.float32)
    return (-s.zipf_s * torch.log(rank)).to(torch.float32)


def activations(tokens: int, hidden: int, seed: int = 1) -> torch.Tensor:
    gen = torch.Generator().manual_seed(seed)
    return torch.randn(tokens, hidden, generator=gen, dtype=torch.float32).to(torch.bfloat16)


def popularity_order(s: LayerShape, layer: int = 0) -> List[int]:
    """Experts from most to least popular under the Zipf bias."""
    b = zipf_bias(s, layer)
    if b is None:
        return list(range(s.num_experts))
    return sorted(range(s.num_experts), key=lambda e: (-float(b[e]), e))
