"""Model description types shared with the reference runners.

Same fields and weight naming as src/plastic_infer/exec/runner.py:35-51, 109-143 so
reference weight dicts and configs can be passed unchanged.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F


@dataclass
class ModelConfig:
    n_layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    hidden_dim: int
    intermediate_dim: int
    vocab_size: int
    max_seq_len: int
    rope_base: float = 10000.0
    dtype: torch.dtype = torch.float32
    qk_norm: bool = False
    n_experts: int = 0
    n_experts_per_tok: int = 0


class DenseWeights:
    """Weights keyed like the reference ("layers.{i}.self_attn.q_proj.weight", ...)."""

    def __init__(self, weights: dict[str, torch.Tensor]) -> None:
        self.w = weights
        first = next(iter(weights.values()))
        self.dtype = first.dtype
        self.device = first.device

    def __getitem__(self, key: str) -> torch.Tensor:
        return self.w[key]


def linear(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """x @ weight.T (nn.Linear layout)."""
    return F.linear(x, weight)
