"""Deterministic token-choice MoE (reference batch_invariant_ops/moe.py:11-92)."""

from __future__ import annotations

import torch


def deterministic_token_choice_moe(
    hidden_states: torch.Tensor,
    routing_weights: torch.Tensor,
    selected_experts: torch.Tensor,
    gate_weight: torch.Tensor,
    up_weight: torch.Tensor,
    down_weight: torch.Tensor,
    workspace: dict[str, torch.Tensor] | None = None,
) -> torch.Tensor:
    raise NotImplementedError
