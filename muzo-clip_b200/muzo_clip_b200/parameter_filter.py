"""Which parameters MuZO-Clip updates (mirror of muzo_clip/parameter_filter.py).

The rule and the default token lists must match the reference exactly: the selected names, in
``named_parameters()`` order, feed the noise keys of every block.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Iterable

import torch

# Projection matrices of a decoder layer (parameter_filter.py:10-18).
DEFAULT_TRAINABLE_SUBSTRINGS = (
    "q_proj",
    "k_proj",
    "v_proj",
    "o_proj",
    "gate_proj",
    "up_proj",
    "down_proj",
)

# Never selected, even when a trainable token matches (parameter_filter.py:20-27).
DEFAULT_FROZEN_SUBSTRINGS = (
    "embed_tokens",
    "lm_head",
    "norm",
    "bias",
    "layernorm",
    "ln_",
)


@dataclass(frozen=True)
class SelectedParameter:
    name: str
    param: torch.nn.Parameter


def should_select_parameter(
    name: str,
    param: torch.Tensor,
    trainable_substrings: Iterable[str] = DEFAULT_TRAINABLE_SUBSTRINGS,
    frozen_substrings: Iterable[str] = DEFAULT_FROZEN_SUBSTRINGS,
) -> bool:
    """2-D, name contains a trainable token and no frozen token (case-insensitive)."""

    if param.ndim != 2:
        return False
    key = name.lower()
    if not any(tok.lower() in key for tok in trainable_substrings):
        return False
    return not any(tok.lower() in key for tok in frozen_substrings)


def select_muzo_parameters(
    model: torch.nn.Module,
    trainable_substrings: Iterable[str] = DEFAULT_TRAINABLE_SUBSTRINGS,
    frozen_substrings: Iterable[str] = DEFAULT_FROZEN_SUBSTRINGS,
) -> list[SelectedParameter]:
    """Selected parameters of ``model`` in ``named_parameters()`` order."""

    trainable = tuple(trainable_substrings)
    frozen = tuple(frozen_substrings)
    return [
        SelectedParameter(name=name, param=param)
        for name, param in model.named_parameters()
        if should_select_parameter(name, param, trainable, frozen)
    ]
