"""Recurrent state, mirroring ``koemi.model.state`` (src/koemi/model/state.py:11-94).

``KoemiState`` keeps the reference's 12 tensor fields, their order, shapes and
dtypes (fp32 memories, bool validity, int64 ids) plus ``step_index``, so the
reference's decode helpers (``to_static_state``, ``clone_state``,
``select_state_rows``, ``stack_states``) work on it unchanged.
``LayeredKoemiState`` carries one ``KoemiState`` per HERM block when
``layer_count > 1``.
"""
from __future__ import annotations

from dataclasses import dataclass, replace

import torch
from torch import Tensor

from koemi_5hom_b200.model.settings import PAD_TOKEN_ID

KOEMI_STATE_FIELDS = (
    "working_state",
    "memory_basis",
    "memory_normalizer",
    "refine_basis",
    "refine_normalizer",
    "local_keys",
    "local_values",
    "local_valid",
    "salient_keys",
    "salient_values",
    "salient_valid",
    "last_token_ids",
)


@dataclass(frozen=True)
class KoemiState:
    working_state: Tensor
    memory_basis: Tensor
    memory_normalizer: Tensor
    refine_basis: Tensor
    refine_normalizer: Tensor
    local_keys: Tensor
    local_values: Tensor
    local_valid: Tensor
    salient_keys: Tensor
    salient_values: Tensor
    salient_valid: Tensor
    last_token_ids: Tensor
    step_index: int

    @classmethod
    def create_static(cls, batch_size: int, embedding_size: int, memory_features: int, local_memory_size: int,
                      salience_memory_size: int, device: torch.device, dtype: torch.dtype = torch.float32) -> "KoemiState":
        """Empty state whose rings already hold their capacity (zero, invalid)."""
        if local_memory_size < 1 or salience_memory_size < 1:
            raise ValueError("static state requires positive ring capacities")
        return cls._build(batch_size, embedding_size, memory_features, local_memory_size, salience_memory_size,
                          device, dtype)

    @classmethod
    def create(cls, batch_size: int, embedding_size: int, memory_features: int, device: torch.device) -> "KoemiState":
        """Empty state with zero-length rings that grow up to capacity."""
        return cls._build(batch_size, embedding_size, memory_features, 0, 0, device, torch.float32)

    @classmethod
    def _build(cls, batch, width, features, local, salient, device, dtype) -> "KoemiState":
        zeros = lambda *shape: torch.zeros(*shape, device=device, dtype=dtype)  # noqa: E731
        flags = lambda n: torch.zeros(batch, n, dtype=torch.bool, device=device)  # noqa: E731
        return cls(
            working_state=zeros(batch, width),
            memory_basis=zeros(batch, width, features),
            memory_normalizer=zeros(batch, features),
            refine_basis=zeros(batch, width, features),
            refine_normalizer=zeros(batch, features),
            local_keys=zeros(batch, local, width),
            local_values=zeros(batch, local, width),
            local_valid=flags(local),
            salient_keys=zeros(batch, salient, width),
            salient_values=zeros(batch, salient, width),
            salient_valid=flags(salient),
            last_token_ids=torch.full((batch,), PAD_TOKEN_ID, dtype=torch.long, device=device),
            step_index=0,
        )


@dataclass(frozen=True)
class LayeredKoemiState:
    """One ``KoemiState`` per stacked HERM block (``layer_count > 1``)."""

    layers: tuple[KoemiState, ...]
    step_index: int

    @property
    def working_state(self) -> Tensor:  # row count for callers that inspect it
        return self.layers[-1].working_state

    def with_step(self, step_index: int) -> "LayeredKoemiState":
        return replace(self, step_index=step_index,
                       layers=tuple(replace(layer, step_index=step_index) for layer in self.layers))
