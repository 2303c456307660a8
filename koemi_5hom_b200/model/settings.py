"""Model settings, mirroring ``koemi.configuration.settings.ModelSettings``.

Same fields, defaults and validation as src/koemi/configuration/settings.py:10-79,
so a reference settings object (or its ``to_dict()``) configures this model
unchanged. Three fields extend it for the B200 build and default to the
reference behaviour:

- ``layer_count``: HERM blocks stacked between the shared embedding and head
  (the reference is one block; >1 is the config-5 workload);
- ``compute_dtype``: "float32" (the reference's arithmetic) or "bfloat16"
  (bf16 weights and GEMM operands, fp32 accumulation, fp32 state);
- ``router_renormalize``: divide learned top-k weights by their sum (the
  reference keeps raw probabilities).
"""
from __future__ import annotations

import math
from dataclasses import asdict, dataclass
from typing import Any

BYTE_VOCABULARY_SIZE = 256
PAD_TOKEN_ID = BYTE_VOCABULARY_SIZE


@dataclass(frozen=True)
class ModelSettings:
    vocabulary_size: int = BYTE_VOCABULARY_SIZE + 1
    embedding_size: int = 64
    memory_features: int = 16
    local_memory_size: int = 16
    salience_memory_size: int = 16
    salience_threshold: float = 0.75
    expert_count: int = 0
    expert_top_k: int = 1
    expert_dispatch: str = "loop"
    cache_capacity: int = 256
    scan_chunk: int = 128
    activation_checkpointing: bool = False
    compile_forward: bool = False
    refine_decay_rate: float = 0.0625
    ablation: str = "no_refine"
    expert_routing: str = "hash"
    expert_load_balance_weight: float = 0.01
    layer_count: int = 1
    compute_dtype: str = "float32"
    router_renormalize: bool = False

    def __post_init__(self) -> None:
        rules = (
            (self.vocabulary_size >= BYTE_VOCABULARY_SIZE + 1, "vocabulary_size must cover every byte value and the padding token"),
            (self.embedding_size >= 8, "embedding_size must be at least 8"),
            (self.memory_features >= 2, "memory_features must be at least 2"),
            (self.local_memory_size >= 1, "local_memory_size must be at least 1"),
            (self.salience_memory_size >= 1, "salience_memory_size must be at least 1"),
            (0.0 <= self.salience_threshold <= 1.0, "salience_threshold must be between zero and one"),
            (self.scan_chunk >= 1, "scan_chunk must be at least 1"),
            (0 <= self.expert_count <= 128, "expert_count must be between 0 and 128"),
            (self.expert_top_k >= 1, "expert_top_k must be at least 1"),
            (self.expert_count == 0 or self.expert_top_k <= self.expert_count, "expert_top_k must not exceed expert_count"),
            (self.expert_dispatch in {"loop", "segments"}, "expert_dispatch must be loop or segments"),
            (self.expert_routing in {"hash", "learned"}, "expert_routing must be hash or learned"),
            (not (self.expert_routing == "learned" and (self.expert_count < 1 or self.ablation == "affine")),
             "learned routing requires experts and a non-affine ablation"),
            (math.isfinite(self.expert_load_balance_weight) and self.expert_load_balance_weight >= 0,
             "expert_load_balance_weight must be finite and non-negative"),
        )
        for passed, message in rules:
            if not passed:
                raise ValueError(message)
        for name in ("activation_checkpointing", "compile_forward"):
            if not isinstance(getattr(self, name), bool):
                raise TypeError(f"{name} must be a boolean")
        extra = (
            (self.cache_capacity >= 1, "cache_capacity must be at least 1"),
            (0.0 < self.refine_decay_rate <= 1.0, "refine_decay_rate must be greater than zero and at most one"),
            (self.ablation in {"herm", "no_refine", "no_surprise", "affine"},
             "ablation must be herm, no_refine, no_surprise or affine"),
            (self.layer_count >= 1, "layer_count must be at least 1"),
            (self.compute_dtype in {"float32", "bfloat16"}, "compute_dtype must be float32 or bfloat16"),
        )
        for passed, message in extra:
            if not passed:
                raise ValueError(message)

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)

    @classmethod
    def from_dict(cls, values: dict[str, Any]) -> "ModelSettings":
        return cls(**values)

    @classmethod
    def coerce(cls, settings: Any) -> "ModelSettings":
        """Accept this class, the reference's ModelSettings or a dict."""
        if isinstance(settings, cls):
            return settings
        values = settings if isinstance(settings, dict) else settings.to_dict()
        known = cls.__dataclass_fields__
        return cls(**{k: v for k, v in values.items() if k in known})
