"""Seeded HERM-block parameters under the reference's state-dict names.

Both the golden-fixture generator (which loads them into the reference
``KoemiModel``) and the tests (which load them into the oracle and into the
B200 model) call :func:`herm_parameters`, so a fixture records only the
settings and the seed, never the weights themselves.

Parameter names and shapes follow ``KoemiModel.__init__``
(src/koemi/model/network.py:80-106) and its submodules.

``init="uniform"`` draws Linear weights and biases from U(-1/sqrt(fan_in),
1/sqrt(fan_in)) (the scale of torch's default Linear init), the embedding from
N(0, 1) and norm weights as 1 + 0.05 N(0, 1). ``init="normal"`` draws every
Linear weight from N(0, 0.02), biases from N(0, 0.002), the embedding from
N(0, 1) and norm weights as above (the config-5 recipe). The padding row of
the embedding is zero, as with ``padding_idx``.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

PAD_TOKEN_ID = 256


@dataclass(frozen=True)
class HermShape:
    vocabulary_size: int = 257
    embedding_size: int = 256
    memory_features: int = 16
    expert_count: int = 4
    expert_routing: str = "hash"
    ablation: str = "no_refine"


def parameter_shapes(shape: HermShape) -> list[tuple[str, tuple[int, ...], str]]:
    """(name, shape, kind) in a fixed order; kind is linear_w/linear_b/embed/norm."""
    v, d, m, e = shape.vocabulary_size, shape.embedding_size, shape.memory_features, shape.expert_count
    out: list[tuple[str, tuple[int, ...], str]] = [("embedding.weight", (v, d), "embed"),
                                                   ("input_normalizer.weight", (d,), "norm")]

    def linear(name: str, rows: int, cols: int, bias: bool = True) -> None:
        out.append((f"{name}.weight", (rows, cols), "linear_w"))
        if bias:
            out.append((f"{name}.bias", (rows,), "linear_b"))

    linear("recurrent_state.retention_projection", d, d)
    linear("recurrent_state.candidate_projection", d, d)
    linear("associative_memory.key_projection", d, d)
    linear("associative_memory.query_projection", d, d)
    linear("associative_memory.value_projection", d, d)
    linear("associative_memory.feature_projection", m, d)
    linear("associative_memory.decay_projection", 1, d)
    linear("associative_memory.write_projection", 1, d)
    linear("local_memory.local_key_projection", d, d)
    linear("local_memory.local_value_projection", d, d)
    if shape.ablation != "no_refine":
        linear("memory_refine_gate", 1, 4 * d)
    linear("fusion_projection", d, 4 * d)
    out.append(("fusion_normalizer.weight", (d,), "norm"))
    for index in range(e):
        linear(f"experts.experts.{index}.value_projection", 2 * d, d)
        linear(f"experts.experts.{index}.gate_projection", 2 * d, d)
        linear(f"experts.experts.{index}.output_projection", d, 2 * d)
    if e > 0:
        out.append(("experts.output_normalizer.weight", (d,), "norm"))
    if shape.expert_routing == "learned" and e > 0:
        linear("experts.gate", e, d, bias=False)
    linear("token_predictor", v, d)
    return out


def herm_parameters(shape: HermShape, seed: int, init: str = "uniform",
                    dtype: torch.dtype = torch.float32) -> dict[str, torch.Tensor]:
    """Deterministic parameters (CPU tensors) keyed by reference state-dict name.

    ``dtype`` is applied last (bf16 rounding for the bf16 configurations); the
    values themselves are always drawn in fp32 from one CPU generator.
    """
    generator = torch.Generator().manual_seed(seed)
    params: dict[str, torch.Tensor] = {}
    fan_in = {}
    for name, dims, kind in parameter_shapes(shape):
        if kind == "linear_w":
            fan_in[name.rsplit(".", 1)[0]] = dims[1]
    for name, dims, kind in parameter_shapes(shape):
        if kind == "embed":
            value = torch.randn(dims, generator=generator)
            if PAD_TOKEN_ID < dims[0]:
                value[PAD_TOKEN_ID] = 0.0
        elif kind == "norm":
            value = 1.0 + 0.05 * torch.randn(dims, generator=generator)
        elif init == "uniform":
            bound = fan_in[name.rsplit(".", 1)[0]] ** -0.5
            value = (torch.rand(dims, generator=generator) * 2.0 - 1.0) * bound
        elif init == "normal":
            std = 0.02 if kind == "linear_w" else 0.002
            value = torch.randn(dims, generator=generator) * std
        else:
            raise ValueError(f"unknown init {init!r}")
        params[name] = value.to(dtype)
    return params
