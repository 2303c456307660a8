"""Expert parallelism: shard bookkeeping, and the all-to-all exchange on CPU
gloo ranks (world size 2 and 4) against the single-rank grouped MLP."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from koemi_5hom_b200.model import KoemiModel, ModelSettings
from koemi_5hom_b200.model.expert_parallel import ExpertOps, ExpertShard, expert_parallel_mlp
from oracle import ops


def test_shard_bookkeeping():
    shard = ExpertShard(world=4, rank=2, expert_count=64)
    assert shard.local_count == 16 and shard.first == 32
    with pytest.raises(ValueError):
        ExpertShard(world=3, rank=0, expert_count=64)
    with pytest.raises(ValueError):
        ExpertShard(world=2, rank=2, expert_count=64)


def test_sharded_model_holds_the_rows_of_the_full_model():
    settings = ModelSettings(vocabulary_size=300, embedding_size=64, memory_features=8, expert_count=8,
                             expert_top_k=2, layer_count=2)
    full = KoemiModel(settings)
    full.initialize_parameters(3)
    for rank in range(4):
        shard = KoemiModel(settings, expert_shard=ExpertShard(4, rank, 8))
        shard.initialize_parameters(3)
        for block, reference in zip(shard.blocks, full.blocks):
            for mine, theirs in zip(block.expert_weights(), reference.expert_weights()):
                assert torch.equal(mine, theirs[2 * rank:2 * rank + 2])
            assert torch.equal(block.gates_weight, reference.gates_weight)
            names = [n for n, *_ in block.reference_map(settings) if n.startswith("experts.experts.")]
            assert sorted({int(n.split(".")[2]) for n in names}) == [2 * rank, 2 * rank + 1]
    with pytest.raises(ValueError):
        KoemiModel(settings, expert_shard=ExpertShard(2, 0, 16))


def _oracle_ops() -> ExpertOps:
    return ExpertOps(permute_topk=ops.permute_rows, grouped_mlp=ops.grouped_mlp, pack=ops.ep_pack,
                     unpack=ops.ep_unpack)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, experts: int, top_k: int) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        width, hidden = 12, 20
        g = torch.Generator().manual_seed(7)  # the same expert weights on every rank
        weights = [torch.randn(*shape, generator=g, dtype=torch.float64) * 0.3 for shape in
                   ((experts, hidden, width), (experts, hidden), (experts, hidden, width), (experts, hidden),
                    (experts, width, hidden), (experts, width))]
        shard = ExpertShard(world, rank, experts)
        local = tuple(w[shard.first:shard.first + shard.local_count] for w in weights)
        tokens = 9 + 4 * rank  # ragged: every rank brings a different number of tokens
        t = torch.Generator().manual_seed(100 + rank)
        rows = torch.randn(tokens, width, generator=t, dtype=torch.float64)
        assignments = torch.randint(-1, experts + 1, (tokens, top_k), generator=t)
        if top_k > 1:
            assignments[::3, 1] = assignments[::3, 0]  # repeated slots are dropped
        valid = torch.rand(tokens, generator=t) > 0.2
        sorted_rows, _, sorted_experts, offsets, _ = ops.permute_rows(rows, assignments, valid, experts)
        expected = ops.grouped_mlp(sorted_rows, sorted_experts, offsets, *weights)
        capacity = (9 + 4 * (world - 1)) * top_k  # the largest rank's pairs, the same on every rank
        for mode in ("padded", "exact"):
            got = expert_parallel_mlp(shard, sorted_rows, sorted_experts, offsets, local, mode=mode,
                                      ops=_oracle_ops(), capacity=capacity)
            torch.testing.assert_close(got, expected, rtol=1e-12, atol=1e-12)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,experts,top_k", [(2, 8, 2), (4, 8, 3), (2, 2, 1)])
def test_exchange_equals_single_rank_mlp(world, experts, top_k):
    mp.spawn(_rank_main, args=(world, _free_port(), experts, top_k), nprocs=world, join=True)


def test_nccl_exchange_is_refused_inside_graph_capture(monkeypatch):
    """The NCCL all-to-all exchange stays out of CUDA graphs: expert_mlp
    refuses it while the stream is capturing, before any collective, and the
    decoder refuses to capture a model that uses it."""
    from koemi_5hom_b200.runtime import BatchDecoder
    settings = ModelSettings(vocabulary_size=300, embedding_size=64, memory_features=8, expert_count=8,
                             expert_top_k=2)
    model = KoemiModel(settings, expert_shard=ExpertShard(2, 0, 8))
    model.exchange = "nccl"
    monkeypatch.setattr(torch.cuda, "is_available", lambda: True)
    monkeypatch.setattr(torch.cuda, "is_current_stream_capturing", lambda: True)
    block = model.blocks[0]
    rows = torch.zeros(4, 64)
    with pytest.raises(RuntimeError, match="not allowed inside CUDA graph capture"):
        model.expert_mlp(block, rows, torch.zeros(4, dtype=torch.long), torch.zeros(9, dtype=torch.long))
    monkeypatch.setattr(type(model), "device", property(lambda self: torch.device("cuda", 0)))
    with pytest.raises(RuntimeError, match="not captured in CUDA graphs"):
        BatchDecoder(model, capture_graph=True, cache_expert_weights=False)
