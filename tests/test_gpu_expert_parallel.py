"""Expert parallelism on GPUs: the pack/unpack slab kernels against the
oracle's slab layout (one GPU), and an expert-parallel model against the
unsharded model on the same streams, two NCCL ranks on two GPUs (skipped with
fewer GPUs)."""
from __future__ import annotations

import os
import socket
from datetime import timedelta

import pytest
import torch

from koemi_5hom_b200.cuda_kernels import _ops
from oracle import ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("ranks,local,tokens,top_k,dtype", [(2, 4, 37, 2, torch.bfloat16), (4, 16, 256, 2, torch.bfloat16),
                                                            (8, 8, 64, 2, torch.float32), (3, 1, 5, 3, torch.float16)])
def test_slab_pack_and_unpack_match_oracle(ranks, local, tokens, top_k, dtype, cuda):
    experts = ranks * local
    g = torch.Generator().manual_seed(tokens + ranks)
    rows = torch.randn(tokens, 64, generator=g).to(dtype)
    assignments = torch.randint(-1, experts + 1, (tokens, top_k), generator=g)
    valid = torch.rand(tokens, generator=g) > 0.2
    sorted_rows, _, sorted_experts, offsets, _ = ops.permute_rows(rows, assignments, valid, experts)
    capacity = tokens * top_k + 3
    slab_ref, ids_ref = ops.ep_pack(sorted_rows, sorted_experts, offsets, ranks, local, capacity)
    s_dev, e_dev, o_dev = sorted_rows.to(cuda), sorted_experts.to(cuda), offsets.to(cuda)
    slab, ids = _ops.ep_pack(s_dev, e_dev, o_dev, ranks, local, capacity)
    assert torch.equal(ids.cpu(), ids_ref)
    live = ids_ref >= 0
    assert torch.equal(slab.cpu()[live], slab_ref[live])
    returned = torch.randn(slab.shape, generator=g).to(dtype)
    back = _ops.ep_unpack(returned.to(cuda), e_dev, o_dev, ranks, local, capacity)
    assert torch.equal(back.cpu(), ops.ep_unpack(returned, sorted_experts, offsets, ranks, local, capacity))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ep_rank(rank: int, world: int, port: int, capture_graph: bool) -> None:
    import torch.distributed as dist
    from koemi_5hom_b200.model import KoemiModel, ModelSettings
    from koemi_5hom_b200.model.expert_parallel import ExpertShard
    from koemi_5hom_b200.runtime import BatchDecoder, SamplingPolicy, TokenSampler
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=device)
    try:
        settings = ModelSettings(vocabulary_size=1024, embedding_size=128, memory_features=16, local_memory_size=16,
                                 salience_memory_size=16, salience_threshold=0.6, expert_count=8, expert_top_k=2,
                                 layer_count=2, compute_dtype="bfloat16")
        full = KoemiModel(settings, device=device)
        full.initialize_parameters(seed=5)
        sharded = KoemiModel(settings, device=device, expert_shard=ExpertShard.from_group(8))
        sharded.initialize_parameters(seed=5)
        g = torch.Generator().manual_seed(40 + rank)  # each rank decodes its own streams
        prompts = torch.randint(0, 1023, (4, 24), generator=g).to(device)
        sampler = TokenSampler(SamplingPolicy(greedy=True), device)
        runs = []
        for model in (full, sharded):
            decoder = BatchDecoder(model, capture_graph=capture_graph)
            logits = decoder.prefill(prompts)
            trace = [logits.clone()]
            for _ in range(12):
                logits = decoder.step(sampler(logits))
                trace.append(logits.clone())
            runs.append(torch.stack(trace))
            del decoder, logits, trace  # graphs holding NCCL calls go before the process group
        torch.cuda.synchronize()
        import gc
        gc.collect()
        assert torch.equal(runs[0], runs[1]), float((runs[0] - runs[1]).abs().max())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("capture_graph", [False, True])
def test_expert_parallel_decode_equals_unsharded_model(capture_graph):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.spawn(_ep_rank, args=(2, _free_port(), capture_graph), nprocs=2, join=True)
