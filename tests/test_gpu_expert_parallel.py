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


@pytest.mark.parametrize("tokens,experts,steps", [(64, 8, 3), (256, 64, 2), (5, 4, 1), (2100, 8, 2)])
@pytest.mark.parametrize("gathered", [False, True])
def test_peer_exchange_with_itself_equals_grouped_mlp(tokens, experts, steps, gathered, cuda):
    """One rank exchanging with its own buffer runs every peer kernel
    (dispatch -- plain, or gathering fp32 token rows --, the one-launch owner
    sort, or past 4096 slots the wait + general permutation, return, collect)
    on one GPU, repeatedly (epochs)."""
    from koemi_5hom_b200 import _native
    from koemi_5hom_b200.model.expert_parallel import ExpertShard, PeerExchange
    g = torch.Generator().manual_seed(tokens)
    width, hidden = 128, 256
    weights = tuple((torch.randn(*shape, generator=g) * 0.05).bfloat16().to(cuda) for shape in
                    ((experts, hidden, width), (experts, hidden), (experts, hidden, width), (experts, hidden),
                     (experts, width, hidden), (experts, width)))
    exchange = PeerExchange(ExpertShard(1, 0, experts), tokens * 2, width, torch.bfloat16, cuda)
    try:
        for step in range(steps):
            context = torch.randn(tokens, width, generator=g).to(cuda)
            rows = context.bfloat16()
            assignments = torch.randint(-1, experts, (tokens, 2), generator=g).to(cuda)
            valid = torch.ones(tokens, dtype=torch.bool, device=cuda)
            sorted_rows, sorted_tokens, sorted_experts, offsets, _ = _ops.permute_topk(rows, assignments, valid,
                                                                                       experts, True)
            expected = _ops.grouped_expert_mlp(sorted_rows, sorted_experts, offsets, *weights)
            if gathered:
                got = exchange.run(None, sorted_experts, offsets, weights, context=context,
                                   sorted_tokens=sorted_tokens)
            else:
                got = exchange.run(sorted_rows, sorted_experts, offsets, weights)
            torch.cuda.synchronize()
            assert _native.device_status(cuda) == 0
            assert torch.equal(got, expected), step
    finally:
        exchange.close()


@pytest.mark.parametrize("tokens,experts,steps", [(64, 8, 3), (256, 64, 2), (5, 4, 1), (1000, 16, 2)])
@pytest.mark.parametrize("normed", [False, True])
def test_fused_return_with_itself_equals_local_combine(tokens, experts, steps, normed, cuda):
    """The fused return on one GPU, one rank exchanging with its own buffer:
    the dispatch (gathering context rows, or normalising the fusion output and
    dispatching in one launch), owner sort (with slots and tile map), the
    expert MLP whose output GEMM stores the rows into the sender's return
    block, and the combine that waits for the return flag and reads them in
    place. It must equal the local norm + grouped MLP + combine bit for bit,
    over several exchanges (epochs)."""
    from koemi_5hom_b200 import _native
    from koemi_5hom_b200.model.expert_parallel import ExpertShard, PeerExchange
    g = torch.Generator().manual_seed(tokens + 7)
    width, hidden, top_k = 128, 256, 2
    weights = tuple((torch.randn(*shape, generator=g) * 0.05).bfloat16().to(cuda) for shape in
                    ((experts, hidden, width), (experts, hidden), (experts, hidden, width), (experts, hidden),
                     (experts, width, hidden), (experts, width)))
    norm = (1.0 + 0.1 * torch.randn(width, generator=g)).to(cuda)
    next_norm = (1.0 + 0.1 * torch.randn(width, generator=g)).to(cuda)
    exchange = PeerExchange(ExpertShard(1, 0, experts), tokens * top_k, width, torch.bfloat16, cuda)
    assert exchange.supports_return_to_combine()
    stream = torch.cuda.current_stream(cuda).cuda_stream
    try:
        fusion_norm = (1.0 + 0.1 * torch.randn(width, generator=g)).to(cuda)
        for step in range(steps):
            fused = torch.randn(tokens, width, generator=g).to(cuda) * 3.0
            context = _ops.rms_norm(fused, None, fusion_norm, None, 1e-6, torch.float32) if normed else fused
            assignments = torch.randint(-1, experts, (tokens, top_k), generator=g).to(cuda)
            valid = (torch.rand(tokens, generator=g) > 0.1).to(cuda)
            sorted_rows, sorted_tokens, sorted_experts, offsets, positions = _ops.permute_topk(
                context.bfloat16(), assignments, valid, experts, True)
            expert_out = _ops.grouped_expert_mlp(sorted_rows, sorted_experts, offsets, *weights)
            expected = _ops.combine_residual_rmsnorm_next(context, expert_out, positions, offsets, None, valid, norm,
                                                          next_norm, top_k, 1e-6, torch.bfloat16)
            if normed:
                mine = exchange.dispatch_normed(fused, fusion_norm, 1e-6, positions, sorted_experts, offsets, top_k)
                assert torch.equal(mine, context), step
                exchange.serve_and_return(weights)
            else:
                exchange.run_to_combine(context, sorted_tokens, sorted_experts, offsets, weights)
            got = torch.empty(tokens, width, dtype=torch.bfloat16, device=cuda)
            _native.call("koemi_ep_combine_residual_rmsnorm_next", context.data_ptr(), positions.data_ptr(),
                         offsets.data_ptr(), None, valid.data_ptr(), norm.data_ptr(), next_norm.data_ptr(),
                         got.data_ptr(), _native.BF16, tokens, width, top_k, experts, 1e-6, _native.BF16,
                         exchange.own, 1, experts, exchange.capacity, stream)
            torch.cuda.synchronize()
            assert _native.device_status(cuda) == 0
            assert torch.equal(got, expected), step
    finally:
        exchange.close()


@pytest.mark.parametrize("stage", ["dispatch", "collect", "combine"])
def test_peer_waits_give_up_when_no_flag_arrives(stage, cuda):
    """The bounded waits of the exchange, made to run out on one GPU: the
    buffer's epoch says an exchange is due but no rank ever raises its flag
    (a peer that never dispatched or never returned). The kernel must end by
    itself, leave KOEMI_ERR_TIMEOUT in the device status word and the host
    must raise on it; the context stays usable afterwards."""
    from koemi_5hom_b200 import _native
    from koemi_5hom_b200.model.expert_parallel import ExpertShard, PeerExchange, _DeviceArray
    # one rank waiting on its own flags: every access stays inside the buffer
    experts, width, capacity, ranks = 4, 64, 8, 1
    exchange = PeerExchange(ExpertShard(1, 0, experts), capacity, width, torch.bfloat16, cuda)
    try:
        header = torch.as_tensor(_DeviceArray(exchange.own, (32,), "<i8"), device=cuda)
        header[16] = 1  # the epoch slot: exchange 1 is expected, every flag still reads 0
        torch.cuda.synchronize()
        stream = torch.cuda.current_stream(cuda).cuda_stream
        if stage == "dispatch":
            _native.call("koemi_ep_wait_dispatch", exchange.own, ranks, stream)
        elif stage == "combine":  # the fused return's combine waits for every owner's return flag
            tokens = 3
            context = torch.randn(tokens, width, device=cuda)
            positions = torch.tensor([0, 1, 2, 3, 4, 5], dtype=torch.int64, device=cuda)
            offsets = torch.tensor([0, 6, 6, 6, 6], dtype=torch.int64, device=cuda)
            valid = torch.ones(tokens, dtype=torch.bool, device=cuda)
            norm = torch.ones(width, device=cuda)
            out = torch.empty(tokens, width, dtype=torch.bfloat16, device=cuda)
            _native.call("koemi_ep_combine_residual_rmsnorm_next", context.data_ptr(), positions.data_ptr(),
                         offsets.data_ptr(), None, valid.data_ptr(), norm.data_ptr(), None, out.data_ptr(),
                         _native.BF16, tokens, width, 2, experts, 1e-6, _native.BF16, exchange.own, ranks,
                         experts // ranks, capacity, stream)
        else:
            pairs = 6
            sorted_experts = torch.zeros(pairs, dtype=torch.int64, device=cuda)
            offsets = torch.tensor([0, pairs, pairs, pairs, pairs], dtype=torch.int64, device=cuda)
            out = torch.empty(pairs, width, dtype=torch.bfloat16, device=cuda)
            peers = torch.tensor([exchange.own], dtype=torch.int64, device=cuda)
            _native.call("koemi_ep_collect", sorted_experts.data_ptr(), offsets.data_ptr(), out.data_ptr(),
                         peers.data_ptr(), exchange.own, pairs, width, 0, ranks, experts // ranks, capacity,
                         _native.BF16, stream)
        torch.cuda.synchronize()  # returns: the wait gave up instead of hanging
        with pytest.raises(_native.KoemiNativeError) as raised:
            _native.raise_for_device_status(cuda)
        assert raised.value.status == _native.KOEMI_ERR_TIMEOUT
        assert _native.device_status(cuda) == 0  # reading cleared it
        assert torch.ones(4, device=cuda).sum().item() == 4.0  # the context still works
    finally:
        exchange.close()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ep_rank(rank: int, world: int, port: int, capture_graph: bool, exchange: str) -> None:
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
        sharded.exchange = exchange
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
        sharded.close_exchanges()
        from koemi_5hom_b200 import _native
        assert _native.device_status(device) == 0
        assert torch.equal(runs[0], runs[1]), float((runs[0] - runs[1]).abs().max())
    finally:
        dist.destroy_process_group()


# the NCCL exchange runs eager only: it is refused inside graph capture
@pytest.mark.parametrize("capture_graph,exchange", [(False, "peer"), (True, "peer"), (False, "nccl")])
def test_expert_parallel_decode_equals_unsharded_model(capture_graph, exchange):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    context = mp.spawn(_ep_rank, args=(2, _free_port(), capture_graph, exchange), nprocs=2, join=False)
    deadline = 300.0
    import time
    start = time.monotonic()
    while not context.join(timeout=5.0):
        if time.monotonic() - start > deadline:  # a rank that never finishes: end both, fail
            for process in context.processes:
                process.kill()
            pytest.fail("expert-parallel ranks did not finish in time")
