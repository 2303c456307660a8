"""Expert parallelism for the MoE block: each rank holds ``E / G`` experts.

The reference has no expert parallelism (its ``moe_submapping.py`` shards
storage, not compute). Here rank ``g`` of ``G`` owns experts
``[g * E/G, (g + 1) * E/G)``. After the usual stable, expert-major
permutation of a rank's own token-expert pairs, the sorted rows are already
grouped by owner, so one all-to-all sends every owner its rows; the owner runs
the same grouped expert MLP on its local experts and a second all-to-all
returns the outputs, which land back in the sender's sorted order. The sender
then combines exactly as on one GPU, so the result for every row equals the
single-GPU result: an expert's output row depends only on that row and the
expert's weights.

Two exchange modes:

- ``padded`` (decode, CUDA-graph capturable): fixed slabs of ``capacity =
  pairs`` rows per owner built on the device by ``ep_pack``; equal-split
  all-to-alls of the rows and of their owner-local expert ids; ``ep_unpack``
  restores the sorted order. No host synchronisation.
- ``exact`` (prefill windows, large row counts): per-owner counts are
  exchanged first and read on the host, then variable-split all-to-alls move
  only the valid rows.

The tensor operations (permute, grouped MLP, pack, unpack) come from an
``ExpertOps`` table, the native kernels by default, so the exchange
bookkeeping can be exercised with other implementations on CPU ranks.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Callable

import torch
from torch import Tensor


@dataclass(frozen=True)
class ExpertShard:
    """This rank's slice of the experts and the group that exchanges rows."""

    world: int
    rank: int
    expert_count: int
    group: Any = None  # torch.distributed process group (None: the default group)

    def __post_init__(self):
        if self.world < 1 or not 0 <= self.rank < self.world:
            raise ValueError("expert shard needs 0 <= rank < world")
        if self.expert_count % self.world != 0:
            raise ValueError(f"{self.expert_count} experts do not split evenly over {self.world} ranks")

    @property
    def local_count(self) -> int:
        return self.expert_count // self.world

    @property
    def first(self) -> int:
        return self.rank * self.local_count

    @classmethod
    def from_group(cls, expert_count: int, group: Any = None) -> "ExpertShard":
        import torch.distributed as dist
        return cls(dist.get_world_size(group), dist.get_rank(group), expert_count, group)


@dataclass(frozen=True)
class ExpertOps:
    """Tensor operations the exchange is built from."""

    permute_topk: Callable[..., tuple]  # (rows, assignments[N,1], valid, experts, gather) -> 5-tuple
    grouped_mlp: Callable[..., Tensor]  # (sorted_rows, sorted_experts, offsets, *weights) -> [P, d]
    pack: Callable[..., tuple]          # (sorted_rows, sorted_experts, offsets, ranks, local, capacity)
    unpack: Callable[..., Tensor]       # (slab, sorted_experts, offsets, ranks, local, capacity)


def native_ops() -> ExpertOps:
    from koemi_5hom_b200.cuda_kernels import _ops
    return ExpertOps(permute_topk=_ops.permute_topk, grouped_mlp=_ops.grouped_expert_mlp, pack=_ops.ep_pack,
                     unpack=_ops.ep_unpack)


def _local_experts(ops: ExpertOps, shard: ExpertShard, rows: Tensor, local_ids: Tensor,
                   weights: tuple[Tensor, ...]) -> Tensor:
    """Owner side: run the received rows through the local experts and return
    the outputs in the received order (padding rows give zero)."""
    assignments = local_ids.reshape(-1, 1)
    valid = local_ids >= 0
    sorted_rows, _, sorted_experts, offsets, positions = ops.permute_topk(rows, assignments, valid,
                                                                         shard.local_count, True)
    out = ops.grouped_mlp(sorted_rows, sorted_experts, offsets, *weights)
    return out.index_select(0, positions)


def expert_parallel_mlp(shard: ExpertShard, sorted_rows: Tensor, sorted_experts: Tensor, offsets: Tensor,
                        weights: tuple[Tensor, ...], mode: str = "padded", ops: ExpertOps | None = None,
                        capacity: int | None = None) -> Tensor:
    """Drop-in for ``grouped_expert_mlp`` over the global experts: the rows of
    ``sorted_rows`` (expert-major, global expert ids, ``offsets`` [E + 1])
    are processed by their owners' local ``weights`` and returned in the same
    order, zero past the valid pairs.

    ``capacity`` (padded mode) is the slab rows per owner and must be the same
    on every rank and at least every rank's pair count; it defaults to this
    rank's pair count, which is right when all ranks hold the same number of
    tokens (the decode step: equal streams per rank)."""
    import torch.distributed as dist
    ops = ops or native_ops()
    group, ranks, local = shard.group, shard.world, shard.local_count
    pairs, width = sorted_rows.shape
    if mode == "padded":
        capacity = max(pairs, 1) if capacity is None else capacity
        if capacity < pairs:
            raise ValueError(f"capacity {capacity} is below this rank's {pairs} pairs")
        slab, slab_ids = ops.pack(sorted_rows, sorted_experts, offsets, ranks, local, capacity)
        recv_ids = torch.empty_like(slab_ids)
        recv = torch.empty_like(slab)
        dist.all_to_all_single(recv_ids, slab_ids, group=group)
        dist.all_to_all_single(recv, slab, group=group)
        back = _local_experts(ops, shard, recv, recv_ids, weights)
        returned = torch.empty_like(back)
        dist.all_to_all_single(returned, back, group=group)
        return ops.unpack(returned, sorted_experts, offsets, ranks, local, capacity)
    if mode != "exact":
        raise ValueError("mode must be 'padded' or 'exact'")
    bounds = offsets[torch.arange(0, ranks + 1, device=offsets.device) * local]
    send_counts = (bounds[1:] - bounds[:-1]).to(torch.int64)
    recv_counts = torch.empty_like(send_counts)
    dist.all_to_all_single(recv_counts, send_counts, group=group)
    send_sizes = send_counts.tolist()
    recv_sizes = recv_counts.tolist()
    valid = int(bounds[-1])
    send = sorted_rows[:valid]
    send_ids = (sorted_experts[:valid] % local).to(torch.int32)
    recv = sorted_rows.new_empty(sum(recv_sizes), width)
    recv_ids = send_ids.new_empty(sum(recv_sizes))
    dist.all_to_all_single(recv_ids, send_ids, recv_sizes, send_sizes, group=group)
    dist.all_to_all_single(recv, send, recv_sizes, send_sizes, group=group)
    back = _local_experts(ops, shard, recv, recv_ids, weights) if recv.shape[0] else recv
    out = sorted_rows.new_zeros(pairs, width)
    dist.all_to_all_single(out[:valid], back, send_sizes, recv_sizes, group=group)
    return out
