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


# limits of the one-launch owner sort (koemi_ep_owner_sort); larger exchanges
# wait, then run the general permutation
OWNER_SORT_MAX_SLOTS = 4096
OWNER_SORT_MAX_EXPERTS = 255


class _DeviceArray:
    """A raw device allocation seen by torch through __cuda_array_interface__."""

    def __init__(self, address: int, shape: tuple[int, ...], typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (address, False),
                                         "version": 3, "strides": None}


class PeerExchange:
    """Buffers of the fused peer-memory exchange (``koemi_ep_*``) for one
    shard, capacity and row shape; created by all ranks together.

    Every rank allocates one buffer with cudaMalloc in the native library and
    shares its CUDA IPC handle through one all-gather on the shard's group;
    after that the exchange needs no collective library call: dispatch and
    return are stores into peer memory followed by epoch flags."""

    def __init__(self, shard: ExpertShard, capacity: int, width: int, dtype: torch.dtype, device: torch.device):
        import ctypes
        import torch.distributed as dist
        from koemi_5hom_b200 import _native
        lib = _native.library()
        self.shard, self.capacity, self.width, self.dtype, self.device = shard, capacity, width, dtype, device
        code = _native.dtype_code(dtype)
        ranks = shard.world
        size = lib.koemi_peer_exchange_bytes(ranks, capacity, width, code)
        if size == 0:
            raise ValueError("bad exchange shape")
        own = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * 64)()
        _native.check("koemi_peer_buffer_alloc", lib.koemi_peer_buffer_alloc(size, ctypes.byref(own), handle))
        self.own = int(own.value)
        self._opened: list[int] = []
        mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=device)
        handles = [torch.empty_like(mine) for _ in range(ranks)]
        if ranks > 1:
            dist.all_gather(handles, mine, group=shard.group)
        addresses = []
        for r, h in enumerate(handles):
            if r == shard.rank:
                addresses.append(self.own)
                continue
            raw = (ctypes.c_uint8 * 64)(*h.cpu().tolist())
            peer = ctypes.c_void_p()
            _native.check("koemi_peer_buffer_open", lib.koemi_peer_buffer_open(raw, ctypes.byref(peer)))
            self._opened.append(int(peer.value))
            addresses.append(int(peer.value))
        # uint64 addresses as int64 bits
        self.peers = torch.tensor([a - (1 << 64) if a >= (1 << 63) else a for a in addresses], dtype=torch.int64,
                                  device=device)
        ids_offset, rows_offset = ctypes.c_size_t(), ctypes.c_size_t()
        _native.check("koemi_peer_exchange_offsets",
                      lib.koemi_peer_exchange_offsets(ranks, capacity, width, code, ctypes.byref(ids_offset),
                                                      ctypes.byref(rows_offset)))
        rows = ranks * capacity
        self.recv_ids = torch.as_tensor(_DeviceArray(self.own + ids_offset.value, (rows,), "<i4"), device=device)
        element = {torch.float32: "<f4", torch.bfloat16: "<i2", torch.float16: "<f2"}[dtype]
        recv = torch.as_tensor(_DeviceArray(self.own + rows_offset.value, (rows, width), element), device=device)
        self.recv_rows = recv.view(dtype) if dtype == torch.bfloat16 else recv
        if ranks > 1:
            dist.barrier(group=shard.group)

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (all ranks together,
        after the last exchange has finished on every rank)."""
        import torch.distributed as dist
        from koemi_5hom_b200 import _native
        lib = _native.library()
        torch.cuda.synchronize(self.device)
        for address in self._opened:
            _native.check("koemi_peer_buffer_close", lib.koemi_peer_buffer_close(address))
        self._opened = []
        if self.shard.world > 1:
            dist.barrier(group=self.shard.group)  # nobody maps this rank's buffer any more
        if self.own:
            _native.check("koemi_peer_buffer_free", lib.koemi_peer_buffer_free(self.own))
            self.own = 0

    def run(self, sorted_rows: Tensor | None, sorted_experts: Tensor, offsets: Tensor, weights: tuple[Tensor, ...],
            *, context: Tensor | None = None, sorted_tokens: Tensor | None = None) -> Tensor:
        """The expert MLP of the global experts over this rank's sorted pairs,
        through the owners (same contract as ``expert_parallel_mlp``). With
        ``context`` and ``sorted_tokens`` instead of ``sorted_rows``, pair i's
        row is ``context[sorted_tokens[i]]``, gathered by the dispatch itself."""
        from koemi_5hom_b200 import _native
        from koemi_5hom_b200.cuda_kernels import _ops
        shard = self.shard
        pairs = sorted_experts.shape[0]
        width = self.width if sorted_rows is None else sorted_rows.shape[1]
        if pairs > self.capacity or width != self.width or (sorted_rows is not None and sorted_rows.dtype != self.dtype):
            raise ValueError("rows do not fit this exchange")
        sorted_experts, offsets = sorted_experts.contiguous(), offsets.contiguous()
        stream = torch.cuda.current_stream(self.device).cuda_stream
        code = _native.dtype_code(self.dtype)
        ptr, call = _native.ptr, _native.call
        if sorted_rows is None:
            context, sorted_tokens = context.contiguous(), sorted_tokens.contiguous()
            call("koemi_ep_dispatch_gather", ptr(context), _native.dtype_code(context.dtype), ptr(sorted_tokens),
                 ptr(sorted_experts), ptr(offsets), ptr(self.peers), self.own, pairs, width, shard.rank, shard.world,
                 shard.local_count, self.capacity, code, stream)
        else:
            sorted_rows = sorted_rows.contiguous()
            call("koemi_ep_dispatch", ptr(sorted_rows), ptr(sorted_experts), ptr(offsets), ptr(self.peers), self.own,
                 pairs, width, shard.rank, shard.world, shard.local_count, self.capacity, code, stream)
        slots = shard.world * self.capacity
        if slots <= OWNER_SORT_MAX_SLOTS and shard.local_count <= OWNER_SORT_MAX_EXPERTS:
            # wait, sort by local expert and gather the received rows in one launch
            local_sorted = torch.empty(slots, width, dtype=self.dtype, device=self.device)
            local_offsets = torch.empty(shard.local_count + 1, dtype=torch.int64, device=self.device)
            local_experts = torch.empty(slots, dtype=torch.int64, device=self.device)
            local_positions = torch.empty(slots, dtype=torch.int64, device=self.device)
            call("koemi_ep_owner_sort", ptr(self.peers), self.own, width, shard.rank, shard.world, shard.local_count,
                 self.capacity, code, ptr(local_sorted), ptr(local_offsets), ptr(local_experts), ptr(local_positions),
                 None, None, stream)
        else:
            call("koemi_ep_wait_dispatch", self.own, shard.world, stream)
            local_sorted, _, local_experts, local_offsets, local_positions = _ops.permute_topk(
                self.recv_rows, self.recv_ids.view(-1, 1), self.recv_ids >= 0, shard.local_count, True)
        local_out = _ops.grouped_expert_mlp(local_sorted, local_experts, local_offsets, *weights)
        call("koemi_ep_return", ptr(local_out), ptr(local_positions), ptr(self.peers), self.own, width, shard.rank,
             shard.world, shard.local_count, self.capacity, code, stream)
        out = torch.empty(pairs, width, dtype=self.dtype, device=self.device)
        call("koemi_ep_collect", ptr(sorted_experts), ptr(offsets), ptr(out), ptr(self.peers), self.own, pairs, width,
             shard.rank, shard.world, shard.local_count, self.capacity, code, stream)
        return out

    def supports_return_to_combine(self) -> bool:
        """The fused return (the owner's output GEMM stores into the senders'
        buffers, the sender's combine reads them in place) needs 16-bit rows
        and the one-launch owner sort."""
        return (self.dtype in (torch.bfloat16, torch.float16) and self.width % 8 == 0
                and self.shard.world * self.capacity <= OWNER_SORT_MAX_SLOTS
                and self.shard.local_count <= OWNER_SORT_MAX_EXPERTS)

    def dispatch_normed(self, fused: Tensor, norm_weight: Tensor, eps: float, pair_positions: Tensor,
                        sorted_experts: Tensor, offsets: Tensor, top_k: int) -> Tensor:
        """The sender's half with the block's fusion RMSNorm fused in: returns
        the fp32 normalised rows (the combine's residual) after storing every
        routed pair's row, in the exchange dtype, into its owner's buffer."""
        from koemi_5hom_b200 import _native
        shard = self.shard
        tokens, width = fused.shape
        if tokens * top_k > self.capacity or width != self.width or not self.supports_return_to_combine():
            raise ValueError("rows do not fit this exchange")
        fused = fused.contiguous()
        context = torch.empty_like(fused)
        _native.call("koemi_ep_norm_dispatch", _native.ptr(fused), _native.ptr(norm_weight.contiguous()), eps,
                     _native.ptr(context), _native.ptr(pair_positions.contiguous()),
                     _native.ptr(sorted_experts.contiguous()), _native.ptr(offsets.contiguous()), tokens, top_k,
                     _native.ptr(self.peers), self.own, width, shard.rank, shard.world, shard.local_count,
                     self.capacity, _native.dtype_code(self.dtype), torch.cuda.current_stream(self.device).cuda_stream)
        return context

    def run_to_combine(self, context: Tensor, sorted_tokens: Tensor, sorted_experts: Tensor, offsets: Tensor,
                       weights: tuple[Tensor, ...]) -> None:
        """One exchange whose expert outputs stay in the senders' buffers:
        the gathering dispatch, then ``serve_and_return``. The caller then
        combines with ``koemi_ep_combine_residual_rmsnorm_next`` on this
        exchange's buffer."""
        from koemi_5hom_b200 import _native
        shard = self.shard
        pairs = sorted_experts.shape[0]
        width = self.width
        if pairs > self.capacity or context.shape[1] != width or not self.supports_return_to_combine():
            raise ValueError("rows do not fit this exchange")
        ptr = _native.ptr
        _native.call("koemi_ep_dispatch_gather", ptr(context.contiguous()), _native.dtype_code(context.dtype),
                     ptr(sorted_tokens.contiguous()), ptr(sorted_experts.contiguous()), ptr(offsets.contiguous()),
                     ptr(self.peers), self.own, pairs, width, shard.rank, shard.world, shard.local_count, self.capacity,
                     _native.dtype_code(self.dtype), torch.cuda.current_stream(self.device).cuda_stream)
        self.serve_and_return(weights)

    def serve_and_return(self, weights: tuple[Tensor, ...]) -> None:
        """The owner's half: the owner sort (which also emits the slot of
        every sorted row and the grouped GEMM's tile map) and the expert MLP
        of the local experts, whose output GEMM stores each row back into its
        sender's buffer and raises the return flags. Three launches fewer
        than ``run`` (the tile map, the return and the collect) and no sorted
        output tensor."""
        from koemi_5hom_b200 import _native
        shard = self.shard
        width = self.width
        stream = torch.cuda.current_stream(self.device).cuda_stream
        code = _native.dtype_code(self.dtype)
        ptr, call = _native.ptr, _native.call
        slots = shard.world * self.capacity
        local_sorted = torch.empty(slots, width, dtype=self.dtype, device=self.device)
        local_offsets = torch.empty(shard.local_count + 1, dtype=torch.int64, device=self.device)
        local_experts = torch.empty(slots, dtype=torch.int64, device=self.device)
        local_positions = torch.empty(slots, dtype=torch.int64, device=self.device)
        local_slots = torch.empty(slots, dtype=torch.int64, device=self.device)
        tile_prefix = torch.empty(shard.local_count + 1, dtype=torch.int32, device=self.device)
        call("koemi_ep_owner_sort", ptr(self.peers), self.own, width, shard.rank, shard.world, shard.local_count,
             self.capacity, code, ptr(local_sorted), ptr(local_offsets), ptr(local_experts), ptr(local_positions),
             ptr(local_slots), ptr(tile_prefix), stream)
        weights = tuple(w.contiguous() for w in weights)
        hidden_width = weights[0].shape[1]
        hidden = torch.empty(slots * hidden_width * 2, dtype=torch.uint8, device=self.device)
        call("koemi_ep_expert_mlp_return", ptr(local_sorted), ptr(local_offsets), ptr(tile_prefix), ptr(local_slots),
             *(ptr(w) for w in weights), slots, width, hidden_width, shard.local_count, code, ptr(hidden),
             hidden.numel(), ptr(self.peers), self.own, shard.rank, shard.world, self.capacity, stream)
