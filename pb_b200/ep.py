"""Expert-parallel host side: which experts each rank owns, and the exchange
of the ranks' combine buffers (CUDA IPC handles gathered over a
torch.distributed process group). The data path is the C-ABI's
pbmoe_ep_moe_layer; nothing here runs on the device.
"""

from __future__ import annotations

from . import capi


def expert_ranges(num_experts: int, world: int):
    """[(begin, count)] per rank: contiguous blocks covering every expert once."""
    return [capi.ep_expert_range(num_experts, r, world) for r in range(world)]


def connect(ctx, group=None, max_tokens: int = 32, hidden: int = 2048):
    """Reserve this rank's exchange buffer and map every rank's, using the
    process group only to all-gather the IPC handles (same collective on every
    rank). Returns (rank, world)."""
    import torch.distributed as dist

    rank, world = dist.get_rank(group), dist.get_world_size(group)
    ctx.ep_reserve(rank, world, max_tokens, hidden)
    handles = [None] * world
    dist.all_gather_object(handles, ctx.ep_ipc_handle(), group=group)
    if any(h is None or len(h) != capi.EP_HANDLE_BYTES for h in handles):
        raise RuntimeError("expert parallelism: a rank sent no exchange-buffer handle")
    ctx.ep_open_peers(handles)
    return rank, world


def shard(table, num_experts: int, rank: int, world: int):
    """(local expert table view, EpShard) of `rank`: slots [begin, begin+count)."""
    begin, count = capi.ep_expert_range(num_experts, rank, world)
    return table[begin:begin + count], capi.EpShard(begin, count, 0)
