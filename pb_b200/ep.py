"""Expert-parallel host side: which experts each rank owns, and the exchange
of the ranks' combine buffers (CUDA IPC handles gathered over a
torch.distributed process group). The data path is the C-ABI's
pbmoe_ep_moe_layer; nothing here runs on the device. For a vocabulary-sharded
LM head: each rank's id range, and the all-gather of the ranks' candidate
lists that pbmoe_head_merge then merges.
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


def vocab_ranges(vocab: int, world: int):
    """[(id_base, rows)] per rank: contiguous shards of the LM head's rows in
    id order (sizes differ by at most one), the order in which
    pbmoe_head_merge takes the ranks' candidate lists."""
    if world <= 0 or vocab < world:
        raise ValueError(f"cannot split {vocab} rows over {world} ranks")
    base, extra = divmod(vocab, world)
    out, b = [], 0
    for r in range(world):
        n = base + (1 if r < extra else 0)
        out.append((b, n))
        b += n
    return out


def gather_candidates(keys, ids, values, group=None):
    """All-gather every rank's [tokens, top_k] candidate lists into
    [world, tokens, top_k] tensors in rank order (the merge input). The same
    collective on every rank; gloo (CPU tensors) or nccl (device tensors)."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    out = []
    for t in (keys, ids, values):
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t.contiguous(), group=group)
        out.append(torch.stack(parts))
    return tuple(out)
