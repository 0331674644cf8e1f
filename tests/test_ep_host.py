"""Expert-parallel host logic on CPU: the expert partition and the exchange of
combine-buffer handles over a world_size-2 gloo process group (the C-ABI
itself is faked here: no device is touched)."""

import os
import socket

import pytest


def test_expert_ranges_cover_every_expert_once():
    from pb_b200 import ep

    for E, world in [(512, 1), (512, 2), (512, 4), (512, 8), (10, 3), (256, 8), (7, 7)]:
        ranges = ep.expert_ranges(E, world)
        owned = [e for b, n in ranges for e in range(b, b + n)]
        assert owned == list(range(E)), (E, world)
        assert all(n >= 1 for _, n in ranges)
        assert max(n for _, n in ranges) - min(n for _, n in ranges) <= 1


def test_expert_range_rejects_bad_partitions():
    from pb_b200 import capi

    for args in [(512, 0, 0), (512, 2, 2), (3, 0, 4)]:
        with pytest.raises(capi.PbmoeError):
            capi.ep_expert_range(*args)


def test_shard_views_the_owned_slots():
    import torch

    from pb_b200 import ep

    table = torch.arange(10 * 4, dtype=torch.uint8).reshape(10, 4)
    local, sh = ep.shard(table, 10, 1, 3)
    assert (sh.expert_begin, sh.expert_count) == (3, 3)
    assert torch.equal(local, table[3:6])


class _FakeCtx:
    """Stands in for capi.Context: records the calls ep.connect makes."""

    def __init__(self, rank):
        self.rank = rank
        self.reserved = None
        self.opened = None

    def ep_reserve(self, rank, world, max_tokens, hidden):
        self.reserved = (rank, world, max_tokens, hidden)

    def ep_ipc_handle(self):
        return bytes([self.rank + 1]) * 64

    def ep_open_peers(self, handles):
        self.opened = list(handles)


def _connect_worker(rank, world, port, out_dir):
    import torch.distributed as dist

    from pb_b200 import ep

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        ctx = _FakeCtx(rank)
        r, w = ep.connect(ctx, max_tokens=8, hidden=256)
        assert (r, w) == (rank, world)
        assert ctx.reserved == (rank, world, 8, 256)
        assert ctx.opened == [bytes([i + 1]) * 64 for i in range(world)]
        open(os.path.join(out_dir, f"ok{rank}"), "w").write("ok")
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_connect_exchanges_handles_in_rank_order(tmp_path):
    import torch.multiprocessing as mp

    world = 2
    mp.spawn(_connect_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    assert sorted(os.listdir(tmp_path)) == ["ok0", "ok1"]
