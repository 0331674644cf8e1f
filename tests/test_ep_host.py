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


def test_vocab_ranges_cover_every_id_once():
    from pb_b200 import ep

    for V, world in [(151936, 8), (151936, 3), (10, 10), (1000, 1)]:
        ranges = ep.vocab_ranges(V, world)
        assert [b for b, _ in ranges] == sorted(b for b, _ in ranges)
        assert sum(n for _, n in ranges) == V and ranges[0][0] == 0
        assert all(b + n == nb for (b, n), (nb, _) in zip(ranges, ranges[1:]))
        assert max(n for _, n in ranges) - min(n for _, n in ranges) <= 1
    with pytest.raises(ValueError):
        ep.vocab_ranges(3, 4)


def _vocab_worker(rank, world, port, out_dir):
    """Each rank selects its shard's candidates (the oracle's topk_vocab with
    ids offset by the shard's base), the lists are gathered in rank order,
    and the best k of the union (value desc, id asc) equal topk_vocab over
    the whole vocabulary."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from oracle import pb_oracle
    from pb_b200 import ep

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        V, T, k = 5000, 3, 16
        rng = np.random.default_rng(0)
        logits = np.round(rng.standard_normal((T, V)) * 8).astype(np.float32) / 8  # many ties
        base, n = ep.vocab_ranges(V, world)[rank]
        ids = np.zeros((T, k), np.int64)
        vals = np.zeros((T, k), np.float32)
        for t in range(T):
            i, v = pb_oracle.topk_vocab(logits[t, base:base + n], k)
            ids[t], vals[t] = i.astype(np.int64) + base, v
        keys = torch.zeros(T, k, dtype=torch.int32)
        gk, gi, gv = ep.gather_candidates(keys, torch.tensor(ids), torch.tensor(vals))
        assert gi.shape == (world, T, k)
        for t in range(T):
            cand = sorted(zip(gv[:, t].reshape(-1).tolist(), gi[:, t].reshape(-1).tolist()),
                          key=lambda c: (-c[0], c[1]))[:k]
            ref_i, ref_v = pb_oracle.topk_vocab(logits[t], k)
            assert [c[1] for c in cand] == ref_i.tolist() and [c[0] for c in cand] == ref_v.tolist()
        open(os.path.join(out_dir, f"ok{rank}"), "w").write("ok")
    finally:
        dist.destroy_process_group()


def test_vocab_shard_candidates_merge_to_the_full_topk(tmp_path):
    import torch.multiprocessing as mp

    mp.spawn(_vocab_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    assert sorted(os.listdir(tmp_path)) == ["ok0", "ok1"]
