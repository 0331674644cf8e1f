"""Expert-parallel decode layer through the C-ABI (pbmoe_ep_moe_layer).

On one GPU: the world-1 path against pbmoe_moe_layer, and the bounded peer
wait (a rank whose partner never arrives latches PBMOE_DEV_ERR_PEER_TIMEOUT
and the context stays usable). On two GPUs (skipped with fewer): two ranks,
each holding half the experts, against the single-GPU layer; both ranks'
outputs must be bit-identical.
"""

import os
import socket

import numpy as np
import pytest

from parity import assert_close

pytestmark = pytest.mark.gpu

TOP_K = 10


def _layer_inputs(device, seed, tokens):
    import torch

    from pb_b200 import synth

    w = synth.MoeLayerWeights(device, seed)
    g = synth.gen(device, seed + 1)
    x = synth.normal_bf16((tokens, w.hidden), 1.0, g, device)
    res = synth.normal_bf16((tokens, w.hidden), 1.0, g, device).float()  # residual is in the output dtype
    norm_w = torch.rand(w.hidden, device=device, generator=g) + 0.5
    return w, x, res, norm_w


def _single(ctx, w, x, res, norm_w, tokens):
    import torch

    from pb_b200 import capi

    cfg = capi.moe_config(w.layout, w.num_experts, TOP_K)
    ctx.reserve(tokens, cfg)
    out = torch.empty(tokens, w.hidden, device=x.device, dtype=torch.float32)
    nn = torch.empty_like(out)
    ctx.moe_layer(cfg, w.c_weights(), x, out, tokens, residual=res, next_norm_weight=norm_w, next_normed=nn)
    return out, nn


def _ep(ctx, w, x, res, norm_w, tokens, rank, world, with_shared, timeout_us=0):
    import torch

    from pb_b200 import capi

    cfg = capi.moe_config(w.layout, w.num_experts, TOP_K)
    ctx.reserve(tokens, cfg)
    begin, count = capi.ep_expert_range(w.num_experts, rank, world)
    local = w.experts[begin:begin + count]
    ptr = lambda t: None if t is None else t.data_ptr()
    cw = capi.MoeWeights(w.router.data_ptr(), local.data_ptr(), ptr(w.shared) if with_shared else None,
                         ptr(w.shared_gate) if with_shared else None)
    out = torch.empty(tokens, w.hidden, device=x.device, dtype=torch.float32)
    nn = torch.empty_like(out)
    ctx.ep_moe_layer(cfg, cw, capi.EpShard(begin, count, timeout_us), x, out, tokens, residual=res,
                     next_norm_weight=norm_w, next_normed=nn)
    return out, nn


@pytest.fixture(scope="module")
def ctx():
    import torch

    from pb_b200 import capi

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    c = capi.Context(0)
    yield c
    c.close()


@pytest.mark.parametrize("tokens", [1, 8])
def test_world1_matches_single_gpu(ctx, tokens):
    import torch

    w, x, res, norm_w = _layer_inputs("cuda", 41, tokens)
    ref, ref_nn = _single(ctx, w, x, res, norm_w, tokens)
    ctx.ep_reserve(0, 1, 32, w.hidden)
    ctx.ep_set_peers([ctx.ep_buffer()])
    for _ in range(3):  # successive epochs reuse both parities
        out, nn = _ep(ctx, w, x, res, norm_w, tokens, 0, 1, True)
        torch.cuda.synchronize()
        assert ctx.device_status() == 0
        assert_close(out.cpu().numpy(), ref.cpu().numpy(), tol=1e-5, what="ep out")
        assert_close(nn.cpu().numpy(), ref_nn.cpu().numpy(), tol=1e-5, what="ep next norm")


def test_missing_peer_times_out(ctx):
    """Rank 0 of a two-rank group runs alone: its wait for rank 1's flag (which
    nothing sets) expires after 200 ms; the status bit is latched and the
    context keeps working."""
    import time

    import torch

    from pb_b200 import capi

    other = capi.Context(0)
    try:
        w, x, res, norm_w = _layer_inputs("cuda", 42, 2)
        ctx.ep_reserve(0, 2, 32, w.hidden)
        other.ep_reserve(1, 2, 32, w.hidden)
        ctx.ep_set_peers([ctx.ep_buffer(), other.ep_buffer()])
        ctx.device_status(clear=True)
        t0 = time.time()
        _ep(ctx, w, x, res, norm_w, 2, 0, 2, True, timeout_us=200_000)
        torch.cuda.synchronize()
        assert time.time() - t0 < 30
        assert ctx.device_status(clear=True) & capi.PBMOE_DEV_ERR_PEER_TIMEOUT
        # still usable
        out, _ = _single(ctx, w, x, res, norm_w, 2)
        torch.cuda.synchronize()
        assert torch.isfinite(out).all()
        assert ctx.device_status() == 0
    finally:
        other.close()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_gpu_worker(rank, world, port, out_dir):
    import torch
    import torch.distributed as dist

    from pb_b200 import capi, ep

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        ctx = capi.Context(rank)
        dev = f"cuda:{rank}"
        tokens = 8
        w, x, res, norm_w = _layer_inputs(dev, 43, tokens)
        ep.connect(ctx, max_tokens=32, hidden=w.hidden)
        stream = torch.cuda.current_stream(rank)
        for step in range(3):
            out, nn = _ep(ctx, w, x, res, norm_w, tokens, rank, world, rank == 0)
            torch.cuda.synchronize(rank)
            assert ctx.device_status() == 0, f"rank {rank} step {step}: device status"
            dist.barrier()
        np.save(os.path.join(out_dir, f"out{rank}.npy"), out.cpu().numpy())
        np.save(os.path.join(out_dir, f"nn{rank}.npy"), nn.cpu().numpy())
        if rank == 0:
            ref, ref_nn = _single(ctx, w, x, res, norm_w, tokens)
            torch.cuda.synchronize(rank)
            np.save(os.path.join(out_dir, "ref.npy"), ref.cpu().numpy())
            np.save(os.path.join(out_dir, "ref_nn.npy"), ref_nn.cpu().numpy())
        dist.barrier()
        ctx.close()
        del stream
    finally:
        dist.destroy_process_group()


def test_two_gpu_expert_parallel(tmp_path):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mp.spawn(_two_gpu_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    o0, o1 = np.load(tmp_path / "out0.npy"), np.load(tmp_path / "out1.npy")
    assert np.array_equal(o0, o1), "ranks disagree"
    assert np.array_equal(np.load(tmp_path / "nn0.npy"), np.load(tmp_path / "nn1.npy"))
    assert_close(o0, np.load(tmp_path / "ref.npy"), tol=1e-5, what="2-GPU out")
    assert_close(np.load(tmp_path / "nn0.npy"), np.load(tmp_path / "ref_nn.npy"), tol=1e-5, what="2-GPU norm")
