"""pbmoe_expert_layer_load: a FIXED_Q4_EXPERT_LAYER_V1 store (config-1 expert
shapes) uploaded into the device expert table byte-exact, whole and as one
expert-parallel rank's range, and a MoE layer run from the loaded table equal
to the same layer from the directly written table."""

import numpy as np
import pytest

from expert_store_writer import write_layer

pytestmark = pytest.mark.gpu


def test_load_matches_and_runs(tmp_path):
    import torch

    from pb_b200 import capi, synth

    ctx = capi.Context(0)
    try:
        w = synth.MoeLayerWeights("cuda", seed=5, hidden=2048, num_experts=64, intermediate=512, group=64)
        lay = w.layout
        slots = w.experts.cpu().numpy().reshape(64, lay.expert_bytes)
        write_layer(str(tmp_path), 2, slots, 2048, 512, 64, list(lay.component_offsets))
        table = torch.zeros(64 * lay.expert_bytes, dtype=torch.uint8, device="cuda")
        ctx.expert_layer_load(tmp_path, 2, lay, 0, 64, table)
        assert torch.equal(table.view(-1), w.experts.view(-1))
        begin, count = capi.ep_expert_range(64, 1, 4)
        part = torch.zeros(count * lay.expert_bytes, dtype=torch.uint8, device="cuda")
        ctx.expert_layer_load(tmp_path, 2, lay, begin, count, part)
        assert torch.equal(part.view(-1), w.experts.view(-1)[begin * lay.expert_bytes:(begin + count) * lay.expert_bytes])
        with pytest.raises(capi.PbmoeError, match="exceed the destination"):
            ctx.expert_layer_load(tmp_path, 2, lay, 0, 64, part)

        cfg = capi.moe_config(lay, 64, 10)
        ctx.reserve(8, cfg)
        x = synth.normal_bf16((8, 2048), 1.0, synth.gen("cuda", 6), "cuda")
        outs = []
        for experts in (w.experts, table):
            cw = capi.MoeWeights(w.router.data_ptr(), experts.data_ptr(), w.shared.data_ptr(),
                                 w.shared_gate.data_ptr())
            out = torch.empty_like(x)
            ctx.moe_layer(cfg, cw, x, out, 8)
            outs.append(out)
        torch.cuda.synchronize()
        assert ctx.device_status() == 0
        assert torch.equal(outs[0], outs[1])
    finally:
        ctx.close()


def test_pbq4_load_equals_host_read(tmp_path):
    """A PBQ4 layer (f32 scales) at config-1 shapes: the device load equals
    the host read, which the CPU tests pin to fixed_q4_pack_from_pbq4_records."""
    import torch

    from expert_store_writer import pbq4_pack, write_pbq4_layer

    from pb_b200 import capi

    ctx = capi.Context(0)
    try:
        H, I, G = 2048, 512, 64
        lay = capi.fixed_q4_layout(H, I, G)
        rng = np.random.default_rng(3)
        packs = []
        for e in range(5):
            parts = []
            for rows, cols in ((I, H), (I, H), (H, I)):
                parts.append((rows, cols, G, rng.integers(0, 256, rows * cols // 2, dtype=np.uint8),
                              rng.uniform(0.004, 0.02, rows * cols // G).astype(np.float32),
                              (rng.standard_normal(rows * cols // G) * 0.1).astype(np.float32)))
            packs.append(pbq4_pack(0, e, parts, True, order=(1, 2, 0)))
        write_pbq4_layer(str(tmp_path), 0, packs, max(len(d) for d, _ in packs))
        host = capi.expert_layer_read(tmp_path, 0, lay, 0, 5)
        dev = torch.zeros(5 * lay.expert_bytes, dtype=torch.uint8, device="cuda")
        ctx.expert_layer_load(tmp_path, 0, lay, 0, 5, dev)
        assert np.array_equal(dev.cpu().numpy(), host.reshape(-1))
    finally:
        ctx.close()
