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
