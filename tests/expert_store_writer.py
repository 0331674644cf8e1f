"""Writes a FIXED_Q4_EXPERT_LAYER_V1 expert layer store as the reference's
writer lays it out (test fixture, not product code): layer_NN.bin with
expert e's slot at e * expert_size (write_test_expert_layer,
test_fixtures.rs:195; rewrite_pbq4_layer_to_fixed_q4, experts/mod.rs:2330-2375)
and layer_NN.json, the serde form of ExpertLayerPackMetadata with one record
per projection (fixed_q4_pack_from_pbq4_records, experts/slots.rs:984-1113)."""

import json
import os

import numpy as np


def records_for(layer, expert, hidden, inter, group, offsets):
    recs = []
    for j, (name, rows, cols) in enumerate((("gate_proj", inter, hidden), ("up_proj", inter, hidden),
                                            ("down_proj", hidden, inter))):
        recs.append({
            "tensor": f"model.layers.{layer}.mlp.experts.{expert}.{name}.weight",
            "dtype": "BF16",
            "shape": [rows, cols],
            "source_offsets": [0, rows * cols * 2],
            "record_offset": int(offsets[3 * j]),
            "packed_bytes": rows * cols // 2,
            "groups": rows * (cols // group),
            "group_size": group,
            "scale_bias_dtype": "BF16",
        })
    return recs


def write_layer(root, layer, slots, hidden, inter, group, offsets, meta_edit=None):
    """slots: uint8 [experts, expert_size]. meta_edit(meta) may alter the
    metadata before it is written (for the invalid-store tests)."""
    experts, size = slots.shape
    os.makedirs(root, exist_ok=True)
    with open(os.path.join(root, f"layer_{layer:02d}.bin"), "wb") as f:
        f.write(np.ascontiguousarray(slots).tobytes())
    meta = {
        "format": "FIXED_Q4_EXPERT_LAYER_V1", "layer": layer, "expert_size": size, "experts": experts,
        "packs": [{"layer": layer, "expert": e, "packed_bytes": size,
                   "records": records_for(layer, e, hidden, inter, group, offsets)} for e in range(experts)],
    }
    if meta_edit:
        meta_edit(meta)
    with open(os.path.join(root, f"layer_{layer:02d}.json"), "w") as f:
        json.dump(meta, f)
