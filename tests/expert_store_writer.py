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


PBQ4_MAGIC = b"PBQ4EXPERT "


def pbq4_pack(layer, expert, parts, f32_scales, order=(0, 1, 2)):
    """A PBQ4 expert pack (parse_pbq4_expert_pack_with_metadata,
    experts/mod.rs:546-653): the magic, then per record u32 name length, name,
    u64 nibble bytes, u64 groups, scales, biases (F32 or BF16 little-endian),
    nibbles. parts[j] = (rows, cols, group, nibbles u8, scales f32, biases f32)
    for gate, up, down. Returns (bytes, metadata records)."""
    import struct

    names = ("gate_proj", "up_proj", "down_proj")
    out = bytearray(PBQ4_MAGIC)
    recs = []
    for j in order:
        rows, cols, group, nib, sc, bi = parts[j]
        name = f"model.layers.{layer}.mlp.experts.{expert}.{names[j]}.weight".encode()
        rec = {"tensor": name.decode(), "dtype": "BF16", "shape": [rows, cols], "source_offsets": [0, 0],
               "record_offset": len(out), "packed_bytes": len(nib), "groups": len(sc), "group_size": group,
               "scale_bias_dtype": "F32" if f32_scales else "BF16"}
        out += struct.pack("<I", len(name)) + name + struct.pack("<QQ", len(nib), len(sc))
        if f32_scales:
            out += np.asarray(sc, np.float32).tobytes() + np.asarray(bi, np.float32).tobytes()
        else:
            out += bf16_bytes(sc) + bf16_bytes(bi)
        out += np.asarray(nib, np.uint8).tobytes()
        recs.append(rec)
    return bytes(out), recs


def bf16_bytes(values):
    """Round-to-nearest-even bf16 of f32 values (experts/slots.rs:1165-1169), as bytes."""
    b = np.asarray(values, np.float32).view(np.uint32).astype(np.uint64)
    lsb = (b >> 16) & 1
    return (((b + 0x7FFF + lsb) >> 16) & 0xFFFF).astype(np.uint16).tobytes()


def write_pbq4_layer(root, layer, packs, slot_size, version="PBQ4EXPERT_LAYER_V2", pack_edit=None):
    """packs: list of (bytes, records) per expert, slot e at e * slot_size."""
    os.makedirs(root, exist_ok=True)
    with open(os.path.join(root, f"layer_{layer:02d}.bin"), "wb") as f:
        for data, _ in packs:
            f.write(data + bytes(slot_size - len(data)))
    meta = {"format": version, "layer": layer, "expert_size": slot_size, "experts": len(packs),
            "packs": [{"layer": layer, "expert": e, "packed_bytes": len(d), "records": r}
                      for e, (d, r) in enumerate(packs)]}
    if pack_edit:
        pack_edit(meta)
    with open(os.path.join(root, f"layer_{layer:02d}.json"), "w") as f:
        json.dump(meta, f)
