"""The fixed-Q4 expert layer store reader (pbmoe_expert_layer_read) on CPU:
slots read back byte-exact, and the metadata checks of
ExpertLayerPackMetadata::validate (experts/mod.rs:372-429) plus the record
checks against the layout, each failing with its message."""

import numpy as np
import pytest

from expert_store_writer import write_layer

H, I, G, E = 128, 64, 32, 6


@pytest.fixture()
def store(tmp_path):
    from pb_b200 import capi

    lay = capi.fixed_q4_layout(H, I, G)
    rng = np.random.default_rng(1)
    slots = rng.integers(0, 256, (E, lay.expert_bytes), dtype=np.uint8)
    offs = list(lay.component_offsets)
    return tmp_path, lay, slots, offs


def test_read_all_and_a_range(store):
    from pb_b200 import capi

    root, lay, slots, offs = store
    write_layer(str(root), 3, slots, H, I, G, offs)
    assert np.array_equal(capi.expert_layer_read(root, 3, lay, 0, E), slots)
    assert np.array_equal(capi.expert_layer_read(root, 3, lay, 2, 3), slots[2:5])


@pytest.mark.parametrize("edit,match", [
    (lambda m: m.update(format="FIXED_DENSE_EXPERT_LAYER_V1"), "unsupported expert storage format"),
    (lambda m: m.update(layer=4), "describes layer 4"),
    (lambda m: m.update(expert_size=m["expert_size"] + 16), "unsupported expert slot size"),
    (lambda m: m.update(experts=0), "zero experts"),
    (lambda m: m["packs"][1].update(expert=0), "duplicate expert 0"),
    (lambda m: m["packs"][1].update(expert=99), "outside 0..6"),
    (lambda m: m["packs"][2].update(packed_bytes=m["expert_size"] + 1), "exceeds slot size"),
    (lambda m: m["packs"].pop(4), "no metadata for expert 4"),
    (lambda m: m["packs"][0]["records"][1].update(record_offset=0), "does not match the layout"),
    (lambda m: m["packs"][0]["records"][2].update(shape=[I, H]), "does not match the layout"),
    (lambda m: m["packs"][0]["records"][0].update(group_size=64), "does not match the layout"),
    (lambda m: m["packs"][0]["records"][0].update(tensor="x.up_proj.weight"), "not a gate_proj.weight record"),
    (lambda m: m["packs"][0].update(records=m["packs"][0]["records"][:2]), "expected gate, up and down"),
])
def test_invalid_metadata(store, edit, match):
    from pb_b200 import capi

    root, lay, slots, offs = store
    write_layer(str(root), 3, slots, H, I, G, offs, meta_edit=edit)
    with pytest.raises(capi.PbmoeError, match=match):
        capi.expert_layer_read(root, 3, lay, 0, E)


def test_range_outside_and_short_file(store):
    from pb_b200 import capi

    root, lay, slots, offs = store
    write_layer(str(root), 0, slots, H, I, G, offs)
    with pytest.raises(capi.PbmoeError, match="outside the 6"):
        capi.expert_layer_read(root, 0, lay, 4, 3)
    with open(root / "layer_00.bin", "r+b") as f:
        f.truncate(lay.expert_bytes * 4 + 10)
    with pytest.raises(capi.PbmoeError, match="shorter than experts"):
        capi.expert_layer_read(root, 0, lay, 0, E)
    assert np.array_equal(capi.expert_layer_read(root, 0, lay, 1, 3), slots[1:4])


def test_missing_and_malformed_metadata(store):
    from pb_b200 import capi

    root, lay, slots, offs = store
    with pytest.raises(capi.PbmoeError, match="cannot be read"):
        capi.expert_layer_read(root, 7, lay, 0, 1)
    write_layer(str(root), 7, slots, H, I, G, offs)
    (root / "layer_07.json").write_text('{"format": "FIXED_Q4_EXPERT_LAYER_V1", "layer": 7,')
    with pytest.raises(capi.PbmoeError, match="failed to parse"):
        capi.expert_layer_read(root, 7, lay, 0, 1)


def test_partial_groups_rejected(tmp_path):
    """The reference's fixed layout allows a partial last group (its test at
    experts/parity_tests.rs:405-461 uses a down projection of 2 columns with
    group 64); the kernels here need whole groups, so such a store is
    refused: pbmoe_fixed_q4_layout rejects the shape outright."""
    from pb_b200 import capi

    with pytest.raises(capi.PbmoeError):
        capi.fixed_q4_layout(64, 2, 64)


def test_record_offsets_are_the_weight_components(store):
    """Each record's record_offset is its projection's nibble offset in the
    slot (gate, up, down), as fixed_q4_pack_from_pbq4_records writes it."""
    from expert_store_writer import records_for

    _, lay, _, offs = store
    recs = records_for(0, 0, H, I, G, offs)
    assert [r["record_offset"] for r in recs] == [offs[0], offs[3], offs[6]]
    assert offs[3] == offs[0] + I * H // 2 + 2 * 2 * I * (H // G)


# ---------------------------------------------------------------- PBQ4 packs
def _pbq4_store(tmp_path, f32, order=(0, 1, 2), pack_edit=None, corrupt=None):
    """Three experts as PBQ4 packs and the fixed-Q4 slot images they must give."""
    from expert_store_writer import bf16_bytes, pbq4_pack, write_pbq4_layer

    from pb_b200 import capi

    lay = capi.fixed_q4_layout(H, I, G)
    offs = list(lay.component_offsets)
    rng = np.random.default_rng(7)
    packs, want = [], []
    for e in range(3):
        parts, slot = [], bytearray(lay.expert_bytes)
        for j, (rows, cols) in enumerate(((I, H), (I, H), (H, I))):
            nib = rng.integers(0, 256, rows * cols // 2, dtype=np.uint8)
            sc = (rng.uniform(0.004, 0.02, rows * cols // G)).astype(np.float32)
            bi = (rng.standard_normal(rows * cols // G) * 0.1).astype(np.float32)
            parts.append((rows, cols, G, nib, sc, bi))
            slot[offs[3 * j]:offs[3 * j] + len(nib)] = nib.tobytes()
            slot[offs[3 * j + 1]:offs[3 * j + 1] + 2 * len(sc)] = bf16_bytes(sc)
            slot[offs[3 * j + 2]:offs[3 * j + 2] + 2 * len(bi)] = bf16_bytes(bi)
        data, recs = pbq4_pack(1, e, parts, f32, order)
        if corrupt:
            data = corrupt(e, data)
        packs.append((data, recs))
        want.append(np.frombuffer(bytes(slot), np.uint8))
    size = max(len(d) for d, _ in packs) + 64
    write_pbq4_layer(str(tmp_path), 1, packs, size, pack_edit=pack_edit)
    return lay, np.stack(want)


@pytest.mark.parametrize("f32", [True, False])
def test_pbq4_becomes_fixed_slots(tmp_path, f32):
    """A PBQ4 layer (PBQ4EXPERT_LAYER_V2) reads as the fixed-Q4 images
    fixed_q4_pack_from_pbq4_records builds: nibbles copied, f32 scales and
    biases rounded to bf16 (experts/slots.rs:984-1169)."""
    from pb_b200 import capi

    lay, want = _pbq4_store(tmp_path, f32)
    assert np.array_equal(capi.expert_layer_read(tmp_path, 1, lay, 0, 3), want)
    assert np.array_equal(capi.expert_layer_read(tmp_path, 1, lay, 1, 2), want[1:])


def test_pbq4_record_order_free(tmp_path):
    from pb_b200 import capi

    lay, want = _pbq4_store(tmp_path, True, order=(2, 0, 1))
    assert np.array_equal(capi.expert_layer_read(tmp_path, 1, lay, 0, 3), want)


@pytest.mark.parametrize("corrupt,edit,match", [
    (lambda e, d: b"XBQ4EXPERT " + d[11:], None, "missing PBQ4EXPERT header"),
    (lambda e, d: d + b"\0", None, "trailing bytes"),
    (None, lambda m: m["packs"][0]["records"][1].update(record_offset=m["packs"][0]["records"][1]["record_offset"] + 4),
     "metadata offset mismatch"),
    (lambda e, d: d.replace(b"up_proj", b"up_prox", 1), None, "name mismatch"),
    (None, lambda m: m["packs"][2]["records"][0].update(scale_bias_dtype="F16"), "does not match the layout"),
])
def test_pbq4_invalid(tmp_path, corrupt, edit, match):
    """Each check of parse_pbq4_expert_pack_with_metadata failing with its message
    (the metadata's pack length always follows the bytes written)."""
    from pb_b200 import capi

    lay, _ = _pbq4_store(tmp_path, True, pack_edit=edit, corrupt=corrupt)
    with pytest.raises(capi.PbmoeError, match=match):
        capi.expert_layer_read(tmp_path, 1, lay, 0, 3)


def test_pbq4_duplicate_projection(tmp_path):
    from pb_b200 import capi

    def dup(meta):
        meta["packs"][0]["records"][1]["tensor"] = meta["packs"][0]["records"][0]["tensor"]

    lay, _ = _pbq4_store(tmp_path, True, pack_edit=dup)
    with pytest.raises(capi.PbmoeError, match="distinct projection"):
        capi.expert_layer_read(tmp_path, 1, lay, 0, 3)


def test_metadata_json_forms(store):
    """serde's output variants parse: pretty-printed, source_hash null or a
    string, escaped characters in other fields, unknown fields ignored."""
    import json

    from pb_b200 import capi

    root, lay, slots, offs = store

    def edit(m):
        m["generator"] = {"name": 'pb "cache"\n', "version": [1, 2.5, -3, True, None]}
        for p in m["packs"]:
            for i, r in enumerate(p["records"]):
                r["source_hash"] = None if i % 2 else "ab\u00e9cd"
                r["dtype"] = "BF16\t"

    write_layer(str(root), 5, slots, H, I, G, offs, meta_edit=edit)
    path = root / "layer_05.json"
    path.write_text(json.dumps(json.loads(path.read_text()), indent=2))
    assert np.array_equal(capi.expert_layer_read(root, 5, lay, 0, E), slots)


def test_metadata_numbers_must_be_integers(store):
    from pb_b200 import capi

    root, lay, slots, offs = store
    write_layer(str(root), 6, slots, H, I, G, offs, meta_edit=lambda m: m.update(expert_size=float(m["expert_size"])))
    with pytest.raises(capi.PbmoeError, match="lacks layer/expert_size/experts"):
        capi.expert_layer_read(root, 6, lay, 0, E)


def test_fixed_mxfp4_layout_offsets():
    """QwenMoeQ4ExpertLayout::fixed_mxfp4 (model_family.rs:846-952): per
    projection the nibbles then one E8M0 byte per group, zero-byte biases."""
    from pb_b200 import capi

    lay = capi.fixed_mxfp4_layout(64, 32, 32)
    gw, gs = 32 * 64 // 2, 32 * (64 // 32)
    dw, ds = 64 * 32 // 2, 64 * (32 // 32)
    assert list(lay.component_offsets) == [0, gw, gw + gs, gw + gs, 2 * gw + gs, 2 * gw + 2 * gs,
                                           2 * gw + 2 * gs, 2 * gw + 2 * gs + dw, 2 * gw + 2 * gs + dw + ds]
    assert lay.expert_bytes == 2 * gw + 2 * gs + dw + ds
    big = capi.fixed_mxfp4_layout(2048, 512, 32)
    assert big.expert_bytes == 3 * (2048 * 512 // 2 + 2048 * 512 // 32)
    with pytest.raises(capi.PbmoeError):
        capi.fixed_mxfp4_layout(64, 48, 32)


def test_mxfp4_layer_reads_as_stored(tmp_path):
    """A FIXED_MXFP4_EXPERT_LAYER_V1 layer: slots as stored, checked at the
    pack level only; a Q4 layout is refused for it."""
    from pb_b200 import capi

    lay = capi.fixed_mxfp4_layout(H, I, 32)
    rng = np.random.default_rng(4)
    slots = rng.integers(0, 256, (E, lay.expert_bytes), dtype=np.uint8)

    def fmt(m):
        m["format"] = "FIXED_MXFP4_EXPERT_LAYER_V1"
        for p in m["packs"]:
            p["records"] = []

    write_layer(str(tmp_path), 2, slots, H, I, 32, list(lay.component_offsets), meta_edit=fmt)
    assert np.array_equal(capi.expert_layer_read(tmp_path, 2, lay, 1, 4), slots[1:5])
    with pytest.raises(capi.PbmoeError, match="MXFP4 layout"):
        capi.expert_layer_read(tmp_path, 2, capi.fixed_q4_layout(H, I, 32), 0, 1)


def test_mxfp4_layer_refuses_other_offsets(tmp_path):
    """An MXFP4 layer read with offsets other than the fixed MXFP4 image's
    (here the up nibbles moved but the slot size and empty biases kept) would
    read its bytes in the wrong places, so it is refused."""
    from pb_b200 import capi

    lay = capi.fixed_mxfp4_layout(H, I, 32)
    rng = np.random.default_rng(5)
    slots = rng.integers(0, 256, (E, lay.expert_bytes), dtype=np.uint8)

    def fmt(m):
        m["format"] = "FIXED_MXFP4_EXPERT_LAYER_V1"
        for p in m["packs"]:
            p["records"] = []

    write_layer(str(tmp_path), 2, slots, H, I, 32, list(lay.component_offsets), meta_edit=fmt)
    bad = capi.fixed_mxfp4_layout(H, I, 32)
    bad.component_offsets[3] += 16  # up nibbles shifted; gate scales now overlap them
    with pytest.raises(capi.PbmoeError, match="fixed MXFP4 layout"):
        capi.expert_layer_read(tmp_path, 2, bad, 0, 1)
    assert np.array_equal(capi.expert_layer_read(tmp_path, 2, lay, 0, 2), slots[:2])
