"""Host-side validation of the MoE layer entry points, on CPU (no GPU call is
reached): pbmoe_moe_layer_static applies the same layout and config checks as
pbmoe_moe_layer (one shared validator), so a slot component that runs past
the slot is refused before anything is launched, with the same status codes."""

import ctypes

import pytest

FAKE = 1 << 20  # a 16-byte aligned stand-in address: validation never dereferences it


def _static(cfg, tokens=1):
    from pb_b200 import capi

    w = capi.MoeWeights(FAKE, FAKE, None, None, None)
    err = ctypes.create_string_buffer(512)
    rc = capi.load().pbmoe_moe_layer_static(ctypes.byref(cfg), ctypes.byref(w), ctypes.c_void_p(FAKE),
                                            capi.PBMOE_BF16, None, ctypes.c_void_p(FAKE), capi.PBMOE_BF16, tokens,
                                            None, None, None, err, len(err), None)
    return rc, err.value.decode()


def _cfg(edit=None, top_k=10):
    from pb_b200 import capi

    lay = capi.fixed_q4_layout(2048, 512, 64)
    if edit:
        edit(lay)
    return capi.moe_config(lay, 512, top_k)


def test_valid_config_with_no_tokens_is_a_no_op():
    from pb_b200 import capi

    rc, msg = _static(_cfg(), tokens=0)
    assert rc == capi.PBMOE_OK and msg == ""


def test_overlong_component_is_refused():
    """down_w's offset stays inside the slot but its 524,288 bytes do not."""
    from pb_b200 import capi

    def edit(lay):
        lay.component_offsets[8] = lay.expert_bytes - 16  # down biases: 32,768 bytes from 16 before the end

    rc, msg = _static(_cfg(edit))
    assert rc == capi.PBMOE_ERR_INVALID_ARGUMENT
    assert "exceeds slot bytes" in msg


def test_misaligned_nibbles_are_unsupported_as_in_pbmoe_moe_layer():
    from pb_b200 import capi

    def edit(lay):
        lay.component_offsets[3] += 8  # up nibbles not 16-byte aligned

    rc, msg = _static(_cfg(edit))
    assert rc == capi.PBMOE_ERR_UNSUPPORTED and "aligned" in msg


@pytest.mark.parametrize("top_k,match", [(0, "top_k"), (33, "top_k")])
def test_config_checks(top_k, match):
    from pb_b200 import capi

    rc, msg = _static(_cfg(top_k=top_k))
    assert rc == capi.PBMOE_ERR_UNSUPPORTED and match in msg


def test_workspace_bytes_match_the_static_capacity():
    """pbmoe_moe_workspace_bytes sizes the static array's capacity: 29
    config-1 tokens fit PBMOE_STATIC_SCRATCH_BYTES (with its 256-byte status
    word), 30 do not."""
    from pb_b200 import capi

    cfg = _cfg()
    need = lambda t: 256 + capi.load().pbmoe_moe_workspace_bytes(t, ctypes.byref(cfg))
    assert need(29) <= 4 << 20 < need(30)


def _mx_cfg(edit=None, hidden=2048, inter=512, group=32):
    from pb_b200 import capi

    lay = capi.fixed_mxfp4_layout(hidden, inter, group)
    if edit:
        edit(lay)
    return capi.moe_config(lay, 512, 10)


def test_expert_layout_struct_and_encodings():
    """pbmoe_expert_layout is 96 bytes with the encoding in its last word; the
    two fixed layouts say which encoding they are."""
    from pb_b200 import capi

    assert ctypes.sizeof(capi.ExpertLayout) == 96
    assert capi.fixed_q4_layout(2048, 512, 64).encoding == capi.PBMOE_EXPERT_AFFINE_Q4
    assert capi.fixed_mxfp4_layout(2048, 512, 32).encoding == capi.PBMOE_EXPERT_MXFP4


def test_mxfp4_layout_is_accepted():
    from pb_b200 import capi

    rc, msg = _static(_mx_cfg(), tokens=0)
    assert rc == capi.PBMOE_OK and msg == ""


def test_mxfp4_group_other_than_32_is_unsupported():
    """The reference builds MXFP4 slots with group 32 only (experts/slots.rs:67-80)."""
    from pb_b200 import capi

    rc, msg = _static(_mx_cfg(group=64))
    assert rc == capi.PBMOE_ERR_UNSUPPORTED and "MXFP4" in msg


def test_mxfp4_overlong_scales_are_refused():
    from pb_b200 import capi

    def edit(lay):
        lay.component_offsets[7] = lay.expert_bytes - 8  # down scales: 32,768 bytes from 8 before the end

    rc, msg = _static(_mx_cfg(edit))
    assert rc == capi.PBMOE_ERR_INVALID_ARGUMENT and "exceeds slot bytes" in msg


def test_unknown_encoding_is_unsupported():
    from pb_b200 import capi

    def edit(lay):
        lay.encoding = 7

    rc, msg = _static(_cfg(edit))
    assert rc == capi.PBMOE_ERR_UNSUPPORTED and "encoding" in msg
