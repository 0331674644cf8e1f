"""CPU checks of the C-ABI library: it builds, loads without a GPU, and
exports exactly the entry points include/pbmoe_cuda.h declares."""

import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "pbmoe_cuda.h")


@pytest.fixture(scope="module")
def lib_path():
    from pb_b200 import build

    return build.build()


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"PBMOE_API\s+[\w\s\*]*?\b(pbmoe_\w+)\s*\(", text)))


def test_header_declares_binding_list():
    from pb_b200 import capi

    assert declared_symbols() == sorted(capi.EXPORTED)


def test_library_exports_every_declared_symbol(lib_path):
    out = subprocess.run(["nm", "-D", "--defined-only", lib_path], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\b(pbmoe_\w+)\b", out))
    missing = set(declared_symbols()) - exported
    assert not missing, f"missing exports: {missing}"
    extra = exported - set(declared_symbols())
    assert not extra, f"undeclared exports: {extra}"


def test_library_loads_without_gpu(lib_path):
    lib = ctypes.CDLL(lib_path)
    for name in declared_symbols():
        assert hasattr(lib, name)
    assert lib.pbmoe_abi_version() == 2


def test_host_only_entry_points(lib_path):
    from pb_b200 import capi

    lay = capi.fixed_q4_layout(2048, 512, 64)
    assert lay.expert_bytes == 1_769_472
    assert list(lay.component_offsets) == [0, 524288, 557056, 589824, 1114112, 1146880, 1179648, 1703936, 1736704]
    with pytest.raises(capi.PbmoeError):
        capi.fixed_q4_layout(2048, 500, 64)
    cfg = capi.moe_config(lay, 512, 10)
    assert capi.load().pbmoe_moe_workspace_bytes(1, ctypes.byref(cfg)) > 0


def test_init_without_device_fails_cleanly(lib_path):
    """With no CUDA device, pbmoe_init reports PBMOE_ERR_CUDA instead of crashing."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from pb_b200 import capi

    h = ctypes.c_void_p()
    assert capi.load().pbmoe_init(0, ctypes.byref(h)) == capi.PBMOE_ERR_CUDA
