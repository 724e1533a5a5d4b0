"""CPU tests: the C-ABI library loads and exports every entry point include/sonic_b200.h declares,
and the Python binding declares a signature for each of them.  No compute calls (no GPU here)."""
import os
import re
import subprocess

import pytest

from conftest import ROOT

HEADER_DIR = os.path.join(ROOT, "include")


def declared_functions():
    names = []
    for fn in sorted(os.listdir(HEADER_DIR)):
        if fn.endswith(".h"):
            text = open(os.path.join(HEADER_DIR, fn)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            names += re.findall(r"\b(sm_[a-z0-9_]+)\s*\(", text)
    return sorted(set(names))


@pytest.fixture(scope="module")
def lib_path():
    import sys

    sys.path.insert(0, os.path.join(ROOT, "sonic-moe_b200"))
    import build  # sonic-moe_b200/build.py

    return build.build()


def test_header_declares_entry_points():
    names = declared_functions()
    for n in ("sm_router_topk", "sm_route_metadata", "sm_moe_forward", "sm_weight_prep", "sm_moe_up",
              "sm_moe_down_combine", "sm_quant_pack", "sm_last_error"):
        assert n in names


def test_library_exports_every_declared_symbol(lib_path):
    out = subprocess.run(["nm", "-D", "--defined-only", lib_path], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (sm_[a-z0-9_]+)", out))
    missing = [n for n in declared_functions() if n not in exported]
    assert not missing, f"declared but not exported: {missing}"


def test_library_loads_and_binding_covers_header(lib_path):
    from sonicmoe import _native

    lib = _native.load()
    assert lib.sm_version().decode().startswith("sonic_b200")
    assert set(declared_functions()) <= set(_native.SIGNATURES), "binding lacks a declared entry point"
    # host-only entry points (no device work)
    assert lib.sm_max_padded_blocks(262144, 128) == 262144 // 128 + 128
    assert lib.sm_moe_workspace_bytes(256, 512, 256, 8, 2) > 0
    assert lib.sm_weight_sf_bytes(8, 512, 512) == 8 * 4 * 1 * 512


def test_argument_validation_without_gpu(lib_path):
    """Shape errors are reported before any CUDA call."""
    from sonicmoe import _native

    lib = _native.load()
    rc = lib.sm_router_topk(None, 0, 4, 8, 9, 1, 0, None, None, None)  # K > E
    assert rc == _native.SM_EINVAL
    assert "K must be" in lib.sm_last_error().decode()
    rc = lib.sm_router_topk(None, 0, 4, 8, 2, 1, 1, None, None, None)  # renorm with softmax-over-topk
    assert rc == _native.SM_EINVAL
    rc = lib.sm_moe_forward(*([None, None, 4, 100, 128, 8, 2, 1, 0, 0] + [None] * 9 + [0, None, None]))
    assert rc == _native.SM_ENOTSUP  # H % 256 != 0
