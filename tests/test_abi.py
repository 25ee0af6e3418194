"""The C-ABI library: it builds for sm_100a, loads without a GPU, and exports
every entry point include/miniep_b200.h declares (no compute calls here)."""
import ctypes as C
import re
from pathlib import Path

import pytest

from miniep_b200 import _lib, build

HEADER = Path(__file__).resolve().parents[1] / "include" / "miniep_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mep_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.lib()


def test_header_declares_the_layer_step():
    names = declared_functions()
    for must in ("mep_ctx_create", "mep_router_topk", "mep_dest_ranks", "mep_moe_forward",
                 "mep_moe_block", "mep_route", "mep_dispatch", "mep_expert_ffn", "mep_combine",
                 "mep_read_stats", "mep_check"):
        assert must in names


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared but not exported"


def test_binding_covers_the_header(lib):
    assert sorted(_lib.SIGNATURES) == declared_functions()


def test_version_and_error_paths_without_gpu(lib):
    assert lib.mep_version() >= 100
    ctx = C.c_void_p()
    # invalid arguments are rejected before any CUDA call
    rc = lib.mep_ctx_create(0, 9, 0, 1, 32, 8, 1024, 512, 16, 1, 0, C.byref(ctx))
    assert rc == 1 and b"world" in lib.mep_last_error(None)
    rc = lib.mep_ctx_create(0, 1, 0, 1, 32, 8, 1000, 512, 16, 1, 0, C.byref(ctx))
    assert rc == 1
    rc = lib.mep_ctx_create(0, 1, 0, 1, 32, 40, 1024, 512, 16, 1, 0, C.byref(ctx))
    assert rc == 1 and b"topk" in lib.mep_last_error(None)
    assert not ctx.value
