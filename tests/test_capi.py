"""The C-ABI library loads without a GPU and exports every entry point that
include/rmlx_kv.h declares (and nothing named rmlx_ that it does not)."""
import ctypes
import os
import re
import subprocess

import rmlx_kv
from rmlx_kv import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "rmlx_kv.h")


def declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^RMLX_API\s+[\w\s\*]+?\b(rmlx_\w+)\s*\(", src, flags=re.M)))


def exported():
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    return sorted({ln.split()[-1] for ln in out.splitlines() if ln.split() and ln.split()[-1].startswith("rmlx_")})


def test_header_declarations_found():
    names = declared()
    assert len(names) >= 60
    assert "rmlx_kv_gather" in names and "rmlx_block_manager_copy_on_write" in names


def test_every_declared_symbol_is_exported():
    assert declared() == exported()


def test_symbols_resolve_through_ctypes():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    for name in declared():
        assert getattr(lib, name) is not None


def test_version_and_status_strings():
    assert _lib.lib.rmlx_version().decode().count(".") == 2
    assert _lib.lib.rmlx_status_string(_lib.E_DOUBLE_FREE).decode() == "double free"


def test_host_errors_carry_messages():
    m = rmlx_kv.PagedCacheManager(16, 2)
    try:
        m.free(5)
    except rmlx_kv.RmlxError as e:
        assert e.status == _lib.E_RANGE and "out of range" in str(e)
    else:
        raise AssertionError("free of an out-of-range block must fail")


def test_bad_pool_config_rejected_before_device_use():
    # Validation runs before any CUDA call, so this passes with no GPU.
    for kw in ({"quant_bits": 3}, {"group_size": 48, "quant_bits": 8}, {"head_dim": 12}):
        args = dict(num_layers=1, num_kv_heads=1, head_dim=128, block_size=16, num_blocks=4)
        args.update(kw)
        try:
            rmlx_kv.KVPool(**args)
        except rmlx_kv.RmlxError as e:
            assert e.status == _lib.E_BAD_ARG
        else:
            raise AssertionError(f"config {kw} must be rejected")
