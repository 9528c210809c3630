"""The C-ABI library loads without a GPU and exports exactly what
include/pageserve_b200.h declares (no compute calls here)."""

import ctypes
import re
from pathlib import Path

import pytest

from pageserve_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent


def _declared():
    txt = (ROOT / "include" / "pageserve_b200.h").read_text()
    return sorted(set(re.findall(r"PS_API\s+[\w\s\*]+?\b(ps_\w+)\s*\(", txt)))


def test_header_declares_entry_points():
    names = _declared()
    assert "ps_paged_attention" in names and "ps_w8a16_linear" in names
    assert len(names) >= 15


def test_library_exports_every_declared_symbol():
    if not _lib.LIB_PATH.exists():
        pytest.skip("libpageserve_b200.so not built (run python -m pageserve_b200.build)")
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in _declared() if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_python_binding_covers_header():
    declared = set(_declared())
    bound = set(_lib.exported_symbols())
    assert declared <= bound, f"no ctypes signature for {sorted(declared - bound)}"
    assert bound <= declared, f"ctypes signature for undeclared {sorted(bound - declared)}"


def test_library_metadata_calls_without_gpu():
    if not _lib.LIB_PATH.exists():
        pytest.skip("library not built")
    lib = _lib.load()
    assert lib.ps_abi_version() == 1
    assert isinstance(lib.ps_launch_count(), int)
    # size queries are pure host arithmetic
    assert lib.ps_paged_attention_workspace_size(64, 1, 4096, 16, 2, 128) > 0
    # a prefill chunk shorter than two key tiles runs unsplit: no scratch
    assert lib.ps_paged_attention_workspace_size(1, 64, 64, 16, 2, 128) == 0


def test_host_validation_errors_without_gpu():
    """Validation runs before any launch, so these never touch a device."""
    if not _lib.LIB_PATH.exists():
        pytest.skip("library not built")
    lib = _lib.load()
    # block table of 1 entry cannot hold position 16 at block size 16 -> IndexError
    rc = lib.ps_write_kv(1, 1, 1, 1, 4, 16, 2, 64, _lib.PS_BF16, 16, 1, 1, 1, None)
    assert rc == _lib.PS_ERR_INDEX
    with pytest.raises(IndexError):
        _lib.check(rc, "write_kv")
    rc = lib.ps_paged_attention(1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 1, 40, 4, 16, 16, 2, 128, _lib.PS_BF16, None, 0, None)
    assert rc == _lib.PS_ERR_INDEX
    rc = lib.ps_paged_attention(1, 1, 1, 1, 1, 4, 1, 1, 1, 1, 1, 40, 4, 16, 15, 2, 128, _lib.PS_BF16, None, 0, None)
    assert rc == _lib.PS_ERR_INVALID  # 15 q heads over 2 kv heads
    with pytest.raises(ValueError):
        _lib.check(rc, "paged_attention")
