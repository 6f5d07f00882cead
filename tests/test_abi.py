"""CPU: the C-ABI library loads and exports every entry point include/tlmg.h
declares; host-only helpers agree with the oracle; no GPU calls."""
from __future__ import annotations

import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def header_functions(path: Path) -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", path.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(tlmg_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_header():
    from tierlm_b200 import _lib
    lib = _lib.load()
    names = []
    for h in sorted((ROOT / "include").glob("*.h")):
        names += header_functions(h)
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    undeclared = [n for n in _lib.declared_symbols() if n not in names]
    assert not undeclared, undeclared


def test_error_and_dtype_codes_match_reference():
    from tierlm_b200 import _lib
    assert (_lib.TLMG_EIO, _lib.TLMG_ENOMEM, _lib.TLMG_EINVAL, _lib.TLMG_EFORMAT, _lib.TLMG_ERANGE,
            _lib.TLMG_ENOTFOUND, _lib.TLMG_EUNSUP, _lib.TLMG_EBUSY) == (-1, -2, -3, -4, -5, -6, -7, -8)
    assert (_lib.F32, _lib.F16, _lib.BF16, _lib.Q8_0, _lib.Q4_K, _lib.Q5_K, _lib.Q6_K, _lib.Q8_K, _lib.MXFP4) == \
        (0, 1, 2, 8, 12, 13, 14, 15, 39)
    hdr = (ROOT / "include" / "tlmg.h").read_text()
    for name, val in (("TLMG_EINVAL", -3), ("TLMG_EUNSUP", -7), ("TLMG_DT_Q6_K", 14), ("TLMG_DT_Q4_K", 12)):
        assert re.search(rf"{name}\s*=\s*{val}\b", hdr), name


def test_host_helpers_match_oracle(orc):
    from tierlm_b200 import _lib
    lib = _lib.load()
    for dt in (0, 1, 2, 8, 12, 13, 14, 15, 39):
        for n in (0, 32, 256, 768, 2048, 100):
            assert lib.tlmg_row_bytes(dt, n) == orc.row_bytes(dt, n)
        assert lib.tlmg_act_kind_for(dt) == orc.act_kind_for(dt)
    for kind in (0, 8, 15):
        for n in (1, 31, 256, 300, 2048):
            assert lib.tlmg_qact_bytes(kind, n) == orc.qact_bytes(kind, n)
    assert lib.tlmg_tier() == b"cuda-sm100a"


def test_no_gpu_fails_loudly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from tierlm_b200 import _lib
    lib = _lib.load()
    rc = lib.tlmg_init(0)
    assert rc == _lib.TLMG_EUNSUP
    assert b"device" in lib.tlmg_errmsg().lower() or b"cuda" in lib.tlmg_errmsg().lower()


def test_product_does_not_import_oracle():
    """The product package never references the CPU checker."""
    for p in (ROOT / "tierlm_b200").rglob("*"):
        if p.suffix in (".py", ".cu", ".cuh", ".h", ".cpp"):
            assert "oracle" not in p.read_text().lower().replace("the oracle", ""), p
