"""The C-ABI library loads and exports every function ``include/*.h`` declares
(no compute call: this runs without a GPU)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]


def _declared() -> list[str]:
    names = []
    for h in sorted((REPO / "include").glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names += re.findall(r"\b(kvd_[a-z0-9_]+)\s*\(", text)
    return sorted(set(names))


def test_library_exports_every_declared_symbol() -> None:
    from kvdlra_b200 import _native
    from kvdlra_b200.build import build

    if not _native.LIB_PATH.exists():
        build()
    lib = ctypes.CDLL(str(_native.LIB_PATH))
    names = _declared()
    assert len(names) >= 10
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_library_reports_errors_without_a_gpu() -> None:
    from kvdlra_b200 import _native as N

    L = N.lib()
    assert L.kvd_version() >= 1
    cfg = N.Config()  # all zeros: invalid
    assert L.kvd_workspace_bytes(ctypes.byref(cfg)) == 0
    assert b"invalid" in L.kvd_last_error()


def test_struct_layouts_match_header() -> None:
    """ctypes mirrors of the C structs have the header's field order."""
    from kvdlra_b200 import _native as N

    text = (REPO / "include" / "kvdlra_b200.h").read_text()
    for struct, cls in (("kvd_config", N.Config), ("kvd_counters", N.Counters)):
        body = re.search(r"typedef struct %s \{(.*?)\} %s;" % (struct, struct), text, re.S).group(1)
        body = re.sub(r"/\*.*?\*/", "", body)
        fields = re.findall(r"([a-z_]+)(?:\[\d\])?\s*;", body.replace(",", ";"))
        assert [f for f, _ in cls._fields_] == fields, struct
