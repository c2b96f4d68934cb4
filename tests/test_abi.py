"""The C-ABI library loads and exports every entry point include/*.h declares
(no compute: this runs without a GPU)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

from cacheslide_b200 import _native as N

HEADERS = sorted((Path(__file__).resolve().parents[1] / "include").glob("*.h"))


def declared() -> set[str]:
    names = set()
    for h in HEADERS:
        text = h.read_text()
        names |= set(re.findall(r"^CS_API\s+[\w\s\*]+?\b(cs_\w+)\s*\(", text, re.M))
    return names


def test_header_declares_entry_points():
    names = declared()
    for required in ("cs_slide_gather", "cs_slide_scatter", "cs_slide_relocate",
                     "cs_wca_deviation", "cs_wca_select_topk", "cs_wca_update",
                     "cs_cope_attn", "cs_cope_attn_prefill", "cs_cope_attn_decode"):
        assert required in names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(N.LIB_PATH))
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_every_declared_symbol():
    assert declared() <= set(N.EXPORTED)
    lib = N.load()
    assert lib.cs_abi_version() == 2
    assert b"sm_100a" in lib.cs_build_info()


def test_struct_layouts_match_the_header():
    # cs_paged_kv: 1 ptr + 8 int64 + 2 ptr + 4 int64 + int32 (+pad) = 128 bytes
    assert ctypes.sizeof(N.PagedKV) == 128
    assert ctypes.sizeof(N.AttnParams) % 8 == 0
