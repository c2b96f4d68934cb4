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
    assert lib.cs_abi_version() == 3
    assert b"sm_100a" in lib.cs_build_info()


def test_struct_layouts_match_the_header():
    # cs_paged_kv: 1 ptr + 8 int64 + 2 ptr + 4 int64 + int32 (+pad) = 128 bytes
    assert ctypes.sizeof(N.PagedKV) == 128
    assert ctypes.sizeof(N.AttnParams) % 8 == 0


def test_struct_sizes_equal_the_c_compilers(tmp_path):
    """Every struct the binding mirrors has the size a C compiler gives the
    header's declaration (fields in the same order, same types)."""
    import shutil
    import subprocess

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        import pytest

        pytest.skip("no C compiler")
    pairs = {"cs_paged_kv": N.PagedKV, "cs_attn_params": N.AttnParams,
             "cs_slide_scatter_item": N.ScatterItem, "cs_wca_initialize_item": N.InitializeItem,
             "cs_wca_update_item": N.UpdateItem, "cs_wca_commit_item": N.CommitItem,
             "cs_qkv_params": N.QKVParams}
    src = tmp_path / "sizes.c"
    src.write_text('#include <stdio.h>\n#include "cacheslide_b200.h"\nint main(void) {\n'
                   + "".join(f'  printf("{k} %zu\\n", sizeof({k}));\n' for k in pairs)
                   + "  return 0;\n}\n")
    exe = tmp_path / "sizes"
    subprocess.run([cc, "-std=c11", "-I", str(HEADERS[0].parent), str(src), "-o", str(exe)],
                   check=True)
    got = dict(line.split() for line in subprocess.run(
        [str(exe)], check=True, capture_output=True, text=True).stdout.splitlines())
    for name, struct in pairs.items():
        assert int(got[name]) == ctypes.sizeof(struct), name
