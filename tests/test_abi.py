"""libgplk.so loads on any machine and exports every symbol the C headers
declare (no compute calls: those need a GPU)."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent


def declared_functions() -> dict[str, list[str]]:
    out = {}
    for h in sorted((REPO / "include").glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        text = re.sub(r"//[^\n]*", "", text)
        names = re.findall(r"\b((?:gplk|gpl)_\w+)\s*\(", text)
        # drop typedef'd function-pointer / macro uses: keep identifiers that
        # appear as a declaration (preceded by a type on the same statement)
        out[h.name] = sorted(set(n for n in names if not n.isupper()))
    return out


def test_headers_declare_entry_points():
    decl = declared_functions()
    assert "gplk.h" in decl and "gplk_triad_f32" in decl["gplk.h"]


def test_library_exports_every_declared_symbol(gplk):
    """include/gplk_nodemon.h is the host-only node sampler
    (libgplk_nodemon.so); every other header is libgplk.so's."""
    from gplk import nodemon

    libs = {"gplk_nodemon.h": ctypes.CDLL(str(nodemon.LIB_PATH))}
    main = ctypes.CDLL(str(gplk.LIB_PATH))
    missing = [(h, n) for h, names in declared_functions().items() for n in names
               if not hasattr(libs.get(h, main), n)]
    assert not missing, missing


def test_status_strings(gplk):
    L = gplk.lib()
    assert L.gplk_status_string(0) == b"ok"
    assert L.gplk_status_string(3) == b"device wait timeout"
    assert L.gplk_abi_version() >= 1


def test_sf_bytes_matches_oracle(gplk, oracle):
    for rows, k in [(1, 256), (128, 256), (129, 512), (16384, 16384), (2048, 4096)]:
        assert gplk.nvfp4_sf_bytes(rows, k) == oracle.sf_bytes(rows, k)
