"""The C-ABI library loads and exports every symbol include/algx.h declares (no GPU needed)."""

import ctypes
import os
import re

from algx import _lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "algx.h")).read()
    return sorted(set(re.findall(r"ALGX_API\s+[\w\s\*]+?\b(algx_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "algx_attn_fwd" in names and "algx_qknorm_bwd" in names
    assert len(names) >= 10


def test_library_exports_every_declared_symbol():
    handle = ctypes.CDLL(L.LIB_PATH)
    missing = [n for n in declared_symbols() if not hasattr(handle, n)]
    assert not missing, missing


def test_binding_covers_every_declared_symbol():
    assert set(declared_symbols()) <= set(L.SIGNATURES)


def test_version_and_error_string_without_gpu():
    lib = L.lib()
    assert lib.algx_version() >= 100
    assert isinstance(lib.algx_last_error(), bytes)


def test_workspace_queries_are_host_only():
    lib = L.lib()
    assert lib.algx_qknorm_bwd_workspace_size(196608, 64) > 0
    assert lib.algx_attn_bwd_workspace_size(8, 12, 2048, 64) >= 8 * 12 * 2048 * 4


def test_every_declaration_cites_the_reference_or_says_it_has_none():
    """Each entry point's comment names the reference function it replaces
    (file.py:line) or states that it has no counterpart in the reference."""
    text = open(os.path.join(ROOT, "include", "algx.h")).read()
    decls = [(m.start(), text.index(";", m.start()), m.group(1))
             for m in re.finditer(r"ALGX_API[^;]*?\b(algx_\w+)\s*\(", text)]
    missing, prev_end = [], 0
    for start, end, name in decls:
        chunk = text[prev_end:start]
        if not (re.search(r"\.py:\d", chunk) or re.search(r"[Nn]o counterpart", chunk)):
            missing.append(name)
        prev_end = end
    assert len(decls) >= 30 and not missing, missing
