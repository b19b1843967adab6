"""The C-ABI library loads on the CPU host and exports every symbol that
include/*.h declares (no compute call is made without a GPU)."""

import ctypes
import glob
import os
import re

from conftest import ROOT


def declared_symbols():
    names = set()
    for header in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(header).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"\b(akv_[a-z0-9_]+)\s*\(", text):
            names.add(m.group(1))
    return names


def test_header_declares_entry_points():
    names = declared_symbols()
    for required in ("akv_reposition_kv_layers", "akv_drop_compact", "akv_context_decode_indices",
                     "akv_context_window_lengths", "akv_write_row_slots",
                     "akv_build_decode_metadata"):
        assert required in names


def test_library_exports_every_declared_symbol():
    from akv_b200 import _native

    lib = ctypes.CDLL(_native.LIB_PATH)
    missing = [n for n in sorted(declared_symbols()) if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_every_declared_symbol():
    from akv_b200 import _native

    assert declared_symbols() == set(_native.SIGNATURES)


def test_host_only_entry_points():
    from akv_b200 import _native

    assert _native.lib.akv_version().startswith(b"akv_b200")
    assert _native.lib.akv_drop_compact_tile_tokens() == 512
    assert _native.lib.akv_drop_compact_workspace_bytes(64, 700) > 0


def test_argument_errors_are_reported_before_any_launch():
    """Bad sizes are rejected on the host: AKV_ERR_INVALID, nothing enqueued."""
    from akv_b200 import _native

    lib = _native.lib
    # rotary_dim odd
    assert lib.akv_reposition_kv_layers(
        None, None, 1, 1, 8, 64, 63, 512, 64, 512, 64, None, None, None, 2, 5, None, None,
        2, 64, 1, 0, 0, 0, None, None) == _native.AKV_ERR_INVALID
    # zero transitions: nothing to do, OK without a GPU
    assert lib.akv_reposition_kv_layers(
        None, None, 1, 1, 8, 64, 64, 512, 64, 512, 64, None, None, None, 2, 0, None, None,
        2, 64, 1, 0, 0, 0, None, None) == _native.AKV_OK
    assert lib.akv_context_decode_indices(
        None, None, 0, None, 0, None, 0, None, 0, None, 0, None, 0, None, 0, 1, 4,
        None) == _native.AKV_ERR_INVALID
    assert lib.akv_write_row_slots(None, None, 0, None, 0, None, 0, 0, None) == _native.AKV_OK
    # reposition options: unknown bits are refused; the bulk V move is a known bit
    assert lib.akv_reposition_kv_layers_ex(
        None, None, 1, 1, 8, 64, 64, 512, 64, 512, 64, None, None, None, 2, 0, None, None,
        2, 64, 1, 0, 0, 0, None, 2, None) == _native.AKV_ERR_INVALID
    assert lib.akv_reposition_kv_layers_ex(
        None, None, 1, 1, 8, 64, 64, 512, 64, 512, 64, None, None, None, 2, 0, None, None,
        2, 64, 1, 0, 0, 0, None, _native.REPOSITION_BULK_V, None) == _native.AKV_OK
    # paged Drop: page sizes other than 1 and powers of two in [4, 128]
    for bad in (2, 12, 256, 0, -16):
        args = [0, None, None, 0, None, None, None, None, None, 0, 1, bad, None, 1]
        assert lib.akv_drop_compact_paged(*args, *([None] * 18)) == _native.AKV_ERR_INVALID
    assert lib.akv_occurrence_advance_indices(None, None) == _native.AKV_ERR_INVALID
    # decode-view read-back: a missing host vector, a negative count, or a
    # view without its device vectors is refused before any copy
    import ctypes

    buf = (ctypes.c_int32 * 16)()
    p1 = ctypes.cast(buf, ctypes.c_void_p)
    assert lib.akv_drop_read_view(None, p1, p1, 1, p1, p1, 1, p1, None) == \
        _native.AKV_ERR_INVALID
    assert lib.akv_drop_read_view(p1, p1, p1, -1, p1, p1, 1, p1, None) == \
        _native.AKV_ERR_INVALID
    assert lib.akv_drop_read_view(p1, None, None, 3, p1, p1, 1, p1, None) == \
        _native.AKV_ERR_INVALID
    assert lib.akv_drop_read_view(p1, p1, p1, 0, None, p1, 1, p1, None) == \
        _native.AKV_ERR_INVALID


def test_layout_batch_struct_matches_the_header():
    """The ctypes mirror of akv_layout_batch has the C struct's size, and
    every field name of the header, in order."""
    import ctypes

    from akv_b200 import _native

    assert ctypes.sizeof(_native.LayoutBatch) == _native.lib.akv_compile_layouts_batch_bytes()
    text = open(os.path.join(ROOT, "include", "akv_b200.h")).read()
    body = text[text.index("typedef struct akv_layout_batch {"):]
    body = re.sub(r"/\*.*?\*/", "", body[: body.index("} akv_layout_batch;")], flags=re.S)
    names = re.findall(r"\b([a-z_0-9]+);", body)
    assert names == [f[0] for f in _native.LayoutBatch._fields_]
    assert _native.lib.akv_compile_layouts_max_repositions() >= 1024
    assert _native.lib.akv_compile_layouts_workspace_bytes(3, 5000, 10, 300) > 0
    assert _native.lib.akv_compile_layouts(None, None) == _native.AKV_ERR_INVALID


def _header_fields(text, typedef_end):
    """Field names of the plain C struct ending at ``} <typedef_end>;``."""
    end = text.index("} " + typedef_end + ";")
    body = text[text.rindex("typedef struct", 0, end): end]
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    names = []
    for decl in body.split("{", 1)[1].split(";"):
        decl = decl.strip()
        if decl:
            names += [n.strip().lstrip("*") for n in decl.split(" ", 1)[1].split(",")] \
                if " " in decl else []
    return [n.split()[-1].lstrip("*") for n in names]


def test_occurrence_structs_match_the_header():
    """The ctypes mirrors of akv_advance_in / akv_advance_out have the
    header's fields, in order."""
    from akv_b200 import context_occurrence as co

    text = open(os.path.join(ROOT, "include", "akv_b200.h")).read()
    assert _header_fields(text, "akv_advance_in") == [f[0] for f in co._AdvanceIn._fields_]
    assert _header_fields(text, "akv_advance_out") == [f[0] for f in co._AdvanceOut._fields_]
