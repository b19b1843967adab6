"""Drop-in decode page-table kernels with the reference's launch syntax.

The reference defines two Triton kernels
(akv/system/sglang/kernels/ops/attention/context_page_table.py:7-76) that
its registry launches as ``kernel[(batch,)](...)``
(srt/layers/attention/context_backend.py:770-783, 791, 804).  The objects
below keep that syntax -- subscripting with a grid returns a launcher with
the same positional and keyword parameters -- and run the sm_100a kernels
of the C ABI (``akv_context_decode_indices``, ``akv_context_window_lengths``)
on the current stream.  The grid's first entry is the batch size, as in the
reference; the native kernel chooses its own block split.
"""

from __future__ import annotations

import torch

from . import _native


class _Launcher:
    def __init__(self, fn, name):
        self._fn = fn
        self.__name__ = name

    def __getitem__(self, grid):
        if callable(grid):
            raise ValueError(f"{self.__name__}: pass an explicit (batch,) grid")
        batch = int(grid[0] if isinstance(grid, (tuple, list)) else grid)
        return lambda *args, **kwargs: self._fn(batch, *args, **kwargs)


def _decode_indices(batch, Registry, Table, Rows, Lengths, Indptr, Output, Starts, Mapping,
                    ROW_STRIDE, TRANSLATE, MULTIPLIER, HAS_START, BLOCK=256):
    """context_page_table.py:34-76: for request b, i < Lengths[b]:
    Output[Indptr[b] + i] = (Mapping[slot] * MULTIPLIER if TRANSLATE else slot)
    with slot = row[raw] and raw from the registry's compacted raw ids."""
    del BLOCK  # the native kernel picks its own tiling
    if Table.dtype != torch.int32 or Registry.dtype != torch.int64:
        raise ValueError("context_decode_indices: int64 registry and int32 req_to_token")
    starts = Starts if HAS_START else None
    mapping = Mapping if TRANSLATE else None
    status = _native.lib.akv_context_decode_indices(
        _native.ptr(Registry), _native.ptr(Table), int(ROW_STRIDE),
        _native.ptr(Rows), _native.is64(Rows), _native.ptr(Lengths), _native.is64(Lengths),
        _native.ptr(Indptr), _native.is64(Indptr), _native.ptr(Output), _native.is64(Output),
        _native.ptr(starts), _native.is64(starts) if starts is not None else 0,
        _native.ptr(mapping), _native.is64(mapping) if mapping is not None else 0,
        int(MULTIPLIER), batch, _native.stream_of(Registry.device),
    )
    _native.check(status, "context_decode_indices")


def _window_lengths(batch, Registry, Rows, Lengths, Output, WINDOW):
    """context_page_table.py:7-31: visible sliding-window length per request."""
    if Registry.dtype != torch.int64:
        raise ValueError("context_window_lengths: int64 registry")
    status = _native.lib.akv_context_window_lengths(
        _native.ptr(Registry), _native.ptr(Rows), _native.is64(Rows), _native.ptr(Lengths),
        _native.is64(Lengths), _native.ptr(Output), _native.is64(Output), int(WINDOW), batch,
        _native.stream_of(Registry.device),
    )
    _native.check(status, "context_window_lengths")


context_decode_indices = _Launcher(_decode_indices, "context_decode_indices")
context_window_lengths = _Launcher(_window_lengths, "context_window_lengths")


def build_decode_metadata(registry, req_to_token, row_ids, seq_lens, kv_indptr, kv_indices, *,
                          window=None, mapping=None, multiplier=1, lengths_out=None,
                          starts_out=None):
    """Window lengths, kv_indptr, starts and kv_indices in two launches (C ABI
    ``akv_build_decode_metadata``), the fused form of
    ``ContextDecodeRegistry.fill_window`` / ``fill``
    (srt/layers/attention/context_backend.py:754-809).  ``row_ids`` and
    ``seq_lens`` are int64; ``kv_indptr`` / ``kv_indices`` int32."""
    batch = len(seq_lens)
    if window is not None and (lengths_out is None or starts_out is None):
        lengths_out = torch.empty(batch, dtype=torch.int64, device=seq_lens.device)
        starts_out = torch.empty(batch, dtype=torch.int64, device=seq_lens.device)
    for t, dt in ((row_ids, torch.int64), (seq_lens, torch.int64), (kv_indptr, torch.int32),
                  (kv_indices, torch.int32)):
        if t.dtype != dt:
            raise ValueError("build_decode_metadata: row_ids/seq_lens int64, indptr/indices int32")
    if mapping is not None and mapping.dtype != torch.int64:
        raise ValueError("build_decode_metadata: int64 mapping")
    status = _native.lib.akv_build_decode_metadata(
        _native.ptr(registry), _native.ptr(req_to_token), req_to_token.stride(0),
        _native.ptr(row_ids), _native.ptr(seq_lens), -1 if window is None else int(window),
        _native.ptr(mapping), int(multiplier), batch, _native.ptr(kv_indptr),
        _native.ptr(lengths_out), _native.ptr(starts_out), _native.ptr(kv_indices),
        _native.stream_of(seq_lens.device),
    )
    _native.check(status, "build_decode_metadata")
    return kv_indptr, lengths_out, starts_out
