"""Drop-in ``write_row_slots`` with the reference's launch syntax.

Replaces the Triton kernel of
akv/system/sglang/kernels/ops/memory/context_rows.py:7-15, which scatters
slot ids into request-owned overflow rows: for i < N,
``((int32*)Pointers[Rows[i]])[Columns[i]] = Values[i]``.  Called as
``write_row_slots[(1,)](Pointers, Rows, Columns, Values, N=n, BLOCK=b)``.
"""

from __future__ import annotations

from . import _native
from .context_page_table import _Launcher


def _write_row_slots(batch, Pointers, Rows, Columns, Values, N, BLOCK=None):
    del batch, BLOCK  # the reference runs one program; the native kernel tiles N itself
    status = _native.lib.akv_write_row_slots(
        _native.ptr(Pointers), _native.ptr(Rows), _native.is64(Rows), _native.ptr(Columns),
        _native.is64(Columns), _native.ptr(Values), _native.is64(Values), int(N),
        _native.stream_of(Pointers.device),
    )
    _native.check(status, "write_row_slots")


write_row_slots = _Launcher(_write_row_slots, "write_row_slots")
