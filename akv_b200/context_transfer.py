"""Active-slot gather for offload / load and PD transfer (C ABI
``akv_active_slots``).

The reference collects a request's surviving KV slots with two device index
operations and a concatenation
(srt/disaggregation/context_transfer.py:110-128): the prompt tokens the
decode view keeps (``row[device_indices[start:]]``, ``start`` from the
sliding window's first visible position) followed by the generated tokens
(``row[generated_start:raw_end]``).  ``request_active_slots`` keeps that
signature and host arithmetic and does the gather in one launch;
``request_active_lengths`` is the reference's host-only length rule
(:131-138).  Requests without a decode view fall back to building it from
the compiled layout, as the reference's ``ContextDecodeLayout.from_layout``
does (srt/context_system/occurrence.py:47-66).
"""

from __future__ import annotations

import numpy as np
import torch

from . import _native


def request_row(pool, index):
    """The request's slot row: an overflow row when the pool keeps one
    (srt/context_system/request_storage.py:240-244), else req_to_token[index]."""
    rows = getattr(pool, "_context_rows", None)
    if rows and index in rows:
        return rows[index]
    return pool.req_to_token[index]


def active_slots(row: torch.Tensor, device_indices: torch.Tensor, start: int,
                 generated_start: int, raw_end: int, *, n_indices: int | None = None,
                 out: torch.Tensor | None = None, error_flag: torch.Tensor | None = None):
    """``concat(row[device_indices[start:n_indices]], row[generated_start:raw_end])``
    as one int32 device tensor; no host synchronisation."""
    if row.dtype != torch.int32 or row.ndim != 1 or not row.is_cuda or row.stride(0) != 1:
        raise ValueError("row must be a contiguous int32 device vector")
    if device_indices.dtype != torch.int32 or device_indices.device != row.device or \
            not device_indices.is_contiguous():
        raise ValueError("device_indices must be contiguous int32 on the row's device")
    n_indices = len(device_indices) if n_indices is None else int(n_indices)
    start, generated_start, raw_end = int(start), int(generated_start), int(raw_end)
    if not 0 <= start <= n_indices <= len(device_indices) or generated_start < 0:
        raise ValueError("active slot ranges out of bounds")
    n_out = (n_indices - start) + max(0, raw_end - generated_start)
    if out is None:
        out = torch.empty(n_out, dtype=torch.int32, device=row.device)
    elif out.dtype != torch.int32 or out.device != row.device or out.numel() < n_out or \
            not out.is_contiguous():
        raise ValueError("out must be a contiguous int32 device vector of the result's length")
    status = _native.lib.akv_active_slots(
        _native.ptr(row), row.numel(), _native.ptr(device_indices), start, n_indices,
        generated_start, raw_end, _native.ptr(out), _native.ptr(error_flag),
        _native.stream_of(row.device))
    _native.check(status, "active_slots")
    return out[:n_out]


def _decode_view(req, device):
    view = req.context_decode_layout
    if view is not None:
        return view
    layout = req.context_program.layout
    raw = np.flatnonzero(layout.keep_mask.numpy()).astype(np.int32)
    positions = layout.positions.numpy()[raw].copy()
    if np.any(np.diff(positions.astype(np.int64)) <= 0):
        raise ValueError("Active decode positions must be strictly increasing")

    class _View:
        pass

    v = _View()
    v.raw_indices, v.positions = raw, positions
    v.device_indices = torch.from_numpy(raw).to(device)
    v.prompt_length, v.next_position = len(layout.positions), layout.next_position
    return v


def request_active_slots(req, pool, raw_end, *, window=None):
    """Drop-in for the reference's ``request_active_slots``: the request's
    active slots up to raw position ``raw_end`` (holes never reach a pool
    copy), optionally only those a sliding ``window`` can still read."""
    row = request_row(pool, req.kv.req_pool_idx)
    view = _decode_view(req, row.device)
    start = 0
    generated_start = view.prompt_length
    if window is not None:
        lower = view.next_position + raw_end - view.prompt_length - window
        start = int(np.searchsorted(view.positions, lower))
        generated_start += max(0, lower - view.next_position)
    indices = view.device_indices
    if indices.dtype != torch.int32:
        indices = indices.to(torch.int32)
    return active_slots(row, indices, start, generated_start, raw_end,
                        n_indices=len(view.raw_indices))


def request_active_lengths(req, raw_end, window):
    """(full active length, length a ``window`` still reads) from the host
    metadata alone, as the reference's ``request_active_lengths``."""
    view = req.context_decode_layout
    generated = max(0, raw_end - view.prompt_length)
    full = len(view.raw_indices) + generated
    lower = view.next_position + generated - window
    start = int(np.searchsorted(view.positions, lower))
    return full, len(view.raw_indices) - start + min(generated, window)


class ActiveSlotGather:
    """``active_slots`` for many requests in one launch (C ABI
    ``akv_active_slots_batch``).  ``plan`` validates the per-request ranges
    on the host and stages them (one host-to-device copy); ``run`` launches
    on the current stream and returns the packed int32 slots, request r's at
    ``offsets[r]:offsets[r + 1]``.  The rows and index vectors must stay
    alive while planned launches may run."""

    def __init__(self, device):
        device = torch.device(device)
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.device = device
        self.total = 0
        self.n = 0

    def plan(self, rows, device_indices, starts, generated_starts, raw_ends, n_indices=None):
        n = len(rows)
        if not (len(device_indices) == len(starts) == len(generated_starts) == len(raw_ends) == n):
            raise ValueError("one row, index vector and range per request")
        if n_indices is None:
            n_indices = [len(x) for x in device_indices]
        meta = np.zeros((max(n, 1), 6), np.int64)
        offsets = np.zeros(n + 1, np.int64)
        for r in range(n):
            row, idx = rows[r], device_indices[r]
            if row.dtype != torch.int32 or row.ndim != 1 or row.device != self.device or \
                    row.stride(0) != 1:
                raise ValueError("rows must be contiguous int32 vectors on the device")
            if idx.dtype != torch.int32 or idx.device != self.device or not idx.is_contiguous():
                raise ValueError("device_indices must be contiguous int32 on the device")
            s, g, e, k = int(starts[r]), int(generated_starts[r]), int(raw_ends[r]), \
                int(n_indices[r])
            if not 0 <= s <= k <= len(idx) or g < 0:
                raise ValueError("active slot ranges out of bounds")
            meta[r] = (row.data_ptr(), row.numel(), idx.data_ptr(), s, k - s, g)
            offsets[r + 1] = offsets[r] + (k - s) + max(0, e - g)
        self._keep = (list(rows), list(device_indices))
        # One block per CHUNK outputs of a request: {request, first output}.
        chunk = int(_native.lib.akv_active_slots_chunk())
        lengths = np.diff(offsets)
        counts = (lengths + chunk - 1) // chunk
        req = np.repeat(np.arange(n, dtype=np.int64), counts)
        first = (np.arange(len(req)) - np.repeat(np.cumsum(counts) - counts, counts)) * chunk
        blocks = np.stack((req, first), 1).astype(np.int64)
        staged = torch.from_numpy(np.concatenate(
            (meta.reshape(-1), offsets, blocks.astype(np.int32).view(np.int64).reshape(-1)
             if len(blocks) else np.zeros(0, np.int64)))).pin_memory()
        dev = staged.to(self.device, non_blocking=True)
        self.meta = dev[: meta.size]
        self.offsets_dev = dev[meta.size: meta.size + n + 1]
        self.chunks = dev[meta.size + n + 1:]
        self.n_chunks = len(blocks)
        self._staged = staged  # the pinned source must outlive the copy
        self.offsets = offsets
        self.n, self.total = n, int(offsets[-1])
        return self

    def run(self, out=None, error_flag=None):
        if out is None:
            out = torch.empty(self.total, dtype=torch.int32, device=self.device)
        elif out.dtype != torch.int32 or out.device != self.device or out.numel() < self.total \
                or not out.is_contiguous():
            raise ValueError("out must be a contiguous int32 device vector of the packed length")
        status = _native.lib.akv_active_slots_batch(
            _native.ptr(self.meta), _native.ptr(self.offsets_dev), _native.ptr(self.chunks),
            self.n_chunks, _native.ptr(out), _native.ptr(error_flag),
            _native.stream_of(self.device))
        _native.check(status, "active_slots_batch")
        return out[: self.total]
