"""Drop + Reposition of a batch of requests on the GPU (C ABI ``akv_drop_compact``).

The reference compiles every request's event program on the CPU
(``compile_context_layout``, srt/context_system/ir.py:113-274, running the
C++ sweep of kernels/ops/attention/context_plan.py:210-532), derives the
decode view on the CPU (``ContextDecodeLayout.from_layout``,
srt/context_system/occurrence.py:47-66), copies it to the device, and
retires dropped slots through the scheduler (occurrence.py:711-714,
936-964).  For the cache operation of an agent turn -- drop a set of spans,
then Reposition at the end of the prompt -- ``DropCompactor`` computes all
of it on the device in three stream-ordered launches:

* keep mask and final positions of every token,
* the compacted decode view (raw indices and positions of the kept tokens),
* the Reposition transitions (source slot, destination slot, old and new
  position), where a radix-shared source is copied to a fresh slot popped
  from the device free ring (copy-on-write) and the request's
  req_to_token entry is updated, while private sources rotate in place,
* the freed slots of dropped private tokens, pushed onto the free ring.

The transition vectors feed ``reposition_kv_layers`` directly, with the
device-side count, so a whole Drop + Reposition runs without a host round
trip.  Host input is the event program (token counts and drop ranges per
request), validated on the CPU with the reference's rules before one packed
host-to-device copy.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from . import _native

TILE = int(_native.lib.akv_drop_compact_tile_tokens())


class FreeSlotRing:
    """Device-resident free list of KV slots.

    ``ring`` holds slot ids; ``state`` = {head, tail} (int64, device).  Free
    entries are ring[head % capacity .. tail % capacity).  Copy-on-write pops
    from the head, freed slots are pushed at the tail, both on the device.
    """

    def __init__(self, free_slots, capacity=None, device=None):
        free = torch.as_tensor(free_slots, dtype=torch.int32)
        device = torch.device(device) if device is not None else free.device
        capacity = int(capacity if capacity is not None else max(1, len(free)))
        if len(free) > capacity:
            raise ValueError("free slots exceed the ring capacity")
        self.capacity = capacity
        self.ring = torch.zeros(capacity, dtype=torch.int32, device=device)
        self.ring[: len(free)] = free.to(device)
        self.state = torch.tensor([0, len(free)], dtype=torch.int64, device=device)

    def free_count(self) -> int:
        """Number of free slots (reads the device state: synchronises)."""
        head, tail = self.state.tolist()
        return tail - head

    def snapshot(self) -> np.ndarray:
        """Free slot ids in ring order (reads the device: synchronises)."""
        head, tail = self.state.tolist()
        idx = torch.arange(head, tail, device=self.ring.device) % self.capacity
        return self.ring[idx].cpu().numpy()


@dataclass
class DropResult:
    """Device views of one call.  Counts live on the device in ``totals``
    ({kept, moved, copy-on-write, freed}); the compacted vectors are valid
    up to those counts and the per-request CSR offsets."""

    keep_mask: torch.Tensor
    positions: torch.Tensor
    active_offsets: torch.Tensor
    raw_indices: torch.Tensor
    active_positions: torch.Tensor
    next_position: torch.Tensor
    transition_offsets: torch.Tensor
    transition_source: torch.Tensor
    transition_destination: torch.Tensor
    transition_pairs: torch.Tensor
    transition_raw: torch.Tensor
    freed_offsets: torch.Tensor
    freed_slots: torch.Tensor
    totals: torch.Tensor
    status: torch.Tensor
    kept_host: int | None = None  # kept tokens, when the host knows them

    @property
    def transition_count(self) -> torch.Tensor:
        """One-element int32 device view: ``count_device`` for reposition."""
        return self.totals[1:2]

    def read_view(self, out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """Copy the decode view to host memory in one library call
        (``akv_drop_read_view``), stream-ordered after the call: one int32
        vector ``[raw_indices(kept) | active_positions(kept) |
        active_offsets(n + 1) | next_position(n) | totals(4) | status]`` for
        n requests, into ``out`` (pinned, for an asynchronous copy) or a new
        pinned tensor.  ``kept`` is the host's count for a validated program
        (``kept_host``), else every token of the call (entries past
        ``totals[0]`` are then unused).  ``stream``: a torch stream (default:
        the current one); record an event on it and wait before reading
        ``out``."""
        n = len(self.next_position)
        kept = self.kept_host if self.kept_host is not None else len(self.keep_mask)
        size = 2 * kept + 2 * n + 6
        if out is None:
            out = torch.empty(size, dtype=torch.int32, pin_memory=True)
        elif out.dtype != torch.int32 or out.device.type != "cpu" or out.numel() < size or \
                not out.is_contiguous():
            raise ValueError(f"out must be a contiguous host int32 tensor of {size} elements")
        handle = _native.stream_of(self.totals.device) if stream is None else \
            ctypes.c_void_p(stream.cuda_stream)
        status = _native.lib.akv_drop_read_view(
            out.data_ptr(), _native.ptr(self.raw_indices), _native.ptr(self.active_positions),
            kept, _native.ptr(self.active_offsets), _native.ptr(self.next_position), n,
            _native.ptr(self.totals), handle)
        _native.check(status, "drop_read_view")
        return out

    def check(self) -> None:
        """Read the device status (synchronises) and raise on failure."""
        st = int(self.status.item())
        if st == 0:
            return
        msgs = []
        if st & _native.DROP_RING_UNDERFLOW:
            msgs.append("not enough free KV slots for copy-on-write")
        if st & _native.DROP_RING_OVERFLOW:
            msgs.append("freed slots exceed the free ring capacity")
        if st & _native.DROP_BAD_RANGE:
            msgs.append("a drop range lies outside its request")
        if st & _native.DROP_NO_ACTIVE:
            msgs.append("Reposition of a request with no active tokens")
        if st & _native.DROP_BAD_PAGE:
            msgs.append("a req_to_token row breaks the page layout (a token's slot offset "
                        "differs from its offset in the page, or one page holds two pages' "
                        "tokens)")
        raise RuntimeError("drop_compact failed: " + "; ".join(msgs))


def validate_program(token_counts, range_offsets, ranges, reposition=True):
    """The reference compiler's rules for one drop event at the end of each
    prompt (context_plan.py:362-411): ranges are half-open, ordered,
    disjoint and inside the prompt; a Reposition needs an active token.
    Checked for every request at once; the error is the one the reference
    raises for the first request (in order) that breaks a rule."""
    token_counts = np.asarray(token_counts, np.int64)
    range_offsets = np.asarray(range_offsets, np.int64)
    ranges = np.asarray(ranges, np.int64).reshape(-1, 2)
    n = len(token_counts)
    if len(range_offsets) != n + 1 or range_offsets[0] != 0 or \
            range_offsets[-1] != len(ranges):
        raise ValueError("drop_range_offsets does not cover drop_ranges")
    per_request = range_offsets[1:] - range_offsets[:-1]
    if (per_request < 0).any():
        raise ValueError("drop_range_offsets does not cover drop_ranges")
    if n and (token_counts.min() < 0 or token_counts.max() > np.iinfo(np.int32).max):
        raise ValueError("token_count exceeds the int32 Reposition limit")
    if not len(ranges):
        return
    starts, ends = ranges[:, 0], ranges[:, 1]
    if n == 1 and len(ranges) <= 256:  # one request, few ranges: a plain walk is cheapest
        t, previous_end, dropped = int(token_counts[0]), -1, 0
        for start, end in ranges.tolist():
            if start < 0 or start >= end or end > t or start <= previous_end:
                raise ValueError("Drop ranges must be ordered, disjoint, and already materialized")
            previous_end, dropped = end, dropped + end - start
        if reposition and t > 0 and dropped == t:
            raise ValueError(f"Reposition at raw boundary {t - 1} has no active tokens.")
        return
    owner = np.repeat(np.arange(n), per_request)  # request of each range
    bad = (starts < 0) | (starts >= ends) | (ends > token_counts[owner])
    # a range that is not its request's first starts after the previous end
    bad[1:] |= (owner[1:] == owner[:-1]) & (starts[1:] <= ends[:-1])
    bad_request = np.bincount(owner, weights=bad, minlength=n) > 0
    dropped = np.bincount(owner, weights=ends - starts, minlength=n)
    no_active = (per_request > 0) & (token_counts > 0) & (dropped == token_counts) if reposition \
        else np.zeros(n, bool)
    failed = bad_request | no_active
    if failed.any():
        r = int(np.argmax(failed))
        if bad_request[r]:
            raise ValueError("Drop ranges must be ordered, disjoint, and already materialized")
        raise ValueError(f"Reposition at raw boundary {int(token_counts[r]) - 1} has no active tokens.")


class DropCompactor:
    """Preallocated device buffers and pinned staging for ``akv_drop_compact``.

    Capacities bound one call: total tokens, requests and ranges.  Outputs
    are views into the buffers and are overwritten by the next call.
    """

    def __init__(self, max_tokens, max_requests, max_ranges, device):
        device = torch.device(device)
        if device.type == "cuda" and device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.device = device
        self.max_tokens = int(max_tokens)
        self.max_requests = int(max_requests)
        self.max_ranges = int(max_ranges)
        max_tiles = (self.max_tokens + TILE - 1) // TILE + self.max_requests
        self.max_tiles = max_tiles
        d, i32 = self.device, torch.int32
        n, r = max(1, self.max_tokens), self.max_requests
        self.keep_mask = torch.empty(n, dtype=torch.uint8, device=d)
        self.positions = torch.empty(n, dtype=i32, device=d)
        self.raw_indices = torch.empty(n, dtype=i32, device=d)
        self.active_positions = torch.empty(n, dtype=i32, device=d)
        self.transition_source = torch.empty(n, dtype=i32, device=d)
        self.transition_destination = torch.empty(n, dtype=i32, device=d)
        self.transition_pairs = torch.empty((n, 2), dtype=i32, device=d)
        self.transition_raw = torch.empty(n, dtype=i32, device=d)
        self.freed_slots = torch.empty(n, dtype=i32, device=d)
        # per-request outputs + counters in one buffer
        self.offsets = torch.empty((3, r + 1), dtype=i32, device=d)
        self.next_position = torch.empty(max(1, r), dtype=i32, device=d)
        self.counters = torch.empty(5, dtype=i32, device=d)  # totals[4], status
        ws = int(_native.lib.akv_drop_compact_workspace_bytes(r, max_tiles))
        self.workspace = torch.empty(ws + 256, dtype=torch.uint8, device=d)
        # Packed program: token_offsets (int64) | row_ids (int64) |
        # tile_offsets | range_offsets | shared_prefix | ranges (int32).
        self._host = torch.empty(self._packed_bytes(), dtype=torch.uint8, pin_memory=True)
        self._host_np = self._host.numpy()
        self._dev = torch.empty_like(self._host, device=d)
        self._prepared = {}
        # The pinned staging buffer is rewritten by the next call only after
        # the previous host-to-device copy has left it.
        self._copied = torch.cuda.Event()
        self._copied.record(torch.cuda.current_stream(d))

    def _packed_bytes(self):
        r, rr = self.max_requests, self.max_ranges
        return 8 * (r + 1) + 8 * r + 4 * ((r + 1) * 2 + r + 2 * rr) + 64

    def _layout(self, nreq, nranges):
        off, views = 0, {}
        for name, count, dtype, size in (
            ("token_offsets", nreq + 1, torch.int64, 8),
            ("row_ids", nreq, torch.int64, 8),
            ("tile_offsets", nreq + 1, torch.int32, 4),
            ("range_offsets", nreq + 1, torch.int32, 4),
            ("shared_prefix", nreq, torch.int32, 4),
            ("ranges", 2 * nranges, torch.int32, 4),
        ):
            off = (off + 7) // 8 * 8
            views[name] = (off, count, dtype)
            off += count * size
        return views, off

    def run(self, token_counts, range_offsets, ranges, req_to_token, row_ids, ring,
            shared_prefix=None, reposition=True, validate=True, page_size=1) -> DropResult:
        """Validate and stage the program (one packed host-to-device copy),
        then launch: ``prepare`` followed by ``launch``."""
        prepared = self.prepare(token_counts, range_offsets, ranges, row_ids,
                                shared_prefix=shared_prefix, reposition=reposition,
                                validate=validate, page_size=page_size)
        return self.launch(prepared, req_to_token, ring)

    def prepare(self, token_counts, range_offsets, ranges, row_ids, shared_prefix=None,
                reposition=True, validate=True, page_size=1) -> dict:
        """Host half: validation, packing and the host-to-device copy.  The
        returned handle can be launched any number of times while the
        staged program stays resident on the device, i.e. until the next
        ``prepare`` or ``run`` of this compactor (which restages; a program
        of the same shape gets the same handle back).

        ``page_size`` > 1 (a power of two from 4 to 128) runs the paged form
        (``akv_drop_compact_paged``): the ring holds page ids, a private
        page is freed once all its tokens are dropped, and a radix-shared
        page holding a moved token is copied whole to a fresh page.  The
        rows must keep each token at offset ``token % page_size`` of its
        page, and every shared prefix must be a whole number of pages."""
        page_size = int(page_size)
        if page_size != 1 and (page_size < 4 or page_size > 128 or page_size & (page_size - 1)):
            raise ValueError("page_size must be 1 or a power of two from 4 to 128")
        if page_size != 1 and shared_prefix is not None and \
                np.any(np.asarray(shared_prefix, np.int64) % page_size):
            raise ValueError("a radix-shared prefix must be a whole number of pages")
        token_counts = np.asarray(token_counts, np.int64)
        nreq = len(token_counts)
        range_offsets = np.asarray(range_offsets, np.int64)
        ranges = np.asarray(ranges, np.int64)
        nranges = len(ranges) // 2
        total = int(token_counts.sum())
        if nreq > self.max_requests or nranges > self.max_ranges or total > self.max_tokens:
            raise ValueError("drop program exceeds the compactor's capacity")
        if validate:
            validate_program(token_counts, range_offsets, ranges, reposition)
        row_ids = np.asarray(row_ids, np.int64)
        if row_ids.shape != (nreq,) or (shared_prefix is not None and
                                        np.shape(shared_prefix) != (nreq,)):
            raise ValueError("row_ids and shared_prefix must hold one entry per request")
        if nreq == 1:  # a single request: plain integers are cheaper than numpy
            n_tiles = -(-total // TILE)
            tile_offsets = (0, n_tiles)
        else:
            tiles = (token_counts + TILE - 1) // TILE
            tile_offsets = np.concatenate(([0], np.cumsum(tiles)))
            n_tiles = int(tile_offsets[-1])
        shared = shared_prefix is not None
        # One handle per layout and size: its device views (fixed offsets of
        # the staging buffer) and its cached launch arguments are reused by
        # every call with the same shape; the staged contents are rewritten.
        key = (nreq, nranges, n_tiles, total, shared, bool(reposition), page_size)
        prepared = self._prepared.get(key)
        if prepared is None:
            views, used = self._layout(nreq, nranges)
            dev = {name: self._dev[off: off + count * (8 if dt == torch.int64 else 4)].view(dt)
                   for name, (off, count, dt) in views.items()}
            host_views = {name: self._host_np[off: off + count * (8 if dt == torch.int64 else 4)]
                          .view(np.int64 if dt == torch.int64 else np.int32)
                          for name, (off, count, dt) in views.items()}
            prepared = dict(dev=dev, nreq=nreq, n_tiles=n_tiles, total=total, shared=shared,
                            reposition=bool(reposition), page_size=page_size, h2d_bytes=used,
                            _host_views=host_views, _src=self._host[:used],
                            _dst=self._dev[:used])
            if len(self._prepared) > 64:
                self._prepared.clear()
            self._prepared[key] = prepared
        # Kept tokens: known on the host once the ranges are validated
        # (half-open, disjoint).
        prepared["kept"] = total - int((ranges[1::2] - ranges[0::2]).sum()) if validate else None
        self._copied.synchronize()
        hv = prepared["_host_views"]
        offsets = hv["token_offsets"]
        offsets[0] = 0
        np.cumsum(token_counts, out=offsets[1:])
        hv["row_ids"][:] = row_ids
        hv["tile_offsets"][:] = tile_offsets
        hv["range_offsets"][:] = range_offsets
        hv["shared_prefix"][:] = 0 if shared_prefix is None else shared_prefix
        hv["ranges"][:] = ranges
        prepared["_dst"].copy_(prepared["_src"], non_blocking=True)
        self._copied.record(torch.cuda.current_stream(self.device))
        return prepared

    def launch(self, prepared, req_to_token, ring) -> DropResult:
        """Device half: the three kernels of ``akv_drop_compact`` over a
        staged program; no host work beyond the launch."""
        # Relaunching the same staged program against the same rows and ring
        # reuses the argument list and the result views (host cost of one
        # ctypes call).
        key = (id(self), req_to_token.data_ptr(), tuple(req_to_token.shape), req_to_token.stride(0),
               req_to_token.dtype, req_to_token.device, ring.ring.data_ptr(), ring.capacity,
               ring.state.data_ptr())
        cached = prepared.get("_launch")
        if cached is None or cached[0] != key:
            cached = (key,) + self._launch_args(prepared, req_to_token, ring)
            prepared["_launch"] = cached
        _, args, result = cached
        result.kept_host = prepared.get("kept")
        page_size = prepared.get("page_size", 1)
        if page_size == 1:
            status = _native.lib.akv_drop_compact(*args, _native.stream_of(self.device))
        else:
            status = _native.lib.akv_drop_compact_paged(*args[:11], page_size, *args[11:],
                                                        _native.stream_of(self.device))
        _native.check(status, "drop_compact")
        return result

    def _launch_args(self, prepared, req_to_token, ring):
        if req_to_token.dtype != torch.int32 or req_to_token.device != self.device or \
                req_to_token.ndim != 2 or req_to_token.stride(1) != 1:
            raise ValueError("req_to_token must be a row-major int32 tensor on the device")
        dev, nreq, n_tiles, total = (prepared["dev"], prepared["nreq"], prepared["n_tiles"],
                                     prepared["total"])
        ws = self.workspace
        ws_aligned = ws[(-ws.data_ptr()) % 256:]
        off3 = self.offsets
        args = (
            nreq, _native.ptr(dev["token_offsets"]), _native.ptr(dev["tile_offsets"]), n_tiles,
            _native.ptr(dev["range_offsets"]), _native.ptr(dev["ranges"]),
            _native.ptr(dev["shared_prefix"]) if prepared["shared"] else None,
            _native.ptr(req_to_token), _native.ptr(dev["row_ids"]), req_to_token.stride(0),
            int(prepared["reposition"]), _native.ptr(ring.ring), ring.capacity,
            _native.ptr(ring.state), _native.ptr(self.keep_mask), _native.ptr(self.positions),
            _native.ptr(off3[0]), _native.ptr(self.raw_indices),
            _native.ptr(self.active_positions), _native.ptr(self.next_position),
            _native.ptr(off3[1]), _native.ptr(self.transition_source),
            _native.ptr(self.transition_destination), _native.ptr(self.transition_pairs),
            _native.ptr(self.transition_raw), _native.ptr(off3[2]), _native.ptr(self.freed_slots),
            _native.ptr(self.counters[:4]), _native.ptr(self.counters[4:]),
            _native.ptr(ws_aligned),
        )
        return args, DropResult(
            keep_mask=self.keep_mask[:total], positions=self.positions[:total],
            active_offsets=off3[0, : nreq + 1], raw_indices=self.raw_indices,
            active_positions=self.active_positions, next_position=self.next_position[:nreq],
            transition_offsets=off3[1, : nreq + 1], transition_source=self.transition_source,
            transition_destination=self.transition_destination,
            transition_pairs=self.transition_pairs, transition_raw=self.transition_raw,
            freed_offsets=off3[2, : nreq + 1], freed_slots=self.freed_slots,
            totals=self.counters[:4], status=self.counters[4:5],
        )


def launch_static(compactor, prepared, req_to_token, ring) -> DropResult:
    """``DropCompactor.launch`` through ``akv_drop_compact_static``: same
    kernels and outputs, but the scratch lives in the library's own device
    array instead of ``compactor.workspace`` -- the entry point for callers
    that cannot allocate device memory for a workspace.  At most
    ``akv_drop_compact_static_max_requests()`` requests and
    ``akv_drop_compact_static_max_tiles()`` tiles per call; calls whose
    kernels overlap on the GPU share the array and must be serialised."""
    c = compactor
    if req_to_token.dtype != torch.int32 or req_to_token.device != c.device or \
            req_to_token.ndim != 2 or req_to_token.stride(1) != 1:
        raise ValueError("req_to_token must be a row-major int32 tensor on the device")
    dev, nreq, n_tiles, total = (prepared["dev"], prepared["nreq"], prepared["n_tiles"],
                                 prepared["total"])
    off3 = c.offsets
    status = _native.lib.akv_drop_compact_static(
        nreq, _native.ptr(dev["token_offsets"]), _native.ptr(dev["tile_offsets"]), n_tiles,
        _native.ptr(dev["range_offsets"]), _native.ptr(dev["ranges"]),
        _native.ptr(dev["shared_prefix"]) if prepared["shared"] else None,
        _native.ptr(req_to_token), _native.ptr(dev["row_ids"]), req_to_token.stride(0),
        int(prepared["reposition"]), _native.ptr(ring.ring), ring.capacity,
        _native.ptr(ring.state), _native.ptr(c.keep_mask), _native.ptr(c.positions),
        _native.ptr(off3[0]), _native.ptr(c.raw_indices), _native.ptr(c.active_positions),
        _native.ptr(c.next_position), _native.ptr(off3[1]), _native.ptr(c.transition_source),
        _native.ptr(c.transition_destination), _native.ptr(c.transition_pairs),
        _native.ptr(c.transition_raw), _native.ptr(off3[2]), _native.ptr(c.freed_slots),
        _native.ptr(c.counters[:4]), _native.ptr(c.counters[4:]), _native.stream_of(c.device),
    )
    if status == _native.AKV_ERR_INVALID:
        raise ValueError(
            "drop_compact_static: the program exceeds the static scratch "
            f"({int(_native.lib.akv_drop_compact_static_max_requests())} requests, "
            f"{int(_native.lib.akv_drop_compact_static_max_tiles())} tiles of {TILE} tokens)")
    _native.check(status, "drop_compact_static")
    return DropResult(
        keep_mask=c.keep_mask[:total], positions=c.positions[:total],
        active_offsets=off3[0, : nreq + 1], raw_indices=c.raw_indices,
        active_positions=c.active_positions, next_position=c.next_position[:nreq],
        transition_offsets=off3[1, : nreq + 1], transition_source=c.transition_source,
        transition_destination=c.transition_destination,
        transition_pairs=c.transition_pairs, transition_raw=c.transition_raw,
        freed_offsets=off3[2, : nreq + 1], freed_slots=c.freed_slots,
        totals=c.counters[:4], status=c.counters[4:5], kept_host=prepared.get("kept"),
    )


def drop_compact(token_counts, range_offsets, ranges, req_to_token, row_ids, ring,
                 shared_prefix=None, reposition=True, page_size=1) -> DropResult:
    """One-shot ``DropCompactor`` sized to this program."""
    token_counts = np.asarray(token_counts, np.int64)
    comp = DropCompactor(int(token_counts.sum()), len(token_counts),
                         max(1, len(np.asarray(ranges)) // 2), req_to_token.device)
    return comp.run(token_counts, range_offsets, ranges, req_to_token, row_ids, ring,
                    shared_prefix=shared_prefix, reposition=reposition, page_size=page_size)
