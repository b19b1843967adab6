"""Occurrence slot binding on the device (C ABI ``akv_gather_slots``).

Between prefill forwards the reference keeps request-local page ownership
on the scheduler CPU (srt/context_system/occurrence.py): ``plan`` picks the
occurrences that need a page, ``advance`` binds the forward's query and
extra pages to them and retires what no later query reads, and
``terminal_slots`` publishes the final-position page table.  Every index is
prepared on the CPU on purpose (no device sync, no ``nonzero`` on the
scheduler path); the device part is a chain of small torch operations per
request -- one concatenation of the state's slots with the new ones, one
gather per output field, int32 casts -- and the scheduler concatenates the
per-request results (akv/system/sglang.patch:3133-3180).

This module keeps the reference's checks and messages in Python, derives
every ownership index natively on the host (``akv_occurrence_advance_indices``,
passes over the arrays described in csrc/occurrence_plan.cu) and does the
device part of a whole forward in ONE host-to-device copy (int32 indices)
and ONE launch:

* ``advance`` is a drop-in for ``OccurrenceState.advance`` (:644-755);
* ``terminal_slots`` for ``OccurrenceState.terminal_slots`` (:757-768);
* ``bind`` for ``OccurrenceMaterialization.bind`` (:315-357);
* ``OccurrenceBatch`` binds every request of a forward (context requests
  through ``advance``, ordinary ones as ``cat(prefix_indices, birth)``)
  and returns the concatenated slots, copy sources, copy destinations and
  copy position pairs the scheduler hands to the prefill.

``SlotGather`` is the launch builder underneath: each task is one output
vector gathered from the virtual concatenation of up to four slot vectors.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

import ctypes
import itertools

from . import _native

_MAX_SEGMENTS = 4
_TASK_WORDS = 12  # first index, outputs, output address, flags, 4 segment addresses, 4 ends
_CHUNK = int(_native.lib.akv_gather_slots_chunk())  # outputs per block of the gather kernel
_P, _I64 = ctypes.c_void_p, ctypes.c_int64


class _AdvanceIn(ctypes.Structure):
    """struct akv_advance_in of include/akv_b200.h, field for field."""

    _fields_ = [("n", _I64), ("start", _I64), ("end", _I64), ("count", _I64), ("n_old", _I64),
                ("n_query", _I64), ("n_extra", _I64), ("n_copy", _I64), ("owned", _P),
                ("canonical_rows", _P), ("terminal_rows", _P), ("canonical_positions", _P),
                ("swa_resident", _P), ("birth_occurrences", _P), ("terminal_occurrences", _P),
                ("occurrence_positions", _P), ("source_rows", _P), ("allocated", _P),
                ("copy_occurrences", _P), ("copy_source_rows", _P), ("plan_terminal", _P),
                ("visible_until", _P)]


class _AdvanceOut(ctypes.Structure):
    """struct akv_advance_out of include/akv_b200.h, field for field."""

    _fields_ = [("occurrence_rows", _P), ("copy_source_rows", _P),
                ("copy_destination_rows", _P), ("retained", _P), ("retired", _P),
                ("unused_swa", _P), ("next_canonical", _P), ("next_terminal", _P),
                ("next_positions", _P), ("next_owned", _P), ("next_swa", _P),
                ("retired_swa", _P), ("n_retained", _I64), ("n_retired", _I64),
                ("n_unused_swa", _I64)]


def _host(t, dtype):
    """A CPU tensor or array as a contiguous numpy array of ``dtype``."""
    a = t.numpy() if isinstance(t, torch.Tensor) else np.asarray(t)
    return np.ascontiguousarray(a, dtype=dtype)


def _addr(a):
    return a.ctypes.data if a.size else None


class SlotGather:
    """Tasks of one ``akv_gather_slots`` launch.

    ``add`` queues one output; ``launch`` packs the task table, the chunk
    table and every index into one pinned buffer, copies it to the device
    once and launches once on the current stream.  The output tensors and
    segment vectors must stay alive until the launch has run (the caller's
    tensors, as with any stream-ordered torch operation)."""

    def __init__(self, device):
        self.device = torch.device(device)
        if self.device.type == "cuda" and self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        # what Tensor.get_device() returns for a tensor on this device
        self._index = self.device.index if self.device.type == "cuda" else -1
        self._reset()

    def _reset(self):
        self._tasks = []      # (out, indices, segments, literal): kept alive until the launch
        self._idx = []        # index vector of each task
        self._meta = []       # (outputs, output address, flags, segment set) per task
        self._sized = None    # the three arrays of _sizes, until the next task
        self._seg_ids = {}    # segment-set key -> row of _seg_table
        self._seg_objs = []   # the segment tuples, by id
        self._seg_table = []  # per segment set: 4 base addresses, 4 cumulative ends
        self._seg_flags = []

    def _segment_set(self, segments, literal=False, m=0):
        """Id of a tuple of segments (checked and registered on first use)."""
        # A tuple is keyed by its identity (registered here, so it stays
        # alive and its id unique); anything else by its tensors' identities.
        key = id(segments) if type(segments) is tuple else tuple(map(id, segments))
        sid = self._seg_ids.get(key)
        if sid is not None:
            if m and not literal and not self._seg_flags[sid] >> 8:
                raise ValueError("a slot gather reads one to four segments")
            return sid
        segments = tuple(segments)
        if len(segments) > _MAX_SEGMENTS or (not literal and not segments and m):
            raise ValueError("a slot gather reads one to four segments")
        for s in segments:
            if s.ndim != 1 or s.dtype != segments[0].dtype or s.dtype not in (
                    torch.int32, torch.int64) or s.get_device() != self._index or \
                    not s.is_contiguous():
                raise ValueError("gather segments must be contiguous int32/int64 vectors "
                                 "of one dtype on the device")
        ptrs, ends, end = [0] * _MAX_SEGMENTS, [0] * _MAX_SEGMENTS, 0
        for i, seg in enumerate(segments):
            size = seg.numel()
            end += size
            ptrs[i] = seg.data_ptr() if size else 0
            ends[i] = end
        flags = len(segments) << 8
        if segments and segments[0].dtype == torch.int64:
            flags |= _native.GATHER_SEG64
        sid = len(self._seg_table)
        self._seg_table.append(ptrs + ends)
        self._seg_flags.append(flags)
        self._seg_objs.append(segments)
        self._seg_ids[key] = sid
        return sid

    def add(self, out: torch.Tensor, indices, segments=(), *, literal: bool = False):
        """out[i] = concat(segments)[indices[i]] (-1 where the index is
        negative), or indices[i] itself with ``literal``; out is int32 or
        int64 (int64 values are cast to int32 as torch does)."""
        idx = np.asarray(indices).reshape(-1)
        if out.dtype not in (torch.int32, torch.int64) or out.get_device() != self._index or \
                not out.is_contiguous() or out.numel() != len(idx):
            raise ValueError("gather output must be a contiguous int32/int64 vector on the "
                             "device with one element per index")
        if idx.dtype.kind not in "iu" and len(idx):
            raise ValueError("gather indices must be integers")
        if len(idx) and (int(idx.min()) < -2**31 or int(idx.max()) > 2**31 - 1):
            raise ValueError("gather indices and literals must fit in int32")
        self._add(out, idx, segments, literal)

    def _add(self, out, idx, segments=(), literal=False):
        """``add`` for an output this module allocated (contiguous, on the
        device, one element per index): the segments are still checked."""
        if type(idx) is not np.ndarray or idx.ndim != 1:
            idx = np.asarray(idx).reshape(-1)
        m = idx.shape[0]
        sid = self._segment_set(segments, literal, m)
        if m > 2**31 - 1:
            raise ValueError("a slot gather task holds at most 2^31 - 1 outputs")
        flags = self._seg_flags[sid] | (_native.GATHER_OUT64 if out.dtype == torch.int64 else 0) \
            | (_native.GATHER_LITERAL if literal else 0)
        self._meta.append((m, out.data_ptr() if m else 0, flags, sid))
        self._idx.append(idx)
        self._tasks.append((out, idx, self._seg_objs[sid], literal))
        self._sized = None

    def _add_fields(self, fields, segments):
        """``_add`` for several outputs gathered from one segment set (the
        fields of one request): one lookup of the set, then one task per
        (out, indices) pair."""
        fields = [(out, idx if type(idx) is np.ndarray and idx.ndim == 1
                   else np.asarray(idx).reshape(-1)) for out, idx in fields]
        m_max = max((idx.shape[0] for _, idx in fields), default=0)
        sid = self._segment_set(segments, False, m_max)
        if m_max > 2**31 - 1:
            raise ValueError("a slot gather task holds at most 2^31 - 1 outputs")
        flags, seg_obj = self._seg_flags[sid], self._seg_objs[sid]
        out64 = _native.GATHER_OUT64
        meta, idxs, tasks = self._meta, self._idx, self._tasks
        for out, idx in fields:
            m = idx.shape[0]
            meta.append((m, out.data_ptr() if m else 0,
                         flags | (out64 if out.dtype == torch.int64 else 0), sid))
            idxs.append(idx)
            tasks.append((out, idx, seg_obj, False))
        self._sized = None

    def __len__(self):
        return len(self._tasks)

    def _sizes(self):
        if self._sized is None:
            meta = np.fromiter(itertools.chain.from_iterable(self._meta), np.int64,
                               4 * len(self._meta)).reshape(-1, 4)
            lengths = meta[:, 0]
            self._sized = (meta, lengths, (lengths + _CHUNK - 1) // _CHUNK)
        return self._sized

    def words(self):
        """Length of the packed program in int64 words (indices are int32,
        two to a word)."""
        _, lengths, counts = self._sizes()
        return _TASK_WORDS * len(self._tasks) + int(counts.sum()) + (int(lengths.sum()) + 1) // 2

    def pack(self, out: np.ndarray | None = None):
        """(words, n_tasks, n_chunks): the int64 task table, the chunk table
        (one word per chunk: the int32 pair {task, first output}) and the
        int32 indices, in that order; written into ``out`` when given."""
        meta, lengths, counts = self._sizes()
        n, n_chunks = len(self._tasks), int(counts.sum())
        if n_chunks > 2**31 - 1:
            raise ValueError("too many slot gather chunks for one launch")
        n_idx = int(lengths.sum())
        total = _TASK_WORDS * n + n_chunks + (n_idx + 1) // 2
        words = np.empty(total, np.int64) if out is None else out[:total]
        if n:
            # row: first index, outputs, output address, flags, segment addresses, ends
            table = words[:_TASK_WORDS * n].reshape(n, _TASK_WORDS)
            table[:, 0] = np.cumsum(lengths) - lengths
            table[:, 1:4] = meta[:, :3]
            table[:, 4:] = np.array(self._seg_table, np.int64)[meta[:, 3]]
        task = np.repeat(np.arange(n, dtype=np.int32), counts)
        start = np.repeat(np.cumsum(counts) - counts, counts)
        pairs = words[_TASK_WORDS * n:_TASK_WORDS * n + n_chunks].view(np.int32).reshape(-1, 2)
        pairs[:, 0] = task
        pairs[:, 1] = (np.arange(n_chunks) - start) * _CHUNK
        if n_idx:
            idx = words[_TASK_WORDS * n + n_chunks:].view(np.int32)[:n_idx]
            np.concatenate(self._idx, out=idx, casting="unsafe")
        return words, n, n_chunks

    def launch(self, error_flag: torch.Tensor | None = None):
        """Copy the packed program to the device and launch; no host sync."""
        if self.device.type != "cuda":
            raise ValueError("slot gathers launch on a CUDA device; this one holds "
                             f"{self.device} tensors")
        if not self._tasks:
            return
        # torch's caching host allocator keeps the pinned block until the
        # copy that reads it has run
        host = torch.empty(self.words(), dtype=torch.int64, pin_memory=True)
        _, n_tasks, n_chunks = self.pack(out=host.numpy())
        self._reset()
        if n_chunks == 0:
            return
        dev = host.to(self.device, non_blocking=True)
        base = dev.data_ptr()  # indices: int32 after the two tables
        status = _native.lib.akv_gather_slots(
            base, base + 8 * _TASK_WORDS * n_tasks, n_chunks,
            base + 8 * (_TASK_WORDS * n_tasks + n_chunks), _native.ptr(error_flag),
            _native.stream_of(self.device))
        _native.check(status, "gather_slots")


@dataclass(frozen=True)
class OccurrenceAdvance:
    """The result fields of the reference's ``OccurrenceAdvance``
    (srt/context_system/occurrence.py:921-933), same names and order."""

    state: object
    occurrence_slots: torch.Tensor
    copy_source_slots: torch.Tensor
    copy_destination_slots: torch.Tensor
    copy_position_pairs: torch.Tensor
    retired_slots: torch.Tensor
    unused_swa_slots: torch.Tensor | None = None
    retired_swa_resident: torch.Tensor | None = None


class _AdvancePlan:
    """The CPU half of ``OccurrenceState.advance`` (occurrence.py:644-755):
    the reference's admission check and messages here, every ownership
    index from ``akv_occurrence_advance_indices`` (host code), no device
    work."""

    def __init__(self, state, window, plan, query_slots, extra_slots, visible_until):
        n = len(window.birth_occurrences)
        start, end = len(state.canonical_rows), len(plan.terminal_occurrences)
        slots = state.slots
        if (
            query_slots.ndim != 1
            or extra_slots.ndim != 1
            or len(query_slots) != end - start
            or len(extra_slots) != plan.extra_page_count
            or query_slots.dtype != slots.dtype
            or extra_slots.dtype != slots.dtype
            or (len(slots) and query_slots.device != slots.device)
            or extra_slots.device != query_slots.device
            or visible_until.device.type != "cpu"
            or visible_until.dtype != torch.int32
            or visible_until.shape != (n,)
        ):
            raise ValueError("Context admission does not cover the selected window")
        n_old, n_query, n_extra = len(slots), len(query_slots), len(extra_slots)
        total = n_old + n_query + n_extra
        count = len(plan.source_rows)
        n_copy = len(plan.copy_occurrences)
        swa_in = state.swa_resident
        arrays = dict(
            owned=_host(state.owned, np.uint8), canonical_rows=_host(state.canonical_rows, np.int64),
            terminal_rows=_host(state.terminal_rows, np.int64),
            canonical_positions=_host(state.canonical_positions, np.int32),
            swa_resident=_host(swa_in, np.uint8) if swa_in is not None else None,
            birth_occurrences=_host(window.birth_occurrences, np.int64),
            terminal_occurrences=_host(window.terminal_occurrences, np.int64),
            occurrence_positions=_host(window.occurrence_positions, np.int32),
            source_rows=_host(plan.source_rows, np.int64),
            allocated=_host(plan.allocated_occurrences, np.int64),
            copy_occurrences=_host(plan.copy_occurrences, np.int64),
            copy_source_rows=_host(plan.copy_source_rows, np.int64),
            plan_terminal=_host(plan.terminal_occurrences, np.int64),
            visible_until=_host(visible_until, np.int32))
        inp = _AdvanceIn(n, start, end, count, n_old, n_query, n_extra, n_copy,
                         *[None if a is None else _addr(a) for a in arrays.values()])
        occ = np.empty(count, np.int32)
        copy_src, copy_dst = np.empty(n_copy, np.int32), np.empty(n_copy, np.int32)
        retained, retired = np.empty(total, np.int32), np.empty(total, np.int32)
        unused_swa = np.empty(n_copy, np.int32)
        canon_rows, term_rows = np.empty(end, np.int64), np.empty(end, np.int64)
        positions = np.empty(end, np.int32)
        owned_next = np.empty(total, np.uint8)
        swa_next = np.empty(total, np.uint8) if swa_in is not None else None
        swa_retired = np.empty(total, np.uint8) if swa_in is not None else None
        out = _AdvanceOut(_addr(occ), _addr(copy_src), _addr(copy_dst), _addr(retained),
                          _addr(retired), _addr(unused_swa), _addr(canon_rows),
                          _addr(term_rows), _addr(positions), _addr(owned_next),
                          None if swa_next is None else _addr(swa_next),
                          None if swa_retired is None else _addr(swa_retired), 0, 0, 0)
        status = _native.lib.akv_occurrence_advance_indices(ctypes.byref(inp),
                                                            ctypes.byref(out))
        if status == _native.AKV_ERR_OCC_MISSING_SOURCE:
            raise ValueError("Context ownership plan references a missing source")
        if status == _native.AKV_ERR_OCC_MISSING_COPY_SOURCE:
            raise ValueError("Context copy references a missing canonical source")
        _native.check(status, "occurrence advance")
        k, r = out.n_retained, out.n_retired
        self.state_type = type(state)
        self.exact_prefix_len = state.exact_prefix_len
        self.segments = tuple(s for s in (slots, query_slots, extra_slots) if len(s)) or \
            (query_slots,)
        self.dtype, self.device = query_slots.dtype, query_slots.device
        self.occurrences = np.maximum(occ, 0, out=occ)
        self.copy_src, self.copy_dst = copy_src, copy_dst
        self.pairs = _host(plan.copy_position_pairs, np.int32).reshape(-1)
        self.retained, self.retired = retained[:k], retired[:r]
        self.unused_swa = unused_swa[: out.n_unused_swa]
        self.successor = (torch.from_numpy(owned_next[:k].view(np.bool_)),
                          torch.from_numpy(canon_rows), torch.from_numpy(term_rows),
                          torch.from_numpy(positions))
        self.swa = None
        if swa_in is not None:
            self.swa_retained = torch.from_numpy(swa_next[:k].view(np.bool_))
            self.swa_retired = torch.from_numpy(swa_retired[:r].view(np.bool_))
            self.swa = True

    def sizes(self):
        """Outputs per field: occurrences, copies, pair words, retained,
        retired, unused SWA slots."""
        return (len(self.occurrences), len(self.copy_src), len(self.pairs), len(self.retained),
                len(self.retired), len(self.unused_swa) if self.swa is not None else 0)

    def add_tasks(self, gather: SlotGather, occurrence_out, src_out, dst_out, pairs_out,
                  succ_slots=None, retired=None, unused=None):
        """Queue this request's fields into the views the caller provides
        (the successor's slots and the retired and unused SWA slots are
        allocated here when not given).  Returns the per-request result."""
        dev, dt, seg = self.device, self.dtype, self.segments
        if succ_slots is None:
            succ_slots = torch.empty(len(self.retained), dtype=dt, device=dev)
        if retired is None:
            retired = torch.empty(len(self.retired), dtype=dt, device=dev)
        fields = [(occurrence_out, self.occurrences), (src_out, self.copy_src),
                  (dst_out, self.copy_dst), (succ_slots, self.retained),
                  (retired, self.retired)]
        if self.swa is not None:
            if unused is None:
                unused = torch.empty(len(self.unused_swa), dtype=dt, device=dev)
            fields.append((unused, self.unused_swa))
        gather._add_fields(fields, seg)
        gather._add(pairs_out, self.pairs, literal=True)
        owned, canon, term, positions = self.successor
        state = self.state_type(
            succ_slots, owned, canon, term, positions, self.exact_prefix_len,
            self.swa_retained if self.swa is not None else None)
        return OccurrenceAdvance(
            state, occurrence_out, src_out, dst_out, pairs_out.view(-1, 2), retired,
            unused if self.swa is not None else None,
            self.swa_retired if self.swa is not None else None)


def advance(state, window, plan, query_slots, extra_slots, visible_until, *,
            error_flag: torch.Tensor | None = None):
    """Drop-in for ``OccurrenceState.advance``: same arguments, checks,
    messages and result fields; the successor has the type of ``state``.
    The device part is one copy and one launch on the current stream."""
    p = _AdvancePlan(state, window, plan, query_slots, extra_slots, visible_until)
    dev = p.device
    occ = torch.empty(len(p.occurrences), dtype=p.dtype, device=dev)
    i32 = torch.empty(len(p.copy_src) + len(p.copy_dst) + len(p.pairs), dtype=torch.int32,
                      device=dev)
    a, b = len(p.copy_src), len(p.copy_src) + len(p.copy_dst)
    gather = SlotGather(dev)
    result = p.add_tasks(gather, occ, i32[:a], i32[a:b], i32[b:])
    gather.launch(error_flag)
    return result


def terminal_slots(state, *, error_flag: torch.Tensor | None = None):
    """Drop-in for ``OccurrenceState.terminal_slots`` (occurrence.py:757-768):
    the raw-order final-position table, -1 at holes, in one launch."""
    rows = state.terminal_rows.numpy()
    slots = state.slots
    out = slots.new_empty((len(rows),))
    gather = SlotGather(slots.device)
    gather._add(out, rows, (slots,) if len(slots) else (slots.new_empty(0),))
    gather.launch(error_flag)
    return out


def bind(materialization, canonical_slots, terminal_slots, allocated_slots, *,
         error_flag: torch.Tensor | None = None):
    """Drop-in for ``OccurrenceMaterialization.bind`` (occurrence.py:315-357):
    (slots, copy source slots int32, copy destination slots int32, copy
    position pairs int32 [k, 2]) in one copy and one launch."""
    n = len(materialization.read_cached)
    if (
        canonical_slots.ndim != 1
        or terminal_slots.ndim != 1
        or allocated_slots.ndim != 1
        or any(
            value.dtype not in (torch.int32, torch.int64)
            for value in (canonical_slots, terminal_slots, allocated_slots)
        )
        or canonical_slots.dtype != terminal_slots.dtype
        or canonical_slots.dtype != allocated_slots.dtype
        or len(canonical_slots) != n
        or len(terminal_slots) != n
        or len(allocated_slots) != materialization.extra_page_count
        or canonical_slots.device != terminal_slots.device
        or canonical_slots.device != allocated_slots.device
    ):
        raise ValueError("Occurrence slot buffers do not match the ownership plan")
    rows = materialization.source_rows.numpy()
    fresh = materialization.allocated_occurrences.numpy()
    # One index per occurrence into concat(canonical, terminal, allocated).
    index = np.where(rows >= 0, rows, -1)
    index[fresh] = 2 * n + np.arange(len(fresh))
    copy_rows = materialization.copy_source_rows.numpy()
    copy_ids = materialization.copy_occurrences.numpy()
    pairs = materialization.copy_position_pairs.numpy().reshape(-1)
    dev = canonical_slots.device
    segments = tuple(s for s in (canonical_slots, terminal_slots, allocated_slots)
                     if len(s)) or (canonical_slots,)
    slots = canonical_slots.new_empty((len(rows),))
    i32 = torch.empty(len(copy_rows) + len(copy_ids) + len(pairs), dtype=torch.int32,
                      device=dev)
    a, b = len(copy_rows), len(copy_rows) + len(copy_ids)
    gather = SlotGather(dev)
    gather._add(slots, index, segments)
    gather._add(i32[:a], copy_rows, segments)
    gather._add(i32[a:b], index[copy_ids], segments)
    gather._add(i32[b:], pairs, literal=True)
    gather.launch(error_flag)
    return slots, i32[:a], i32[a:b], i32[b:].view(-1, 2)


class OccurrenceBatch:
    """Every request of one prefill forward in one launch.

    ``add_context(state, window, plan, birth, allocated, visible_until)``
    for a context request (the arguments of ``OccurrenceState.advance``) and
    ``add_ordinary(prefix_indices, birth)`` for an ordinary one, in batch
    order; ``launch()`` returns ``(advances, slots, sources, destinations,
    positions)``: one ``OccurrenceAdvance`` per context request (None for
    ordinary ones) and the concatenations the scheduler builds with
    ``torch.cat`` (akv/system/sglang.patch:3133-3180).  Per-request outputs
    are views of the concatenated tensors, and the successors' slots and
    the retired and unused SWA slots are views of one more batch buffer
    (each view is its request's own elements; the buffer lives as long as
    any of them)."""

    def __init__(self, device):
        self.device = torch.device(device)
        self._items = []

    def add_context(self, state, window, plan, birth, allocated, visible_until):
        self._items.append(("context", _AdvancePlan(state, window, plan, birth, allocated,
                                                    visible_until)))

    def add_ordinary(self, prefix_indices, birth):
        if prefix_indices.ndim != 1 or birth.ndim != 1 or prefix_indices.dtype != birth.dtype:
            raise ValueError("ordinary prefix and birth slots must be aligned vectors")
        self._items.append(("ordinary", (prefix_indices, birth)))

    def launch(self, error_flag: torch.Tensor | None = None):
        gather, result = self._queue()
        gather.launch(error_flag)
        return result

    def _queue(self):
        """Allocate the outputs and queue every task without launching."""
        if not self._items:
            raise ValueError("Context attention batch cannot be empty")
        dtypes = {p.dtype if kind == "context" else p[1].dtype for kind, p in self._items}
        if len(dtypes) != 1:
            raise ValueError("all requests of a forward bind slots of one dtype")
        dtype = dtypes.pop()
        # Per item: slots (occurrences, or prefix + birth), copies, pair
        # words, retained, retired, unused SWA slots; every field of the
        # batch is one buffer split into per-item views.
        sizes = np.array([p.sizes() if kind == "context" else
                          (len(p[0]) + len(p[1]), 0, 0, 0, 0, 0) for kind, p in self._items],
                         np.int64).reshape(-1, 6)
        totals = sizes.sum(axis=0)
        slots = torch.empty(int(totals[0]), dtype=dtype, device=self.device)
        n_copy, n_pairs = int(totals[1]), int(totals[2])
        i32 = torch.empty(2 * n_copy + n_pairs, dtype=torch.int32, device=self.device)
        sources, destinations = i32[:n_copy], i32[n_copy:2 * n_copy]
        positions = i32[2 * n_copy:]
        kept = torch.empty(int(totals[3] + totals[4] + totals[5]), dtype=dtype, device=self.device)
        split = lambda t, col: t.split_with_sizes(sizes[:, col].tolist())  # noqa: E731
        v_slots, v_src, v_dst = split(slots, 0), split(sources, 1), split(destinations, 1)
        v_pairs = split(positions, 2)
        v_succ, v_retired, v_unused = kept.split_with_sizes(
            [int(totals[3]), int(totals[4]), int(totals[5])])
        v_succ, v_retired, v_unused = split(v_succ, 3), split(v_retired, 4), split(v_unused, 5)
        gather = SlotGather(self.device)
        advances = []
        for i, (kind, p) in enumerate(self._items):
            if kind == "context":
                advances.append(p.add_tasks(gather, v_slots[i], v_src[i], v_dst[i], v_pairs[i],
                                            v_succ[i], v_retired[i], v_unused[i]))
            else:
                prefix, birth = p
                seg = tuple(x for x in (prefix, birth) if len(x)) or (birth,)
                gather._add(v_slots[i], np.arange(int(sizes[i, 0])), seg)
                advances.append(None)
        self._items = []
        return gather, (advances, slots, sources, destinations, positions.view(-1, 2))
