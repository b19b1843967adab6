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

This module keeps the CPU decisions (restated from the reference, same
checks and messages) and does the device part of a whole forward in ONE
host-to-device copy and ONE launch:

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

from . import _native

_MAX_SEGMENTS = 4
_TASK_WORDS = 12


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
        self._tasks = []
        self._rows = []
        self._segments = {}

    def add(self, out: torch.Tensor, indices, segments=(), *, literal: bool = False):
        """out[i] = concat(segments)[indices[i]] (-1 where the index is
        negative), or indices[i] itself with ``literal``; out is int32 or
        int64 (int64 values are cast to int32 as torch does)."""
        idx = np.asarray(indices, dtype=np.int64).reshape(-1)
        if out.dtype not in (torch.int32, torch.int64) or out.get_device() != self._index or \
                not out.is_contiguous() or out.numel() != len(idx):
            raise ValueError("gather output must be a contiguous int32/int64 vector on the "
                             "device with one element per index")
        self._add(out, idx, segments, literal)

    def _add(self, out, idx, segments=(), literal=False):
        """``add`` for an output this module allocated (contiguous, on the
        device, one element per index): the segments are still checked."""
        idx = np.asarray(idx, dtype=np.int64).reshape(-1)
        m = len(idx)
        segments = tuple(segments)
        key = tuple(id(s) for s in segments)
        info = self._segments.get(key)
        if info is None:
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
            info = (flags, ptrs + ends)
            # the task list holds the segments, so their ids stay unique
            self._segments[key] = info
        if m > 2**31 - 1:
            raise ValueError("a slot gather task holds at most 2^31 - 1 outputs")
        flags = info[0] | (_native.GATHER_OUT64 if out.dtype == torch.int64 else 0) | \
            (_native.GATHER_LITERAL if literal else 0)
        self._rows.append([0, m, out.data_ptr() if m else 0, flags, *info[1]])
        self._tasks.append((out, idx, segments, literal))

    def __len__(self):
        return len(self._tasks)

    def _sizes(self):
        chunk = int(_native.lib.akv_gather_slots_chunk())
        lengths = np.fromiter((len(t[1]) for t in self._tasks), np.int64, len(self._tasks))
        counts = (lengths + chunk - 1) // chunk
        return chunk, lengths, counts

    def words(self):
        """Length of the packed program in int64 words."""
        _, lengths, counts = self._sizes()
        return _TASK_WORDS * len(self._tasks) + int(counts.sum()) + int(lengths.sum())

    def pack(self, out: np.ndarray | None = None):
        """(words, n_tasks, n_chunks): the int64 task table, the chunk table
        (one word per chunk: the int32 pair {task, first output}) and the
        indices, in that order; written into ``out`` when given."""
        chunk, lengths, counts = self._sizes()
        n, n_chunks = len(self._tasks), int(counts.sum())
        if n_chunks > 2**31 - 1:
            raise ValueError("too many slot gather chunks for one launch")
        total = _TASK_WORDS * n + n_chunks + int(lengths.sum())
        words = np.empty(total, np.int64) if out is None else out[:total]
        if n:
            table = words[:_TASK_WORDS * n].reshape(n, _TASK_WORDS)
            table[:] = np.asarray(self._rows, np.int64)
            table[:, 0] = np.cumsum(lengths) - lengths
        task = np.repeat(np.arange(n, dtype=np.int32), counts)
        start = np.repeat(np.cumsum(counts) - counts, counts)
        pairs = words[_TASK_WORDS * n:_TASK_WORDS * n + n_chunks].view(np.int32).reshape(-1, 2)
        pairs[:, 0] = task
        pairs[:, 1] = (np.arange(n_chunks) - start) * chunk
        at = _TASK_WORDS * n + n_chunks
        for _, idx, _, _ in self._tasks:
            words[at:at + len(idx)] = idx
            at += len(idx)
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
        self._tasks, self._rows, self._segments = [], [], {}
        if n_chunks == 0:
            return
        dev = host.to(self.device, non_blocking=True)
        base = dev.data_ptr()
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
    every ownership decision and index, no device work."""

    def __init__(self, state, window, plan, query_slots, extra_slots, visible_until):
        birth_occ = window.birth_occurrences.numpy()
        n = len(birth_occ)
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
        owned = np.concatenate((state.owned.numpy(), np.ones(n_query + n_extra, np.bool_)))
        # Rows of `sources` address the state's canonical owners [0, n) and
        # its terminal owners [n, 2n); values are indices into all slots.
        canonical = np.full(n, -1, np.int64)
        canonical[:start] = state.canonical_rows.numpy()
        canonical[start:end] = np.arange(n_old, n_old + n_query)
        terminal = np.full(n, -1, np.int64)
        terminal[:start] = state.terminal_rows.numpy()
        sources = np.concatenate((canonical, terminal))
        rows = plan.source_rows.numpy()
        occurrences = np.full(len(rows), -1, np.int64)
        reuse = rows >= 0
        occurrences[reuse] = sources[rows[reuse]]
        if np.any(occurrences[reuse] < 0):
            raise ValueError("Context ownership plan references a missing source")
        occurrences[plan.allocated_occurrences.numpy()] = np.arange(n_old + n_query, total)
        copy_src = sources[plan.copy_source_rows.numpy()]
        if np.any(copy_src < 0):
            raise ValueError("Context copy references a missing canonical source")
        copy_dst = occurrences[plan.copy_occurrences.numpy()]
        swa = None
        unused_swa = np.empty(0, np.int64)
        if state.swa_resident is not None:
            swa = np.concatenate((state.swa_resident.numpy(),
                                  np.ones(n_query + n_extra, np.bool_)))
            swa[copy_dst] = swa[copy_src]
            # only fresh private copy destinations without an SWA source
            unused_swa = copy_dst[~swa[copy_dst]]
        picked = plan.terminal_occurrences.numpy()
        kept = picked >= 0
        next_term = np.full(end, -1, np.int64)
        next_term[kept] = occurrences[picked[kept]]
        occ_pos = window.occurrence_positions.numpy()
        positions = occ_pos[birth_occ[:end]].copy()
        positions[:start] = state.canonical_positions.numpy()
        same = positions == occ_pos[window.terminal_occurrences.numpy()[:end]]
        # a same-position copy is bit-identical: read the terminal owner
        next_canon = np.where(kept & same, next_term, canonical[:end])
        # no later prefill query reads a source whose token is invisible by then
        if end == n:
            next_canon[:] = -1
        else:
            next_canon = np.where(visible_until.numpy()[:end] > end, next_canon, -1)
        retained = np.unique(np.concatenate((next_canon[next_canon >= 0],
                                             next_term[next_term >= 0])))
        live = np.zeros(total, np.bool_)
        live[retained] = True
        retired = np.flatnonzero(owned & ~live)
        remap = np.full(total, -1, np.int64)
        remap[retained] = np.arange(len(retained))
        self.state_type = type(state)
        self.exact_prefix_len = state.exact_prefix_len
        self.segments = tuple(s for s in (slots, query_slots, extra_slots) if len(s)) or \
            (query_slots,)
        self.dtype, self.device = query_slots.dtype, query_slots.device
        self.occurrences = np.maximum(occurrences, 0)
        self.copy_src, self.copy_dst = copy_src, copy_dst
        self.pairs = plan.copy_position_pairs.numpy().reshape(-1)
        self.retained, self.retired, self.unused_swa = retained, retired, unused_swa
        canon_rows = np.full(end, -1, np.int64)
        has = next_canon >= 0
        canon_rows[has] = remap[next_canon[has]]
        term_rows = np.full(end, -1, np.int64)
        term_rows[kept] = remap[next_term[kept]]
        self.successor = (torch.from_numpy(owned[retained]), torch.from_numpy(canon_rows),
                          torch.from_numpy(term_rows), torch.from_numpy(positions))
        self.swa = swa

    def add_tasks(self, gather: SlotGather, occurrence_out, src_out, dst_out, pairs_out):
        """Queue this request's fields; the batch-level outputs are views the
        caller provides.  Returns the per-request device tensors."""
        dev, dt = self.device, self.dtype
        succ_slots = torch.empty(len(self.retained), dtype=dt, device=dev)
        retired = torch.empty(len(self.retired), dtype=dt, device=dev)
        seg = self.segments
        gather._add(occurrence_out, self.occurrences, seg)
        gather._add(src_out, self.copy_src, seg)
        gather._add(dst_out, self.copy_dst, seg)
        gather._add(pairs_out, self.pairs, literal=True)
        gather._add(succ_slots, self.retained, seg)
        gather._add(retired, self.retired, seg)
        unused = None
        if self.swa is not None:
            unused = torch.empty(len(self.unused_swa), dtype=dt, device=dev)
            gather._add(unused, self.unused_swa, seg)
        owned, canon, term, positions = self.successor
        state = self.state_type(
            succ_slots, owned, canon, term, positions, self.exact_prefix_len,
            torch.from_numpy(self.swa[self.retained]) if self.swa is not None else None)
        return OccurrenceAdvance(
            state, occurrence_out, src_out, dst_out, pairs_out.view(-1, 2), retired, unused,
            torch.from_numpy(self.swa[self.retired]) if self.swa is not None else None)


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
    are views of the concatenated tensors."""

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
        n_slots = n_copy = n_pairs = 0
        for kind, p in self._items:
            if kind == "context":
                n_slots += len(p.occurrences)
                n_copy += len(p.copy_src)
                n_pairs += len(p.pairs)
            else:
                n_slots += len(p[0]) + len(p[1])
        slots = torch.empty(n_slots, dtype=dtype, device=self.device)
        i32 = torch.empty(2 * n_copy + n_pairs, dtype=torch.int32, device=self.device)
        sources, destinations = i32[:n_copy], i32[n_copy:2 * n_copy]
        positions = i32[2 * n_copy:]
        gather = SlotGather(self.device)
        advances = []
        s = c = q = 0
        for kind, p in self._items:
            if kind == "context":
                k, m, r = len(p.occurrences), len(p.copy_src), len(p.pairs)
                advances.append(p.add_tasks(gather, slots[s:s + k], sources[c:c + m],
                                            destinations[c:c + m], positions[q:q + r]))
                s, c, q = s + k, c + m, q + r
            else:
                prefix, birth = p
                k = len(prefix) + len(birth)
                seg = tuple(x for x in (prefix, birth) if len(x)) or (birth,)
                gather._add(slots[s:s + k], np.arange(k), seg)
                advances.append(None)
                s += k
        self._items = []
        return gather, (advances, slots, sources, destinations, positions.view(-1, 2))
