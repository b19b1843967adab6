"""The event compiler on the GPU (C ABI ``akv_compile_layouts``).

The reference compiles each request's immutable event program -- Drop
events (insertion offset + half-open raw-token ranges) and Reposition events
(raw boundaries) -- on the scheduler CPU: ``compile_context_layout``
(srt/context_system/ir.py:113-274) runs the C++ count and compile sweeps of
kernels/ops/attention/context_plan.py:80-532 and returns a
``ContextLayout``.  ``LayoutCompiler`` computes the same ``ContextLayout``
for a batch of requests on the device in four stream-ordered launches, and
``compile_context_layout`` is a drop-in for the reference function (same
inputs, checks, error messages and output tensors, on the CPU by default).

Host work is the reference's metadata validation (O(events + ranges +
Repositions) with numpy) and one packed host-to-device copy; the per-token
work runs on the device.
"""

from __future__ import annotations

import time
from dataclasses import dataclass

import numpy as np
import torch

from . import _native

TILE = 512
MAX_REPOSITIONS = int(_native.lib.akv_compile_layouts_max_repositions())
_INT32_MAX = 2**31 - 1


@dataclass(frozen=True)
class ContextLayout:
    """Field for field the reference's ContextLayout
    (srt/context_system/ir.py:37-59)."""

    drop_insert_offsets: torch.Tensor
    drop_range_offsets: torch.Tensor
    drop_ranges: torch.Tensor
    records: torch.Tensor
    virtual_mask: torch.Tensor
    key_to_token: torch.Tensor
    token_to_key: torch.Tensor
    positions: torch.Tensor
    keep_mask: torch.Tensor
    materialized_stage: torch.Tensor
    birth_positions: torch.Tensor
    birth_stages: torch.Tensor
    transition_offsets: torch.Tensor
    transition_raw_tokens: torch.Tensor
    transition_old_positions: torch.Tensor
    transition_new_positions: torch.Tensor
    effective_reposition_stages: torch.Tensor
    drop_event_to_key: torch.Tensor
    effective_repositions: torch.Tensor
    ignored_repositions: torch.Tensor
    next_position: int
    compile_ns: int

    @property
    def keys(self) -> torch.Tensor:
        return self.records


def validate_program(token_count, drop_insert_offsets, drop_range_offsets, drop_ranges,
                     reposition_raw_boundaries, reposition_insert_offsets):
    """The reference's metadata checks, in the order its count pass makes
    them (context_plan.py:88-130, range check :155-157), with its messages.
    The reference's ``require`` failures surface in Python as RuntimeError
    (std::invalid_argument through its FFI), so these raise RuntimeError too.
    Arguments are 1-D integer numpy arrays."""
    drops = np.asarray(drop_insert_offsets, np.int64)
    offsets = np.asarray(drop_range_offsets, np.int64)
    ranges = np.asarray(drop_ranges, np.int64)
    bounds = np.asarray(reposition_raw_boundaries, np.int64)
    inserts = np.asarray(reposition_insert_offsets, np.int64)
    if token_count < 0 or token_count > _INT32_MAX:
        raise RuntimeError("token_count exceeds the int32 Reposition limit")
    if len(offsets) != len(drops) + 1 or len(ranges) % 2 or len(inserts) != len(bounds):
        raise RuntimeError("Reposition transition-count tensor lengths are inconsistent")
    if offsets[0] != 0 or offsets[-1] != len(ranges) // 2:
        raise RuntimeError("drop_range_offsets does not cover drop_ranges")
    if len(drops) and (np.any(drops < 0) or np.any(drops > token_count)
                       or np.any(np.diff(drops) <= 0) or np.any(np.diff(offsets) <= 0)):
        raise RuntimeError("Invalid Drop event metadata")
    if len(bounds) and (np.any(inserts != bounds + 1) or np.any(inserts <= 0)
                        or np.any(inserts > token_count) or np.any(np.diff(bounds) <= 0)):
        raise RuntimeError("Invalid Reposition event metadata")
    if len(ranges):
        starts, ends = ranges[0::2], ranges[1::2]
        owner = np.repeat(np.arange(len(drops)), np.diff(offsets))
        first = np.zeros(len(starts), bool)
        first[offsets[:-1]] = True
        prev_end = np.concatenate(([-1], ends[:-1]))
        ok = (starts >= 0) & (starts < ends) & (ends <= drops[owner]) & (first | (prev_end < starts))
        if not ok.all():
            raise RuntimeError("Drop ranges must be ordered, disjoint, and already materialized")
    if len(bounds) > MAX_REPOSITIONS:
        raise ValueError(f"at most {MAX_REPOSITIONS} Reposition events per request are supported")


@dataclass
class Program:
    """One request's event program (request-local values, as the reference
    takes them)."""

    token_ids: np.ndarray
    drop_insert_offsets: np.ndarray
    drop_range_offsets: np.ndarray
    drop_ranges: np.ndarray
    reposition_raw_boundaries: np.ndarray

    @staticmethod
    def of(token_ids, drop_insert_offsets=(), drop_range_offsets=(0,), drop_ranges=(),
           reposition_raw_boundaries=(), reposition_insert_offsets=None, validate=True):
        p = Program(np.asarray(token_ids), np.asarray(drop_insert_offsets, np.int32),
                    np.asarray(drop_range_offsets, np.int32), np.asarray(drop_ranges, np.int32),
                    np.asarray(reposition_raw_boundaries, np.int32))
        if validate:
            ins = (p.reposition_raw_boundaries.astype(np.int64) + 1
                   if reposition_insert_offsets is None else reposition_insert_offsets)
            validate_program(len(p.token_ids), p.drop_insert_offsets, p.drop_range_offsets,
                             p.drop_ranges, p.reposition_raw_boundaries, ins)
        return p


class BatchLayout:
    """Device outputs of one ``LayoutCompiler.compile`` call.  Per-request
    transition and decode-view offsets, counts and status live on the
    device; ``status()`` and ``request()`` read them (and synchronise)."""

    def __init__(self, compiler, plan):
        self._c = compiler
        self._plan = plan

    @property
    def totals(self) -> torch.Tensor:
        """{transitions, kept tokens, keys, AKV_LAYOUT_* bits} on the device."""
        return self._c.totals

    def status(self) -> np.ndarray:
        return self._c.status[: self._plan["n"]].cpu().numpy()

    def check(self):
        """Raise the reference's ValueError for the first failed request."""
        totals = self._c.totals.cpu().tolist()
        if totals[3] & _native.LAYOUT_CAPACITY:
            raise RuntimeError("transition capacity exceeded")
        for code, _, _, _, arg in self.status():
            if code == 1:
                raise ValueError(f"Reposition at raw boundary {arg} has no active tokens.")
            if code == 2:
                raise ValueError(
                    f"Reposition Radix token ID {arg} is outside the non-negative int32 range.")
            if code < 0:
                raise ValueError("too many Reposition events")

    def request(self, b, to_cpu=True, compile_ns=0) -> ContextLayout:
        """The reference's ContextLayout of request ``b`` (synchronises)."""
        c, plan = self._c, self._plan
        status = c.status[b].cpu().tolist()
        key_len, stages, next_position = status[1], status[2], status[3]
        t0, t1 = plan["tokens"][b], plan["tokens"][b + 1]
        e0, e1 = plan["events"][b], plan["events"][b + 1]
        r0, r1 = plan["reps"][b], plan["reps"][b + 1]
        g0, g1 = plan["ranges"][b], plan["ranges"][b + 1]
        k0 = t0 + g0 + r0
        tr = c.transition_request_offsets[b: b + 2].cpu().tolist()
        col = r0 + b
        dev = {
            "records": c.records[k0: k0 + key_len],
            "virtual_mask": c.virtual_mask[k0: k0 + key_len].view(torch.bool),
            "key_to_token": c.key_to_token[k0: k0 + key_len],
            "token_to_key": c.token_to_key[t0:t1],
            "positions": c.positions[t0:t1],
            "keep_mask": c.keep_mask[t0:t1].view(torch.bool),
            "materialized_stage": c.materialized_stage[t0:t1],
            "birth_positions": c.birth_positions[t0:t1],
            "birth_stages": c.birth_stages[t0:t1],
            "transition_offsets": c.transition_offsets[col: col + stages + 1],
            "transition_raw_tokens": c.transition_raw[tr[0]: tr[1]],
            "transition_old_positions": c.transition_old[tr[0]: tr[1]],
            "transition_new_positions": c.transition_new[tr[0]: tr[1]],
            "effective_reposition_stages": c.effective_stages[r0:r1],
            "drop_event_to_key": c.drop_event_to_key[e0:e1],
            "effective_repositions": c.effective[r0:r1].view(torch.bool),
            "ignored_repositions": c.ignored[r0:r1].view(torch.bool),
        }
        if to_cpu:
            dev = {k: v.cpu() for k, v in dev.items()}
        prog = plan["programs"][b]
        return ContextLayout(
            drop_insert_offsets=torch.from_numpy(prog.drop_insert_offsets.astype(np.int32)),
            drop_range_offsets=torch.from_numpy(prog.drop_range_offsets.astype(np.int32)),
            drop_ranges=torch.from_numpy(prog.drop_ranges.astype(np.int32)),
            next_position=int(next_position), compile_ns=int(compile_ns), **dev)

    def decode_view(self, b):
        """(raw_indices, positions) of request b's kept tokens, device views
        (ContextDecodeLayout.from_layout, occurrence.py:47-66; synchronises)."""
        a0, a1 = self._c.active_offsets[b: b + 2].cpu().tolist()
        return self._c.raw_indices[a0:a1], self._c.active_positions[a0:a1]


class LayoutCompiler:
    """Device-resident buffers for compiling batches of event programs.

    Capacities are fixed at construction so ``compile`` allocates nothing on
    the device; ``transition_capacity`` bounds the transitions of one batch
    (a batch that needs more raises on ``check`` -- rebuild with a larger
    capacity; the count is in ``totals[0]``).
    """

    def __init__(self, device, max_tokens, max_requests=1, max_events=64, max_ranges=4096,
                 max_repositions=64, transition_capacity=None, token_ids_64=True):
        dev = torch.device(device)
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        self.max_tokens, self.max_requests = int(max_tokens), int(max_requests)
        self.max_events, self.max_ranges = int(max_events), int(max_ranges)
        self.max_repositions = int(max_repositions)
        self.max_tiles = self.max_tokens // TILE + self.max_requests
        self.max_cells = self.max_tiles * (self.max_repositions + self.max_requests)
        if transition_capacity is None:
            transition_capacity = self.max_tokens * max(1, min(self.max_repositions, 4))
        self.capacity = int(transition_capacity)
        n, T, R, P = self.max_requests, self.max_tokens, self.max_ranges, self.max_repositions
        E = self.max_events
        keys = T + R + P
        i32 = dict(dtype=torch.int32, device=dev)
        self.token_ids = torch.empty(max(T, 1), dtype=torch.int64 if token_ids_64 else torch.int32,
                                     device=dev)
        self.ids64 = 1 if token_ids_64 else 0
        self.positions = torch.empty(max(T, 1), **i32)
        self.keep_mask = torch.empty(max(T, 1), dtype=torch.uint8, device=dev)
        self.materialized_stage = torch.empty(max(T, 1), **i32)
        self.birth_positions = torch.empty(max(T, 1), **i32)
        self.birth_stages = torch.empty(max(T, 1), **i32)
        self.token_to_key = torch.empty(max(T, 1), dtype=torch.int64, device=dev)
        self.records = torch.empty((max(keys, 1), 3), **i32)
        self.virtual_mask = torch.empty(max(keys, 1), dtype=torch.uint8, device=dev)
        self.key_to_token = torch.empty(max(keys, 1), dtype=torch.int64, device=dev)
        self.transition_offsets = torch.empty(P + n, **i32)
        self.transition_request_offsets = torch.empty(n + 1, **i32)
        self.transition_raw = torch.empty(max(self.capacity, 1), **i32)
        self.transition_old = torch.empty(max(self.capacity, 1), **i32)
        self.transition_new = torch.empty(max(self.capacity, 1), **i32)
        self.effective_stages = torch.empty(max(P, 1), **i32)
        self.effective = torch.empty(max(P, 1), dtype=torch.uint8, device=dev)
        self.ignored = torch.empty(max(P, 1), dtype=torch.uint8, device=dev)
        self.drop_event_to_key = torch.empty(max(E, 1), dtype=torch.int64, device=dev)
        self.status = torch.empty((n, 5), dtype=torch.int64, device=dev)
        self.active_offsets = torch.empty(n + 1, **i32)
        self.raw_indices = torch.empty(max(T, 1), **i32)
        self.active_positions = torch.empty(max(T, 1), **i32)
        self.totals = torch.empty(4, dtype=torch.int64, device=dev)
        ws = int(_native.lib.akv_compile_layouts_workspace_bytes(n, T, P, self.max_cells))
        self.workspace = torch.empty(ws, dtype=torch.uint8, device=dev)
        # Packed int32 metadata: offsets and event vectors, one copy per call.
        self._meta_len = 3 * (n + 1) + E + (E + 1) + 2 * R + P + 4 * (n + 1) + 9
        self._meta_host = torch.empty(self._meta_len, dtype=torch.int32, pin_memory=True)
        self._meta_dev = torch.empty(self._meta_len, **i32)
        self._ids_host = torch.empty(max(T, 1), dtype=self.token_ids.dtype, pin_memory=True)
        self._copied = torch.cuda.Event()
        self._copied.record(torch.cuda.current_stream(dev))

    def compile(self, programs) -> BatchLayout:
        """Compile a list of ``Program`` (validated) on the current stream."""
        return self.launch(self.prepare(programs))

    def launch(self, prepared) -> BatchLayout:
        """Run the four launches on inputs already copied by ``prepare``
        (stream-ordered, no host synchronisation)."""
        batch, plan = prepared
        _native.check(_native.lib.akv_compile_layouts(batch, _native.stream_of(self.device)),
                      "compile_layouts")
        return BatchLayout(self, plan)

    def prepare(self, programs):
        """Pack the programs and copy them to the device (one pinned copy for
        the metadata, one for the token ids); returns what ``launch`` takes."""
        n = len(programs)
        T = [len(p.token_ids) for p in programs]
        E = [len(p.drop_insert_offsets) for p in programs]
        R = [len(p.drop_ranges) // 2 for p in programs]
        P = [len(p.reposition_raw_boundaries) for p in programs]
        tokens = np.concatenate(([0], np.cumsum(T))).astype(np.int64)
        events = np.concatenate(([0], np.cumsum(E))).astype(np.int64)
        ranges = np.concatenate(([0], np.cumsum(R))).astype(np.int64)
        reps = np.concatenate(([0], np.cumsum(P))).astype(np.int64)
        tiles = np.concatenate(([0], np.cumsum([-(-t // TILE) for t in T]))).astype(np.int64)
        cells = np.concatenate(([0], np.cumsum(np.diff(tiles) * (np.asarray(P) + 1)))).astype(
            np.int64)
        if (n > self.max_requests or tokens[-1] > self.max_tokens or events[-1] > self.max_events
                or ranges[-1] > self.max_ranges or reps[-1] > self.max_repositions):
            raise ValueError("batch exceeds the compiler's capacities")
        # Global range offsets of every event (request-local offsets shifted).
        dro = np.concatenate([p.drop_range_offsets[:-1].astype(np.int64) + ranges[i]
                              for i, p in enumerate(programs)] + [ranges[-1:]])
        empty = np.zeros(0, np.int32)
        parts = [  # int32 words; the two int64 vectors last (kept 8-byte aligned)
            tiles.astype(np.int32), events.astype(np.int32), reps.astype(np.int32),
            np.concatenate([p.drop_insert_offsets for p in programs] + [empty]),
            dro.astype(np.int32),
            np.concatenate([p.drop_ranges for p in programs] + [empty]),
            np.concatenate([p.reposition_raw_boundaries for p in programs] + [empty]),
            tokens.view(np.int32), cells.view(np.int32),
        ]
        self._copied.synchronize()
        host = self._meta_host.numpy()
        offs, o = [], 0
        for part in parts:
            part = np.ascontiguousarray(part).view(np.int32)
            offs.append(o)
            host[o: o + len(part)] = part
            o += len(part) + (len(part) & 1)  # even word offsets
        n_ids = int(tokens[-1])
        if n_ids:  # one pass straight into the pinned staging buffer
            np.concatenate([np.asarray(p.token_ids) for p in programs],
                           out=self._ids_host.numpy()[:n_ids], casting="unsafe")
        stream = torch.cuda.current_stream(self.device)
        self._meta_dev[:o].copy_(self._meta_host[:o], non_blocking=True)
        if n_ids:
            self.token_ids[:n_ids].copy_(self._ids_host[:n_ids], non_blocking=True)
        self._copied.record(stream)
        md = self._meta_dev
        addr = lambda i: md.data_ptr() + 4 * offs[i]  # noqa: E731
        b = _native.LayoutBatch()
        b.n_requests, b.n_tiles = n, int(tiles[-1])
        b.n_tokens, b.n_repositions, b.n_count_cells = int(tokens[-1]), int(reps[-1]), int(cells[-1])
        b.token_offsets, b.count_offsets = addr(7), addr(8)
        b.token_ids, b.token_ids_is64 = self.token_ids.data_ptr(), self.ids64
        b.tile_offsets, b.drop_event_offsets, b.reposition_offsets = addr(0), addr(1), addr(2)
        b.drop_insert_offsets, b.drop_range_offsets = addr(3), addr(4)
        b.drop_ranges, b.reposition_raw_boundaries = addr(5), addr(6)
        for name, t in (("positions", self.positions), ("keep_mask", self.keep_mask),
                        ("materialized_stage", self.materialized_stage),
                        ("birth_positions", self.birth_positions),
                        ("birth_stages", self.birth_stages), ("token_to_key", self.token_to_key),
                        ("records", self.records), ("virtual_mask", self.virtual_mask),
                        ("key_to_token", self.key_to_token),
                        ("transition_offsets", self.transition_offsets),
                        ("transition_request_offsets", self.transition_request_offsets),
                        ("transition_raw_tokens", self.transition_raw),
                        ("transition_old_positions", self.transition_old),
                        ("transition_new_positions", self.transition_new),
                        ("effective_reposition_stages", self.effective_stages),
                        ("effective_repositions", self.effective),
                        ("ignored_repositions", self.ignored),
                        ("drop_event_to_key", self.drop_event_to_key), ("status", self.status),
                        ("active_offsets", self.active_offsets), ("raw_indices", self.raw_indices),
                        ("active_positions", self.active_positions), ("totals", self.totals),
                        ("workspace", self.workspace)):
            setattr(b, name, t.data_ptr())
        b.transition_capacity = self.capacity
        if int(cells[-1]) > self.max_cells or int(_native.lib.akv_compile_layouts_workspace_bytes(
                n, int(tokens[-1]), int(reps[-1]), int(cells[-1]))) > self.workspace.numel():
            raise ValueError("batch exceeds the compiler's workspace")
        plan = dict(n=n, tokens=tokens.tolist(), events=events.tolist(), ranges=ranges.tolist(),
                    reps=reps.tolist(), programs=programs,
                    h2d_bytes=4 * o + self._ids_host.element_size() * n_ids)
        return b, plan


def _check_vector(name, value):
    if (not isinstance(value, torch.Tensor) or value.device.type != "cpu" or value.ndim != 1
            or value.dtype not in (torch.int32, torch.int64)):
        raise ValueError(f"{name} must be a one-dimensional CPU integer tensor.")
    if value.dtype == torch.int64 and len(value) and (
            int(value.min()) < -(2**31) or int(value.max()) >= 2**31):
        raise ValueError(f"{name} exceeds the signed int32 range.")


def compile_context_layout(token_ids, drop_insert_offsets, drop_range_offsets, drop_ranges,
                           reposition_raw_boundaries, reposition_insert_offsets, *, device=None,
                           to_cpu=True) -> ContextLayout:
    """Drop-in for the reference's compile_context_layout (ir.py:113-274):
    same inputs (CPU int32/int64 vectors), checks and messages; the layout
    is compiled on ``device`` (default: the current CUDA device) and, with
    ``to_cpu``, returned as CPU tensors like the reference's."""
    started = time.perf_counter_ns()
    vectors = {
        "token_ids": token_ids, "drop_insert_offsets": drop_insert_offsets,
        "drop_range_offsets": drop_range_offsets, "drop_ranges": drop_ranges,
        "reposition_raw_boundaries": reposition_raw_boundaries,
        "reposition_insert_offsets": reposition_insert_offsets,
    }
    for name, value in vectors.items():
        _check_vector(name, value)
    arrays = {k: v.numpy() for k, v in vectors.items()}
    prog = Program.of(arrays["token_ids"], arrays["drop_insert_offsets"],
                      arrays["drop_range_offsets"], arrays["drop_ranges"],
                      arrays["reposition_raw_boundaries"], arrays["reposition_insert_offsets"])
    T = len(prog.token_ids)
    compiler = LayoutCompiler(
        device if device is not None else torch.device("cuda", torch.cuda.current_device()),
        max_tokens=T, max_requests=1, max_events=len(prog.drop_insert_offsets),
        max_ranges=len(prog.drop_ranges) // 2,
        max_repositions=len(prog.reposition_raw_boundaries),
        token_ids_64=token_ids.dtype == torch.int64,
        transition_capacity=max(1, T * max(1, min(len(prog.reposition_raw_boundaries), 4))))
    batch = compiler.compile([prog])
    totals = compiler.totals.cpu().tolist()
    if totals[3] & _native.LAYOUT_CAPACITY:  # more transitions than guessed: exact size
        compiler = LayoutCompiler(
            compiler.device, max_tokens=T, max_requests=1,
            max_events=compiler.max_events, max_ranges=compiler.max_ranges,
            max_repositions=compiler.max_repositions, token_ids_64=compiler.ids64 == 1,
            transition_capacity=int(totals[0]))
        batch = compiler.compile([prog])
    batch.check()
    return batch.request(0, to_cpu=to_cpu, compile_ns=time.perf_counter_ns() - started)
