"""Seeded synthetic workloads with the shapes of the benchmark configurations.

No public dataset is involved: every input is drawn from
``numpy.random.default_rng(seed)`` with the shapes, sizes and distributions
of the five configurations this package is measured on.

* c1 -- one request, 1 layer, 8 KV heads, head_dim 64, 4096 tokens, three
  dropped spans of 128..512 tokens, plain RoPE theta 10000.
* c2 -- GPT-OSS-120B-shaped cache: 36 layers, 8 KV heads, head_dim 64, one
  65536-token request, about 40 % dropped in 20 spans, YaRN RoPE (theta
  150000, factor 32, original 4096).  Span lengths are drawn uniform in
  [256, 4096] and then rescaled so that they total 0.4 T (20 spans drawn
  uniform in that range would average 66 % of T), clipped to [256, 4096].
* c3 -- 64 requests, lengths uniform 2K..32K, one shared radix prefix of
  1K..4K tokens, per-request drop fraction uniform 10..60 % in
  ceil(f L / 1024) spans, the first span starting inside the first half of
  the prefix so that shared tokens behind it must be copied (COW).
* c4 -- ragged decode attention: batch 128, 64 q heads / 8 KV heads,
  head_dim 64, lognormal KV lengths (median 8192, sigma 1.0, clipped to
  [1, 65536]), sinks ~ N(0, 1).
* c5 -- Llama-3-70B-shaped cache: 80 layers, 8 KV heads, head_dim 128,
  8 requests of 131072 tokens, 30 % dropped, plain RoPE theta 500000.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np


def place_spans(rng, token_count, lengths, lo=0):
    """Place spans of the given lengths, in order and disjoint, inside
    [lo, token_count), with the free tokens split by a sorted uniform draw.
    Returns an int32 array of (start, end) pairs, flattened."""
    lengths = np.asarray(lengths, np.int64)
    free = token_count - lo - int(lengths.sum())
    if free < 0:
        raise ValueError("spans do not fit")
    cuts = np.sort(rng.integers(0, free + 1, size=len(lengths)))
    starts = lo + cuts + np.concatenate(([0], np.cumsum(lengths)[:-1]))
    return np.stack((starts, starts + lengths), 1).reshape(-1).astype(np.int32)


def rescaled_lengths(rng, count, lo, hi, total):
    """``count`` lengths drawn uniform in [lo, hi], rescaled to sum to about
    ``total`` and clipped back into [lo, hi]."""
    raw = rng.uniform(lo, hi, size=count)
    scaled = np.clip(np.round(raw * (total / raw.sum())), lo, hi).astype(np.int64)
    return scaled


@dataclass
class DropProgram:
    """Batched Drop + Reposition program in request-local raw indices."""

    token_counts: np.ndarray  # int64 [R]
    range_offsets: np.ndarray  # int32 [R+1], in pairs
    ranges: np.ndarray  # int32 [2 * n_ranges], (start, end) pairs
    shared_prefix: np.ndarray  # int64 [R], borrowed radix tokens per request
    meta: dict = field(default_factory=dict)

    @property
    def requests(self):
        return len(self.token_counts)

    @property
    def total_tokens(self):
        return int(self.token_counts.sum())

    def request_ranges(self, r):
        a, b = self.range_offsets[r], self.range_offsets[r + 1]
        return self.ranges[2 * a: 2 * b]

    def keep_mask(self, r):
        keep = np.ones(int(self.token_counts[r]), bool)
        rr = self.request_ranges(r).reshape(-1, 2)
        for s, e in rr:
            keep[s:e] = False
        return keep


def _program(counts, per_request, shared=None, meta=None):
    offsets = [0]
    for spans in per_request:
        offsets.append(offsets[-1] + len(spans) // 2)
    ranges = (np.concatenate(per_request) if per_request else np.zeros(0)).astype(np.int32)
    shared = np.zeros(len(counts), np.int64) if shared is None else np.asarray(shared, np.int64)
    return DropProgram(np.asarray(counts, np.int64), np.asarray(offsets, np.int32), ranges,
                       shared, meta or {})


def c1_program(seed=0, tokens=4096):
    rng = np.random.default_rng(seed)
    lengths = rng.integers(128, 513, size=3)
    return _program([tokens], [place_spans(rng, tokens, lengths)], meta=dict(config="c1"))


def c2_program(seed=0, tokens=65536, spans=20, frac=0.4):
    rng = np.random.default_rng(seed)
    lengths = rescaled_lengths(rng, spans, 256, 4096, frac * tokens)
    return _program([tokens], [place_spans(rng, tokens, lengths)], meta=dict(config="c2"))


def c3_program(seed=0, requests=64, min_len=2048, max_len=32768, page_align=1):
    """``page_align``: round the shared prefix down to a whole number of
    pages of that size (a radix cache over a paged pool shares whole
    pages); 1 keeps the drawn length."""
    rng = np.random.default_rng(seed)
    prefix = int(rng.integers(1024, 4097)) // page_align * page_align
    counts = rng.integers(max(min_len, prefix + 2), max_len + 1, size=requests)
    per_request = []
    for length in counts:
        length = int(length)
        frac = rng.uniform(0.1, 0.6)
        total = int(round(frac * length))
        count = max(1, int(np.ceil(total / 1024)))
        lengths = np.maximum(1, rescaled_lengths(rng, count, 1, 2048, total))
        first_start = int(rng.integers(0, prefix // 2))
        first_end = first_start + int(lengths[0])
        rest = lengths[1:]
        while first_end + int(rest.sum()) > length:
            rest = rest[:-1]
        spans = [np.array([first_start, first_end], np.int32)]
        if len(rest):
            spans.append(place_spans(rng, length, rest, lo=first_end))
        per_request.append(np.concatenate(spans))
    return _program(counts, per_request, shared=np.full(requests, prefix),
                    meta=dict(config="c3", prefix=prefix))


def c5_program(seed=0, requests=8, tokens=131072, spans=20, frac=0.3):
    rng = np.random.default_rng(seed)
    per_request = []
    for _ in range(requests):
        lengths = rescaled_lengths(rng, spans, 256, 4096, frac * tokens)
        per_request.append(place_spans(rng, tokens, lengths))
    return _program([tokens] * requests, per_request, meta=dict(config="c5"))


def slot_rows(rng, program, shared_slots=None, first_slot=1):
    """req_to_token rows: each request's private tokens get distinct slots
    from a random permutation of ``first_slot..``; slot 0 is the padding slot.
    Tokens below the shared prefix all map to the same shared slots."""
    prefix = int(program.shared_prefix.max()) if program.requests else 0
    private = int((program.token_counts - program.shared_prefix).sum())
    perm = rng.permutation(prefix + private).astype(np.int64) + first_slot
    shared = perm[:prefix]
    cursor = prefix
    rows = []
    for r in range(program.requests):
        t, p = int(program.token_counts[r]), int(program.shared_prefix[r])
        row = np.empty(t, np.int32)
        row[:p] = shared[:p]
        row[p:] = perm[cursor: cursor + t - p]
        cursor += t - p
        rows.append(row)
    return rows, prefix + private + first_slot


def paged_slot_rows(rng, program, page_size, first_page=1):
    """req_to_token rows over a paged pool (slot = page * page_size +
    offset): the shared prefix (a whole number of pages) maps every request
    to the same pages; each request's private tokens fill their own pages,
    token t at offset t % page_size, the pages drawn from a random
    permutation and handed to each request in ascending order (as an
    allocator with a sorted free list does).  Page 0 stays unused (slot 0
    is SGLang's padding slot).  Returns (rows, number of pages including
    the unused ones)."""
    ps = int(page_size)
    prefix = int(program.shared_prefix.max()) if program.requests else 0
    if prefix % ps:
        raise ValueError("the shared prefix must be a whole number of pages")
    private = [-(-(int(t) - int(p)) // ps) for t, p in
               zip(program.token_counts, program.shared_prefix)]
    n_pages = prefix // ps + sum(private)
    perm = rng.permutation(n_pages).astype(np.int64) + first_page
    shared = np.sort(perm[: prefix // ps])
    cursor = prefix // ps
    rows = []
    for r in range(program.requests):
        t, p = int(program.token_counts[r]), int(program.shared_prefix[r])
        pages = np.concatenate((shared[: p // ps], np.sort(perm[cursor: cursor + private[r]])))
        cursor += private[r]
        tok = np.arange(t)
        rows.append((pages[tok // ps] * ps + tok % ps).astype(np.int32))
    return rows, n_pages + first_page


@dataclass
class DecodeBatch:
    lengths: np.ndarray  # int64 [bs]
    meta: dict = field(default_factory=dict)


def c4_lengths(seed=0, batch=128, median=8192, sigma=1.0, max_len=65536):
    rng = np.random.default_rng(seed)
    lengths = np.clip(np.round(rng.lognormal(np.log(median), sigma, size=batch)), 1, max_len)
    return lengths.astype(np.int64)


def event_program(rng, tokens, events, repositions, max_ranges=4, span=None):
    """A seeded multi-event program in the reference's input format
    (compile_context_layout, ir.py:113-121): ``events`` Drop events at
    distinct insertion offsets in [1, tokens], each with 1..max_ranges
    ordered, disjoint, already materialized ranges (later events may cover
    tokens an earlier one dropped), and ``repositions`` Repositions at
    distinct raw boundaries.  ``span`` caps a range's length (None: up to
    the insertion offset).  Returns (token_ids int64, drop_insert_offsets,
    drop_range_offsets, drop_ranges, reposition_raw_boundaries), int32
    except the ids."""
    tokens = int(tokens)
    events = min(int(events), tokens)
    inserts = (np.sort(rng.choice(np.arange(1, tokens + 1), size=events, replace=False))
               if events else np.zeros(0, np.int64))
    offsets, ranges = [0], []
    for ins in inserts:
        k = int(min(rng.integers(1, max_ranges + 1), (ins + 1) // 2))
        if span is None:
            points = np.sort(rng.choice(np.arange(0, ins + 1), size=2 * k, replace=False))
        else:
            starts = np.sort(rng.choice(np.arange(0, ins), size=k, replace=False))
            ends = np.minimum(starts + rng.integers(1, span + 1, size=k), ins)
            ends = np.minimum(ends, np.append(starts[1:] - 1, ins))  # keep previous_end < start
            keep = ends > starts
            points = np.stack((starts[keep], ends[keep]), 1).reshape(-1)
            k = len(points) // 2
            if k == 0:
                points, k = np.array([ins - 1, ins]), 1
        ranges += [int(x) for x in points]
        offsets.append(offsets[-1] + k)
    reps = min(int(repositions), tokens)
    bounds = (np.sort(rng.choice(np.arange(0, tokens), size=reps, replace=False))
              if reps else np.zeros(0, np.int64))
    ids = rng.integers(0, 200000, size=tokens).astype(np.int64)
    return (ids, inserts.astype(np.int32), np.asarray(offsets, np.int32),
            np.asarray(ranges, np.int32), bounds.astype(np.int32))


def agent_turn_programs(seed=0, requests=64, turns=8, min_len=2048, max_len=32768,
                        drop_frac=0.3, max_span=1024):
    """Multi-turn agent programs for the general event compiler ("c3m"):
    the c3 request lengths (lengths U{min_len..max_len}, seeded), each prompt
    cut into ``turns`` turns at sorted random raw boundaries; at the end of
    every turn one Drop event removes spans (each at most ``max_span``
    tokens, about ``drop_frac`` of the turn's new tokens in total) from the
    text materialized so far, and a Reposition at the same insertion offset
    compacts the positions -- the cache operation an agent runs per turn.
    Returns a list of (token_ids, drop_insert_offsets, drop_range_offsets,
    drop_ranges, reposition_raw_boundaries)."""
    rng = np.random.default_rng(seed)
    counts = rng.integers(min_len, max_len + 1, size=requests)
    programs = []
    for length in counts:
        length = int(length)
        bounds = np.sort(rng.choice(np.arange(turns, length - 1), size=turns, replace=False))
        inserts, offsets, ranges = [], [0], []
        prev = 0
        for b in bounds:
            ins = int(b) + 1
            budget = max(1, int(drop_frac * (ins - prev)))
            count = max(1, -(-budget // max_span))
            lengths = np.maximum(1, rescaled_lengths(rng, count, 1, max_span, budget))
            spans = place_spans(rng, ins, lengths)
            inserts.append(ins)
            ranges += [int(x) for x in spans]
            offsets.append(offsets[-1] + len(spans) // 2)
            prev = ins
        ids = rng.integers(0, 200000, size=length).astype(np.int64)
        programs.append((ids, np.asarray(inserts, np.int32), np.asarray(offsets, np.int32),
                         np.asarray(ranges, np.int32), bounds.astype(np.int32)))
    return programs
