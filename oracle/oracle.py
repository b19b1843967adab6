"""numpy-facing wrapper of the CPU oracle (test infrastructure only).

Only tests/, ``__graft_entry__.smoke()`` and the cpu_baseline leg of
bench.py import this module.  It is the checker, never the product: the
``akv_b200`` package does not import it and has no CPU fallback.

Functions and the reference code they restate (paths relative to the
reference project root):

* ``compile_layout``     context_plan.py:210-532 via ir.py:113-274
* ``decode_layout``      context_system/occurrence.py:47-66
* ``reposition``         kernels/ops/attention/context_reposition.py:28-123
* ``decode_indices``     kernels/ops/attention/context_page_table.py:34-76
* ``window_lengths``     kernels/ops/attention/context_page_table.py:7-31
* ``window_lengths_cpu`` layers/attention/context_backend.py:742-752
* ``write_row_slots``    kernels/ops/memory/context_rows.py:7-15
* ``drop_compact``       the batched Drop + single Reposition operation of
  this build, composed from ``compile_layout`` per request (one drop event at
  the end of the prompt, one Reposition at its last token), the decode view
  and the freed-slot rule of occurrence.py:711-714 / 936-964
* ``active_slots``, ``active_lengths``
                         srt/disaggregation/context_transfer.py:110-138
* ``occurrence_advance``, ``occurrence_bind``, ``terminal_slots``
                         srt/context_system/occurrence.py:644-755, 315-357,
                         757-768 (request-local page ownership)
* ``gather_slots``       the contract of ``akv_gather_slots`` (include/akv_b200.h)
                         run over a packed program, to check the host packing
* ``decode_attention``   paged GQA decode with learned sinks, the math of
  layers/attention/context_backend.py:254-272 (sink LSE correction) over the
  registry's ``kv_indptr / kv_indices``; float64.
"""

from __future__ import annotations

import ctypes
import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np

from .build_oracle import ORACLE_SO, build_oracle

_lib = None

OK, INVALID, NO_ACTIVE, TOKEN_RANGE, CAPACITY = 0, 1, 2, 3, 4
DT_F16, DT_BF16, DT_F32 = 0, 1, 2


def lib():
    global _lib
    if _lib is None:
        path = ORACLE_SO if os.path.exists(ORACLE_SO) else build_oracle()
        _lib = ctypes.CDLL(path)
    return _lib


def _p(a):
    return ctypes.c_void_p(0 if a is None else a.ctypes.data)


def _i32(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32))


def _i64(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.int64))


# --------------------------------------------------------------------------
# Event compiler
# --------------------------------------------------------------------------


def compile_layout(token_ids, drop_insert_offsets, drop_range_offsets, drop_ranges,
                   reposition_raw_boundaries, reposition_insert_offsets):
    """Return the ContextLayout fields (ir.py:37-60) as numpy arrays.

    Raises ValueError where the reference raises (ir.py:176-178, 240-247, and
    every ``require`` of context_plan.py).
    """
    tokens = _i64(token_ids)
    drops, offsets, ranges = _i32(drop_insert_offsets), _i32(drop_range_offsets), _i32(drop_ranges)
    bounds, inserts = _i32(reposition_raw_boundaries), _i32(reposition_insert_offsets)
    t, e, p = len(tokens), len(drops), len(bounds)
    if len(offsets) != e + 1 or len(ranges) % 2 or len(inserts) != p:
        raise ValueError("Reposition transition-count tensor lengths are inconsistent")
    rcount = len(ranges) // 2
    cap = t + rcount + p
    out = dict(
        positions=np.zeros(t, np.int32), keep_mask=np.zeros(t, np.uint8),
        materialized_stage=np.zeros(t, np.int32), birth_positions=np.zeros(t, np.int32),
        birth_stages=np.zeros(t, np.int32), transition_offsets=np.zeros(p + 1, np.int32),
        effective_reposition_stages=np.zeros(p, np.int32),
        effective_repositions=np.zeros(p, np.uint8), ignored_repositions=np.zeros(p, np.uint8),
        records=np.zeros((cap, 3), np.int32), virtual_mask=np.zeros(cap, np.uint8),
        key_to_token=np.zeros(cap, np.int64), token_to_key=np.zeros(t, np.int64),
        drop_event_to_key=np.zeros(e, np.int64),
    )
    tcap = max(1, t * max(1, p))
    traw, told, tnew = (np.zeros(tcap, np.int32) for _ in range(3))
    ntrans = ctypes.c_int64(0)
    status = np.zeros(5, np.int64)
    rc = lib().akvo_compile_layout(
        ctypes.c_int64(t), _p(tokens), ctypes.c_int64(e), _p(drops), _p(offsets),
        ctypes.c_int64(rcount), _p(ranges), ctypes.c_int64(p), _p(bounds), _p(inserts),
        _p(out["positions"]), _p(out["keep_mask"]), _p(out["materialized_stage"]),
        _p(out["birth_positions"]), _p(out["birth_stages"]), _p(out["transition_offsets"]),
        _p(traw), _p(told), _p(tnew), ctypes.c_int64(tcap), ctypes.byref(ntrans),
        _p(out["effective_reposition_stages"]), _p(out["effective_repositions"]),
        _p(out["ignored_repositions"]), _p(out["records"]), _p(out["virtual_mask"]),
        _p(out["key_to_token"]), _p(out["token_to_key"]), _p(out["drop_event_to_key"]),
        ctypes.c_int64(cap), _p(status),
    )
    if rc == NO_ACTIVE:
        raise ValueError(f"Reposition at raw boundary {int(status[4])} has no active tokens.")
    if rc == TOKEN_RANGE:
        raise ValueError(
            f"Reposition Radix token ID {int(status[4])} is outside the non-negative int32 range."
        )
    if rc != OK:
        raise ValueError(f"invalid Context event program (oracle code {rc})")
    n = ntrans.value
    key_len, stages = int(status[1]), int(status[2])
    out.update(
        transition_raw_tokens=traw[:n].copy(), transition_old_positions=told[:n].copy(),
        transition_new_positions=tnew[:n].copy(),
    )
    out["transition_offsets"] = out["transition_offsets"][: stages + 1]
    for k in ("records", "virtual_mask", "key_to_token"):
        out[k] = out[k][:key_len]
    out["keep_mask"] = out["keep_mask"].astype(bool)
    out["virtual_mask"] = out["virtual_mask"].astype(bool)
    out["effective_repositions"] = out["effective_repositions"].astype(bool)
    out["ignored_repositions"] = out["ignored_repositions"].astype(bool)
    out["next_position"] = int(status[3])
    return out


def decode_layout(layout):
    """ContextDecodeLayout.from_layout (occurrence.py:47-66), host half."""
    raw = np.flatnonzero(layout["keep_mask"]).astype(np.int32)
    positions = layout["positions"][raw].copy()
    if np.any(np.diff(positions.astype(np.int64)) <= 0):
        raise ValueError("Active decode positions must be strictly increasing")
    return raw, positions, len(layout["positions"]), layout["next_position"]


# --------------------------------------------------------------------------
# Drop + Reposition (batched)
# --------------------------------------------------------------------------


def drop_compact(token_counts, range_offsets, ranges, slot_rows, shared_prefix=None,
                 reposition=True, free_ring=None, free_head=0, free_tail=0):
    """Per request r with ``token_counts[r]`` raw tokens born at positions
    0..T-1: drop the half-open ranges ``ranges[range_offsets[r]:range_offsets[r+1]]``
    (pairs, request-local), then Reposition at the last token.

    ``slot_rows[r]`` is the request's req_to_token row (int32 slot ids).
    Tokens below ``shared_prefix[r]`` are borrowed from the radix cache: a
    moved one is copied to a fresh slot popped from ``free_ring`` at
    ``free_head`` (copy-on-write) and the row is updated; a dropped one is not
    freed.  Private moved tokens are rotated in place (source == destination).
    Private dropped tokens' slots are freed, in request then raw order.

    Returns a dict with per-request layouts and flat transition / freed
    vectors in the order the GPU kernel emits them.
    """
    nreq = len(token_counts)
    shared_prefix = np.zeros(nreq, np.int64) if shared_prefix is None else np.asarray(shared_prefix)
    rows = [np.array(r, dtype=np.int32, copy=True) for r in slot_rows]
    res = dict(layouts=[], raw_indices=[], active_positions=[], next_position=[],
               src=[], dst=[], pairs=[], raw=[], freed=[], rows=rows)
    head = free_head
    for r in range(nreq):
        t = int(token_counts[r])
        rr = np.asarray(ranges[2 * range_offsets[r]: 2 * range_offsets[r + 1]], np.int32)
        has_drop = len(rr) > 0
        lay = compile_layout(
            np.zeros(t, np.int64),
            [t] if has_drop else [], [0, len(rr) // 2] if has_drop else [0], rr,
            [t - 1] if (reposition and t > 0) else [], [t] if (reposition and t > 0) else [],
        )
        res["layouts"].append(lay)
        raw, pos, _, nxt = decode_layout(lay)
        res["raw_indices"].append(raw)
        res["active_positions"].append(pos)
        res["next_position"].append(nxt)
        for k in range(len(lay["transition_raw_tokens"])):
            tok = int(lay["transition_raw_tokens"][k])
            src = int(rows[r][tok])
            if tok < shared_prefix[r]:
                dst = int(free_ring[head % len(free_ring)])
                head += 1
                rows[r][tok] = dst
            else:
                dst = src
            res["src"].append(src)
            res["dst"].append(dst)
            res["pairs"].append((int(lay["transition_old_positions"][k]),
                                 int(lay["transition_new_positions"][k])))
            res["raw"].append(tok)
        dropped = np.flatnonzero(~lay["keep_mask"])
        dropped = dropped[dropped >= shared_prefix[r]]
        res["freed"].extend(int(rows[r][i]) for i in dropped)
    res["free_head"] = head
    res["free_tail"] = free_tail + len(res["freed"])
    for k in ("src", "dst", "raw", "freed"):
        res[k] = np.asarray(res[k], np.int32)
    res["pairs"] = np.asarray(res["pairs"], np.int32).reshape(-1, 2)
    return res


def drop_compact_paged(token_counts, range_offsets, ranges, slot_rows, page_size,
                       shared_prefix=None, reposition=True, free_pages=None, free_head=0,
                       free_tail=0):
    """``drop_compact`` over a paged pool (slot = page * page_size + offset,
    token t of a request at offset t % page_size; the reference has no
    paged Reposition, so these rules are this package's contract):

    * a private page (tokens at or after ``shared_prefix[r]``, which is a
      whole number of pages) is freed when every token it holds is
      dropped; its page id is pushed in token order;
    * a shared page that holds a moved token is copied to the next free
      page: every kept token of the page gets a transition to the same
      offset of the new page (old == new position for the tokens before the
      first drop) and every row entry of the page points there afterwards;
    * private moved tokens rotate in place.

    Per request the loop walks pages in token order, exactly as the
    transitions, copies and frees are emitted."""
    nreq = len(token_counts)
    ps = int(page_size)
    shared_prefix = np.zeros(nreq, np.int64) if shared_prefix is None else np.asarray(shared_prefix)
    rows = [np.array(r, dtype=np.int32, copy=True) for r in slot_rows]
    res = dict(raw_indices=[], active_positions=[], next_position=[], src=[], dst=[], pairs=[],
               raw=[], freed=[], rows=rows, copied_pages=0)
    head = free_head
    for r in range(nreq):
        t_count = int(token_counts[r])
        rr = np.asarray(ranges[2 * range_offsets[r]: 2 * range_offsets[r + 1]], np.int64)
        keep = np.ones(t_count, bool)
        for a, b in rr.reshape(-1, 2):
            keep[a:b] = False
        first = int(rr[0]) if len(rr) else t_count
        rank = np.cumsum(keep) - keep  # kept tokens before t
        moved = keep & (np.arange(t_count) > first) & bool(reposition)
        pos = np.where(keep & bool(reposition), rank, np.arange(t_count))
        res["raw_indices"].append(np.flatnonzero(keep).astype(np.int32))
        res["active_positions"].append(pos[keep].astype(np.int32))
        res["next_position"].append(int(keep.sum()) if moved.any() else t_count)
        p_len = int(shared_prefix[r])
        row = rows[r]
        for g0 in range(0, t_count, ps):
            g1 = min(g0 + ps, t_count)
            shared = g0 < p_len
            cow = shared and bool(moved[g0:g1].any())
            if cow:
                new_page = int(free_pages[head % len(free_pages)])
                head += 1
                res["copied_pages"] += 1
            for t in range(g0, g1):
                if keep[t] and (moved[t] or cow):
                    fresh = new_page * ps + t % ps if cow else int(row[t])
                    res["src"].append(int(row[t]))
                    res["dst"].append(fresh)
                    res["pairs"].append((t, int(pos[t])))
                    res["raw"].append(t)
            if cow:
                row[g0:g1] = new_page * ps + np.arange(g0, g1) % ps
            if not shared and not keep[g0:g1].any():
                res["freed"].append(int(row[g0]) // ps)
    res["free_head"] = head
    res["free_tail"] = free_tail + len(res["freed"])
    for k in ("src", "dst", "raw", "freed"):
        res[k] = np.asarray(res[k], np.int32)
    res["pairs"] = np.asarray(res["pairs"], np.int32).reshape(-1, 2)
    return res


# --------------------------------------------------------------------------
# Reposition
# --------------------------------------------------------------------------

_DT = {np.dtype(np.float16): DT_F16, np.dtype(np.float32): DT_F32}


def _dtype_code(a, bf16):
    if bf16:
        assert a.dtype == np.uint16
        return DT_BF16
    return _DT[a.dtype]


def reposition(k_layers, v_layers, source_slots, destination_slots, position_pairs,
               cos_sin_cache, *, is_neox_style=True, skip_unmapped=False, rotary_dim=None,
               bf16=False, cache_bf16=False, threads=1):
    """In-place update of numpy K/V layer arrays shaped [slots, heads, dim].

    bf16 arrays are passed as uint16 bit patterns with ``bf16=True``.
    ``threads`` > 1 splits tokens across a thread pool (the C code releases
    the GIL through ctypes).
    """
    k0 = k_layers[0]
    dtype = _dtype_code(k0, bf16)
    isz = k0.itemsize
    ks0, kh0 = k0.strides[0] // isz, k0.strides[1] // isz
    v0 = v_layers[0]
    vs0, vh0 = v0.strides[0] // isz, v0.strides[1] // isz
    heads, dim = k0.shape[1], k0.shape[2]
    rdim = dim if rotary_dim is None else rotary_dim
    kp = (ctypes.c_void_p * len(k_layers))(*[a.ctypes.data for a in k_layers])
    vp = (ctypes.c_void_p * len(v_layers))(*[a.ctypes.data for a in v_layers])
    src, dst = _i32(source_slots), _i32(destination_slots)
    pairs = _i32(position_pairs).reshape(-1, 2)
    cs = np.ascontiguousarray(cos_sin_cache)
    cs_code = DT_BF16 if cache_bf16 else _DT[cs.dtype]
    n = len(src)

    def run(a, b):
        return lib().akvo_reposition(
            kp, vp, ctypes.c_int32(len(k_layers)), ctypes.c_int32(dtype),
            ctypes.c_int64(ks0), ctypes.c_int64(kh0), ctypes.c_int64(vs0), ctypes.c_int64(vh0),
            ctypes.c_int32(heads), ctypes.c_int32(dim), ctypes.c_int32(rdim),
            ctypes.c_int32(int(is_neox_style)), ctypes.c_int32(int(skip_unmapped)),
            _p(src), _p(dst), _p(pairs), ctypes.c_int64(2), ctypes.c_int64(a), ctypes.c_int64(b),
            _p(cs), ctypes.c_int32(cs_code), ctypes.c_int64(cs.strides[0] // cs.itemsize),
        )

    if threads <= 1 or n < 2 * threads:
        rc = run(0, n)
        if rc != OK:
            raise ValueError("Reposition requires a native cos/sin cache matching rotary_dim")
        return
    bounds = np.linspace(0, n, threads + 1).astype(np.int64)
    with ThreadPoolExecutor(threads) as pool:
        rcs = list(pool.map(run, bounds[:-1], bounds[1:]))
    if any(rc != OK for rc in rcs):
        raise ValueError("Reposition requires a native cos/sin cache matching rotary_dim")


# --------------------------------------------------------------------------
# Page table
# --------------------------------------------------------------------------


class HostRegistry:
    """Host twin of ContextDecodeRegistry.rows (context_backend.py:680-684).

    Each row is six int64 cells; the pointer cells hold host addresses of
    numpy arrays kept alive by this object.
    """

    def __init__(self, max_rows):
        self.rows = np.zeros((max_rows, 6), np.int64)
        self._keep = []

    def set_context(self, row, raw_ids, positions, prompt_len, next_pos, row_array=None):
        raw_ids, positions = _i32(raw_ids), _i32(positions)
        active = len(raw_ids)
        if active == 0:
            raw_ids = np.zeros(1, np.int32)  # non-null marker (occurrence.py:56-58)
            positions = raw_ids
        self._keep += [raw_ids, positions]
        rp = 0
        if row_array is not None:
            row_array = _i32(row_array)
            self._keep.append(row_array)
            rp = row_array.ctypes.data
        self.rows[row] = (raw_ids.ctypes.data, positions.ctypes.data, prompt_len, active,
                          next_pos, rp)

    def set_ordinary(self, row):
        self.rows[row] = 0


def decode_indices(registry, table, row_ids, lengths, indptr, output_len, starts=None,
                   mapping=None, multiplier=1):
    table = _i32(table)
    out = np.zeros(output_len, np.int64)
    row_ids, lengths, indptr = _i64(row_ids), _i64(lengths), _i64(indptr)
    st = None if starts is None else _i64(starts)
    mp = None if mapping is None else _i64(mapping)
    lib().akvo_decode_indices(
        _p(registry.rows), _p(table), ctypes.c_int64(table.shape[1]), _p(row_ids), _p(lengths),
        _p(indptr), _p(out), _p(st), _p(mp), ctypes.c_int64(multiplier),
        ctypes.c_int64(len(row_ids)),
    )
    return out


def window_lengths(registry, row_ids, lengths, window):
    row_ids, lengths = _i64(row_ids), _i64(lengths)
    out = np.zeros(len(row_ids), np.int64)
    lib().akvo_window_lengths(_p(registry.rows), _p(row_ids), _p(lengths), _p(out),
                              ctypes.c_int64(window), ctypes.c_int64(len(row_ids)))
    return out


def window_lengths_cpu(batch_layouts, window, batch_size):
    """context_backend.py:742-752: (positions, next_position) or None rows."""
    lengths = []
    for layout, generated in batch_layouts:
        if layout is None:
            lengths.append(min(generated, window + 1))
        else:
            positions, next_position = layout
            lower = next_position + generated - 1 - window
            start = np.searchsorted(positions, lower)
            lengths.append(len(positions) - start + min(generated, window + 1))
    return np.asarray(lengths + [1] * (batch_size - len(lengths)), np.int64)


def write_row_slots(row_arrays, rows, columns, values):
    ptrs = _i64([a.ctypes.data for a in row_arrays])
    rows, columns, values = _i64(rows), _i64(columns), _i64(values)
    lib().akvo_write_row_slots(_p(ptrs), _p(rows), _p(columns), _p(values),
                               ctypes.c_int64(len(rows)))


# --------------------------------------------------------------------------
# Decode attention
# --------------------------------------------------------------------------


def decode_attention(q, k_pool, v_pool, kv_indptr, kv_indices, sinks=None, scale=None):
    """Paged GQA decode in float64.

    q: [bs, Hq, D]; k_pool/v_pool: [slots, Hkv, D]; keys of request b are
    ``kv_indices[kv_indptr[b]:kv_indptr[b+1]]``.  With ``sinks`` ([Hq] natural
    log logits) the output is multiplied by sigmoid(lse - sink), i.e. the sink
    is an extra softmax column whose value row is zero
    (context_backend.py:266-268).  Returns (out [bs, Hq, D], lse [bs, Hq]).
    Empty key sets give zero output and lse = -inf.
    """
    q = np.asarray(q, np.float64)
    bs, hq, d = q.shape
    hkv = k_pool.shape[1]
    group = hq // hkv
    scale = 1.0 / np.sqrt(d) if scale is None else scale
    out = np.zeros((bs, hq, d))
    lse = np.full((bs, hq), -np.inf)
    for b in range(bs):
        idx = np.asarray(kv_indices[kv_indptr[b]: kv_indptr[b + 1]], np.int64)
        if len(idx) == 0:
            continue
        k = np.asarray(k_pool[idx], np.float64)  # [n, Hkv, D]
        v = np.asarray(v_pool[idx], np.float64)
        for h in range(hq):
            g = h // group
            s = (k[:, g, :] @ q[b, h]) * scale
            m = s.max()
            w = np.exp(s - m)
            tot = w.sum()
            out[b, h] = (w @ v[:, g, :]) / tot
            lse[b, h] = m + np.log(tot)
    if sinks is not None:
        sig = 1.0 / (1.0 + np.exp(-(lse - np.asarray(sinks, np.float64)[None, :])))
        sig = np.where(np.isfinite(lse), sig, 0.0)
        out = out * sig[:, :, None]
    return out, lse


def prefill_attention(q, k_pool, v_pool, qo_indptr, kv_indptr, kv_indices, birth_slots,
                      q_positions, kv_positions, sinks=None, window=-1, scale=None):
    """Ragged prefill attention with context positions, in float64.

    Follows the reference's position-aware extend mask (sglang.patch:524-541,
    725-741; ContextAttentionMetadata.native_plan, context_backend.py:184-222):
    request b's keys are its prefix (kv_indices / kv_positions at
    kv_indptr[b]..) followed by its new tokens (birth_slots / q_positions at
    qo_indptr[b]..); query i sees prefix key j when window < 0 or
    q_pos - k_pos <= window, and new-token key j when also j <= i.  The sink
    multiplies the output by sigmoid(lse - sink) (context_backend.py:266-268).
    Returns (out [tokens, Hq, D], lse [tokens, Hq]).
    """
    q = np.asarray(q, np.float64)
    n, hq, d = q.shape
    hkv = k_pool.shape[1]
    group = hq // hkv
    scale = 1.0 / np.sqrt(d) if scale is None else scale
    out = np.zeros((n, hq, d))
    lse = np.full((n, hq), -np.inf)
    for b in range(len(qo_indptr) - 1):
        a, e = int(qo_indptr[b]), int(qo_indptr[b + 1])
        x, y = int(kv_indptr[b]), int(kv_indptr[b + 1])
        slots = np.concatenate((np.asarray(kv_indices[x:y], np.int64),
                                np.asarray(birth_slots[a:e], np.int64)))
        kpos = np.concatenate((np.asarray(kv_positions[x:y], np.int64),
                               np.asarray(q_positions[a:e], np.int64)))
        if len(slots) == 0:
            continue
        k = np.asarray(k_pool[slots], np.float64)
        v = np.asarray(v_pool[slots], np.float64)
        p_count = y - x
        j = np.arange(len(slots))
        for i in range(e - a):
            qp = int(q_positions[a + i])
            vis = (j < p_count) | (j - p_count <= i)
            if window is not None and window >= 0:
                vis &= qp - kpos <= window
            for h in range(hq):
                s = (k[vis, h // group, :] @ q[a + i, h]) * scale
                mx = s.max()
                wgt = np.exp(s - mx)
                tot = wgt.sum()
                out[a + i, h] = (wgt @ v[vis, h // group, :]) / tot
                lse[a + i, h] = mx + np.log(tot)
    if sinks is not None:
        sig = 1.0 / (1.0 + np.exp(-(lse - np.asarray(sinks, np.float64)[None, :])))
        sig = np.where(np.isfinite(lse), sig, 0.0)
        out = out * sig[:, :, None]
    return out, lse


# --------------------------------------------------------------------------
# Active-slot gather (offload / load / PD transfer)
# --------------------------------------------------------------------------


def active_slot_ranges(raw_indices, positions, prompt_length, next_position, raw_end,
                       window=None):
    """(start, generated_start) of srt/disaggregation/context_transfer.py:116-122:
    the first decode-view entry a sliding window still reads and the first
    generated raw position it reads."""
    start = 0
    generated_start = int(prompt_length)
    if window is not None:
        lower = int(next_position) + int(raw_end) - int(prompt_length) - int(window)
        start = int(np.searchsorted(np.asarray(positions), lower))
        generated_start += max(0, lower - int(next_position))
    return start, generated_start


def active_slots(row, raw_indices, positions, prompt_length, next_position, raw_end,
                 window=None):
    """context_transfer.py:110-128: row[raw_indices[start:]] followed by
    row[generated_start:raw_end] (int32)."""
    row = np.asarray(row)
    start, generated_start = active_slot_ranges(raw_indices, positions, prompt_length,
                                                next_position, raw_end, window)
    prefix = row[np.asarray(raw_indices, np.int64)[start:]]
    tail = row[generated_start:int(raw_end)]
    return np.concatenate((prefix, tail)).astype(np.int32)


def active_lengths(raw_indices, positions, prompt_length, next_position, raw_end, window):
    """context_transfer.py:131-138: (full active length, windowed length)."""
    generated = max(0, int(raw_end) - int(prompt_length))
    full = len(raw_indices) + generated
    lower = int(next_position) + generated - int(window)
    start = int(np.searchsorted(np.asarray(positions), lower))
    return full, len(raw_indices) - start + min(generated, int(window))


def gather_slots(words, n_tasks, n_chunks, memory, chunk):
    """The contract of ``akv_gather_slots`` (include/akv_b200.h) executed on
    the CPU over a packed program: ``memory`` maps each address in the task
    table to a writable numpy vector.  Returns how many times each output
    element was written (every element must be written exactly once)."""
    words = np.asarray(words, np.int64)
    table = words[: 12 * n_tasks].reshape(n_tasks, 12)
    chunks = words[12 * n_tasks: 12 * n_tasks + n_chunks].view(np.int32).reshape(-1, 2)
    indices = words[12 * n_tasks + n_chunks:].view(np.int32)
    writes = {t: np.zeros(int(table[t, 1]), np.int64) for t in range(n_tasks)}
    for task, first in chunks:
        first_idx, n, out_addr, flags = (int(x) for x in table[task, :4])
        n_seg = (flags >> 8) & 0xFF
        ends = [int(e) for e in table[task, 8:8 + n_seg]]
        segs = [memory[int(a)] if e > b else None
                for a, e, b in zip(table[task, 4:4 + n_seg], ends, [0] + ends[:-1])]
        out = memory[out_addr]
        for k in range(first, min(first + chunk, n)):
            v = int(indices[first_idx + k])
            if not flags & 2:
                if v < 0:
                    v = -1
                else:
                    s = next((i for i, e in enumerate(ends) if v < e), None)
                    if s is None:
                        raise IndexError("slot gather index past its segments")
                    v = int(segs[s][v - (ends[s - 1] if s else 0)])
            out[k] = np.int64(v).astype(out.dtype)  # int32: the low 32 bits
            writes[task][k] += 1
    return writes


def occurrence_advance(state, window, plan, query_slots, extra_slots, visible_until):
    """srt/context_system/occurrence.py:644-755 (``OccurrenceState.advance``)
    over numpy dicts: ``state`` holds slots, owned, canonical_rows,
    terminal_rows, canonical_positions, exact_prefix_len and optionally
    swa_resident; ``window`` and ``plan`` hold the fields of
    ``OccurrenceWindow`` / ``OccurrenceMaterialization``.  Returns the
    advance's fields and the successor state as numpy values."""
    n = len(window["birth_occurrences"])
    start, end = len(state["canonical_rows"]), len(plan["terminal_occurrences"])
    n_old, n_q = len(state["slots"]), len(query_slots)
    all_slots = np.concatenate((state["slots"], query_slots, extra_slots))
    all_owned = np.r_[state["owned"], np.ones(n_q + len(extra_slots), bool)]
    canonical = np.full(n, -1, np.int64)
    canonical[:start] = state["canonical_rows"]
    canonical[start:end] = np.arange(n_old, n_old + n_q)
    terminal = np.full(n, -1, np.int64)
    terminal[:start] = state["terminal_rows"]
    source_rows = np.r_[canonical, terminal]
    rows = plan["source_rows"]
    occurrences = np.full(len(rows), -1, np.int64)
    occurrences[rows >= 0] = source_rows[rows[rows >= 0]]
    occurrences[plan["allocated_occurrences"]] = np.arange(n_old + n_q, len(all_slots))
    copy_rows = source_rows[plan["copy_source_rows"]]
    swa = state.get("swa_resident")
    unused = None
    if swa is not None:
        swa = np.r_[swa, np.ones(n_q + len(extra_slots), bool)]
        dst = occurrences[plan["copy_occurrences"]]
        swa[dst] = swa[copy_rows]
        unused = dst[~swa[dst]]
    picked = plan["terminal_occurrences"]
    kept = picked >= 0
    terminal = np.full(end, -1, np.int64)
    terminal[kept] = occurrences[picked[kept]]
    pos = window["occurrence_positions"]
    positions = pos[window["birth_occurrences"][:end]].copy()
    positions[:start] = state["canonical_positions"]
    same = positions == pos[window["terminal_occurrences"][:end]]
    canonical = np.where(kept & same, terminal, canonical[:end])
    future = visible_until[:end] > end
    if end == n:
        future[:] = False
    canonical = np.where(future, canonical, -1)
    retained = np.unique(np.r_[canonical[canonical >= 0], terminal[terminal >= 0]])
    live = np.zeros(len(all_slots), bool)
    live[retained] = True
    retired = np.flatnonzero(all_owned & ~live)
    remap = np.full(len(all_slots), -1, np.int64)
    remap[retained] = np.arange(len(retained))
    next_canonical = np.full(end, -1, np.int64)
    next_canonical[canonical >= 0] = remap[canonical[canonical >= 0]]
    next_terminal = np.full(end, -1, np.int64)
    next_terminal[kept] = remap[terminal[kept]]
    out = {
        "occurrence_slots": all_slots[np.maximum(occurrences, 0)],
        "copy_source_slots": all_slots[copy_rows].astype(np.int32),
        "copy_destination_slots":
            all_slots[occurrences[plan["copy_occurrences"]]].astype(np.int32),
        "copy_position_pairs": np.asarray(plan["copy_position_pairs"]).reshape(-1, 2)
        .astype(np.int32),
        "retired_slots": all_slots[retired],
        "successor": {
            "slots": all_slots[retained], "owned": all_owned[retained],
            "canonical_rows": next_canonical, "terminal_rows": next_terminal,
            "canonical_positions": positions, "exact_prefix_len": state["exact_prefix_len"],
        },
    }
    if swa is not None:
        out["unused_swa_slots"] = all_slots[unused]
        out["retired_swa_resident"] = swa[retired]
        out["successor"]["swa_resident"] = swa[retained]
    return out


def occurrence_bind(plan, canonical_slots, terminal_slots, allocated_slots):
    """srt/context_system/occurrence.py:315-357 (``OccurrenceMaterialization.bind``):
    (slots, copy sources int32, copy destinations int32, pairs int32 [k, 2])."""
    rows = plan["source_rows"]
    sources = np.r_[canonical_slots, terminal_slots]
    slots = np.full(len(rows), -1, np.asarray(canonical_slots).dtype)
    reused = np.flatnonzero(rows >= 0)
    slots[reused] = sources[rows[reused]]
    slots[plan["allocated_occurrences"]] = allocated_slots
    return (slots, sources[plan["copy_source_rows"]].astype(np.int32),
            slots[plan["copy_occurrences"]].astype(np.int32),
            np.asarray(plan["copy_position_pairs"]).reshape(-1, 2).astype(np.int32))


def terminal_slots(slots, terminal_rows):
    """srt/context_system/occurrence.py:757-768: slots[terminal_rows], -1 at holes."""
    rows = np.asarray(terminal_rows)
    out = np.full(len(rows), -1, np.asarray(slots).dtype)
    present = rows >= 0
    out[present] = np.asarray(slots)[rows[present]]
    return out
