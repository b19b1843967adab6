"""Generate tests/golden/occurrence.npz by running the REFERENCE's occurrence
ownership code on the CPU:

* ``compile_context_layout`` (srt/context_system/ir.py:113-274) over the
  reference's C++ event compiler, as make_golden.py builds it;
* ``OccurrenceState.from_match / prefill_terminal_keep / plan / advance /
  terminal_slots``, ``compile_occurrence_window`` and
  ``OccurrenceMaterialization.bind`` (srt/context_system/occurrence.py),
  driven the way the scheduler drives them for a request prefilled in
  several chunks (akv/system/sglang.patch:2894-2933 plans a chunk,
  :3133-3180 admits it and calls ``advance``).

Each program is prefilled in 1-4 chunks, from nothing or from a matched
prefix (optionally with non-resident tokens and SWA residency).  Query and
extra slots are synthetic distinct slot numbers.  Every ``advance`` call
records its inputs and outputs; every plan records a ``bind``.

    python tests/golden/make_occurrence_golden.py

Nothing here is needed at test time: the tests read the .npz file only.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import make_golden as mg  # noqa: E402

STATE = ("slots", "owned", "canonical_rows", "terminal_rows", "canonical_positions")
WINDOW = ("occurrence_raw_tokens", "occurrence_positions", "birth_occurrences",
          "terminal_occurrences", "segment_query_starts", "segment_query_ends",
          "segment_key_offsets", "segment_key_occurrences")
PLAN = ("source_rows", "allocated_occurrences", "copy_occurrences", "copy_source_rows",
        "copy_position_pairs", "terminal_occurrences", "read_cached", "repositioned_cached")
ADVANCE = ("occurrence_slots", "copy_source_slots", "copy_destination_slots",
           "copy_position_pairs", "retired_slots", "unused_swa_slots", "retired_swa_resident")


def visible_until(inp, n):
    """Earliest insertion offset of a drop range covering each raw token
    (srt/context_system/planner.py:167-181), int32 max when never dropped."""
    out = np.full(n, np.iinfo(np.int32).max, np.int32)
    ins, offs, rng = inp["drop_insert_offsets"], inp["drop_range_offsets"], inp["drop_ranges"]
    for e, pos in enumerate(ins):
        for r in range(int(offs[e]), int(offs[e + 1])):
            s, t = int(rng[2 * r]), int(rng[2 * r + 1])
            out[s:t] = np.minimum(out[s:t], pos)
    return out


def record_state(out, key, st):
    for f in STATE:
        out[f"{key}/{f}"] = getattr(st, f).numpy()
    out[f"{key}/exact_prefix_len"] = np.asarray(st.exact_prefix_len, np.int64)
    if st.swa_resident is not None:
        out[f"{key}/swa_resident"] = st.swa_resident.numpy()


def run_case(occ, ir, out, name, rng, inp, chunks, match, dtype):
    lay = ir.compile_context_layout(*(mg._t(inp[k]) for k in mg.INPUT_FIELDS))
    n = len(lay.positions)
    vis = torch.from_numpy(visible_until(inp, n))
    m = match.get("length", 0)
    next_slot = [1000]

    def fresh(count):
        s = torch.arange(next_slot[0], next_slot[0] + count, dtype=dtype)
        next_slot[0] += count + int(rng.integers(0, 50))
        return s

    positions = (lay.birth_positions if match.get("birth") else lay.positions)[:m].clone()
    resident = None
    if match.get("holes"):
        # tokens no query at or after m can read and the policy never publishes
        resident = torch.from_numpy(~((vis.numpy()[:m] <= m) & ~lay.keep_mask.numpy()[:m]))
    swa = torch.from_numpy(rng.random(m) < 0.7) if match.get("swa") else None
    state = occ.OccurrenceState.from_match(
        fresh(m), positions.to(torch.int32), exact_prefix_len=match.get("exact", m),
        resident=resident, swa_resident=swa)
    bounds = sorted(set(int(x) for x in rng.integers(m + 1, n, size=chunks - 1))) if n - m > 1 \
        else []
    ends = [b for b in bounds if b > m] + [n]
    out[f"{name}/n"] = np.asarray(n, np.int64)
    out[f"{name}/visible_until"] = vis.numpy()
    out[f"{name}/steps"] = np.asarray(len(ends), np.int64)
    for k, qe in enumerate(ends):
        key = f"{name}/{k}"
        start = len(state.canonical_rows)
        window = occ.compile_occurrence_window(lay, vis, lay.positions, query_start=start,
                                               query_end=qe)
        keep = state.prefill_terminal_keep(lay, qe)
        plan = state.plan(window, keep)
        query_slots, extra_slots = fresh(qe - start), fresh(plan.extra_page_count)
        record_state(out, f"{key}/state", state)
        for f in WINDOW:
            out[f"{key}/window/{f}"] = getattr(window, f).numpy()
        for f in PLAN:
            out[f"{key}/plan/{f}"] = getattr(plan, f).numpy()
        out[f"{key}/query_slots"] = query_slots.numpy()
        out[f"{key}/extra_slots"] = extra_slots.numpy()
        # bind over synthetic canonical / terminal slot vectors
        cs = torch.from_numpy(rng.permutation(10**6)[:n].astype(np.int64)).to(dtype)
        ts = torch.from_numpy(rng.permutation(10**6)[:n].astype(np.int64)).to(dtype)
        b = plan.bind(cs, ts, extra_slots)
        out[f"{key}/bind/canonical_slots"] = cs.numpy()
        out[f"{key}/bind/terminal_slots"] = ts.numpy()
        for f, v in zip(("slots", "copy_source_slots", "copy_destination_slots",
                         "copy_position_pairs"), b):
            out[f"{key}/bind/{f}"] = v.numpy()
        step = state.advance(window, plan, query_slots, extra_slots, vis)
        for f in ADVANCE:
            v = getattr(step, f)
            if v is not None:
                out[f"{key}/advance/{f}"] = v.numpy()
        state = step.state
        record_state(out, f"{key}/successor", state)
        out[f"{key}/terminal_slots"] = state.terminal_slots().numpy()


def main():
    ir = mg.reference_modules()[0]
    occ = mg._load("akv_ref_occurrence", f"{mg.SG}/srt/context_system/occurrence.py")
    rng = np.random.default_rng(20261202)
    out, names = {}, []
    plans = [
        (40, 1, {}), (40, 3, {}), (200, 2, {}), (200, 4, {"length": 50}),
        (900, 3, {"length": 300, "birth": True}), (900, 2, {"length": 400, "swa": True}),
        (1500, 4, {"length": 700, "holes": True, "exact": 500}),
        (1500, 3, {"length": 200, "holes": True, "swa": True, "birth": True, "exact": 0}),
        (300, 4, {"length": 120, "swa": True, "exact": 60}),
    ]
    for i, (t, chunks, match) in enumerate(plans):
        for dtype in (torch.int64, torch.int32) if i % 3 == 0 else (torch.int64,):
            name = f"case{len(names)}"
            inp = mg.random_program(rng, t)
            try:
                run_case(occ, ir, out, name, rng, inp, chunks, match, dtype)
            except ValueError as exc:
                print(f"{name}: skipped ({exc})")
                out = {k: v for k, v in out.items() if not k.startswith(f"{name}/")}
                continue
            names.append(name)
    out["cases"] = np.asarray(names)
    path = os.path.join(HERE, "occurrence.npz")
    np.savez_compressed(path, **out)
    steps = sum(int(out[f"{c}/steps"]) for c in names)
    print(f"wrote {path}: {len(names)} programs, {steps} advances")


if __name__ == "__main__":
    main()
