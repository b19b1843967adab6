"""Generate tests/golden/cow.npz: which tokens the REFERENCE copies when a
request with a radix-shared prefix drops spans and repositions, from the
reference's own ownership code (srt/context_system/occurrence.py), so that
the copy-on-write selection of ``DropCompactor`` is pinned to it.

Every case is c3-shaped, scaled down: a prompt of T tokens whose first P
were matched in the radix cache (borrowed, ``exact_prefix_len = P``), a
Drop at insertion T whose first range starts inside the first half of the
prefix, a Reposition at raw boundary T - 1, then the next turn's q new
tokens.  The scheduler's sequence (akv/system/sglang.patch:2894-2933,
:3133-3180) is driven on the CPU:

1. ``compile_context_layout`` over all T + q tokens (the reference's C++);
2. ``OccurrenceState.from_match`` with the P matched slots;
3. forward 1: queries [P, T) -- the private prompt tokens, born before the
   Drop -- planned (``prefill_terminal_keep``, ``plan``) and admitted
   (``advance``) with fresh query slots;
4. forward 2: queries [T, T + q) after the Drop + Reposition; its plan's
   copies (raw tokens, position pairs, source slots) and the slots that its
   ``advance`` retires are recorded, with those that forward 1 retired.

    python tests/golden/make_cow_golden.py

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
from make_occurrence_golden import visible_until  # noqa: E402


def c3_like_case(rng, tokens, prefix, new):
    """Drop spans of a c3 request (about 10-60 % of the prompt, the first
    starting in [0, prefix / 2)) as the reference's program inputs."""
    frac = rng.uniform(0.1, 0.6)
    total = max(1, int(round(frac * tokens)))
    count = max(1, -(-total // 256))
    lengths = np.maximum(1, np.round(rng.uniform(1, 512, size=count) *
                                     (total / max(1.0, count * 256.0))).astype(np.int64))
    first = int(rng.integers(0, max(1, prefix // 2)))
    spans = [(first, first + int(lengths[0]))]
    cursor = spans[0][1]
    for length in lengths[1:]:
        gap = int(rng.integers(1, 200))
        s, e = cursor + gap, cursor + gap + int(length)
        if e > tokens:
            break
        spans.append((s, e))
        cursor = e
    ranges = np.asarray([x for s in spans for x in s], np.int32)
    n = tokens + new
    return dict(
        token_ids=rng.integers(0, 2**31, size=n).astype(np.int64),
        drop_insert_offsets=np.asarray([tokens], np.int32),
        drop_range_offsets=np.asarray([0, len(spans)], np.int32),
        drop_ranges=ranges,
        reposition_raw_boundaries=np.asarray([tokens - 1], np.int32),
        reposition_insert_offsets=np.asarray([tokens], np.int32),
    )


def run_case(occ, ir, rng, tokens, prefix, new):
    inp = c3_like_case(rng, tokens, prefix, new)
    lay = ir.compile_context_layout(*(mg._t(inp[k]) for k in mg.INPUT_FIELDS))
    n = len(lay.positions)
    vis = torch.from_numpy(visible_until(inp, n))
    slot_pool = rng.permutation(10**6)[: n + 10000].astype(np.int64) + 1
    cursor = [0]

    def fresh(count):
        s = torch.from_numpy(slot_pool[cursor[0]: cursor[0] + count].copy())
        cursor[0] += count
        return s

    # The matched prefix was written by another request at its birth
    # positions (0..P-1), as a radix cache holds it.
    prefix_slots = fresh(prefix)
    state = occ.OccurrenceState.from_match(
        prefix_slots, lay.birth_positions[:prefix].clone().to(torch.int32),
        exact_prefix_len=prefix)
    out = {}
    for k, (qs, qe) in enumerate(((prefix, tokens), (tokens, n))):
        window = occ.compile_occurrence_window(lay, vis, lay.positions, query_start=qs,
                                               query_end=qe)
        keep = state.prefill_terminal_keep(lay, qe)
        plan = state.plan(window, keep)
        query_slots, extra_slots = fresh(qe - qs), fresh(plan.extra_page_count)
        step = state.advance(window, plan, query_slots, extra_slots, vis)
        if k == 0:
            out["row"] = torch.cat((prefix_slots, query_slots)).numpy().astype(np.int32)
            out["forward1_extra"] = np.asarray(plan.extra_page_count, np.int64)
            # dropped private tokens: no later query reads them
            out["forward1_retired_slots"] = step.retired_slots.numpy().astype(np.int64)
        else:
            raw = window.occurrence_raw_tokens.numpy()
            out["copy_raw"] = raw[plan.copy_occurrences.numpy()].astype(np.int32)
            out["copy_pairs"] = plan.copy_position_pairs.numpy().astype(np.int32)
            out["copy_source_slots"] = step.copy_source_slots.numpy().astype(np.int32)
            out["retired_slots"] = step.retired_slots.numpy().astype(np.int64)
        state = step.state
    out.update(tokens=np.asarray(tokens, np.int64), prefix=np.asarray(prefix, np.int64),
               new=np.asarray(new, np.int64), ranges=inp["drop_ranges"])
    return out


def main():
    ir = mg.reference_modules()[0]
    occ = mg._load("akv_ref_occurrence", f"{mg.SG}/srt/context_system/occurrence.py")
    rng = np.random.default_rng(20261203)
    shapes = [(600, 160, 1), (1200, 400, 7), (2000, 1024, 3), (3000, 1500, 16),
              (900, 64, 2), (4096, 2048, 5), (2500, 1000, 1), (1800, 700, 9)]
    out, names = {}, []
    for i, (tokens, prefix, new) in enumerate(shapes):
        case = run_case(occ, ir, rng, tokens, prefix, new)
        name = f"case{i}"
        for key, value in case.items():
            out[f"{name}/{key}"] = value
        names.append(name)
        print(f"{name}: T={tokens} P={prefix}: {len(case['copy_raw'])} copies, "
              f"{len(case['retired_slots'])} retired, forward-1 extras {case['forward1_extra']}")
    out["cases"] = np.asarray(names)
    path = os.path.join(HERE, "cow.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}")


if __name__ == "__main__":
    main()
