"""Occurrence ownership on the host (no GPU): the oracle against the
reference's golden vectors, and the host half of ``context_occurrence``
(every ownership decision and the packed gather program) executed by the
oracle's restatement of the ``akv_gather_slots`` contract.

Golden: tests/golden/occurrence.npz, made by make_occurrence_golden.py from
the reference's OccurrenceState / compile_occurrence_window /
OccurrenceMaterialization (srt/context_system/occurrence.py)."""

from __future__ import annotations

import dataclasses

import numpy as np
import pytest
import torch

from occurrence_cases import (ADVANCE, PLAN, WINDOW, Plan, State, as_numpy,
                              check_advance, golden, np_state, steps, torch_state, window_plan)

def test_golden_covers_the_ownership_paths():
    z = golden()
    cases = list(steps(z))
    assert len(cases) >= 30
    copies = sum(len(z[f"{c}/{k}/plan/copy_occurrences"]) for c, k in cases)
    retired = sum(len(z[f"{c}/{k}/advance/retired_slots"]) for c, k in cases)
    unused = sum(len(z[f"{c}/{k}/advance/unused_swa_slots"]) for c, k in cases
                 if f"{c}/{k}/advance/unused_swa_slots" in z)
    dtypes = {str(z[f"{c}/{k}/query_slots"].dtype) for c, k in cases}
    assert copies > 0 and retired > 0 and unused > 0 and dtypes == {"int32", "int64"}


def test_oracle_matches_the_reference_advance():
    from oracle import oracle

    z = golden()
    for c, k in steps(z):
        key = f"{c}/{k}"
        got = oracle.occurrence_advance(
            np_state(z, f"{key}/state"),
            {f: z[f"{key}/window/{f}"] for f in WINDOW},
            {f: z[f"{key}/plan/{f}"] for f in PLAN},
            z[f"{key}/query_slots"], z[f"{key}/extra_slots"], z[f"{c}/visible_until"])
        check_advance(got, z, key)
        succ = np_state(z, f"{key}/successor")
        np.testing.assert_array_equal(
            oracle.terminal_slots(succ["slots"], succ["terminal_rows"]),
            z[f"{key}/terminal_slots"])


def test_oracle_matches_the_reference_bind():
    from oracle import oracle

    z = golden()
    for c, k in steps(z):
        key = f"{c}/{k}"
        got = oracle.occurrence_bind({f: z[f"{key}/plan/{f}"] for f in PLAN},
                                     z[f"{key}/bind/canonical_slots"],
                                     z[f"{key}/bind/terminal_slots"], z[f"{key}/extra_slots"])
        for f, v in zip(("slots", "copy_source_slots", "copy_destination_slots",
                         "copy_position_pairs"), got):
            want = z[f"{key}/bind/{f}"]
            assert v.dtype == want.dtype
            np.testing.assert_array_equal(v, want, err_msg=f"{key} bind {f}")


def run_on_host(gather):
    """Execute a queued SlotGather with the oracle; every output element
    must be written exactly once."""
    from akv_b200 import _native
    from oracle import oracle

    memory = {}
    for out, _, segments, _ in gather._tasks:
        for t in (out, *segments):
            if t.numel():
                memory[t.data_ptr()] = t.numpy()
    words, n_tasks, n_chunks = gather.pack()
    writes = oracle.gather_slots(words, n_tasks, n_chunks, memory,
                                 int(_native.lib.akv_gather_slots_chunk()))
    for t, w in writes.items():
        assert np.all(w == 1), f"task {t} elements written {set(w.tolist())} times"


def host_advance(state, window, plan, query, extra, vis):
    from akv_b200 import context_occurrence as co

    p = co._AdvancePlan(state, window, plan, query, extra, vis)
    occ = torch.empty(len(p.occurrences), dtype=p.dtype)
    i32 = torch.empty(len(p.copy_src) + len(p.copy_dst) + len(p.pairs), dtype=torch.int32)
    a, b = len(p.copy_src), len(p.copy_src) + len(p.copy_dst)
    gather = co.SlotGather("cpu")
    res = p.add_tasks(gather, occ, i32[:a], i32[a:b], i32[b:])
    run_on_host(gather)
    return res


def test_host_advance_program_matches_the_reference_chain():
    """Each request's whole prefill, chained through this module's own
    successors: only the first state comes from the fixture."""
    z = golden()
    for c in z["cases"]:
        c = str(c)
        vis = torch.from_numpy(z[f"{c}/visible_until"])
        state = torch_state(z, f"{c}/0/state")
        for k in range(int(z[f"{c}/steps"])):
            key = f"{c}/{k}"
            window, plan = window_plan(z, key)
            res = host_advance(state, window, plan, torch.from_numpy(z[f"{key}/query_slots"]),
                               torch.from_numpy(z[f"{key}/extra_slots"]), vis)
            assert type(res.state) is State
            check_advance(as_numpy(res), z, key)
            state = res.state


def test_host_batch_program_matches_the_reference():
    """Every request's step k (and ordinary requests between them) in one
    program; the concatenations are the scheduler's torch.cat of the
    per-request results."""
    from akv_b200 import context_occurrence as co

    z = golden()
    gen = torch.Generator().manual_seed(5)
    for k in range(2):
        batch = co.OccurrenceBatch("cpu")
        keys, ordinary = [], []
        for i, c in enumerate(z["cases"]):
            key = f"{c}/{k}"
            if k >= int(z[f"{c}/steps"]):
                continue
            if i % 3 == 1:
                pre = torch.randint(0, 10**6, (int(i * 7),), generator=gen)
                birth = torch.randint(0, 10**6, (5,), generator=gen)
                batch.add_ordinary(pre, birth)
                ordinary.append((len(keys), pre, birth))
            q = torch.from_numpy(z[f"{key}/query_slots"]).to(torch.int64)
            e = torch.from_numpy(z[f"{key}/extra_slots"]).to(torch.int64)
            st = torch_state(z, f"{key}/state")
            st = dataclasses.replace(st, slots=st.slots.to(torch.int64))
            window, plan = window_plan(z, key)
            batch.add_context(st, window, plan, q, e, torch.from_numpy(z[f"{c}/visible_until"]))
            keys.append(key)
        gather, (advances, slots, src, dst, pairs) = batch._queue()
        assert len(ordinary) >= 2
        run_on_host(gather)
        want_slots, want_src, want_dst, want_pairs = [], [], [], []
        ctx = [a for a in advances if a is not None]
        assert len(ctx) == len(keys)
        j = 0
        for a in advances:
            if a is None:
                _, pre, birth = next(o for o in ordinary if o[0] == j)
                want_slots.append(torch.cat((pre, birth)).numpy())
                continue
            key = keys[j]
            got = as_numpy(a)
            for f in ADVANCE:
                want = z[f"{key}/advance/{f}"]
                np.testing.assert_array_equal(got[f], want.astype(got[f].dtype))
            want_slots.append(z[f"{key}/advance/occurrence_slots"].astype(np.int64))
            want_src.append(z[f"{key}/advance/copy_source_slots"])
            want_dst.append(z[f"{key}/advance/copy_destination_slots"])
            want_pairs.append(z[f"{key}/advance/copy_position_pairs"].reshape(-1, 2))
            j += 1
        np.testing.assert_array_equal(slots.numpy(), np.concatenate(want_slots))
        np.testing.assert_array_equal(src.numpy(), np.concatenate(want_src))
        np.testing.assert_array_equal(dst.numpy(), np.concatenate(want_dst))
        np.testing.assert_array_equal(pairs.numpy(), np.concatenate(want_pairs))


def test_host_bind_and_terminal_programs_match_the_reference():
    from akv_b200 import context_occurrence as co

    z = golden()
    for c, k in steps(z):
        key = f"{c}/{k}"
        _, plan = window_plan(z, key)
        p = co.SlotGather("cpu")
        # the index composition of bind, executed on the host
        cs = torch.from_numpy(z[f"{key}/bind/canonical_slots"])
        ts = torch.from_numpy(z[f"{key}/bind/terminal_slots"])
        al = torch.from_numpy(z[f"{key}/extra_slots"])
        rows = plan.source_rows.numpy()
        n = len(cs)
        index = np.where(rows >= 0, rows, -1)
        index[plan.allocated_occurrences.numpy()] = 2 * n + np.arange(len(al))
        out = torch.empty(len(rows), dtype=cs.dtype)
        p.add(out, index, tuple(s for s in (cs, ts, al) if len(s)))
        run_on_host(p)
        np.testing.assert_array_equal(out.numpy(), z[f"{key}/bind/slots"])
        succ = torch_state(z, f"{key}/successor")
        p = co.SlotGather("cpu")
        term = torch.empty(len(succ.terminal_rows), dtype=succ.slots.dtype)
        p.add(term, succ.terminal_rows.numpy(), (succ.slots,))
        run_on_host(p)
        np.testing.assert_array_equal(term.numpy(), z[f"{key}/terminal_slots"])


def test_gather_program_chunks_and_literals():
    """Tasks longer than a chunk, empty tasks, literal tasks and four
    segments of int32 slots into int64 outputs."""
    from akv_b200 import context_occurrence as co

    rng = np.random.default_rng(3)
    segs = tuple(torch.from_numpy(rng.integers(0, 2**31, size=m).astype(np.int32))
                 for m in (700, 0, 3000, 5))
    total = sum(s.numel() for s in segs)
    g = co.SlotGather("cpu")
    idx = rng.integers(-3, total, size=5000)
    a = torch.empty(5000, dtype=torch.int64)
    g.add(a, idx, segs)
    b = torch.empty(0, dtype=torch.int32)
    g.add(b, [], segs)
    lit = rng.integers(-2**31, 2**31, size=2100)
    c = torch.empty(2100, dtype=torch.int32)
    g.add(c, lit, literal=True)
    with pytest.raises(ValueError, match="fit in int32"):
        g.add(torch.empty(1, dtype=torch.int64), [2**31], literal=True)
    run_on_host(g)
    flat = torch.cat(segs).numpy().astype(np.int64)
    np.testing.assert_array_equal(a.numpy(), np.where(idx < 0, -1, flat[np.maximum(idx, 0)]))
    np.testing.assert_array_equal(c.numpy(), lit.astype(np.int32))


def test_host_checks_and_messages():
    from akv_b200 import context_occurrence as co

    z = golden()
    key = "case0/0"
    state = torch_state(z, f"{key}/state")
    window, plan = window_plan(z, key)
    q = torch.from_numpy(z[f"{key}/query_slots"])
    e = torch.from_numpy(z[f"{key}/extra_slots"])
    vis = torch.from_numpy(z["case0/visible_until"])
    with pytest.raises(ValueError, match="Context admission does not cover the selected window"):
        co.advance(state, window, plan, q[:-1], e, vis)
    with pytest.raises(ValueError, match="Context admission does not cover the selected window"):
        co.advance(state, window, plan, q, e, vis.to(torch.int64))
    bad = Plan(**{**plan.__dict__, "source_rows": plan.source_rows.clone()})
    reused = np.flatnonzero(bad.source_rows.numpy() >= 0)
    if len(reused):
        n = len(window.birth_occurrences)
        bad.source_rows[reused[0]] = 2 * n - 1  # a terminal row the state does not hold
        with pytest.raises(ValueError, match="references a missing source"):
            co.advance(state, window, bad, q, e, vis)
    cs = torch.from_numpy(z[f"{key}/bind/canonical_slots"])
    with pytest.raises(ValueError, match="Occurrence slot buffers do not match"):
        co.bind(plan, cs, cs[:-1], e)
    with pytest.raises(ValueError, match="Occurrence slot buffers do not match"):
        co.bind(plan, cs, cs.to(torch.int32), e)
    g = co.SlotGather("cpu")
    with pytest.raises(ValueError):
        g.add(torch.empty(3, dtype=torch.int64), [0, 1, 2])  # no segments
    with pytest.raises(ValueError):
        g.add(torch.empty(3, dtype=torch.float32), [0, 1, 2], (cs,))
    with pytest.raises(ValueError):
        g.add(torch.empty(2, dtype=torch.int64), [0, 1, 2], (cs,))
    with pytest.raises(ValueError, match="cannot be empty"):
        co.OccurrenceBatch("cpu").launch()
    # host tensors never reach the kernel
    g = co.SlotGather("cpu")
    g.add(torch.empty(2, dtype=torch.int64), [0, 1], (cs,))
    with pytest.raises(ValueError, match="CUDA device"):
        g.launch()
    with pytest.raises(ValueError, match="CUDA device"):
        co.terminal_slots(torch_state(z, f"{key}/successor"))
