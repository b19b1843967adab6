"""Occurrence slot binding on the GPU (C ABI ``akv_gather_slots``), bit-exact
against the reference's golden vectors (tests/golden/occurrence.npz) and,
at large sizes, against a numpy gather."""

from __future__ import annotations

import dataclasses

import numpy as np
import pytest
import torch

from occurrence_cases import (ADVANCE, State, as_numpy, check_advance, golden, steps,
                              torch_state, window_plan)

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def on_device(state):
    return dataclasses.replace(state, slots=state.slots.to(DEV))


def host_numpy(res):
    """as_numpy after bringing the device tensors back."""
    moved = {f: getattr(res, f).cpu() for f in ADVANCE}
    for f in ("unused_swa_slots",):
        v = getattr(res, f)
        moved[f] = None if v is None else v.cpu()
    st = dataclasses.replace(res.state, slots=res.state.slots.cpu())
    return as_numpy(dataclasses.replace(res, state=st, **moved))


def test_advance_chain_matches_the_reference():
    """Every request's prefill chained through the drop-in ``advance``: only
    the first state comes from the fixture; every step, every field."""
    from akv_b200 import context_occurrence as co

    z = golden()
    flag = torch.zeros(1, dtype=torch.int32, device=DEV)
    for c in z["cases"]:
        c = str(c)
        vis = torch.from_numpy(z[f"{c}/visible_until"])
        state = on_device(torch_state(z, f"{c}/0/state"))
        for k in range(int(z[f"{c}/steps"])):
            key = f"{c}/{k}"
            window, plan = window_plan(z, key)
            q = torch.from_numpy(z[f"{key}/query_slots"]).to(DEV)
            e = torch.from_numpy(z[f"{key}/extra_slots"]).to(DEV)
            res = co.advance(state, window, plan, q, e, vis, error_flag=flag)
            assert type(res.state) is State and res.state.slots.is_cuda
            assert res.occurrence_slots.is_cuda and res.copy_source_slots.dtype == torch.int32
            check_advance(host_numpy(res), z, key)
            term = co.terminal_slots(res.state, error_flag=flag)
            np.testing.assert_array_equal(term.cpu().numpy(), z[f"{key}/terminal_slots"])
            state = res.state
    assert int(flag.item()) == 0


def test_bind_matches_the_reference():
    from akv_b200 import context_occurrence as co

    z = golden()
    flag = torch.zeros(1, dtype=torch.int32, device=DEV)
    for c, k in steps(z):
        key = f"{c}/{k}"
        _, plan = window_plan(z, key)
        args = [torch.from_numpy(z[f"{key}/{f}"]).to(DEV)
                for f in ("bind/canonical_slots", "bind/terminal_slots", "extra_slots")]
        got = co.bind(plan, *args, error_flag=flag)
        for f, v in zip(("slots", "copy_source_slots", "copy_destination_slots",
                         "copy_position_pairs"), got):
            want = z[f"{key}/bind/{f}"]
            assert v.is_cuda and str(v.dtype).endswith(str(want.dtype))
            np.testing.assert_array_equal(v.cpu().numpy(), want, err_msg=f"{key} {f}")
    assert int(flag.item()) == 0


def test_batch_matches_the_scheduler_concatenation():
    """Step k of every request plus ordinary requests, one launch; the
    concatenations equal the scheduler's torch.cat of the reference's
    per-request results."""
    from akv_b200 import context_occurrence as co

    z = golden()
    gen = torch.Generator().manual_seed(11)
    for k in range(3):
        batch = co.OccurrenceBatch(DEV)
        want = {"slots": [], "src": [], "dst": [], "pairs": []}
        keys = []
        for i, c in enumerate(z["cases"]):
            if k >= int(z[f"{c}/steps"]):
                continue
            key = f"{c}/{k}"
            if i % 2:
                pre = torch.randint(0, 10**6, (i * 13,), generator=gen)
                birth = torch.randint(0, 10**6, (i + 1,), generator=gen)
                batch.add_ordinary(pre.to(DEV), birth.to(DEV))
                want["slots"].append(torch.cat((pre, birth)).numpy())
                keys.append(None)
            st = on_device(torch_state(z, f"{key}/state"))
            st = dataclasses.replace(st, slots=st.slots.to(torch.int64))
            window, plan = window_plan(z, key)
            batch.add_context(st, window, plan,
                              torch.from_numpy(z[f"{key}/query_slots"]).to(DEV, torch.int64),
                              torch.from_numpy(z[f"{key}/extra_slots"]).to(DEV, torch.int64),
                              torch.from_numpy(z[f"{c}/visible_until"]))
            keys.append(key)
            want["slots"].append(z[f"{key}/advance/occurrence_slots"].astype(np.int64))
            want["src"].append(z[f"{key}/advance/copy_source_slots"])
            want["dst"].append(z[f"{key}/advance/copy_destination_slots"])
            want["pairs"].append(z[f"{key}/advance/copy_position_pairs"].reshape(-1, 2))
        advances, slots, src, dst, pairs = batch.launch()
        assert len(advances) == len(keys)
        for key, a in zip(keys, advances):
            assert (a is None) == (key is None)
            if a is not None:
                np.testing.assert_array_equal(a.retired_slots.cpu().numpy(),
                                              z[f"{key}/advance/retired_slots"])
                np.testing.assert_array_equal(a.state.slots.cpu().numpy(),
                                              z[f"{key}/successor/slots"])
        np.testing.assert_array_equal(slots.cpu().numpy(), np.concatenate(want["slots"]))
        np.testing.assert_array_equal(src.cpu().numpy(), np.concatenate(want["src"]))
        np.testing.assert_array_equal(dst.cpu().numpy(), np.concatenate(want["dst"]))
        np.testing.assert_array_equal(pairs.cpu().numpy(), np.concatenate(want["pairs"]))


@pytest.mark.parametrize("seg_dtype,out_dtype", [(torch.int64, torch.int64),
                                                 (torch.int32, torch.int64),
                                                 (torch.int64, torch.int32),
                                                 (torch.int32, torch.int32)])
def test_gather_kernel_at_scale(seg_dtype, out_dtype):
    """Millions of outputs over one to four segments (empty ones among
    them), negative indices, literal tasks; a numpy gather is the check."""
    from akv_b200 import context_occurrence as co

    rng = np.random.default_rng(17)
    g = co.SlotGather(DEV)
    checks = []
    for t in range(9):
        lens = [int(x) for x in rng.integers(0, 400_000, size=int(rng.integers(1, 5)))]
        if t == 4:
            lens[0] = 0
        segs = [torch.from_numpy(rng.integers(0, 2**31 - 1, size=m)).to(DEV, seg_dtype)
                for m in lens]
        total = sum(lens)
        n = int(rng.integers(0, 1_500_000))
        if total == 0:
            n = 0
        idx = rng.integers(-5, max(total, 1), size=n)
        out = torch.empty(n, dtype=out_dtype, device=DEV)
        g.add(out, idx, segs)
        flat = np.concatenate([s.cpu().numpy().astype(np.int64) for s in segs]) if total \
            else np.zeros(0, np.int64)
        expect = np.where(idx < 0, -1, flat[np.clip(idx, 0, max(total - 1, 0))] if total
                          else -1)
        checks.append((out, expect))
    lit = rng.integers(-2**31, 2**31, size=300_000)  # literals are int32 values
    lit_out = torch.empty(len(lit), dtype=out_dtype, device=DEV)
    g.add(lit_out, lit, literal=True)
    checks.append((lit_out, lit))
    flag = torch.zeros(1, dtype=torch.int32, device=DEV)
    g.launch(flag)
    torch.cuda.synchronize()
    assert int(flag.item()) == 0
    for out, expect in checks:
        want = expect.astype(np.int32) if out_dtype == torch.int32 else expect
        np.testing.assert_array_equal(out.cpu().numpy(), want)


def test_index_past_the_segments_sets_the_error_flag():
    """The kernel's bounds check: an index at or past the end of the
    concatenation writes -1 and raises the flag (no access past it)."""
    from akv_b200 import context_occurrence as co

    segs = (torch.arange(10, 20, device=DEV), torch.arange(100, 105, device=DEV))
    out = torch.empty(4, dtype=torch.int64, device=DEV)
    g = co.SlotGather(DEV)
    g.add(out, [0, 14, 15, 1000], segs)
    flag = torch.zeros(1, dtype=torch.int32, device=DEV)
    g.launch(flag)
    assert out.cpu().tolist() == [10, 104, -1, -1]
    assert int(flag.item()) == 1


def test_graph_capture_of_a_batch_replays():
    """One batch bound inside a CUDA graph (the copy from pinned memory and
    the launch are both capturable) and replayed."""
    from akv_b200 import context_occurrence as co

    z = golden()
    key = "case3/0"
    st = on_device(torch_state(z, f"{key}/state"))
    window, plan = window_plan(z, key)
    args = (torch.from_numpy(z[f"{key}/query_slots"]).to(DEV),
            torch.from_numpy(z[f"{key}/extra_slots"]).to(DEV),
            torch.from_numpy(z["case3/visible_until"]))
    batch = co.OccurrenceBatch(DEV)
    batch.add_context(st, window, plan, *args)
    gather, (_, slots, src, dst, pairs) = batch._queue()
    stream = torch.cuda.Stream(DEV)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        words, n_tasks, n_chunks = gather.pack()
        host = torch.from_numpy(words).pin_memory()
        dev = torch.empty(len(words), dtype=torch.int64, device=DEV)
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=stream):
            dev.copy_(host, non_blocking=True)
            from akv_b200 import _native
            base = dev.data_ptr()
            status = _native.lib.akv_gather_slots(
                base, base + 96 * n_tasks, n_chunks, base + 8 * (12 * n_tasks + n_chunks),
                None, _native.stream_of(DEV))
            assert status == 0
    slots.fill_(-7)
    graph.replay()
    torch.cuda.synchronize()
    np.testing.assert_array_equal(slots.cpu().numpy(), z[f"{key}/advance/occurrence_slots"])
    np.testing.assert_array_equal(pairs.cpu().numpy(),
                                  z[f"{key}/advance/copy_position_pairs"].reshape(-1, 2))
    del graph
