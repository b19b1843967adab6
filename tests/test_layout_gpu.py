"""The general event compiler on the device (C ABI akv_compile_layouts).

Every output of the reference's ContextLayout is compared bit for bit: with
the reference's own golden vectors (tests/golden/event_compiler.npz, made by
running its C++ compiler), and with the pinned oracle on seeded multi-event
programs of several size regimes, batched several requests per call.
"""

import numpy as np
import pytest
import torch

from conftest import golden

pytestmark = pytest.mark.gpu

EC = golden("event_compiler")
FIELDS = (
    "positions", "keep_mask", "materialized_stage", "birth_positions", "birth_stages",
    "transition_offsets", "transition_raw_tokens", "transition_old_positions",
    "transition_new_positions", "effective_reposition_stages", "drop_event_to_key",
    "effective_repositions", "ignored_repositions", "records", "virtual_mask",
    "key_to_token", "token_to_key",
)
INPUTS = (
    "token_ids", "drop_insert_offsets", "drop_range_offsets", "drop_ranges",
    "reposition_raw_boundaries", "reposition_insert_offsets",
)


def _compiler(programs, **kw):
    from akv_b200.context_plan import LayoutCompiler

    # Upper bound: every token moves at every Reposition.
    kw.setdefault("transition_capacity", max(1, sum(
        len(p.token_ids) * max(1, len(p.reposition_raw_boundaries)) for p in programs)))
    return LayoutCompiler(
        "cuda", max_tokens=max(1, sum(len(p.token_ids) for p in programs)),
        max_requests=len(programs),
        max_events=max(1, sum(len(p.drop_insert_offsets) for p in programs)),
        max_ranges=max(1, sum(len(p.drop_ranges) // 2 for p in programs)),
        max_repositions=max(1, sum(len(p.reposition_raw_boundaries) for p in programs)), **kw)


def _assert_layout(layout, want, what):
    for f in FIELDS:
        got = getattr(layout, f)
        assert got.device.type == "cpu"
        w = np.asarray(want[f])
        np.testing.assert_array_equal(got.numpy().astype(w.dtype), w, err_msg=f"{what}: {f}")
    assert layout.next_position == int(want["next_position"]), what


def _golden_cases():
    cases = sorted({k.split("/")[0] for k in EC.files})
    return [c for c in cases if f"{c}/error" not in EC.files]


def test_golden_cases_in_one_batch():
    """All of the reference's golden programs compiled as one batch."""
    from akv_b200.context_plan import Program

    cases = _golden_cases()
    programs = [Program.of(*[EC[f"{c}/in/{k}"] for k in INPUTS]) for c in cases]
    batch = _compiler(programs).compile(programs)
    batch.check()
    for b, case in enumerate(cases):
        want = {f: EC[f"{case}/out/{f}"] for f in FIELDS + ("next_position",)}
        _assert_layout(batch.request(b), want, case)


REGIMES = {
    # name: (programs, batch, T range, E range, P range, max ranges, span)
    "dense_small": (240, 60, (1, 80), (0, 9), (0, 9), 4, None),
    "medium": (48, 16, (100, 6000), (0, 30), (0, 30), 6, 400),
    "many_stages": (6, 3, (2000, 9000), (40, 120), (60, 200), 3, 60),
    "multi_tile": (4, 2, (60000, 70000), (10, 40), (5, 25), 8, 3000),
    # more than 256 Repositions / Drop events: tables read from global memory
    "wide": (3, 3, (6000, 12000), (260, 400), (280, 500), 3, 40),
}


def _random_programs(name, seed):
    from akv_b200 import workloads
    from akv_b200.context_plan import Program

    count, _, (tlo, thi), (elo, ehi), (plo, phi), mr, span = REGIMES[name]
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(count):
        T = int(rng.integers(tlo, thi + 1))
        prog = workloads.event_program(rng, T, int(rng.integers(elo, ehi + 1)),
                                       int(rng.integers(plo, phi + 1)), max_ranges=mr, span=span)
        out.append(Program.of(*prog))
    return out


@pytest.mark.parametrize("regime", sorted(REGIMES))
def test_random_programs_match_oracle(regime):
    from oracle import oracle

    programs = _random_programs(regime, seed=len(regime))
    per_batch = REGIMES[regime][1]
    checked = errors = 0
    for i in range(0, len(programs), per_batch):
        chunk = programs[i: i + per_batch]
        batch = _compiler(chunk).compile(chunk)
        assert batch.totals[3].item() & 1 == 0  # capacity suffices
        status = batch.status()
        for b, p in enumerate(chunk):
            args = (p.token_ids, p.drop_insert_offsets, p.drop_range_offsets, p.drop_ranges,
                    p.reposition_raw_boundaries, p.reposition_raw_boundaries.astype(np.int64) + 1)
            try:
                want = oracle.compile_layout(*args)
            except ValueError as exc:
                assert "no active tokens" in str(exc)
                assert status[b][0] == 1 and f"boundary {status[b][4]} " in str(exc)
                errors += 1
                continue
            assert status[b][0] == 0, status[b]
            _assert_layout(batch.request(b), want, f"{regime}[{i + b}]")
            raw, pos = batch.decode_view(b)
            want_raw, want_pos, _, _ = oracle.decode_layout(want)
            np.testing.assert_array_equal(raw.cpu().numpy(), want_raw)
            np.testing.assert_array_equal(pos.cpu().numpy(), want_pos)
            checked += 1
    assert checked > errors


def test_empty_and_event_free_requests_in_a_batch():
    from akv_b200 import workloads
    from akv_b200.context_plan import Program
    from oracle import oracle

    rng = np.random.default_rng(5)
    programs = [
        Program.of(np.zeros(0, np.int64)),                      # no tokens
        Program.of(np.arange(700)),                             # no events
        Program.of(*workloads.event_program(rng, 1300, 4, 3)),
        Program.of(np.arange(5), reposition_raw_boundaries=[1, 4]),  # compact: ignored
        Program.of(np.zeros(0, np.int64)),
        Program.of(np.arange(3000), [3000], [0, 1], [0, 2999], [2999]),  # one token survives
    ]
    batch = _compiler(programs).compile(programs)
    batch.check()
    for b, p in enumerate(programs):
        want = oracle.compile_layout(p.token_ids, p.drop_insert_offsets, p.drop_range_offsets,
                                     p.drop_ranges, p.reposition_raw_boundaries,
                                     p.reposition_raw_boundaries.astype(np.int64) + 1)
        _assert_layout(batch.request(b), want, f"request {b}")
    totals = batch.totals.cpu().tolist()
    assert totals[3] == 0


def test_int32_token_ids_and_device_outputs():
    from akv_b200 import workloads
    from akv_b200.context_plan import Program
    from oracle import oracle

    rng = np.random.default_rng(11)
    prog = Program.of(*workloads.event_program(rng, 4000, 12, 9, span=300))
    prog.token_ids = prog.token_ids.astype(np.int32)
    batch = _compiler([prog], token_ids_64=False).compile([prog])
    layout = batch.request(0, to_cpu=False)
    assert layout.positions.device.type == "cuda"
    want = oracle.compile_layout(prog.token_ids, prog.drop_insert_offsets,
                                 prog.drop_range_offsets, prog.drop_ranges,
                                 prog.reposition_raw_boundaries,
                                 prog.reposition_raw_boundaries.astype(np.int64) + 1)
    cpu = {f: getattr(layout, f).cpu() for f in FIELDS}
    for f in FIELDS:
        np.testing.assert_array_equal(cpu[f].numpy().astype(np.asarray(want[f]).dtype), want[f])


def test_drop_in_compile_context_layout_matches_reference_tensors():
    """Same dtypes, shapes and values as the reference's ContextLayout."""
    from akv_b200.context_plan import compile_context_layout

    for case in ("c1", "random13", "same_insertion", "suffix_drop_ignored"):
        args = [torch.from_numpy(np.ascontiguousarray(EC[f"{case}/in/{k}"])) for k in INPUTS]
        layout = compile_context_layout(*args)
        assert layout.records.dtype == torch.int32 and layout.records.shape[1] == 3
        assert layout.keep_mask.dtype == torch.bool and layout.virtual_mask.dtype == torch.bool
        assert layout.key_to_token.dtype == torch.int64 and layout.token_to_key.dtype == torch.int64
        assert layout.drop_event_to_key.dtype == torch.int64
        assert layout.effective_repositions.dtype == torch.bool
        for f in ("positions", "materialized_stage", "birth_positions", "birth_stages",
                  "transition_offsets", "transition_raw_tokens", "effective_reposition_stages"):
            assert getattr(layout, f).dtype == torch.int32, f
        want = {f: EC[f"{case}/out/{f}"] for f in FIELDS + ("next_position",)}
        _assert_layout(layout, want, case)
        assert layout.drop_insert_offsets.dtype == torch.int32


def test_errors_match_reference_messages():
    from akv_b200.context_plan import compile_context_layout

    def args(case):
        return [torch.from_numpy(np.ascontiguousarray(EC[f"{case}/in/{k}"])) for k in INPUTS]

    for case in ("err_no_active", "err_token_id", "err_unmaterialized", "err_unordered"):
        kind, message = str(EC[f"{case}/error"]).split(": ", 1)
        with pytest.raises((ValueError, RuntimeError)) as exc:
            compile_context_layout(*args(case))
        assert type(exc.value).__name__ == kind and str(exc.value) == message, case
    # A negative id passes the int32 range check and fails in the compiler.
    ids = torch.tensor([4, 9, -3, 7], dtype=torch.int32)
    empty = torch.zeros(0, dtype=torch.int32)
    with pytest.raises(ValueError, match=r"token ID -3 is outside"):
        compile_context_layout(ids, empty, torch.zeros(1, dtype=torch.int32), empty, empty, empty)


def test_transition_capacity_overflow_is_flagged_then_retried():
    from akv_b200 import _native, workloads
    from akv_b200.context_plan import Program, compile_context_layout
    from oracle import oracle

    rng = np.random.default_rng(21)
    prog = Program.of(*workloads.event_program(rng, 3000, 30, 40, span=20))
    batch = _compiler([prog], transition_capacity=7).compile([prog])
    totals = batch.totals.cpu().tolist()
    assert totals[3] & _native.LAYOUT_CAPACITY and totals[0] > 7
    with pytest.raises(RuntimeError, match="capacity"):
        batch.check()
    # compile_context_layout sizes its guess, then retries with the exact count.
    args = [torch.from_numpy(np.ascontiguousarray(x)) for x in (
        prog.token_ids, prog.drop_insert_offsets, prog.drop_range_offsets, prog.drop_ranges,
        prog.reposition_raw_boundaries, prog.reposition_raw_boundaries.astype(np.int64) + 1)]
    layout = compile_context_layout(*args)
    want = oracle.compile_layout(*[a.numpy() for a in args])
    _assert_layout(layout, want, "retried")
