"""Host half of the device event compiler: the reference's metadata checks
and messages (context_plan.py:88-157, ir.py:144-153), checked on the CPU."""

import numpy as np
import pytest
import torch

from conftest import golden

EC = golden("event_compiler")
INPUTS = (
    "token_ids", "drop_insert_offsets", "drop_range_offsets", "drop_ranges",
    "reposition_raw_boundaries", "reposition_insert_offsets",
)


def _validate(T, drops, offsets, ranges, bounds=(), inserts=None):
    from akv_b200.context_plan import validate_program

    bounds = np.asarray(bounds, np.int64)
    validate_program(T, drops, offsets, ranges, bounds,
                     bounds + 1 if inserts is None else inserts)


@pytest.mark.parametrize("case", ["err_unmaterialized", "err_unordered"])
def test_golden_metadata_errors(case):
    kind, message = str(EC[f"{case}/error"]).split(": ", 1)
    inp = [EC[f"{case}/in/{k}"] for k in INPUTS]
    with pytest.raises(RuntimeError) as exc:
        _validate(len(inp[0]), *inp[1:])
    assert kind == "RuntimeError" and str(exc.value) == message


@pytest.mark.parametrize("args, message", [
    ((10, [3], [0, 1], [0, 1, 2]), "tensor lengths are inconsistent"),
    ((10, [3], [0, 1, 1], [0, 1]), "tensor lengths are inconsistent"),
    ((10, [3], [1, 1], [0, 1]), "does not cover drop_ranges"),
    ((10, [11], [0, 1], [0, 1]), "Invalid Drop event metadata"),
    ((10, [5, 5], [0, 1, 2], [0, 1, 2, 3]), "Invalid Drop event metadata"),
    ((10, [5, 7], [0, 1, 1], [0, 1]), "Invalid Drop event metadata"),  # empty event
    ((10, [], [0], [], [10]), "Invalid Reposition event metadata"),
    ((10, [], [0], [], [4, 4]), "Invalid Reposition event metadata"),
    ((10, [5], [0, 1], [3, 3]), "already materialized"),
    ((10, [5], [0, 1], [3, 6]), "already materialized"),
    ((10, [5], [0, 2], [0, 2, 2, 4]), "already materialized"),  # previous_end < start
])
def test_metadata_checks(args, message):
    with pytest.raises(RuntimeError, match=message):
        _validate(*args)


def test_valid_programs_pass():
    from akv_b200 import workloads

    rng = np.random.default_rng(0)
    for _ in range(50):
        ids, drops, offsets, ranges, bounds = workloads.event_program(
            rng, int(rng.integers(1, 5000)), int(rng.integers(0, 20)), int(rng.integers(0, 20)))
        _validate(len(ids), drops, offsets, ranges, bounds)


def test_mismatched_insert_offsets_rejected():
    with pytest.raises(RuntimeError, match="Invalid Reposition event metadata"):
        _validate(10, [], [0], [], [4], inserts=np.array([4]))


def test_too_many_repositions():
    from akv_b200.context_plan import MAX_REPOSITIONS

    n = MAX_REPOSITIONS + 1
    with pytest.raises(ValueError, match="Reposition events per request"):
        _validate(n + 5, [], [0], [], np.arange(n))


def test_drop_in_input_checks():
    from akv_b200.context_plan import compile_context_layout

    ok = torch.zeros(0, dtype=torch.int32)
    with pytest.raises(ValueError, match="token_ids must be a one-dimensional CPU integer"):
        compile_context_layout(torch.zeros(3, dtype=torch.float32), ok,
                               torch.zeros(1, dtype=torch.int32), ok, ok, ok)
    with pytest.raises(ValueError, match="drop_ranges exceeds the signed int32 range"):
        compile_context_layout(torch.zeros(3, dtype=torch.int64), ok,
                               torch.zeros(1, dtype=torch.int32),
                               torch.tensor([0, 2**31], dtype=torch.int64), ok, ok)
