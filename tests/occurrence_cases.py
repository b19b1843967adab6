"""Shared fixtures of the occurrence tests: the golden file
(tests/golden/occurrence.npz, made by make_occurrence_golden.py from the
reference's srt/context_system/occurrence.py) read back into the shapes
the reference's OccurrenceState / OccurrenceWindow /
OccurrenceMaterialization have."""

from __future__ import annotations

import os
from dataclasses import dataclass
from types import SimpleNamespace

import numpy as np
import torch

from conftest import ROOT

GOLDEN = os.path.join(ROOT, "tests", "golden", "occurrence.npz")
STATE = ("slots", "owned", "canonical_rows", "terminal_rows", "canonical_positions")
WINDOW = ("occurrence_raw_tokens", "occurrence_positions", "birth_occurrences",
          "terminal_occurrences", "segment_query_starts", "segment_query_ends",
          "segment_key_offsets", "segment_key_occurrences")
PLAN = ("source_rows", "allocated_occurrences", "copy_occurrences", "copy_source_rows",
        "copy_position_pairs", "terminal_occurrences", "read_cached", "repositioned_cached")
ADVANCE = ("occurrence_slots", "copy_source_slots", "copy_destination_slots",
           "copy_position_pairs", "retired_slots")


@dataclass(frozen=True)
class State:
    """Field-for-field stand-in for the reference's OccurrenceState."""

    slots: torch.Tensor
    owned: torch.Tensor
    canonical_rows: torch.Tensor
    terminal_rows: torch.Tensor
    canonical_positions: torch.Tensor
    exact_prefix_len: int
    swa_resident: torch.Tensor | None = None


class Plan(SimpleNamespace):
    @property
    def extra_page_count(self):
        return len(self.allocated_occurrences)


def golden():
    return np.load(GOLDEN)


def steps(z):
    for c in z["cases"]:
        for k in range(int(z[f"{c}/steps"])):
            yield str(c), k


def np_state(z, key):
    d = {f: z[f"{key}/{f}"] for f in STATE}
    d["exact_prefix_len"] = int(z[f"{key}/exact_prefix_len"])
    if f"{key}/swa_resident" in z:
        d["swa_resident"] = z[f"{key}/swa_resident"]
    return d


def torch_state(z, key, device="cpu"):
    d = np_state(z, key)
    swa = d.get("swa_resident")
    return State(torch.from_numpy(d["slots"]).to(device), torch.from_numpy(d["owned"]),
                 torch.from_numpy(d["canonical_rows"]), torch.from_numpy(d["terminal_rows"]),
                 torch.from_numpy(d["canonical_positions"]), d["exact_prefix_len"],
                 torch.from_numpy(swa) if swa is not None else None)


def window_plan(z, key):
    window = SimpleNamespace(**{f: torch.from_numpy(z[f"{key}/window/{f}"]) for f in WINDOW})
    plan = Plan(**{f: torch.from_numpy(z[f"{key}/plan/{f}"]) for f in PLAN})
    return window, plan


def check_advance(got, z, key):
    """``got``: dict of numpy outputs and a successor dict."""
    for f in ADVANCE + ("unused_swa_slots", "retired_swa_resident"):
        if f"{key}/advance/{f}" in z:
            want = z[f"{key}/advance/{f}"]
            assert got[f].dtype == want.dtype, (key, f)
            np.testing.assert_array_equal(got[f], want, err_msg=f"{key} {f}")
        else:
            assert got.get(f) is None, (key, f)
    for f in STATE:
        want = z[f"{key}/successor/{f}"]
        assert got["successor"][f].dtype == want.dtype, (key, f)
        np.testing.assert_array_equal(got["successor"][f], want, err_msg=f"{key} successor {f}")
    if f"{key}/successor/swa_resident" in z:
        np.testing.assert_array_equal(got["successor"]["swa_resident"],
                                      z[f"{key}/successor/swa_resident"])


def as_numpy(res):
    got = {f: getattr(res, f).numpy() for f in ADVANCE}
    for f in ("unused_swa_slots", "retired_swa_resident"):
        v = getattr(res, f)
        got[f] = None if v is None else v.numpy()
    got["successor"] = {f: getattr(res.state, f).numpy() for f in STATE}
    if res.state.swa_resident is not None:
        got["successor"]["swa_resident"] = res.state.swa_resident.numpy()
    return got
