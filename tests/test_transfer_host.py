"""Active-slot gather (srt/disaggregation/context_transfer.py:110-138): the
oracle restatement and the host arithmetic of akv_b200.context_transfer
against goldens made by running the reference's own functions
(tests/golden/make_transfer_golden.py)."""

import os
import types

import numpy as np

from conftest import ROOT

GOLDEN = os.path.join(ROOT, "tests", "golden", "active_slots.npz")


def golden_cases():
    g = np.load(GOLDEN)
    windows = g["windows"]
    for n in range(int(g["count"])):
        keep = g[f"c{n}_keep"]
        raw = np.flatnonzero(keep).astype(np.int32)
        case = dict(row=g[f"c{n}_row"], raw=raw, positions=g[f"c{n}_positions"][raw],
                    prompt=len(keep), next_position=int(g[f"c{n}_next_position"]),
                    raw_end=int(g[f"c{n}_raw_end"]))
        for j, w in enumerate(windows):
            yield case, (None if w < 0 else int(w)), g[f"c{n}_w{j}_out"], \
                tuple(g[f"c{n}_w{j}_lengths"])


def test_oracle_matches_reference_goldens():
    from oracle import oracle

    count = 0
    for c, window, want, lengths in golden_cases():
        got = oracle.active_slots(c["row"], c["raw"], c["positions"], c["prompt"],
                                  c["next_position"], c["raw_end"], window)
        np.testing.assert_array_equal(got, want)
        if window is not None:
            assert oracle.active_lengths(c["raw"], c["positions"], c["prompt"],
                                         c["next_position"], c["raw_end"], window) == lengths
        count += 1
    assert count >= 50


def test_request_active_lengths_matches_reference_goldens():
    from akv_b200.context_transfer import request_active_lengths

    for c, window, _, lengths in golden_cases():
        if window is None:
            continue
        view = types.SimpleNamespace(raw_indices=c["raw"], positions=c["positions"],
                                     prompt_length=c["prompt"], next_position=c["next_position"])
        req = types.SimpleNamespace(context_decode_layout=view)
        assert request_active_lengths(req, c["raw_end"], window) == lengths
