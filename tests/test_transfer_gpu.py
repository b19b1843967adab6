"""Active-slot gather on the device (C ABI akv_active_slots) through the
drop-in request_active_slots, against goldens made by running the
reference's request_active_slots (srt/disaggregation/context_transfer.py:110-128).
Integer outputs: bit-exact."""

import types

import numpy as np
import pytest
import torch

from test_transfer_host import golden_cases

pytestmark = pytest.mark.gpu


def test_request_active_slots_matches_reference_goldens():
    from akv_b200.context_transfer import request_active_slots

    dev = torch.device("cuda")
    count = 0
    for c, window, want, _ in golden_cases():
        table = np.zeros((2, len(c["row"])), np.int32)
        table[1] = c["row"]
        view = types.SimpleNamespace(
            raw_indices=c["raw"], positions=c["positions"],
            device_indices=torch.from_numpy(c["raw"]).to(dev), prompt_length=c["prompt"],
            next_position=c["next_position"])
        req = types.SimpleNamespace(context_decode_layout=view,
                                    kv=types.SimpleNamespace(req_pool_idx=1))
        pool = types.SimpleNamespace(req_to_token=torch.from_numpy(table).to(dev))
        got = request_active_slots(req, pool, c["raw_end"], window=window)
        np.testing.assert_array_equal(got.cpu().numpy(), want)
        count += 1
    assert count >= 50


def test_overflow_row_is_used_when_the_pool_keeps_one():
    from akv_b200.context_transfer import request_active_slots

    dev = torch.device("cuda")
    raw = np.array([0, 2, 5], np.int32)
    view = types.SimpleNamespace(raw_indices=raw, positions=np.arange(3, dtype=np.int32),
                                 device_indices=torch.from_numpy(raw).to(dev), prompt_length=6,
                                 next_position=3)
    req = types.SimpleNamespace(context_decode_layout=view,
                                kv=types.SimpleNamespace(req_pool_idx=7))
    row = torch.arange(100, 110, dtype=torch.int32, device=dev)
    pool = types.SimpleNamespace(req_to_token=torch.zeros(2, 4, dtype=torch.int32, device=dev),
                                 _context_rows={7: row})
    got = request_active_slots(req, pool, 8)
    assert got.cpu().tolist() == [100, 102, 105, 106, 107]


def test_out_of_row_index_reads_minus_one_and_sets_the_flag():
    from akv_b200.context_transfer import active_slots

    dev = torch.device("cuda")
    row = torch.arange(10, 20, dtype=torch.int32, device=dev)
    idx = torch.tensor([1, 50, 3], dtype=torch.int32, device=dev)
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    got = active_slots(row, idx, 0, 9, 12, error_flag=flag)
    torch.cuda.synchronize()
    assert got.cpu().tolist() == [11, -1, 13, 19, -1, -1]
    assert int(flag.item()) == 1


def test_empty_gather_returns_an_empty_vector():
    from akv_b200.context_transfer import active_slots

    dev = torch.device("cuda")
    row = torch.arange(4, dtype=torch.int32, device=dev)
    idx = torch.tensor([0, 1], dtype=torch.int32, device=dev)
    assert active_slots(row, idx, 2, 4, 4).numel() == 0


def test_batched_gather_matches_per_request_goldens():
    from akv_b200.context_transfer import ActiveSlotGather
    from oracle import oracle

    dev = torch.device("cuda")
    rows, idxs, starts, gens, ends, wants = [], [], [], [], [], []
    for c, window, want, _ in golden_cases():
        start, gen0 = oracle.active_slot_ranges(c["raw"], c["positions"], c["prompt"],
                                                c["next_position"], c["raw_end"], window)
        rows.append(torch.from_numpy(c["row"]).to(dev))
        idxs.append(torch.from_numpy(c["raw"]).to(dev))
        starts.append(start)
        gens.append(gen0)
        ends.append(c["raw_end"])
        wants.append(want)
    g = ActiveSlotGather(dev).plan(rows, idxs, starts, gens, ends)
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    out = g.run(error_flag=flag).cpu().numpy()
    assert int(flag.item()) == 0
    for r, want in enumerate(wants):
        np.testing.assert_array_equal(out[g.offsets[r]: g.offsets[r + 1]], want)
