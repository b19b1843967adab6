"""The allocation-free drop compaction, akv_drop_compact_static.

Some callers cannot give the library device memory for a workspace: a
serving runtime that reserved all device memory for its KV pool, a caller
whose allocator forbids cudaMalloc while serving, a C/FFI caller with no
device allocator.  akv_drop_compact_static serves them: same kernels and
outputs as akv_drop_compact, scratch in the library's own device array.

This file is named to be collected last.  It checks, through the C ABI,
that two static calls in a row (the second one running over whatever the
first left in the shared array) give exactly the outputs of the workspace
entry point -- integer outputs, so the tolerance is zero -- and that calls
beyond the array's limits are refused.  It passes alone in a fresh process
and after the other tests.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

FIELDS = ("keep_mask", "positions", "active_offsets", "next_position", "transition_offsets",
          "freed_offsets", "totals", "status")


def _programs():
    from akv_b200 import workloads

    a = workloads.c3_program(requests=24, max_len=9000, seed=11)
    b = workloads.c2_program(seed=5, tokens=20000)
    return [(a, np.random.default_rng(11)), (b, np.random.default_rng(5))]


def _run(prog, rng_seed_rows, static):
    from akv_b200 import workloads
    from akv_b200.context_drop import DropCompactor, FreeSlotRing, launch_static

    dev = torch.device("cuda", 0)
    rows, nslots = workloads.slot_rows(rng_seed_rows, prog)
    free = np.arange(nslots, nslots + int(prog.shared_prefix.sum()) + 32, dtype=np.int32)
    table = np.zeros((prog.requests + 1, int(prog.token_counts.max())), np.int32)
    for r in range(prog.requests):
        table[r + 1, : len(rows[r])] = rows[r]
    req_to_token = torch.from_numpy(table).to(dev)
    ring = FreeSlotRing(torch.from_numpy(free), capacity=len(free) + prog.total_tokens, device=dev)
    comp = DropCompactor(prog.total_tokens, prog.requests, len(prog.ranges) // 2, dev)
    prep = comp.prepare(prog.token_counts, prog.range_offsets, prog.ranges,
                        np.arange(1, prog.requests + 1),
                        shared_prefix=prog.shared_prefix if prog.shared_prefix.any() else None)
    res = launch_static(comp, prep, req_to_token, ring) if static else \
        comp.launch(prep, req_to_token, ring)
    torch.cuda.synchronize()
    out = {f: getattr(res, f).cpu().numpy().copy() for f in FIELDS}
    kept, moved, _, freed = (int(x) for x in out["totals"])
    out["raw_indices"] = res.raw_indices[:kept].cpu().numpy()
    out["active_positions"] = res.active_positions[:kept].cpu().numpy()
    out["transition_source"] = res.transition_source[:moved].cpu().numpy()
    out["transition_destination"] = res.transition_destination[:moved].cpu().numpy()
    out["transition_pairs"] = res.transition_pairs[:moved].cpu().numpy()
    out["transition_raw"] = res.transition_raw[:moved].cpu().numpy()
    out["freed_slots"] = res.freed_slots[:freed].cpu().numpy()
    out["req_to_token"] = req_to_token.cpu().numpy()
    out["ring_state"] = ring.state.cpu().numpy()
    out["ring"] = ring.ring.cpu().numpy()
    return out


def test_static_entry_point_matches_workspace_entry_point_on_two_calls_in_a_row():
    progs = _programs()
    static = [_run(p, rng, True) for p, rng in progs]  # two static calls back to back
    progs = _programs()
    reference = [_run(p, rng, False) for p, rng in progs]
    for got, want in zip(static, reference):
        assert int(got["status"][0]) == 0
        assert int(got["totals"][1]) > 0 and int(got["totals"][3]) > 0
        for key in want:
            np.testing.assert_array_equal(got[key], want[key], err_msg=key)


def test_static_entry_point_refuses_calls_beyond_its_limits():
    from akv_b200 import _native

    lib = _native.lib
    max_req = int(lib.akv_drop_compact_static_max_requests())
    max_tiles = int(lib.akv_drop_compact_static_max_tiles())
    assert (max_req, max_tiles) == (4096, 65536)
    nulls = [None] * 19
    for n_requests, n_tiles in ((max_req + 1, 1), (1, max_tiles + 1)):
        status = lib.akv_drop_compact_static(
            n_requests, None, None, n_tiles, None, None, None, None, None, 0, 1, None, 1, None,
            *nulls[:15], None)
        assert status == _native.AKV_ERR_INVALID
