"""The reference's own CPU event compiler, built by oracle/build_oracle.py.

TEST INFRASTRUCTURE ONLY: loaded by tests/ and by bench.py's reference arm
and cpu_baseline leg to time and check against the reference itself.  The
library in oracle/_ref/ is compiled from the C++ that
akv/system/sglang/kernels/ops/attention/context_plan.py carries
(:48-540); ``compile_context_layout`` below drives its two exported
functions the way the reference's ``compile_context_layout`` does
(srt/context_system/ir.py:113-274): count pass, exact-size allocation,
compile pass, status check.
"""

from __future__ import annotations

import os

import numpy as np
import torch

from .build_oracle import REF_SO

_mod = None


def available() -> bool:
    return os.path.exists(REF_SO)


def module():
    global _mod
    if _mod is None:
        import tvm_ffi

        _mod = tvm_ffi.load_module(REF_SO)
    return _mod


def _t(x, dtype):
    x = np.ascontiguousarray(np.asarray(x), dtype=dtype)
    out = torch.empty(x.shape, dtype={np.int32: torch.int32, np.int64: torch.int64}[dtype])
    out.copy_(torch.from_numpy(x))
    return out


def compile_context_layout(token_ids, drop_insert_offsets, drop_range_offsets, drop_ranges,
                           reposition_raw_boundaries, reposition_insert_offsets):
    mod = module()
    tokens = _t(token_ids, np.int32)
    drops = _t(drop_insert_offsets, np.int32)
    offsets = _t(drop_range_offsets, np.int32)
    ranges = _t(drop_ranges, np.int32)
    bounds = _t(reposition_raw_boundaries, np.int32)
    inserts = _t(reposition_insert_offsets, np.int32)
    t, p = len(tokens), len(bounds)
    counts = torch.zeros(p, dtype=torch.int32)
    count_status = torch.zeros(2, dtype=torch.int64)
    mod.count_radix_reposition_transitions(t, drops, offsets, ranges, bounds, inserts, counts,
                                           count_status)
    if int(count_status[0]) == 1:
        raise ValueError(f"Reposition at raw boundary {int(count_status[1])} has no active tokens.")
    n = int(counts.sum())
    cap = t + len(ranges) // 2 + p
    out = dict(
        records=torch.empty((cap, 3), dtype=torch.int32),
        virtual_mask=torch.empty(cap, dtype=torch.bool),
        key_to_token=torch.empty(cap, dtype=torch.int64),
        token_to_key=torch.empty(t, dtype=torch.int64),
        positions=torch.empty(t, dtype=torch.int32),
        keep_mask=torch.empty(t, dtype=torch.bool),
        materialized_stage=torch.empty(t, dtype=torch.int32),
        birth_positions=torch.empty(t, dtype=torch.int32),
        birth_stages=torch.empty(t, dtype=torch.int32),
        transition_offsets=torch.empty(p + 1, dtype=torch.int32),
        transition_raw_tokens=torch.empty(n, dtype=torch.int32),
        transition_old_positions=torch.empty(n, dtype=torch.int32),
        transition_new_positions=torch.empty(n, dtype=torch.int32),
        effective_reposition_stages=torch.full((p,), -1, dtype=torch.int32),
        drop_event_to_key=torch.full((len(drops),), -1, dtype=torch.int64),
        effective_repositions=torch.zeros(p, dtype=torch.bool),
        ignored_repositions=torch.zeros(p, dtype=torch.bool),
    )
    status = torch.zeros(5, dtype=torch.int64)
    mod.compile_radix_reposition_layout(
        tokens, drops, offsets, ranges, bounds, inserts, out["records"], out["virtual_mask"],
        out["key_to_token"], out["token_to_key"], out["positions"], out["keep_mask"],
        out["materialized_stage"], out["birth_positions"], out["birth_stages"],
        out["transition_offsets"], out["transition_raw_tokens"], out["transition_old_positions"],
        out["transition_new_positions"], out["effective_reposition_stages"],
        out["drop_event_to_key"], out["effective_repositions"], out["ignored_repositions"],
        status,
    )
    if int(status[0]) == 1:
        raise ValueError(f"Reposition at raw boundary {int(status[4])} has no active tokens.")
    if int(status[0]) == 2:
        raise ValueError(f"Reposition Radix token ID {int(status[4])} is outside the range.")
    key_len, stages = int(status[1]), int(status[2])
    res = {k: v.numpy() for k, v in out.items()}
    res["records"] = res["records"][:key_len]
    res["virtual_mask"] = res["virtual_mask"][:key_len]
    res["key_to_token"] = res["key_to_token"][:key_len]
    res["transition_offsets"] = res["transition_offsets"][: stages + 1]
    res["next_position"] = int(status[3])
    return res
