"""Generate tests/golden/active_slots.npz by running the REFERENCE's
``request_active_slots`` and ``request_active_lengths``
(akv/system/sglang/srt/disaggregation/context_transfer.py:110-138) on the
CPU, with its own ``request_row`` (srt/context_system/request_storage.py)
and ``ContextDecodeLayout.from_layout`` (srt/context_system/occurrence.py).

Run in a container that has the reference tree (its root in
AKV_REFERENCE_ROOT, else the default of oracle/build_oracle.py):

    python tests/golden/make_transfer_golden.py

Nothing here is needed at test time: the tests read the .npz file only.
"""

from __future__ import annotations

import importlib.util
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle.build_oracle import REFERENCE_ROOT  # noqa: E402
SG = os.path.join(REFERENCE_ROOT, "akv/system/sglang")


def _load(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def reference_transfer():
    for pkg in ("sglang", "sglang.srt", "sglang.srt.context_system"):
        sys.modules.setdefault(pkg, types.ModuleType(pkg))
    _load("sglang.srt.context_system.request_storage",
          f"{SG}/srt/context_system/request_storage.py")
    _load("sglang.srt.context_system.occurrence", f"{SG}/srt/context_system/occurrence.py")
    _load("sglang.srt.context_system.usage", f"{SG}/srt/context_system/usage.py")
    return _load("akv_ref_transfer", f"{SG}/srt/disaggregation/context_transfer.py")


class _Layout:
    def __init__(self, keep, positions, next_position):
        self.keep_mask = torch.from_numpy(keep)
        self.positions = torch.from_numpy(positions)
        self.next_position = next_position


WINDOWS = (-1, 1, 64, 1000, 10**6)  # -1: no window


def cases(tr, occ):
    rng = np.random.default_rng(2026)
    out = {"windows": np.asarray(WINDOWS, np.int64)}
    n = 0
    for prompt in (1, 7, 300, 2000):
        for _ in range(5):
            keep = rng.random(prompt) < rng.uniform(0.2, 1.0)
            if not keep.any():
                keep[rng.integers(prompt)] = True
            kept = int(keep.sum())
            positions = np.arange(prompt, dtype=np.int32)
            positions[keep] = np.arange(kept, dtype=np.int32)  # compacted after the Reposition
            next_position = kept
            raw_end = prompt + int(rng.integers(0, 200))
            width = raw_end + int(rng.integers(0, 50))
            table = rng.permutation(50 * width)[: 3 * width].astype(np.int32).reshape(3, width)
            row_idx = int(rng.integers(3))
            view = occ.ContextDecodeLayout.from_layout(_Layout(keep, positions, next_position),
                                                       "cpu")
            req = types.SimpleNamespace(context_decode_layout=view,
                                        kv=types.SimpleNamespace(req_pool_idx=row_idx),
                                        context_program=None)
            pool = types.SimpleNamespace(req_to_token=torch.from_numpy(table))
            out[f"c{n}_keep"] = keep
            out[f"c{n}_positions"] = positions
            out[f"c{n}_next_position"] = np.int64(next_position)
            out[f"c{n}_raw_end"] = np.int64(raw_end)
            out[f"c{n}_row"] = table[row_idx]
            for j, window in enumerate(WINDOWS):
                w = None if window < 0 else window
                got = tr.request_active_slots(req, pool, raw_end, window=w)
                lengths = (-1, -1) if w is None else tr.request_active_lengths(req, raw_end, w)
                out[f"c{n}_w{j}_out"] = got.numpy().astype(np.int32)
                out[f"c{n}_w{j}_lengths"] = np.asarray(lengths, np.int64)
            n += 1
    out["count"] = np.int64(n)
    return out


def main():
    tr = reference_transfer()
    occ = sys.modules["sglang.srt.context_system.occurrence"]
    path = os.path.join(HERE, "active_slots.npz")
    np.savez_compressed(path, **cases(tr, occ))
    print(path, os.path.getsize(path))


if __name__ == "__main__":
    main()
