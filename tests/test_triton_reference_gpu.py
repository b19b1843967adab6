"""This build against the reference's own Triton kernels run on the GPU.

The kernels are loaded unmodified from the reference package installed in
baseline/_ref (``pip install --target baseline/_ref`` of the reference's
akv/system project); the test is skipped when it is not installed.  On the
GPU the Triton stores round to nearest even, so K is compared bit for bit
(the CPU interpreter truncates, which is why the committed goldens are fp32
runs); V and the index outputs are copies and must match exactly.
"""

import importlib.util
import os

import numpy as np
import pytest
import torch

from conftest import ROOT

pytestmark = pytest.mark.gpu

BASE = os.path.join(ROOT, "baseline", "_ref", "akv", "system", "sglang", "kernels", "ops",
                    "attention")


def _load(name):
    path = os.path.join(BASE, f"{name}.py")
    if not os.path.exists(path):
        pytest.skip("the reference package is not installed in baseline/_ref")
    spec = importlib.util.spec_from_file_location(f"akv_reference_{name}", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _pools(slots, layers, heads, dim, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    k = [torch.randn(slots, heads, dim, device=dev, generator=g).to(torch.bfloat16)
         for _ in range(layers)]
    v = [torch.randn(slots, heads, dim, device=dev, generator=g).to(torch.bfloat16)
         for _ in range(layers)]
    return k, v


@pytest.mark.parametrize("neox,rotary", [(True, 64), (False, 64), (True, 32)])
@pytest.mark.parametrize("in_place", [False, True])
def test_reposition_matches_the_reference_triton_kernel(neox, rotary, in_place):
    from akv_b200 import workloads
    from akv_b200.context_reposition import layer_pointer_table, reposition_kv_layers
    from akv_b200.rope import yarn_cos_sin_cache
    from oracle import oracle

    ref = _load("context_reposition")
    dev = torch.device("cuda")
    prog = workloads.c2_program()
    rows, nslots = workloads.slot_rows(np.random.default_rng(0), prog)
    lay = oracle.compile_layout(np.zeros(prog.total_tokens, np.int64), [prog.total_tokens],
                                [0, len(prog.ranges) // 2], prog.ranges,
                                [prog.total_tokens - 1], [prog.total_tokens])
    rng = np.random.default_rng(1)
    pick = np.sort(rng.choice(len(lay["transition_raw_tokens"]), size=3000, replace=False))
    src = rows[0][lay["transition_raw_tokens"][pick]].astype(np.int32)
    dst = src if in_place else (nslots + np.arange(len(src))).astype(np.int32)
    pairs = np.stack((lay["transition_old_positions"][pick],
                      lay["transition_new_positions"][pick]), 1).astype(np.int32)
    layers, heads, dim = 3, 8, 64
    cache = yarn_cos_sin_cache(65536, rotary, 150000.0, 32.0, 4096).to(dev)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
    outs = []
    for which in ("reference", "ours"):
        k, v = _pools(nslots + len(src), layers, heads, dim, 5, dev)
        args = (layer_pointer_table(k), layer_pointer_table(v), k[0], v[0], t(src), t(dst),
                t(pairs), cache)
        if which == "reference":
            ref.reposition_kv_layers(*args, is_neox_style=neox, rotary_dim=rotary)
        else:
            reposition_kv_layers(*args, is_neox_style=neox, rotary_dim=rotary)
        torch.cuda.synchronize()
        outs.append((k, v))
    d = torch.from_numpy(dst.astype(np.int64)).to(dev)
    (k_ref, v_ref), (k_ours, v_ours) = outs
    for kr, vr, ko, vo in zip(k_ref, v_ref, k_ours, v_ours):
        assert torch.equal(kr[d].view(torch.int16), ko[d].view(torch.int16))
        assert torch.equal(vr[d].view(torch.int16), vo[d].view(torch.int16))
        # nothing else in the pools changed differently
        assert torch.equal(kr.view(torch.int16), ko.view(torch.int16))


def test_page_table_kernels_match_the_reference_triton_kernels():
    from akv_b200.context_page_table import build_decode_metadata

    pt = _load("context_page_table")
    dev = torch.device("cuda")
    rng = np.random.default_rng(3)
    batch, generated = 40, 3
    lengths = rng.integers(1, 5000, size=batch)
    table = torch.from_numpy(rng.integers(1, 1 << 24, size=(batch, int(lengths.max()) + 8))
                             .astype(np.int32)).to(dev)
    registry = torch.zeros((batch, 6), dtype=torch.int64, device=dev)
    keep, seq = [], []
    for b, n in enumerate(lengths.tolist()):
        if b % 7 == 3:  # an ordinary request (registry row of zeros)
            seq.append(n)
            continue
        raw = np.flatnonzero(rng.random(n) < 0.6).astype(np.int32)
        if len(raw) == 0:
            raw = np.zeros(1, np.int32)
        pos = np.cumsum(rng.integers(1, 3, size=len(raw))).astype(np.int32)
        packed = torch.from_numpy(np.concatenate((raw, pos))).to(dev)
        keep.append(packed)
        registry[b] = torch.tensor([packed.data_ptr(), packed.data_ptr() + 4 * len(raw), n,
                                    len(raw), int(pos[-1]) + 1, 0], dtype=torch.int64)
        seq.append(len(raw) + generated)
    rows = torch.arange(batch, dtype=torch.int64, device=dev)
    seq_lens = torch.tensor(seq, dtype=torch.int64, device=dev)
    n_full = int(sum(seq))
    for window in (None, 128, 5):
        ours_indptr = torch.empty(batch + 1, dtype=torch.int32, device=dev)
        ours_idx = torch.empty(n_full, dtype=torch.int32, device=dev)
        ref_indptr = torch.zeros(batch + 1, dtype=torch.int32, device=dev)
        ref_idx = torch.full((n_full,), -7, dtype=torch.int32, device=dev)
        if window is None:
            build_decode_metadata(registry, table, rows, seq_lens, ours_indptr, ours_idx)
            ref_indptr[1:] = seq_lens.cumsum(0)
            pt.context_decode_indices[(batch,)](
                registry, table, rows, seq_lens, ref_indptr, ref_idx, None, None,
                ROW_STRIDE=table.stride(0), TRANSLATE=False, MULTIPLIER=1, HAS_START=False)
            n = n_full
        else:
            w_len = torch.empty(batch, dtype=torch.int64, device=dev)
            w_start = torch.empty(batch, dtype=torch.int64, device=dev)
            build_decode_metadata(registry, table, rows, seq_lens, ours_indptr, ours_idx,
                                  window=window, lengths_out=w_len, starts_out=w_start)
            r_len = torch.empty_like(seq_lens)
            pt.context_window_lengths[(batch,)](registry, rows, seq_lens, r_len, window)
            ref_indptr[1:] = r_len.cumsum(0)
            starts = seq_lens - r_len
            pt.context_decode_indices[(batch,)](
                registry, table, rows, r_len, ref_indptr, ref_idx, starts, None,
                ROW_STRIDE=table.stride(0), TRANSLATE=False, MULTIPLIER=1, HAS_START=True)
            torch.cuda.synchronize()
            assert torch.equal(w_len, r_len)
            assert torch.equal(w_start, starts)
            n = int(r_len.sum().item())
        torch.cuda.synchronize()
        assert torch.equal(ours_indptr, ref_indptr)
        assert torch.equal(ours_idx[:n], ref_idx[:n])
