"""Generate the golden fixtures in this directory by running the REFERENCE.

Run in a container that has the reference tree (its root in
AKV_REFERENCE_ROOT, else the default of oracle/build_oracle.py):

    python tests/golden/make_golden.py

What runs, all on the CPU:

* the reference's C++ event compiler (the ``_SOURCE`` of
  akv/system/sglang/kernels/ops/attention/context_plan.py), built by
  ``oracle/build_oracle.build_reference`` with tvm_ffi, driven through the
  reference's own ``compile_context_layout`` (srt/context_system/ir.py:113-274);
* the reference's Triton kernels ``context_decode_indices``,
  ``context_window_lengths`` (kernels/ops/attention/context_page_table.py),
  ``write_row_slots`` (kernels/ops/memory/context_rows.py) and
  ``_reposition_layers_kernel`` (kernels/ops/attention/context_reposition.py)
  under the Triton CPU interpreter (TRITON_INTERPRET=1).  The interpreter
  truncates fp32 -> bf16 stores, so the reposition goldens are produced with
  fp32 K/V holding bf16-representable values: they pin the fp32 arithmetic
  bit for bit, and a bf16 store is the round-to-nearest-even of that value
  (what the GPU store does);
* ``flash_attention_with_sink`` (srt/layers/attention/context_backend.py:254-272)
  with a stand-in attention kernel, pinning the sink LSE correction.

Nothing here is needed at test time: the tests read the .npz files only.
"""

from __future__ import annotations

import importlib.util
import os
import sys
import types

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from akv_b200 import workloads  # noqa: E402
from oracle.build_oracle import REFERENCE_ROOT, build_reference  # noqa: E402

SG = os.path.join(REFERENCE_ROOT, "akv/system/sglang")


def _t(x):
    # A fresh torch tensor: numpy-backed empty tensors carry stride 0, which
    # tvm_ffi rejects as non-contiguous; the server's own tensors never do.
    x = np.ascontiguousarray(x)
    out = torch.empty(x.shape, dtype=torch.from_numpy(x.reshape(-1)[:0].copy()).dtype)
    out.copy_(torch.from_numpy(x))
    return out


def _load(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def reference_modules():
    import tvm_ffi

    ir = _load("akv_ref_ir", f"{SG}/srt/context_system/ir.py")
    plan = tvm_ffi.load_module(build_reference())
    ir._load_module = lambda: plan
    page_table = _load("akv_ref_page_table", f"{SG}/kernels/ops/attention/context_page_table.py")
    rows = _load("akv_ref_rows", f"{SG}/kernels/ops/memory/context_rows.py")
    repos = _load("akv_ref_reposition", f"{SG}/kernels/ops/attention/context_reposition.py")
    # context_backend.py imports one helper from the (absent) SGLang tree.
    for pkg in ("sglang", "sglang.srt", "sglang.srt.context_system"):
        sys.modules.setdefault(pkg, types.ModuleType(pkg))
    storage = types.ModuleType("sglang.srt.context_system.request_storage")
    storage.request_row = lambda *a, **k: None
    sys.modules["sglang.srt.context_system.request_storage"] = storage
    backend = _load("akv_ref_backend", f"{SG}/srt/layers/attention/context_backend.py")
    return ir, page_table, rows, repos, backend


LAYOUT_FIELDS = (
    "positions", "keep_mask", "materialized_stage", "birth_positions", "birth_stages",
    "transition_offsets", "transition_raw_tokens", "transition_old_positions",
    "transition_new_positions", "effective_reposition_stages", "drop_event_to_key",
    "effective_repositions", "ignored_repositions", "records", "virtual_mask",
    "key_to_token", "token_to_key",
)
INPUT_FIELDS = (
    "token_ids", "drop_insert_offsets", "drop_range_offsets", "drop_ranges",
    "reposition_raw_boundaries", "reposition_insert_offsets",
)


def random_program(rng, token_count):
    drops, offsets, ranges = [], [0], []
    inserts = np.sort(rng.choice(np.arange(1, token_count + 1),
                                 size=min(token_count, int(rng.integers(1, 7))), replace=False))
    for ins in inserts:
        n = int(rng.integers(1, 4))
        cuts = np.sort(rng.choice(np.arange(0, ins + 1), size=min(ins + 1, 2 * n), replace=False))
        pairs = [(int(cuts[2 * i]), int(cuts[2 * i + 1])) for i in range(len(cuts) // 2)
                 if cuts[2 * i] < cuts[2 * i + 1]]
        if not pairs:
            continue
        drops.append(int(ins))
        for s, e in pairs:
            ranges += [s, e]
        offsets.append(offsets[-1] + len(pairs))
    nrep = int(rng.integers(1, 6))
    bounds = np.sort(rng.choice(np.arange(0, token_count), size=min(token_count, nrep),
                                replace=False))
    token_ids = rng.integers(0, 2**31, size=token_count)
    return dict(
        token_ids=np.asarray(token_ids, np.int64),
        drop_insert_offsets=np.asarray(drops, np.int32),
        drop_range_offsets=np.asarray(offsets, np.int32),
        drop_ranges=np.asarray(ranges, np.int32),
        reposition_raw_boundaries=np.asarray(bounds, np.int32),
        reposition_insert_offsets=np.asarray(bounds + 1, np.int32),
    )


def single_stage(program, r=0):
    t = int(program.token_counts[r])
    rr = program.request_ranges(r)
    return dict(
        token_ids=np.arange(t, dtype=np.int64) % 50000,
        drop_insert_offsets=np.asarray([t] if len(rr) else [], np.int32),
        drop_range_offsets=np.asarray([0, len(rr) // 2] if len(rr) else [0], np.int32),
        drop_ranges=np.asarray(rr, np.int32),
        reposition_raw_boundaries=np.asarray([t - 1], np.int32),
        reposition_insert_offsets=np.asarray([t], np.int32),
    )


def event_compiler_cases(ir):
    rng = np.random.default_rng(20261201)
    cases = {"c1": single_stage(workloads.c1_program(seed=0))}
    for i in range(32):
        cases[f"random{i}"] = random_program(rng, int(rng.integers(1, 1500)))
    i32 = lambda x: np.asarray(x, np.int32)  # noqa: E731
    cases["prewarm"] = dict(token_ids=np.zeros(1, np.int64), drop_insert_offsets=i32([]),
                            drop_range_offsets=i32([0]), drop_ranges=i32([]),
                            reposition_raw_boundaries=i32([]), reposition_insert_offsets=i32([]))
    cases["ten_tokens"] = dict(token_ids=np.arange(10, dtype=np.int64),
                               drop_insert_offsets=i32([5]), drop_range_offsets=i32([0, 1]),
                               drop_ranges=i32([2, 5]), reposition_raw_boundaries=i32([7]),
                               reposition_insert_offsets=i32([8]))
    cases["suffix_drop_ignored"] = dict(
        token_ids=np.arange(12, dtype=np.int64), drop_insert_offsets=i32([12]),
        drop_range_offsets=i32([0, 1]), drop_ranges=i32([8, 12]),
        reposition_raw_boundaries=i32([11]), reposition_insert_offsets=i32([12]))
    cases["same_insertion"] = dict(
        token_ids=np.arange(20, dtype=np.int64), drop_insert_offsets=i32([6, 14]),
        drop_range_offsets=i32([0, 1, 3]), drop_ranges=i32([1, 3, 7, 9, 10, 12]),
        reposition_raw_boundaries=i32([5, 13, 19]), reposition_insert_offsets=i32([6, 14, 20]))
    cases["err_no_active"] = dict(
        token_ids=np.arange(5, dtype=np.int64), drop_insert_offsets=i32([5]),
        drop_range_offsets=i32([0, 1]), drop_ranges=i32([0, 5]),
        reposition_raw_boundaries=i32([4]), reposition_insert_offsets=i32([5]))
    cases["err_token_id"] = dict(
        token_ids=np.asarray([1, 2, 2**31, 3], np.int64), drop_insert_offsets=i32([]),
        drop_range_offsets=i32([0]), drop_ranges=i32([]),
        reposition_raw_boundaries=i32([]), reposition_insert_offsets=i32([]))
    cases["err_unordered"] = dict(
        token_ids=np.arange(10, dtype=np.int64), drop_insert_offsets=i32([10]),
        drop_range_offsets=i32([0, 2]), drop_ranges=i32([5, 7, 1, 3]),
        reposition_raw_boundaries=i32([9]), reposition_insert_offsets=i32([10]))
    cases["err_unmaterialized"] = dict(
        token_ids=np.arange(10, dtype=np.int64), drop_insert_offsets=i32([4]),
        drop_range_offsets=i32([0, 1]), drop_ranges=i32([2, 6]),
        reposition_raw_boundaries=i32([]), reposition_insert_offsets=i32([]))

    out = {}
    for name, inp in cases.items():
        for k in INPUT_FIELDS:
            out[f"{name}/in/{k}"] = inp[k]
        try:
            lay = ir.compile_context_layout(*(_t(inp[k]) for k in INPUT_FIELDS))
        except Exception as exc:  # the reference's own error contract
            out[f"{name}/error"] = np.asarray(f"{type(exc).__name__}: {exc}")
            continue
        for k in LAYOUT_FIELDS:
            out[f"{name}/out/{k}"] = getattr(lay, k).numpy()
        out[f"{name}/out/next_position"] = np.asarray(lay.next_position, np.int64)
    return out


def page_table_cases(ir, pt):
    rng = np.random.default_rng(7)
    max_rows, ctx = 10, 4096
    table = rng.integers(1, 1 << 14, size=(max_rows, ctx)).astype(np.int32)
    overflow = {3: rng.integers(1, 1 << 14, size=5000).astype(np.int32)}
    rows = torch.zeros((max_rows, 6), dtype=torch.int64)
    keep_alive, logical = [], {}
    programs = {1: 700, 3: 3000, 5: 1200, 8: 64}
    for row, t in programs.items():
        inp = single_stage(workloads.c1_program(seed=row, tokens=max(t, 2000))) if t >= 2000 \
            else random_program(np.random.default_rng(row), t)
        if t >= 2000:
            inp = {k: v for k, v in inp.items()}
        lay = ir.compile_context_layout(*(_t(inp[k]) for k in INPUT_FIELDS))
        keep = lay.keep_mask.numpy()
        raw = np.flatnonzero(keep).astype(np.int32)
        pos = lay.positions.numpy()[raw].copy()
        packed = torch.from_numpy(np.concatenate((raw, pos)).astype(np.int32))
        if len(raw) == 0:
            packed = torch.zeros(1, dtype=torch.int32)
        keep_alive.append(packed)
        ids = packed[: len(raw)] if len(raw) else packed
        poss = packed[len(raw):] if len(raw) else packed
        row_ptr = 0
        if row in overflow:
            o = torch.from_numpy(overflow[row])
            keep_alive.append(o)
            row_ptr = o.data_ptr()
        prompt = len(keep)
        rows[row] = torch.tensor([ids.data_ptr(), poss.data_ptr(), prompt, len(raw),
                                  lay.next_position, row_ptr])
        logical[row] = dict(raw=raw, pos=pos, prompt=prompt, next_pos=lay.next_position)
    tbl = torch.from_numpy(table)
    out = {"table": table, "overflow_row": np.asarray(3), "overflow": overflow[3]}
    for row, d in logical.items():
        for k, v in d.items():
            out[f"row{row}/{k}"] = np.asarray(v)
    batch_rows = np.asarray([1, 0, 3, 5, 2, 8, 1], np.int64)
    generated = np.asarray([1, 0, 17, 3, 0, 1, 40], np.int64)
    seq = []
    for r, g in zip(batch_rows, generated):
        if r in logical:
            seq.append(len(logical[r]["raw"]) + g)
        else:
            seq.append(int(rng.integers(1, 3000)))
    seq_lens = torch.tensor(seq, dtype=torch.int64)
    row_ids = torch.from_numpy(batch_rows)
    out["batch_rows"], out["seq_lens"] = batch_rows, seq_lens.numpy()
    mapping = torch.from_numpy(rng.integers(0, 1 << 16, size=1 << 14).astype(np.int64))
    out["mapping"] = mapping.numpy()
    for window in (4, 128):
        lengths = torch.empty_like(seq_lens)
        pt.context_window_lengths[(len(seq_lens),)](rows, row_ids, seq_lens, lengths, window)
        out[f"window{window}/lengths"] = lengths.numpy().copy()
        starts = seq_lens - lengths
        indptr = torch.zeros(len(seq_lens) + 1, dtype=torch.int32)
        indptr[1:] = lengths.cumsum(0)
        for translate, mult in ((False, 1), (True, 1), (True, 4)):
            output = torch.full((int(indptr[-1]) + 3,), -7, dtype=torch.int32)
            pt.context_decode_indices[(len(seq_lens),)](
                rows, tbl, row_ids, lengths, indptr, output, starts,
                mapping if translate else None, ROW_STRIDE=tbl.stride(0), TRANSLATE=translate,
                MULTIPLIER=mult, HAS_START=True)
            out[f"window{window}/indices_t{int(translate)}_m{mult}"] = output.numpy().copy()
    indptr = torch.zeros(len(seq_lens) + 1, dtype=torch.int32)
    indptr[1:] = seq_lens.cumsum(0)
    output = torch.full((int(indptr[-1]) + 3,), -7, dtype=torch.int32)
    pt.context_decode_indices[(len(seq_lens),)](
        rows, tbl, row_ids, seq_lens, indptr, output, None, None,
        ROW_STRIDE=tbl.stride(0), TRANSLATE=False, MULTIPLIER=1, HAS_START=False)
    out["full/indices"] = output.numpy().copy()
    del keep_alive
    return out


def reposition_cases(rp):
    rng = np.random.default_rng(11)

    def bf16_values(shape):
        return torch.from_numpy(rng.standard_normal(shape).astype(np.float32)).bfloat16().float()

    specs = {
        "neox_d64": dict(n=32, layers=2, heads=8, dim=64, rot=64, neox=True, pad=0, skip=False),
        "gptj_d64": dict(n=30, layers=2, heads=4, dim=64, rot=64, neox=False, pad=0, skip=False),
        "neox_tail": dict(n=25, layers=2, heads=2, dim=128, rot=64, neox=True, pad=0, skip=False),
        "gptj_tail_pad": dict(n=20, layers=2, heads=3, dim=96, rot=32, neox=False, pad=16,
                              skip=False),
        "skip_unmapped": dict(n=30, layers=2, heads=2, dim=64, rot=64, neox=True, pad=0, skip=True),
        "odd_half": dict(n=12, layers=1, heads=2, dim=40, rot=24, neox=True, pad=0, skip=False),
    }
    out = {}
    for name, s in specs.items():
        slots = 2 * s["n"] + 8
        width = s["dim"] + s["pad"]
        k_full = [bf16_values((slots, s["heads"], width)) for _ in range(s["layers"])]
        v_full = [bf16_values((slots, s["heads"], width)) for _ in range(s["layers"])]
        ks = [k[..., : s["dim"]] for k in k_full]
        vs = [v[..., : s["dim"]] for v in v_full]
        perm = rng.permutation(np.arange(1, slots))
        src = perm[: s["n"]].astype(np.int32)
        dst = perm[s["n"]: 2 * s["n"]].astype(np.int32)
        if s["skip"]:
            src[::5] = 0
            dst[1::7] = -1
        max_pos = 300
        old = rng.integers(0, max_pos, size=s["n"])
        new = rng.integers(0, max_pos, size=s["n"])
        new[::6] = old[::6]  # same-position copies
        pairs = np.stack((old, new), 1).astype(np.int32)
        if name == "neox_d64":
            from akv_b200.rope import yarn_cos_sin_cache

            cache = yarn_cos_sin_cache(max_pos, s["rot"], 150000.0, 32.0, 4096)
        else:
            cache = bf16_values((max_pos, s["rot"]))  # bf16-representable table
        k_in = [k.clone() for k in k_full]
        v_in = [v.clone() for v in v_full]
        kp = torch.tensor([k.data_ptr() for k in ks], dtype=torch.int64)
        vp = torch.tensor([v.data_ptr() for v in vs], dtype=torch.int64)
        pairs_t = torch.from_numpy(pairs)
        rp._reposition_layers_kernel[(s["n"], s["layers"], s["heads"])](
            ks[0], kp, vp, torch.from_numpy(src), torch.from_numpy(dst), pairs_t, cache,
            ks[0].stride(0), ks[0].stride(1), vs[0].stride(0), vs[0].stride(1),
            pairs_t.stride(0), cache.stride(0), NEOX_STYLE=s["neox"], SKIP_UNMAPPED=s["skip"],
            head_dim=s["dim"], rotary_dim=s["rot"], half_dim=s["rot"] // 2,
            BLOCK_HALF=1 << max(0, (s["rot"] // 2 - 1).bit_length()),
            BLOCK_HEAD=1 << max(0, (s["dim"] - 1).bit_length()), num_warps=4,
            enable_fp_fusion=False)
        out[f"{name}/spec"] = np.asarray([s["n"], s["layers"], s["heads"], s["dim"], s["rot"],
                                          int(s["neox"]), s["pad"], int(s["skip"])])
        out[f"{name}/src"], out[f"{name}/dst"], out[f"{name}/pairs"] = src, dst, pairs
        out[f"{name}/cache"] = cache.numpy()
        # Inputs are bf16-representable: store their bf16 bit patterns.  Only
        # destination rows change; store those rows of the fp32 result.
        out[f"{name}/k_in"] = torch.stack(k_in).bfloat16().view(torch.int16).numpy()
        out[f"{name}/v_in"] = torch.stack(v_in).bfloat16().view(torch.int16).numpy()
        rows = torch.from_numpy(dst.astype(np.int64)).clamp(min=0)
        out[f"{name}/k_out_dst"] = torch.stack(k_full)[:, rows].numpy()
        out[f"{name}/v_out_dst"] = torch.stack(v_full)[:, rows].numpy()
        changed = np.zeros(slots, bool)
        changed[rows.numpy()] = True
        same = torch.stack(k_full)[:, ~torch.from_numpy(changed)] == torch.stack(k_in)[:, ~torch.from_numpy(changed)]
        assert bool(same.all()), "reference wrote outside its destination rows"
    return out


def row_slot_cases(rows_mod):
    rng = np.random.default_rng(5)
    arrays = [torch.from_numpy(rng.integers(0, 100, size=64).astype(np.int32)) for _ in range(4)]
    before = torch.stack(arrays).numpy().copy()
    pointers = torch.tensor([a.data_ptr() for a in arrays], dtype=torch.int64)
    n = 37
    rows = torch.from_numpy(rng.integers(0, 4, size=n).astype(np.int64))
    cols = torch.from_numpy(rng.choice(256, size=n, replace=False).astype(np.int64) % 64)
    # distinct (row, col) so the result does not depend on write order
    key = rows.numpy() * 64 + cols.numpy()
    _, first = np.unique(key, return_index=True)
    rows, cols = rows[np.sort(first)], cols[np.sort(first)]
    vals = torch.from_numpy(rng.integers(1000, 2000, size=len(rows)).astype(np.int32))
    block = 1 << (len(rows) - 1).bit_length()
    rows_mod.write_row_slots[(1,)](pointers, rows, cols, vals, N=len(rows), BLOCK=block)
    return dict(before=before, after=torch.stack(arrays).numpy(), rows=rows.numpy(),
                cols=cols.numpy(), values=vals.numpy())


def sink_cases(backend):
    rng = np.random.default_rng(3)
    bs, hq, d = 5, 8, 16
    o = rng.standard_normal((bs, hq, d)).astype(np.float32)
    lse = rng.standard_normal((bs, hq)).astype(np.float32) * 3
    sinks = rng.standard_normal(hq).astype(np.float32)

    def fake_kernel(*args, sinks=None, return_softmax_lse=False, **kwargs):
        # FA layout: lse is [heads, tokens]
        return torch.from_numpy(o.copy()), torch.from_numpy(lse.T.copy())

    res, res_lse = backend.flash_attention_with_sink(
        fake_kernel, sinks=torch.from_numpy(sinks), return_softmax_lse=True)
    return dict(o=o, lse=lse, sinks=sinks, out=res.numpy(), out_lse=res_lse.numpy().T.copy())


def main():
    ir, pt, rows_mod, rp, backend = reference_modules()
    np.savez_compressed(os.path.join(HERE, "event_compiler.npz"), **event_compiler_cases(ir))
    np.savez_compressed(os.path.join(HERE, "page_table.npz"), **page_table_cases(ir, pt))
    np.savez_compressed(os.path.join(HERE, "reposition.npz"), **reposition_cases(rp))
    np.savez_compressed(os.path.join(HERE, "row_slots.npz"), **row_slot_cases(rows_mod))
    np.savez_compressed(os.path.join(HERE, "sinks.npz"), **sink_cases(backend))
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
