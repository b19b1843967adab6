"""The CPU oracle against golden vectors produced by the reference itself.

Golden vectors come from tests/golden/make_golden.py, which ran the
reference's C++ event compiler and its Triton kernels (CPU interpreter).
These tests pin the oracle; the GPU tests then compare the CUDA path with
the pinned oracle.
"""

import numpy as np
import pytest

from conftest import golden
from oracle import oracle

EC = golden("event_compiler")
EC_CASES = sorted({k.split("/")[0] for k in EC.files})
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


@pytest.mark.parametrize("case", EC_CASES)
def test_event_compiler_matches_reference(case):
    inp = [EC[f"{case}/in/{k}"] for k in INPUTS]
    err_key = f"{case}/error"
    if err_key in EC.files:
        message = str(EC[err_key])
        if "exceeds the signed int32 range" in message:
            # ir.py:148-153 rejects before the compiler runs; the oracle sees
            # the same out-of-range id through status[0] == 2.
            with pytest.raises(ValueError):
                oracle.compile_layout(*inp)
            return
        with pytest.raises(ValueError) as exc:
            oracle.compile_layout(*inp)
        if "no active tokens" in message:
            assert str(exc.value) == message.split(": ", 1)[1]
        return
    got = oracle.compile_layout(*inp)
    for f in FIELDS:
        want = EC[f"{case}/out/{f}"]
        np.testing.assert_array_equal(np.asarray(got[f]).astype(want.dtype), want, err_msg=f)
    assert got["next_position"] == int(EC[f"{case}/out/next_position"])


def test_decode_layout_is_strictly_increasing():
    inp = [EC[f"c1/in/{k}"] for k in INPUTS]
    raw, pos, prompt, nxt = oracle.decode_layout(oracle.compile_layout(*inp))
    assert prompt == 4096 and np.all(np.diff(pos) > 0)
    np.testing.assert_array_equal(pos, np.arange(len(raw)))
    assert nxt == len(raw)


PT = golden("page_table")


def _registry():
    reg = oracle.HostRegistry(10)
    overflow_row = int(PT["overflow_row"])
    for row in (1, 3, 5, 8):
        reg.set_context(row, PT[f"row{row}/raw"], PT[f"row{row}/pos"], int(PT[f"row{row}/prompt"]),
                        int(PT[f"row{row}/next_pos"]),
                        PT["overflow"] if row == overflow_row else None)
    return reg


@pytest.mark.parametrize("window", [4, 128])
def test_window_lengths_match_reference(window):
    reg = _registry()
    got = oracle.window_lengths(reg, PT["batch_rows"], PT["seq_lens"], window)
    np.testing.assert_array_equal(got, PT[f"window{window}/lengths"])


@pytest.mark.parametrize("window", [4, 128])
@pytest.mark.parametrize("translate,mult", [(0, 1), (1, 1), (1, 4)])
def test_decode_indices_match_reference(window, translate, mult):
    reg = _registry()
    lengths = PT[f"window{window}/lengths"]
    starts = PT["seq_lens"] - lengths
    indptr = np.concatenate(([0], np.cumsum(lengths)))
    want = PT[f"window{window}/indices_t{translate}_m{mult}"]
    got = oracle.decode_indices(reg, PT["table"], PT["batch_rows"], lengths, indptr, len(want),
                                starts=starts, mapping=PT["mapping"] if translate else None,
                                multiplier=mult)
    n = int(indptr[-1])
    np.testing.assert_array_equal(got[:n].astype(np.int32), want[:n])
    assert np.all(want[n:] == -7)


def test_decode_indices_full_match_reference():
    reg = _registry()
    seq = PT["seq_lens"]
    indptr = np.concatenate(([0], np.cumsum(seq)))
    want = PT["full/indices"]
    got = oracle.decode_indices(reg, PT["table"], PT["batch_rows"], seq, indptr, len(want))
    n = int(indptr[-1])
    np.testing.assert_array_equal(got[:n].astype(np.int32), want[:n])


def test_window_lengths_cpu_twin_agrees_for_context_rows():
    # context_backend.py:742-752 vs the device kernel for rows with context.
    reg = _registry()
    rows, seq = PT["batch_rows"], PT["seq_lens"]
    for window in (4, 128):
        dev = oracle.window_lengths(reg, rows, seq, window)
        layouts = []
        for r, s in zip(rows, seq):
            if int(r) in (1, 3, 5, 8):
                layouts.append(((PT[f"row{r}/pos"], int(PT[f"row{r}/next_pos"])),
                                int(s) - len(PT[f"row{r}/raw"])))
            else:
                layouts.append((None, int(s)))
        cpu = oracle.window_lengths_cpu(layouts, window, len(rows))
        ctx = np.isin(rows, [1, 3, 5, 8])
        np.testing.assert_array_equal(cpu[ctx], dev[ctx])


RP = golden("reposition")
RP_CASES = sorted({k.split("/")[0] for k in RP.files})


def _bits_to_f32(bits):
    return (bits.astype(np.uint16).astype(np.uint32) << 16).view(np.float32)


def _f32_to_bf16_bits(x):
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), r)


def _reposition_case(case, storage):
    n, layers, heads, dim, rot, neox, pad, skip = (int(x) for x in RP[f"{case}/spec"])
    k_bits, v_bits = RP[f"{case}/k_in"], RP[f"{case}/v_in"]
    if storage == "f32":
        k_full = [np.ascontiguousarray(_bits_to_f32(k_bits[i])) for i in range(layers)]
        v_full = [np.ascontiguousarray(_bits_to_f32(v_bits[i])) for i in range(layers)]
    else:
        k_full = [np.ascontiguousarray(k_bits[i].view(np.uint16)) for i in range(layers)]
        v_full = [np.ascontiguousarray(v_bits[i].view(np.uint16)) for i in range(layers)]
    ks = [k[..., :dim] for k in k_full]
    vs = [v[..., :dim] for v in v_full]
    oracle.reposition(ks, vs, RP[f"{case}/src"], RP[f"{case}/dst"], RP[f"{case}/pairs"],
                      RP[f"{case}/cache"], is_neox_style=bool(neox), skip_unmapped=bool(skip),
                      rotary_dim=rot, bf16=(storage == "bf16"))
    return k_full, v_full, dim


@pytest.mark.parametrize("case", RP_CASES)
def test_reposition_fp32_bit_exact(case):
    k_full, v_full, dim = _reposition_case(case, "f32")
    dst = np.clip(RP[f"{case}/dst"].astype(np.int64), 0, None)
    for layer in range(len(k_full)):
        np.testing.assert_array_equal(k_full[layer][dst], RP[f"{case}/k_out_dst"][layer])
        np.testing.assert_array_equal(v_full[layer][dst], RP[f"{case}/v_out_dst"][layer])


@pytest.mark.parametrize("case", RP_CASES)
def test_reposition_bf16_is_rne_of_reference_fp32(case):
    k_full, v_full, dim = _reposition_case(case, "bf16")
    dst = np.clip(RP[f"{case}/dst"].astype(np.int64), 0, None)
    for layer in range(len(k_full)):
        np.testing.assert_array_equal(k_full[layer][dst],
                                      _f32_to_bf16_bits(RP[f"{case}/k_out_dst"][layer]))
        np.testing.assert_array_equal(v_full[layer][dst],
                                      _f32_to_bf16_bits(RP[f"{case}/v_out_dst"][layer]))


def test_write_row_slots_match_reference():
    z = golden("row_slots")
    arrays = [np.array(r, np.int32) for r in z["before"]]
    oracle.write_row_slots(arrays, z["rows"], z["cols"], z["values"])
    np.testing.assert_array_equal(np.stack(arrays), z["after"])


def test_sink_correction_matches_reference():
    z = golden("sinks")
    # Reproduce flash_attention_with_sink's output from (o, lse, sinks) with
    # the oracle's definition: o * sigmoid(lse - sink).
    o, lse, sinks = z["o"].astype(np.float64), z["lse"].astype(np.float64), z["sinks"]
    want = o * (1 / (1 + np.exp(-(lse - sinks[None, :]))))[..., None]
    np.testing.assert_allclose(z["out"], want, rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(z["out_lse"], np.logaddexp(lse, sinks[None, :]), rtol=1e-6,
                               atol=1e-6)


def test_attention_oracle_sink_is_extra_softmax_column():
    rng = np.random.default_rng(0)
    bs, hq, hkv, d, slots = 3, 8, 2, 16, 50
    q = rng.standard_normal((bs, hq, d))
    k = rng.standard_normal((slots, hkv, d))
    v = rng.standard_normal((slots, hkv, d))
    sinks = rng.standard_normal(hq)
    lens = [5, 0, 17]
    indptr = np.concatenate(([0], np.cumsum(lens)))
    idx = rng.integers(0, slots, size=indptr[-1])
    out, _ = oracle.decode_attention(q, k, v, indptr, idx, sinks)
    for b in range(bs):
        ids = idx[indptr[b]: indptr[b + 1]]
        for h in range(hq):
            s = k[ids, h // 4] @ q[b, h] / np.sqrt(d)
            col = np.concatenate((s, [sinks[h]]))
            w = np.exp(col - col.max())
            w /= w.sum()
            np.testing.assert_allclose(out[b, h], w[:-1] @ v[ids, h // 4], atol=1e-12)
