"""Decode page-table kernels against the reference's Triton kernels.

Golden values come from the reference's context_decode_indices /
context_window_lengths / write_row_slots run under the Triton CPU
interpreter (tests/golden/make_golden.py); a large lognormal batch is
checked against the pinned CPU oracle.  Integer outputs: bit-exact.
"""

import numpy as np
import pytest
import torch

from conftest import golden

pytestmark = pytest.mark.gpu

PT = golden("page_table")
CTX_ROWS = (1, 3, 5, 8)


class DeviceRegistry:
    """Registry rows on the device, pointing at device copies of each row's
    compacted raw ids / positions (context_backend.py:680-684, 716-725)."""

    def __init__(self, max_rows, dev):
        self.rows = torch.zeros((max_rows, 6), dtype=torch.int64, device=dev)
        self.keep = []
        self.dev = dev

    def set(self, row, raw, pos, prompt, next_pos, overflow=None):
        packed = torch.from_numpy(np.concatenate((raw, pos)).astype(np.int32)).to(self.dev)
        if len(raw) == 0:
            packed = torch.zeros(1, dtype=torch.int32, device=self.dev)
        self.keep.append(packed)
        ids = packed[: len(raw)] if len(raw) else packed
        poss = packed[len(raw):] if len(raw) else packed
        rp = 0
        if overflow is not None:
            o = torch.from_numpy(np.asarray(overflow, np.int32)).to(self.dev)
            self.keep.append(o)
            rp = o.data_ptr()
        self.rows[row] = torch.tensor([ids.data_ptr(), poss.data_ptr(), prompt, len(raw),
                                       next_pos, rp], dtype=torch.int64)


def _golden_registry(dev):
    reg = DeviceRegistry(10, dev)
    for row in CTX_ROWS:
        reg.set(row, PT[f"row{row}/raw"], PT[f"row{row}/pos"], int(PT[f"row{row}/prompt"]),
                int(PT[f"row{row}/next_pos"]),
                PT["overflow"] if row == int(PT["overflow_row"]) else None)
    return reg


@pytest.mark.parametrize("window", [4, 128])
@pytest.mark.parametrize("idx_dtype", [torch.int64, torch.int32])
def test_window_lengths_match_reference(window, idx_dtype):
    from akv_b200.context_page_table import context_window_lengths

    dev = torch.device("cuda")
    reg = _golden_registry(dev)
    rows = torch.from_numpy(PT["batch_rows"]).to(dev).to(idx_dtype)
    seq = torch.from_numpy(PT["seq_lens"]).to(dev).to(idx_dtype)
    out = torch.empty_like(seq)
    context_window_lengths[(len(seq),)](reg.rows, rows, seq, out, window)
    np.testing.assert_array_equal(out.cpu().numpy(), PT[f"window{window}/lengths"])


@pytest.mark.parametrize("window", [4, 128])
@pytest.mark.parametrize("translate,mult", [(False, 1), (True, 1), (True, 4)])
@pytest.mark.parametrize("out_dtype", [torch.int32, torch.int64])
def test_decode_indices_match_reference(window, translate, mult, out_dtype):
    from akv_b200.context_page_table import context_decode_indices

    dev = torch.device("cuda")
    reg = _golden_registry(dev)
    table = torch.from_numpy(PT["table"]).to(dev)
    rows = torch.from_numpy(PT["batch_rows"]).to(dev)
    seq = torch.from_numpy(PT["seq_lens"]).to(dev)
    lengths = torch.from_numpy(PT[f"window{window}/lengths"]).to(dev)
    starts = seq - lengths
    indptr = torch.zeros(len(seq) + 1, dtype=torch.int32, device=dev)
    indptr[1:] = lengths.cumsum(0)
    want = PT[f"window{window}/indices_t{int(translate)}_m{mult}"]
    out = torch.full((len(want),), -7, dtype=out_dtype, device=dev)
    mapping = torch.from_numpy(PT["mapping"]).to(dev) if translate else None
    context_decode_indices[(len(seq),)](reg.rows, table, rows, lengths, indptr, out, starts,
                                        mapping, ROW_STRIDE=table.stride(0), TRANSLATE=translate,
                                        MULTIPLIER=mult, HAS_START=True)
    np.testing.assert_array_equal(out.cpu().numpy().astype(np.int32), want)


def test_decode_indices_full_match_reference():
    from akv_b200.context_page_table import context_decode_indices

    dev = torch.device("cuda")
    reg = _golden_registry(dev)
    table = torch.from_numpy(PT["table"]).to(dev)
    rows = torch.from_numpy(PT["batch_rows"]).to(dev)
    seq = torch.from_numpy(PT["seq_lens"]).to(dev)
    indptr = torch.zeros(len(seq) + 1, dtype=torch.int32, device=dev)
    indptr[1:] = seq.cumsum(0)
    want = PT["full/indices"]
    out = torch.full((len(want),), -7, dtype=torch.int32, device=dev)
    context_decode_indices[(len(seq),)](reg.rows, table, rows, seq, indptr, out, None, None,
                                        ROW_STRIDE=table.stride(0), TRANSLATE=False,
                                        MULTIPLIER=1, HAS_START=False)
    np.testing.assert_array_equal(out.cpu().numpy(), want)


def test_write_row_slots_match_reference():
    from akv_b200.context_rows import write_row_slots

    z = golden("row_slots")
    dev = torch.device("cuda")
    arrays = [torch.from_numpy(r.copy()).to(dev) for r in z["before"]]
    pointers = torch.tensor([a.data_ptr() for a in arrays], dtype=torch.int64, device=dev)
    rows = torch.from_numpy(z["rows"]).to(dev)
    cols = torch.from_numpy(z["cols"]).to(dev)
    vals = torch.from_numpy(z["values"]).to(dev)
    write_row_slots[(1,)](pointers, rows, cols, vals, N=len(rows), BLOCK=64)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(torch.stack(arrays).cpu().numpy(), z["after"])


def _c4_registry(dev, rng, batch=128, gapped=False, median=8192):
    """A c4-shaped batch: lognormal prompt lengths, drops applied through the
    oracle compiler, a few generated tokens per request."""
    from oracle import oracle
    from akv_b200 import workloads

    lengths = workloads.c4_lengths(batch=batch, median=median)
    max_ctx = int(lengths.max()) + 64
    table = rng.integers(1, 1 << 24, size=(batch + 1, max_ctx)).astype(np.int32)
    host = oracle.HostRegistry(batch + 1)
    reg = DeviceRegistry(batch + 1, dev)
    seq = []
    for b, t in enumerate(lengths):
        t = int(t)
        n_spans = int(rng.integers(0, 4))
        spans = np.sort(rng.choice(np.arange(t), size=2 * n_spans, replace=False)) \
            if t > 2 * n_spans + 1 else np.zeros(0, int)
        spans = spans.astype(np.int32)
        has = len(spans) > 0
        lay = oracle.compile_layout(np.zeros(t, np.int64), [t] if has else [],
                                    [0, len(spans) // 2] if has else [0], spans,
                                    [] if gapped else [t - 1], [] if gapped else [t])
        raw, pos, prompt, nxt = oracle.decode_layout(lay)
        row = b + 1 if b % 7 else 0  # row 0 is an ordinary request
        gen = int(rng.integers(1, 9))
        if row == 0:
            seq.append(int(rng.integers(1, max_ctx)))
            continue
        host.set_context(row, raw, pos, prompt, nxt)
        reg.set(row, raw, pos, prompt, nxt)
        seq.append(len(raw) + gen)
    rows = np.asarray([b + 1 if b % 7 else 0 for b in range(batch)], np.int64)
    return host, reg, table, rows, np.asarray(seq, np.int64)


@pytest.mark.parametrize("window", [None, 128, 1])
@pytest.mark.parametrize("gapped", [False, True])
@pytest.mark.parametrize("batch,median", [(128, 8192), (1, 8192), (3, 300), (1100, 200)])
def test_build_decode_metadata_c4_matches_oracle(window, gapped, batch, median):
    """Batches up to 1,024 requests take the key-balanced kernel, larger ones
    the per-request split; both against the oracle."""
    from oracle import oracle
    from akv_b200.context_page_table import build_decode_metadata

    dev = torch.device("cuda")
    rng = np.random.default_rng(11 + batch)
    host, reg, table, rows, seq = _c4_registry(dev, rng, batch=batch, gapped=gapped,
                                               median=median)
    if window is None:
        lengths = seq
        starts = None
    else:
        lengths = oracle.window_lengths(host, rows, seq, window)
        starts = seq - lengths
    indptr = np.concatenate(([0], np.cumsum(lengths)))
    want = oracle.decode_indices(host, table, rows, lengths, indptr, int(indptr[-1]),
                                 starts=starts)
    kv_indptr = torch.empty(len(seq) + 1, dtype=torch.int32, device=dev)
    kv_indices = torch.empty(int(indptr[-1]), dtype=torch.int32, device=dev)
    _, lens, sts = build_decode_metadata(reg.rows, torch.from_numpy(table).to(dev),
                                         torch.from_numpy(rows).to(dev),
                                         torch.from_numpy(seq).to(dev), kv_indptr, kv_indices,
                                         window=window)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(kv_indptr.cpu().numpy(), indptr)
    np.testing.assert_array_equal(kv_indices.cpu().numpy(), want.astype(np.int32))
    if window is not None:
        np.testing.assert_array_equal(lens.cpu().numpy(), lengths)
        np.testing.assert_array_equal(sts.cpu().numpy(), starts)


@pytest.mark.parametrize("window", [None, 128])
@pytest.mark.parametrize("batch,median", [(128, 2000), (1100, 100)])
def test_decode_indices_padded_table_matches_oracle(window, batch, median):
    """The registry's fill_table layout (context_backend.py:785-796): one
    table row per request, kv_indptr = arange(bs + 1) * row stride, so the
    index space has gaps that must stay untouched.  Up to 1,000 requests
    take the key-balanced kernel, more the per-request split."""
    from oracle import oracle
    from akv_b200.context_page_table import context_decode_indices

    dev = torch.device("cuda")
    rng = np.random.default_rng(5 + batch)
    host, reg, table, rows, seq = _c4_registry(dev, rng, batch=batch, median=median)
    if window is None:
        lengths, starts = seq, None
    else:
        lengths = oracle.window_lengths(host, rows, seq, window)
        starts = seq - lengths
    stride = int(seq.max()) + 5
    indptr = np.arange(batch + 1, dtype=np.int64) * stride
    want = oracle.decode_indices(host, table, rows, lengths, indptr, batch * stride,
                                 starts=starts)
    out = torch.zeros(batch * stride, dtype=torch.int32, device=dev)
    t = lambda a, dt: torch.from_numpy(np.asarray(a)).to(dev, dt)  # noqa: E731
    context_decode_indices[(batch,)](
        reg.rows, torch.from_numpy(table).to(dev), t(rows, torch.int64),
        t(lengths, torch.int64), t(indptr, torch.int32), out,
        None if starts is None else t(starts, torch.int64), None,
        ROW_STRIDE=table.shape[1], TRANSLATE=False, MULTIPLIER=1,
        HAS_START=starts is not None)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), want.astype(np.int32))


@pytest.mark.parametrize("window", [None, 128])
def test_decode_metadata_replays_from_a_cuda_graph(window):
    """The reference keeps its decode registry capture-stable so a decode
    step's metadata launches can live in a CUDA graph
    (context_backend.py:667-672): here the metadata launches of one step
    are captured once, then the sequence lengths grow in place between
    replays, as decode steps do; every replay equals the oracle."""
    from oracle import oracle
    from akv_b200.context_page_table import build_decode_metadata, context_window_lengths

    dev = torch.device("cuda")
    rng = np.random.default_rng(21)
    host, reg, table, rows, seq = _c4_registry(dev, rng, batch=96, median=1500)
    steps = 4
    # ordinary requests read their table row directly: keep them inside it
    seq = np.minimum(seq, table.shape[1] - steps - 1)
    cap = int((seq + steps).sum())
    d_table = torch.from_numpy(table).to(dev)
    d_rows = torch.from_numpy(rows).to(dev)
    d_seq = torch.from_numpy(seq).to(dev)
    kv_indptr = torch.empty(len(seq) + 1, dtype=torch.int32, device=dev)
    kv_indices = torch.full((cap,), -7, dtype=torch.int32, device=dev)
    lens = torch.empty(len(seq), dtype=torch.int64, device=dev)
    starts = torch.empty(len(seq), dtype=torch.int64, device=dev)
    wl = torch.empty(len(seq), dtype=torch.int64, device=dev)

    def step():
        build_decode_metadata(reg.rows, d_table, d_rows, d_seq, kv_indptr, kv_indices,
                              window=window, lengths_out=lens, starts_out=starts)
        if window is not None:
            context_window_lengths[(len(seq),)](reg.rows, d_rows, d_seq, wl, window)

    step()  # first launch outside the capture
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(steps):
        seq = seq + 1
        d_seq.copy_(torch.from_numpy(seq))
        graph.replay()
        torch.cuda.synchronize()
        lengths = seq if window is None else oracle.window_lengths(host, rows, seq, window)
        indptr = np.concatenate(([0], np.cumsum(lengths)))
        want = oracle.decode_indices(host, table, rows, lengths, indptr, int(indptr[-1]),
                                     starts=None if window is None else seq - lengths)
        np.testing.assert_array_equal(kv_indptr.cpu().numpy(), indptr)
        np.testing.assert_array_equal(kv_indices[: int(indptr[-1])].cpu().numpy(),
                                      want.astype(np.int32))
        if window is not None:
            np.testing.assert_array_equal(lens.cpu().numpy(), lengths)
            np.testing.assert_array_equal(wl.cpu().numpy(), lengths)
    del graph
