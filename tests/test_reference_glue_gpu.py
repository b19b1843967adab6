"""The reference's own glue code calling this package as its overlay.

The reference imports its kernels lazily under
``sglang.kernels.ops.attention.context_reposition`` and
``...context_page_table`` (srt/layers/attention/context_backend.py:325, 438,
755-757, 789, 798-800).  Here those module names are bound to
``akv_b200.context_reposition`` / ``akv_b200.context_page_table`` and the
reference's unmodified ``context_backend.py`` (with its ``occurrence.py``
and ``request_storage.py``) is loaded from the reference package installed
in baseline/_ref (the ``reference_backend`` fixture of conftest.py); the test
is skipped when it is not installed.  Then the
reference's own classes run on the GPU:

* ``ContextModelBinding.reposition_existing`` (:432-472): layers grouped by
  shape / RoPE into one all-layer launch per group;
* ``ContextModelBinding.bind`` + ``ContextLayerCopy.apply`` (:302-341,
  :474-528): one launch per layer;
* ``ContextDecodeRegistry.bind_batch / fill / fill_table / fill_window``
  (:686-809): the decode page table, full and sliding-window.

K/V are compared bit for bit with the oracle's reposition, the page tables
with a numpy statement of context_page_table.py.
"""

from types import SimpleNamespace

import numpy as np
import pytest
import torch


pytestmark = pytest.mark.gpu



class Translator:
    """Identity slot translation (native pools without hybrid SWA memory)."""

    page_size = 1
    defer_read_translate = False
    is_translating = False

    def __init__(self, req_to_token=None):
        self.req_to_token = req_to_token

    def translate_full_attn_ids(self, ids):
        return ids

    def sliding_window_write_loc_for(self, ids):
        return None


def _model(n_layers, slots, heads, dim, rotary, cache, dev, seed):
    """A stand-in model (modules with ``attn`` and ``rotary_emb``) and pool,
    alternating sliding-window and full layers as GPT-OSS does."""
    g = torch.Generator(device=dev).manual_seed(seed)
    kv = {}
    modules = []
    for layer in range(n_layers):
        kv[layer] = (torch.randn(slots, heads, dim, device=dev, generator=g).to(torch.bfloat16),
                     torch.randn(slots, heads, dim, device=dev, generator=g).to(torch.bfloat16))
        attn = SimpleNamespace(layer_id=layer, sliding_window_size=128 if layer % 2 == 0 else -1)
        rope = SimpleNamespace(cos_sin_cache=cache, rotary_dim=rotary, is_neox_style=True)
        modules.append(SimpleNamespace(attn=attn, rotary_emb=rope))
    model = SimpleNamespace(modules=lambda: iter(modules))
    pool = SimpleNamespace(get_kv_buffer=lambda layer: kv[layer])
    return model, pool, kv


def _transitions(rng, n, slots, tokens):
    src = rng.choice(slots // 2, size=n, replace=False).astype(np.int32) + 1
    dst = (slots // 2 + 1 + rng.choice(slots // 2 - 2, size=n, replace=False)).astype(np.int32)
    old = rng.integers(0, tokens, size=n)
    new = np.maximum(0, old - rng.integers(0, 300, size=n))
    return src, dst, np.stack((old, new), 1).astype(np.int32)


def _expected(kv, src, dst, pairs, cache, rotary):
    from oracle import oracle

    ks = [kv[l][0].cpu().view(torch.int16).numpy().view(np.uint16).copy() for l in sorted(kv)]
    vs = [kv[l][1].cpu().view(torch.int16).numpy().view(np.uint16).copy() for l in sorted(kv)]
    oracle.reposition(ks, vs, src, dst, pairs, cache.cpu().numpy(), bf16=True,
                      rotary_dim=rotary)
    return ks, vs


def _compare(kv, ks, vs):
    for layer in sorted(kv):
        k, v = kv[layer]
        assert np.array_equal(k.cpu().view(torch.int16).numpy().view(np.uint16), ks[layer])
        assert np.array_equal(v.cpu().view(torch.int16).numpy().view(np.uint16), vs[layer])


@pytest.mark.parametrize("rotary", [64, 32])
def test_reposition_existing_through_the_reference_binding(reference_backend, rotary):
    from akv_b200.rope import yarn_cos_sin_cache

    dev = torch.device("cuda")
    cache = yarn_cos_sin_cache(8192, rotary, 150000.0, 32.0, 4096).to(dev)
    model, pool, kv = _model(4, 6000, 8, 64, rotary, cache, dev, seed=3)
    binding = reference_backend.ContextModelBinding(model, pool, Translator(), page_size=1)
    src, dst, pairs = _transitions(np.random.default_rng(1), 1500, 6000, 8000)
    ks, vs = _expected(kv, src, dst, pairs, cache, rotary)
    binding.reposition_existing(torch.from_numpy(src.astype(np.int64)).to(dev),
                                torch.from_numpy(dst.astype(np.int64)).to(dev),
                                torch.from_numpy(pairs).to(dev))
    torch.cuda.synchronize()
    _compare(kv, ks, vs)


def test_bind_and_layer_copies_through_the_reference_binding(reference_backend):
    from akv_b200.rope import yarn_cos_sin_cache

    dev = torch.device("cuda")
    cache = yarn_cos_sin_cache(8192, 64, 150000.0, 32.0, 4096).to(dev)
    model, pool, kv = _model(3, 5000, 8, 64, 64, cache, dev, seed=4)
    binding = reference_backend.ContextModelBinding(model, pool, Translator(), page_size=1)
    src, dst, pairs = _transitions(np.random.default_rng(2), 900, 5000, 8000)
    ks, vs = _expected(kv, src, dst, pairs, cache, 64)
    inputs = SimpleNamespace(
        occurrence_slots=torch.arange(10, device=dev),
        copy_sources=torch.from_numpy(src.astype(np.int64)).to(dev),
        copy_destinations=torch.from_numpy(dst.astype(np.int64)).to(dev),
        copy_positions=torch.from_numpy(pairs).to(dev),
        attention_plan=SimpleNamespace(bind=lambda slots: slots))
    metadata = binding.bind(inputs)
    assert sorted(metadata.layer_copies) == [0, 1, 2]
    for layer in sorted(metadata.layer_copies):
        metadata.layer_copies[layer].apply()
    torch.cuda.synchronize()
    _compare(kv, ks, vs)


def _decode_expect(layouts, table, rows, generated, window=None):
    """context_page_table.py:7-76 in numpy: each request's key slots (the
    compacted prompt then the generated tokens), or the last keys the
    window reaches."""
    out, lens = [], []
    for b, (lay, g) in enumerate(zip(layouts, generated)):
        row = table[rows[b]]
        if lay is None:  # ordinary request: min(length, window) keys (:16)
            raw = np.arange(g)
            n = min(g, window) if window is not None else g
            out.append(row[raw[len(raw) - n:]])
            lens.append(n)
            continue
        raw_ids, pos, prompt, nxt = lay
        keys = np.concatenate((raw_ids, prompt + np.arange(g)))
        n = len(keys)
        if window is not None:
            lower = nxt + g - 1 - window
            lo = int(np.searchsorted(pos, lower))
            n = len(raw_ids) - lo + g - max(0, lower - nxt)
        out.append(row[keys[len(keys) - n:]])
        lens.append(n)
    return out, np.asarray(lens)


def test_decode_registry_through_the_reference_code(reference_backend):
    from oracle import oracle

    dev = torch.device("cuda")
    rng = np.random.default_rng(5)
    batch = 12
    prompts = rng.integers(50, 3000, size=batch)
    generated = rng.integers(1, 40, size=batch)
    width = int((prompts + generated).max())
    table_np = rng.integers(1, 1 << 20, size=(batch + 3, width)).astype(np.int32)
    translator = Translator(torch.from_numpy(table_np).to(dev))
    registry = reference_backend.ContextDecodeRegistry(translator, SimpleNamespace())
    reqs, layouts, raw_lengths = [], [], []
    for b in range(batch):
        t = int(prompts[b])
        if b % 5 == 2:  # an ordinary request
            reqs.append(SimpleNamespace(context_program=None))
            layouts.append(None)
            raw_lengths.append(int(generated[b]))
            continue
        spans = np.sort(rng.choice(np.arange(t), size=6, replace=False)).astype(np.int32)
        lay = oracle.compile_layout(np.zeros(t, np.int64), [t], [0, 3], spans, [t - 1], [t])
        keep = np.asarray(lay["keep_mask"], bool)
        layout = SimpleNamespace(keep_mask=torch.from_numpy(keep),
                                 positions=torch.from_numpy(np.asarray(lay["positions"], np.int32)),
                                 next_position=int(lay["next_position"]))
        reqs.append(SimpleNamespace(context_program=SimpleNamespace(layout=layout),
                                    context_decode_layout=None))
        raw = np.flatnonzero(keep).astype(np.int32)
        layouts.append((raw, np.asarray(lay["positions"], np.int64)[raw], t,
                        int(lay["next_position"])))
        raw_lengths.append(t + int(generated[b]))
    gen = [g if lay is not None else raw_lengths[b] for b, (lay, g) in
           enumerate(zip(layouts, generated.tolist()))]
    rows = np.arange(batch) + 2
    row_ids = torch.from_numpy(rows.astype(np.int64)).to(dev)
    lengths, positions, _, refs = registry.bind_batch(reqs, raw_lengths, row_ids)
    seq_lens = lengths.to(dev)

    # fill: full attention over explicit CSR offsets
    want, want_len = _decode_expect(layouts, table_np, rows, gen)
    np.testing.assert_array_equal(lengths.numpy(), want_len)
    indptr = torch.from_numpy(np.concatenate(([0], np.cumsum(want_len))).astype(np.int32)).to(dev)
    out = torch.full((int(want_len.sum()),), -1, dtype=torch.int32, device=dev)
    registry.fill(row_ids, seq_lens, indptr, out)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), np.concatenate(want))

    # fill_table: the padded native table, full and window 128
    for window in (None, 128):
        table_out = torch.full((batch, width), -1, dtype=torch.int32, device=dev)
        got_len = registry.fill_table(row_ids, seq_lens, table_out, window=window)
        torch.cuda.synchronize()
        w, wl = _decode_expect(layouts, table_np, rows, gen, window)
        np.testing.assert_array_equal(got_len.cpu().numpy(), wl)
        t_np = table_out.cpu().numpy()
        for b in range(batch):
            np.testing.assert_array_equal(t_np[b, : wl[b]], w[b])
            assert np.all(t_np[b, wl[b]:] == -1)

    # fill_window: CSR over window 64
    win_indptr = torch.zeros(batch + 1, dtype=torch.int32, device=dev)
    win_out = torch.full((batch * 65,), -1, dtype=torch.int32, device=dev)
    indptr_w, _, wlen, starts = registry.fill_window(row_ids, seq_lens, win_indptr, 64, win_out)
    torch.cuda.synchronize()
    w, wl = _decode_expect(layouts, table_np, rows, gen, 64)
    np.testing.assert_array_equal(wlen.cpu().numpy(), wl)
    np.testing.assert_array_equal(starts.cpu().numpy(), want_len - wl)
    np.testing.assert_array_equal(win_out[: int(wl.sum())].cpu().numpy(), np.concatenate(w))
    del refs
