"""Drop + Reposition over a paged KV pool (C ABI akv_drop_compact_paged).

The reference has no paged Reposition (context_reposition.py:153-154 and
capabilities.py:11-12 require page_size 1), so parity is pinned two ways:

* every integer output against ``oracle.drop_compact_paged``, whose
  positions, decode view and transition pairs are those of the page_size 1
  oracle (itself pinned to the reference's compiler);
* the data: a batch run at page_size 1 and at page_size 16 from the same
  logical K/V must leave the same logical K/V behind when each request's
  compacted view is gathered through its own rows, bit for bit.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _table(program, rows, dev):
    nreq = program.requests
    width = max(1, int(program.token_counts.max()) if nreq else 1)
    table = np.zeros((nreq + 1, width), np.int32)
    row_ids = np.arange(nreq, dtype=np.int64) + 1
    for r in range(nreq):
        table[row_ids[r], : len(rows[r])] = rows[r]
    return torch.from_numpy(table).to(dev), row_ids


def _run(program, rows, free_pages, page_size, reposition=True, capacity=None):
    from akv_b200.context_drop import DropCompactor, FreeSlotRing

    dev = torch.device("cuda")
    req_to_token, row_ids = _table(program, rows, dev)
    ring = FreeSlotRing(torch.from_numpy(np.asarray(free_pages, np.int32)),
                        capacity=capacity or len(free_pages) + program.total_tokens + 1,
                        device=dev)
    comp = DropCompactor(program.total_tokens, program.requests,
                         max(1, len(program.ranges) // 2), dev)
    shared = program.shared_prefix if program.shared_prefix.any() else None
    res = comp.run(program.token_counts, program.range_offsets, program.ranges, req_to_token,
                   row_ids, ring, shared_prefix=shared, reposition=reposition,
                   page_size=page_size)
    torch.cuda.synchronize()
    return res, req_to_token, row_ids, ring


def _check(program, rows, free_pages, page_size, reposition=True):
    from oracle import oracle

    res, req_to_token, row_ids, ring = _run(program, rows, free_pages, page_size, reposition)
    want = oracle.drop_compact_paged(program.token_counts, program.range_offsets,
                                     program.ranges, rows, page_size,
                                     shared_prefix=program.shared_prefix, reposition=reposition,
                                     free_pages=np.asarray(free_pages, np.int32),
                                     free_tail=len(free_pages))
    res.check()
    kept = sum(len(x) for x in want["raw_indices"])
    n, f = len(want["src"]), len(want["freed"])
    assert res.totals.cpu().tolist() == [kept, n, want["copied_pages"], f]
    ao = res.active_offsets.cpu().numpy()
    raw = res.raw_indices[:kept].cpu().numpy()
    apos = res.active_positions[:kept].cpu().numpy()
    for r in range(program.requests):
        np.testing.assert_array_equal(raw[ao[r]: ao[r + 1]], want["raw_indices"][r])
        np.testing.assert_array_equal(apos[ao[r]: ao[r + 1]], want["active_positions"][r])
    np.testing.assert_array_equal(res.next_position.cpu().numpy(), want["next_position"])
    np.testing.assert_array_equal(res.transition_source[:n].cpu().numpy(), want["src"])
    np.testing.assert_array_equal(res.transition_destination[:n].cpu().numpy(), want["dst"])
    np.testing.assert_array_equal(res.transition_pairs[:n].cpu().numpy(), want["pairs"])
    np.testing.assert_array_equal(res.transition_raw[:n].cpu().numpy(), want["raw"])
    np.testing.assert_array_equal(res.freed_slots[:f].cpu().numpy(), want["freed"])
    assert ring.state.cpu().tolist() == [want["free_head"], want["free_tail"]]
    idx = np.arange(len(free_pages), want["free_tail"]) % ring.capacity
    np.testing.assert_array_equal(ring.ring.cpu().numpy()[idx], want["freed"])
    table = req_to_token.cpu().numpy()
    for r in range(program.requests):
        np.testing.assert_array_equal(table[row_ids[r], : len(rows[r])], want["rows"][r])
        # the layout rule still holds after copy-on-write
        t = np.arange(len(rows[r]))
        row = table[row_ids[r], : len(rows[r])]
        assert np.all(row % page_size == t % page_size)
    return res, want


@pytest.mark.parametrize("page_size", [16, 64, 4, 128])
def test_paged_c3_shape_matches_oracle(page_size):
    from akv_b200 import workloads

    prog = workloads.c3_program(requests=12, max_len=9000, seed=5, page_align=page_size)
    rows, n_pages = workloads.paged_slot_rows(np.random.default_rng(5), prog, page_size)
    need = -(-int(prog.shared_prefix.sum()) // page_size) + prog.requests
    free = np.arange(n_pages, n_pages + need)
    res, want = _check(prog, rows, free, page_size)
    assert want["copied_pages"] > 0 and len(want["freed"]) > 0


def test_paged_reposition_off_matches_oracle():
    from akv_b200 import workloads

    prog = workloads.c3_program(requests=5, max_len=6000, seed=8, page_align=16)
    rows, n_pages = workloads.paged_slot_rows(np.random.default_rng(8), prog, 16)
    _, want = _check(prog, rows, np.arange(n_pages, n_pages + 4), 16, reposition=False)
    assert len(want["src"]) == 0


def test_paged_edge_cases_match_oracle():
    """Partial last pages, pages dropped whole at the ends and in the middle,
    an empty request, a request with no drop, one dropped token per page."""
    from akv_b200 import workloads
    from akv_b200.workloads import DropProgram

    counts = np.array([1000, 0, 77, 2049, 16, 530])
    per = [[32, 64, 100, 101, 990, 1000], [], [], [0, 16, 2040, 2049],
           [3, 4], [i for p in range(0, 512, 16) for i in (p + 5, p + 6)] + [512, 530]]
    offsets = np.cumsum([0] + [len(p) // 2 for p in per]).astype(np.int32)
    ranges = np.concatenate([np.asarray(p, np.int32) for p in per])
    shared = np.array([48, 0, 32, 0, 16, 0])
    prog = DropProgram(counts, offsets, ranges, shared)
    rows, n_pages = workloads.paged_slot_rows(np.random.default_rng(2), prog, 16)
    _check(prog, rows, np.arange(n_pages, n_pages + 50), 16)


def test_paged_layout_violation_is_rejected_whole():
    """A row whose slot offsets do not follow the tokens: status
    AKV_DROP_BAD_PAGE, nothing emitted, ring and rows untouched."""
    from akv_b200 import _native, workloads

    prog = workloads.c3_program(requests=4, max_len=5000, seed=2, page_align=16)
    rows, n_pages = workloads.paged_slot_rows(np.random.default_rng(2), prog, 16)
    rows[2] = rows[2].copy()
    rows[2][[40, 41]] = rows[2][[41, 40]]  # two tokens of one page swapped
    res, req_to_token, row_ids, ring = _run(prog, rows, np.arange(n_pages, n_pages + 300), 16)
    assert int(res.status.item()) & _native.DROP_BAD_PAGE
    assert res.totals[1:].cpu().tolist() == [0, 0, 0]
    assert ring.state.cpu().tolist() == [0, 300]
    table = req_to_token.cpu().numpy()
    for r in range(prog.requests):
        np.testing.assert_array_equal(table[row_ids[r], : len(rows[r])], rows[r])
    with pytest.raises(RuntimeError, match="page layout"):
        res.check()


def test_paged_rejects_unaligned_prefix_and_bad_page_size():
    from akv_b200 import workloads
    from akv_b200.context_drop import DropCompactor

    prog = workloads.c3_program(requests=2, max_len=4000, seed=1)
    comp = DropCompactor(prog.total_tokens, 2, 64, "cuda")
    shared = prog.shared_prefix.copy()
    shared[:] = 33
    with pytest.raises(ValueError, match="whole number of pages"):
        comp.prepare(prog.token_counts, prog.range_offsets, prog.ranges, [0, 1],
                     shared_prefix=shared, page_size=16)
    with pytest.raises(ValueError, match="power of two"):
        comp.prepare(prog.token_counts, prog.range_offsets, prog.ranges, [0, 1], page_size=12)


def _logical_pools(rng_seed, program, rows, n_slots, layers, heads, dim, dev):
    """K/V pools that hold the same logical content (one value per request
    token, shared prefix tokens the same for every request) at each
    request's slots."""
    g = torch.Generator(device=dev).manual_seed(rng_seed)
    prefix = int(program.shared_prefix.max())
    private = int((program.token_counts - program.shared_prefix).sum())
    content = [(torch.randn(prefix + private, heads, dim, device=dev, generator=g)
                .to(torch.bfloat16),
                torch.randn(prefix + private, heads, dim, device=dev, generator=g)
                .to(torch.bfloat16)) for _ in range(layers)]
    logical, cursor = [], prefix
    for r in range(program.requests):
        t, p = int(program.token_counts[r]), int(program.shared_prefix[r])
        logical.append(np.concatenate((np.arange(p), cursor + np.arange(t - p))))
        cursor += t - p
    slots = torch.from_numpy(np.concatenate(rows).astype(np.int64)).to(dev)
    ids = torch.from_numpy(np.concatenate(logical)).to(dev)
    k_pools, v_pools = [], []
    for kc, vc in content:
        k = torch.zeros(n_slots, heads, dim, device=dev, dtype=torch.bfloat16)
        v = torch.zeros_like(k)
        k[slots] = kc[ids]
        v[slots] = vc[ids]
        k_pools.append(k)
        v_pools.append(v)
    return k_pools, v_pools


@pytest.mark.parametrize("bulk", [False, True])
@pytest.mark.parametrize("page_size", [16])
def test_paged_and_unpaged_runs_leave_the_same_logical_kv(page_size, bulk):
    from akv_b200 import workloads
    from akv_b200.context_reposition import layer_pointer_table, reposition_kv_layers
    from akv_b200.rope import yarn_cos_sin_cache

    dev = torch.device("cuda")
    layers, heads, dim = 3, 8, 64
    prog = workloads.c3_program(requests=10, max_len=7000, seed=4, page_align=page_size)
    cache = yarn_cos_sin_cache(8192, dim, 150000.0, 32.0, 4096).to(dev)
    views = {}
    for ps in (1, page_size):
        if ps == 1:
            rows, n_slots = workloads.slot_rows(np.random.default_rng(4), prog)
            free = np.arange(n_slots, n_slots + int(prog.shared_prefix.sum()))
            total_slots = n_slots + len(free)
        else:
            rows, n_pages = workloads.paged_slot_rows(np.random.default_rng(4), prog, ps)
            need = -(-int(prog.shared_prefix.sum()) // ps) + prog.requests
            free = np.arange(n_pages, n_pages + need)
            total_slots = (n_pages + need) * ps
        k_pools, v_pools = _logical_pools(77, prog, rows, total_slots, layers, heads, dim, dev)
        res, req_to_token, row_ids, _ = _run(prog, rows, free, ps)
        res.check()
        reposition_kv_layers(layer_pointer_table(k_pools), layer_pointer_table(v_pools),
                             k_pools[0], v_pools[0], res.transition_source,
                             res.transition_destination, res.transition_pairs, cache,
                             count_device=res.transition_count, page_size=ps,
                             bulk_copy_v=bulk)
        torch.cuda.synchronize()
        ao = res.active_offsets.cpu().numpy()
        raw = res.raw_indices[: ao[-1]].cpu().numpy()
        table = req_to_token.cpu().numpy()
        slots = np.concatenate([table[row_ids[r], raw[ao[r]: ao[r + 1]]]
                                for r in range(prog.requests)])
        sl = torch.from_numpy(slots.astype(np.int64)).to(dev)
        views[ps] = [(k[sl].cpu(), v[sl].cpu()) for k, v in zip(k_pools, v_pools)]
        views[(ps, "pos")] = res.active_positions[: ao[-1]].cpu().numpy()
    np.testing.assert_array_equal(views[(1, "pos")], views[(page_size, "pos")])
    for (k1, v1), (k2, v2) in zip(views[1], views[page_size]):
        assert torch.equal(k1.view(torch.int16), k2.view(torch.int16))
        assert torch.equal(v1.view(torch.int16), v2.view(torch.int16))
