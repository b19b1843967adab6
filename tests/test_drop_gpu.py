"""Drop + Reposition on the device (C ABI akv_drop_compact) against the oracle.

The oracle's ``drop_compact`` composes the CPU event compiler restatement,
which tests/test_oracle_golden.py pins to the reference's own C++ compiler,
with the decode view (occurrence.py:47-66) and the freed-slot rule.  Every
integer output must match bit for bit.
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _run(program, rows, ring_free, ring_capacity=None, reposition=True, max_slots=None):
    from akv_b200.context_drop import DropCompactor, FreeSlotRing

    dev = torch.device("cuda")
    nreq = program.requests
    width = max(1, int(program.token_counts.max()) if nreq else 1)
    table = np.zeros((nreq + 2, width), np.int32)
    row_ids = np.arange(nreq, dtype=np.int64) + 1  # row 0 unused: rows need not start at 0
    for r in range(nreq):
        table[row_ids[r], : len(rows[r])] = rows[r]
    req_to_token = torch.from_numpy(table).to(dev)
    ring = FreeSlotRing(torch.from_numpy(np.asarray(ring_free, np.int32)),
                        capacity=ring_capacity or len(ring_free) + program.total_tokens + 1,
                        device=dev)
    comp = DropCompactor(program.total_tokens, nreq, max(1, len(program.ranges) // 2), dev)
    res = comp.run(program.token_counts, program.range_offsets, program.ranges, req_to_token,
                   row_ids, ring, shared_prefix=program.shared_prefix if
                   program.shared_prefix.any() else None, reposition=reposition)
    torch.cuda.synchronize()
    return res, req_to_token, row_ids, ring


def _check(program, rows, ring_free, reposition=True, ring_capacity=None):
    from oracle import oracle

    res, req_to_token, row_ids, ring = _run(program, rows, ring_free, ring_capacity, reposition)
    want = oracle.drop_compact(program.token_counts, program.range_offsets, program.ranges, rows,
                               shared_prefix=program.shared_prefix, reposition=reposition,
                               free_ring=np.asarray(ring_free, np.int32), free_head=0,
                               free_tail=len(ring_free))
    assert int(res.status.item()) == 0
    totals = res.totals.cpu().numpy()
    kept = sum(len(x) for x in want["raw_indices"])
    assert totals.tolist() == [kept, len(want["src"]),
                               int(sum(1 for s, d in zip(want["src"], want["dst"]) if s != d)),
                               len(want["freed"])]
    # per-token outputs
    keep = np.concatenate([lay["keep_mask"] for lay in want["layouts"]]) if want["layouts"] else []
    pos = np.concatenate([lay["positions"] for lay in want["layouts"]]) if want["layouts"] else []
    np.testing.assert_array_equal(res.keep_mask.cpu().numpy().astype(bool), keep)
    np.testing.assert_array_equal(res.positions.cpu().numpy(), pos)
    # decode view (CSR)
    ao = res.active_offsets.cpu().numpy()
    np.testing.assert_array_equal(np.diff(ao), [len(x) for x in want["raw_indices"]])
    raw = res.raw_indices[:kept].cpu().numpy()
    apos = res.active_positions[:kept].cpu().numpy()
    for r in range(program.requests):
        np.testing.assert_array_equal(raw[ao[r]: ao[r + 1]], want["raw_indices"][r])
        np.testing.assert_array_equal(apos[ao[r]: ao[r + 1]], want["active_positions"][r])
    np.testing.assert_array_equal(res.next_position.cpu().numpy(), want["next_position"])
    # transitions
    n = len(want["src"])
    np.testing.assert_array_equal(res.transition_source[:n].cpu().numpy(), want["src"])
    np.testing.assert_array_equal(res.transition_destination[:n].cpu().numpy(), want["dst"])
    np.testing.assert_array_equal(res.transition_pairs[:n].cpu().numpy(), want["pairs"])
    np.testing.assert_array_equal(res.transition_raw[:n].cpu().numpy(), want["raw"])
    to = res.transition_offsets.cpu().numpy()
    np.testing.assert_array_equal(np.diff(to), [len(lay["transition_raw_tokens"])
                                                for lay in want["layouts"]])
    # freed slots and the free ring
    f = len(want["freed"])
    np.testing.assert_array_equal(res.freed_slots[:f].cpu().numpy(), want["freed"])
    head, tail = ring.state.cpu().tolist()
    assert (head, tail) == (want["free_head"], want["free_tail"])
    ring_now = ring.ring.cpu().numpy()
    idx = np.arange(len(ring_free), tail) % ring.capacity
    np.testing.assert_array_equal(ring_now[idx], want["freed"])
    # rows after copy-on-write
    table = req_to_token.cpu().numpy()
    for r in range(program.requests):
        np.testing.assert_array_equal(table[row_ids[r], : len(rows[r])], want["rows"][r])
    return res


def test_drop_c1_matches_oracle():
    from akv_b200 import workloads

    prog = workloads.c1_program()
    rows, nslots = workloads.slot_rows(np.random.default_rng(0), prog)
    _check(prog, rows, ring_free=np.arange(nslots, nslots + 16))


def test_drop_c2_full_size_matches_oracle():
    from akv_b200 import workloads

    prog = workloads.c2_program()
    rows, nslots = workloads.slot_rows(np.random.default_rng(0), prog)
    res = _check(prog, rows, ring_free=np.arange(nslots, nslots + 16))
    totals = res.totals.cpu().tolist()
    assert totals[1] == 38902 and totals[3] == 26425  # the c2 program's seed-0 counts


def test_drop_c3_shared_prefix_cow_matches_oracle():
    from akv_b200 import workloads

    prog = workloads.c3_program(requests=16, max_len=12000)
    rows, nslots = workloads.slot_rows(np.random.default_rng(1), prog)
    free = np.arange(nslots, nslots + int(prog.shared_prefix.sum()) + 10)
    res = _check(prog, rows, ring_free=free, ring_capacity=len(free) + 400000)
    assert int(res.totals[2].item()) > 0  # some copy-on-write happened


def test_drop_reposition_off_matches_oracle():
    from akv_b200 import workloads

    prog = workloads.c3_program(requests=6, max_len=5000, seed=3)
    rows, nslots = workloads.slot_rows(np.random.default_rng(3), prog)
    _check(prog, rows, ring_free=np.arange(nslots, nslots + 4), reposition=False,
           ring_capacity=100000)


def test_drop_edge_cases_match_oracle():
    from akv_b200.workloads import DropProgram

    # request 0: no ranges; 1: empty request; 2: a suffix drop (Reposition
    # ignored); 3: spans crossing 512-token tile boundaries; 4: one token
    # kept at the end; 5: a range covering the first token only.
    counts = np.array([300, 0, 40, 7000, 3000, 2])
    per = [[], [], [30, 40], [100, 2047, 2049, 4097, 6000, 6999], [0, 2999], [0, 1]]
    offsets = np.cumsum([0] + [len(p) // 2 for p in per])
    ranges = np.concatenate([np.asarray(p, np.int32) for p in per])
    prog = DropProgram(counts, offsets.astype(np.int32), ranges, np.zeros(len(counts), np.int64))
    rng = np.random.default_rng(9)
    rows = [rng.permutation(int(c)).astype(np.int32) + 1 + 10000 * r for r, c in enumerate(counts)]
    _check(prog, rows, ring_free=np.arange(90000, 90004), ring_capacity=20000)


def test_drop_ring_underflow_changes_nothing():
    from akv_b200 import workloads

    prog = workloads.c3_program(requests=4, max_len=6000, seed=2)
    rows, nslots = workloads.slot_rows(np.random.default_rng(2), prog)
    res, req_to_token, row_ids, ring = _run(prog, rows, ring_free=np.arange(nslots, nslots + 3),
                                            ring_capacity=100000)
    st = int(res.status.item())
    from akv_b200 import _native

    assert st & _native.DROP_RING_UNDERFLOW
    assert ring.state.cpu().tolist() == [0, 3]
    assert res.totals[1:].cpu().tolist() == [0, 0, 0]
    table = req_to_token.cpu().numpy()
    for r in range(prog.requests):
        np.testing.assert_array_equal(table[row_ids[r], : len(rows[r])], rows[r])
    with pytest.raises(RuntimeError, match="copy-on-write"):
        res.check()


def test_drop_host_validation_errors():
    from akv_b200.context_drop import validate_program

    with pytest.raises(ValueError, match="ordered, disjoint"):
        validate_program([10], [0, 2], [5, 7, 1, 3])
    with pytest.raises(ValueError, match="ordered, disjoint"):
        validate_program([10], [0, 1], [5, 11])
    with pytest.raises(ValueError, match="no active tokens"):
        validate_program([5], [0, 1], [0, 5])
    validate_program([5], [0, 1], [0, 5], reposition=False)


def test_drop_then_reposition_without_host_round_trip():
    """drop_compact's device-side transition count drives the reposition
    kernel; the K rows end up exactly as the oracle pipeline leaves them."""
    from oracle import oracle
    from akv_b200 import workloads
    from akv_b200.context_reposition import layer_pointer_table, reposition_kv_layers
    from akv_b200.rope import yarn_cos_sin_cache

    dev = torch.device("cuda")
    prog = workloads.c3_program(requests=8, max_len=9000, seed=4)
    rows, nslots = workloads.slot_rows(np.random.default_rng(4), prog)
    free = np.arange(nslots, nslots + int(prog.shared_prefix.sum()) + 8, dtype=np.int32)
    slots = int(free.max()) + 1
    layers, heads, dim = 3, 8, 64
    ks = [torch.randn(slots, heads, dim).to(torch.bfloat16) for _ in range(layers)]
    vs = [torch.randn(slots, heads, dim).to(torch.bfloat16) for _ in range(layers)]
    cache = yarn_cos_sin_cache(40000, dim, 150000.0, 32.0, 4096)
    hk = [k.view(torch.int16).numpy().view(np.uint16).copy() for k in ks]
    hv = [v.view(torch.int16).numpy().view(np.uint16).copy() for v in vs]
    want = oracle.drop_compact(prog.token_counts, prog.range_offsets, prog.ranges, rows,
                               shared_prefix=prog.shared_prefix, free_ring=free, free_head=0,
                               free_tail=len(free))
    oracle.reposition(hk, hv, want["src"], want["dst"], want["pairs"], cache.numpy(), bf16=True,
                      threads=4)

    res, _, _, _ = _run(prog, rows, free, ring_capacity=len(free) + 200000)
    dk = [k.to(dev) for k in ks]
    dv = [v.to(dev) for v in vs]
    reposition_kv_layers(layer_pointer_table(dk), layer_pointer_table(dv), dk[0], dv[0],
                         res.transition_source, res.transition_destination,
                         res.transition_pairs, cache.to(dev),
                         count_device=res.transition_count)
    torch.cuda.synchronize()
    for layer in range(layers):
        np.testing.assert_array_equal(dk[layer].cpu().view(torch.int16).numpy().view(np.uint16),
                                      hk[layer])
        np.testing.assert_array_equal(dv[layer].cpu().view(torch.int16).numpy().view(np.uint16),
                                      hv[layer])


def test_drop_then_reposition_replayed_from_a_cuda_graph():
    """The Drop launches (plan and scatter as programmatic dependent
    launches) and the reposition launch are stream-ordered, allocate nothing
    and read no host state, so one captured graph replays the whole cache
    operation; the result equals the oracle pipeline's."""
    from oracle import oracle
    from akv_b200 import workloads
    from akv_b200.context_drop import DropCompactor, FreeSlotRing
    from akv_b200.context_reposition import layer_pointer_table, reposition_kv_layers
    from akv_b200.rope import yarn_cos_sin_cache

    dev = torch.device("cuda")
    prog = workloads.c3_program(requests=6, max_len=7000, seed=5)
    rows, nslots = workloads.slot_rows(np.random.default_rng(5), prog)
    free = np.arange(nslots, nslots + int(prog.shared_prefix.sum()) + 8, dtype=np.int32)
    slots = int(free.max()) + 1
    layers, heads, dim = 2, 8, 64
    ks = [torch.randn(slots, heads, dim).to(torch.bfloat16) for _ in range(layers)]
    vs = [torch.randn(slots, heads, dim).to(torch.bfloat16) for _ in range(layers)]
    cache = yarn_cos_sin_cache(40000, dim, 150000.0, 32.0, 4096)
    hk = [k.view(torch.int16).numpy().view(np.uint16).copy() for k in ks]
    hv = [v.view(torch.int16).numpy().view(np.uint16).copy() for v in vs]
    want = oracle.drop_compact(prog.token_counts, prog.range_offsets, prog.ranges, rows,
                               shared_prefix=prog.shared_prefix, free_ring=free, free_head=0,
                               free_tail=len(free))
    oracle.reposition(hk, hv, want["src"], want["dst"], want["pairs"], cache.numpy(), bf16=True,
                      threads=4)

    nreq = prog.requests
    table = np.zeros((nreq + 1, int(prog.token_counts.max())), np.int32)
    for r in range(nreq):
        table[r + 1, : len(rows[r])] = rows[r]
    req_to_token = torch.from_numpy(table).to(dev)
    row_ids = np.arange(1, nreq + 1)
    ring = FreeSlotRing(torch.from_numpy(free), capacity=len(free) + prog.total_tokens + 1,
                        device=dev)
    comp = DropCompactor(prog.total_tokens, nreq, max(1, len(prog.ranges) // 2), dev)
    prepared = comp.prepare(prog.token_counts, prog.range_offsets, prog.ranges, row_ids,
                            shared_prefix=prog.shared_prefix)
    dk = [k.to(dev) for k in ks]
    dv = [v.to(dev) for v in vs]
    kp, vp, dcache = layer_pointer_table(dk), layer_pointer_table(dv), cache.to(dev)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        res = comp.launch(prepared, req_to_token, ring)
        reposition_kv_layers(kp, vp, dk[0], dv[0], res.transition_source,
                             res.transition_destination, res.transition_pairs, dcache,
                             count_device=res.transition_count)
    graph.replay()
    torch.cuda.synchronize()
    assert int(res.status.item()) == 0
    n = len(want["src"])
    assert int(res.totals[1].item()) == n
    np.testing.assert_array_equal(res.transition_source[:n].cpu().numpy(), want["src"])
    np.testing.assert_array_equal(res.transition_destination[:n].cpu().numpy(), want["dst"])
    for layer in range(layers):
        np.testing.assert_array_equal(dk[layer].cpu().view(torch.int16).numpy().view(np.uint16),
                                      hk[layer])
        np.testing.assert_array_equal(dv[layer].cpu().view(torch.int16).numpy().view(np.uint16),
                                      hv[layer])
    del graph


def test_same_shape_programs_restage_through_one_compactor():
    """A compactor hands the same staging handle back for programs of the
    same shape; each call must still stage its own program (A, B, A again
    through one compactor, each against the oracle)."""
    from akv_b200.context_drop import DropCompactor, FreeSlotRing
    from akv_b200.workloads import DropProgram
    from oracle import oracle

    dev = torch.device("cuda")
    counts = np.array([3000, 2000])
    programs = [DropProgram(counts, np.array([0, 2, 3], np.int32),
                            np.asarray(r, np.int32), np.zeros(2, np.int64))
                for r in ([10, 200, 700, 900, 5, 1500], [1000, 1100, 2500, 2990, 400, 401])]
    rng = np.random.default_rng(5)
    rows = [rng.permutation(int(c)).astype(np.int32) + 1 + 5000 * r for r, c in enumerate(counts)]
    table = np.zeros((3, 3000), np.int32)
    table[1, :3000], table[2, :2000] = rows
    req_to_token = torch.from_numpy(table).to(dev)
    comp = DropCompactor(5000, 2, 3, dev)
    handles = []
    for p in (programs[0], programs[1], programs[0]):
        ring = FreeSlotRing(torch.zeros(0, dtype=torch.int32), capacity=6000, device=dev)
        handles.append(comp.prepare(p.token_counts, p.range_offsets, p.ranges, [1, 2]))
        res = comp.launch(handles[-1], req_to_token, ring)
        want = oracle.drop_compact(p.token_counts, p.range_offsets, p.ranges, rows,
                                   shared_prefix=p.shared_prefix, reposition=True,
                                   free_ring=np.zeros(0, np.int32), free_head=0, free_tail=0)
        torch.cuda.synchronize()
        res.check()
        keep = np.concatenate([lay["keep_mask"] for lay in want["layouts"]])
        pos = np.concatenate([lay["positions"] for lay in want["layouts"]])
        np.testing.assert_array_equal(res.keep_mask.cpu().numpy().astype(bool), keep)
        np.testing.assert_array_equal(res.positions.cpu().numpy(), pos)
        n = int(res.totals[1].item())
        np.testing.assert_array_equal(res.transition_source[:n].cpu().numpy(), want["src"])
    assert handles[0] is handles[1] is handles[2]


@pytest.mark.parametrize("validate", [True, False])
def test_read_view_copies_the_decode_view_in_one_call(validate):
    """``DropResult.read_view`` (C ABI akv_drop_read_view): the host vector
    holds the device's raw indices and positions (the first ``kept``, the
    host's count for a validated program, else every token), the CSR
    offsets, next positions, totals and status, in that order, and the
    oracle's decode view; the copies run on the stream given."""
    from oracle import oracle
    from akv_b200 import workloads
    from akv_b200.context_drop import DropCompactor, FreeSlotRing

    dev = torch.device("cuda")
    prog = workloads.c3_program(requests=6, max_len=7000, seed=9)
    rows, nslots = workloads.slot_rows(np.random.default_rng(9), prog)
    free = np.arange(nslots, nslots + int(prog.shared_prefix.sum()) + 8, dtype=np.int32)
    nreq = prog.requests
    table = np.zeros((nreq + 1, int(prog.token_counts.max())), np.int32)
    for r in range(nreq):
        table[r + 1, : len(rows[r])] = rows[r]
    rtt = torch.from_numpy(table).to(dev)
    ring = FreeSlotRing(torch.from_numpy(free), capacity=len(free) + prog.total_tokens + 1,
                        device=dev)
    comp = DropCompactor(prog.total_tokens, nreq, len(prog.ranges) // 2, dev)
    res = comp.run(prog.token_counts, prog.range_offsets, prog.ranges, rtt,
                   np.arange(1, nreq + 1), ring, shared_prefix=prog.shared_prefix,
                   validate=validate)
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    out = res.read_view(stream=side)
    side.synchronize()
    want = oracle.drop_compact(prog.token_counts, prog.range_offsets, prog.ranges, rows,
                               shared_prefix=prog.shared_prefix, free_ring=free, free_head=0,
                               free_tail=len(free))
    kept = sum(len(x) for x in want["raw_indices"])
    assert res.kept_host == (kept if validate else None)
    k = kept if validate else prog.total_tokens
    host = out.numpy()
    assert len(host) == 2 * k + 2 * nreq + 6
    np.testing.assert_array_equal(host[:kept], np.concatenate(want["raw_indices"]))
    np.testing.assert_array_equal(host[k: k + kept], np.concatenate(want["active_positions"]))
    o = 2 * k
    np.testing.assert_array_equal(host[o: o + nreq + 1], res.active_offsets.cpu().numpy())
    np.testing.assert_array_equal(np.diff(host[o: o + nreq + 1]),
                                  [len(x) for x in want["raw_indices"]])
    o += nreq + 1
    np.testing.assert_array_equal(host[o: o + nreq], want["next_position"])
    o += nreq
    np.testing.assert_array_equal(host[o: o + 4], res.totals.cpu().numpy())
    assert host[o] == kept and host[o + 4] == 0
    with pytest.raises(ValueError):
        res.read_view(out=torch.empty(3, dtype=torch.int32))
