"""Copy-on-write selection pinned to the reference's ownership code.

tests/golden/cow.npz (made by tests/golden/make_cow_golden.py) records what
the reference's OccurrenceState does for c3-shaped requests -- a
radix-matched prefix, a Drop whose first range starts inside it, a
Reposition, the next turn: which tokens its second forward copies (with
position pairs and source slots) and which slots each forward retires.

The reference copies every moved token to a fresh slot and later retires
the old one if the request owns it; this package rotates owned tokens in
place and copies only borrowed (radix-shared) ones.  So, per request:
  transitions (raw token, pair, source slot) == the reference's copies;
  copy-on-write transitions == its copies of borrowed tokens (raw < P);
  freed slots == what its first forward retires (the dropped private
    tokens, which no later query reads), in the same order;
  in-place sources == what its second forward retires (the superseded
    versions of moved private tokens), in the same order.
"""

import numpy as np
import pytest
import torch

from conftest import ROOT

GOLDEN = f"{ROOT}/tests/golden/cow.npz"


def cases():
    z = np.load(GOLDEN)
    return z, [str(c) for c in z["cases"]]


def expect(z, c):
    g = lambda k: z[f"{c}/{k}"]  # noqa: E731
    order = np.argsort(g("copy_raw"), kind="stable")
    return dict(T=int(g("tokens")), P=int(g("prefix")), ranges=g("ranges"), row=g("row"),
                raw=g("copy_raw")[order], pairs=g("copy_pairs")[order],
                src=g("copy_source_slots")[order], freed=g("forward1_retired_slots"),
                in_place=g("retired_slots"))


def check(e, raw, pairs, src, dst, freed):
    np.testing.assert_array_equal(raw, e["raw"])
    np.testing.assert_array_equal(pairs, e["pairs"])
    np.testing.assert_array_equal(src, e["src"])
    cow = raw < e["P"]
    assert np.all(dst[cow] != src[cow])
    np.testing.assert_array_equal(dst[~cow], src[~cow])
    np.testing.assert_array_equal(freed, e["freed"])
    np.testing.assert_array_equal(src[~cow], e["in_place"])


def test_golden_has_copy_on_write_and_in_place_cases():
    z, names = cases()
    kinds = [(int((expect(z, c)["raw"] < expect(z, c)["P"]).sum()) > 0,
              len(expect(z, c)["freed"]) > 0) for c in names]
    assert any(k[0] for k in kinds) and any(not k[0] for k in kinds)
    assert any(k[1] for k in kinds)


def test_oracle_selection_matches_the_reference():
    from oracle import oracle

    z, names = cases()
    for c in names:
        e = expect(z, c)
        fresh = np.arange(2 * 10**6, 2 * 10**6 + e["P"], dtype=np.int32)
        w = oracle.drop_compact([e["T"]], [0, len(e["ranges"]) // 2], e["ranges"], [e["row"]],
                                shared_prefix=[e["P"]], free_ring=fresh, free_tail=len(fresh))
        check(e, w["raw"], w["pairs"], w["src"], w["dst"], w["freed"])


@pytest.mark.gpu
def test_drop_compactor_selection_matches_the_reference():
    """All cases in one batched call through the C ABI."""
    from akv_b200.context_drop import DropCompactor, FreeSlotRing

    z, names = cases()
    es = [expect(z, c) for c in names]
    dev = torch.device("cuda")
    counts = np.array([e["T"] for e in es])
    offsets = np.cumsum([0] + [len(e["ranges"]) // 2 for e in es]).astype(np.int32)
    ranges = np.concatenate([e["ranges"] for e in es]).astype(np.int32)
    table = np.zeros((len(es), int(counts.max())), np.int32)
    for r, e in enumerate(es):
        table[r, : e["T"]] = e["row"]
    rtt = torch.from_numpy(table).to(dev)
    fresh = np.arange(2 * 10**6, 2 * 10**6 + sum(e["P"] for e in es), dtype=np.int32)
    ring = FreeSlotRing(torch.from_numpy(fresh), capacity=len(fresh) + int(counts.sum()),
                        device=dev)
    comp = DropCompactor(int(counts.sum()), len(es), len(ranges) // 2, dev)
    res = comp.run(counts, offsets, ranges, rtt, np.arange(len(es)), ring,
                   shared_prefix=np.array([e["P"] for e in es]))
    torch.cuda.synchronize()
    res.check()
    to = res.transition_offsets.cpu().numpy()
    fo = res.freed_offsets.cpu().numpy()
    n = int(to[-1])
    raw = res.transition_raw[:n].cpu().numpy()
    pairs = res.transition_pairs[:n].cpu().numpy()
    src = res.transition_source[:n].cpu().numpy()
    dst = res.transition_destination[:n].cpu().numpy()
    freed = res.freed_slots[: int(fo[-1])].cpu().numpy()
    for r, e in enumerate(es):
        a, b = to[r], to[r + 1]
        check(e, raw[a:b], pairs[a:b], src[a:b], dst[a:b], freed[fo[r]: fo[r + 1]])
