"""The paged Drop oracle (``oracle.drop_compact_paged``) on the CPU.

Its decode view and positions must equal those of the page_size 1 oracle,
which tests/test_oracle_golden.py pins to the reference's compiler; a
hand-worked case fixes the page rules (freed pages, whole-page copies and
bit copies of the tokens before the first drop).
"""

import numpy as np
import pytest


@pytest.mark.parametrize("page_size", [4, 16, 64])
def test_paged_oracle_keeps_the_unpaged_decode_view(page_size):
    from akv_b200 import workloads
    from oracle import oracle

    prog = workloads.c3_program(requests=8, max_len=6000, seed=5, page_align=page_size)
    rows, n_pages = workloads.paged_slot_rows(np.random.default_rng(5), prog, page_size)
    need = -(-int(prog.shared_prefix.sum()) // page_size) + prog.requests
    paged = oracle.drop_compact_paged(prog.token_counts, prog.range_offsets, prog.ranges, rows,
                                      page_size, shared_prefix=prog.shared_prefix,
                                      free_pages=np.arange(n_pages, n_pages + need),
                                      free_tail=need)
    flat = oracle.drop_compact(prog.token_counts, prog.range_offsets, prog.ranges, rows,
                               shared_prefix=prog.shared_prefix,
                               free_ring=np.arange(10**7, 10**7 + 10**6))
    for a, b in zip(paged["raw_indices"], flat["raw_indices"]):
        np.testing.assert_array_equal(a, b)
    for a, b in zip(paged["active_positions"], flat["active_positions"]):
        np.testing.assert_array_equal(a, b)
    assert paged["next_position"] == flat["next_position"]
    # every moved token of the flat run is a transition of the paged run
    # with the same position pair
    moved = set(zip(flat["raw"].tolist(), map(tuple, flat["pairs"].tolist())))
    assert moved <= set(zip(paged["raw"].tolist(), map(tuple, paged["pairs"].tolist())))
    # freed pages hold only dropped private tokens
    freed_slots = set(flat["freed"].tolist())
    for page in paged["freed"]:
        assert set(range(page * page_size, (page + 1) * page_size)) & set(
            np.concatenate(rows).tolist()) <= freed_slots


def test_paged_oracle_hand_worked_case():
    from oracle import oracle

    # one request of 40 tokens, pages of 4, the first 8 tokens shared (two
    # pages); drop [2, 3) and [20, 28) (two whole private pages).
    ps = 4
    rows = [np.array([(10 + t // ps) * ps + t % ps for t in range(40)], np.int32)]
    out = oracle.drop_compact_paged([40], [0, 2], [2, 3, 20, 28], rows, ps, shared_prefix=[8],
                                    free_pages=np.array([90, 91, 92], np.int32), free_tail=3)
    # shared page 10 (tokens 0-3) holds moved token 3: copied to page 90,
    # tokens 0 and 1 bit-copied (old == new), token 3 moves 3 -> 2; shared
    # page 11 (tokens 4-7) is copied to page 91.
    assert out["copied_pages"] == 2 and out["free_head"] == 2
    assert out["src"][:5].tolist() == [40, 41, 43, 44, 45]
    assert out["dst"][:5].tolist() == [360, 361, 363, 364, 365]
    assert out["pairs"][:3].tolist() == [[0, 0], [1, 1], [3, 2]]
    # private tokens rotate in place
    assert out["src"][7:].tolist() == out["dst"][7:].tolist()
    # pages 15 and 16 (tokens 20-27) are freed, in token order
    assert out["freed"].tolist() == [15, 16]
    assert out["rows"][0][:8].tolist() == [360, 361, 362, 363, 364, 365, 366, 367]
