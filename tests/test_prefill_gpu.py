"""Ragged prefill attention with context positions (C ABI akv_context_attention)
against a plain torch fp32 reference and the float64 oracle.

Tolerance: atol 2e-3 / rtol 1e-2 on the bf16 output (bf16 inputs, fp32
softmax and accumulation; P enters P.V as a bf16 hi + lo pair, except in
variants 5 and 6, which round it to bf16 like FlashInfer and get that
rounding's bound on top, stated at their test).
"""

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2


def make_batch(rng, prefix_lens, query_lens, hkv, d, gap=5, dev="cuda"):
    """Prefix positions with holes (dropped tokens), new tokens consecutive
    after a gap; every key at a distinct random pool slot."""
    qo = np.concatenate(([0], np.cumsum(query_lens))).astype(np.int64)
    kv = np.concatenate(([0], np.cumsum(prefix_lens))).astype(np.int64)
    qpos, kpos = [], []
    for p, q in zip(prefix_lens, query_lens):
        steps = rng.integers(1, gap + 1, size=p)
        pp = np.cumsum(steps) - 1
        start = (pp[-1] if p else -1) + int(rng.integers(1, gap + 1))
        kpos.append(pp)
        qpos.append(start + np.arange(q))
    qpos = np.concatenate(qpos).astype(np.int32)
    kpos = np.concatenate(kpos).astype(np.int32) if kv[-1] else np.zeros(0, np.int32)
    n_slots = int(kv[-1] + qo[-1]) + 7
    perm = rng.permutation(n_slots - 1).astype(np.int32) + 1
    kv_idx = perm[: kv[-1]]
    births = perm[kv[-1]: kv[-1] + qo[-1]]
    g = torch.Generator(device=dev).manual_seed(int(rng.integers(1 << 30)))
    k_pool = torch.randn(n_slots, hkv, d, device=dev, generator=g, dtype=torch.bfloat16)
    v_pool = torch.randn(n_slots, hkv, d, device=dev, generator=g, dtype=torch.bfloat16)
    q = torch.randn(int(qo[-1]), 8 * hkv, d, device=dev, generator=g, dtype=torch.bfloat16)
    return dict(qo=qo, kv=kv, qpos=qpos, kpos=kpos, kv_idx=kv_idx, births=births,
                k_pool=k_pool, v_pool=v_pool, q=q)


def torch_reference(x, window, sinks, scale):
    q, kp, vp = x["q"].float(), x["k_pool"].float(), x["v_pool"].float()
    hq = q.shape[1]
    group = hq // kp.shape[1]
    out = torch.zeros_like(q)
    for b in range(len(x["qo"]) - 1):
        a, e, s0, s1 = int(x["qo"][b]), int(x["qo"][b + 1]), int(x["kv"][b]), int(x["kv"][b + 1])
        if e == a:
            continue
        slots = np.concatenate((x["kv_idx"][s0:s1], x["births"][a:e])).astype(np.int64)
        kpos = torch.tensor(np.concatenate((x["kpos"][s0:s1], x["qpos"][a:e])).astype(np.int64),
                            device=q.device)
        qpos = torch.tensor(x["qpos"][a:e].astype(np.int64), device=q.device)
        sl = torch.from_numpy(slots).to(q.device)
        k = kp[sl].repeat_interleave(group, dim=1)  # [n, Hq, D]
        v = vp[sl].repeat_interleave(group, dim=1)
        n_prefix = s1 - s0
        j = torch.arange(len(slots), device=q.device)
        i = torch.arange(e - a, device=q.device)
        vis = (j[None, :] < n_prefix) | (j[None, :] - n_prefix <= i[:, None])
        if window >= 0:
            vis &= (qpos[:, None] - kpos[None, :]) <= window
        sc = torch.einsum("qhd,khd->hqk", q[a:e], k) * scale
        sc = sc.masked_fill(~vis[None], float("-inf"))
        if sinks is not None:
            col = sinks.float()[:, None, None].expand(hq, e - a, 1)
            w = torch.softmax(torch.cat((sc, col), dim=2), dim=2)[..., :-1]
        else:
            w = torch.softmax(sc, dim=2)
        out[a:e] = torch.einsum("hqk,khd->qhd", w, v)
    return out


def run_ours(x, hkv, d, window, sinks, lse=None, variant=0):
    from akv_b200.context_prefill import ContextPrefillAttention

    dev = x["q"].device
    att = ContextPrefillAttention(8 * hkv, hkv, d, dev).plan(
        x["qo"], x["kv"], x["qpos"], x["kpos"], window=window)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.int32)).to(dev)  # noqa: E731
    out = att.run(x["q"], x["k_pool"], x["v_pool"], t(x["kv_idx"]), t(x["births"]),
                  t(x["qpos"]), t(x["kpos"]), sinks=sinks, lse=lse, variant=variant)
    torch.cuda.synchronize()
    assert att.errors() == 0
    return out, att


CASES = [
    # (prefix lens, query lens, hkv, d, window, sinks)
    ([300, 0, 1000, 17], [40, 33, 1, 200], 8, 64, -1, True),
    ([300, 0, 1000, 17], [40, 33, 1, 200], 8, 64, 128, True),
    ([2000, 5], [300, 64], 8, 64, 7, False),
    ([64, 128], [16, 17], 2, 128, -1, True),
    ([900], [130], 1, 128, 100, True),
    ([0], [1], 8, 64, -1, True),
    ([5000, 3000, 1], [96, 250, 70], 8, 64, 128, True),
    ([2000, 5], [300, 64], 4, 128, 7, False),
    ([3000, 700, 0], [130, 200, 33], 8, 128, 128, True),
]


@pytest.mark.parametrize("variant", [0, 1, 2, 3, 4],
                         ids=["auto", "mma_sync", "tcgen05", "tcgen05_ws", "tcgen05_ws_2tiles"])
@pytest.mark.parametrize("case", range(len(CASES)))
def test_prefill_matches_torch(case, variant):
    """variant 1 runs the mma.sync kernel, 2 the tcgen05 one (head_dim 64), 3 its
    warp-specialised form (head_dim 64 and 128), 4 that form with two query
    tiles per CTA."""
    prefix, queries, hkv, d, window, use_sinks = CASES[case]
    if variant == 2 and d != 64:
        pytest.skip("the simpler tcgen05 kernel covers head_dim 64")
    rng = np.random.default_rng(case)
    x = make_batch(rng, prefix, queries, hkv, d)
    sinks = torch.randn(8 * hkv, device="cuda") if use_sinks else None
    scale = 1.0 / np.sqrt(d)
    out, _ = run_ours(x, hkv, d, window, sinks, variant=variant)
    want = torch_reference(x, window, sinks, scale)
    torch.testing.assert_close(out.float(), want, atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("variant,d", [(1, 64), (2, 64), (3, 64), (4, 64), (1, 128), (3, 128),
                                       (4, 128)])
def test_prefill_matches_float64_oracle_with_lse(variant, d):
    from oracle import oracle

    rng = np.random.default_rng(42)
    hkv, window = 2, 33
    x = make_batch(rng, [150, 40], [37, 20], hkv, d)
    sinks = torch.randn(8 * hkv, device="cuda")
    lse = torch.empty(x["q"].shape[0], 8 * hkv, device="cuda")
    out, _ = run_ours(x, hkv, d, window, sinks, lse=lse, variant=variant)
    want, want_lse = oracle.prefill_attention(
        x["q"].float().cpu().numpy(), x["k_pool"].float().cpu().numpy(),
        x["v_pool"].float().cpu().numpy(), x["qo"], x["kv"], x["kv_idx"], x["births"],
        x["qpos"], x["kpos"], sinks=sinks.cpu().numpy(), window=window)
    np.testing.assert_allclose(out.float().cpu().numpy(), want, atol=ATOL, rtol=RTOL)
    # lse includes the sink: logaddexp(lse_scores, sink)
    full = np.logaddexp(want_lse, sinks.cpu().numpy()[None, :].astype(np.float64))
    np.testing.assert_allclose(lse.cpu().numpy(), full, atol=1e-3, rtol=1e-4)


def test_bad_slot_sets_error_flag_and_stays_in_bounds():
    rng = np.random.default_rng(3)
    x = make_batch(rng, [100], [20], 8, 64)
    x["kv_idx"] = x["kv_idx"].copy()
    x["kv_idx"][5] = 10**6  # outside the pool
    from akv_b200.context_prefill import ContextPrefillAttention

    att = ContextPrefillAttention(64, 8, 64, "cuda").plan(x["qo"], x["kv"], x["qpos"], x["kpos"])
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.int32)).cuda()  # noqa: E731
    att.run(x["q"], x["k_pool"], x["v_pool"], t(x["kv_idx"]), t(x["births"]), t(x["qpos"]),
            t(x["kpos"]))
    torch.cuda.synchronize()
    assert att.errors() == 1
    with pytest.raises(RuntimeError, match="outside the KV pools"):
        att.check()
    assert att.errors() == 0  # check() clears the bits
    att.check()


def test_abort_word_of_an_earlier_launch_does_not_stop_the_next():
    """A wait that ran out leaves the abort word set; the next launch
    clears it before it starts, so it runs fully and matches the oracle,
    while the error bits stay until check()."""
    rng = np.random.default_rng(11)
    x = make_batch(rng, [300, 40], [70, 33], 8, 64)
    from akv_b200.context_prefill import ContextPrefillAttention

    att = ContextPrefillAttention(64, 8, 64, "cuda").plan(x["qo"], x["kv"], x["qpos"], x["kpos"])
    att.error_flag.copy_(torch.tensor([2, 1], dtype=torch.int32))  # as a timed-out launch leaves it
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.int32)).cuda()  # noqa: E731
    for variant in (0, 2, 3):
        att.error_flag[1].fill_(1)
        out = att.run(x["q"], x["k_pool"], x["v_pool"], t(x["kv_idx"]), t(x["births"]),
                      t(x["qpos"]), t(x["kpos"]), variant=variant)
        torch.cuda.synchronize()
        assert int(att.error_flag[1].item()) == 0
        want = torch_reference(x, -1, None, 1.0 / 8.0)
        torch.testing.assert_close(out.float(), want, atol=ATOL, rtol=RTOL)
    assert att.errors() == 2
    with pytest.raises(RuntimeError, match="wait ran out"):
        att.check()


def test_plan_rejects_unsorted_positions():
    from akv_b200.context_prefill import ContextPrefillAttention

    att = ContextPrefillAttention(64, 8, 64, "cuda")
    with pytest.raises(ValueError, match="increase"):
        att.plan([0, 2], [0, 2], [5, 6], [3, 3])


@pytest.mark.parametrize("variant", [5, 6], ids=["tcgen05_ws_bf16p", "tcgen05_ws_2tiles_bf16p"])
@pytest.mark.parametrize("case", range(len(CASES)))
def test_prefill_bf16_p_forms_match_torch_within_their_bound(case, variant):
    """Variants 5 and 6 round P to bf16 for P.V, as FlashInfer's prefill
    does (one MMA per key block instead of the hi + lo pair): each output is
    within atol 2e-3 + rtol 1e-2 |ref| plus that rounding's bound,
    2^-8 * sum_i p_i |v_i|, of the exact fp32 attention."""
    prefix, queries, hkv, d, window, use_sinks = CASES[case]
    rng = np.random.default_rng(case)
    x = make_batch(rng, prefix, queries, hkv, d)
    sinks = torch.randn(8 * hkv, device="cuda") if use_sinks else None
    scale = 1.0 / np.sqrt(d)
    out, _ = run_ours(x, hkv, d, window, sinks, variant=variant)
    want = torch_reference(x, window, sinks, scale)
    p_abs_v = torch_reference(dict(x, v_pool=x["v_pool"].abs()), window, sinks, scale)
    bound = ATOL + RTOL * want.abs() + 2.0 ** -8 * p_abs_v
    excess = (out.float() - want).abs() - bound
    assert float(excess.max()) <= 0.0, f"max excess {float(excess.max()):.3g}"


@pytest.mark.parametrize("variant", [5, 6])
def test_prefill_bf16_p_forms_keep_the_exact_lse(variant):
    """The row sums of variants 5 and 6 add the fp32 exponentials, so their
    log-sum-exp is as exact as the other kernels'."""
    from oracle import oracle

    rng = np.random.default_rng(42)
    hkv, d, window = 2, 64, 33
    x = make_batch(rng, [150, 40], [37, 20], hkv, d)
    sinks = torch.randn(8 * hkv, device="cuda")
    lse = torch.empty(x["q"].shape[0], 8 * hkv, device="cuda")
    run_ours(x, hkv, d, window, sinks, lse=lse, variant=variant)
    _, want_lse = oracle.prefill_attention(
        x["q"].float().cpu().numpy(), x["k_pool"].float().cpu().numpy(),
        x["v_pool"].float().cpu().numpy(), x["qo"], x["kv"], x["kv_idx"], x["births"],
        x["qpos"], x["kpos"], sinks=sinks.cpu().numpy(), window=window)
    full = np.logaddexp(want_lse, sinks.cpu().numpy()[None, :].astype(np.float64))
    np.testing.assert_allclose(lse.cpu().numpy(), full, atol=1e-3, rtol=1e-4)
