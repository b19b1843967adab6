"""The prefill mask of the device kernel and the oracle against the
reference's own planning rule, on the CPU.

ContextAttentionMetadata.native_plan (srt/layers/attention/context_backend.py
:191-222) turns every query of a sliding-window segment whose positions have
holes into a single-query segment with the gathered keys
``indices[start:end]``, ``end = prefix + i + 1`` and ``start`` the first key
whose position reaches ``q_pos - window``.  The kernel and the oracle use
the rule "prefix key j, or new-token key j <= i, with q_pos - k_pos <=
window"; this test checks the two select the same keys.
"""

import numpy as np


def native_plan_keys(positions, n_prefix, qpos, i, window):
    """Request-local key indices native_plan gathers for query i of a gapped
    segment (the per-query branch, context_backend.py:203-208)."""
    end = n_prefix + i + 1
    start = int(np.searchsorted(positions[:end], qpos - window))
    return np.arange(start, end)


def rule_keys(positions, n_prefix, qpos, i, window):
    j = np.arange(len(positions))
    vis = (j < n_prefix) | (j - n_prefix <= i)
    if window >= 0:
        vis &= qpos - positions <= window
    return np.flatnonzero(vis)


def test_mask_rule_matches_native_plan_on_gapped_segments():
    rng = np.random.default_rng(0)
    for _ in range(300):
        n_prefix = int(rng.integers(0, 400))
        n_query = int(rng.integers(1, 60))
        window = int(rng.integers(0, 300))
        prefix = np.cumsum(rng.integers(1, 6, size=n_prefix)) - 1
        start = (prefix[-1] if n_prefix else -1) + int(rng.integers(1, 6))
        queries = start + np.arange(n_query)
        positions = np.concatenate((prefix, queries))
        for i in range(n_query):
            np.testing.assert_array_equal(
                rule_keys(positions, n_prefix, queries[i], i, window),
                native_plan_keys(positions, n_prefix, queries[i], i, window))


def test_oracle_applies_the_rule():
    """The float64 oracle's output for one query equals softmax attention
    over exactly the rule's keys."""
    from oracle import oracle

    rng = np.random.default_rng(1)
    d, hkv = 16, 1
    n_prefix, n_query, window = 50, 9, 20
    prefix = np.cumsum(rng.integers(1, 4, size=n_prefix)) - 1
    queries = prefix[-1] + 3 + np.arange(n_query)
    slots = rng.permutation(n_prefix + n_query + 1)[: n_prefix + n_query] + 0
    k = rng.standard_normal((n_prefix + n_query + 1, hkv, d))
    v = rng.standard_normal((n_prefix + n_query + 1, hkv, d))
    q = rng.standard_normal((n_query, 8, d))
    out, _ = oracle.prefill_attention(q, k, v, [0, n_query], [0, n_prefix], slots[:n_prefix],
                                      slots[n_prefix:], queries, prefix, window=window)
    positions = np.concatenate((prefix, queries))
    for i in range(n_query):
        keys = rule_keys(positions, n_prefix, queries[i], i, window)
        kk, vv = k[slots[keys], 0], v[slots[keys], 0]
        s = kk @ q[i, 3] / np.sqrt(d)
        w = np.exp(s - s.max())
        np.testing.assert_allclose(out[i, 3], (w / w.sum()) @ vv, rtol=1e-12, atol=1e-12)
