"""Decode and context-prefill attention pinned to the reference's runtime
attention path (FlashInfer plus the sink correction of its SGLang patch).

The reference serves decode through SGLang's FlashInfer backend with its
sink patch (akv/system/sglang.patch:1535-1551): FlashInfer's
BatchDecodeWithPagedKVCacheWrapper runs without sinks and returns the
log2-sum-exp of the scaled scores, and the backend rescales the bf16 output
in place by sigmoid(lse * ln 2 - sink).  These tests run exactly that on the
same page-size-1 pools, kv_indptr and kv_indices as akv_decode_attention.

FlashInfer is a library of the serving stack, not part of this build; it is
the checker here, JIT-compiled from its own sources on first use.  It has
two decode variants, and the tolerances follow what each computes:

* tensor-core decode (upstream SGLang's choice for 16-bit KV at GQA groups
  of 4 or more, so the one GPT-OSS and Llama shapes run): P enters the PV
  product in bf16, as in this build.  Outputs agree within the path's
  attention tolerance, atol 2e-3 / rtol 1e-2.  FlashInfer also sums the
  bf16-rounded P into its softmax denominator, so its log-sum-exp carries a
  relative error of up to 2^-8 in the sum: |dlse| <= ln(1 + 2^-8) < 3.9e-3.
* CUDA-core decode: P stays fp32 end to end.  Its log-sum-exp is the exact
  one (atol 1e-3, rtol 1e-4 against this build's); its output differs from
  this build's by the bf16 rounding of P in this build's PV product, which
  is bounded per element by 2^-8 * sum_i p_i |v_i| on top of the tolerance.

This build's lse includes the sink, so it must equal
logaddexp(lse_flashinfer * ln 2, sink).

The prefill half (below) builds the reference's ragged segments with its
own ``ContextAttentionMetadata.native_plan`` and runs FlashInfer's ragged
prefill over them; its tolerances are stated there.
"""

import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

flashinfer = pytest.importorskip("flashinfer")

ATOL, RTOL = 2e-3, 1e-2
LN2 = 0.6931471805599453
BF16_ROUND = 2.0 ** -8          # relative rounding bound of one bf16 value


def _reference_decode(q, k_pool, v_pool, indptr, indices, sinks, scale, tensor_cores):
    """FlashInfer decode + the reference backend's sink correction."""
    dev = q.device
    bs, hq, d = q.shape
    hkv = k_pool.shape[1]
    work = torch.zeros(128 << 20, dtype=torch.uint8, device=dev)
    wrapper = flashinfer.BatchDecodeWithPagedKVCacheWrapper(
        work, kv_layout="NHD", use_tensor_cores=tensor_cores)
    wrapper.plan(torch.from_numpy(indptr.astype(np.int32)).to(dev),
                 torch.from_numpy(indices).to(dev),
                 torch.ones(bs, dtype=torch.int32, device=dev),
                 hq, hkv, d, 1, pos_encoding_mode="NONE",
                 q_data_type=torch.bfloat16, kv_data_type=torch.bfloat16, sm_scale=scale)
    o, lse = wrapper.run(q, (k_pool.unsqueeze(1), v_pool.unsqueeze(1)), return_lse=True)
    if sinks is not None:
        o.mul_(torch.sigmoid(lse * LN2 - sinks.float()).unsqueeze(-1))
    return o, lse


@pytest.fixture(scope="module")
def flashinfer_ready():
    """FlashInfer builds its kernels from source on first use (a JIT cache in
    the home directory).  When that cannot happen on this machine the
    checker is missing, not this build's kernel: skip with the reason."""
    dev = torch.device("cuda")
    try:
        q = torch.zeros(1, 8, 64, dtype=torch.bfloat16, device=dev)
        pool = torch.zeros(4, 1, 64, dtype=torch.bfloat16, device=dev)
        for tc in (False, True):
            _reference_decode(q, pool, pool, np.array([0, 2]), np.array([1, 2], np.int32), None,
                              0.125, tc)
        work = torch.zeros(128 << 20, dtype=torch.uint8, device=dev)
        w = flashinfer.BatchPrefillWithRaggedKVCacheWrapper(work, "NHD", backend="fa2")
        ind = torch.tensor([0, 2], dtype=torch.int32)
        w.plan(ind, ind, 8, 1, 64, causal=True, q_data_type=torch.bfloat16,
               kv_data_type=torch.bfloat16)
        w.run(torch.zeros(2, 8, 64, dtype=torch.bfloat16, device=dev), pool[:2], pool[:2],
              return_lse=True)
        torch.cuda.synchronize()
    except Exception as exc:  # a JIT build or load failure of the library
        pytest.skip(f"FlashInfer cannot build or run its kernels here: "
                    f"{type(exc).__name__}: {str(exc).splitlines()[0][:200]}")


def _p_abs_v(q, k_pool, v_pool, indptr, indices, sinks, scale):
    """sum_i p_i |v_i| per (request, head, dim) in fp32: the scale of the
    rounding error a bf16 P contributes to the PV product."""
    bs, hq, d = q.shape
    group = hq // k_pool.shape[1]
    out = torch.zeros(bs, hq, d, dtype=torch.float32, device=q.device)
    idx_all = torch.from_numpy(indices).to(q.device).long()
    for b in range(bs):
        idx = idx_all[indptr[b]: indptr[b + 1]]
        k = k_pool[idx].float().repeat_interleave(group, dim=1)
        v = v_pool[idx].float().repeat_interleave(group, dim=1)
        s = torch.einsum("hd,nhd->hn", q[b].float(), k) * scale
        if sinks is not None:
            s = torch.cat((s, sinks.float()[:, None]), dim=1)
        p = torch.softmax(s, dim=1)[:, : idx.numel()]
        out[b] = torch.einsum("hn,nhd->hd", p, v.abs())
    return out


@pytest.mark.parametrize("tensor_cores", [False, True])
@pytest.mark.parametrize("hkv,d", [(8, 64), (1, 64), (8, 128), (2, 128)])
@pytest.mark.parametrize("sinks", [True, False])
def test_matches_flashinfer_decode_with_sink_correction(flashinfer_ready, tensor_cores, hkv, d,
                                                        sinks):
    from akv_b200.context_attention import DecodeAttention

    dev = torch.device("cuda")
    seed = 7 * hkv + d + int(sinks)
    rng = np.random.default_rng(seed)
    g = torch.Generator(device="cpu").manual_seed(seed)
    # Lengths from one token to long enough that both sides split the keys.
    lengths = np.array([1, 3, 17, 128, 129, 1000, 4099, 20000, 2, 777], dtype=np.int64)
    hq, bs = 8 * hkv, len(lengths)
    total = int(lengths.sum())
    slots = total + 64
    k_pool = torch.randn(slots, hkv, d, generator=g).to(torch.bfloat16).to(dev)
    v_pool = torch.randn(slots, hkv, d, generator=g).to(torch.bfloat16).to(dev)
    q = torch.randn(bs, hq, d, generator=g).to(torch.bfloat16).to(dev)
    indptr = np.concatenate(([0], np.cumsum(lengths))).astype(np.int64)
    # A compacted index list: distinct slots in a shuffled order, as Drop leaves them.
    indices = rng.permutation(slots)[:total].astype(np.int32)
    sk = (3.0 * torch.randn(hq, generator=g)).to(dev) if sinks else None
    scale = 1.0 / math.sqrt(d)

    attn = DecodeAttention(hq, hkv, d, bs, dev, sm_scale=scale)
    lse = torch.empty(bs, hq, device=dev)
    out = attn.plan(indptr).run(q, k_pool, v_pool, torch.from_numpy(indices).to(dev),
                                sinks=sk, lse=lse)
    ref_out, ref_lse2 = _reference_decode(q, k_pool, v_pool, indptr, indices, sk, scale,
                                          tensor_cores)
    torch.cuda.synchronize()
    assert int(attn.error_flag.item()) == 0

    expect_lse = ref_lse2.float() * LN2
    if sinks:
        expect_lse = torch.logaddexp(expect_lse, sk.float()[None, :])
    if tensor_cores:
        torch.testing.assert_close(out.float(), ref_out.float(), atol=ATOL, rtol=RTOL)
        torch.testing.assert_close(lse, expect_lse, atol=3.9e-3, rtol=0)
    else:
        torch.testing.assert_close(lse, expect_lse, atol=1e-3, rtol=1e-4)
        bound = ATOL + RTOL * ref_out.float().abs() + BF16_ROUND * _p_abs_v(
            q, k_pool, v_pool, indptr, indices, sk, scale)
        excess = (out.float() - ref_out.float()).abs() - bound
        assert float(excess.max()) <= 0.0, f"max excess {float(excess.max()):.3g}"


def test_matches_flashinfer_on_a_dropped_cache_layout(flashinfer_ready):
    """The decode index list a Drop leaves (kept slots of a compacted
    request), read by both kernels from the same pools."""
    from akv_b200.context_attention import DecodeAttention

    dev = torch.device("cuda")
    rng = np.random.default_rng(11)
    g = torch.Generator(device="cpu").manual_seed(11)
    hkv, d = 8, 64
    hq = 8 * hkv
    lengths = [6000, 900, 33000]
    slots = sum(lengths) + 16
    k_pool = torch.randn(slots, hkv, d, generator=g).to(torch.bfloat16).to(dev)
    v_pool = torch.randn(slots, hkv, d, generator=g).to(torch.bfloat16).to(dev)
    kept_lists = []
    base = 0
    for n in lengths:
        keep = np.ones(n, dtype=bool)
        for _ in range(12):
            s = int(rng.integers(0, n - 1))
            keep[s: s + int(rng.integers(1, max(2, n // 30)))] = False
        row = np.arange(base, base + n, dtype=np.int32)
        kept_lists.append(row[keep])
        base += n
    indptr = np.concatenate(([0], np.cumsum([len(k) for k in kept_lists]))).astype(np.int64)
    indices = np.concatenate(kept_lists).astype(np.int32)
    q = torch.randn(len(lengths), hq, d, generator=g).to(torch.bfloat16).to(dev)
    sk = (2.0 * torch.randn(hq, generator=g)).to(dev)
    scale = 1.0 / math.sqrt(d)

    attn = DecodeAttention(hq, hkv, d, len(lengths), dev, sm_scale=scale)
    out = attn.plan(indptr).run(q, k_pool, v_pool, torch.from_numpy(indices).to(dev), sinks=sk)
    ref_out, _ = _reference_decode(q, k_pool, v_pool, indptr, indices, sk, scale, True)
    torch.cuda.synchronize()
    assert int(attn.error_flag.item()) == 0
    torch.testing.assert_close(out.float(), ref_out.float(), atol=ATOL, rtol=RTOL)


# Prefill: the reference's native FlashInfer path for context attention
# (sglang.patch:1303-1331): ContextAttentionMetadata.native_plan
# (context_backend.py:184-222) turns the occurrence metadata into ragged
# segments -- one per query block, or one per query where a sliding window
# meets position gaps -- and gathers their keys; FlashInfer's ragged prefill
# (backend "fa2", causal, window_left = the window) runs over them, then the
# same sink correction.  The plan is the reference's own code, loaded from
# the reference package in baseline/_ref.

PREFILL_CASES = [
    # (prefix lens, query lens, hkv, d, window, sinks, gap): gap 1 keeps every
    # request's positions consecutive (one ragged segment per request).
    ([300, 0, 1000, 17], [40, 33, 1, 200], 8, 64, -1, True, 5),
    ([300, 0, 1000, 17], [40, 33, 1, 200], 8, 64, 128, True, 5),
    ([2000, 5], [300, 64], 8, 64, 7, False, 5),
    ([64, 128], [16, 17], 2, 128, -1, True, 5),
    ([900], [130], 1, 128, 100, True, 5),
    ([5000, 3000, 1], [96, 250, 70], 8, 64, 128, True, 1),
    ([3000, 700, 0], [130, 200, 33], 8, 128, 128, True, 1),
    ([4000, 1500], [700, 300], 8, 64, -1, True, 1),
]


def _flashinfer_prefill(reference_backend, x, hkv, d, window, sinks, scale):
    dev = x["q"].device
    hq = 8 * hkv
    t64 = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.int64)).to(dev)  # noqa: E731
    cpu_fields = (x["qo"], x["kv"], None, x["qpos"].astype(np.int64),
                  x["kpos"].astype(np.int64))
    q_lengths = tuple(int(v) for v in np.diff(x["qo"]))
    metadata = reference_backend.ContextAttentionMetadata(
        t64(x["qo"]), t64(x["kv"]), t64(x["kv_idx"]), t64(x["qpos"]), t64(x["kpos"]),
        q_lengths, int(x["qo"][-1]), max(q_lengths), cpu_fields)
    cpu_qo, cpu_kv, _, _, slots, _, _ = metadata.native_plan(t64(x["births"]), window)
    work = torch.zeros(128 << 20, dtype=torch.uint8, device=dev)
    wrapper = flashinfer.BatchPrefillWithRaggedKVCacheWrapper(work, "NHD", backend="fa2")
    wrapper.plan(cpu_qo, cpu_kv, hq, hkv, d, causal=True, window_left=window,
                 logits_soft_cap=0.0, sm_scale=scale, q_data_type=torch.bfloat16,
                 kv_data_type=torch.bfloat16)
    o, lse = wrapper.run(x["q"], x["k_pool"][slots], x["v_pool"][slots], return_lse=True)
    if sinks is not None:
        o.mul_(torch.sigmoid(lse * LN2 - sinks.float()).unsqueeze(-1))
    return o, lse


@pytest.mark.parametrize("variant", [0, 5])
@pytest.mark.parametrize("case", range(len(PREFILL_CASES)))
def test_prefill_matches_flashinfer_through_the_reference_native_plan(flashinfer_ready,
                                                                      reference_backend, case,
                                                                      variant):
    """FlashInfer's fa2 prefill rounds P to bf16 for its PV product; this
    build's prefill kernels carry P as a bf16 hi + lo pair (P to about 16
    bits).  So this build's output is held to the path's tolerance against
    the exact fp32 attention, and to that tolerance plus the bound of
    FlashInfer's P rounding, 2^-8 * sum_i p_i |v_i| per element, against the
    reference's runtime output.  Variant 5 rounds P to bf16 like FlashInfer:
    it gets that bound once more against the exact attention, and twice
    against FlashInfer (two independent roundings)."""
    from test_prefill_gpu import make_batch, run_ours, torch_reference

    prefix, queries, hkv, d, window, use_sinks, gap = PREFILL_CASES[case]
    rng = np.random.default_rng(100 + case)
    x = make_batch(rng, prefix, queries, hkv, d, gap=gap)
    sinks = (2.0 * torch.randn(8 * hkv, device="cuda")) if use_sinks else None
    scale = 1.0 / math.sqrt(d)
    lse = torch.empty(x["q"].shape[0], 8 * hkv, device="cuda")
    out, _ = run_ours(x, hkv, d, window, sinks, lse=lse, variant=variant)
    ref, ref_lse2 = _flashinfer_prefill(reference_backend, x, hkv, d, window, sinks, scale)
    torch.cuda.synchronize()
    exact = torch_reference(x, window, sinks, scale)
    p_abs_v = torch_reference(dict(x, v_pool=x["v_pool"].abs()), window, sinks, scale)
    ours_round = 0 if variant == 0 else 1  # this build's P roundings of P.V
    gap = (out.float() - exact).abs() - (ATOL + RTOL * exact.abs() +
                                          ours_round * BF16_ROUND * p_abs_v)
    assert float(gap.max()) <= 0.0, f"against exact: max excess {float(gap.max()):.3g}"
    bound = ATOL + RTOL * ref.float().abs() + (1 + ours_round) * BF16_ROUND * p_abs_v
    excess = (out.float() - ref.float()).abs() - bound
    assert float(excess.max()) <= 0.0, f"max excess {float(excess.max()):.3g}"
    expect_lse = ref_lse2.float() * LN2
    if use_sinks:
        expect_lse = torch.logaddexp(expect_lse, sinks.float()[None, :])
    # FlashInfer's ragged prefill also sums bf16-rounded P into its denominator.
    torch.testing.assert_close(lse, expect_lse, atol=3.9e-3, rtol=0)
