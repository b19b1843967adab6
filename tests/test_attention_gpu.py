"""Paged GQA decode attention with sinks (C ABI akv_decode_attention).

Checked against the float64 CPU oracle and a plain PyTorch fp32 reference
of the same op, within the tolerance the path states for attention:
atol 2e-3, rtol 1e-2 on the bf16 output.  The sink correction itself is
pinned to the reference's flash_attention_with_sink by
tests/test_oracle_golden.py, and the kernel to the reference's runtime
decode path (FlashInfer plus the sink patch) by
tests/test_flashinfer_pin_gpu.py.
"""

import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2


def torch_reference(q, k_pool, v_pool, indptr, indices, sinks, scale):
    """fp32 torch: gather keys, softmax over [scores | sink], drop the sink column."""
    bs, hq, d = q.shape
    hkv = k_pool.shape[1]
    out = torch.zeros(bs, hq, d, dtype=torch.float32, device=q.device)
    lse = torch.full((bs, hq), float("-inf"), device=q.device)
    for b in range(bs):
        idx = indices[indptr[b]: indptr[b + 1]].long()
        k = k_pool[idx].float().repeat_interleave(hq // hkv, dim=1)  # [n, hq, d]
        v = v_pool[idx].float().repeat_interleave(hq // hkv, dim=1)
        s = torch.einsum("hd,nhd->hn", q[b].float(), k) * scale
        if sinks is not None:
            s = torch.cat((s, sinks.float()[:, None]), dim=1)
        if s.shape[1] == 0:
            continue
        lse[b] = torch.logsumexp(s, dim=1)
        p = torch.softmax(s, dim=1)
        if sinks is not None:
            p = p[:, :-1]
        out[b] = torch.einsum("hn,nhd->hd", p, v)
    return out, lse


def _case(lengths, hkv, d, sinks, seed=0, chunk=None, slots=None, ctas=None):
    from akv_b200.context_attention import DecodeAttention

    dev = torch.device("cuda")
    rng = np.random.default_rng(seed)
    g = torch.Generator(device="cpu").manual_seed(seed)
    hq = 8 * hkv
    bs = len(lengths)
    total = int(np.sum(lengths))
    slots = slots or max(16, total + 8)
    k_pool = torch.randn(slots, hkv, d, generator=g).to(torch.bfloat16)
    v_pool = torch.randn(slots, hkv, d, generator=g).to(torch.bfloat16)
    q = torch.randn(bs, hq, d, generator=g).to(torch.bfloat16)
    indptr = np.concatenate(([0], np.cumsum(lengths))).astype(np.int64)
    indices = rng.integers(1, slots, size=total).astype(np.int32)
    sk = torch.randn(hq, generator=g) if sinks else None
    scale = 1.0 / np.sqrt(d)
    attn = DecodeAttention(hq, hkv, d, bs, dev, ctas=ctas,
                           max_items=4096 if ctas is not None else None)
    lse = torch.empty(bs, hq, device=dev)
    out = attn.plan(indptr, chunk=chunk).run(
        q.to(dev), k_pool.to(dev), v_pool.to(dev), torch.from_numpy(indices).to(dev),
        sinks=sk.to(dev) if sk is not None else None, lse=lse)
    torch.cuda.synchronize()
    assert int(attn.error_flag.item()) == 0
    ref_out, ref_lse = torch_reference(q.to(dev), k_pool.to(dev), v_pool.to(dev), indptr,
                                       torch.from_numpy(indices).to(dev),
                                       sk.to(dev) if sk is not None else None, scale)
    torch.testing.assert_close(out.float(), ref_out, atol=ATOL, rtol=RTOL)
    finite = torch.isfinite(ref_lse)
    torch.testing.assert_close(lse[finite], ref_lse[finite], atol=1e-3, rtol=1e-4)
    assert torch.equal(torch.isfinite(lse), finite)
    return q, k_pool, v_pool, indptr, indices, sk, out


@pytest.mark.parametrize("hkv", [1, 2, 4, 8])
@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("sinks", [False, True])
def test_decode_attention_matches_torch_fp32(hkv, d, sinks):
    lengths = [1, 17, 0, 300, 64, 2049, 5]
    _case(lengths, hkv, d, sinks, seed=hkv * 10 + d)


@pytest.mark.parametrize("ctas", [None, 3])
@pytest.mark.parametrize("chunk", [32, 96, 1024])
def test_decode_attention_split_and_combine(chunk, ctas):
    """Requests split into several key ranges combine to the same result,
    with one CTA per range and with 3 persistent CTAs running lists."""
    lengths = [3000, 1, 33, 700, 0, 4097]
    _case(lengths, 8, 64, True, seed=chunk, chunk=chunk, ctas=ctas)


def test_decode_attention_matches_float64_oracle():
    q, k_pool, v_pool, indptr, indices, sk, out = _case([513, 40, 1500], 8, 64, True, seed=3)
    want, _ = oracle.decode_attention(q.float().numpy(), k_pool.float().numpy(),
                                      v_pool.float().numpy(), indptr, indices,
                                      sinks=sk.numpy())
    np.testing.assert_allclose(out.float().cpu().numpy(), want, atol=ATOL, rtol=RTOL)


def test_decode_attention_c4_batch():
    """Batch 128, 64 q heads / 8 KV heads, head_dim 64, lognormal lengths
    (median 8K, capped here at 16K to keep the fp32 torch check quick)."""
    from akv_b200 import workloads

    lengths = np.minimum(workloads.c4_lengths(batch=128), 16384)
    _case(lengths, 8, 64, True, seed=4)


def test_decode_attention_rejects_bad_shapes():
    from akv_b200.context_attention import DecodeAttention

    with pytest.raises(ValueError):
        DecodeAttention(48, 8, 64, 4, "cuda")  # group 6
    with pytest.raises(ValueError):
        DecodeAttention(64, 8, 96, 4, "cuda")  # head_dim 96
