"""Paged GQA decode attention with learned sinks (C ABI ``akv_decode_attention``).

The reference decodes through SGLang's native backends over the registry's
``kv_indptr / kv_indices`` (FlashInfer's decode wrapper, FA3's
``flash_attn_with_kvcache``; akv/system/sglang.patch:2170-2183) and applies
GPT-OSS sinks after the kernel, ``o *= sigmoid(lse - sink)``
(srt/layers/attention/context_backend.py:254-272, patch :2154, :2182).
``DecodeAttention`` is this package's decode kernel for the same inputs,
with the sink folded into the softmax denominator.

Like FlashInfer's ``plan`` / ``run`` split, ``plan`` takes the host-known
per-request key counts (the registry computes them on the host too:
``window_lengths_cpu``, context_backend.py:742-752) and builds the work list
-- each request cut into key ranges of at most ``chunk`` keys so that the
whole batch fills every SM -- with one pinned host-to-device copy; ``run``
launches the kernel (and, when some request was split, the combine kernel)
on the current stream with no host synchronisation.
"""

from __future__ import annotations

import math

import numpy as np
import torch

from . import _native

NUM_SMS = 148
ITEMS_PER_CTA = 4   # key ranges per persistent CTA
MAX_SPLITS = 512    # key ranges per request the combine kernel merges


class DecodeAttention:
    def __init__(self, num_q_heads, num_kv_heads, head_dim, max_batch, device, *,
                 max_items=None, sm_scale=None, ctas=None):
        if num_q_heads != 8 * num_kv_heads or num_kv_heads not in (1, 2, 4, 8):
            raise ValueError("decode attention supports GQA groups of 8 and 1-8 KV heads")
        if head_dim not in (64, 128):
            raise ValueError("decode attention supports head_dim 64 and 128")
        device = torch.device(device)
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.device = device
        self.hq, self.hkv, self.d = num_q_heads, num_kv_heads, head_dim
        self.sm_scale = 1.0 / math.sqrt(head_dim) if sm_scale is None else float(sm_scale)
        self.max_batch = int(max_batch)
        if ctas is None:
            per_sm = int(_native.lib.akv_decode_attention_ctas_per_sm(num_kv_heads, head_dim))
            if per_sm <= 0:
                raise RuntimeError("decode attention: occupancy query failed")
            sms = torch.cuda.get_device_properties(device).multi_processor_count
            ctas = per_sm * sms
        self.ctas = int(ctas)
        # Enough items for the default plan: ITEMS_PER_CTA per CTA, plus one
        # rounding remainder per request.
        self.max_items = int(max_items if max_items is not None else
                             max(ITEMS_PER_CTA, 1) * self.ctas + self.max_batch)
        n = self.max_items
        self._host = torch.empty(4 * n + 2 * self.max_batch + self.ctas + 1, dtype=torch.int32,
                                 pin_memory=True)
        self._dev = torch.empty_like(self._host, device=device)
        self.part_acc = torch.empty((n, num_q_heads, head_dim), dtype=torch.float32, device=device)
        self.part_ml = torch.empty((n, num_q_heads, 2), dtype=torch.float32, device=device)
        self.error_flag = torch.zeros(1, dtype=torch.int32, device=device)
        self._copied = torch.cuda.Event()
        self._copied.record(torch.cuda.current_stream(device))
        self.n_items = 0
        self.n_ctas = 0
        self.batch = 0
        self.split = False

    def plan(self, kv_indptr_host, chunk=None, items_per_cta=None):
        """Work list from host-known CSR offsets of the key lists.

        With ``items_per_cta`` (default ``ITEMS_PER_CTA``) the launch is
        persistent when there are more items than resident CTAs: ``ctas``
        CTAs (all that fit on the GPU at once) each run a list of items, the
        key ranges cut ``items_per_cta`` times finer than one range per CTA
        and dealt to the CTAs longest first in a back-and-forth order, so
        that every CTA ends at about the same time.  ``items_per_cta=0`` (or
        a work list no longer than the resident CTAs) launches one CTA per
        item instead."""
        indptr = np.asarray(kv_indptr_host, np.int64)
        lengths = np.diff(indptr)
        batch = len(lengths)
        if batch > self.max_batch:
            raise ValueError("batch exceeds the planned maximum")
        total = int(lengths.sum())
        per_cta = ITEMS_PER_CTA if items_per_cta is None else int(items_per_cta)
        if chunk is None:
            # Whole 32-key tiles, at least 256 keys; about `per_cta` items per
            # resident CTA (one per CTA when not persistent).
            chunk = max(256, -(-total // (self.ctas * max(1, per_cta))))
            chunk = -(-chunk // 32) * 32
        items, merge, partials = [], np.zeros((batch, 2), np.int64), 0
        for b, n in enumerate(lengths):
            start = int(indptr[b])
            if n <= chunk:
                items.append((b, start, start + int(n), -1))
                continue
            k = min(-(-int(n) // chunk), MAX_SPLITS)
            cuts = start + (np.arange(k + 1) * int(n)) // k
            merge[b] = (partials, k)
            for i in range(k):
                items.append((b, int(cuts[i]), int(cuts[i + 1]), partials + i))
            partials += k
        if len(items) > self.max_items:
            raise ValueError("work list exceeds max_items; raise max_items or the chunk")
        # Longest ranges first: the short tails fill the last wave.
        items.sort(key=lambda it: it[1] - it[2])
        work = np.asarray(items, np.int32).reshape(-1, 4)
        n = len(work)
        ctas = 0
        # With no more items than resident CTAs each item gets a CTA of its
        # own either way; the plain launch then skips the per-CTA list (one
        # dependent load: a sliding-window layer of the c4 batch, 128 items,
        # 16.5 instead of 19.6 us).
        if per_cta > 0 and n > self.ctas:
            ctas = min(self.ctas, n)
            i = np.arange(n)
            lap, pos = i // ctas, i % ctas
            owner = np.where(lap % 2 == 0, pos, ctas - 1 - pos)
            order = np.argsort(owner, kind="stable")
            work = work[order]
            cta_items = np.searchsorted(owner[order], np.arange(ctas + 1)).astype(np.int32)
        self._copied.synchronize()
        host = self._host
        mo, co = 4 * self.max_items, 4 * self.max_items + 2 * self.max_batch
        host[: 4 * n].copy_(torch.from_numpy(work.reshape(-1)))
        host[mo: mo + 2 * batch].copy_(torch.from_numpy(merge.astype(np.int32).reshape(-1)))
        if ctas:
            host[co: co + ctas + 1].copy_(torch.from_numpy(cta_items))
        self._dev[: 4 * n].copy_(host[: 4 * n], non_blocking=True)
        self._dev[mo: mo + 2 * batch].copy_(host[mo: mo + 2 * batch], non_blocking=True)
        if ctas:
            self._dev[co: co + ctas + 1].copy_(host[co: co + ctas + 1], non_blocking=True)
        self._copied.record(torch.cuda.current_stream(self.device))
        self.n_items, self.batch, self.split = n, batch, partials > 0
        self.n_ctas = ctas
        self.chunk = chunk
        return self

    def run(self, q, k_pool, v_pool, kv_indices, sinks=None, out=None, lse=None):
        """q [batch, Hq, D] bf16; pools [slots, Hkv, D] bf16; kv_indices int32."""
        if q.dtype != torch.bfloat16 or k_pool.dtype != torch.bfloat16 or \
                v_pool.dtype != torch.bfloat16:
            raise ValueError("decode attention runs on bf16 q / K / V")
        if q.shape[0] != self.batch or q.shape[1:] != (self.hq, self.d) or q.stride(-1) != 1:
            raise ValueError("q must be [batch, num_q_heads, head_dim] with unit last stride")
        for pool in (k_pool, v_pool):
            if pool.ndim != 3 or pool.shape[1:] != (self.hkv, self.d) or pool.stride(-1) != 1:
                raise ValueError("KV pools must be [slots, num_kv_heads, head_dim]")
        if kv_indices.dtype != torch.int32:
            raise ValueError("kv_indices must be int32")
        if sinks is not None and (sinks.dtype != torch.float32 or sinks.numel() != self.hq):
            raise ValueError("sinks must be fp32 [num_q_heads]")
        if out is None:
            out = torch.empty((self.batch, self.hq, self.d), dtype=torch.bfloat16,
                              device=self.device)
        mo, co = 4 * self.max_items, 4 * self.max_items + 2 * self.max_batch
        merge = self._dev[mo:] if self.split else None
        cta_items = self._dev[co:] if self.n_ctas else None
        status = _native.lib.akv_decode_attention(
            _native.ptr(q), q.stride(0), q.stride(1), _native.ptr(k_pool), _native.ptr(v_pool),
            k_pool.stride(0), k_pool.stride(1), v_pool.stride(0), v_pool.stride(1),
            min(k_pool.shape[0], v_pool.shape[0]), _native.ptr(kv_indices), _native.ptr(sinks),
            self.sm_scale, self.batch, self.hq, self.hkv, self.d, _native.ptr(self._dev),
            self.n_items, _native.ptr(cta_items), self.n_ctas, _native.ptr(merge),
            _native.ptr(self.part_acc),
            _native.ptr(self.part_ml), _native.ptr(out), out.stride(0), out.stride(1),
            _native.ptr(lse), _native.ptr(self.error_flag), _native.stream_of(self.device),
        )
        _native.check(status, "decode_attention")
        return out


def decode_attention(q, k_pool, v_pool, kv_indptr_host, kv_indices, sinks=None, sm_scale=None,
                     lse=None):
    """One-shot plan + run."""
    bs, hq, d = q.shape
    attn = DecodeAttention(hq, k_pool.shape[1], d, bs, q.device, sm_scale=sm_scale,
                           max_items=None)
    return attn.plan(kv_indptr_host).run(q, k_pool, v_pool, kv_indices, sinks=sinks, lse=lse)
