"""Ragged prefill attention with context positions (C ABI ``akv_context_attention``).

In the reference, each layer's prefill over a context request writes the new
tokens' K/V, applies the layer's copy-on-write, then
``ContextAttentionMetadata.forward`` launches a native ragged kernel
(srt/layers/attention/context_backend.py:184-241).  Native kernels assume
contiguous positions, so for sliding-window layers whose positions have
holes ``native_plan`` splits every query of a gapped segment into its own
single-query segment and gathers its visible slots on the host
(:191-222); the sink is applied after the kernel (:244-272).

``ContextPrefillAttention`` takes the same metadata (qo_indptr, kv_indptr,
kv_indices, query and KV positions) plus the new tokens' slots, and applies
the window by position inside the kernel, so no per-query gather or dense
mask is built; the sink is part of the softmax denominator.  ``plan`` runs
once per forward on the host-known metadata (as ``native_plan`` is cached
per window); ``run`` launches on the current stream without host
synchronisation.
"""

from __future__ import annotations

import math

import numpy as np
import torch

from . import _native

QUERY_BLOCK = int(_native.lib.akv_context_attention_query_block())


class ContextPrefillAttention:
    def __init__(self, num_q_heads, num_kv_heads, head_dim, device, *, sm_scale=None):
        if num_q_heads != 8 * num_kv_heads:
            raise ValueError("context attention supports GQA groups of 8")
        if head_dim not in (64, 128):
            raise ValueError("context attention supports head_dim 64 and 128")
        device = torch.device(device)
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.device = device
        self.hq, self.hkv, self.d = num_q_heads, num_kv_heads, head_dim
        self.sm_scale = 1.0 / math.sqrt(head_dim) if sm_scale is None else float(sm_scale)
        # [0]: error bits kept across launches until check() clears them
        # (1: a slot outside the pools was read as slot 0; 2: a tensor-core
        # wait ran out and that launch's output is invalid); [1]: the abort
        # word of the current launch, cleared by every launch.
        self.error_flag = torch.zeros(2, dtype=torch.int32, device=device)
        self.n_items = 0
        self.tokens = 0
        self.window = -1

    def plan(self, qo_indptr, kv_indptr, q_positions, kv_positions, window=None):
        """Host metadata (CPU int vectors, as the reference's cpu_fields):
        one work item per block of QUERY_BLOCK queries with the key range
        its queries can reach; largest ranges first."""
        qo = np.asarray(qo_indptr, np.int64)
        kv = np.asarray(kv_indptr, np.int64)
        qpos = np.asarray(q_positions, np.int64)
        kpos = np.asarray(kv_positions, np.int64)
        if len(qo) != len(kv) or len(qo) < 1 or qo[0] != 0 or kv[0] != 0:
            raise ValueError("qo_indptr and kv_indptr must be CSR offsets of one batch")
        if len(qpos) != qo[-1] or len(kpos) != kv[-1]:
            raise ValueError("Context attention positions must align with Q/KV")
        window = -1 if window is None or window < 0 else int(window)
        # Items of QUERY_BLOCK queries, paired: consecutive blocks of one
        # request sit next to each other (a padding item {-1, 0, 0, 0}
        # completes a request's odd block), so a CTA with two query tiles
        # takes a pair and shares its K/V tiles; kernels with one tile per
        # CTA skip the padding.  Pairs with the most keys come first.
        pairs = []
        for b in range(len(qo) - 1):
            a, e, x, y = int(qo[b]), int(qo[b + 1]), int(kv[b]), int(kv[b + 1])
            n_prefix = y - x
            positions = np.concatenate((kpos[x:y], qpos[a:e]))
            if len(positions) > 1 and np.any(np.diff(positions) <= 0):
                raise ValueError("context positions must increase along each request")
            blocks = []
            for q0 in range(0, e - a, QUERY_BLOCK):
                q1 = min(q0 + QUERY_BLOCK, e - a)
                hi = n_prefix + q1
                lo = 0
                if window >= 0:
                    lo = int(np.searchsorted(positions[:hi], qpos[a + q0] - window))
                blocks.append((b, q0, lo, hi))
            for i in range(0, len(blocks), 2):
                second = blocks[i + 1] if i + 1 < len(blocks) else (-1, 0, 0, 0)
                pairs.append((blocks[i], second))
        pairs.sort(key=lambda pr: -max(it[3] - it[2] for it in pr if it[0] >= 0))
        items = [it for pr in pairs for it in pr]
        work = torch.tensor(items if items else np.zeros((0, 4)), dtype=torch.int32)
        self.work = work.reshape(-1, 4).pin_memory().to(self.device, non_blocking=True)
        self.qo_indptr = torch.from_numpy(qo.astype(np.int32)).to(self.device, non_blocking=True)
        self.kv_indptr = torch.from_numpy(kv.astype(np.int32)).to(self.device, non_blocking=True)
        self.n_items = len(items)
        self.tokens = int(qo[-1])
        self.window = window
        self.visible = self._count_visible(qo, kv, qpos, kpos, window)
        return self

    @staticmethod
    def _count_visible(qo, kv, qpos, kpos, window):
        """Number of (query, key) pairs the mask admits (for FLOP counts)."""
        total = 0
        for b in range(len(qo) - 1):
            a, e, x, y = int(qo[b]), int(qo[b + 1]), int(kv[b]), int(kv[b + 1])
            positions = np.concatenate((kpos[x:y], qpos[a:e]))
            hi = (y - x) + np.arange(1, e - a + 1)
            lo = np.zeros(e - a, np.int64) if window < 0 else \
                np.searchsorted(positions, qpos[a:e] - window)
            total += int(np.maximum(hi - lo, 0).sum())
        return total

    def run(self, q, k_pool, v_pool, kv_indices, birth_slots, q_positions, kv_positions,
            sinks=None, out=None, lse=None, variant=0):
        """q [tokens, Hq, D] bf16; pools [slots, Hkv, D] bf16; index and
        position vectors int32 on the device.  ``variant``: 0 the faster
        kernel for the shape (3 at head_dim 64, 4 at 128), 1 the mma.sync
        kernel, 2 the tcgen05 / TMEM kernel (head_dim 64), 3 its
        warp-specialised form (head_dim 64 and 128), 4 the warp-specialised
        form with two query tiles per CTA; 5 and 6 the forms of 3 and 4 with
        P rounded to bf16 for P.V (the precision of FlashInfer's prefill:
        one MMA per key block instead of the hi + lo pair, |error| up to
        2^-8 * sum p|v| more than the others)."""
        if q.dtype != torch.bfloat16 or k_pool.dtype != torch.bfloat16 or \
                v_pool.dtype != torch.bfloat16:
            raise ValueError("context attention runs on bf16 q / K / V")
        if q.shape[0] != self.tokens or q.shape[1:] != (self.hq, self.d) or q.stride(-1) != 1:
            raise ValueError("q must be [tokens, num_q_heads, head_dim] with unit last stride")
        for pool in (k_pool, v_pool):
            if pool.ndim != 3 or pool.shape[1:] != (self.hkv, self.d) or pool.stride(-1) != 1:
                raise ValueError("KV pools must be [slots, num_kv_heads, head_dim]")
        for name, t in (("kv_indices", kv_indices), ("birth_slots", birth_slots),
                        ("q_positions", q_positions), ("kv_positions", kv_positions)):
            if t.dtype != torch.int32 or t.device != q.device:
                raise ValueError(f"{name} must be an int32 tensor on the device of q")
        if sinks is not None and (sinks.dtype != torch.float32 or sinks.numel() != self.hq):
            raise ValueError("sinks must be fp32 [num_q_heads]")
        if out is None:
            out = torch.empty((self.tokens, self.hq, self.d), dtype=torch.bfloat16,
                              device=self.device)
        status = _native.lib.akv_context_attention(
            _native.ptr(q), q.stride(0), q.stride(1), _native.ptr(k_pool), _native.ptr(v_pool),
            k_pool.stride(0), k_pool.stride(1), v_pool.stride(0), v_pool.stride(1),
            min(k_pool.shape[0], v_pool.shape[0]), _native.ptr(self.qo_indptr),
            _native.ptr(self.kv_indptr), _native.ptr(kv_indices), _native.ptr(birth_slots),
            _native.ptr(q_positions), _native.ptr(kv_positions), _native.ptr(sinks),
            self.sm_scale, self.window, self.hq, self.hkv, self.d, _native.ptr(self.work),
            self.n_items, _native.ptr(out), out.stride(0), out.stride(1), _native.ptr(lse),
            _native.ptr(self.error_flag), int(variant), _native.stream_of(self.device),
        )
        _native.check(status, "context_attention")
        return out

    ERRORS = {1: "a key slot outside the KV pools was read as slot 0",
              2: "a tensor-core wait ran out; the output of that launch is invalid"}

    def errors(self) -> int:
        """Error bits of the launches since the last ``check`` (reads the
        device flag: synchronises with the current stream)."""
        return int(self.error_flag[0].item())

    def check(self):
        """Raise RuntimeError if any launch since the last check reported
        an error, and clear the error bits."""
        bits = self.errors()
        if bits:
            self.error_flag[0].zero_()
            why = "; ".join(msg for bit, msg in self.ERRORS.items() if bits & bit)
            raise RuntimeError(f"context attention: {why}")
