"""KV-head sharding on two CPU ranks (gloo).

Each rank repositions its half of the KV heads with the oracle over the
same replicated Drop metadata; gathered back, the halves equal the
unsharded result bit for bit, every rank computed identical metadata, and
the timing reduction returns the maximum.  Needs no GPU.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from akv_b200 import tp, workloads
        from akv_b200.rope import rope_cos_sin_cache
        from oracle import oracle

        prog = workloads.c1_program(seed=3, tokens=1500)
        rows, nslots = workloads.slot_rows(np.random.default_rng(3), prog)
        res = oracle.drop_compact(prog.token_counts, prog.range_offsets, prog.ranges, rows,
                                  free_ring=np.arange(nslots, nslots + 4, dtype=np.int32),
                                  free_tail=4)
        # Replicated metadata: identical on every rank.
        digest = torch.tensor([int(np.asarray(res["src"], np.int64).sum()),
                               int(np.asarray(res["pairs"], np.int64).sum()),
                               len(res["freed"])], dtype=torch.int64)
        gathered = [torch.zeros_like(digest) for _ in range(world)]
        dist.all_gather(gathered, digest)
        same_meta = all(torch.equal(g, gathered[0]) for g in gathered)

        layers, heads, dim = 2, 8, 64
        g = np.random.default_rng(11)  # same full pools on every rank
        full_k = [g.integers(0, 1 << 16, size=(nslots, heads, dim), dtype=np.uint16) & 0x3FFF
                  for _ in range(layers)]
        cache = rope_cos_sin_cache(2048, dim, 10000.0).numpy()
        a, b = tp.kv_head_range(rank, world, heads)
        local_k = [np.ascontiguousarray(k[:, a:b]) for k in full_k]
        oracle.reposition(local_k, [np.zeros_like(k) for k in local_k], res["src"], res["dst"],
                          res["pairs"], cache, bf16=True)
        mine = torch.from_numpy(np.stack(local_k).astype(np.int32))
        parts = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(parts, mine)
        slowest = tp.max_over_ranks(float(rank + 1))
        if rank == 0:
            whole = [k.copy() for k in full_k]
            oracle.reposition(whole, [np.zeros_like(k) for k in whole], res["src"], res["dst"],
                              res["pairs"], cache, bf16=True)
            stitched = torch.cat(parts, dim=2).numpy().astype(np.uint16)
            out.put((same_meta, bool(np.array_equal(stitched, np.stack(whole))), slowest))
    finally:
        dist.destroy_process_group()


def test_head_sharded_reposition_equals_unsharded_on_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    same_meta, equal, slowest = out.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert same_meta and equal and slowest == 2.0


def test_kv_head_range():
    from akv_b200.tp import kv_head_range, shard_heads

    assert [kv_head_range(r, 4, 8) for r in range(4)] == [(0, 2), (2, 4), (4, 6), (6, 8)]
    with pytest.raises(ValueError):
        kv_head_range(0, 3, 8)
    pool = torch.arange(2 * 8 * 4).view(2, 8, 4)
    assert torch.equal(shard_heads(pool, 1, 2), pool[:, 4:8])
