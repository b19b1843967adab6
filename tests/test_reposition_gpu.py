"""Reposition kernel (C ABI akv_reposition_kv_layers) against the reference.

* golden cases: outputs of the reference's Triton kernel
  (context_reposition.py:28-123) run by tests/golden/make_golden.py -- fp32
  storage bit for bit, bf16 storage as the round-to-nearest-even of the
  reference's fp32 values (what a GPU store does);
* random and benchmark-shaped cases against the pinned CPU oracle, bit for
  bit, for bf16 / fp16 / fp32 storage, NEOX and GPT-J styles, partial
  rotary_dim, copy-on-write and in-place transitions.
"""

import numpy as np
import pytest
import torch

from conftest import golden

pytestmark = pytest.mark.gpu

RP = golden("reposition")
RP_CASES = sorted({k.split("/")[0] for k in RP.files})


def _rp():
    from akv_b200.context_reposition import reposition_kv_layers, layer_pointer_table

    return reposition_kv_layers, layer_pointer_table


def _bits_to_f32(bits):
    return (bits.astype(np.uint16).astype(np.uint32) << 16).view(np.float32)


def _f32_to_bf16_bits(x):
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), r)


def _golden_layers(case, storage):
    n, layers, heads, dim, rot, neox, pad, skip = (int(x) for x in RP[f"{case}/spec"])
    k_bits, v_bits = RP[f"{case}/k_in"], RP[f"{case}/v_in"]
    dev = torch.device("cuda")
    if storage == "f32":
        ks = [torch.from_numpy(_bits_to_f32(k_bits[i])).to(dev) for i in range(layers)]
        vs = [torch.from_numpy(_bits_to_f32(v_bits[i])).to(dev) for i in range(layers)]
    else:
        ks = [torch.from_numpy(k_bits[i].copy()).to(dev).view(torch.bfloat16) for i in range(layers)]
        vs = [torch.from_numpy(v_bits[i].copy()).to(dev).view(torch.bfloat16) for i in range(layers)]
    return (n, layers, heads, dim, rot, neox, pad, skip), ks, vs


@pytest.mark.parametrize("storage", ["f32", "bf16"])
@pytest.mark.parametrize("case", RP_CASES)
def test_reposition_matches_reference_golden(case, storage):
    reposition_kv_layers, table = _rp()
    (n, layers, heads, dim, rot, neox, pad, skip), k_full, v_full = _golden_layers(case, storage)
    ks = [k[..., :dim] for k in k_full]
    vs = [v[..., :dim] for v in v_full]
    dev = ks[0].device
    cache = torch.from_numpy(RP[f"{case}/cache"]).to(dev)
    src = torch.from_numpy(RP[f"{case}/src"]).to(dev)
    dst = torch.from_numpy(RP[f"{case}/dst"]).to(dev)
    pairs = torch.from_numpy(RP[f"{case}/pairs"]).to(dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    reposition_kv_layers(table(ks), table(vs), ks[0], vs[0], src, dst, pairs, cache,
                         is_neox_style=bool(neox), skip_unmapped=bool(skip), rotary_dim=rot,
                         error_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    rows = np.clip(RP[f"{case}/dst"].astype(np.int64), 0, None)
    for layer in range(layers):
        got_k = k_full[layer].cpu()
        got_v = v_full[layer].cpu()
        want_k, want_v = RP[f"{case}/k_out_dst"][layer], RP[f"{case}/v_out_dst"][layer]
        if storage == "f32":
            np.testing.assert_array_equal(got_k.numpy()[rows], want_k)
            np.testing.assert_array_equal(got_v.numpy()[rows], want_v)
        else:
            np.testing.assert_array_equal(got_k.view(torch.int16).numpy().view(np.uint16)[rows],
                                          _f32_to_bf16_bits(want_k))
            np.testing.assert_array_equal(got_v.view(torch.int16).numpy().view(np.uint16)[rows],
                                          _f32_to_bf16_bits(want_v))
        # rows that are not destinations are untouched (padding included)
        mask = np.ones(got_k.shape[0], bool)
        mask[rows] = False
        k_in = RP[f"{case}/k_in"][layer]
        if storage == "f32":
            np.testing.assert_array_equal(got_k.numpy()[mask], _bits_to_f32(k_in)[mask])
        else:
            np.testing.assert_array_equal(got_k.view(torch.int16).numpy()[mask], k_in[mask])


def _random_case(rng, *, dtype, layers, heads, dim, rot, neox, n, slots, in_place, pad=0,
                 cache_dtype=torch.float32, max_pos=4096, yarn=False, bulk=False):
    """``in_place``: True (every transition in place), False (every one a
    copy) or "mixed" (every third in place, the rest copies)."""
    from oracle import oracle
    from akv_b200.rope import rope_cos_sin_cache, yarn_cos_sin_cache

    reposition_kv_layers, table = _rp()
    width = dim + pad
    k_full = [torch.randn(slots, heads, width).to(dtype) for _ in range(layers)]
    v_full = [torch.randn(slots, heads, width).to(dtype) for _ in range(layers)]
    perm = rng.permutation(np.arange(1, slots))
    src = perm[:n].astype(np.int32)
    dst = src.copy() if in_place is True else perm[n: 2 * n].astype(np.int32)
    if in_place == "mixed":
        dst[::3] = src[::3]
    old = rng.integers(0, max_pos, size=n)
    new = rng.integers(0, max_pos, size=n)
    new[::9] = old[::9]
    pairs = np.stack((old, new), 1).astype(np.int32)
    if yarn:
        cache = yarn_cos_sin_cache(max_pos, rot, 150000.0, 32.0, 4096)
    else:
        cache = rope_cos_sin_cache(max_pos, rot, 10000.0)
    cache = cache.to(cache_dtype)

    # oracle on host copies
    def host(t):
        if t.dtype == torch.bfloat16:
            return t.view(torch.int16).numpy().view(np.uint16).copy()
        return t.numpy().copy()

    hk = [host(k) for k in k_full]
    hv = [host(v) for v in v_full]
    cache_host = host(cache)
    oracle.reposition([a[..., :dim] for a in hk], [a[..., :dim] for a in hv], src, dst, pairs,
                      cache_host, is_neox_style=neox, rotary_dim=rot,
                      bf16=dtype == torch.bfloat16, cache_bf16=cache_dtype == torch.bfloat16,
                      threads=4)
    dev = torch.device("cuda")
    dk = [k.to(dev) for k in k_full]
    dv = [v.to(dev) for v in v_full]
    ks = [k[..., :dim] for k in dk]
    vs = [v[..., :dim] for v in dv]
    reposition_kv_layers(table(ks), table(vs), ks[0], vs[0], torch.from_numpy(src).to(dev),
                         torch.from_numpy(dst).to(dev), torch.from_numpy(pairs).to(dev),
                         cache.to(dev), is_neox_style=neox, rotary_dim=rot, bulk_copy_v=bulk)
    torch.cuda.synchronize()
    for layer in range(layers):
        np.testing.assert_array_equal(host(dk[layer].cpu()), hk[layer])
        np.testing.assert_array_equal(host(dv[layer].cpu()), hv[layer])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("neox", [True, False])
@pytest.mark.parametrize("in_place", [True, False])
def test_reposition_random_matches_oracle(dtype, neox, in_place):
    rng = np.random.default_rng(1)
    _random_case(rng, dtype=dtype, layers=3, heads=8, dim=64, rot=64, neox=neox, n=300,
                 slots=1000, in_place=in_place, yarn=True)


@pytest.mark.parametrize(
    "heads,dim,rot,pad,cache_dtype,layers",
    [(4, 128, 128, 0, torch.float32, 5), (2, 128, 64, 0, torch.bfloat16, 5),
     (3, 96, 32, 8, torch.float32, 5), (1, 40, 24, 0, torch.float16, 5),
     (8, 64, 64, 4, torch.float32, 5), (5, 80, 80, 0, torch.float32, 5),
     # one rank's share of 8-way KV-head sharding: c2 (36 layers) and c5 (80 layers)
     (1, 64, 64, 0, torch.float32, 36), (1, 128, 128, 0, torch.float32, 80),
     (2, 128, 128, 0, torch.float32, 80)],
)
def test_reposition_shapes_match_oracle(heads, dim, rot, pad, cache_dtype, layers):
    rng = np.random.default_rng(heads * 1000 + dim)
    for in_place in (True, False):
        _random_case(rng, dtype=torch.bfloat16, layers=layers, heads=heads, dim=dim, rot=rot,
                     neox=True, n=257, slots=800, in_place=in_place, pad=pad,
                     cache_dtype=cache_dtype)


@pytest.mark.parametrize(
    "dtype,heads,dim,rot,pad,neox,in_place",
    [(torch.bfloat16, 8, 64, 64, 0, True, "mixed"), (torch.bfloat16, 8, 64, 64, 0, False, False),
     (torch.float16, 4, 128, 128, 0, True, "mixed"), (torch.bfloat16, 1, 64, 64, 0, True, False),
     (torch.bfloat16, 2, 128, 128, 0, True, "mixed"), (torch.bfloat16, 8, 128, 128, 0, True, True),
     # the option does not apply (the main kernel moves V): padded heads,
     # partial rotary, fp32 storage
     (torch.bfloat16, 8, 64, 64, 8, True, "mixed"), (torch.bfloat16, 4, 128, 64, 0, True, False),
     (torch.float32, 4, 64, 64, 0, True, "mixed")],
)
def test_reposition_bulk_v_move_matches_oracle(dtype, heads, dim, rot, pad, neox, in_place):
    """AKV_REPOSITION_BULK_V (copy V rows moved by TMA bulk copies in a
    second kernel): bit for bit the oracle's result, as without it."""
    rng = np.random.default_rng(heads * 100 + dim + pad)
    _random_case(rng, dtype=dtype, layers=7, heads=heads, dim=dim, rot=rot, neox=neox, n=700,
                 slots=2000, in_place=in_place, pad=pad, yarn=True, bulk=True)


def test_reposition_bulk_v_move_with_device_count_and_skips():
    """Bulk V move over a device-counted prefix of the list, with
    skip_unmapped rows and an out-of-range destination."""
    from oracle import oracle
    from akv_b200.rope import rope_cos_sin_cache

    reposition_kv_layers, table = _rp()
    rng = np.random.default_rng(21)
    dev = torch.device("cuda")
    slots, heads, dim, layers, n = 1500, 8, 64, 4, 600
    ks = [torch.randn(slots, heads, dim).to(torch.bfloat16) for _ in range(layers)]
    vs = [torch.randn(slots, heads, dim).to(torch.bfloat16) for _ in range(layers)]
    perm = rng.permutation(np.arange(1, slots))
    src, dst = perm[:n].astype(np.int32), perm[n: 2 * n].astype(np.int32)
    dst[1::4] = src[1::4]
    src[5] = 0  # skip_unmapped: slot 0 is not mapped
    dst[9] = slots + 7  # outside the pool: skipped and flagged
    pairs = rng.integers(0, 3000, size=(n, 2)).astype(np.int32)
    cache = rope_cos_sin_cache(3000, dim, 10000.0)
    used = 450
    keep = np.arange(used)
    keep = keep[(keep != 5) & (keep != 9)]
    host = lambda t: t.view(torch.int16).numpy().view(np.uint16).copy()  # noqa: E731
    hk, hv = [host(k) for k in ks], [host(v) for v in vs]
    oracle.reposition(hk, hv, src[keep], dst[keep], pairs[keep], cache.numpy(), bf16=True)
    dk, dv = [k.to(dev) for k in ks], [v.to(dev) for v in vs]
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    cnt = torch.tensor([used], dtype=torch.int32, device=dev)
    reposition_kv_layers(table(dk), table(dv), dk[0], dv[0], torch.from_numpy(src).to(dev),
                         torch.from_numpy(dst).to(dev), torch.from_numpy(pairs).to(dev),
                         cache.to(dev), skip_unmapped=True, count_device=cnt, error_flag=err,
                         bulk_copy_v=True)
    torch.cuda.synchronize()
    assert int(err.item()) == 1
    for layer in range(layers):
        np.testing.assert_array_equal(host(dk[layer].cpu()), hk[layer])
        np.testing.assert_array_equal(host(dv[layer].cpu()), hv[layer])


def test_reposition_misaligned_layer_matches_oracle():
    """A layer whose base address is not 16-byte aligned takes the element path."""
    from oracle import oracle
    from akv_b200.rope import rope_cos_sin_cache

    reposition_kv_layers, table = _rp()
    rng = np.random.default_rng(5)
    dev = torch.device("cuda")
    slots, heads, dim = 300, 8, 64
    base = torch.randn(slots * heads * dim + 8).to(torch.bfloat16)
    k0 = base[4: 4 + slots * heads * dim].view(slots, heads, dim)  # 8-byte offset
    k1 = torch.randn(slots, heads, dim).to(torch.bfloat16)
    v0 = torch.randn(slots, heads, dim).to(torch.bfloat16)
    v1 = torch.randn(slots, heads, dim).to(torch.bfloat16)
    n = 100
    perm = rng.permutation(np.arange(1, slots))
    src, dst = perm[:n].astype(np.int32), perm[n: 2 * n].astype(np.int32)
    pairs = rng.integers(0, 1000, size=(n, 2)).astype(np.int32)
    cache = rope_cos_sin_cache(1000, dim, 10000.0)
    host = [t.view(torch.int16).numpy().view(np.uint16).copy() for t in (k0, k1, v0, v1)]
    oracle.reposition(host[:2], host[2:], src, dst, pairs, cache.numpy(), bf16=True)
    for bulk in (False, True):
        dbase = base.to(dev)
        dk0 = dbase[4: 4 + slots * heads * dim].view(slots, heads, dim)
        dk1, dv0, dv1 = k1.to(dev), v0.to(dev), v1.to(dev)
        reposition_kv_layers(table([dk0, dk1]), table([dv0, dv1]), dk1, dv1,
                             torch.from_numpy(src).to(dev), torch.from_numpy(dst).to(dev),
                             torch.from_numpy(pairs).to(dev), cache.to(dev), bulk_copy_v=bulk)
        torch.cuda.synchronize()
        for got, want in zip((dk0, dk1, dv0, dv1), host):
            np.testing.assert_array_equal(got.cpu().view(torch.int16).numpy().view(np.uint16),
                                          want)


def test_reposition_count_device_and_bounds():
    from akv_b200.rope import rope_cos_sin_cache

    reposition_kv_layers, table = _rp()
    dev = torch.device("cuda")
    k = torch.randn(64, 2, 64, device=dev).to(torch.bfloat16)
    v = torch.randn(64, 2, 64, device=dev).to(torch.bfloat16)
    k0, v0 = k.clone(), v.clone()
    src = torch.tensor([1, 2, 3, 4], dtype=torch.int32, device=dev)
    dst = torch.tensor([11, 12, 13, 999], dtype=torch.int32, device=dev)  # 999 out of range
    pairs = torch.tensor([[5, 1], [6, 2], [7, 3], [8, 4]], dtype=torch.int32, device=dev)
    cache = rope_cos_sin_cache(16, 64, 10000.0).to(dev)
    count = torch.tensor([2], dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    reposition_kv_layers(table([k]), table([v]), k, v, src, dst, pairs, cache, count_device=count,
                         error_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert not torch.equal(k[11], k0[11]) and torch.equal(v[12], v0[2])
    assert torch.equal(k[13], k0[13])  # beyond the device count: untouched
    count.fill_(4)
    reposition_kv_layers(table([k]), table([v]), k, v, src, dst, pairs, cache, count_device=count,
                         error_flag=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 1  # the out-of-range destination was skipped and reported
    assert torch.equal(v[13], v0[3])


def test_reposition_validation_errors():
    reposition_kv_layers, table = _rp()
    dev = torch.device("cuda")
    k = torch.zeros(8, 2, 64, device=dev, dtype=torch.bfloat16)
    ptrs = table([k])
    s = torch.zeros(1, dtype=torch.int32, device=dev)
    pairs = torch.zeros(1, 2, dtype=torch.int32, device=dev)
    cache = torch.zeros(4, 64, device=dev)
    for bad in (2, 12, 256):  # the paged Drop's page sizes are powers of two in [4, 128]
        with pytest.raises(ValueError, match="page_size=1"):
            reposition_kv_layers(ptrs, ptrs, k, k, s, s, pairs, cache, page_size=bad)
    reposition_kv_layers(ptrs, ptrs, k, k, s, s, pairs, cache, page_size=16)  # token slots
    with pytest.raises(ValueError, match="int32 slot vectors"):
        reposition_kv_layers(ptrs, ptrs, k, k, s.long(), s, pairs, cache)
    with pytest.raises(ValueError, match="cos/sin cache"):
        reposition_kv_layers(ptrs, ptrs, k, k, s, s, pairs, cache[:, :32])
    with pytest.raises(ValueError, match="cos/sin cache"):
        reposition_kv_layers(ptrs, ptrs, k, k, s, s, pairs, cache, rotary_dim=63)
    with pytest.raises(ValueError, match="one CUDA device"):
        reposition_kv_layers(ptrs, ptrs, k, k, s.cpu(), s, pairs, cache)
    # empty transition list: no launch, no error
    e = torch.zeros(0, dtype=torch.int32, device=dev)
    reposition_kv_layers(ptrs, ptrs, k, k, e, e, e.view(0, 2), cache)


def test_reposition_c2_shape_sampled_rows_match_oracle():
    """Full GPT-OSS-shaped launch (36 layers, 8 heads, head_dim 64, YaRN,
    38.9K transitions in place); every row depends only on its own input, so
    a sample of transitions checked on the CPU is an exact check of them."""
    from oracle import oracle
    from akv_b200 import workloads
    from akv_b200.rope import yarn_cos_sin_cache

    reposition_kv_layers, table = _rp()
    dev = torch.device("cuda")
    prog = workloads.c2_program()
    T = int(prog.token_counts[0])
    keep = prog.keep_mask(0)
    rank = np.cumsum(keep) - 1
    moved = np.flatnonzero(keep & (np.arange(T) > np.flatnonzero(~keep)[0]))
    rng = np.random.default_rng(0)
    row = rng.permutation(T).astype(np.int32) + 1
    src = row[moved]
    pairs = np.stack((moved, rank[moved]), 1).astype(np.int32)
    layers, heads, dim = 36, 8, 64
    g = torch.Generator(device=dev).manual_seed(0)
    ks = [torch.randn(T + 1, heads, dim, device=dev, generator=g).to(torch.bfloat16)
          for _ in range(layers)]
    vs = [torch.empty(T + 1, heads, dim, device=dev, dtype=torch.bfloat16) for _ in range(layers)]
    cache = yarn_cos_sin_cache(131072, dim, 150000.0, 32.0, 4096)
    sample = rng.choice(len(moved), size=2000, replace=False)
    before = [k[torch.from_numpy(src[sample].astype(np.int64)).to(dev)].cpu() for k in ks]
    s = torch.from_numpy(src).to(dev)
    reposition_kv_layers(table(ks), table(vs), ks[0], vs[0], s, s,
                         torch.from_numpy(pairs).to(dev), cache.to(dev))
    torch.cuda.synchronize()
    hk = [b.view(torch.int16).numpy().view(np.uint16).copy() for b in before]
    hv = [np.zeros_like(a) for a in hk]
    idx = np.arange(len(sample), dtype=np.int32)
    oracle.reposition(hk, hv, idx, idx, pairs[sample], cache.numpy(), bf16=True, threads=4)
    for layer in range(layers):
        got = ks[layer][torch.from_numpy(src[sample].astype(np.int64)).to(dev)].cpu()
        np.testing.assert_array_equal(got.view(torch.int16).numpy().view(np.uint16), hk[layer])


def _random_floats(rng, n, lo_exp, hi_exp):
    """fp32 values with uniformly random exponents and mantissas, both signs."""
    exp = rng.integers(lo_exp + 127, hi_exp + 127 + 1, size=n).astype(np.uint32)
    mant = rng.integers(0, 1 << 23, size=n, dtype=np.uint32)
    sign = rng.integers(0, 2, size=n, dtype=np.uint32) << 31
    return (sign | (np.clip(exp, 0, 254) << 23) | mant).view(np.float32)


def test_reposition_division_matches_ieee():
    """The kernel's division (Markstein correction over a per-token
    reciprocal, IEEE fallback outside its range) returns exactly what IEEE
    division returns, over 48M quotients: realistic RoPE scales (plain ~1,
    YaRN ~1.81, bf16 tables), log-uniform denominators across the fast-path
    bounds, numerators over every binade, and special values."""
    from akv_b200 import _native

    dev = torch.device("cuda")
    rng = np.random.default_rng(2024)
    n = 1 << 24
    cases = []
    # 1. realistic: numerators ~ products of N(0,1) K values with cos/sin
    num = (rng.standard_normal(n) * rng.standard_normal(n)).astype(np.float32)
    den = np.where(rng.random(n) < 0.5, 1.0 + (rng.random(n) - 0.5) * 2e-7,
                   (0.1 * np.log(32) + 1) ** 2 * (1 + (rng.random(n) - 0.5) * 1e-6))
    cases.append((num, den.astype(np.float32)))
    # 2. every binade of the numerator, denominators across and beyond the bounds
    cases.append((_random_floats(rng, n, -149, 127), np.abs(_random_floats(rng, n, -80, 80))))
    # 3. numerators near the fast-path edges, random denominators near 1
    edge = np.concatenate([_random_floats(rng, n // 4, -102, -98),
                           _random_floats(rng, n // 4, 98, 102),
                           _random_floats(rng, n // 2, -30, 30)])
    cases.append((edge, np.abs(_random_floats(rng, n, -2, 2))))
    special = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-45, -1e-45, 1e-38, 3.4e38,
                        -3.4e38, 1.0, -1.0], np.float32)
    sp_n, sp_d = np.meshgrid(special, np.abs(special))
    cases.append((sp_n.reshape(-1), sp_d.reshape(-1).astype(np.float32)))
    for num, den in cases:
        a = torch.from_numpy(np.ascontiguousarray(num, np.float32)).to(dev)
        b = torch.from_numpy(np.ascontiguousarray(den, np.float32)).to(dev)
        q0 = torch.empty_like(a)
        q1 = torch.empty_like(a)
        stream = _native.stream_of(dev)
        _native.check(_native.lib.akv_reposition_divide(_native.ptr(a), _native.ptr(b),
                                                         _native.ptr(q0), a.numel(), 0, stream),
                      "divide")
        _native.check(_native.lib.akv_reposition_divide(_native.ptr(a), _native.ptr(b),
                                                         _native.ptr(q1), a.numel(), 1, stream),
                      "divide")
        torch.cuda.synchronize()
        x0, x1 = q0.view(torch.int32), q1.view(torch.int32)
        both_nan = torch.isnan(q0) & torch.isnan(q1)
        bad = (x0 != x1) & ~both_nan
        assert int(bad.sum().item()) == 0, (
            f"{int(bad.sum())} quotients differ, e.g. "
            f"{a[bad][:4].tolist()} / {b[bad][:4].tolist()}")


def test_launches_follow_the_current_torch_stream():
    """Every entry point takes the stream torch has current for the device:
    the fast lookup agrees with torch.cuda.current_stream inside and
    outside a stream context, for every way a device is named."""
    from akv_b200 import _native

    dev = torch.device("cuda", torch.cuda.current_device())
    forms = (dev, dev.index, f"cuda:{dev.index}", torch.device("cuda"))
    for s in (torch.cuda.current_stream(dev), torch.cuda.Stream(dev)):
        with torch.cuda.stream(s):
            for form in forms:
                assert _native.stream_of(form).value == s.cuda_stream or \
                    (_native.stream_of(form).value is None and s.cuda_stream == 0)
