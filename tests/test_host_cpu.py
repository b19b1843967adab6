"""Host-side logic that needs no GPU: program validation, workload
generators, the closed form the drop kernels implement, RoPE tables."""

import numpy as np
import pytest

from oracle import oracle


def test_validate_program_follows_reference_rules():
    from akv_b200.context_drop import validate_program

    validate_program([10, 0, 5], [0, 2, 2, 3], [1, 3, 5, 7, 0, 2])
    with pytest.raises(ValueError, match="ordered, disjoint"):
        validate_program([10], [0, 2], [1, 5, 4, 7])  # overlapping
    with pytest.raises(ValueError, match="ordered, disjoint"):
        validate_program([10], [0, 1], [3, 3])  # empty range
    with pytest.raises(ValueError, match="does not cover"):
        validate_program([10], [0, 2], [1, 3])
    with pytest.raises(ValueError, match="ordered, disjoint"):
        validate_program([4], [0, 2], [0, 2, 2, 4])  # adjacent: previous_end < start fails
    with pytest.raises(ValueError, match="no active tokens"):
        validate_program([4], [0, 1], [0, 4])


def _validate_request_by_request(token_counts, range_offsets, ranges, reposition):
    """The rules checked one request at a time, in order, as the reference
    compiler meets them (context_plan.py:362-411); returns the message of
    the first violation or None."""
    ranges = np.asarray(ranges, np.int64).reshape(-1, 2)
    for r, t in enumerate(token_counts):
        rr = ranges[range_offsets[r]: range_offsets[r + 1]]
        if not len(rr):
            continue
        s, e = rr[:, 0], rr[:, 1]
        if np.any(s < 0) or np.any(s >= e) or np.any(e > t) or np.any(s[1:] <= e[:-1]):
            return "Drop ranges must be ordered, disjoint, and already materialized"
        if reposition and t > 0 and int((e - s).sum()) == t:
            return f"Reposition at raw boundary {int(t) - 1} has no active tokens."
    return None


@pytest.mark.parametrize("seed", range(40))
def test_validate_program_reports_the_first_failing_request(seed):
    """The vectorised check raises what a request-by-request walk raises
    first, on random batches with overlapping, empty, out-of-range and
    all-covering ranges sprinkled in."""
    from akv_b200.context_drop import validate_program

    rng = np.random.default_rng(seed)
    n = int(rng.integers(1, 12))
    counts = rng.integers(0, 40, n)
    offsets, ranges = [0], []
    for t in counts:
        k = int(rng.integers(0, 4))
        cuts = np.sort(rng.choice(np.arange(t + 1), size=min(2 * k, t + 1), replace=False))
        cuts = cuts if len(cuts) % 2 == 0 else cuts[:-1]
        pairs = cuts.reshape(-1, 2).tolist()
        kind = rng.integers(0, 30)
        if kind == 0 and pairs:
            pairs[0] = [pairs[0][1], pairs[0][0]]  # reversed
        elif kind == 1 and len(pairs) > 1:
            pairs[1][0] = pairs[0][0]  # overlap
        elif kind == 2:
            pairs.append([int(t), int(t) + 3])  # past the prompt
        elif kind == 3 and t > 0:
            pairs = [[0, int(t)]]  # everything dropped
        ranges += [x for pr in pairs for x in pr]
        offsets.append(offsets[-1] + len(pairs))
    for reposition in (True, False):
        want = _validate_request_by_request(counts, offsets, ranges, reposition)
        if want is None:
            validate_program(counts, offsets, ranges, reposition)
        else:
            with pytest.raises(ValueError) as err:
                validate_program(counts, offsets, ranges, reposition)
            assert str(err.value) == want


@pytest.mark.parametrize("seed", range(6))
def test_single_stage_closed_form_matches_compiler(seed):
    """The formulas the drop kernels evaluate (keep = not covered, rank =
    kept tokens before, moved = kept after the first drop) equal the
    reference-pinned compiler's output for one drop event + one Reposition."""
    from akv_b200 import workloads

    prog = workloads.c3_program(requests=3, max_len=6000, seed=seed)
    for r in range(prog.requests):
        t = int(prog.token_counts[r])
        rr = prog.request_ranges(r)
        lay = oracle.compile_layout(np.zeros(t), [t], [0, len(rr) // 2], rr, [t - 1], [t])
        keep = prog.keep_mask(r)
        rank = np.cumsum(keep) - keep
        first = np.flatnonzero(~keep)[0]
        moved = keep & (np.arange(t) > first)
        np.testing.assert_array_equal(lay["keep_mask"], keep)
        np.testing.assert_array_equal(lay["positions"], np.where(keep, rank, np.arange(t)))
        np.testing.assert_array_equal(lay["transition_raw_tokens"], np.flatnonzero(moved))
        np.testing.assert_array_equal(lay["transition_new_positions"], rank[moved])
        assert lay["next_position"] == (int(keep.sum()) if moved.any() else t)


def test_workloads_match_configuration():
    from akv_b200 import workloads

    c2 = workloads.c2_program()
    keep = c2.keep_mask(0)
    assert c2.total_tokens == 65536 and len(c2.ranges) == 40
    assert int((~keep).sum()) == 26425  # about 40 % dropped
    lengths = np.diff(c2.ranges.reshape(-1, 2), axis=1)
    assert lengths.min() >= 256 and lengths.max() <= 4096
    c3 = workloads.c3_program()
    assert c3.requests == 64 and 1024 <= c3.meta["prefix"] <= 4096
    for r in range(c3.requests):
        rr = c3.request_ranges(r)
        assert rr[0] < c3.meta["prefix"] // 2  # first span inside the shared prefix
    c4 = workloads.c4_lengths()
    assert len(c4) == 128 and c4.max() <= 65536 and abs(np.median(c4) - 8192) < 2500
    c5 = workloads.c5_program(requests=2)
    assert abs(int((~c5.keep_mask(0)).sum()) / 131072 - 0.3) < 0.02


def test_yarn_table_magnitude():
    from akv_b200.rope import rope_cos_sin_cache, yarn_cos_sin_cache

    t = yarn_cos_sin_cache(1024, 64, 150000.0, 32.0, 4096).numpy()
    mag = t[:, :32] ** 2 + t[:, 32:] ** 2
    want = (0.1 * np.log(32.0) + 1.0) ** 2
    np.testing.assert_allclose(mag, want, rtol=1e-5)
    p = rope_cos_sin_cache(16, 8, 10000.0).numpy()
    np.testing.assert_allclose(p[:, :4] ** 2 + p[:, 4:] ** 2, 1.0, rtol=1e-6)
    np.testing.assert_allclose(p[3, 0], np.cos(3.0), rtol=1e-6)


def test_reference_compiler_matches_oracle_at_c2_size():
    """When the reference's own compiler is built (oracle/_ref), it agrees
    with the oracle on the full GPT-OSS-shaped program."""
    from oracle import reference
    from akv_b200 import workloads

    if not reference.available():
        pytest.skip("reference compiler not built here")
    prog = workloads.c2_program()
    t = prog.total_tokens
    rr = prog.request_ranges(0)
    args = (np.arange(t) % 1000, [t], [0, len(rr) // 2], rr, [t - 1], [t])
    a = reference.compile_context_layout(*args)
    b = oracle.compile_layout(*args)
    for k in ("positions", "keep_mask", "transition_raw_tokens", "transition_old_positions",
              "transition_new_positions", "records", "birth_positions", "materialized_stage"):
        np.testing.assert_array_equal(np.asarray(a[k]).astype(np.int64),
                                      np.asarray(b[k]).astype(np.int64), err_msg=k)
    assert a["next_position"] == b["next_position"]


@pytest.mark.parametrize("truncate", [True, False])
def test_yarn_table_matches_the_serving_stacks(truncate):
    """The YaRN table of akv_b200.rope against the two serving-stack
    implementations present in this image, for the GPT-OSS settings (head_dim 64,
    theta 150,000, factor 32 over 4,096 positions, beta 32 / 1): vLLM's
    YaRN rotary module's cos/sin buffer (the class SGLang's is adapted
    from) and transformers' YaRN inverse frequencies and attention factor,
    with the ramp bounds rounded out (truncate) and left fractional, as the
    GPT-OSS checkpoints ask."""
    import torch

    from akv_b200.rope import yarn_cos_sin_cache

    ours = yarn_cos_sin_cache(8192, 64, 150000.0, 32.0, 4096, truncate=truncate)
    rope_mod = pytest.importorskip("vllm.model_executor.layers.rotary_embedding")
    from vllm.model_executor.layers.rotary_embedding.common import yarn_get_mscale

    # The class's own table methods, on an object holding the attributes its
    # constructor sets (the constructor itself wants a vLLM device config).
    yarn = rope_mod.YaRNScalingRotaryEmbedding

    class Stand:
        _compute_inv_freq = yarn._compute_inv_freq
        _compute_cos_sin_cache = yarn._compute_cos_sin_cache

    emb = Stand()
    emb.rotary_dim, emb.base, emb.max_position_embeddings = 64, 150000.0, 4096
    emb.scaling_factor, emb.extrapolation_factor, emb.attn_factor = 32.0, 1, 1
    emb.beta_fast, emb.beta_slow, emb.truncate = 32, 1, truncate
    emb.mscale = float(yarn_get_mscale(32.0))
    theirs = emb._compute_cos_sin_cache()[:8192]
    assert torch.equal(ours, theirs)  # bit for bit

    from transformers import PretrainedConfig
    from transformers.modeling_rope_utils import ROPE_INIT_FUNCTIONS

    cfg = PretrainedConfig()
    cfg.hidden_size, cfg.num_attention_heads, cfg.head_dim = 64 * 64, 64, 64
    cfg.max_position_embeddings = 131072
    cfg.rope_parameters = {"rope_type": "yarn", "rope_theta": 150000.0, "factor": 32.0,
                           "beta_fast": 32.0, "beta_slow": 1.0,
                           "original_max_position_embeddings": 4096, "truncate": truncate}
    inv_freq, attention_factor = ROPE_INIT_FUNCTIONS["yarn"](cfg, "cpu")
    n = 100
    pos = torch.arange(n, dtype=torch.float32)
    ang = torch.outer(pos, inv_freq.float())
    want = torch.cat((ang.cos(), ang.sin()), dim=-1) * attention_factor
    torch.testing.assert_close(ours[:n], want, atol=2e-6, rtol=0)
