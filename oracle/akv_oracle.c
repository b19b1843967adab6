/*
 * akv_oracle.c -- CPU restatement of the AKV cache-operation path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker that the CUDA product
 * path is compared against.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py load it.  The product (akv_b200/) never links,
 * imports or calls anything here, and it has no CPU fallback.
 *
 * Parity pins: every function below is checked against golden vectors that
 * tests/golden/make_golden.py produced by running the reference itself (its
 * C++ event compiler built with tvm_ffi, its Triton kernels under the Triton
 * CPU interpreter).  The reference file:line that each function restates is
 * cited at the function.  Paths are relative to the reference project root.
 *
 * Build: see oracle/build_oracle.py (gcc -O2 -ffp-contract=off, so that every
 * float operation below rounds to fp32 exactly once, as the reference kernel
 * does with enable_fp_fusion=False).
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* Return codes shared with oracle/oracle.py. */
#define AKVO_OK 0
#define AKVO_INVALID 1     /* a reference `require(...)` would throw        */
#define AKVO_NO_ACTIVE 2   /* status[0] == 1 in the reference              */
#define AKVO_TOKEN_RANGE 3 /* status[0] == 2 in the reference              */
#define AKVO_CAPACITY 4    /* caller-provided output capacity too small     */

/* Record kinds of the radix key stream (context_system/ir.py:32-34). */
#define KIND_TOKEN 0
#define KIND_DELTA 1
#define KIND_REPOSITION 2

/* ------------------------------------------------------------------------ */
/* Event compiler                                                            */
/* ------------------------------------------------------------------------ */

/*
 * Restates compile_radix_reposition_layout
 * (akv/system/sglang/kernels/ops/attention/context_plan.py:210-532) and the
 * status contract of compile_context_layout (context_system/ir.py:113-274).
 *
 * The reference walks a doubly linked list of active tokens and tracks the
 * first non-compact token.  This restatement keeps the active tokens in a
 * plain ordered array instead and, at each Reposition, re-ranks every active
 * token, emitting a transition exactly for those whose position differs
 * from their rank.  The two formulations are equivalent: every active token
 * before the reference's `first_noncompact` already sits at its rank, and
 * every one from it onward sits strictly above its rank
 * (context_plan.py:421-423).
 *
 * status[0..4] = {0, key_len, stages, next_position, -1} on success,
 * {1, ., ., ., boundary} when a Reposition finds no active token, and
 * {2, ., ., ., token_id} for a token id outside [0, 2^31).
 */
int akvo_compile_layout(
    int64_t token_count, const int64_t *token_ids,
    int64_t drop_count, const int32_t *drop_insert, const int32_t *drop_range_offsets,
    int64_t range_count, const int32_t *drop_ranges,
    int64_t reposition_count, const int32_t *reposition_boundaries,
    const int32_t *reposition_insert,
    int32_t *positions, uint8_t *keep, int32_t *materialized_stage,
    int32_t *birth_positions, int32_t *birth_stages,
    int32_t *transition_offsets, int32_t *transition_raw, int32_t *transition_old,
    int32_t *transition_new, int64_t transition_capacity, int64_t *transition_count,
    int32_t *effective_stage, uint8_t *effective, uint8_t *ignored,
    int32_t *records, uint8_t *virtual_mask, int64_t *key_to_token,
    int64_t *token_to_key, int64_t *drop_event_to_key, int64_t record_capacity,
    int64_t *status)
{
    if (token_count < 0 || token_count > INT32_MAX) return AKVO_INVALID;
    if (drop_range_offsets[0] != 0 || drop_range_offsets[drop_count] != range_count)
        return AKVO_INVALID;
    for (int64_t i = 0; i < drop_count; ++i) {
        if (drop_insert[i] < 0 || drop_insert[i] > token_count) return AKVO_INVALID;
        if (i > 0 && drop_insert[i - 1] >= drop_insert[i]) return AKVO_INVALID;
        if (drop_range_offsets[i] >= drop_range_offsets[i + 1]) return AKVO_INVALID;
    }
    for (int64_t i = 0; i < reposition_count; ++i) {
        if (reposition_insert[i] != reposition_boundaries[i] + 1) return AKVO_INVALID;
        if (reposition_insert[i] <= 0 || reposition_insert[i] > token_count) return AKVO_INVALID;
        if (i > 0 && reposition_boundaries[i - 1] >= reposition_boundaries[i]) return AKVO_INVALID;
    }
    if (record_capacity < token_count + range_count + reposition_count) return AKVO_CAPACITY;

    for (int64_t i = 0; i < reposition_count; ++i) {
        effective[i] = 0;
        ignored[i] = 0;
        effective_stage[i] = -1;
    }
    for (int64_t i = 0; i < drop_count; ++i) drop_event_to_key[i] = -1;
    transition_offsets[0] = 0;
    status[0] = 0;
    status[4] = -1;

    int32_t *active = (int32_t *)malloc(sizeof(int32_t) * (size_t)(token_count + 1));
    if (!active) return AKVO_CAPACITY;
    int64_t n_active = 0;
    int32_t next_position = 0;
    int32_t stage = 0;
    int64_t cursor = 0;
    int64_t d = 0, r = 0;
    int rc = AKVO_OK;

    for (int64_t ins = 0; ins <= token_count; ++ins) {
        if (d < drop_count && drop_insert[d] == ins) {
            int32_t previous_end = -1;
            for (int32_t k = drop_range_offsets[d]; k < drop_range_offsets[d + 1]; ++k) {
                int32_t s = drop_ranges[2 * k], e = drop_ranges[2 * k + 1];
                if (!(s >= 0 && s < e && e <= ins &&
                      (k == drop_range_offsets[d] || previous_end < s))) {
                    rc = AKVO_INVALID;
                    goto done;
                }
                previous_end = e;
                for (int32_t t = s; t < e; ++t) keep[t] = 0;
            }
            int64_t w = 0;
            for (int64_t i = 0; i < n_active; ++i)
                if (keep[active[i]]) active[w++] = active[i];
            n_active = w;
            ++d;
        }
        if (r < reposition_count && reposition_insert[r] == ins) {
            if (n_active == 0) {
                status[0] = 1;
                status[4] = reposition_boundaries[r];
                rc = AKVO_NO_ACTIVE;
                goto done;
            }
            int noncompact = 0;
            for (int64_t i = 0; i < n_active; ++i)
                if (positions[active[i]] != (int32_t)i) { noncompact = 1; break; }
            if (!noncompact) {
                ignored[r] = 1;
            } else {
                ++stage;
                effective[r] = 1;
                effective_stage[r] = stage;
                for (int64_t i = 0; i < n_active; ++i) {
                    int32_t t = active[i];
                    if (positions[t] == (int32_t)i) continue;
                    if (positions[t] < (int32_t)i) { rc = AKVO_INVALID; goto done; }
                    if (cursor >= transition_capacity) { rc = AKVO_CAPACITY; goto done; }
                    transition_raw[cursor] = t;
                    transition_old[cursor] = positions[t];
                    transition_new[cursor] = (int32_t)i;
                    ++cursor;
                    positions[t] = (int32_t)i;
                    materialized_stage[t] = stage;
                }
                next_position = (int32_t)n_active;
                transition_offsets[stage] = (int32_t)cursor;
            }
            ++r;
        }
        if (ins == token_count) break;
        int32_t t = (int32_t)ins;
        keep[t] = 1;
        positions[t] = next_position++;
        birth_positions[t] = positions[t];
        birth_stages[t] = stage;
        materialized_stage[t] = stage;
        active[n_active++] = t;
    }

    /* Second pass: the radix key stream (context_plan.py:465-522). */
    {
        int64_t key = 0;
        d = 0;
        r = 0;
        for (int64_t ins = 0; ins <= token_count; ++ins) {
            if (d < drop_count && drop_insert[d] == ins) {
                drop_event_to_key[d] = key;
                for (int32_t k = drop_range_offsets[d]; k < drop_range_offsets[d + 1]; ++k) {
                    records[3 * key] = KIND_DELTA;
                    records[3 * key + 1] = (int32_t)(-(int64_t)drop_ranges[2 * k] - 1);
                    records[3 * key + 2] = (int32_t)(-(int64_t)drop_ranges[2 * k + 1] - 1);
                    virtual_mask[key] = 1;
                    key_to_token[key++] = -1;
                }
                ++d;
            }
            if (r < reposition_count && reposition_insert[r] == ins) {
                if (effective[r]) {
                    records[3 * key] = KIND_REPOSITION;
                    records[3 * key + 1] = reposition_boundaries[r];
                    records[3 * key + 2] = -1;
                    virtual_mask[key] = 1;
                    key_to_token[key++] = -1;
                }
                ++r;
            }
            if (ins == token_count) break;
            token_to_key[ins] = key;
            int64_t id = token_ids[ins];
            if (id < 0 || id > INT32_MAX) {
                status[0] = 2;
                status[4] = id;
                rc = AKVO_TOKEN_RANGE;
                goto done;
            }
            records[3 * key] = KIND_TOKEN;
            records[3 * key + 1] = (int32_t)id;
            records[3 * key + 2] = positions[ins];
            virtual_mask[key] = 0;
            key_to_token[key++] = ins;
        }
        status[0] = 0;
        status[1] = key;
        status[2] = stage;
        status[3] = next_position;
        status[4] = -1;
    }
done:
    *transition_count = cursor;
    free(active);
    return rc;
}

/* ------------------------------------------------------------------------ */
/* Reposition                                                                */
/* ------------------------------------------------------------------------ */

#define DT_F16 0
#define DT_BF16 1
#define DT_F32 2

static float bf16_to_f32(uint16_t h)
{
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* Round-to-nearest-even fp32 -> bf16, NaN kept quiet. */
static uint16_t f32_to_bf16(float f)
{
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static float load_elem(const void *base, int64_t idx, int dtype)
{
    switch (dtype) {
    case DT_F16: return (float)((const _Float16 *)base)[idx];
    case DT_BF16: return bf16_to_f32(((const uint16_t *)base)[idx]);
    default: return ((const float *)base)[idx];
    }
}

static void store_elem(void *base, int64_t idx, int dtype, float v)
{
    switch (dtype) {
    case DT_F16: ((_Float16 *)base)[idx] = (_Float16)v; break;
    case DT_BF16: ((uint16_t *)base)[idx] = f32_to_bf16(v); break;
    default: ((float *)base)[idx] = v; break;
    }
}

static void copy_elem(void *dst, const void *src, int64_t d, int64_t s, int dtype)
{
    if (dtype == DT_F32) ((float *)dst)[d] = ((const float *)src)[s];
    else ((uint16_t *)dst)[d] = ((const uint16_t *)src)[s];
}

/*
 * Restates _reposition_layers_kernel
 * (akv/system/sglang/kernels/ops/attention/context_reposition.py:28-123):
 * explicit fp32 inverse rotation by the old position (IEEE division by
 * cos^2+sin^2, :92-97), forward rotation by the new one (:101-102), the
 * same-position bit copy (:100-112), then the non-rotary K tail and all of V
 * (:114-123).  Each (token, layer, head) row is read before it is written,
 * so src == dst (in place) gives the same result as a copy.
 * Tokens are processed in [token_begin, token_end) so callers can split
 * the work across threads.
 */
int akvo_reposition(
    void *const *k_layers, void *const *v_layers, int32_t n_layers, int32_t dtype,
    int64_t k_stride_slot, int64_t k_stride_head, int64_t v_stride_slot, int64_t v_stride_head,
    int32_t num_heads, int32_t head_dim, int32_t rotary_dim, int32_t neox, int32_t skip_unmapped,
    const int32_t *src_slots, const int32_t *dst_slots, const int32_t *pairs, int64_t pair_stride,
    int64_t token_begin, int64_t token_end,
    const void *cos_sin, int32_t cs_dtype, int64_t cs_stride)
{
    if (rotary_dim <= 0 || rotary_dim > head_dim || (rotary_dim & 1)) return AKVO_INVALID;
    const int32_t half = rotary_dim / 2;
    for (int64_t t = token_begin; t < token_end; ++t) {
        int64_t src = src_slots[t], dst = dst_slots[t];
        if (skip_unmapped && (src <= 0 || dst <= 0)) continue;
        int64_t p_old = pairs[t * pair_stride], p_new = pairs[t * pair_stride + 1];
        int same = p_old == p_new;
        for (int32_t l = 0; l < n_layers; ++l) {
            void *kb = k_layers[l];
            void *vb = v_layers[l];
            for (int32_t h = 0; h < num_heads; ++h) {
                int64_t ks = src * k_stride_slot + h * k_stride_head;
                int64_t kd = dst * k_stride_slot + h * k_stride_head;
                for (int32_t i = 0; i < half; ++i) {
                    int64_t i1 = neox ? i : 2 * i;
                    int64_t i2 = neox ? half + i : 2 * i + 1;
                    float x1 = load_elem(kb, ks + i1, dtype);
                    float x2 = load_elem(kb, ks + i2, dtype);
                    float oc = load_elem(cos_sin, p_old * cs_stride + i, cs_dtype);
                    float os = load_elem(cos_sin, p_old * cs_stride + half + i, cs_dtype);
                    float nc = load_elem(cos_sin, p_new * cs_stride + i, cs_dtype);
                    float ns = load_elem(cos_sin, p_new * cs_stride + half + i, cs_dtype);
                    float oc2 = oc * oc;
                    float os2 = os * os;
                    float scale = oc2 + os2;
                    float a1 = x1 * oc;
                    float a2 = x2 * os;
                    float u1 = (a1 + a2) / scale;
                    float b1 = x2 * oc;
                    float b2 = x1 * os;
                    float u2 = (b1 - b2) / scale;
                    float c1 = u1 * nc;
                    float c2 = u2 * ns;
                    float y1 = c1 - c2;
                    float e1 = u2 * nc;
                    float e2 = u1 * ns;
                    float y2 = e1 + e2;
                    store_elem(kb, kd + i1, dtype, same ? x1 : y1);
                    store_elem(kb, kd + i2, dtype, same ? x2 : y2);
                }
                /* In place (src == dst) these copies write every element
                 * onto itself; skipping them leaves the same bytes. */
                if (src == dst) continue;
                for (int32_t j = rotary_dim; j < head_dim; ++j) copy_elem(kb, kb, kd + j, ks + j, dtype);
                int64_t vs = src * v_stride_slot + h * v_stride_head;
                int64_t vd = dst * v_stride_slot + h * v_stride_head;
                for (int32_t j = 0; j < head_dim; ++j) copy_elem(vb, vb, vd + j, vs + j, dtype);
            }
        }
    }
    return AKVO_OK;
}

/* ------------------------------------------------------------------------ */
/* Decode page table                                                         */
/* ------------------------------------------------------------------------ */

/*
 * Registry rows are six int64 cells, {raw_ids*, positions*, prompt_len,
 * active, next_pos, row*} (layers/attention/context_backend.py:716-725).
 * In the oracle the two pointers and the row pointer are host addresses.
 *
 * Restates context_decode_indices
 * (akv/system/sglang/kernels/ops/attention/context_page_table.py:34-76).
 * `starts`, `mapping` may be NULL.  All index vectors are int64 here; the
 * Python wrapper widens whatever the caller passed.
 */
int akvo_decode_indices(
    const int64_t *registry, const int32_t *table, int64_t row_stride,
    const int64_t *row_ids, const int64_t *lengths, const int64_t *indptr,
    int64_t *output, const int64_t *starts, const int64_t *mapping, int64_t multiplier,
    int64_t batch)
{
    for (int64_t b = 0; b < batch; ++b) {
        int64_t row = row_ids[b];
        int64_t length = lengths[b];
        int64_t offset = indptr[b];
        int64_t start = starts ? starts[b] : 0;
        const int64_t *entry = registry + row * 6;
        const int32_t *raw_ids = (const int32_t *)(intptr_t)entry[0];
        int32_t prompt = (int32_t)entry[2];
        int32_t active = (int32_t)entry[3];
        const int32_t *raw_row = table + row * row_stride;
        if (entry[5] != 0) raw_row = (const int32_t *)(intptr_t)entry[5];
        for (int64_t i = 0; i < length; ++i) {
            int64_t logical = start + i;
            int64_t raw = logical;
            if (entry[0] != 0)
                raw = logical < active ? (int64_t)raw_ids[logical] : prompt + logical - active;
            int64_t slot = raw_row[raw];
            if (mapping) slot = mapping[slot] * multiplier;
            output[offset + i] = slot;
        }
    }
    return AKVO_OK;
}

/*
 * Restates context_window_lengths
 * (akv/system/sglang/kernels/ops/attention/context_page_table.py:7-31):
 * the number of visible keys of a sliding-window layer, found by a binary
 * search for the first active position >= q_pos - window.
 */
int akvo_window_lengths(
    const int64_t *registry, const int64_t *row_ids, const int64_t *lengths,
    int64_t *output, int64_t window, int64_t batch)
{
    for (int64_t b = 0; b < batch; ++b) {
        const int64_t *entry = registry + row_ids[b] * 6;
        int64_t length = lengths[b];
        int64_t result = length < window ? length : window;
        if (entry[0] != 0) {
            const int32_t *pos = (const int32_t *)(intptr_t)entry[1];
            int32_t active = (int32_t)entry[3];
            int32_t next_pos = (int32_t)entry[4];
            int64_t generated = length - active;
            int64_t lower = next_pos + generated - 1 - window;
            int32_t lo = 0, hi = active;
            while (lo < hi) {
                int32_t mid = (lo + hi) / 2;
                if (pos[mid] < lower) lo = mid + 1;
                else hi = mid;
            }
            int64_t skipped = lower - next_pos > 0 ? lower - next_pos : 0;
            result = active - lo + generated - skipped;
        }
        output[b] = result;
    }
    return AKVO_OK;
}

/*
 * Restates write_row_slots
 * (akv/system/sglang/kernels/ops/memory/context_rows.py:7-15):
 * pointers[rows[i]] addresses an int32 row; write values[i] at columns[i].
 */
int akvo_write_row_slots(const int64_t *pointers, const int64_t *rows, const int64_t *columns,
                         const int64_t *values, int64_t n)
{
    for (int64_t i = 0; i < n; ++i) {
        int32_t *row = (int32_t *)(intptr_t)pointers[rows[i]];
        row[columns[i]] = (int32_t)values[i];
    }
    return AKVO_OK;
}
