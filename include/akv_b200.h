/*
 * akv_b200.h -- C ABI of the B200 (sm_100a) cache-operation kernels.
 *
 * Every entry point:
 *   - takes plain device pointers, sizes and strides (strides in elements),
 *     and a cudaStream_t passed as `void*` (NULL = legacy default stream);
 *   - is stream-ordered: it enqueues work and returns, with no host
 *     synchronisation, no device-to-host copy and no allocation, so it can
 *     be captured in a CUDA graph;
 *   - returns an AKV_* status.  A non-zero status means nothing was
 *     enqueued (argument errors) or the launch failed (AKV_ERR_CUDA).
 * The one host-only entry point, akv_occurrence_advance_indices, reads and
 * writes host memory and touches no device.
 *
 * Reference interfaces are cited as file:line relative to the reference
 * project root (thu-nics/AKV).
 */
#ifndef AKV_B200_H_
#define AKV_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define AKV_OK 0
#define AKV_ERR_INVALID 1     /* bad argument (shape, dtype, stride, count) */
#define AKV_ERR_CUDA 2        /* the CUDA launch failed                      */
#define AKV_ERR_UNSUPPORTED 3 /* valid but not supported by this build       */
#define AKV_ERR_OCC_MISSING_SOURCE 4      /* an ownership plan row has no owner */
#define AKV_ERR_OCC_MISSING_COPY_SOURCE 5 /* a copy's source version is absent  */

/* Device-side status bits written by akv_drop_compact into `status`. */
#define AKV_DROP_RING_UNDERFLOW 1 /* not enough free slots for copy-on-write */
#define AKV_DROP_RING_OVERFLOW 2  /* freed slots exceed the ring capacity    */
#define AKV_DROP_BAD_RANGE 4      /* a drop range lies outside its request   */
#define AKV_DROP_NO_ACTIVE 8      /* Reposition of a request with no token   */
#define AKV_DROP_BAD_PAGE 16      /* page mode: a row breaks the page layout */

/* Element types. */
#define AKV_F16 0
#define AKV_BF16 1
#define AKV_F32 2

/* Library identification: returns a static string. */
const char* akv_version(void);

/*
 * Reposition: rotate retained K rows from their old to their new RoPE
 * position and move them (and V) from source to destination slots, for
 * every layer in the pointer tables, in one launch.
 *
 * Replaces reposition_kv_layers / _reposition_layers_kernel
 * (akv/system/sglang/kernels/ops/attention/context_reposition.py:126-236,
 * :28-123).  Same arithmetic: explicit fp32 inverse rotation by the old
 * angle with IEEE division by cos^2+sin^2, forward rotation by the new one,
 * no FMA contraction, bit copy when the two positions are equal; the K
 * dims [rotary_dim, head_dim) and all of V are copied.
 *
 * k_data_ptrs / v_data_ptrs: DEVICE arrays of n_layers 64-bit base
 *   addresses of [slots, heads, head_dim] NHD pools (stride(-1) == 1).
 * source_slots / destination_slots: int32 [count]; position_pairs: int32
 *   [count, position_stride] holding (old, new) in columns 0 and 1.
 * cos_sin_cache: [max_position, rotary_dim] rows of (cos | sin), element
 *   type cache_dtype, row stride cache_stride.
 * count_device: optional DEVICE int32 holding the number of transitions to
 *   process; when non-NULL the kernel processes min(count, *count_device),
 *   so a count produced on the device needs no host round trip.
 *
 * num_slots / max_position (0 = unchecked) bound the slots and positions a
 * transition may name; a transition outside them is skipped and, when
 * error_flag (DEVICE int32, may be NULL) is given, 1 is stored there.
 *
 * A transition whose source equals its destination is rotated in place:
 * every (token, layer, head) row is read completely before it is written,
 * and the K tail and V (copies onto themselves) are skipped.  Results are
 * the same as the reference's for such rows.
 */
int akv_reposition_kv_layers(
    const void* k_data_ptrs, const void* v_data_ptrs, int32_t n_layers, int32_t kv_dtype,
    int32_t num_heads, int32_t head_dim, int32_t rotary_dim, int64_t k_stride_slot,
    int64_t k_stride_head, int64_t v_stride_slot, int64_t v_stride_head,
    const int32_t* source_slots, const int32_t* destination_slots,
    const int32_t* position_pairs, int64_t position_stride, int64_t count,
    const int32_t* count_device, const void* cos_sin_cache, int32_t cache_dtype,
    int64_t cache_stride, int32_t is_neox_style, int32_t skip_unmapped, int64_t num_slots,
    int64_t max_position, int32_t* error_flag, void* stream);

/*
 * akv_reposition_kv_layers with options; akv_reposition_kv_layers is this
 * with options 0.  No reference counterpart.
 *
 * AKV_REPOSITION_BULK_V: the V rows of copy transitions (source !=
 * destination) are moved by a second kernel that streams whole token rows
 * through shared memory with TMA bulk copies (cp.async.bulk global ->
 * shared on an mbarrier, then shared -> global), and the reposition kernel
 * moves only their K rows.  Used when the token's V row over the local
 * heads is contiguous (v_stride_head == head_dim), 16-byte aligned, at most
 * 2 KiB, and rotary_dim == head_dim; otherwise the option is ignored.  It
 * pays when copies are a minority of the list (a Drop's mixed list of
 * in-place rotations and copy-on-write: c3 step 6 % faster) and costs when
 * every transition is a copy (two passes instead of one: about 11 % slower),
 * so the caller chooses.  A bulk-copy wait that runs out (100 ms) sets bit 2
 * of *error_flag.
 */
#define AKV_REPOSITION_BULK_V 1
int akv_reposition_kv_layers_ex(
    const void* k_data_ptrs, const void* v_data_ptrs, int32_t n_layers, int32_t kv_dtype,
    int32_t num_heads, int32_t head_dim, int32_t rotary_dim, int64_t k_stride_slot,
    int64_t k_stride_head, int64_t v_stride_slot, int64_t v_stride_head,
    const int32_t* source_slots, const int32_t* destination_slots,
    const int32_t* position_pairs, int64_t position_stride, int64_t count,
    const int32_t* count_device, const void* cos_sin_cache, int32_t cache_dtype,
    int64_t cache_stride, int32_t is_neox_style, int32_t skip_unmapped, int64_t num_slots,
    int64_t max_position, int32_t* error_flag, int32_t options, void* stream);

/*
 * The correctly rounded fp32 division the reposition kernel uses, exported
 * so a caller can check it against IEEE division on its own GPU: method 0
 * is IEEE division (__fdiv_rn, the reference's tl.div_rn), method 1 the
 * kernel's path (Markstein's FMA correction over a per-token reciprocal,
 * with an IEEE fallback outside its safe range).  quotients[i] =
 * numerators[i] / denominators[i] for i < count, all DEVICE fp32.  No
 * reference counterpart: a self-check of this build's arithmetic.
 */
int akv_reposition_divide(const float* numerators, const float* denominators,
                          float* quotients, int64_t count, int32_t method, void* stream);

/*
 * Drop + Reposition of a batch of requests, on the device.
 *
 * Replaces, for programs with one Drop event and one Reposition at the end
 * of the prompt, the CPU event compiler compile_radix_reposition_layout
 * (akv/system/sglang/kernels/ops/attention/context_plan.py:210-532, via
 * srt/context_system/ir.py:113-274: keep mask, final positions, transitions
 * (raw, old, new), next_position), the decode view
 * ContextDecodeLayout.from_layout (srt/context_system/occurrence.py:47-66:
 * raw = flatnonzero(keep), positions[raw]) and the slot retirement of
 * OccurrenceState.advance / free_context_slots (occurrence.py:711-714,
 * 936-964), with copy-on-write for radix-shared slots.
 *
 * Request r owns tokens [token_offsets[r], token_offsets[r+1]) of the flat
 * per-token outputs, born at positions 0..T_r-1; its drop ranges are the
 * request-local half-open pairs ranges[2*range_offsets[r] .. 2*range_offsets[r+1]).
 * Its req_to_token row is req_to_token + row_ids[r] * row_stride (int32).
 * Tokens below shared_prefix[r] (NULL = none) are borrowed radix slots: one
 * that moves is copied to a fresh slot popped from the free ring and its row
 * entry is updated; one that is dropped is not freed.  Other moved tokens
 * are repositioned in place (source == destination).  Dropped private
 * tokens' slots are pushed onto the free ring (and listed in freed_slots).
 *
 * Free ring: ring[capacity] int32 slot ids; ring_state = {head, tail} int64
 * on the device (free entries are ring[head % capacity .. tail % capacity)).
 *
 * Outputs (device): keep_mask (uint8) and positions (int32) per flat token;
 * active_offsets[R+1], raw_indices, active_positions (compacted decode view);
 * next_position[R]; transition_offsets[R+1], transition_source,
 * transition_destination, transition_pairs [N,2], transition_raw;
 * freed_offsets[R+1], freed_slots; totals[4] = {active, transitions, cow,
 * freed}; status (AKV_DROP_* bits, 0 = ok).  Per-request counts are on the
 * device only: totals[1] can be handed to akv_reposition_kv_layers as
 * count_device without a host round trip.
 *
 * tile_offsets[R+1]: prefix sum over requests of ceil(T_r / tile_tokens),
 * n_tiles its last entry (the host knows the request lengths).
 * workspace: akv_drop_compact_workspace_bytes(n_requests, n_tiles) bytes of
 * device scratch, no initial contents required.
 */
int64_t akv_drop_compact_tile_tokens(void);
int64_t akv_drop_compact_workspace_bytes(int32_t n_requests, int32_t n_tiles);
int akv_drop_compact(
    int32_t n_requests, const int64_t* token_offsets, const int32_t* tile_offsets,
    int32_t n_tiles, const int32_t* range_offsets, const int32_t* ranges,
    const int32_t* shared_prefix, int32_t* req_to_token, const int64_t* row_ids,
    int64_t row_stride, int32_t reposition, int32_t* ring, int64_t ring_capacity,
    int64_t* ring_state, uint8_t* keep_mask, int32_t* positions, int32_t* active_offsets,
    int32_t* raw_indices, int32_t* active_positions, int32_t* next_position,
    int32_t* transition_offsets, int32_t* transition_source, int32_t* transition_destination,
    int32_t* transition_pairs, int32_t* transition_raw, int32_t* freed_offsets,
    int32_t* freed_slots, int32_t* totals, int32_t* status, void* workspace, void* stream);

/*
 * akv_drop_compact over a paged KV pool: the same computation with
 * page_size slots per page.  page_size 1 is akv_drop_compact; otherwise a
 * power of two from 4 to 128.  No counterpart in the reference, whose
 * Reposition requires page_size 1 (context_reposition.py:153-154,
 * capabilities.py:11-12); this extends it to SGLang's paged pools.
 *
 * Layout rule (checked on the device, AKV_DROP_BAD_PAGE if broken): slot s
 * is offset s % page_size of page s / page_size, and a request's token t
 * sits at offset t % page_size, so tokens [g*page_size, (g+1)*page_size)
 * of a request share one page; shared_prefix[r] is a multiple of
 * page_size.  The free ring and freed_slots hold PAGE ids, not slots.
 *   - A private page whose every token is dropped is freed (pushed in the
 *     order of its tokens; dropped tokens of other pages stay as holes).
 *   - A shared (radix) page holding a moved token is copied to one fresh
 *     page popped from the ring: each kept token of the page gets a
 *     transition to the same offset of the new page (moved tokens rotate;
 *     tokens before the first drop keep their position and are copied bit
 *     for bit) and every row entry of the page is rewritten to the new page.
 *   - Private moved tokens rotate in place.
 * totals = {active, transitions, copied pages, freed pages}.
 */
int akv_drop_compact_paged(
    int32_t n_requests, const int64_t* token_offsets, const int32_t* tile_offsets,
    int32_t n_tiles, const int32_t* range_offsets, const int32_t* ranges,
    const int32_t* shared_prefix, int32_t* req_to_token, const int64_t* row_ids,
    int64_t row_stride, int32_t reposition, int32_t page_size, int32_t* ring,
    int64_t ring_capacity, int64_t* ring_state, uint8_t* keep_mask, int32_t* positions,
    int32_t* active_offsets, int32_t* raw_indices, int32_t* active_positions,
    int32_t* next_position, int32_t* transition_offsets, int32_t* transition_source,
    int32_t* transition_destination, int32_t* transition_pairs, int32_t* transition_raw,
    int32_t* freed_offsets, int32_t* freed_slots, int32_t* totals, int32_t* status,
    void* workspace, void* stream);

/*
 * akv_drop_compact without a workspace argument: the same computation and
 * outputs, with its scratch in a file-scope device array of this library
 * instead of caller memory.  No counterpart in the reference: it is for
 * callers that cannot allocate device memory for a workspace -- a runtime
 * whose memory is all reserved for its KV pool, a caller whose allocator
 * forbids cudaMalloc on the serving path, or a C/FFI caller without a device
 * allocator.  It allocates nothing and frees nothing.
 *
 * Limits: n_requests <= akv_drop_compact_static_max_requests() (4096) and
 * n_tiles <= akv_drop_compact_static_max_tiles() (65536, i.e. 32M tokens);
 * larger calls return AKV_ERR_INVALID before any launch.  The array (about
 * 2.4 MB) is held by every GPU that loads the library until exit.  The first
 * call on a device looks the array's device address up
 * (cudaGetSymbolAddress) and caches it; make that first call before any
 * stream capture.  The cached address belongs to the device's primary
 * context as it was at that first call: after cudaDeviceReset (or anything
 * else that destroys that context) it is stale, so a process that resets a
 * device must not call this entry point on it again.  All calls on a device
 * share the array, which keeps the
 * last call's contents (nothing in it needs to start at zero): calls whose
 * kernels may overlap on the GPU race and must be ordered by the caller.
 */
int64_t akv_drop_compact_static_max_requests(void);
int64_t akv_drop_compact_static_max_tiles(void);
int akv_drop_compact_static(
    int32_t n_requests, const int64_t* token_offsets, const int32_t* tile_offsets,
    int32_t n_tiles, const int32_t* range_offsets, const int32_t* ranges,
    const int32_t* shared_prefix, int32_t* req_to_token, const int64_t* row_ids,
    int64_t row_stride, int32_t reposition, int32_t* ring, int64_t ring_capacity,
    int64_t* ring_state, uint8_t* keep_mask, int32_t* positions, int32_t* active_offsets,
    int32_t* raw_indices, int32_t* active_positions, int32_t* next_position,
    int32_t* transition_offsets, int32_t* transition_source, int32_t* transition_destination,
    int32_t* transition_pairs, int32_t* transition_raw, int32_t* freed_offsets,
    int32_t* freed_slots, int32_t* totals, int32_t* status, void* stream);

/*
 * The decode view of one akv_drop_compact (or _paged / _static) call read
 * back to host memory, stream-ordered after it on `stream`: one int32 vector
 *   [raw_indices(kept) | active_positions(kept) | active_offsets(n_requests + 1)
 *    | next_position(n_requests) | totals(4) | status]
 * at host_out (pinned memory makes the copies asynchronous).  `counters` is
 * the call's totals pointer, with the status word right after it.  This is
 * the host-side result the reference builds with
 * ContextDecodeLayout.from_layout (srt/context_system/occurrence.py:47-66),
 * here for a layout computed on the device.  `kept` is the host's count of
 * kept tokens (known from a validated program) or any larger value up to the
 * buffers' capacity.  Copies only: no launch, no synchronisation.
 */
int akv_drop_read_view(int32_t* host_out, const int32_t* raw_indices,
                       const int32_t* active_positions, int64_t kept,
                       const int32_t* active_offsets, const int32_t* next_position,
                       int32_t n_requests, const int32_t* counters, void* stream);

/*
 * General event compiler for a batch of request programs.  Replaces
 * compile_radix_reposition_layout and count_radix_reposition_transitions
 * (akv/system/sglang/kernels/ops/attention/context_plan.py:80-532) as called
 * by compile_context_layout (srt/context_system/ir.py:113-274): any number
 * of Drop events and Reposition events per request, in the reference's
 * order (a Drop runs before a Reposition at the same insertion offset), with
 * every output tensor of the reference's ContextLayout, plus the decode view
 * of ContextDecodeLayout.from_layout (srt/context_system/occurrence.py:47-66).
 *
 * Batch layout (all device pointers, request-local values as in the
 * reference): request b owns tokens [token_offsets[b], token_offsets[b+1])
 * of the flat per-token arrays; its Drop events are
 * [drop_event_offsets[b], drop_event_offsets[b+1]) of drop_insert_offsets,
 * event e owning the range pairs [drop_range_offsets[e], drop_range_offsets[e+1])
 * of drop_ranges (drop_range_offsets is one increasing vector over the whole
 * batch); its Reposition events are [reposition_offsets[b],
 * reposition_offsets[b+1]) of reposition_raw_boundaries (insertion offset =
 * boundary + 1).  The metadata must satisfy the reference's checks
 * (context_plan.py:309-325 and the range check at :367-371); the host
 * validates it before the call, the device does not re-check it.
 *
 * Outputs, per request at the same offsets as the inputs:
 *   per token: positions, keep_mask, materialized_stage, birth_positions,
 *     birth_stages (int32 / uint8), token_to_key (int64, request-local key);
 *   per key, at key offset token_offsets[b] + (ranges before b) +
 *     reposition_offsets[b], capacity T + R + P per request: records
 *     [.,3] int32, virtual_mask uint8, key_to_token int64;
 *   per Reposition: effective_reposition_stages (int32, -1 if ignored),
 *     effective_repositions, ignored_repositions (uint8);
 *   transition_offsets: P_b + 1 int32 entries at reposition_offsets[b] + b,
 *     stage-indexed and relative to the request's first transition (entries
 *     past the request's stage count hold its total);
 *   per Drop event: drop_event_to_key (int64);
 *   transitions (raw token, old, new position; int32) of request b at
 *     [transition_request_offsets[b], transition_request_offsets[b+1]), at
 *     most transition_capacity in total (more sets AKV_LAYOUT_CAPACITY and
 *     the excess is not written);
 *   status [n][5] int64, the reference's status vector per request:
 *     {0, key_len, stages, next_position, -1} or {1 (no active token at a
 *     Reposition), ., ., ., boundary} or {2 (token id outside [0, 2^31)), .,
 *     ., ., token id};
 *   decode view (optional, all three NULL to skip): active_offsets [n+1],
 *     raw_indices, active_positions;
 *   totals [4] int64: {transitions, kept tokens, keys, AKV_LAYOUT_* bits}.
 *
 * tile_offsets[n+1]: prefix over requests of ceil(T_b / 512); count_offsets
 * [n+1] int64: prefix over requests of tiles_b * (P_b + 1).  The workspace
 * (akv_compile_layouts_workspace_bytes with the batch's n_requests,
 * n_tokens, n_repositions, n_count_cells) needs no initial contents.  At
 * most akv_compile_layouts_max_repositions() Reposition events per request.
 * Work: linear in tokens and ranges (times log P for a binary search), plus
 * one 512-token block scan per pair of tile and effective Reposition whose
 * transitions reach into the tile.
 */
#define AKV_LAYOUT_CAPACITY 1  /* transitions exceed transition_capacity      */
#define AKV_LAYOUT_ERROR 2     /* some request's status[0] is non-zero         */
#define AKV_LAYOUT_TOO_MANY 4  /* a request has more Repositions than allowed;
                                  its outputs are not written (status[0] = -1) */

typedef struct akv_layout_batch {
  int32_t n_requests;
  int32_t n_tiles;
  int64_t n_tokens;       /* token_offsets[n_requests] */
  int64_t n_repositions;  /* reposition_offsets[n_requests] */
  int64_t n_count_cells;  /* count_offsets[n_requests] */
  const int64_t* token_offsets;
  const void* token_ids;
  int32_t token_ids_is64;
  const int32_t* tile_offsets;
  const int64_t* count_offsets;
  const int32_t* drop_event_offsets;
  const int32_t* drop_insert_offsets;
  const int32_t* drop_range_offsets;
  const int32_t* drop_ranges;
  const int32_t* reposition_offsets;
  const int32_t* reposition_raw_boundaries;
  int32_t* positions;
  uint8_t* keep_mask;
  int32_t* materialized_stage;
  int32_t* birth_positions;
  int32_t* birth_stages;
  int64_t* token_to_key;
  int32_t* records;
  uint8_t* virtual_mask;
  int64_t* key_to_token;
  int32_t* transition_offsets;
  int32_t* transition_request_offsets;
  int32_t* transition_raw_tokens;
  int32_t* transition_old_positions;
  int32_t* transition_new_positions;
  int64_t transition_capacity;
  int32_t* effective_reposition_stages;
  uint8_t* effective_repositions;
  uint8_t* ignored_repositions;
  int64_t* drop_event_to_key;
  int64_t* status;
  int32_t* active_offsets;
  int32_t* raw_indices;
  int32_t* active_positions;
  int64_t* totals;
  void* workspace;
} akv_layout_batch;

int64_t akv_compile_layouts_max_repositions(void);
int64_t akv_compile_layouts_batch_bytes(void); /* sizeof(akv_layout_batch), for FFI checks */
int64_t akv_compile_layouts_workspace_bytes(int32_t n_requests, int64_t n_tokens,
                                            int64_t n_repositions, int64_t n_count_cells);
int akv_compile_layouts(const akv_layout_batch* batch, void* stream);

/*
 * Decode read indices.  Replaces the Triton kernel context_decode_indices
 * (akv/system/sglang/kernels/ops/attention/context_page_table.py:34-76),
 * same contract: registry rows of six int64 cells {raw_ids*, positions*,
 * prompt_len, active, next_pos, row*}
 * (srt/layers/attention/context_backend.py:716-725); for request b and
 * i < lengths[b], logical = starts[b] + i; raw = raw_ids[logical] if the
 * row has context and logical < active, else prompt + logical - active (or
 * logical without context); slot = row[raw] (row* or req_to_token row);
 * slot = mapping[slot] * multiplier if mapping != NULL; stored at
 * output[indptr[b] + i].  The *_is64 flags give each index vector's width.
 */
int akv_context_decode_indices(
    const int64_t* registry, const int32_t* req_to_token, int64_t row_stride,
    const void* row_ids, int32_t row_ids_is64, const void* lengths, int32_t lengths_is64,
    const void* indptr, int32_t indptr_is64, void* output, int32_t output_is64,
    const void* starts, int32_t starts_is64, const void* mapping, int32_t mapping_is64,
    int64_t multiplier, int32_t batch, void* stream);

/*
 * Sliding-window visible lengths.  Replaces the Triton kernel
 * context_window_lengths
 * (akv/system/sglang/kernels/ops/attention/context_page_table.py:7-31):
 * rows without context get min(length, window); context rows count the
 * active keys with position >= q_pos - window (binary search over the
 * row's positions) plus the visible generated tokens.
 */
int akv_context_window_lengths(
    const int64_t* registry, const void* row_ids, int32_t row_ids_is64, const void* lengths,
    int32_t lengths_is64, void* output, int32_t output_is64, int64_t window, int32_t batch,
    void* stream);

/*
 * Ragged decode metadata in one call: optional window lengths (window >= 0),
 * kv_indptr (exclusive scan of the lengths), starts = seq_lens - lengths and
 * the decode indices.  Replaces ContextDecodeRegistry.fill_window / fill
 * (srt/layers/attention/context_backend.py:754-809), whose torch cumsum and
 * subtraction run as separate kernels.  kv_indptr: int32 [batch+1];
 * lengths_out, starts_out: int64 [batch] (may be NULL); kv_indices: int32.
 */
int akv_build_decode_metadata(
    const int64_t* registry, const int32_t* req_to_token, int64_t row_stride,
    const int64_t* row_ids, const int64_t* seq_lens, int64_t window, const int64_t* mapping,
    int64_t multiplier, int32_t batch, int32_t* kv_indptr, int64_t* lengths_out,
    int64_t* starts_out, int32_t* kv_indices, void* stream);

/*
 * Paged GQA decode attention with learned sinks over a compacted index
 * list.  Replaces the native decode kernels the reference runs over the
 * registry's kv_indptr / kv_indices (FlashInfer decode wrapper / FA3
 * flash_attn_with_kvcache, upstream, not vendored; AKV glue at
 * akv/system/sglang.patch:2170-2183) and AKV's sink correction
 * o *= sigmoid(lse - sink) (srt/layers/attention/context_backend.py:254-272),
 * computed here as out = sum e^s v / (sum e^s + e^sink).
 *
 * q: bf16 [batch, num_q_heads, head_dim] (strides in elements); K / V pools:
 * bf16 [slots, num_kv_heads, head_dim] with the given strides (16-byte
 * aligned rows); kv_indices: int32 slots.  num_q_heads = 8 * num_kv_heads,
 * num_kv_heads in {1, 2, 4, 8}, head_dim in {64, 128}.  sinks: fp32
 * [num_q_heads] natural-log logits or NULL.  sm_scale multiplies q.k.
 * work: DEVICE int32 [n_items, 4] rows {request, kv_begin, kv_end, partial}
 * (kv_begin/kv_end index kv_indices; partial = -1 writes the request's
 * output directly, else the item's slot in partial_acc [P, q_heads, D] and
 * partial_ml [P, q_heads, 2]); merge: DEVICE int32 [batch, 2] rows
 * {first partial, count} (count 0 = written directly) or NULL when no item
 * is split.  cta_items: DEVICE int32 [n_ctas + 1] or NULL: with it, n_ctas
 * persistent CTAs run, CTA c processing work rows [cta_items[c],
 * cta_items[c+1]) in order (the host balances the lists); NULL launches one
 * CTA per work row.  out: bf16 [batch, q_heads, head_dim]; lse: fp32 [batch, q_heads]
 * natural-log LSE including the sink, or NULL.  A slot outside [0, num_slots)
 * is read as slot 0 and sets *error_flag (DEVICE int32, may be NULL).
 * The host side (akv_b200/context_attention.py) builds work/merge from
 * host-known lengths, as FlashInfer's plan() does.
 */
int akv_decode_attention(
    const void* q, int64_t q_stride_batch, int64_t q_stride_head, const void* k_pool,
    const void* v_pool, int64_t k_stride_slot, int64_t k_stride_head, int64_t v_stride_slot,
    int64_t v_stride_head, int64_t num_slots, const int32_t* kv_indices, const float* sinks,
    float sm_scale, int32_t batch, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
    const int32_t* work, int32_t n_items, const int32_t* cta_items, int32_t n_ctas,
    const int32_t* merge, float* partial_acc, float* partial_ml, void* out,
    int64_t out_stride_batch, int64_t out_stride_head, float* lse, int32_t* error_flag,
    void* stream);

/*
 * Ragged prefill (extend) attention with context positions and sinks.
 * Replaces the native ragged prefill launch of ContextAttentionMetadata.forward
 * and its host-side native_plan gathers
 * (srt/layers/attention/context_backend.py:184-241; the position-aware
 * extend kernel of akv/system/sglang.patch:106-237) and the sink correction
 * of flash_attention_with_sink (context_backend.py:244-272).
 *
 * Request b: Q_b = qo_indptr[b+1] - qo_indptr[b] new tokens (rows of q and
 * out, DEVICE int32 birth_slots and q_positions at the same rows; their K/V
 * already written to the pools) after P_b = kv_indptr[b+1] - kv_indptr[b]
 * prefix keys (kv_indices, kv_positions).  Query i sees prefix key j when
 * window < 0 or q_pos - k_pos <= window, and new-token key j when j <= i and
 * the same window test holds (positions increase along each request's key
 * list).  q / out: bf16 [tokens, q_heads, head_dim] (strides in elements);
 * pools bf16 [slots, kv_heads, head_dim]; num_q_heads = 8 * num_kv_heads,
 * head_dim 64 or 128; sinks fp32 [q_heads] or NULL; lse fp32 [tokens,
 * q_heads] (natural log, including the sink) or NULL.
 * work: DEVICE int32 [n_items, 4] rows {request, first query (request-local,
 * a multiple of akv_context_attention_query_block()), key_lo, key_hi}: the
 * block's queries read keys [key_lo, key_hi) of the request's key list
 * (key_hi = P_b + last query + 1; key_lo = first key the window can reach);
 * built on the host from the CPU positions (akv_b200/context_prefill.py).
 * error_flag: DEVICE int32[2] or NULL.  Word 0 collects error bits and is
 * never cleared by the library: bit 1 = a slot outside [0, num_slots) was
 * read as slot 0; bit 2 = a tcgen05 wait did not complete (the CTA freed its
 * tensor memory and returned; the output of that launch is not valid).
 * Word 1 is the launch's abort word: this call clears it on the stream
 * before launching, a CTA whose wait ran out sets it, and CTAs that start
 * after that skip their work.
 * work may hold padding items {-1, 0, 0, 0}; items 2i and 2i + 1 are two
 * consecutive blocks of one request or a block and a padding item (the plan
 * of akv_b200/context_prefill.py lays them out so), which variant 4 needs.
 * variant: 0 = the faster kernel for the shape, 1 = the mma.sync kernel,
 * 2 = the tcgen05 / TMEM kernel (head_dim 64), 3 = its warp-specialised
 * form (head_dim 64 and 128), 4 = the warp-specialised form with the two
 * items of a pair in one CTA (n_items even); 5 and 6 = the forms of 3 and 4
 * with P rounded to bf16 for P.V (one MMA per key block instead of the hi +
 * lo pair of the others: FlashInfer's precision, |error| <= 2^-8 sum p|v|
 * more); 2-6 need 16-byte aligned q and out rows and sm_scale > 0
 * (AKV_ERR_UNSUPPORTED otherwise).
 */
int64_t akv_context_attention_query_block(void);
int akv_context_attention(
    const void* q, int64_t q_stride_token, int64_t q_stride_head, const void* k_pool,
    const void* v_pool, int64_t k_stride_slot, int64_t k_stride_head, int64_t v_stride_slot,
    int64_t v_stride_head, int64_t num_slots, const int32_t* qo_indptr, const int32_t* kv_indptr,
    const int32_t* kv_indices, const int32_t* birth_slots, const int32_t* q_positions,
    const int32_t* kv_positions, const float* sinks, float sm_scale, int64_t window,
    int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, const int32_t* work,
    int32_t n_items, void* out, int64_t out_stride_token, int64_t out_stride_head, float* lse,
    int32_t* error_flag, int32_t variant, void* stream);

/* Resident CTAs per SM of akv_decode_attention for this shape (the size of
 * a persistent launch is this times the SM count); a negative AKV_* status
 * on error.  Needs a CUDA device.  No reference counterpart. */
int32_t akv_decode_attention_ctas_per_sm(int32_t num_kv_heads, int32_t head_dim);

/*
 * Overflow-row slot scatter.  Replaces the Triton kernel write_row_slots
 * (akv/system/sglang/kernels/ops/memory/context_rows.py:7-15):
 * ((int32*)pointers[rows[i]])[columns[i]] = values[i] for i < n.
 */
int akv_write_row_slots(const int64_t* pointers, const void* rows, int32_t rows_is64,
                        const void* columns, int32_t columns_is64, const void* values,
                        int32_t values_is64, int64_t n, void* stream);

/*
 * Active slots of one request row, for offload / load and PD transfer.
 * Replaces the gather of request_active_slots
 * (akv/system/sglang/srt/disaggregation/context_transfer.py:110-128):
 * out = concat(row[device_indices[start:n_indices]],
 *              row[generated_start:raw_end]),
 * n_indices - start + max(0, raw_end - generated_start) int32 slots, in one
 * launch.  row: DEVICE int32 [row_len] (a req_to_token row); device_indices:
 * DEVICE int32 raw indices of the surviving prompt tokens.  The caller
 * computes start and generated_start on the host from the decode view (the
 * window's first visible position), as the reference does.  An index outside
 * the row reads as slot -1 and sets *error_flag (NULL: not reported).
 */
int akv_active_slots(const int32_t* row, int64_t row_len, const int32_t* device_indices,
                     int64_t start, int64_t n_indices, int64_t generated_start, int64_t raw_end,
                     int32_t* out, int32_t* error_flag, void* stream);

/*
 * akv_active_slots for a batch of requests in one launch (an offload or a
 * transfer of many requests; no reference counterpart -- the reference
 * gathers request by request).  meta: DEVICE int64 [n_requests][6] =
 * {row address, row length, raw-index address, start, n_prefix =
 * n_indices - start, generated_start}; out_offsets: DEVICE int64
 * [n_requests + 1], request r's slots at out[out_offsets[r] ..], each of
 * length n_prefix + max(0, raw_end - generated_start); chunks: DEVICE int32
 * [n_chunks][2] = {request, first output of the request}, every request cut
 * into pieces of akv_active_slots_chunk() outputs (one block each).
 */
int64_t akv_active_slots_chunk(void);
int akv_active_slots_batch(const int64_t* meta, const int64_t* out_offsets, const int32_t* chunks,
                           int32_t n_chunks, int32_t* out, int32_t* error_flag, void* stream);

/*
 * Occurrence slot gathers: the device binding of request-local page
 * ownership between prefill forwards, for every request of a forward in one
 * launch.  Replaces the per-request torch concatenation, gathers and casts of
 * OccurrenceMaterialization.bind
 * (akv/system/sglang/srt/context_system/occurrence.py:315-357),
 * OccurrenceState.advance (:644-755) and OccurrenceState.terminal_slots
 * (:757-768), and the scheduler's concatenation of their results
 * (akv/system/sglang.patch:3133-3180).  The scheduler CPU keeps every
 * ownership decision; only the slot binding runs here.
 *
 * tasks: DEVICE int64 [n_tasks][12], one output vector each:
 *   [0] first index of the task in `indices`   [1] n outputs
 *   [2] output address                         [3] flags (AKV_GATHER_*)
 *       | n_segments << 8 (0..4)
 *   [4..7] segment addresses                   [8..11] cumulative segment
 *                                                      lengths
 * For i < n: v = indices[first + i] (int32: a row below 2^31, or a literal
 * of that range); with AKV_GATHER_LITERAL, out[i] = v;
 * else out[i] = -1 if v < 0, else element v of the concatenation of the
 * segments (an index at or past its end writes -1 and sets *error_flag).
 * Segments are int64 with AKV_GATHER_SEG64, else int32; out is int64 with
 * AKV_GATHER_OUT64, else int32 (the low 32 bits, as a torch int32 cast).
 * chunks: DEVICE int32 [n_chunks][2] = {task, first output of the task},
 * every task cut into pieces of akv_gather_slots_chunk() outputs (one block
 * each).  indices: DEVICE int32.  No reference counterpart as one call.
 */
/*
 * Host half of OccurrenceState.advance
 * (akv/system/sglang/srt/context_system/occurrence.py:644-755): every
 * ownership index of one prefill forward of one request, computed on the
 * CPU (no device memory is touched).  All pointers are HOST memory.
 *
 * Rows index all = state slots ++ query slots ++ extra slots (fewer than
 * 2^31 rows, else AKV_ERR_INVALID).  Outputs (int32 row vectors, ready to be
 * akv_gather_slots indices): occurrence_rows[count] (-1 = unbound), copy_source_rows /
 * copy_destination_rows [n_copy], retained / retired (ascending rows; room
 * for n_old + n_query + n_extra each) with their counts, unused_swa (room
 * for n_copy), the successor's canonical / terminal rows and positions
 * [end], owned flags of the retained rows and, with swa_resident, the
 * residency of retained and retired rows (next_swa / retired_swa may be
 * NULL without it).  Returns AKV_OK, AKV_ERR_OCC_MISSING_SOURCE (a reused
 * occurrence's version has no owner: "Context ownership plan references a
 * missing source"), AKV_ERR_OCC_MISSING_COPY_SOURCE ("Context copy
 * references a missing canonical source") or AKV_ERR_INVALID (indices out
 * of range).  The passes are described in akv_b200/csrc/occurrence_plan.cu.
 */
typedef struct {
  int64_t n;          /* tokens of the occurrence window */
  int64_t start, end; /* the state covers [0, start); this forward's queries [start, end) */
  int64_t count;      /* occurrences of the window */
  int64_t n_old, n_query, n_extra, n_copy;
  const uint8_t* owned;               /* [n_old] */
  const int64_t* canonical_rows;      /* [start] */
  const int64_t* terminal_rows;       /* [start] */
  const int32_t* canonical_positions; /* [start] */
  const uint8_t* swa_resident;        /* [n_old] or NULL */
  const int64_t* birth_occurrences;   /* [n] */
  const int64_t* terminal_occurrences; /* [n] */
  const int32_t* occurrence_positions; /* [count] */
  const int64_t* source_rows;         /* [count] */
  const int64_t* allocated;           /* [n_extra] */
  const int64_t* copy_occurrences;    /* [n_copy] */
  const int64_t* copy_source_rows;    /* [n_copy] */
  const int64_t* plan_terminal;       /* [end] */
  const int32_t* visible_until;       /* [n] */
} akv_advance_in;

typedef struct {
  int32_t* occurrence_rows; /* rows are below 2^31: n_old + n_query + n_extra must be */
  int32_t* copy_source_rows;
  int32_t* copy_destination_rows;
  int32_t* retained;
  int32_t* retired;
  int32_t* unused_swa;
  int64_t* next_canonical;
  int64_t* next_terminal;
  int32_t* next_positions;
  uint8_t* next_owned;
  uint8_t* next_swa;
  uint8_t* retired_swa;
  int64_t n_retained, n_retired, n_unused_swa;
} akv_advance_out;

int akv_occurrence_advance_indices(const akv_advance_in* in, akv_advance_out* out);

#define AKV_GATHER_OUT64 1
#define AKV_GATHER_LITERAL 2
#define AKV_GATHER_SEG64 4
int64_t akv_gather_slots_chunk(void);
int akv_gather_slots(const int64_t* tasks, const int32_t* chunks, int32_t n_chunks,
                     const int32_t* indices, int32_t* error_flag, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* AKV_B200_H_ */
