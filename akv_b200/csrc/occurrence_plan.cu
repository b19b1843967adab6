// Host half of occurrence ownership: which slot rows a prefill forward binds,
// copies, keeps and retires (the slot gather of occurrence.cu binds them on
// the device).
//
// The reference derives these indices on the scheduler CPU with numpy
// (OccurrenceState.advance, akv/system/sglang/srt/context_system/
// occurrence.py:644-755).  Here they are the passes below over plain arrays,
// written from the contract the scheduler relies on (which occurrence reads
// which version of which token, which versions a later query can still
// read), so that a request's ownership costs one native call.
//
// Rows.  all = state.slots ++ query slots ++ extra slots; a row is an index
// into `all`: [0, n_old) the state's, [n_old, n_old + n_query) the query
// slots (token start + i), then the extra slots in the order of
// plan.allocated_occurrences.  A plan row r in [0, 2n) names a version of a
// token: r < n the canonical (birth-stage) version of token r, r >= n the
// terminal (final-position) version of token r - n.  Its owner row:
//   canonical(t) = state.canonical_rows[t] if t < start,
//                  n_old + t - start       if start <= t < end,  else none;
//   terminal(t)  = state.terminal_rows[t]  if t < start,          else none.
//
//   1. occurrences: an occurrence with a plan row >= 0 binds that version's
//      owner (none is an error); plan.allocated_occurrences take the extra
//      slots in order; any other occurrence stays unbound (row 0 in the
//      output, as the reference reports it).
//   2. copies: source = owner of copy_source_rows[j] (none is an error),
//      destination = the row of occurrence copy_occurrences[j].
//   3. SWA residency (only with per-row residency): the state's rows keep
//      theirs, new rows start resident; every copy destination takes the
//      residency its source had before any copy of this pass; destinations
//      that end non-resident are listed as unused SWA slots.
//   4. tokens t < end: terminal row = row of plan.terminal_occurrences[t]
//      (if any); position = state.canonical_positions[t] for t < start, else
//      the position of t's birth occurrence; the next canonical row is the
//      terminal row when the terminal occurrence sits at that position (a
//      same-position copy is bit-identical), else canonical(t); it is
//      dropped when no later query of this prefill reads t
//      (visible_until[t] <= end, or end == n).
//   5. liveness: the next canonical and terminal rows are marked live;
//      retained = live rows ascending (a row's rank is its row in the
//      successor), retired = owned rows that are not live, ascending.

#include <string.h>

#include <vector>

#include "akv_b200.h"

namespace {

struct Owner {
  const akv_advance_in* in;
  int64_t n;
  int64_t operator()(int64_t r) const {
    if (r < 0 || r >= 2 * n) return -2;  // outside the plan's rows
    if (r < n) {
      if (r < in->start) return in->canonical_rows[r];
      if (r < in->end) return in->n_old + (r - in->start);
      return -1;
    }
    const int64_t t = r - n;
    return t < in->start ? in->terminal_rows[t] : -1;
  }
};

}  // namespace

extern "C" int akv_occurrence_advance_indices(const akv_advance_in* in, akv_advance_out* out) {
  if (!in || !out) return AKV_ERR_INVALID;
  const int64_t n = in->n, start = in->start, end = in->end, count = in->count;
  const int64_t n_old = in->n_old, n_query = in->n_query, n_extra = in->n_extra;
  const int64_t total = n_old + n_query + n_extra;
  if (n < 0 || start < 0 || start > end || end > n || count < 0 || n_old < 0 ||
      n_query != end - start || n_extra < 0 || in->n_copy < 0 || total > INT32_MAX)
    return AKV_ERR_INVALID;
  const Owner owner{in, n};
  const int64_t row_limit = total;

  // 1. occurrences
  for (int64_t o = 0; o < count; ++o) {
    const int64_t r = in->source_rows[o];
    int64_t row = -1;
    if (r >= 0) {
      row = owner(r);
      if (row < 0 || row >= row_limit) return AKV_ERR_OCC_MISSING_SOURCE;
    }
    out->occurrence_rows[o] = (int32_t)row;
  }
  for (int64_t i = 0; i < n_extra; ++i) {
    const int64_t o = in->allocated[i];
    if (o < 0 || o >= count) return AKV_ERR_INVALID;
    out->occurrence_rows[o] = (int32_t)(n_old + n_query + i);
  }
  // 2. copies
  for (int64_t j = 0; j < in->n_copy; ++j) {
    const int64_t src = owner(in->copy_source_rows[j]);
    if (src < 0 || src >= row_limit) return AKV_ERR_OCC_MISSING_COPY_SOURCE;
    const int64_t o = in->copy_occurrences[j];
    if (o < 0 || o >= count) return AKV_ERR_INVALID;
    out->copy_source_rows[j] = (int32_t)src;
    out->copy_destination_rows[j] = out->occurrence_rows[o];
  }
  // 3. SWA residency
  std::vector<uint8_t> swa;
  out->n_unused_swa = 0;
  if (in->swa_resident) {
    swa.assign(total, 1);
    memcpy(swa.data(), in->swa_resident, (size_t)n_old);
    std::vector<uint8_t> before(in->n_copy);
    for (int64_t j = 0; j < in->n_copy; ++j) before[j] = swa[out->copy_source_rows[j]];
    for (int64_t j = 0; j < in->n_copy; ++j) {
      const int64_t d = out->copy_destination_rows[j];
      if (d < 0) return AKV_ERR_INVALID;
      swa[d] = before[j];
    }
    for (int64_t j = 0; j < in->n_copy; ++j) {
      const int64_t d = out->copy_destination_rows[j];
      if (!swa[d]) out->unused_swa[out->n_unused_swa++] = (int32_t)d;
    }
  }
  // 4. tokens of the successor
  std::vector<int64_t> next_canonical(end), next_terminal(end);
  for (int64_t t = 0; t < end; ++t) {
    const int64_t picked = in->plan_terminal[t];
    if (picked >= count) return AKV_ERR_INVALID;
    const int64_t term = picked >= 0 ? out->occurrence_rows[picked] : -1;
    int32_t pos;
    if (t < start) {
      pos = in->canonical_positions[t];
    } else {
      const int64_t b = in->birth_occurrences[t];
      if (b < 0 || b >= count) return AKV_ERR_INVALID;
      pos = in->occurrence_positions[b];
    }
    out->next_positions[t] = pos;
    const int64_t to = in->terminal_occurrences[t];
    if (to < 0 || to >= count) return AKV_ERR_INVALID;
    const bool same = pos == in->occurrence_positions[to];
    int64_t canon = (picked >= 0 && same) ? term : owner(t);
    if (canon >= total) return AKV_ERR_INVALID;  // a state row past its slots
    const bool read_later = end < n && in->visible_until[t] > end;
    if (!read_later) canon = -1;
    next_canonical[t] = canon;
    next_terminal[t] = picked >= 0 ? term : -1;
  }
  // 5. liveness
  std::vector<int64_t> rank(total, -1);
  for (int64_t t = 0; t < end; ++t) {
    if (next_canonical[t] >= 0) rank[next_canonical[t]] = 0;
    if (next_terminal[t] >= 0) rank[next_terminal[t]] = 0;
  }
  int64_t kept = 0, retired = 0;
  for (int64_t row = 0; row < total; ++row) {
    const bool owned = row < n_old ? in->owned[row] != 0 : true;
    if (rank[row] == 0) {
      rank[row] = kept;
      out->retained[kept] = (int32_t)row;
      out->next_owned[kept] = owned;
      if (out->next_swa && in->swa_resident) out->next_swa[kept] = swa[row];
      ++kept;
    } else if (owned) {
      out->retired[retired] = (int32_t)row;
      if (out->retired_swa && in->swa_resident) out->retired_swa[retired] = swa[row];
      ++retired;
    }
  }
  for (int64_t t = 0; t < end; ++t) {
    out->next_canonical[t] = next_canonical[t] >= 0 ? rank[next_canonical[t]] : -1;
    out->next_terminal[t] = next_terminal[t] >= 0 ? rank[next_terminal[t]] : -1;
  }
  out->n_retained = kept;
  out->n_retired = retired;
  return AKV_OK;
}
