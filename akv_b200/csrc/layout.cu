// General event compiler (Drop / Reposition programs) for a batch of
// requests, on the device.
//
// Replaces compile_radix_reposition_layout and
// count_radix_reposition_transitions
// (akv/system/sglang/kernels/ops/attention/context_plan.py:80-532), which
// sweep the insertion offsets 0..T of one request with a doubly linked list
// of active tokens.  This file computes the same outputs from a closed form.
// For one request with Reposition insertion offsets I_r = boundary_r + 1
// (r = 0..P-1, increasing):
//
//   drop(t)   = smallest insertion offset of a Drop event whose ranges cover
//               t, or infinity; keep(t) = drop(t) is infinite.
//   A_r       = { t < I_r : drop(t) > I_r }, the active tokens Reposition r
//               sees (a Drop at the same offset runs first).
//   rank_r(t) = |A_r ∩ [0, t)|.
//
// After Reposition r, effective or ignored, every token of A_r sits at
// rank_r(t).  With NP_r the next position right after Reposition r
// (NP_{-1} = 0, I_{-1} = 0), a token born in [I_{r-1}, I_r) gets
// NP_{r-1} + (t - I_{r-1}).  Reposition r moves exactly the tokens of A_r at
// or after
//   F_r = min(D_r, I_{r-1} if NP_{r-1} > |A_{r-1}|),
//   D_r = the smallest token with drop(t) in (I_{r-1}, I_r],
// which is the reference's first non-compact token: the successor of the
// first token dropped since the previous Reposition (context_plan.py:383-394)
// or the first token born after an ignored Reposition left a gap in the
// positions (:460-463).  It is effective iff n_r = |A_r| - rank_r(F_r) > 0,
// and then NP_r = |A_r|; otherwise NP_r = NP_{r-1} + (I_r - I_{r-1}).  Only
// this recurrence over the P Repositions is sequential.
//
// Launches (no inter-block waiting):
//   1. classify -- per 512-token tile: drop(t) by painting the request's
//      ranges in shared memory; per token the interval [r0, r1] of
//      Repositions whose A_r contain it, as a difference array over the
//      P + 1 columns (column P counts kept tokens); per-window minima D_r.
//   2. stages   -- per request: column-wise exclusive scans over the tiles
//      (rank_r at every tile start), rank_r(D_r) and rank_r(I_{r-1}) from one
//      partial tile each, the recurrence, status and the virtual radix
//      records (Drop ranges, effective Repositions).
//   3. offsets  -- one block: per-request transition and decode-view bases.
//   4. emit     -- per tile: for every effective Reposition whose moved
//      tokens reach the tile, one block scan of (A_r, A_{r-1}) membership
//      gives each transition's index, old and new position; then the final
//      per-token outputs, token records and the decode view.

#include <climits>

#include "common.cuh"

namespace akv {
namespace {

constexpr int kTile = 512;
constexpr int kThreads = 256;
constexpr int kPer = kTile / kThreads;  // tokens per thread: threadIdx.x + k * kThreads
constexpr int kMaxRepositions = 4094;
constexpr int kListCap = 256;  // ranges overlapping one tile, painted cooperatively
// Requests with at most this many Repositions and Drop events keep their
// per-Reposition tables in shared memory while a block works on them (one
// parallel load instead of a dependent global load per step); longer
// programs read the same tables from global memory.
constexpr int kColCap = 256;
constexpr int kOffsetThreads = 1024;

// Record kinds of the radix key stream (srt/context_system/ir.py:32-34).
constexpr int kToken = 0, kDelta = 1, kReposition = 2;

__host__ __device__ inline size_t align_up(size_t x) { return (x + 255) & ~size_t(255); }

// Device scratch.  `dinv` and `bad_inv` accumulate minima as atomicMax of
// INT_MAX - value and start at zero (one memset per call).
struct LayoutWs {
  int* dinv;        // [columns] INT_MAX - D_r (0: no token dropped in the window)
  int* bad_inv;     // [n] INT_MAX - first token with an out-of-range id
  int* dt;          // [n_tokens] drop(t), INT_MAX if kept
  int* counts;      // [count cells] per request [P+1][tiles]: tile counts, then exclusive prefixes
  int* nA;          // [columns] |A_r|; column P: kept tokens
  int* rankD;       // [columns] rank_r(D_r)
  int* rankI;       // [columns] rank_r(I_{r-1})
  int* F;           // [columns] F_r (INT_MAX if ignored)
  int* rankF;       // [columns] rank_r(F_r)
  int* tbase;       // [columns] first transition of Reposition r within its request
  int* stage_of;    // [columns] stage number of an effective Reposition, else 0
  int* np_before;   // [columns] NP_{r-1}
  int* seg_np;      // [columns] NP_{s-1}: next position at the start of segment s
  int* seg_stage;   // [columns] effective Repositions before segment s
  int* trans_count; // [n]
  int* key_len;     // [n]
  uintptr_t end;    // one past the last array
};

__host__ __device__ inline LayoutWs carve(void* base, int n, long long n_tokens, long long columns,
                                         long long cells) {
  uintptr_t p = reinterpret_cast<uintptr_t>(base);
  auto take = [&](size_t count) {
    int* r = reinterpret_cast<int*>(p);
    p += align_up(sizeof(int) * (count > 0 ? count : 1));
    return r;
  };
  LayoutWs w;
  w.dinv = take(columns);
  w.bad_inv = take(n);
  w.dt = take(n_tokens);
  w.counts = take(cells);
  w.nA = take(columns);
  w.rankD = take(columns);
  w.rankI = take(columns);
  w.F = take(columns);
  w.rankF = take(columns);
  w.tbase = take(columns);
  w.stage_of = take(columns);
  w.np_before = take(columns);
  w.seg_np = take(columns);
  w.seg_stage = take(columns);
  w.trans_count = take(n);
  w.key_len = take(n);
  w.end = p;
  return w;
}

inline size_t workspace_bytes(int n, long long n_tokens, long long n_repositions,
                              long long cells) {
  return carve(nullptr, n, n_tokens, n_repositions + n, cells).end;  // offsets from 0
}

struct LayoutArgs {
  akv_layout_batch b;
  LayoutWs ws;
};

// One request's slice of the batch.
struct Req {
  long long tok0;   // first flat token
  int T;            // tokens
  int ev0, E;       // Drop events [ev0, ev0 + E)
  int rg0;          // drop_range_offsets[ev0] (global range index)
  int rg1;
  int rep0, P;      // Repositions [rep0, rep0 + P)
  int col0;         // first column (rep0 + request index)
  int tile0, ntiles;
  long long cbase;  // first count cell
  long long key0;   // first key
};

__device__ Req request_meta(const LayoutArgs& a, int b) {
  const akv_layout_batch& x = a.b;
  Req q;
  q.tok0 = x.token_offsets[b];
  q.T = (int)(x.token_offsets[b + 1] - q.tok0);
  q.ev0 = x.drop_event_offsets[b];
  q.E = x.drop_event_offsets[b + 1] - q.ev0;
  q.rg0 = x.drop_range_offsets[q.ev0];
  q.rg1 = x.drop_range_offsets[q.ev0 + q.E];
  q.rep0 = x.reposition_offsets[b];
  q.P = x.reposition_offsets[b + 1] - q.rep0;
  q.col0 = q.rep0 + b;
  q.tile0 = x.tile_offsets[b];
  q.ntiles = x.tile_offsets[b + 1] - q.tile0;
  q.cbase = x.count_offsets[b];
  q.key0 = q.tok0 + q.rg0 + q.rep0;  // drop_range_offsets starts at 0
  return q;
}

// Number of entries of the increasing array a[0, n) below x; a may be in
// shared or global memory.
__device__ __forceinline__ int count_below_any(const int32_t* a, int n, long long x) {
  int lo = 0, hi = n;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if ((long long)a[mid] < x) lo = mid + 1;
    else hi = mid;
  }
  return lo;
}

__device__ int tile_request(const int32_t* tile_offsets, int n, int tile) {
  int lo = 0, hi = n;  // first b with tile_offsets[b] > tile, minus one
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (__ldg(tile_offsets + mid) <= tile) lo = mid + 1;
    else hi = mid;
  }
  return lo - 1;
}

// ---------------------------------------------------------------------------
// 1. classify
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) layout_classify_kernel(const LayoutArgs a) {
  __shared__ int s_dt[kTile];
  __shared__ int s_hist[kMaxRepositions + 2];  // difference array over columns 0..P
  __shared__ int s_dmin[kMaxRepositions];
  __shared__ int3 s_list[kListCap];
  __shared__ int s_nlist, s_bad;
  __shared__ int32_t s_bnd[kColCap];
  pdl_launch_dependents();  // the stages blocks may be scheduled; they wait for this grid
  const int tile = blockIdx.x;
  const int b = tile_request(a.b.tile_offsets, a.b.n_requests, tile);
  const Req q = request_meta(a, b);
  if (q.P > kMaxRepositions) return;  // reported by the stages kernel
  const int tl = tile - q.tile0;
  const int t0 = tl * kTile, n = min(kTile, q.T - t0);
  const bool staged = q.P <= kColCap;
  const int32_t* bnd = a.b.reposition_raw_boundaries + q.rep0;
  if (staged) {
    for (int r = threadIdx.x; r < q.P; r += blockDim.x) s_bnd[r] = bnd[r];
    bnd = s_bnd;
  }
  for (int i = threadIdx.x; i < kTile; i += blockDim.x) s_dt[i] = INT_MAX;
  for (int c = threadIdx.x; c <= q.P + 1; c += blockDim.x) s_hist[c] = 0;
  for (int c = threadIdx.x; c < q.P; c += blockDim.x) s_dmin[c] = INT_MAX;
  if (threadIdx.x == 0) {
    s_nlist = 0;
    s_bad = INT_MAX;
  }
  __syncthreads();

  // Ranges overlapping the tile, with their event's insertion offset.
  const int32_t* dro = a.b.drop_range_offsets;
  for (int k = q.rg0 + threadIdx.x; k < q.rg1; k += blockDim.x) {
    const int s = a.b.drop_ranges[2 * (long long)k], e = a.b.drop_ranges[2 * (long long)k + 1];
    const int cs = max(s, t0), ce = min(e, t0 + n);
    if (cs >= ce) continue;
    int lo = q.ev0, hi = q.ev0 + q.E;  // owner: last event whose first range is <= k
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (__ldg(dro + mid) <= k) lo = mid + 1;
      else hi = mid;
    }
    const int ins = a.b.drop_insert_offsets[lo - 1];
    const int slot = atomicAdd(&s_nlist, 1);
    if (slot < kListCap) {
      s_list[slot] = make_int3(cs - t0, ce - t0, ins);
    } else {
      for (int i = cs - t0; i < ce - t0; ++i) atomicMin(&s_dt[i], ins);
    }
  }
  __syncthreads();
  const int nl = min(s_nlist, kListCap);
  for (int j = 0; j < nl; ++j) {
    const int3 r = s_list[j];
    for (int i = r.x + threadIdx.x; i < r.y; i += blockDim.x) atomicMin(&s_dt[i], r.z);
  }
  __syncthreads();

  // Neighbouring tokens mostly share their interval [r0, r1]: the shared
  // histogram and minima are updated once per distinct value in a warp.
  const unsigned full = 0xffffffffu;
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int i = threadIdx.x + k * kThreads;
    const bool valid = i < n;
    const int t = t0 + i;
    int r0 = -1, r1 = -2, w = -1;
    if (valid) {
      const int dt = s_dt[i];
      a.ws.dt[q.tok0 + t] = dt;
      r0 = count_below_any(bnd, q.P, t);  // Repositions with I_r <= t
      if (dt == INT_MAX) {
        r1 = q.P;  // kept: active to the end, counted in the final column
      } else {
        r1 = count_below_any(bnd, q.P, (long long)dt - 1) - 1;  // last r with I_r < drop(t)
        w = r1 + 1;  // window (I_{w-1}, I_w] holding drop(t)
        if (w >= q.P) w = -1;
      }
      const long long id = ld_index(a.b.token_ids, q.tok0 + t, a.b.token_ids_is64);
      if (id < 0 || id > INT_MAX) atomicMin(&s_bad, t);
    }
    const bool span = r1 >= r0;
    const int lo_key = span ? r0 : -1, hi_key = span ? r1 + 1 : -1;
    const unsigned g_lo = __match_any_sync(full, lo_key);
    if (lo_key >= 0 && lane == __ffs(g_lo) - 1) atomicAdd(&s_hist[lo_key], __popc(g_lo));
    const unsigned g_hi = __match_any_sync(full, hi_key);
    if (hi_key >= 0 && lane == __ffs(g_hi) - 1) atomicAdd(&s_hist[hi_key], -__popc(g_hi));
    const unsigned g_w = __match_any_sync(full, w);
    if (w >= 0) {
      const int m = (int)__reduce_min_sync(g_w, (unsigned)t);
      if (lane == __ffs(g_w) - 1) atomicMin(&s_dmin[w], m);
    }
  }
  __syncthreads();

  int carry = 0;
  for (int c0 = 0; c0 <= q.P; c0 += blockDim.x) {
    const int c = c0 + threadIdx.x;
    const int v = c <= q.P ? s_hist[c] : 0;
    int tot;
    const int ex = block_exclusive_scan<int>(v, &tot);
    if (c <= q.P) a.ws.counts[q.cbase + (long long)c * q.ntiles + tl] = carry + ex + v;
    carry += tot;
  }
  for (int c = threadIdx.x; c < q.P; c += blockDim.x)
    if (s_dmin[c] != INT_MAX) atomicMax(&a.ws.dinv[q.col0 + c], INT_MAX - s_dmin[c]);
  if (threadIdx.x == 0 && s_bad != INT_MAX) atomicMax(&a.ws.bad_inv[b], INT_MAX - s_bad);
}

// ---------------------------------------------------------------------------
// 2. stages
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) layout_stages_kernel(const LayoutArgs a) {
  __shared__ int s_bnd[kColCap], s_nA[kColCap], s_dinv[kColCap], s_rankD[kColCap],
      s_rankI[kColCap];
  pdl_wait();
  pdl_launch_dependents();
  const int b = blockIdx.x;
  const Req q = request_meta(a, b);
  int64_t* status = a.b.status + 5 * (long long)b;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  if (q.P > kMaxRepositions) {
    if (threadIdx.x == 0) {
      status[0] = -1;
      status[1] = status[2] = status[3] = 0;
      status[4] = q.P;
      a.ws.trans_count[b] = 0;
      a.ws.key_len[b] = 0;
      a.ws.nA[q.col0 + q.P] = 0;
    }
    return;
  }
  int* counts = a.ws.counts + q.cbase;
  const bool staged = q.P <= kColCap;
  if (staged) {
    for (int r = threadIdx.x; r < q.P; r += blockDim.x) {
      s_bnd[r] = a.b.reposition_raw_boundaries[q.rep0 + r];
      s_dinv[r] = a.ws.dinv[q.col0 + r];
    }
  }

  // Column-wise exclusive scans over the request's tiles.
  for (int c = warp; c <= q.P; c += nwarps) {
    int carry = 0;
    for (int j0 = 0; j0 < q.ntiles; j0 += 32) {
      const int j = j0 + lane;
      const long long cell = (long long)c * q.ntiles + j;
      const int v = j < q.ntiles ? counts[cell] : 0;
      const int inc = warp_inclusive_scan<int>(v);
      if (j < q.ntiles) counts[cell] = carry + inc - v;
      carry += __shfl_sync(0xffffffffu, inc, 31);
    }
    if (lane == 0) {
      a.ws.nA[q.col0 + c] = carry;
      if (staged && c < q.P) s_nA[c] = carry;
    }
  }
  __syncthreads();

  // rank_r(D_r) and rank_r(I_{r-1}): the tile-start prefix plus a count over
  // the part of one tile before the token.
  const int32_t* bnd = a.b.reposition_raw_boundaries + q.rep0;
  for (int job = warp; job < 2 * q.P; job += nwarps) {
    const int r = job >> 1, which = job & 1;
    long long x = -1;
    if (which == 0) {
      const int dinv = a.ws.dinv[q.col0 + r];
      if (dinv != 0) x = INT_MAX - dinv;
    } else if (r > 0) {
      x = (long long)bnd[r - 1] + 1;
    }
    int rank = -1;
    if (x >= 0) {
      const long long I = (long long)bnd[r] + 1;
      const int tl = (int)(x / kTile);
      int cnt = 0;
      for (long long t = (long long)tl * kTile + lane; t < x; t += 32)
        cnt += (long long)a.ws.dt[q.tok0 + t] > I;
      cnt = warp_sum<int>(cnt);
      rank = counts[(long long)r * q.ntiles + tl] + cnt;
    }
    if (lane == 0) {
      (which == 0 ? a.ws.rankD : a.ws.rankI)[q.col0 + r] = rank;
      if (staged) (which == 0 ? s_rankD : s_rankI)[r] = rank;
    }
  }
  __syncthreads();

  // The recurrence over the Repositions (context_plan.py:405-440).
  int32_t* toff = a.b.transition_offsets + q.col0;
  if (threadIdx.x == 0) {
    // Inputs of the recurrence: shared-memory copies when staged.
    const int* c_bnd = staged ? s_bnd : bnd;
    const int* c_nA = staged ? s_nA : a.ws.nA + q.col0;
    const int* c_dinv = staged ? s_dinv : a.ws.dinv + q.col0;
    const int* c_rankD = staged ? s_rankD : a.ws.rankD + q.col0;
    const int* c_rankI = staged ? s_rankI : a.ws.rankI + q.col0;
    long long np_prev = 0, i_prev = 0, na_prev = 0, arg = -1;
    int stage = 0, cum = 0, code = 0;
    a.ws.seg_np[q.col0] = 0;
    a.ws.seg_stage[q.col0] = 0;
    toff[0] = 0;
    for (int r = 0; r < q.P; ++r) {
      const long long I = (long long)c_bnd[r] + 1;
      const int na = c_nA[r];
      const int col = q.col0 + r;
      int st = 0;
      long long np = np_prev + (I - i_prev);
      if (code == 0 && na == 0) {
        code = 1;  // "Reposition at raw boundary ... has no active tokens."
        arg = c_bnd[r];
      }
      int F = INT_MAX, rank_f = 0;
      if (code == 0) {
        const int dinv = c_dinv[r];
        if (dinv != 0) {
          F = INT_MAX - dinv;
          rank_f = c_rankD[r];
        }
        if (r > 0 && np_prev > na_prev && i_prev < F) {
          F = (int)i_prev;
          rank_f = c_rankI[r];
        }
        const int moved = F != INT_MAX ? na - rank_f : 0;
        a.ws.tbase[col] = cum;
        a.ws.np_before[col] = (int)np_prev;
        if (moved > 0) {
          st = ++stage;
          cum += moved;
          toff[stage] = cum;
          np = na;
        } else {
          F = INT_MAX;
        }
      }
      a.ws.F[col] = F;
      a.ws.rankF[col] = rank_f;
      a.ws.stage_of[col] = st;
      a.b.effective_repositions[q.rep0 + r] = st > 0;
      a.b.ignored_repositions[q.rep0 + r] = code == 0 && st == 0;
      a.b.effective_reposition_stages[q.rep0 + r] = st > 0 ? st : -1;
      np_prev = np;
      i_prev = I;
      na_prev = na;
      a.ws.seg_np[col + 1] = (int)np;
      a.ws.seg_stage[col + 1] = stage;
    }
    for (int s = stage + 1; s <= q.P; ++s) toff[s] = cum;
    const int bad = a.ws.bad_inv[b];
    if (code == 0 && bad != 0) {
      code = 2;  // "Reposition Radix token ID ... is outside the non-negative int32 range."
      arg = ld_index(a.b.token_ids, q.tok0 + (INT_MAX - bad), a.b.token_ids_is64);
    }
    const long long key_len = (long long)q.T + (q.rg1 - q.rg0) + stage;
    status[0] = code;
    status[1] = code == 0 ? key_len : 0;
    status[2] = code == 0 ? stage : 0;
    status[3] = code == 0 ? np_prev + (q.T - i_prev) : 0;
    status[4] = code == 0 ? -1 : arg;
    a.ws.trans_count[b] = cum;
    a.ws.key_len[b] = code == 0 ? (int)key_len : 0;
  }
  __syncthreads();

  // Virtual records of the radix key stream (context_plan.py:467-498).
  const int32_t* ins = a.b.drop_insert_offsets + q.ev0;
  const int32_t* dro = a.b.drop_range_offsets + q.ev0;
  for (int r = threadIdx.x; r < q.P; r += blockDim.x) {
    const int st = a.ws.stage_of[q.col0 + r];
    if (st == 0) continue;
    const long long I = (long long)bnd[r] + 1;
    const int ev = count_below(ins, q.E, I + 1);  // Drop events at or before I_r
    const long long key = I + (dro[ev] - dro[0]) + (st - 1);
    int32_t* rec = a.b.records + 3 * (q.key0 + key);
    rec[0] = kReposition;
    rec[1] = bnd[r];
    rec[2] = -1;
    a.b.virtual_mask[q.key0 + key] = 1;
    a.b.key_to_token[q.key0 + key] = -1;
  }
  for (int e = threadIdx.x; e < q.E; e += blockDim.x) {
    const long long I = ins[e];
    const int before = count_below(bnd, q.P, I - 1);  // Repositions with I_r < I
    const long long key = I + (dro[e] - dro[0]) + a.ws.seg_stage[q.col0 + before];
    a.b.drop_event_to_key[q.ev0 + e] = key;
    for (int k = dro[e]; k < dro[e + 1]; ++k) {
      const long long kk = q.key0 + key + (k - dro[e]);
      int32_t* rec = a.b.records + 3 * kk;
      rec[0] = kDelta;
      rec[1] = (int32_t)(-(long long)a.b.drop_ranges[2 * (long long)k] - 1);
      rec[2] = (int32_t)(-(long long)a.b.drop_ranges[2 * (long long)k + 1] - 1);
      a.b.virtual_mask[kk] = 1;
      a.b.key_to_token[kk] = -1;
    }
  }
}

// ---------------------------------------------------------------------------
// 3. offsets
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kOffsetThreads) layout_offsets_kernel(const LayoutArgs a) {
  __shared__ long long s_carry[3];
  __shared__ int s_err;
  pdl_wait();
  pdl_launch_dependents();
  if (threadIdx.x == 0) {
    s_carry[0] = s_carry[1] = s_carry[2] = 0;
    s_err = 0;
  }
  __syncthreads();
  const int n = a.b.n_requests;
  for (int b0 = 0; b0 < n; b0 += blockDim.x) {
    const int b = b0 + threadIdx.x;
    long long tr = 0, kept = 0, keys = 0;
    if (b < n) {
      const int col = a.b.reposition_offsets[b + 1] + b;  // the request's final column
      tr = a.ws.trans_count[b];
      kept = a.ws.nA[col];
      keys = a.ws.key_len[b];
      const long long code = a.b.status[5 * (long long)b];
      if (code > 0) atomicOr(&s_err, AKV_LAYOUT_ERROR);
      if (code < 0) atomicOr(&s_err, AKV_LAYOUT_TOO_MANY);
    }
    long long tot_tr, tot_kept, tot_keys;
    const long long ex_tr = block_exclusive_scan<long long>(tr, &tot_tr);
    const long long ex_kept = block_exclusive_scan<long long>(kept, &tot_kept);
    block_exclusive_scan<long long>(keys, &tot_keys);
    if (b < n) {
      a.b.transition_request_offsets[b] = (int32_t)(s_carry[0] + ex_tr);
      if (a.b.active_offsets) a.b.active_offsets[b] = (int32_t)(s_carry[1] + ex_kept);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      s_carry[0] += tot_tr;
      s_carry[1] += tot_kept;
      s_carry[2] += tot_keys;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    a.b.transition_request_offsets[n] = (int32_t)s_carry[0];
    if (a.b.active_offsets) a.b.active_offsets[n] = (int32_t)s_carry[1];
    int err = s_err;
    if (s_carry[0] > a.b.transition_capacity) err |= AKV_LAYOUT_CAPACITY;
    a.b.totals[0] = s_carry[0];
    a.b.totals[1] = s_carry[1];
    a.b.totals[2] = s_carry[2];
    a.b.totals[3] = err;
  }
}

// ---------------------------------------------------------------------------
// 4. emit
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads, 4) layout_emit_kernel(const LayoutArgs a) {
  // Per-Reposition tables of the request (and its Drop events), staged.
  __shared__ int32_t s_bnd[kColCap], s_stage[kColCap], s_F[kColCap], s_rankF[kColCap],
      s_npb[kColCap], s_tbase[kColCap], s_next[kColCap];
  __shared__ int32_t s_cnt[kColCap + 1], s_segnp[kColCap + 1], s_segst[kColCap + 1];
  __shared__ int32_t s_ins[kColCap], s_dro[kColCap + 1];
  pdl_wait();
  const int tile = blockIdx.x;
  const int b = tile_request(a.b.tile_offsets, a.b.n_requests, tile);
  const Req q = request_meta(a, b);
  if (q.P > kMaxRepositions) return;
  const int tl = tile - q.tile0;
  const int t0 = tl * kTile, n = min(kTile, q.T - t0);
  const int* counts = a.ws.counts + q.cbase;

  // Table views: shared-memory copies (one parallel load) for requests with
  // at most kColCap Repositions and Drop events, global memory otherwise.
  //   cnt[r]  = rank_r at this tile's start (r = 0..P; P: kept tokens);
  //   next[r] = rank_r at the next tile's start, or |A_r| for the last tile.
  const bool staged = q.P <= kColCap && q.E <= kColCap;
  const int32_t* bnd = a.b.reposition_raw_boundaries + q.rep0;
  const int32_t* ins = a.b.drop_insert_offsets + q.ev0;
  const int32_t* dro = a.b.drop_range_offsets + q.ev0;
  const int* stage_of = a.ws.stage_of + q.col0;
  const int* Fv = a.ws.F + q.col0;
  const int* rankFv = a.ws.rankF + q.col0;
  const int* npbv = a.ws.np_before + q.col0;
  const int* tbasev = a.ws.tbase + q.col0;
  const int* segnp = a.ws.seg_np + q.col0;
  const int* segst = a.ws.seg_stage + q.col0;
  auto cnt_at = [&](int r) -> int {
    return staged ? s_cnt[r] : counts[(long long)r * q.ntiles + tl];
  };
  auto cnt_next = [&](int r) -> int {
    if (staged) return s_next[r];
    return tl + 1 < q.ntiles ? counts[(long long)r * q.ntiles + tl + 1] : a.ws.nA[q.col0 + r];
  };
  if (staged) {
    for (int r = threadIdx.x; r <= q.P; r += blockDim.x) {
      s_cnt[r] = counts[(long long)r * q.ntiles + tl];
      s_segnp[r] = segnp[r];
      s_segst[r] = segst[r];
      if (r < q.P) {
        s_bnd[r] = bnd[r];
        s_stage[r] = stage_of[r];
        s_F[r] = Fv[r];
        s_rankF[r] = rankFv[r];
        s_npb[r] = npbv[r];
        s_tbase[r] = tbasev[r];
        s_next[r] = tl + 1 < q.ntiles ? counts[(long long)r * q.ntiles + tl + 1]
                                      : a.ws.nA[q.col0 + r];
      }
    }
    for (int e = threadIdx.x; e <= q.E; e += blockDim.x) {
      if (e < q.E) s_ins[e] = ins[e];
      s_dro[e] = dro[e];
    }
    __syncthreads();
    bnd = s_bnd;
    ins = s_ins;
    dro = s_dro;
    stage_of = s_stage;
    Fv = s_F;
    rankFv = s_rankF;
    npbv = s_npb;
    tbasev = s_tbase;
    segnp = s_segnp;
    segst = s_segst;
  }

  // Thread x holds tokens x and x + kThreads of the tile, so each store
  // instruction of a warp covers 32 consecutive tokens.
  int dt[kPer], seg[kPer], pos[kPer], ms[kPer];
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int i = threadIdx.x + k * kThreads, t = t0 + i;
    dt[k] = INT_MAX;
    seg[k] = 0;
    pos[k] = 0;
    ms[k] = 0;
    if (i >= n) continue;
    dt[k] = a.ws.dt[q.tok0 + t];
    seg[k] = count_below_any(bnd, q.P, t);
    const long long i_seg = seg[k] ? (long long)bnd[seg[k] - 1] + 1 : 0;
    pos[k] = (int)(segnp[seg[k]] + (t - i_seg));
    ms[k] = segst[seg[k]];
    a.b.birth_positions[q.tok0 + t] = pos[k];
    a.b.birth_stages[q.tok0 + t] = ms[k];
  }

  // Transitions of every effective Reposition whose moved tokens reach here.
  const int tr_base = a.b.transition_request_offsets[b];
  const long long cap = a.b.transition_capacity;
  for (int r = count_below_any(bnd, q.P, t0); r < q.P; ++r) {
    const int st = stage_of[r];
    if (st == 0) continue;
    const int F = Fv[r];
    if (F >= t0 + n) continue;
    const int Rr = cnt_at(r);
    if (cnt_next(r) == Rr) continue;  // no token of A_r in this tile
    const long long I = (long long)bnd[r] + 1;
    const long long Ip = r > 0 ? (long long)bnd[r - 1] + 1 : 0;
    // Ranks in A_r and A_{r-1} in token order: one scan of four 16-bit
    // counters (A_r, A_{r-1}) x (first, second token of each thread).
    bool in_r[kPer], in_p[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int i = threadIdx.x + k * kThreads;
      const long long t = t0 + i;
      in_r[k] = i < n && t < I && dt[k] > I;
      in_p[k] = i < n && t < Ip && dt[k] > Ip;
    }
    static_assert(kPer == 2, "four 16-bit scan fields");
    const unsigned long long local = (unsigned long long)in_r[0] |
                                     ((unsigned long long)in_p[0] << 16) |
                                     ((unsigned long long)in_r[1] << 32) |
                                     ((unsigned long long)in_p[1] << 48);
    unsigned long long tot;
    const unsigned long long ex = block_exclusive_scan<unsigned long long>(local, &tot);
    const int er[kPer] = {(int)(ex & 0xffffu), (int)(tot & 0xffffu) + (int)((ex >> 32) & 0xffffu)};
    const int ep[kPer] = {(int)((ex >> 16) & 0xffffu),
                          (int)((tot >> 16) & 0xffffu) + (int)((ex >> 48) & 0xffffu)};
    const int Rp = r > 0 ? cnt_at(r - 1) : 0;
    const int rank_f = rankFv[r], npb = npbv[r];
    const long long base = (long long)tr_base + tbasev[r] - rank_f;
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int t = t0 + threadIdx.x + k * kThreads;
      if (in_r[k] && t >= F) {
        const int rank = Rr + er[k];
        const long long idx = base + rank;
        const int old = t < Ip ? Rp + ep[k] : (int)(npb + (t - Ip));
        if (idx >= 0 && idx < cap) {  // the capacity may be short (flagged)
          a.b.transition_raw_tokens[idx] = t;
          a.b.transition_old_positions[idx] = old;
          a.b.transition_new_positions[idx] = rank;
        }
        pos[k] = rank;
        ms[k] = st;
      }
    }
  }

  // Final per-token outputs and token records (context_plan.py:499-514).
  // A record is three int32 at 12-byte stride: with an 8-byte aligned array
  // it is one 8-byte and one 4-byte store (which comes first depends on the
  // key's parity).
  const bool rec8 = (reinterpret_cast<uintptr_t>(a.b.records) & 7) == 0;
  int kept[kPer];
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int i = threadIdx.x + k * kThreads, t = t0 + i;
    kept[k] = 0;
    if (i >= n) continue;
    const long long f = q.tok0 + t;
    const bool keep = dt[k] == INT_MAX;
    kept[k] = keep;
    a.b.positions[f] = pos[k];
    a.b.keep_mask[f] = keep;
    a.b.materialized_stage[f] = ms[k];
    const int ev = count_below_any(ins, q.E, (long long)t + 1);  // Drop events at or before t
    const long long key = t + (dro[ev] - dro[0]) + segst[seg[k]];
    a.b.token_to_key[f] = key;
    const long long gk = q.key0 + key;
    int32_t* rec = a.b.records + 3 * gk;
    const int32_t id = (int32_t)ld_index(a.b.token_ids, f, a.b.token_ids_is64);
    if (rec8 && (gk & 1) == 0) {
      *reinterpret_cast<int2*>(rec) = make_int2(kToken, id);
      rec[2] = pos[k];
    } else if (rec8) {
      rec[0] = kToken;
      *reinterpret_cast<int2*>(rec + 1) = make_int2(id, pos[k]);
    } else {
      rec[0] = kToken;
      rec[1] = id;
      rec[2] = pos[k];
    }
    a.b.virtual_mask[gk] = 0;
    a.b.key_to_token[gk] = t;
  }

  // Decode view: raw = flatnonzero(keep), positions[raw] (occurrence.py:47-66).
  if (a.b.active_offsets != nullptr) {
    unsigned tot;
    const unsigned ex = block_exclusive_scan<unsigned>((unsigned)kept[0] | ((unsigned)kept[1] << 16),
                                                       &tot);
    const long long kbase = (long long)a.b.active_offsets[b] + cnt_at(q.P);
    const int rank[kPer] = {(int)(ex & 0xffffu), (int)(tot & 0xffffu) + (int)(ex >> 16)};
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      if (!kept[k]) continue;
      a.b.raw_indices[kbase + rank[k]] = t0 + threadIdx.x + k * kThreads;
      a.b.active_positions[kbase + rank[k]] = pos[k];
    }
  }
}

}  // namespace
}  // namespace akv

extern "C" int64_t akv_compile_layouts_max_repositions(void) { return akv::kMaxRepositions; }

extern "C" int64_t akv_compile_layouts_workspace_bytes(int32_t n_requests, int64_t n_tokens,
                                                       int64_t n_repositions,
                                                       int64_t n_count_cells) {
  if (n_requests < 0 || n_tokens < 0 || n_repositions < 0 || n_count_cells < 0) return -1;
  return (int64_t)akv::workspace_bytes(n_requests, n_tokens, n_repositions, n_count_cells);
}

extern "C" int akv_compile_layouts(const akv_layout_batch* batch, void* stream) {
  AKV_NVTX_RANGE("akv_compile_layouts");
  using namespace akv;
  if (batch == nullptr) return AKV_ERR_INVALID;
  const akv_layout_batch& x = *batch;
  if (x.n_requests < 0 || x.n_tiles < 0 || x.n_tokens < 0 || x.n_repositions < 0 ||
      x.n_count_cells < 0 || x.transition_capacity < 0 || x.n_tokens > INT_MAX)
    return AKV_ERR_INVALID;
  const bool view = x.active_offsets != nullptr;
  if (view != (x.raw_indices != nullptr) || view != (x.active_positions != nullptr))
    return AKV_ERR_INVALID;
  if (!x.token_offsets || !x.tile_offsets || !x.count_offsets || !x.drop_event_offsets ||
      !x.drop_range_offsets || !x.reposition_offsets || !x.status || !x.totals ||
      !x.transition_offsets || !x.transition_request_offsets || !x.workspace)
    return AKV_ERR_INVALID;
  if (x.n_tokens > 0 && (!x.token_ids || !x.positions || !x.keep_mask || !x.materialized_stage ||
                         !x.birth_positions || !x.birth_stages || !x.token_to_key ||
                         !x.records || !x.virtual_mask || !x.key_to_token))
    return AKV_ERR_INVALID;
  if (x.n_repositions > 0 &&
      (!x.reposition_raw_boundaries || !x.effective_reposition_stages ||
       !x.effective_repositions || !x.ignored_repositions))
    return AKV_ERR_INVALID;
  if (x.transition_capacity > 0 &&
      (!x.transition_raw_tokens || !x.transition_old_positions || !x.transition_new_positions))
    return AKV_ERR_INVALID;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const long long columns = x.n_repositions + x.n_requests;
  LayoutArgs a;
  a.b = x;
  a.ws = carve(x.workspace, x.n_requests, x.n_tokens, columns, x.n_count_cells);
  const size_t zeroed = reinterpret_cast<uintptr_t>(a.ws.dt) - reinterpret_cast<uintptr_t>(a.ws.dinv);
  if (cudaMemsetAsync(a.ws.dinv, 0, zeroed, s) != cudaSuccess)
    return AKV_ERR_CUDA;
  // classify follows the memset as an ordinary launch; stages, offsets and
  // emit are programmatic dependent launches (each waits for its
  // predecessor before reading anything).
  if (x.n_tiles > 0) layout_classify_kernel<<<x.n_tiles, kThreads, 0, s>>>(a);
  if (x.n_requests > 0 &&
      launch_pdl(layout_stages_kernel, x.n_requests, kThreads, 0, s, a) != cudaSuccess)
    return AKV_ERR_CUDA;
  if (launch_pdl(layout_offsets_kernel, 1, kOffsetThreads, 0, s, a) != cudaSuccess)
    return AKV_ERR_CUDA;
  if (x.n_tiles > 0 &&
      launch_pdl(layout_emit_kernel, x.n_tiles, kThreads, 0, s, a) != cudaSuccess)
    return AKV_ERR_CUDA;
  return launch_status();
}

extern "C" int64_t akv_compile_layouts_batch_bytes(void) { return sizeof(akv_layout_batch); }
