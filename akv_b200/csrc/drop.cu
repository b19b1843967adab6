// Drop + Reposition of a batch of requests, computed on the device.
//
// For a program with one Drop event and one Reposition at the end of the
// prompt, the reference's CPU event compiler
// (akv/system/sglang/kernels/ops/attention/context_plan.py:210-532) walks a
// linked list token by token.  Its result has a closed form that maps onto
// one exclusive scan per request:
//   keep(t)     = t is covered by no drop range
//   rank(t)     = number of kept tokens before t (the scan)
//   position(t) = rank(t) if kept (after the Reposition), else t
//   moved(t)    = kept and rank(t) != t, i.e. t lies after the first drop
// (tokens are born at positions 0..T-1; the first non-compact token of the
// reference is the first kept token after the first dropped one, and from
// there on every kept token moves -- context_plan.py:405-440).
//
// Three launches, no inter-block waiting:
//   1. count   -- per 512-token tile: keep mask from a difference array of
//                 the request's drop ranges (shared-memory atomics + block
//                 scan), four per-tile counters {kept, moved, cow, freed};
//   2. plan    -- one block: exclusive scan of the tile counters, per-request
//                 offsets, next_position, free-ring reservation;
//   3. scatter -- per tile: block scan again, write positions, the compacted
//                 decode view, transitions (with copy-on-write destinations
//                 popped from the free ring) and freed slots (pushed on it).
// Tiles never straddle requests (the host gives per-request tile offsets),
// so a request's base is the scan value at its first tile.

#include <mutex>

#include "common.cuh"

namespace akv {
namespace {

constexpr int kTile = 512;
constexpr int kThreads = 128;
constexpr int kPerThread = kTile / kThreads;  // 4 contiguous tokens per thread
constexpr int kPlanThreads = 256;
constexpr int kFields = 4;  // kept, moved, cow, freed

// Field packing for the block scan: 16 bits per counter (a tile holds at
// most 512 tokens, so no field overflows into the next).
__device__ __forceinline__ unsigned long long pack4(int a, int b, int c, int d) {
  return (unsigned long long)a | ((unsigned long long)b << 16) | ((unsigned long long)c << 32) |
         ((unsigned long long)d << 48);
}
__device__ __forceinline__ int field(unsigned long long v, int f) {
  return (int)((v >> (16 * f)) & 0xffffull);
}

struct Workspace {
  int* tile_sums;   // [n_tiles][5]: four counters + bad-input bits (1 range, 2 page layout)
  int* tile_base;   // [n_tiles][4]: exclusive scan of the counters
  int* first_drop;  // [R]: smallest drop start of the request (INT_MAX if none)
  long long* plan;  // {ring head, ring tail, status}
};

__host__ __device__ inline size_t align_up(size_t x) { return (x + 255) & ~size_t(255); }

__host__ __device__ inline Workspace carve(void* base, int n_requests, int n_tiles) {
  char* p = static_cast<char*>(base);
  Workspace w;
  w.tile_sums = reinterpret_cast<int*>(p);
  p += align_up(sizeof(int) * 5 * (size_t)(n_tiles > 0 ? n_tiles : 1));
  w.tile_base = reinterpret_cast<int*>(p);
  p += align_up(sizeof(int) * 4 * (size_t)(n_tiles > 0 ? n_tiles : 1));
  w.first_drop = reinterpret_cast<int*>(p);
  p += align_up(sizeof(int) * (size_t)(n_requests > 0 ? n_requests : 1));
  w.plan = reinterpret_cast<long long*>(p);
  return w;
}

inline size_t workspace_bytes(int n_requests, int n_tiles) {
  const size_t nt = n_tiles > 0 ? n_tiles : 1, nr = n_requests > 0 ? n_requests : 1;
  return align_up(sizeof(int) * 5 * nt) + align_up(sizeof(int) * 4 * nt) +
         align_up(sizeof(int) * nr) + align_up(sizeof(long long) * 4);
}

struct DropArgs {
  int n_requests;
  const int64_t* token_offsets;
  const int32_t* tile_offsets;
  int n_tiles;
  const int32_t* range_offsets;
  const int32_t* ranges;
  const int32_t* shared_prefix;
  int32_t* req_to_token;
  const int64_t* row_ids;
  int64_t row_stride;
  int reposition;
  int page_shift;  // 0: page_size 1; else log2(page_size), page_size in [4, 128]
  int32_t* ring;
  int64_t ring_capacity;
  int64_t* ring_state;
  uint8_t* keep_mask;
  int32_t* positions;
  int32_t* active_offsets;
  int32_t* raw_indices;
  int32_t* active_positions;
  int32_t* next_position;
  int32_t* transition_offsets;
  int32_t* transition_source;
  int32_t* transition_destination;
  int32_t* transition_pairs;
  int32_t* transition_raw;
  int32_t* freed_offsets;
  int32_t* freed_slots;
  int32_t* totals;
  int32_t* status;
  Workspace ws;
};

// Request owning tile `tile`: the r with tile_offsets[r] <= tile < tile_offsets[r+1].
__device__ int tile_request(const int32_t* tile_offsets, int n_requests, int tile) {
  int lo = 0, hi = n_requests;  // search in [0, R]
  while (lo < hi) {             // first r with tile_offsets[r] > tile
    const int mid = (lo + hi) >> 1;
    if (__ldg(tile_offsets + mid) <= tile) lo = mid + 1;
    else hi = mid;
  }
  return lo - 1;
}

struct TileCtx {
  int r, t0, n, T, P;
  long long flat0;
};

__device__ TileCtx tile_context(const DropArgs& a, int tile) {
  TileCtx c;
  c.r = tile_request(a.tile_offsets, a.n_requests, tile);
  const long long begin = a.token_offsets[c.r];
  c.T = (int)(a.token_offsets[c.r + 1] - begin);
  c.t0 = (tile - a.tile_offsets[c.r]) * kTile;
  const int t1 = min(c.T, c.t0 + kTile);
  c.n = t1 - c.t0;
  c.P = a.shared_prefix ? a.shared_prefix[c.r] : 0;
  c.flat0 = begin + c.t0;
  return c;
}

// ---- page mode (page_size = 2^page_shift, 4 <= page_size <= 128) ----
// Slot s of a request's token t lies in page s >> page_shift at offset
// s & (page_size - 1), and the layout keeps offset == t mod page_size, so
// the tokens [g * page_size, (g + 1) * page_size) of a request share one
// page.  A thread's four tokens lie in one page; a page is page_size / 4
// consecutive lanes of a warp (tiles and requests start on page
// boundaries).  The radix-shared prefix P is a whole number of pages.
//   * A private page is freed when every token it holds is dropped (its id
//     goes to freed_slots and the free ring, in token order).
//   * A shared page that holds a moved token is copied to one fresh page
//     popped from the ring: every kept token of the page gets a transition
//     to the same offset of the new page (moved tokens rotated, tokens
//     before the first drop copied bit for bit, old == new position), and
//     the row entries of all its tokens are rewritten, so the layout rule
//     holds for the next call.
//   * Private moved tokens rotate in place, as with page_size 1.
struct PageFlags {
  bool keep[kPerThread], mv[kPerThread];
  bool lead;  // first lane of the page and the page holds a token of the request
  bool cow;   // shared page with a moved token
  bool freed; // private page whose tokens are all dropped
};

__device__ __forceinline__ unsigned page_or(unsigned v, int lanes) {
  for (int o = 1; o < lanes; o <<= 1) v |= __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ unsigned page_and(unsigned v, int lanes) {
  for (int o = 1; o < lanes; o <<= 1) v &= __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Every thread of the block calls this (warp shuffles over whole warps).
__device__ PageFlags page_flags(const DropArgs& a, const TileCtx& c, int first_drop, int base) {
  PageFlags f;
  const int lanes = (1 << a.page_shift) / kPerThread;
  bool any_mv = false, all_drop = true;
#pragma unroll
  for (int k = 0; k < kPerThread; ++k) {
    const int i = base + k;
    const int t = c.t0 + i;
    f.keep[k] = i < c.n && a.keep_mask[c.flat0 + i] != 0;
    f.mv[k] = a.reposition && f.keep[k] && t > first_drop;
    any_mv |= f.mv[k];
    if (i < c.n) all_drop &= !f.keep[k];
  }
  const bool shared = c.t0 + base < c.P;  // pages never straddle P
  f.lead = ((threadIdx.x & (lanes - 1)) == 0) && base < c.n;
  f.cow = shared && page_or(any_mv, lanes) != 0;
  f.freed = !shared && page_and(all_drop, lanes) != 0;
  return f;
}

// True if this thread's tokens break the page layout rule.
__device__ bool page_layout_bad(const DropArgs& a, const TileCtx& c, int base) {
  const int mask = (1 << a.page_shift) - 1;
  const int lanes = (1 << a.page_shift) / kPerThread;
  const int32_t* row = a.req_to_token + a.row_ids[c.r] * a.row_stride;
  int page = -1;
  bool bad = false;
#pragma unroll
  for (int k = 0; k < kPerThread; ++k) {
    const int i = base + k;
    if (i >= c.n) break;
    const int t = c.t0 + i;
    const int slot = row[t];
    bad |= (slot & mask) != (t & mask);
    if (k == 0) page = slot >> a.page_shift;
    bad |= (slot >> a.page_shift) != page;
  }
  const int lead_lane = (threadIdx.x & 31) & ~(lanes - 1);
  const int lead_page = __shfl_sync(0xffffffffu, page, lead_lane);
  return bad || (base < c.n && page != lead_page);
}

__global__ void __launch_bounds__(kThreads) drop_count_kernel(const DropArgs a) {
  __shared__ int diff[kTile + 1];
  __shared__ int s_first, s_bad;
  pdl_launch_dependents();  // the plan block may be scheduled now; it waits for this grid
  const int tile = blockIdx.x;
  const TileCtx c = tile_context(a, tile);
  for (int i = threadIdx.x; i <= kTile; i += blockDim.x) diff[i] = 0;
  if (threadIdx.x == 0) {
    s_first = INT_MAX;
    s_bad = 0;
  }
  __syncthreads();
  const int rb = a.range_offsets[c.r], re = a.range_offsets[c.r + 1];
  int first = INT_MAX, bad = 0;
  for (int i = rb + threadIdx.x; i < re; i += blockDim.x) {
    const int s = a.ranges[2 * i], e = a.ranges[2 * i + 1];
    if (s < 0 || e > c.T || s >= e) {
      bad = 1;
      continue;
    }
    first = min(first, s);
    const int cs = max(s, c.t0), ce = min(e, c.t0 + c.n);
    if (cs < ce) {
      atomicAdd(&diff[cs - c.t0], 1);
      atomicAdd(&diff[ce - c.t0], -1);
    }
  }
  if (first != INT_MAX) atomicMin(&s_first, first);
  if (bad) atomicOr(&s_bad, 1);
  __syncthreads();

  const int base = threadIdx.x * kPerThread;
  int local = 0;
#pragma unroll
  for (int k = 0; k < kPerThread; ++k) local += diff[base + k];
  int unused;
  int cover = block_exclusive_scan<int>(local, &unused);
  const int first_drop = s_first;
  int kept = 0, moved = 0, cow = 0, freed = 0;
#pragma unroll
  for (int k = 0; k < kPerThread; ++k) {
    const int i = base + k;
    cover += diff[i];
    if (i < c.n) {
      const int t = c.t0 + i;
      const bool keep = cover == 0;
      const bool mv = a.reposition && keep && t > first_drop;
      kept += keep;
      moved += mv;
      cow += mv && t < c.P;
      freed += !keep && t >= c.P;
      a.keep_mask[c.flat0 + i] = keep ? 1 : 0;
    }
  }
  if (a.page_shift != 0) {
    // Page mode: the counters of the tile are recomputed per page (the
    // token loop above still wrote the keep mask).
    __shared__ int s_bad_page;
    if (threadIdx.x == 0) s_bad_page = c.P & ((1 << a.page_shift) - 1) ? 1 : 0;
    __syncthreads();
    const PageFlags f = page_flags(a, c, first_drop, base);
    const bool bad = page_layout_bad(a, c, base);
    kept = moved = cow = freed = 0;
#pragma unroll
    for (int k = 0; k < kPerThread; ++k) {
      if (base + k >= c.n) break;
      kept += f.keep[k];
      moved += f.keep[k] && (f.mv[k] || f.cow);
    }
    cow = f.lead && f.cow;
    freed = f.lead && f.freed;
    if (bad) atomicOr(&s_bad_page, 1);
    __syncthreads();
    if (threadIdx.x == 0 && s_bad_page) atomicOr(&s_bad, 2);
    __syncthreads();
  }
  unsigned long long tot;
  block_exclusive_scan<unsigned long long>(pack4(kept, moved, cow, freed), &tot);
  if (threadIdx.x == 0) {
    int* ts = a.ws.tile_sums + 5 * (size_t)tile;
    for (int f = 0; f < kFields; ++f) ts[f] = field(tot, f);
    ts[4] = s_bad;
    if (c.t0 == 0) a.ws.first_drop[c.r] = first_drop;
  }
}

// Pairs of 32-bit counters in one 64-bit word: {kept, moved} and {cow,
// freed}.  Every prefix is a count of tokens or pages of the call, below
// 2^31, so the low field never carries into the high one.
__device__ __forceinline__ unsigned long long pair32(int lo, int hi) {
  return (unsigned long long)(unsigned)lo | ((unsigned long long)(unsigned)hi << 32);
}

__global__ void __launch_bounds__(kPlanThreads) drop_plan_kernel(const DropArgs a) {
  __shared__ int s_bad, s_no_active;
  // The ring state is written by no kernel of this call (last by the plan
  // of the previous call, which completed before this call's count kernel
  // started), so it is read before waiting for the tile counters.
  // So are the staged program's offsets of this thread's first request.
  long long ring_head = 0, ring_tail = 0;
  if (threadIdx.x == 0) {
    ring_head = a.ring_state[0];
    ring_tail = a.ring_state[1];
    s_bad = 0;
    s_no_active = 0;
  }
  int first_tb = 0, first_te = 0, first_T = 0;
  if ((int)threadIdx.x < a.n_requests) {
    first_tb = a.tile_offsets[threadIdx.x];
    first_te = a.tile_offsets[threadIdx.x + 1];
    first_T = (int)(a.token_offsets[threadIdx.x + 1] - a.token_offsets[threadIdx.x]);
  }
  pdl_wait();
  pdl_launch_dependents();
  // Exclusive scan of the per-tile counters: thread i sums a contiguous run
  // of tiles, one block scan gives each run its base, and the run is walked
  // again to write the tiles' bases.
  const int per = (a.n_tiles + (int)blockDim.x - 1) / (int)blockDim.x;
  const int t_begin = min((int)threadIdx.x * per, a.n_tiles);
  const int t_end = min(t_begin + per, a.n_tiles);
  unsigned long long km = 0, cf = 0;
  int bad = 0;
#pragma unroll 4
  for (int t = t_begin; t < t_end; ++t) {
    const int* ts = a.ws.tile_sums + 5 * (size_t)t;
    km += pair32(ts[0], ts[1]);
    cf += pair32(ts[2], ts[3]);
    bad |= ts[4];
  }
  unsigned long long km_total, cf_total;
  unsigned long long km_base = block_exclusive_scan<unsigned long long>(km, &km_total);
  if (bad) atomicOr(&s_bad, bad);  // s_bad was set before the scan's barriers
  unsigned long long cf_base = block_exclusive_scan<unsigned long long>(cf, &cf_total);
  for (int t = t_begin; t < t_end; ++t) {
    *reinterpret_cast<int4*>(a.ws.tile_base + 4 * (size_t)t) =
        make_int4((int)(unsigned)km_base, (int)(km_base >> 32), (int)(unsigned)cf_base,
                  (int)(cf_base >> 32));
    const int* ts = a.ws.tile_sums + 5 * (size_t)t;
    km_base += pair32(ts[0], ts[1]);
    cf_base += pair32(ts[2], ts[3]);
  }
  __syncthreads();  // the bases are read back below by other threads
  const long long carry[kFields] = {(long long)(unsigned)km_total, (long long)(km_total >> 32),
                                    (long long)(unsigned)cf_total, (long long)(cf_total >> 32)};
  const long long total_kept = carry[0], total_moved = carry[1], total_cow = carry[2],
                  total_freed = carry[3];
  auto base_at = [&](int tile, int f) -> int {
    return tile < a.n_tiles ? a.ws.tile_base[4 * (size_t)tile + f] : (int)carry[f];
  };
  for (int r = threadIdx.x; r < a.n_requests; r += blockDim.x) {
    const bool first = r == (int)threadIdx.x;
    const int tb = first ? first_tb : a.tile_offsets[r];
    const int te = first ? first_te : a.tile_offsets[r + 1];
    const int T = first ? first_T : (int)(a.token_offsets[r + 1] - a.token_offsets[r]);
    const int kb = base_at(tb, 0), ke = base_at(te, 0);
    const int mb = base_at(tb, 1), me = base_at(te, 1);
    a.active_offsets[r] = kb;
    a.transition_offsets[r] = mb;
    a.freed_offsets[r] = base_at(tb, 3);
    const int active = ke - kb, moved = me - mb;
    a.next_position[r] = (a.reposition && moved > 0) ? active : T;
    if (a.reposition && T > 0 && active == 0) atomicOr(&s_no_active, 1);
    if (te == tb) a.ws.first_drop[r] = INT_MAX;  // empty request: no tile wrote it
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    a.active_offsets[a.n_requests] = (int)total_kept;
    a.transition_offsets[a.n_requests] = (int)total_moved;
    a.freed_offsets[a.n_requests] = (int)total_freed;
    a.totals[0] = (int)total_kept;
    a.totals[1] = (int)total_moved;
    a.totals[2] = (int)total_cow;
    a.totals[3] = (int)total_freed;
    int st = 0;
    if (s_bad & 1) st |= AKV_DROP_BAD_RANGE;
    if (s_bad & 2) st |= AKV_DROP_BAD_PAGE;
    if (s_no_active) st |= AKV_DROP_NO_ACTIVE;
    const long long head = ring_head, tail = ring_tail;
    if (total_cow > tail - head) st |= AKV_DROP_RING_UNDERFLOW;
    else if (tail - head - total_cow + total_freed > a.ring_capacity) st |= AKV_DROP_RING_OVERFLOW;
    a.ws.plan[0] = head;
    a.ws.plan[1] = tail;
    a.ws.plan[2] = st;
    if (st == 0) {
      a.ring_state[0] = head + total_cow;
      a.ring_state[1] = tail + total_freed;
    } else {
      // All or nothing: no transition, copy-on-write or freed slot is
      // emitted, so a failed call leaves the free ring and rows untouched.
      a.totals[1] = 0;
      a.totals[2] = 0;
      a.totals[3] = 0;
    }
    *a.status = st;
  }
}

// Scatter of one tile in page mode (the rules above drop_count_kernel).
__device__ void scatter_pages(const DropArgs& a, const TileCtx& c, int first_drop, int base,
                              const int (&slots)[kPerThread], int4 tb, int req_kept_base,
                              long long head, long long tail) {
  const int shift = a.page_shift, mask = (1 << shift) - 1;
  const int lanes = (1 << shift) / kPerThread;
  const PageFlags f = page_flags(a, c, first_drop, base);
  int kept = 0, moved = 0;
#pragma unroll
  for (int k = 0; k < kPerThread; ++k) {
    if (base + k >= c.n) break;
    kept += f.keep[k];
    moved += f.keep[k] && (f.mv[k] || f.cow);
  }
  unsigned long long tot;
  const unsigned long long ex = block_exclusive_scan<unsigned long long>(
      pack4(kept, moved, f.lead && f.cow, f.lead && f.freed), &tot);
  int gk = tb.x + field(ex, 0);
  int gm = tb.y + field(ex, 1);
  const int gc = tb.z + field(ex, 2);  // ring index of this page's copy (lead lane)
  const int gf = tb.w + field(ex, 3);
  const int lead_lane = (threadIdx.x & 31) & ~(lanes - 1);
  const int page_gc = __shfl_sync(0xffffffffu, gc, lead_lane);
  int32_t* row = a.req_to_token + a.row_ids[c.r] * a.row_stride;
  const int new_page = f.cow ? a.ring[(head + page_gc) % a.ring_capacity] : 0;
#pragma unroll
  for (int k = 0; k < kPerThread; ++k) {
    const int i = base + k;
    if (i >= c.n) break;
    const int t = c.t0 + i;
    const int fresh = (new_page << shift) | (t & mask);
    if (f.keep[k]) {
      const int rank = gk - req_kept_base;
      const int pos = a.reposition ? rank : t;
      a.positions[c.flat0 + i] = pos;
      a.raw_indices[gk] = t;
      a.active_positions[gk] = pos;
      ++gk;
      if (f.mv[k] || f.cow) {
        a.transition_source[gm] = slots[k];
        a.transition_destination[gm] = f.cow ? fresh : slots[k];
        a.transition_pairs[2 * (size_t)gm] = t;
        a.transition_pairs[2 * (size_t)gm + 1] = pos;
        a.transition_raw[gm] = t;
        ++gm;
      }
    } else {
      a.positions[c.flat0 + i] = t;
    }
    if (f.cow) row[t] = fresh;
  }
  if (f.lead && f.freed) {
    const int page = slots[0] >> shift;
    a.freed_slots[gf] = page;
    a.ring[(tail + gf) % a.ring_capacity] = page;
  }
}

__global__ void __launch_bounds__(kThreads) drop_scatter_kernel(const DropArgs a) {
  // This kernel always follows the plan kernel of the same call, which
  // follows count; count is an ordinary launch, so all earlier work of the
  // stream has completed.  The staged program and the request's row are
  // written by no kernel of this call before this one, so the tile's request
  // and the slots of its tokens are read before waiting for the plan.
  const int tile = blockIdx.x;
  const TileCtx c = tile_context(a, tile);
  const int base = threadIdx.x * kPerThread;
  int32_t* row = a.req_to_token + a.row_ids[c.r] * a.row_stride;
  // All of this thread's slot loads go out before any store: the stores
  // below may alias the row (copy-on-write rewrites it) so the compiler
  // would otherwise serialise load, store, load, ...
  int slots[kPerThread];
#pragma unroll
  for (int k = 0; k < kPerThread; ++k) slots[k] = base + k < c.n ? row[c.t0 + base + k] : 0;
  pdl_wait();
  pdl_launch_dependents();  // lets a following reposition launch be scheduled
  // What count and plan wrote for this tile, loaded together.
  const long long status = a.ws.plan[2], head = a.ws.plan[0], tail = a.ws.plan[1];
  const int first_drop = a.ws.first_drop[c.r];
  const int4 tb = *reinterpret_cast<const int4*>(a.ws.tile_base + 4 * (size_t)tile);
  const int req_kept_base = a.active_offsets[c.r];
  bool keep[kPerThread];
#pragma unroll
  for (int k = 0; k < kPerThread; ++k) keep[k] = base + k < c.n && a.keep_mask[c.flat0 + base + k] != 0;
  if (status != 0) return;
  if (a.page_shift != 0) {
    scatter_pages(a, c, first_drop, base, slots, tb, req_kept_base, head, tail);
    return;
  }
  int kept = 0, moved = 0, cow = 0, freed = 0;
#pragma unroll
  for (int k = 0; k < kPerThread; ++k) {
    const int i = base + k;
    if (i < c.n) {
      const int t = c.t0 + i;
      const bool mv = a.reposition && keep[k] && t > first_drop;
      kept += keep[k];
      moved += mv;
      cow += mv && t < c.P;
      freed += !keep[k] && t >= c.P;
    }
  }
  unsigned long long tot;
  const unsigned long long ex =
      block_exclusive_scan<unsigned long long>(pack4(kept, moved, cow, freed), &tot);
  int gk = tb.x + field(ex, 0);
  int gm = tb.y + field(ex, 1);
  int gc = tb.z + field(ex, 2);
  int gf = tb.w + field(ex, 3);
#pragma unroll
  for (int k = 0; k < kPerThread; ++k) {
    const int i = base + k;
    if (i >= c.n) break;
    const int t = c.t0 + i;
    if (keep[k]) {
      const int rank = gk - req_kept_base;
      const int pos = a.reposition ? rank : t;
      a.positions[c.flat0 + i] = pos;
      a.raw_indices[gk] = t;
      a.active_positions[gk] = pos;
      ++gk;
      if (a.reposition && t > first_drop) {
        const int slot = slots[k];
        int dst = slot;
        if (t < c.P) {
          dst = a.ring[(head + gc) % a.ring_capacity];
          row[t] = dst;
          ++gc;
        }
        a.transition_source[gm] = slot;
        a.transition_destination[gm] = dst;
        a.transition_pairs[2 * (size_t)gm] = t;
        a.transition_pairs[2 * (size_t)gm + 1] = rank;
        a.transition_raw[gm] = t;
        ++gm;
      }
    } else {
      a.positions[c.flat0 + i] = t;
      if (t >= c.P) {
        const int slot = slots[k];
        a.freed_slots[gf] = slot;
        a.ring[(tail + gf) % a.ring_capacity] = slot;
        ++gf;
      }
    }
  }
}

}  // namespace
}  // namespace akv

extern "C" int64_t akv_drop_compact_tile_tokens(void) { return akv::kTile; }

extern "C" int64_t akv_drop_compact_workspace_bytes(int32_t n_requests, int32_t n_tiles) {
  return (int64_t)akv::workspace_bytes(n_requests, n_tiles);
}

namespace akv {
namespace {
int drop_compact(
    int32_t n_requests, const int64_t* token_offsets, const int32_t* tile_offsets,
    int32_t n_tiles, const int32_t* range_offsets, const int32_t* ranges,
    const int32_t* shared_prefix, int32_t* req_to_token, const int64_t* row_ids,
    int64_t row_stride, int32_t reposition, int32_t page_size, int32_t* ring,
    int64_t ring_capacity, int64_t* ring_state, uint8_t* keep_mask, int32_t* positions,
    int32_t* active_offsets, int32_t* raw_indices, int32_t* active_positions,
    int32_t* next_position, int32_t* transition_offsets, int32_t* transition_source,
    int32_t* transition_destination, int32_t* transition_pairs, int32_t* transition_raw,
    int32_t* freed_offsets, int32_t* freed_slots, int32_t* totals, int32_t* status,
    void* workspace, void* stream) {
  int page_shift = 0;
  if (page_size != 1) {
    // Powers of two from 4 to 128: a thread's four tokens lie in one page
    // and a page is at most one warp; tiles (512 tokens) hold whole pages.
    if (page_size < 4 || page_size > 128 || (page_size & (page_size - 1))) return AKV_ERR_INVALID;
    while ((1 << page_shift) < page_size) ++page_shift;
  }
  if (n_requests < 0 || n_tiles < 0 || ring_capacity <= 0 || !token_offsets || !tile_offsets ||
      !range_offsets || !req_to_token || !row_ids || !ring || !ring_state || !keep_mask ||
      !positions || !active_offsets || !raw_indices || !active_positions || !next_position ||
      !transition_offsets || !transition_source || !transition_destination ||
      !transition_pairs || !transition_raw || !freed_offsets || !freed_slots || !totals ||
      !status || !workspace)
    return AKV_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0) return AKV_ERR_INVALID;
  DropArgs a;
  a.n_requests = n_requests;
  a.token_offsets = token_offsets;
  a.tile_offsets = tile_offsets;
  a.n_tiles = n_tiles;
  a.range_offsets = range_offsets;
  a.ranges = ranges;
  a.shared_prefix = shared_prefix;
  a.req_to_token = req_to_token;
  a.row_ids = row_ids;
  a.row_stride = row_stride;
  a.reposition = reposition != 0;
  a.page_shift = page_shift;
  a.ring = ring;
  a.ring_capacity = ring_capacity;
  a.ring_state = ring_state;
  a.keep_mask = keep_mask;
  a.positions = positions;
  a.active_offsets = active_offsets;
  a.raw_indices = raw_indices;
  a.active_positions = active_positions;
  a.next_position = next_position;
  a.transition_offsets = transition_offsets;
  a.transition_source = transition_source;
  a.transition_destination = transition_destination;
  a.transition_pairs = transition_pairs;
  a.transition_raw = transition_raw;
  a.freed_offsets = freed_offsets;
  a.freed_slots = freed_slots;
  a.totals = totals;
  a.status = status;
  a.ws = carve(workspace, n_requests, n_tiles);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // count is an ordinary launch (it overwrites outputs that earlier work in
  // the stream may still read); plan and scatter follow it with
  // programmatic dependent launches.
  if (n_tiles > 0) drop_count_kernel<<<n_tiles, kThreads, 0, s>>>(a);
  if (launch_pdl(drop_plan_kernel, 1, kPlanThreads, 0, s, a) != cudaSuccess) return AKV_ERR_CUDA;
  if (n_tiles > 0 &&
      launch_pdl(drop_scatter_kernel, n_tiles, kThreads, 0, s, a) != cudaSuccess)
    return AKV_ERR_CUDA;
  return launch_status();
}
}  // namespace
}  // namespace akv

extern "C" int akv_drop_compact(
    int32_t n_requests, const int64_t* token_offsets, const int32_t* tile_offsets,
    int32_t n_tiles, const int32_t* range_offsets, const int32_t* ranges,
    const int32_t* shared_prefix, int32_t* req_to_token, const int64_t* row_ids,
    int64_t row_stride, int32_t reposition, int32_t* ring, int64_t ring_capacity,
    int64_t* ring_state, uint8_t* keep_mask, int32_t* positions, int32_t* active_offsets,
    int32_t* raw_indices, int32_t* active_positions, int32_t* next_position,
    int32_t* transition_offsets, int32_t* transition_source, int32_t* transition_destination,
    int32_t* transition_pairs, int32_t* transition_raw, int32_t* freed_offsets,
    int32_t* freed_slots, int32_t* totals, int32_t* status, void* workspace, void* stream) {
  AKV_NVTX_RANGE("akv_drop_compact");
  return akv::drop_compact(n_requests, token_offsets, tile_offsets, n_tiles, range_offsets,
                           ranges, shared_prefix, req_to_token, row_ids, row_stride, reposition,
                           1, ring, ring_capacity, ring_state, keep_mask, positions,
                           active_offsets, raw_indices, active_positions, next_position,
                           transition_offsets, transition_source, transition_destination,
                           transition_pairs, transition_raw, freed_offsets, freed_slots, totals,
                           status, workspace, stream);
}

extern "C" int akv_drop_compact_paged(
    int32_t n_requests, const int64_t* token_offsets, const int32_t* tile_offsets,
    int32_t n_tiles, const int32_t* range_offsets, const int32_t* ranges,
    const int32_t* shared_prefix, int32_t* req_to_token, const int64_t* row_ids,
    int64_t row_stride, int32_t reposition, int32_t page_size, int32_t* ring,
    int64_t ring_capacity, int64_t* ring_state, uint8_t* keep_mask, int32_t* positions,
    int32_t* active_offsets, int32_t* raw_indices, int32_t* active_positions,
    int32_t* next_position, int32_t* transition_offsets, int32_t* transition_source,
    int32_t* transition_destination, int32_t* transition_pairs, int32_t* transition_raw,
    int32_t* freed_offsets, int32_t* freed_slots, int32_t* totals, int32_t* status,
    void* workspace, void* stream) {
  AKV_NVTX_RANGE("akv_drop_compact_paged");
  return akv::drop_compact(n_requests, token_offsets, tile_offsets, n_tiles, range_offsets,
                           ranges, shared_prefix, req_to_token, row_ids, row_stride, reposition,
                           page_size, ring, ring_capacity, ring_state, keep_mask, positions,
                           active_offsets, raw_indices, active_positions, next_position,
                           transition_offsets, transition_source, transition_destination,
                           transition_pairs, transition_raw, freed_offsets, freed_slots, totals,
                           status, workspace, stream);
}

// ---------------------------------------------------------------------------
// Allocation-free variant.
//
// Some callers cannot hand this library a workspace: a serving runtime that
// has reserved every byte of device memory for its KV pool up front, a
// caller running inside a CUDA-graph capture or a custom allocator that
// forbids cudaMalloc on its hot path, or a plain C/FFI caller with no device
// allocator of its own.  For them the drop compaction keeps its scratch
// (per-tile counters, their scan, per-request first-drop positions and the
// ring plan) in one file-scope device array instead.  Every GPU that loads
// this library holds the array until the process exits.
//
// Limits: at most kStaticMaxRequests requests and kStaticMaxTiles tiles
// (kStaticMaxTiles * 512 = 32M tokens) per call; larger calls are refused
// with AKV_ERR_INVALID before anything is launched.  No part of the scratch
// needs to start at zero -- each call writes every entry before reading it --
// so nothing is cleared between calls.  All calls on a device share the one
// array: two calls whose kernels overlap on the GPU (different streams
// without ordering between them) race on it and must be serialised by the
// caller.
namespace akv {
namespace {
constexpr int kStaticMaxRequests = 4096;
constexpr int kStaticMaxTiles = 65536;
constexpr size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
// The workspace layout of carve() at the maximum sizes (about 2.4 MB).
constexpr size_t kStaticScratchBytes =
    align256(sizeof(int) * 5 * kStaticMaxTiles) + align256(sizeof(int) * 4 * kStaticMaxTiles) +
    align256(sizeof(int) * kStaticMaxRequests) + align256(sizeof(long long) * 4);
}  // namespace
}  // namespace akv

static __device__ __align__(256) unsigned char g_drop_scratch[akv::kStaticScratchBytes];

namespace akv {
namespace {
constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of g_drop_scratch on the current device, looked up once
// per device (cudaGetSymbolAddress; the host-side name is only a stand-in).
// The address is that of the primary context current at the first call; a
// cudaDeviceReset destroys it, and the library does not look it up again.
int static_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return AKV_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_drop_scratch) != cudaSuccess || p == nullptr)
      return AKV_ERR_CUDA;
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return AKV_OK;
}
}  // namespace
}  // namespace akv

extern "C" int64_t akv_drop_compact_static_max_requests(void) {
  return akv::kStaticMaxRequests;
}
extern "C" int64_t akv_drop_compact_static_max_tiles(void) { return akv::kStaticMaxTiles; }

extern "C" int akv_drop_compact_static(
    int32_t n_requests, const int64_t* token_offsets, const int32_t* tile_offsets,
    int32_t n_tiles, const int32_t* range_offsets, const int32_t* ranges,
    const int32_t* shared_prefix, int32_t* req_to_token, const int64_t* row_ids,
    int64_t row_stride, int32_t reposition, int32_t* ring, int64_t ring_capacity,
    int64_t* ring_state, uint8_t* keep_mask, int32_t* positions, int32_t* active_offsets,
    int32_t* raw_indices, int32_t* active_positions, int32_t* next_position,
    int32_t* transition_offsets, int32_t* transition_source, int32_t* transition_destination,
    int32_t* transition_pairs, int32_t* transition_raw, int32_t* freed_offsets,
    int32_t* freed_slots, int32_t* totals, int32_t* status, void* stream) {
  AKV_NVTX_RANGE("akv_drop_compact_static");
  using namespace akv;
  if (n_requests < 0 || n_tiles < 0 || n_requests > kStaticMaxRequests ||
      n_tiles > kStaticMaxTiles)
    return AKV_ERR_INVALID;
  if (workspace_bytes(n_requests, n_tiles) > kStaticScratchBytes) return AKV_ERR_INVALID;
  void* scratch = nullptr;
  const int st = static_scratch(&scratch);
  if (st != AKV_OK) return st;
  return akv_drop_compact(n_requests, token_offsets, tile_offsets, n_tiles, range_offsets, ranges,
                          shared_prefix, req_to_token, row_ids, row_stride, reposition, ring,
                          ring_capacity, ring_state, keep_mask, positions, active_offsets,
                          raw_indices, active_positions, next_position, transition_offsets,
                          transition_source, transition_destination, transition_pairs,
                          transition_raw, freed_offsets, freed_slots, totals, status, scratch,
                          stream);
}

// The decode view of one call, read back to host memory: five
// stream-ordered device-to-host copies into one int32 vector, so a serving
// loop reads a Drop's result with one library call (no launch, no sync).
extern "C" int akv_drop_read_view(int32_t* host_out, const int32_t* raw_indices,
                                  const int32_t* active_positions, int64_t kept,
                                  const int32_t* active_offsets, const int32_t* next_position,
                                  int32_t n_requests, const int32_t* counters, void* stream) {
  if (host_out == nullptr || kept < 0 || n_requests < 0 || active_offsets == nullptr ||
      counters == nullptr || (kept > 0 && (raw_indices == nullptr || active_positions == nullptr)) ||
      (n_requests > 0 && next_position == nullptr))
    return AKV_ERR_INVALID;
  const auto s = static_cast<cudaStream_t>(stream);
  const struct {
    const int32_t* src;
    int64_t count;
  } parts[] = {{raw_indices, kept},
               {active_positions, kept},
               {active_offsets, (int64_t)n_requests + 1},
               {next_position, n_requests},
               {counters, 5}};
  int32_t* dst = host_out;
  for (const auto& part : parts) {
    if (part.count > 0 && cudaMemcpyAsync(dst, part.src, (size_t)part.count * sizeof(int32_t),
                                          cudaMemcpyDeviceToHost, s) != cudaSuccess)
      return AKV_ERR_CUDA;
    dst += part.count;
  }
  return AKV_OK;
}
