// Decode page-table kernels over the compacted active-index view.
//
// Replace the reference's Triton kernels context_decode_indices and
// context_window_lengths
// (akv/system/sglang/kernels/ops/attention/context_page_table.py:7-76) and
// write_row_slots (akv/system/sglang/kernels/ops/memory/context_rows.py:7-15).
// The Triton decode-index kernel runs one program per request that walks
// the request's whole length 256 indices at a time, so a 64K-token request
// serialises on one SM.  Here each request is split over several blocks
// (grid = splits x batch) that stride through it, so the batch's total
// length is spread over every SM whatever the length distribution.

#include "common.cuh"

namespace akv {
namespace {

constexpr int kThreads = 256;

// Registry row: {raw_ids*, positions*, prompt_len, active, next_pos, row*}
// (srt/layers/attention/context_backend.py:716-725).
struct Entry {
  const int32_t* raw_ids;
  const int32_t* positions;
  int32_t prompt;
  int32_t active;
  int32_t next_pos;
  const int32_t* row;
};

__device__ __forceinline__ Entry load_entry(const int64_t* registry, int64_t row) {
  const long long* e = reinterpret_cast<const long long*>(registry) + row * 6;
  Entry x;
  x.raw_ids = reinterpret_cast<const int32_t*>(e[0]);
  x.positions = reinterpret_cast<const int32_t*>(e[1]);
  x.prompt = (int32_t)e[2];
  x.active = (int32_t)e[3];
  x.next_pos = (int32_t)e[4];
  x.row = reinterpret_cast<const int32_t*>(e[5]);
  return x;
}

struct IndexArgs {
  const int64_t* registry;
  const int32_t* table;
  int64_t row_stride;
  const void* row_ids;
  int row_ids_is64;
  const void* lengths;
  int lengths_is64;
  const void* indptr;
  int indptr_is64;
  void* output;
  int output_is64;
  const void* starts;
  int starts_is64;
  const void* mapping;
  int mapping_is64;
  int64_t multiplier;
};

__global__ void __launch_bounds__(kThreads) decode_indices_kernel(const IndexArgs a) {
  const int b = blockIdx.y;
  const int64_t row = ld_index(a.row_ids, b, a.row_ids_is64);
  const int64_t length = ld_index(a.lengths, b, a.lengths_is64);
  const int64_t offset = ld_index(a.indptr, b, a.indptr_is64);
  const int64_t start = a.starts ? ld_index(a.starts, b, a.starts_is64) : 0;
  const Entry e = load_entry(a.registry, row);
  const bool context = e.raw_ids != nullptr;
  const int32_t* raw_row = e.row != nullptr ? e.row : a.table + row * a.row_stride;
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < length; i += step) {
    const int64_t logical = start + i;
    int64_t raw = logical;
    if (context)
      raw = logical < e.active ? (int64_t)__ldg(e.raw_ids + logical)
                               : (int64_t)e.prompt + logical - e.active;
    int64_t slot = __ldg(raw_row + raw);
    if (a.mapping) slot = ld_index(a.mapping, slot, a.mapping_is64) * a.multiplier;
    st_index(a.output, offset + i, a.output_is64, slot);
  }
}

// Key-balanced decode indices: the batch's keys are spread evenly over the
// grid instead of splitting each request a fixed number of ways.  Each block
// scans the lengths into shared memory (key k of the batch belongs to the
// last request whose first key is at or before k), takes 1,024 consecutive
// keys at a time, finds each key's request by a binary search of that scan
// and writes it at kv_indptr[request] + its index in the request, exactly
// where the per-request kernel writes it for any lengths and indptr
// (padded tables included).  A 64K-key request thus does not leave a few
// blocks running long after the rest.  Each thread loads its four raw
// indices, then its four slots, then stores.  Batches up to kFlatMaxBatch.
constexpr int kFlatChunk = 1024;
constexpr int kFlatPer = kFlatChunk / kThreads;
// The request table of 1,000 requests and their scan fill 48,008 bytes, under
// the 48 KiB a launch gets without opting in.
constexpr int kFlatMaxBatch = 1000;
constexpr int kFlatScanPer = (kFlatMaxBatch + kThreads - 1) / kThreads;  // lengths per thread

struct FlatRequest {
  const int32_t* raw_ids;  // null: ordinary request
  const int32_t* row;
  int64_t start;
  int64_t out;             // kv_indptr[b]
  int32_t active;
  int32_t prompt;
};

__global__ void __launch_bounds__(kThreads) decode_indices_flat_kernel(const IndexArgs a,
                                                                       int batch) {
  extern __shared__ __align__(16) unsigned char flat_smem[];
  int64_t* s_cum = reinterpret_cast<int64_t*>(flat_smem);                   // [batch + 1]
  FlatRequest* s_req = reinterpret_cast<FlatRequest*>(s_cum + batch + 1);  // [batch]
  __shared__ int64_t s_warp[kThreads / 32];
  // Per-request table and the exclusive scan of the lengths (negative: 0).
  int64_t len[kFlatScanPer];
  int64_t mine = 0;
#pragma unroll
  for (int j = 0; j < kFlatScanPer; ++j) {
    const int b = threadIdx.x * kFlatScanPer + j;
    len[j] = 0;
    if (b < batch) {
      const int64_t row = ld_index(a.row_ids, b, a.row_ids_is64);
      const Entry e = load_entry(a.registry, row);
      FlatRequest r;
      r.raw_ids = e.raw_ids;
      r.row = e.row != nullptr ? e.row : a.table + row * a.row_stride;
      r.start = a.starts ? ld_index(a.starts, b, a.starts_is64) : 0;
      r.out = ld_index(a.indptr, b, a.indptr_is64);
      r.active = e.active;
      r.prompt = e.prompt;
      s_req[b] = r;
      const int64_t l = ld_index(a.lengths, b, a.lengths_is64);
      len[j] = l > 0 ? l : 0;
    }
    mine += len[j];
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int64_t inc = mine;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int64_t o = __shfl_up_sync(0xffffffffu, inc, d);
    if (lane >= d) inc += o;
  }
  if (lane == 31) s_warp[warp] = inc;
  __syncthreads();
  int64_t before = 0;
#pragma unroll
  for (int w = 0; w < kThreads / 32; ++w)
    if (w < warp) before += s_warp[w];
  int64_t run = before + inc - mine;
#pragma unroll
  for (int j = 0; j < kFlatScanPer; ++j) {
    const int b = threadIdx.x * kFlatScanPer + j;
    if (b < batch) s_cum[b] = run;
    run += len[j];
  }
  if (threadIdx.x == kThreads - 1) s_cum[batch] = run;  // the last thread ends the scan
  __syncthreads();
  const int64_t total = s_cum[batch];
  for (int64_t base = (int64_t)blockIdx.x * kFlatChunk; base < total;
       base += (int64_t)gridDim.x * kFlatChunk) {
    int64_t raw[kFlatPer], dst[kFlatPer];
    const int32_t* rowp[kFlatPer];
#pragma unroll
    for (int j = 0; j < kFlatPer; ++j) {
      const int64_t k = base + j * kThreads + threadIdx.x;
      rowp[j] = nullptr;
      raw[j] = dst[j] = 0;
      if (k >= total) continue;
      int lo = 0, hi = batch;  // the last request whose first key is at or before k
      while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (s_cum[mid] <= k) lo = mid;
        else hi = mid;
      }
      const FlatRequest& r = s_req[lo];
      const int64_t i = k - s_cum[lo];
      const int64_t logical = r.start + i;
      rowp[j] = r.row;
      dst[j] = r.out + i;
      raw[j] = r.raw_ids == nullptr ? logical
               : logical < r.active ? (int64_t)__ldg(r.raw_ids + logical)
                                    : (int64_t)r.prompt + logical - r.active;
    }
    int64_t slot[kFlatPer];
#pragma unroll
    for (int j = 0; j < kFlatPer; ++j) slot[j] = rowp[j] ? (int64_t)__ldg(rowp[j] + raw[j]) : 0;
    if (a.mapping) {
#pragma unroll
      for (int j = 0; j < kFlatPer; ++j)
        if (rowp[j]) slot[j] = ld_index(a.mapping, slot[j], a.mapping_is64) * a.multiplier;
    }
#pragma unroll
    for (int j = 0; j < kFlatPer; ++j)
      if (rowp[j]) st_index(a.output, dst[j], a.output_is64, slot[j]);
  }
}

// Window length of one request computed by the eight lanes of a lane group
// (lanes 8g .. 8g + 7 of a warp; every lane of the warp calls this, `has`
// false for lanes without a request): each round the eight lanes probe
// eight evenly spaced positions of the request's active range and keep the
// ninth part that holds the first position at or above the window's lower
// edge, so a 64K range takes six dependent loads instead of sixteen.  Every
// lane of the group returns the length.
__device__ __forceinline__ long long group_window_length(bool has, const Entry& e, long long seq,
                                                         int64_t window) {
  const int lane = threadIdx.x & 31, sub = threadIdx.x & 7, first_lane = lane & 24;
  const unsigned group = 0xffu << first_lane;
  long long lower = 0, generated = 0;
  int32_t lo = 0, hi = 0;
  if (has && e.raw_ids != nullptr) {
    generated = seq - e.active;
    // the window is the inclusive distance q_pos - k_pos (context_page_table.py:19-20)
    lower = (long long)e.next_pos + generated - 1 - window;
    hi = e.active;
  }
  while (__any_sync(0xffffffffu, hi > lo)) {
    int32_t probe = lo;
    bool below = false;
    if (hi > lo) {
      probe = lo + (int32_t)(((long long)(hi - lo) * (sub + 1)) / 9);
      below = (long long)__ldg(e.positions + probe) < lower;
    }
    const int c = __popc(__ballot_sync(0xffffffffu, below) & group);
    const int32_t p_below = __shfl_sync(0xffffffffu, probe, first_lane + (c > 0 ? c - 1 : 0));
    const int32_t p_above = __shfl_sync(0xffffffffu, probe, first_lane + (c < 8 ? c : 7));
    if (hi > lo) {
      if (c > 0) lo = p_below + 1;
      if (c < 8) hi = p_above;
    }
  }
  if (e.raw_ids == nullptr) return seq < window ? seq : window;
  const long long skipped = lower - e.next_pos > 0 ? lower - e.next_pos : 0;
  return (long long)e.active - lo + generated - skipped;
}

// The drop-in context_window_lengths: eight lanes per request.
__global__ void __launch_bounds__(kThreads) window_lengths_kernel(
    const int64_t* registry, const void* row_ids, int row_ids_is64, const void* lengths,
    int lengths_is64, void* output, int output_is64, int64_t window, int batch) {
  const int b = (int)(((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 3);
  const bool has = b < batch;
  Entry e{};
  long long seq = 0;
  if (has) {
    seq = ld_index(lengths, b, lengths_is64);
    e = load_entry(registry, ld_index(row_ids, b, row_ids_is64));
  }
  const long long len = group_window_length(has, e, seq, window);
  if (has && (threadIdx.x & 7) == 0) st_index(output, b, output_is64, len);
}

// One block: lengths (windowed or not), their exclusive scan into kv_indptr,
// and starts = seq_len - length.  Windowed lengths are found first, eight
// lanes per request (group_window_length), into lengths_out, which the scan
// then reads.
__global__ void __launch_bounds__(1024) decode_lengths_scan_kernel(
    const int64_t* registry, const int64_t* row_ids, const int64_t* seq_lens, int64_t window,
    int batch, int32_t* kv_indptr, int64_t* lengths_out, int64_t* starts_out) {
  __shared__ long long warp_sums[32];
  __shared__ long long carry;
  if (threadIdx.x == 0) carry = 0;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (window >= 0) {
    for (int b0 = 0; b0 < batch; b0 += blockDim.x >> 3) {
      const int b = b0 + (threadIdx.x >> 3);
      const bool has = b < batch;
      Entry e{};
      long long seq = 0;
      if (has) {
        seq = seq_lens[b];
        e = load_entry(registry, row_ids[b]);
      }
      const long long len = group_window_length(has, e, seq, window);
      if (has && (threadIdx.x & 7) == 0) lengths_out[b] = len;
    }
  }
  __syncthreads();
  for (int b0 = 0; b0 < batch; b0 += blockDim.x) {
    const int b = b0 + threadIdx.x;
    long long len = 0, seq = 0;
    if (b < batch) {
      seq = seq_lens[b];
      len = window >= 0 ? lengths_out[b] : seq;
    }
    long long inc = len;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const long long o = __shfl_up_sync(0xffffffffu, inc, d);
      if (lane >= d) inc += o;
    }
    if (lane == 31) warp_sums[warp] = inc;
    __syncthreads();
    if (warp == 0) {
      const long long w = warp_sums[lane];
      long long winc = w;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const long long o = __shfl_up_sync(0xffffffffu, winc, d);
        if (lane >= d) winc += o;
      }
      warp_sums[lane] = winc - w;
    }
    __syncthreads();
    const long long excl = carry + warp_sums[warp] + inc - len;
    if (b < batch) {
      kv_indptr[b] = (int32_t)excl;
      if (lengths_out) lengths_out[b] = len;
      if (starts_out) starts_out[b] = seq - len;
      if (b == batch - 1) kv_indptr[batch] = (int32_t)(excl + len);
    }
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = excl + len;
    __syncthreads();
  }
  if (batch == 0 && threadIdx.x == 0) kv_indptr[0] = 0;
}

__global__ void write_row_slots_kernel(const int64_t* pointers, const void* rows, int rows_is64,
                                       const void* cols, int cols_is64, const void* values,
                                       int values_is64, int64_t n) {
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += step) {
    int32_t* row = reinterpret_cast<int32_t*>(pointers[ld_index(rows, i, rows_is64)]);
    row[ld_index(cols, i, cols_is64)] = (int32_t)ld_index(values, i, values_is64);
  }
}

// Active slots of one request row for an offload / load / PD transfer:
// out[i] = row[device_indices[start + i]] for the n_prefix surviving prompt
// tokens, then out[n_prefix + j] = row[generated_start + j] for the generated
// tail.  A raw index or row position outside the row reads as slot -1 and
// sets *error_flag.
__global__ void active_slots_kernel(const int32_t* row, int64_t row_len,
                                    const int32_t* device_indices, int64_t start,
                                    int64_t n_prefix, int64_t generated_start, int64_t n_out,
                                    int32_t* out, int32_t* error_flag) {
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_out; i += step) {
    const int64_t col =
        i < n_prefix ? (int64_t)__ldg(device_indices + start + i) : generated_start + (i - n_prefix);
    int32_t v = -1;
    if (col >= 0 && col < row_len) v = __ldg(row + col);
    else if (error_flag != nullptr) *error_flag = 1;
    out[i] = v;
  }
}

// The same gather for a batch of requests in one launch.  meta holds, per
// request, {row address, row length, raw-index address, start, n_prefix,
// generated_start}; out_offsets is the CSR of the packed output; block b
// covers outputs [chunk[b].y, chunk[b].y + kGatherChunk) of request
// chunk[b].x (the host splits each request into such chunks).
constexpr int kGatherChunk = 1024;

__global__ void __launch_bounds__(kThreads) active_slots_batch_kernel(
    const int64_t* meta, const int64_t* out_offsets, const int2* chunks, int32_t* out,
    int32_t* error_flag) {
  const int2 c = chunks[blockIdx.x];
  const int64_t* m = meta + 6 * (int64_t)c.x;
  const int32_t* row = reinterpret_cast<const int32_t*>(__ldg(m));
  const int64_t row_len = __ldg(m + 1);
  const int32_t* idx = reinterpret_cast<const int32_t*>(__ldg(m + 2));
  const int64_t start = __ldg(m + 3), n_prefix = __ldg(m + 4), gen0 = __ldg(m + 5);
  const int64_t o0 = __ldg(out_offsets + c.x), n = __ldg(out_offsets + c.x + 1) - o0;
  // Every raw index of the thread, then every slot, then the stores: two
  // dependent memory round trips per thread instead of one per output.
  constexpr int kPer = kGatherChunk / kThreads;
  int64_t col[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int64_t k = (int64_t)c.y + j * kThreads + threadIdx.x;
    col[j] = k >= n ? -1 : k < n_prefix ? (int64_t)__ldg(idx + start + k) : gen0 + (k - n_prefix);
  }
  int32_t v[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) v[j] = col[j] >= 0 && col[j] < row_len ? __ldg(row + col[j]) : -1;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int64_t k = (int64_t)c.y + j * kThreads + threadIdx.x;
    if (k >= n) break;
    if ((col[j] < 0 || col[j] >= row_len) && error_flag != nullptr) *error_flag = 1;
    out[o0 + k] = v[j];
  }
}

int split_count(int batch) {
  // About 8 resident blocks per SM in total, at most 256 per request.
  long long want = (long long)kNumSMs * 8 / (batch > 0 ? batch : 1);
  if (want < 1) want = 1;
  if (want > 256) want = 256;
  return (int)want;
}

// Launch decode indices: the key-balanced kernel up to kFlatMaxBatch
// requests, else the per-request split.  max_keys (< 0: unknown) bounds the
// keys and so the chunks the key-balanced grid needs.
void launch_decode_indices(const IndexArgs& a, int batch, long long max_keys, cudaStream_t s) {
  if (batch <= kFlatMaxBatch) {
    // about four resident blocks per SM, fewer for a small batch
    long long blocks = batch * 8 < kNumSMs * 4 ? batch * 8 : kNumSMs * 4;
    if (max_keys >= 0) {
      const long long chunks = (max_keys + kFlatChunk - 1) / kFlatChunk;
      if (chunks < blocks) blocks = chunks > 0 ? chunks : 1;
    }
    const size_t smem = sizeof(int64_t) * (batch + 1) + sizeof(FlatRequest) * batch;
    decode_indices_flat_kernel<<<(unsigned)blocks, kThreads, smem, s>>>(a, batch);
  } else {
    dim3 grid(split_count(batch), batch);
    decode_indices_kernel<<<grid, kThreads, 0, s>>>(a);
  }
}

}  // namespace
}  // namespace akv

extern "C" int akv_context_decode_indices(
    const int64_t* registry, const int32_t* req_to_token, int64_t row_stride,
    const void* row_ids, int32_t row_ids_is64, const void* lengths, int32_t lengths_is64,
    const void* indptr, int32_t indptr_is64, void* output, int32_t output_is64,
    const void* starts, int32_t starts_is64, const void* mapping, int32_t mapping_is64,
    int64_t multiplier, int32_t batch, void* stream) {
  AKV_NVTX_RANGE("akv_context_decode_indices");
  using namespace akv;
  if (batch < 0 || batch > 65535 || !registry || !req_to_token || !row_ids || !lengths ||
      !indptr || !output)
    return AKV_ERR_INVALID;
  if (batch == 0) return AKV_OK;
  IndexArgs a{registry, req_to_token, row_stride, row_ids, row_ids_is64, lengths, lengths_is64,
              indptr, indptr_is64, output, output_is64, starts, starts_is64, mapping,
              mapping_is64, multiplier};
  launch_decode_indices(a, batch, -1, static_cast<cudaStream_t>(stream));
  return launch_status();
}

extern "C" int akv_context_window_lengths(
    const int64_t* registry, const void* row_ids, int32_t row_ids_is64, const void* lengths,
    int32_t lengths_is64, void* output, int32_t output_is64, int64_t window, int32_t batch,
    void* stream) {
  AKV_NVTX_RANGE("akv_context_window_lengths");
  using namespace akv;
  if (batch < 0 || !registry || !row_ids || !lengths || !output) return AKV_ERR_INVALID;
  if (batch == 0) return AKV_OK;
  window_lengths_kernel<<<(int)(((long long)batch * 8 + kThreads - 1) / kThreads), kThreads, 0,
                          static_cast<cudaStream_t>(stream)>>>(
      registry, row_ids, row_ids_is64, lengths, lengths_is64, output, output_is64, window, batch);
  return launch_status();
}

extern "C" int akv_build_decode_metadata(
    const int64_t* registry, const int32_t* req_to_token, int64_t row_stride,
    const int64_t* row_ids, const int64_t* seq_lens, int64_t window, const int64_t* mapping,
    int64_t multiplier, int32_t batch, int32_t* kv_indptr, int64_t* lengths_out,
    int64_t* starts_out, int32_t* kv_indices, void* stream) {
  AKV_NVTX_RANGE("akv_build_decode_metadata");
  using namespace akv;
  if (batch < 0 || batch > 65535 || !registry || !req_to_token || !row_ids || !seq_lens ||
      !kv_indptr || !kv_indices)
    return AKV_ERR_INVALID;
  if (window >= 0 && (!lengths_out || !starts_out)) return AKV_ERR_INVALID;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  decode_lengths_scan_kernel<<<1, 1024, 0, s>>>(registry, row_ids, seq_lens, window, batch,
                                                 kv_indptr, lengths_out, starts_out);
  if (batch == 0) return launch_status();
  IndexArgs a{registry, req_to_token, row_stride, row_ids, 1,
              window >= 0 ? (const void*)lengths_out : (const void*)seq_lens, 1, kv_indptr, 0,
              kv_indices, 0, window >= 0 ? starts_out : nullptr, 1, mapping, 1, multiplier};
  // A window keeps at most window + 1 keys of a request (the positions from
  // q_pos - window to q_pos).
  const long long max_keys =
      window >= 0 && window < (1LL << 40) ? (long long)batch * (window + 1) : -1;
  launch_decode_indices(a, batch, max_keys, s);
  return launch_status();
}

extern "C" int akv_write_row_slots(const int64_t* pointers, const void* rows, int32_t rows_is64,
                                   const void* columns, int32_t columns_is64, const void* values,
                                   int32_t values_is64, int64_t n, void* stream) {
  AKV_NVTX_RANGE("akv_write_row_slots");
  using namespace akv;
  if (n < 0 || (n > 0 && (!pointers || !rows || !columns || !values))) return AKV_ERR_INVALID;
  if (n == 0) return AKV_OK;
  const int blocks = (int)((n + kThreads - 1) / kThreads < 1024 ? (n + kThreads - 1) / kThreads
                                                                 : 1024);
  write_row_slots_kernel<<<blocks, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      pointers, rows, rows_is64, columns, columns_is64, values, values_is64, n);
  return launch_status();
}

extern "C" int akv_active_slots(const int32_t* row, int64_t row_len,
                                const int32_t* device_indices, int64_t start, int64_t n_indices,
                                int64_t generated_start, int64_t raw_end, int32_t* out,
                                int32_t* error_flag, void* stream) {
  AKV_NVTX_RANGE("akv_active_slots");
  using namespace akv;
  if (row_len < 0 || start < 0 || n_indices < start || generated_start < 0)
    return AKV_ERR_INVALID;
  const int64_t n_prefix = n_indices - start;
  const int64_t n_gen = raw_end > generated_start ? raw_end - generated_start : 0;
  const int64_t n_out = n_prefix + n_gen;
  if (n_out == 0) return AKV_OK;
  if (!row || !out || (n_prefix > 0 && !device_indices)) return AKV_ERR_INVALID;
  const int64_t want = (n_out + kThreads - 1) / kThreads;
  const int blocks = (int)(want < (int64_t)kNumSMs * 4 ? want : (int64_t)kNumSMs * 4);
  active_slots_kernel<<<blocks, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      row, row_len, device_indices, start, n_prefix, generated_start, n_out, out, error_flag);
  return launch_status();
}

extern "C" int64_t akv_active_slots_chunk(void) { return akv::kGatherChunk; }

extern "C" int akv_active_slots_batch(const int64_t* meta, const int64_t* out_offsets,
                                      const int32_t* chunks, int32_t n_chunks, int32_t* out,
                                      int32_t* error_flag, void* stream) {
  AKV_NVTX_RANGE("akv_active_slots_batch");
  using namespace akv;
  if (n_chunks < 0) return AKV_ERR_INVALID;
  if (n_chunks == 0) return AKV_OK;
  if (!meta || !out_offsets || !chunks || !out) return AKV_ERR_INVALID;
  active_slots_batch_kernel<<<n_chunks, kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      meta, out_offsets, reinterpret_cast<const int2*>(chunks), out, error_flag);
  return launch_status();
}

extern "C" const char* akv_version(void) { return "akv_b200 0.1 (sm_100a)"; }
