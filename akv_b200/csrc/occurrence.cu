// Occurrence slot gathers: the device side of request-local page ownership
// between prefill forwards.
//
// The reference prepares every index on the scheduler CPU and then binds
// physical slots on the device with a chain of small torch operations per
// request: a concatenation of the state's slots with the new query and extra
// slots, one gather per output field and int32 casts
// (srt/context_system/occurrence.py:315-357 OccurrenceMaterialization.bind,
// :644-755 OccurrenceState.advance, :757-768 OccurrenceState.terminal_slots),
// and the scheduler concatenates the per-request results
// (akv/system/sglang.patch:3133-3180).  Here one launch runs every field of
// every request of a forward: a task reads its indices from one packed
// host-to-device copy and gathers from the virtual concatenation of up to
// four slot vectors, so neither the concatenation nor the per-request
// outputs are materialised separately.
//
// Work: one block per chunk of kSlotChunk outputs of one task (the host cuts
// each task into chunks).  Each output is one 4-byte index load, at most one
// 4- or 8-byte slot load and one store; the kernel is bound by launch and
// latency at the sizes a forward binds (thousands of slots), and by HBM at
// large ones.
#include "akv_b200.h"
#include "common.cuh"

namespace akv {
namespace {

constexpr int kSlotChunk = 1024;
constexpr int kSlotThreads = 256;
constexpr int kTaskWords = 12;
constexpr int kMaxSegments = 4;

__global__ void __launch_bounds__(kSlotThreads) gather_slots_kernel(
    const int64_t* __restrict__ tasks, const int2* __restrict__ chunks,
    const int32_t* __restrict__ indices, int32_t* error_flag) {
  const int2 c = chunks[blockIdx.x];
  const int64_t* t = tasks + (int64_t)kTaskWords * c.x;
  const int64_t first = __ldg(t), n = __ldg(t + 1);
  const int64_t flags = __ldg(t + 3);
  const bool out64 = flags & AKV_GATHER_OUT64;
  const bool literal = flags & AKV_GATHER_LITERAL;
  const bool seg64 = flags & AKV_GATHER_SEG64;
  const int n_seg = (int)((flags >> 8) & 0xff);
  const void* seg[kMaxSegments];
  int64_t seg_end[kMaxSegments];
#pragma unroll
  for (int s = 0; s < kMaxSegments; ++s) {
    seg[s] = reinterpret_cast<const void*>(__ldg(t + 4 + s));
    seg_end[s] = s < n_seg ? __ldg(t + 8 + s) : -1;
  }
  void* out = reinterpret_cast<void*>(__ldg(t + 2));
  // Every index of the thread is loaded, then every slot, then every store
  // is made: two dependent memory round trips per thread, not eight.
  constexpr int kPer = kSlotChunk / kSlotThreads;
  int64_t v[kPer];
  bool live[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int64_t k = (int64_t)c.y + j * kSlotThreads + threadIdx.x;
    live[j] = k < n;
    v[j] = live[j] ? (int64_t)__ldg(indices + first + k) : -1;
  }
  if (!literal) {
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      if (!live[j] || v[j] < 0) {
        v[j] = -1;
        continue;
      }
      int64_t base = 0, local = -1;
      int s_hit = -1;
#pragma unroll
      for (int s = 0; s < kMaxSegments; ++s) {
        if (s_hit < 0 && v[j] < seg_end[s]) {
          s_hit = s;
          local = v[j] - base;
        }
        if (s < n_seg) base = seg_end[s];
      }
      if (s_hit < 0) {
        if (error_flag != nullptr) *error_flag = 1;
        v[j] = -1;
        continue;
      }
      const void* p = seg[0];
#pragma unroll
      for (int s = 1; s < kMaxSegments; ++s)
        if (s_hit == s) p = seg[s];
      v[j] = seg64 ? __ldg(static_cast<const int64_t*>(p) + local)
                   : (int64_t)__ldg(static_cast<const int32_t*>(p) + local);
    }
  }
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    if (!live[j]) continue;
    const int64_t k = (int64_t)c.y + j * kSlotThreads + threadIdx.x;
    if (out64) static_cast<int64_t*>(out)[k] = v[j];
    else static_cast<int32_t*>(out)[k] = (int32_t)v[j];
  }
}

}  // namespace
}  // namespace akv

extern "C" int64_t akv_gather_slots_chunk(void) { return akv::kSlotChunk; }

extern "C" int akv_gather_slots(const int64_t* tasks, const int32_t* chunks, int32_t n_chunks,
                                const int32_t* indices, int32_t* error_flag, void* stream) {
  AKV_NVTX_RANGE("akv_gather_slots");
  using namespace akv;
  if (n_chunks < 0) return AKV_ERR_INVALID;
  if (n_chunks == 0) return AKV_OK;
  if (!tasks || !chunks || !indices) return AKV_ERR_INVALID;
  gather_slots_kernel<<<n_chunks, kSlotThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      tasks, reinterpret_cast<const int2*>(chunks), indices, error_flag);
  return launch_status();
}
