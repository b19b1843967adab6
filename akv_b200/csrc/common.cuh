// Shared device helpers for the akv_b200 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>
#include <stdint.h>

#include "akv_b200.h"

namespace akv {

// A named NVTX range over an entry point's host scope (its checks and
// launches).  Header-only NVTX v3: without a profiler attached each push and
// pop is a check of an unset function pointer; nsys / ncu show the range
// and the kernels it enqueued under it.
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};
#define AKV_NVTX_RANGE(name) ::akv::NvtxRange akv_nvtx_range_(name)

constexpr int kNumSMs = 148;

// Grid sized for a persistent launch: `per_sm` resident blocks on every SM.
inline int persistent_grid(int per_sm, long long work_blocks) {
  int device = 0;
  int sms = kNumSMs;
  if (cudaGetDevice(&device) == cudaSuccess) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) == cudaSuccess && v > 0)
      sms = v;
  }
  long long cap = (long long)sms * per_sm;
  long long g = work_blocks < cap ? work_blocks : cap;
  return g < 1 ? 1 : (int)g;
}

inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? AKV_OK : AKV_ERR_CUDA;
}

// Programmatic dependent launch.  A kernel launched by launch_pdl may be
// scheduled while the previous kernel of the stream is still running, once
// every block of that kernel has called pdl_launch_dependents() (or exited);
// it calls pdl_wait() before its first global memory access, which returns
// when the previous kernel has completed and its writes are visible.  This
// hides the launch gap between short dependent kernels.  After work that is
// not one of these kernels, the launch behaves like an ordinary one.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KernelArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KernelArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

// Load an index stored as int32 or int64 (dtype chosen at run time; the
// branch is uniform across the grid).
__device__ __forceinline__ int64_t ld_index(const void* p, int64_t i, int is64) {
  return is64 ? __ldg(static_cast<const long long*>(p) + i)
              : (int64_t)__ldg(static_cast<const int*>(p) + i);
}

__device__ __forceinline__ void st_index(void* p, int64_t i, int is64, int64_t v) {
  if (is64)
    static_cast<long long*>(p)[i] = (long long)v;
  else
    static_cast<int*>(p)[i] = (int)v;
}

// Element <-> fp32 conversions.  Loads are exact; stores round to nearest
// even, as a GPU store of an fp32 value into a 16-bit tensor does.
template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float to_f32(float x) { return x; }
  static __device__ __forceinline__ float from_f32(float x) { return x; }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_f32(float x) { return __float2bfloat16_rn(x); }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_f32(float x) { return __float2half_rn(x); }
};

// 16-byte vector of T.
template <typename T> struct Vec16 {
  static constexpr int N = 16 / sizeof(T);
  union {
    uint4 raw;
    T e[N];
  };
};

template <typename T>
__device__ __forceinline__ Vec16<T> ld16(const T* p) {
  Vec16<T> v;
  v.raw = *reinterpret_cast<const uint4*>(p);
  return v;
}

template <typename T>
__device__ __forceinline__ void st16(T* p, const Vec16<T>& v) {
  *reinterpret_cast<uint4*>(p) = v.raw;
}

// Streaming variants: the KV rows are touched once per call, keep them out
// of L1 and mark them evict-first in L2.
template <typename T>
__device__ __forceinline__ Vec16<T> ld16_stream(const T* p) {
  Vec16<T> v;
  asm volatile("ld.global.cs.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.raw.x), "=r"(v.raw.y), "=r"(v.raw.z), "=r"(v.raw.w)
               : "l"(p));
  return v;
}

template <typename T>
__device__ __forceinline__ void st16_stream(T* p, const Vec16<T>& v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.raw.x), "r"(v.raw.y),
               "r"(v.raw.z), "r"(v.raw.w)
               : "memory");
}

// Block-wide exclusive scan built from warp shuffles.  Returns the
// exclusive prefix of `v` and writes the block total to *total.  Every
// thread of the block must call it (it synchronises the block).
template <typename U>
__device__ U block_exclusive_scan(U v, U* total) {
  __shared__ U warp_sums[32];
  __shared__ U block_total;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  U inc = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    U o = __shfl_up_sync(0xffffffffu, inc, d);
    if (lane >= d) inc += o;
  }
  if (lane == 31) warp_sums[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    U w = lane < nwarps ? warp_sums[lane] : U(0);
    U winc = w;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      U o = __shfl_up_sync(0xffffffffu, winc, d);
      if (lane >= d) winc += o;
    }
    if (lane < nwarps) warp_sums[lane] = winc - w;  // exclusive base of each warp
    if (lane == 31) block_total = winc;
  }
  __syncthreads();
  const U base = warp_sums[warp];
  *total = block_total;
  __syncthreads();  // the next call may overwrite warp_sums
  return base + inc - v;
}

// Inclusive scan across one warp.
template <typename U>
__device__ __forceinline__ U warp_inclusive_scan(U v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    U o = __shfl_up_sync(0xffffffffu, v, d);
    if (lane >= d) v += o;
  }
  return v;
}

template <typename U>
__device__ __forceinline__ U warp_sum(U v) {
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
  return v;
}

// Number of entries of the sorted vector a[0, n) that are < x.
__device__ __forceinline__ int count_below(const int32_t* a, int n, long long x) {
  int lo = 0, hi = n;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if ((long long)__ldg(a + mid) < x) lo = mid + 1;
    else hi = mid;
  }
  return lo;
}

}  // namespace akv
