// Reposition: RoPE re-rotation of retained K rows plus the K-tail / V move,
// for every layer of a pointer table, in one persistent launch.
//
// Replaces _reposition_layers_kernel / reposition_kv_layers
// (akv/system/sglang/kernels/ops/attention/context_reposition.py:28-123,
// :126-236).  The reference launches one 4-warp program per
// (token, layer, head) that moves a single 128-byte row.  Here one thread
// ("unit") owns V consecutive rotary pairs of one (token, head) -- two
// 16-byte vectors -- and walks all layers, so the token's slots, positions
// and cos/sin values are loaded once and reused across layers, and every
// warp moves whole contiguous [heads x head_dim] rows with 16-byte accesses.
//
// Arithmetic is the reference's, operation for operation, with explicitly
// rounded intrinsics (no FMA contraction):
//   s  = oc*oc + os*os
//   u1 = (x1*oc + x2*os) / s         u2 = (x2*oc - x1*os) / s
//   y1 = u1*nc - u2*ns               y2 = u2*nc + u1*ns
// and the source values are stored unchanged when old == new position.

#include "common.cuh"

namespace akv {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxLayers = 512;

struct RepositionParams {
  const unsigned long long* k_ptrs;
  const unsigned long long* v_ptrs;
  int n_layers;
  int num_heads;
  int head_dim;
  int rotary_dim;
  int half;
  long long k_ss, k_sh, v_ss, v_sh;
  const int* src;
  const int* dst;
  const int* pairs;
  long long pstride;
  long long count;
  const int* count_dev;
  const void* cache;
  long long cache_stride;
  int skip_unmapped;
  long long num_slots;     // 0 = unchecked
  long long max_position;  // 0 = unchecked
  int* error_flag;
};

// V consecutive elements of T, moved with one 16- or 8-byte access when
// V * sizeof(T) is 16 or 8 bytes, element by element otherwise.
template <typename T, int V> struct alignas(V * sizeof(T) >= 16 ? 16 : 8) Chunk {
  T e[V];
  // `vec` is false for a layer whose base address is not 16-byte aligned;
  // the branch is uniform across the grid for a given layer.
  __device__ __forceinline__ void load(const T* p, bool vec) {
    if constexpr (V * sizeof(T) == 16) {
      if (vec) {
        uint4 r;
        asm volatile("ld.global.cs.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                     : "l"(p));
        *reinterpret_cast<uint4*>(e) = r;
        return;
      }
    } else if constexpr (V * sizeof(T) == 8) {
      if (vec) {
        uint2 r;
        asm volatile("ld.global.cs.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
        *reinterpret_cast<uint2*>(e) = r;
        return;
      }
    }
#pragma unroll
    for (int i = 0; i < V; ++i) e[i] = p[i];
  }
  __device__ __forceinline__ void store(T* p, bool vec) const {
    if constexpr (V * sizeof(T) == 16) {
      if (vec) {
        const uint4 r = *reinterpret_cast<const uint4*>(e);
        asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(r.x), "r"(r.y),
                     "r"(r.z), "r"(r.w)
                     : "memory");
        return;
      }
    } else if constexpr (V * sizeof(T) == 8) {
      if (vec) {
        const uint2 r = *reinterpret_cast<const uint2*>(e);
        asm volatile("st.global.cs.v2.u32 [%0], {%1,%2};" ::"l"(p), "r"(r.x), "r"(r.y)
                     : "memory");
        return;
      }
    }
#pragma unroll
    for (int i = 0; i < V; ++i) p[i] = e[i];
  }
};

template <typename C>
__device__ __forceinline__ float cache_at(const void* base, long long idx) {
  return Elem<C>::to_f32(static_cast<const C*>(base)[idx]);
}

// Correctly rounded n / s for both numerators of a pair, given
// y = RN(1/s) (computed once per token and pair with __frcp_rn and reused
// across every layer and head).
//
// Method: Markstein's FMA correction (P. Markstein, "Computation of
// elementary functions on the IBM RISC System/6000 processor", IBM J. Res.
// Dev. 34(1), 1990; "IA-64 and Elementary Functions", 2000): if y is within
// half an ulp of 1/s and q within one ulp of n/s, then r = n - s*q is exact
// in one FMA and RN(q + r*y) is the correctly rounded quotient.  q0 = RN(n*y)
// can be up to about 1.5 ulp away, so one correction step first brings it
// within (0.5 + 2^-23) ulp and a second one, under the theorem, gives
// RN(n/s) -- the value IEEE division (__fdiv_rn, the reference's tl.div_rn)
// returns.  The theorem needs no underflow or overflow in the remainders:
// the fast path is taken only when s lies in [2^-60, 2^60] (checked once per
// token) and |n| in [2^-100, 2^100]; anything else, zeros (whose sign the
// FMA chain would not keep) and non-finite values included, uses __fdiv_rn.
// tests/test_reposition_gpu.py compares the two over adversarial inputs.
constexpr float kDivMin = 0x1p-60f, kDivMax = 0x1p60f;
constexpr float kNumMin = 0x1p-100f, kNumMax = 0x1p100f;

__device__ __forceinline__ float markstein_div(float n, float s, float y) {
  float q = __fmul_rn(n, y);
  float r = __fmaf_rn(-s, q, n);
  q = __fmaf_rn(r, y, q);
  r = __fmaf_rn(-s, q, n);
  return __fmaf_rn(r, y, q);
}

__device__ __forceinline__ void div2_rn(float n1, float n2, float s, float y, bool s_ok,
                                        float& u1, float& u2) {
  const float a1 = fabsf(n1), a2 = fabsf(n2);
  if (s_ok && a1 >= kNumMin && a1 <= kNumMax && a2 >= kNumMin && a2 <= kNumMax) {
    u1 = markstein_div(n1, s, y);
    u2 = markstein_div(n2, s, y);
  } else {
    u1 = __fdiv_rn(n1, s);
    u2 = __fdiv_rn(n2, s);
  }
}

// Layers loaded before any is rotated, so that 2 * LU independent 16-byte
// loads are in flight per thread.
#ifndef AKV_REPOSITION_UNROLL
#define AKV_REPOSITION_UNROLL 2
#endif
// Bytes per vector access (16 or 8) and resident blocks per SM the register
// budget is sized for.
#ifndef AKV_REPOSITION_VECTOR_BYTES
#define AKV_REPOSITION_VECTOR_BYTES 16
#endif
#ifndef AKV_REPOSITION_MIN_BLOCKS
#define AKV_REPOSITION_MIN_BLOCKS 2
#endif
template <typename T> struct Unroll { static constexpr int value = AKV_REPOSITION_UNROLL; };

template <typename T, typename C, bool NEOX, int V>
__global__ void __launch_bounds__(kThreads, AKV_REPOSITION_MIN_BLOCKS)
reposition_kernel(const RepositionParams p) {
  constexpr int LU = Unroll<T>::value;
  __shared__ unsigned long long s_k[kMaxLayers];
  __shared__ unsigned long long s_v[kMaxLayers];
  __shared__ bool s_vec[kMaxLayers];
  for (int i = threadIdx.x; i < p.n_layers; i += blockDim.x) {
    s_k[i] = p.k_ptrs[i];
    s_v[i] = p.v_ptrs[i];
    s_vec[i] = ((s_k[i] | s_v[i]) & (V * sizeof(T) - 1)) == 0;
  }
  __syncthreads();

  long long count = p.count;
  if (p.count_dev != nullptr) {
    const long long c = *p.count_dev;
    count = c < count ? c : count;
  }
  const int chunks = p.half / V;             // units per head
  const int upt = p.num_heads * chunks;      // units per token
  const long long total = count * upt;
  // Vectors of V elements per head that a copy moves: K tail then all of V.
  const int tail_vecs = (p.head_dim - p.rotary_dim) / V;
  const int copy_vecs = tail_vecs + p.head_dim / V;
  const long long stride = (long long)gridDim.x * blockDim.x;

  for (long long u = (long long)blockIdx.x * blockDim.x + threadIdx.x; u < total; u += stride) {
    const long long tok = u / upt;
    const int rem = (int)(u - tok * upt);
    const int head = rem / chunks;
    const int chunk = rem - head * chunks;
    const long long src = __ldg(p.src + tok);
    const long long dst = __ldg(p.dst + tok);
    if (p.skip_unmapped && (src <= 0 || dst <= 0)) continue;
    const long long po = __ldg(p.pairs + tok * p.pstride);
    const long long pn = __ldg(p.pairs + tok * p.pstride + 1);
    if ((p.num_slots > 0 && (src < 0 || dst < 0 || src >= p.num_slots || dst >= p.num_slots)) ||
        (p.max_position > 0 && (po < 0 || pn < 0 || po >= p.max_position || pn >= p.max_position))) {
      if (p.error_flag != nullptr) *p.error_flag = 1;
      continue;
    }
    const bool same = po == pn;
    const bool in_place = src == dst;
    if (same && in_place) continue;  // rewriting identical bits: nothing to do

    const int j = chunk * V;  // first pair of this unit
    const int o1 = NEOX ? j : 2 * j;
    const int o2 = NEOX ? p.half + j : 2 * j + V;

    float oc[V], os[V], nc[V], ns[V], sc[V], rc[V];
    bool scale_ok = true;
    {
      const long long ro = po * p.cache_stride, rn = pn * p.cache_stride;
#pragma unroll
      for (int i = 0; i < V; ++i) {
        oc[i] = cache_at<C>(p.cache, ro + j + i);
        os[i] = cache_at<C>(p.cache, ro + p.half + j + i);
        nc[i] = cache_at<C>(p.cache, rn + j + i);
        ns[i] = cache_at<C>(p.cache, rn + p.half + j + i);
        sc[i] = __fadd_rn(__fmul_rn(oc[i], oc[i]), __fmul_rn(os[i], os[i]));
        rc[i] = __frcp_rn(sc[i]);
        scale_ok = scale_ok && sc[i] >= kDivMin && sc[i] <= kDivMax;
      }
    }
    const long long ks = src * p.k_ss + head * p.k_sh;
    const long long kd = dst * p.k_ss + head * p.k_sh;
    const long long vs = src * p.v_ss + head * p.v_sh;
    const long long vd = dst * p.v_ss + head * p.v_sh;

    for (int l0 = 0; l0 < p.n_layers; l0 += LU) {
      Chunk<T, V> a[LU], b[LU];
#pragma unroll
      for (int q = 0; q < LU; ++q) {
        if (l0 + q < p.n_layers) {
          const T* kb = reinterpret_cast<const T*>(s_k[l0 + q]);
          a[q].load(kb + ks + o1, s_vec[l0 + q]);
          b[q].load(kb + ks + o2, s_vec[l0 + q]);
        }
      }
#pragma unroll
      for (int q = 0; q < LU; ++q) {
        if (l0 + q < p.n_layers) {
          float x[2 * V];
#pragma unroll
          for (int i = 0; i < V; ++i) {
            x[i] = Elem<T>::to_f32(a[q].e[i]);
            x[V + i] = Elem<T>::to_f32(b[q].e[i]);
          }
          float y[2 * V];
          if (same) {
            // Old == new position: the reference stores the source values.
#pragma unroll
            for (int i = 0; i < 2 * V; ++i) y[i] = x[i];
          } else {
#pragma unroll
            for (int i = 0; i < V; ++i) {
              // NEOX pairs (i, half + i) -> (x[i], x[V + i]); GPT-J pairs
              // (2i, 2i + 1) of the 2V contiguous elements.
              const int i1 = NEOX ? i : 2 * i;
              const int i2 = NEOX ? V + i : 2 * i + 1;
              const float x1 = x[i1], x2 = x[i2];
              const float n1 = __fadd_rn(__fmul_rn(x1, oc[i]), __fmul_rn(x2, os[i]));
              const float n2 = __fsub_rn(__fmul_rn(x2, oc[i]), __fmul_rn(x1, os[i]));
              float u1, u2;
              div2_rn(n1, n2, sc[i], rc[i], scale_ok, u1, u2);
              y[i1] = __fsub_rn(__fmul_rn(u1, nc[i]), __fmul_rn(u2, ns[i]));
              y[i2] = __fadd_rn(__fmul_rn(u2, nc[i]), __fmul_rn(u1, ns[i]));
            }
          }
          Chunk<T, V> ra, rb;
#pragma unroll
          for (int i = 0; i < V; ++i) {
            ra.e[i] = Elem<T>::from_f32(y[i]);
            rb.e[i] = Elem<T>::from_f32(y[V + i]);
          }
          T* kb = reinterpret_cast<T*>(s_k[l0 + q]);
          ra.store(kb + kd + o1, s_vec[l0 + q]);
          rb.store(kb + kd + o2, s_vec[l0 + q]);
        }
      }
      if (!in_place) {
        // Copy-on-write: this unit moves vectors chunk, chunk + chunks, ...
        // of the head's K tail followed by its V row.
        for (int c = chunk; c < copy_vecs; c += chunks) {
          Chunk<T, V> t[LU];
#pragma unroll
          for (int q = 0; q < LU; ++q) {
            if (l0 + q < p.n_layers) {
              if (c < tail_vecs) {
                t[q].load(reinterpret_cast<const T*>(s_k[l0 + q]) + ks + p.rotary_dim + c * V,
                          s_vec[l0 + q]);
              } else {
                t[q].load(reinterpret_cast<const T*>(s_v[l0 + q]) + vs + (c - tail_vecs) * V,
                          s_vec[l0 + q]);
              }
            }
          }
#pragma unroll
          for (int q = 0; q < LU; ++q) {
            if (l0 + q < p.n_layers) {
              if (c < tail_vecs) {
                t[q].store(reinterpret_cast<T*>(s_k[l0 + q]) + kd + p.rotary_dim + c * V,
                           s_vec[l0 + q]);
              } else {
                t[q].store(reinterpret_cast<T*>(s_v[l0 + q]) + vd + (c - tail_vecs) * V,
                           s_vec[l0 + q]);
              }
            }
          }
        }
      }
    }
  }
}

template <typename T, typename C, bool NEOX, int V>
int launch(const RepositionParams& p, cudaStream_t stream) {
  auto kernel = reposition_kernel<T, C, NEOX, V>;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, 0) != cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  const long long units = p.count * (long long)p.num_heads * (p.half / V);
  const long long blocks = (units + kThreads - 1) / kThreads;
  const int grid = persistent_grid(per_sm, blocks);
  kernel<<<grid, kThreads, 0, stream>>>(p);
  return launch_status();
}

template <typename T, typename C>
int dispatch_style(const RepositionParams& p, bool neox, bool vec, cudaStream_t s) {
  constexpr int VV = AKV_REPOSITION_VECTOR_BYTES / sizeof(T);
  if (vec) return neox ? launch<T, C, true, VV>(p, s) : launch<T, C, false, VV>(p, s);
  return neox ? launch<T, C, true, 1>(p, s) : launch<T, C, false, 1>(p, s);
}

template <typename T>
int dispatch_cache(const RepositionParams& p, int cache_dtype, bool neox, bool vec,
                   cudaStream_t s) {
  switch (cache_dtype) {
    case AKV_F32: return dispatch_style<T, float>(p, neox, vec, s);
    case AKV_BF16: return dispatch_style<T, __nv_bfloat16>(p, neox, vec, s);
    case AKV_F16: return dispatch_style<T, __half>(p, neox, vec, s);
  }
  return AKV_ERR_INVALID;
}


}  // namespace
}  // namespace akv

extern "C" int akv_reposition_kv_layers(
    const void* k_data_ptrs, const void* v_data_ptrs, int32_t n_layers, int32_t kv_dtype,
    int32_t num_heads, int32_t head_dim, int32_t rotary_dim, int64_t k_stride_slot,
    int64_t k_stride_head, int64_t v_stride_slot, int64_t v_stride_head,
    const int32_t* source_slots, const int32_t* destination_slots,
    const int32_t* position_pairs, int64_t position_stride, int64_t count,
    const int32_t* count_device, const void* cos_sin_cache, int32_t cache_dtype,
    int64_t cache_stride, int32_t is_neox_style, int32_t skip_unmapped, int64_t num_slots,
    int64_t max_position, int32_t* error_flag, void* stream) {
  using namespace akv;
  if (count < 0 || n_layers < 0 || n_layers > kMaxLayers || num_heads <= 0 || head_dim <= 0 ||
      rotary_dim <= 0 || rotary_dim > head_dim || (rotary_dim & 1) || position_stride < 2)
    return AKV_ERR_INVALID;
  if (count == 0 || n_layers == 0) return AKV_OK;
  if (!k_data_ptrs || !v_data_ptrs || !source_slots || !destination_slots || !position_pairs ||
      !cos_sin_cache)
    return AKV_ERR_INVALID;
  RepositionParams p;
  p.k_ptrs = static_cast<const unsigned long long*>(k_data_ptrs);
  p.v_ptrs = static_cast<const unsigned long long*>(v_data_ptrs);
  p.n_layers = n_layers;
  p.num_heads = num_heads;
  p.head_dim = head_dim;
  p.rotary_dim = rotary_dim;
  p.half = rotary_dim / 2;
  p.k_ss = k_stride_slot;
  p.k_sh = k_stride_head;
  p.v_ss = v_stride_slot;
  p.v_sh = v_stride_head;
  p.src = source_slots;
  p.dst = destination_slots;
  p.pairs = position_pairs;
  p.pstride = position_stride;
  p.count = count;
  p.count_dev = count_device;
  p.cache = cos_sin_cache;
  p.cache_stride = cache_stride;
  p.skip_unmapped = skip_unmapped;
  p.num_slots = num_slots;
  p.max_position = max_position;
  p.error_flag = error_flag;

  const int esize = kv_dtype == AKV_F32 ? 4 : 2;
  const int V = AKV_REPOSITION_VECTOR_BYTES / esize;
  // The vector path needs every vector to start on a vector boundary:
  // shapes and strides are checked here, each layer's base address in the
  // kernel (a misaligned layer falls back to element accesses).
  const bool vec = (p.half % V == 0) && (head_dim % V == 0) && (rotary_dim % V == 0) &&
                   (k_stride_slot % V == 0) && (k_stride_head % V == 0) &&
                   (v_stride_slot % V == 0) && (v_stride_head % V == 0);
  const bool neox = is_neox_style != 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (kv_dtype) {
    case AKV_F32: return dispatch_cache<float>(p, cache_dtype, neox, vec, s);
    case AKV_BF16: return dispatch_cache<__nv_bfloat16>(p, cache_dtype, neox, vec, s);
    case AKV_F16: return dispatch_cache<__half>(p, cache_dtype, neox, vec, s);
  }
  return AKV_ERR_INVALID;
}

namespace akv {
namespace {

__global__ void divide_kernel(const float* n, const float* s, float* q, int64_t count,
                              int method) {
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += step) {
    const float d = s[i];
    if (method == 0) {
      q[i] = __fdiv_rn(n[i], d);
    } else {
      const bool d_ok = d >= kDivMin && d <= kDivMax;
      float u1, u2;
      div2_rn(n[i], n[i], d, __frcp_rn(d), d_ok, u1, u2);
      q[i] = u1;
    }
  }
}

}  // namespace
}  // namespace akv

extern "C" int akv_reposition_divide(const float* numerators, const float* denominators,
                                     float* quotients, int64_t count, int32_t method,
                                     void* stream) {
  using namespace akv;
  if (count < 0 || (method != 0 && method != 1) ||
      (count > 0 && (!numerators || !denominators || !quotients)))
    return AKV_ERR_INVALID;
  if (count == 0) return AKV_OK;
  const int blocks = (int)((count + 255) / 256 < 4096 ? (count + 255) / 256 : 4096);
  divide_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      numerators, denominators, quotients, count, method);
  return launch_status();
}
