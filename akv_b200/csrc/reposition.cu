// Reposition: RoPE re-rotation of retained K rows plus the K-tail / V move,
// for every layer of a pointer table, in one persistent launch.
//
// Replaces _reposition_layers_kernel / reposition_kv_layers
// (akv/system/sglang/kernels/ops/attention/context_reposition.py:28-123,
// :126-236).  The reference launches one 4-warp program per
// (token, layer, head) that moves a single 128-byte row.  Here one thread
// ("unit") owns V consecutive rotary pairs of one (token, head) -- two
// 16-byte vectors per layer -- and walks all layers: the token's slots,
// positions and cos/sin values are loaded once and reused across layers,
// and a warp moves whole contiguous [heads x head_dim] rows.
//
// Memory pipeline: a unit's rows for the next S-1 layers are in flight
// while it rotates the current one.  They are fetched with per-thread
// cp.async into the thread's own shared-memory slots (no registers held,
// no barrier: a thread only reads what it fetched), so the loads of up to
// eight layers overlap the arithmetic of the current layer.  Results are
// stored straight back with streaming (evict-first) 16-byte stores.
//
// Arithmetic is the reference's, operation for operation, with explicitly
// rounded intrinsics (no FMA contraction):
//   s  = oc*oc + os*os
//   u1 = (x1*oc + x2*os) / s         u2 = (x2*oc - x1*os) / s
//   y1 = u1*nc - u2*ns               y2 = u2*nc + u1*ns
// the divisions correctly rounded (div2_rn below), and the source values
// stored unchanged when old == new position.

#include <type_traits>

#include "common.cuh"

namespace akv {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxLayers = 512;
// 16-byte staging slots per thread: 8 layers of a K pair in flight for an
// in-place unit, 4 layers of (K pair + 2 copied vectors) for copy-on-write.
constexpr int kSlots = 16;
constexpr int kStageBytes = kSlots * kThreads * 16;  // 64 KiB per block

#ifndef AKV_REPOSITION_MIN_BLOCKS
#define AKV_REPOSITION_MIN_BLOCKS 2
#endif

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
  float one;  // 1.0f, passed at run time (see the packed sums in rotate)
  int v_moved;  // copy-on-write V rows are moved by reposition_v_move_kernel
};

// V consecutive elements of T, moved with one 16-byte access when
// V * sizeof(T) is 16 and the layer is aligned, element by element otherwise.
template <typename T, int V> struct alignas(V * sizeof(T) >= 16 ? 16 : alignof(T)) Chunk {
  T e[V];
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
    }
#pragma unroll
    for (int i = 0; i < V; ++i) p[i] = e[i];
  }
  __device__ __forceinline__ void load_shared(uint32_t addr) {
    uint4 r;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "r"(addr));
    *reinterpret_cast<uint4*>(e) = r;
  }
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Cache element types.  F32Rows is an fp32 cache whose rows and halves
// start on 16-byte boundaries, read with vector loads.
struct F32Rows {};
template <typename C> struct CacheElem {
  using type = C;
  static constexpr bool kRows = false;
};
template <> struct CacheElem<F32Rows> {
  using type = float;
  static constexpr bool kRows = true;
};

template <typename C>
__device__ __forceinline__ float cache_at(const void* base, long long idx) {
  using E = typename CacheElem<C>::type;
  return Elem<E>::to_f32(static_cast<const E*>(base)[idx]);
}

// Correctly rounded n / s for both numerators of a pair, given
// y = RN(1/s) (computed once per token and pair with __frcp_rn and reused
// across every layer).
//
// Method: Markstein's FMA correction (P. Markstein, "Computation of
// elementary functions on the IBM RISC System/6000 processor", IBM J. Res.
// Dev. 34(1), 1990; "IA-64 and Elementary Functions", 2000): if y is within
// half an ulp of 1/s and q within one ulp of n/s, then r = n - s*q is exact
// in one FMA and RN(q + r*y) is the correctly rounded quotient.  q0 = RN(n*y)
// can be up to about 1.5 ulp away, so one correction step first brings it
// within (0.5 + 2^-23) ulp and a second one, under the theorem, gives
// RN(n/s) -- the value IEEE division (__fdiv_rn, the reference's tl.div_rn)
// returns.  The theorem needs the quotient and remainders clear of overflow
// and underflow: the fast path is taken only when s lies in [2^-30, 2^30]
// (checked once per token) and |n| in [2^-60, 2^60], so the quotient stays
// within [2^-90, 2^90]; anything else, zeros (whose sign the FMA chain would
// not keep) and non-finite values included, uses __fdiv_rn.
// tests/test_reposition_gpu.py compares the two over adversarial inputs.
constexpr float kDivMin = 0x1p-30f, kDivMax = 0x1p30f;
constexpr float kNumMin = 0x1p-60f, kNumMax = 0x1p60f;

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

// Per-unit constants: the V pairs' old/new cos and sin, s = cos^2+sin^2 of
// the old angle and its reciprocal.
template <int V> struct Trig {
  float oc[V], os[V], nc[V], ns[V], sc[V], rc[V];
  bool scale_ok;
  float one;
};

// V consecutive fp32 cache values as 16-byte read-only loads.
template <int V>
__device__ __forceinline__ void load_f32_vec(const float* src, float* out) {
#pragma unroll
  for (int i = 0; i < V; i += 4) {
    float4 v;
    asm("ld.global.nc.v4.f32 {%0,%1,%2,%3}, [%4];"
        : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
        : "l"(src + i));
    out[i] = v.x;
    out[i + 1] = v.y;
    out[i + 2] = v.z;
    out[i + 3] = v.w;
  }
}

template <typename C, int V>
__device__ __forceinline__ void load_trig(const RepositionParams& p, long long po, long long pn,
                                          int j, Trig<V>& tr) {
  const long long ro = po * p.cache_stride, rn = pn * p.cache_stride;
  tr.scale_ok = true;
  tr.one = p.one;
  constexpr bool kVec = CacheElem<C>::kRows && V % 4 == 0;
  if constexpr (kVec) {
    const float* c = static_cast<const float*>(p.cache);
    load_f32_vec<V>(c + ro + j, tr.oc);
    load_f32_vec<V>(c + ro + p.half + j, tr.os);
    load_f32_vec<V>(c + rn + j, tr.nc);
    load_f32_vec<V>(c + rn + p.half + j, tr.ns);
  }
#pragma unroll
  for (int i = 0; i < V; ++i) {
    if constexpr (!kVec) {
      tr.oc[i] = cache_at<C>(p.cache, ro + j + i);
      tr.os[i] = cache_at<C>(p.cache, ro + p.half + j + i);
      tr.nc[i] = cache_at<C>(p.cache, rn + j + i);
      tr.ns[i] = cache_at<C>(p.cache, rn + p.half + j + i);
    }
    tr.sc[i] = __fadd_rn(__fmul_rn(tr.oc[i], tr.oc[i]), __fmul_rn(tr.os[i], tr.os[i]));
    tr.rc[i] = __frcp_rn(tr.sc[i]);
    tr.scale_ok = tr.scale_ok && tr.sc[i] >= kDivMin && tr.sc[i] <= kDivMax;
  }
}

// Packed fp32 pairs: Blackwell's f32x2 add / sub / mul / fma (PTX ISA 8.6,
// sm_100a) round each lane exactly like the scalar .rn instruction, so two
// rotary pairs go through the reference's operation sequence per
// instruction with bit-identical results.
using f2 = unsigned long long;
__device__ __forceinline__ f2 pk(float lo, float hi) {
  f2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void upk(f2 r, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(r));
}
__device__ __forceinline__ f2 mul2(f2 a, f2 b) {
  f2 d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f2 add2(f2 a, f2 b) {
  f2 d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f2 sub2(f2 a, f2 b) {
  f2 d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f2 fma2(f2 a, f2 b, f2 c) {
  f2 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// Markstein division (see markstein_div) on two lanes at once; ns = -s.
__device__ __forceinline__ f2 markstein_div2(f2 n, f2 ns, f2 y) {
  f2 q = mul2(n, y);
  f2 r = fma2(ns, q, n);
  q = fma2(r, y, q);
  r = fma2(ns, q, n);
  return fma2(r, y, q);
}

__device__ __forceinline__ bool num_ok(float n) {
  const float a = fabsf(n);
  return a >= kNumMin && a <= kNumMax;
}

// Two adjacent elements of a chunk pair as fp32 (word w of the 2V elements
// a ++ b) and back, rounding to nearest even on the way back.
template <typename T, int V>
__device__ __forceinline__ void get2(const Chunk<T, V>& a, const Chunk<T, V>& b, int w, float& lo,
                                     float& hi) {
  const Chunk<T, V>& c = w < V / 2 ? a : b;
  const int i = 2 * (w < V / 2 ? w : w - V / 2);
  lo = Elem<T>::to_f32(c.e[i]);
  hi = Elem<T>::to_f32(c.e[i + 1]);
}
template <typename T, int V>
__device__ __forceinline__ void put2(Chunk<T, V>& a, Chunk<T, V>& b, int w, float lo, float hi) {
  Chunk<T, V>& c = w < V / 2 ? a : b;
  const int i = 2 * (w < V / 2 ? w : w - V / 2);
  if constexpr (sizeof(T) == 2) {
    uint32_t packed;
    if constexpr (std::is_same<T, __nv_bfloat16>::value)
      asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(packed) : "f"(hi), "f"(lo));
    else
      asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(packed) : "f"(hi), "f"(lo));
    *reinterpret_cast<uint32_t*>(&c.e[i]) = packed;
  } else {
    c.e[i] = Elem<T>::from_f32(lo);
    c.e[i + 1] = Elem<T>::from_f32(hi);
  }
}

// Rotate one unit's two chunks (a: first V elements, b: second) in place.
template <typename T, bool NEOX, int V>
__device__ __forceinline__ void rotate(Chunk<T, V>& a, Chunk<T, V>& b, const Trig<V>& tr,
                                       bool same) {
  if (same) return;  // old == new position: the reference stores the source values
  if constexpr (V % 2 == 0) {
#pragma unroll
    for (int k = 0; k < V / 2; ++k) {
      // Pairs 2k and 2k + 1 of the unit.  NEOX: x1 are elements 2k, 2k+1 of
      // a and x2 the same of b.  GPT-J: the pairs are elements (4k, 4k+1)
      // and (4k+2, 4k+3) of a ++ b.
      float x1l, x1h, x2l, x2h;
      if constexpr (NEOX) {
        get2(a, b, k, x1l, x1h);
        get2(a, b, V / 2 + k, x2l, x2h);
      } else {
        get2(a, b, 2 * k, x1l, x2l);
        get2(a, b, 2 * k + 1, x1h, x2h);
      }
      const int i = 2 * k;
      const f2 x1 = pk(x1l, x1h), x2 = pk(x2l, x2h);
      const f2 oc = pk(tr.oc[i], tr.oc[i + 1]), os = pk(tr.os[i], tr.os[i + 1]);
      // Sums of two rounded products are formed as fma(p, +-1, q) with the
      // 1 known only at run time: RN(p * 1 + q) is exactly RN(p + q), and
      // the assembler cannot fold a single-use packed product into an FMA
      // with the other product, which it otherwise does for f32x2 add/sub
      // despite the .rn modifier (the fused result differs in the last bit).
      const f2 one = pk(tr.one, tr.one), mone = pk(-tr.one, -tr.one);
      const f2 n1 = fma2(mul2(x1, oc), one, mul2(x2, os));
      const f2 n2 = fma2(mul2(x1, os), mone, mul2(x2, oc));
      float n1l, n1h, n2l, n2h;
      upk(n1, n1l, n1h);
      upk(n2, n2l, n2h);
      f2 u1, u2;
      if (tr.scale_ok && num_ok(n1l) && num_ok(n1h) && num_ok(n2l) && num_ok(n2h)) {
        const f2 ns = pk(-tr.sc[i], -tr.sc[i + 1]), y = pk(tr.rc[i], tr.rc[i + 1]);
        u1 = markstein_div2(n1, ns, y);
        u2 = markstein_div2(n2, ns, y);
      } else {
        u1 = pk(__fdiv_rn(n1l, tr.sc[i]), __fdiv_rn(n1h, tr.sc[i + 1]));
        u2 = pk(__fdiv_rn(n2l, tr.sc[i]), __fdiv_rn(n2h, tr.sc[i + 1]));
      }
      const f2 nc = pk(tr.nc[i], tr.nc[i + 1]), nsn = pk(tr.ns[i], tr.ns[i + 1]);
      const f2 y1 = fma2(mul2(u2, nsn), mone, mul2(u1, nc));
      const f2 y2 = fma2(mul2(u2, nc), one, mul2(u1, nsn));
      float y1l, y1h, y2l, y2h;
      upk(y1, y1l, y1h);
      upk(y2, y2l, y2h);
      if constexpr (NEOX) {
        put2(a, b, k, y1l, y1h);
        put2(a, b, V / 2 + k, y2l, y2h);
      } else {
        put2(a, b, 2 * k, y1l, y2l);
        put2(a, b, 2 * k + 1, y1h, y2h);
      }
    }
    return;
  }
  float x[2 * V];
#pragma unroll
  for (int i = 0; i < V; ++i) {
    x[i] = Elem<T>::to_f32(a.e[i]);
    x[V + i] = Elem<T>::to_f32(b.e[i]);
  }
  float y[2 * V];
#pragma unroll
  for (int i = 0; i < V; ++i) {
    // NEOX pairs (i, half + i) -> (x[i], x[V + i]); GPT-J pairs (2i, 2i + 1)
    // of the 2V contiguous elements.
    const int i1 = NEOX ? i : 2 * i;
    const int i2 = NEOX ? V + i : 2 * i + 1;
    const float x1 = x[i1], x2 = x[i2];
    const float n1 = __fadd_rn(__fmul_rn(x1, tr.oc[i]), __fmul_rn(x2, tr.os[i]));
    const float n2 = __fsub_rn(__fmul_rn(x2, tr.oc[i]), __fmul_rn(x1, tr.os[i]));
    float u1, u2;
    div2_rn(n1, n2, tr.sc[i], tr.rc[i], tr.scale_ok, u1, u2);
    y[i1] = __fsub_rn(__fmul_rn(u1, tr.nc[i]), __fmul_rn(u2, tr.ns[i]));
    y[i2] = __fadd_rn(__fmul_rn(u2, tr.nc[i]), __fmul_rn(u1, tr.ns[i]));
  }
#pragma unroll
  for (int i = 0; i < V; ++i) {
    a.e[i] = Elem<T>::from_f32(y[i]);
    b.e[i] = Elem<T>::from_f32(y[V + i]);
  }
}

struct UnitGeom {
  long long ks, kd, vs, vd;  // element offsets of the (slot, head) rows
  int o1, o2;                // offsets of the unit's two chunks in the head row
  int chunk, chunks, tail_vecs, copy_vecs;
  bool in_place, same;
};

// Element offset of copy vector c (K tail first, then V) and its table.
__device__ __forceinline__ long long copy_src(const UnitGeom& g, int c, int rot, int V) {
  return c < g.tail_vecs ? g.ks + rot + (long long)c * V : g.vs + (long long)(c - g.tail_vecs) * V;
}
__device__ __forceinline__ long long copy_dst(const UnitGeom& g, int c, int rot, int V) {
  return c < g.tail_vecs ? g.kd + rot + (long long)c * V : g.vd + (long long)(c - g.tail_vecs) * V;
}

// Unpipelined walk over the layers (element path, misaligned layers, or a
// copy-on-write that moves more than two vectors per unit and layer).
template <typename T, bool NEOX, int V>
__device__ void unit_direct(const RepositionParams& p, const unsigned long long* s_k,
                            const unsigned long long* s_v, const bool* s_vec, const UnitGeom& g,
                            const Trig<V>& tr, int l0, int l1) {
  for (int l = l0; l < l1; ++l) {
    T* kb = reinterpret_cast<T*>(s_k[l]);
    Chunk<T, V> a, b;
    a.load(kb + g.ks + g.o1, s_vec[l]);
    b.load(kb + g.ks + g.o2, s_vec[l]);
    rotate<T, NEOX, V>(a, b, tr, g.same);
    a.store(kb + g.kd + g.o1, s_vec[l]);
    b.store(kb + g.kd + g.o2, s_vec[l]);
    if (!g.in_place) {
      T* vb = reinterpret_cast<T*>(s_v[l]);
      for (int c = g.chunk; c < g.copy_vecs; c += g.chunks) {
        T* base = c < g.tail_vecs ? kb : vb;
        Chunk<T, V> t;
        t.load(base + copy_src(g, c, p.rotary_dim, V), s_vec[l]);
        t.store(base + copy_dst(g, c, p.rotary_dim, V), s_vec[l]);
      }
    }
  }
}

// Pipelined walk: S layers in flight, NV staged 16-byte vectors per layer
// (2 = the K pair; 4 = the K pair plus two copy vectors).  The first S-1
// layers are requested before the unit's cos/sin values are loaded, so the
// two memory round trips overlap.
template <typename T, typename C, bool NEOX, int V, int S, int NV>
__device__ void unit_pipelined(const RepositionParams& p, const unsigned long long* s_k,
                               const unsigned long long* s_v, uint32_t stage, const UnitGeom& g,
                               long long po, long long pn, int j, int l0, int l1) {
  static_assert(S * NV <= kSlots, "staging slots");
  constexpr uint32_t kSlotStride = kThreads * 16;
  const int c0 = g.chunk, c1 = g.chunk + g.chunks;
  auto issue = [&](int l) {
    const T* kb = reinterpret_cast<const T*>(s_k[l]);
    const uint32_t base = stage + (uint32_t)((l % S) * NV) * kSlotStride;
    cp_async16(base, kb + g.ks + g.o1);
    cp_async16(base + kSlotStride, kb + g.ks + g.o2);
    if constexpr (NV == 4) {
      const T* vb = reinterpret_cast<const T*>(s_v[l]);
      if (c0 < g.copy_vecs)
        cp_async16(base + 2 * kSlotStride,
                   (c0 < g.tail_vecs ? kb : vb) + copy_src(g, c0, p.rotary_dim, V));
      if (c1 < g.copy_vecs)
        cp_async16(base + 3 * kSlotStride,
                   (c1 < g.tail_vecs ? kb : vb) + copy_src(g, c1, p.rotary_dim, V));
    }
  };
#pragma unroll
  for (int i = 0; i < S - 1; ++i) {
    if (l0 + i < l1) issue(l0 + i);
    cp_async_commit();
  }
  Trig<V> tr;
  load_trig<C, V>(p, po, pn, j, tr);
  for (int l = l0; l < l1; ++l) {
    if (l + S - 1 < l1) issue(l + S - 1);
    cp_async_commit();
    cp_async_wait<S - 1>();
    const uint32_t base = stage + (uint32_t)((l % S) * NV) * kSlotStride;
    Chunk<T, V> a, b;
    a.load_shared(base);
    b.load_shared(base + kSlotStride);
    rotate<T, NEOX, V>(a, b, tr, g.same);
    T* kb = reinterpret_cast<T*>(s_k[l]);
    a.store(kb + g.kd + g.o1, true);
    b.store(kb + g.kd + g.o2, true);
    if constexpr (NV == 4) {
      T* vb = reinterpret_cast<T*>(s_v[l]);
      if (c0 < g.copy_vecs) {
        Chunk<T, V> t;
        t.load_shared(base + 2 * kSlotStride);
        t.store((c0 < g.tail_vecs ? kb : vb) + copy_dst(g, c0, p.rotary_dim, V), true);
      }
      if (c1 < g.copy_vecs) {
        Chunk<T, V> t;
        t.load_shared(base + 3 * kSlotStride);
        t.store((c1 < g.tail_vecs ? kb : vb) + copy_dst(g, c1, p.rotary_dim, V), true);
      }
    }
  }
  cp_async_wait<0>();
}

template <typename T, typename C, bool NEOX, int V>
__global__ void __launch_bounds__(kThreads, AKV_REPOSITION_MIN_BLOCKS)
reposition_kernel(const RepositionParams p) {
  constexpr bool kVector = V * sizeof(T) == 16;
  extern __shared__ __align__(16) unsigned char stage_smem[];
  __shared__ unsigned long long s_k[kMaxLayers];
  __shared__ unsigned long long s_v[kMaxLayers];
  __shared__ bool s_vec[kMaxLayers];
  __shared__ int s_all_vec;
  pdl_wait();  // transitions and their count may come from the kernel before
  if (threadIdx.x == 0) s_all_vec = 1;
  __syncthreads();
  for (int i = threadIdx.x; i < p.n_layers; i += blockDim.x) {
    s_k[i] = p.k_ptrs[i];
    s_v[i] = p.v_ptrs[i];
    s_vec[i] = ((s_k[i] | s_v[i]) & (V * sizeof(T) - 1)) == 0;
    if (!s_vec[i]) s_all_vec = 0;
  }
  __syncthreads();
  const bool all_vec = kVector && s_all_vec;
  // The staging slots start on a 128-byte boundary.  Dynamic shared memory
  // follows the static tables above at only 16-byte alignment, and a warp's
  // cp.async whose 512-byte shared destination is not 128-byte aligned
  // makes the L1 request 24 instead of 16 global sectors (measured on the
  // c2 shape: 58% more L2 read sectors, 8% longer kernel).
  const uint32_t stage =
      ((static_cast<uint32_t>(__cvta_generic_to_shared(stage_smem)) + 127u) & ~127u) +
      threadIdx.x * 16;

  long long count = p.count;
  if (p.count_dev != nullptr) {
    const long long c = *p.count_dev;
    count = c < count ? c : count;
  }
  UnitGeom g;
  g.chunks = p.half / V;  // units per head
  const int upt = p.num_heads * g.chunks;
  const long long total = count * upt;
  // Vectors of V elements per head that a copy moves: K tail then all of V.
  g.tail_vecs = (p.head_dim - p.rotary_dim) / V;
  g.copy_vecs = g.tail_vecs + p.head_dim / V;
  const bool cow_pipelined = g.copy_vecs <= 2 * g.chunks;

  // Work is split over warps as equal spans of (warp unit, layer) pairs, a
  // warp unit being 32 consecutive units (the lanes of a warp).  A span
  // covers a few warp units, the first and last possibly over part of the
  // layers; every (unit, layer) row belongs to exactly one span.  Giving
  // each thread whole units over all layers left a partial last wave when
  // units are few (one KV head per GPU: 1.37 units per resident thread ran
  // as two rounds).
  const int n_layers = p.n_layers;
  const long long warp_units = (total + 31) >> 5;
  const long long n_warps = (long long)gridDim.x * (blockDim.x >> 5);
  const long long warp = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const long long work = warp_units * n_layers;
  const long long per = work / n_warps, rest = work % n_warps;
  long long pos = warp * per + (warp < rest ? warp : rest);
  const long long end = pos + per + (warp < rest ? 1 : 0);
  while (pos < end) {
    const long long wu = pos / n_layers;
    const int l0 = (int)(pos - wu * n_layers);
    const int l1 = end - pos < n_layers - l0 ? l0 + (int)(end - pos) : n_layers;
    pos += l1 - l0;
    const long long u = (wu << 5) + (threadIdx.x & 31);
    if (u >= total) continue;
    const long long tok = u / upt;
    const int rem = (int)(u - tok * upt);
    const int head = rem / g.chunks;
    g.chunk = rem - head * g.chunks;
    const long long src = __ldg(p.src + tok);
    const long long dst = __ldg(p.dst + tok);
    if (p.skip_unmapped && (src <= 0 || dst <= 0)) continue;
    const long long po = __ldg(p.pairs + tok * p.pstride);
    const long long pn = __ldg(p.pairs + tok * p.pstride + 1);
    if ((p.num_slots > 0 && (src < 0 || dst < 0 || src >= p.num_slots || dst >= p.num_slots)) ||
        (p.max_position > 0 && (po < 0 || pn < 0 || po >= p.max_position || pn >= p.max_position))) {
      if (p.error_flag != nullptr) atomicOr(p.error_flag, 1);
      continue;
    }
    g.same = po == pn;
    g.in_place = src == dst;
    if (g.same && g.in_place) continue;  // rewriting identical bits: nothing to do

    const int j = g.chunk * V;  // first pair of this unit
    g.o1 = NEOX ? j : 2 * j;
    g.o2 = NEOX ? p.half + j : 2 * j + V;
    g.ks = src * p.k_ss + head * p.k_sh;
    g.kd = dst * p.k_ss + head * p.k_sh;
    g.vs = src * p.v_ss + head * p.v_sh;
    g.vd = dst * p.v_ss + head * p.v_sh;

    if constexpr (kVector) {
      // In place, or a copy whose V rows the move kernel carries: only the
      // K pair of the unit moves (rotated into the destination row).
      if (all_vec && (g.in_place || (p.v_moved && g.tail_vecs == 0))) {
        unit_pipelined<T, C, NEOX, V, 8, 2>(p, s_k, s_v, stage, g, po, pn, j, l0, l1);
        continue;
      }
      if (all_vec && cow_pipelined) {
        unit_pipelined<T, C, NEOX, V, 4, 4>(p, s_k, s_v, stage, g, po, pn, j, l0, l1);
        continue;
      }
    }
    Trig<V> tr;
    load_trig<C, V>(p, po, pn, j, tr);
    unit_direct<T, NEOX, V>(p, s_k, s_v, s_vec, g, tr, l0, l1);
  }
}

// ---------------------------------------------------------------------------
// V rows of copy-on-write transitions, moved by the TMA engine.
//
// For a copy (source != destination) the whole V row of a token over the
// local heads -- num_heads * head_dim contiguous elements when heads are
// contiguous in the [slot, head, dim] pool -- moves unchanged.  Here one
// thread per warp (a "mover") streams such rows through a ring of
// kMoveSlots row buffers in its own shared memory: a 1-D bulk copy global ->
// shared completes on the slot's mbarrier (bounded wait), then a 1-D bulk
// copy shared -> global writes the destination row, and a slot is refilled
// only after the store that read it has finished reading
// (cp.async.bulk.wait_group.read).  No register or thread touches the data.
// All addresses are this GPU's own pools; no cluster multicast.
// Work: mover m takes transitions m, m + M, m + 2M, ... (M movers in the
// grid), each with all its layers, so that copies clustered in the list
// (a request's shared prefix) spread over every mover; in-place, skipped
// and out-of-range transitions are passed over whole (the main kernel
// reports the latter).
constexpr int kMoveWarps = 8;
constexpr int kMoveSlots = 8;
constexpr int kMoveAhead = kMoveSlots - 2;  // loads in flight; the store two rows back is read
constexpr int kMaxMoveRow = 2048;           // bytes: 8 heads x 128 dims x 2 B
constexpr unsigned long long kMoveWaitNs = 100000000ull;  // 100 ms per row

__device__ __forceinline__ bool move_bar_wait(uint32_t bar, uint32_t parity) {
  auto done = [&]() {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
  };
  if (done()) return true;
  unsigned long long t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (;;) {
    if (done()) return true;
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (t - t0 > kMoveWaitNs) return false;
  }
}

__global__ void __launch_bounds__(kMoveWarps * 32) reposition_v_move_kernel(
    const RepositionParams p, int row_bytes) {
  extern __shared__ __align__(128) unsigned char move_smem[];
  __shared__ __align__(8) unsigned long long move_bars[kMoveWarps][kMoveSlots];
  pdl_wait();  // transitions and their count may come from the kernel before
  pdl_launch_dependents();
  const int warp = threadIdx.x >> 5;
  if ((threadIdx.x & 31) != 0) return;  // one thread per mover
  long long count = p.count;
  if (p.count_dev != nullptr) {
    const long long c = *p.count_dev;
    count = c < count ? c : count;
  }
  const long long movers = (long long)gridDim.x * kMoveWarps;
  long long tr = (long long)blockIdx.x * kMoveWarps + warp;  // this mover's current transition
  int layer = 0;                                             // its next layer
  long long tr_src = 0, tr_dst = 0;

  const uint32_t slots = (uint32_t)__cvta_generic_to_shared(move_smem) +
                         (uint32_t)(warp * kMoveSlots * row_bytes);
  const uint32_t bars = (uint32_t)__cvta_generic_to_shared(&move_bars[warp][0]);
  for (int s = 0; s < kMoveSlots; ++s)
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bars + 8 * s));
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");

  unsigned long long dst_of[kMoveSlots];
  uint32_t parity = 0;  // bit s: parity of slot s's next completion
  long long issued = 0, done = 0;
  // The next row of this mover: source and destination addresses.
  auto next_row = [&](unsigned long long& src, unsigned long long& dst) -> bool {
    while (tr < count) {
      if (layer == 0) {  // a new transition: is it a copy to move?
        tr_src = __ldg(p.src + tr);
        tr_dst = __ldg(p.dst + tr);
        const bool skip =
            tr_src == tr_dst || (p.skip_unmapped && (tr_src <= 0 || tr_dst <= 0)) ||
            (p.num_slots > 0 &&
             (tr_src < 0 || tr_dst < 0 || tr_src >= p.num_slots || tr_dst >= p.num_slots));
        if (skip) {
          tr += movers;
          continue;
        }
      }
      const unsigned long long vb = __ldg(p.v_ptrs + layer);
      src = vb + (unsigned long long)(tr_src * p.v_ss) * 2ull;
      dst = vb + (unsigned long long)(tr_dst * p.v_ss) * 2ull;
      if (++layer == p.n_layers) {
        layer = 0;
        tr += movers;
      }
      if (((src | dst) & 15ull) == 0) return true;  // misaligned layer: the main kernel moves it
    }
    return false;
  };
  auto load = [&](unsigned long long src, unsigned long long dst) {
    const int s = (int)(issued % kMoveSlots);
    const uint32_t bar = bars + 8 * s, buf = slots + (uint32_t)(s * row_bytes);
    dst_of[s] = dst;
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
                 "r"(row_bytes)
                 : "memory");
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, "
        "[%3];" ::"r"(buf),
        "l"(src), "r"(row_bytes), "r"(bar)
        : "memory");
    ++issued;
  };
  unsigned long long src, dst;
  while (issued < kMoveAhead && next_row(src, dst)) load(src, dst);
  bool failed = false;
  while (done < issued) {
    const int s = (int)(done % kMoveSlots);
    if (!move_bar_wait(bars + 8 * s, (parity >> s) & 1u)) {
      failed = true;
      break;
    }
    parity ^= 1u << s;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst_of[s]),
                 "r"(slots + (uint32_t)(s * row_bytes)), "r"(row_bytes)
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    ++done;
    if (next_row(src, dst)) {
      // The slot to fill last held row issued - kMoveSlots, whose store is
      // older than the newest kMoveSlots - kMoveAhead stores.
      asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(kMoveSlots - kMoveAhead) : "memory");
      load(src, dst);
    }
  }
  if (failed) {
    if (p.error_flag != nullptr) atomicOr(p.error_flag, 2);
    // The loads still in flight land in this CTA's shared memory: wait for
    // each (bounded) before the CTA leaves.
    for (long long k = done; k < issued; ++k) {
      const int s = (int)(k % kMoveSlots);
      if (move_bar_wait(bars + 8 * s, (parity >> s) & 1u)) parity ^= 1u << s;
    }
  }
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

template <typename T, typename C, bool NEOX, int V>
int launch(const RepositionParams& p, cudaStream_t stream) {
  auto kernel = reposition_kernel<T, C, NEOX, V>;
  // + 128 bytes of alignment slack; the element path stages nothing.
  constexpr int smem = (V * sizeof(T) == 16) ? kStageBytes + 128 : 0;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
      cudaSuccess)
    return AKV_ERR_CUDA;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, smem) !=
          cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  // Enough warps for spans of at least kMinSpan layers (so the per-thread
  // pipeline still has layers in flight), at most one wave.
  constexpr long long kMinSpan = 8;
  const long long units = p.count * (long long)p.num_heads * (p.half / V);
  const long long spans = ((units + 31) / 32 * p.n_layers + kMinSpan - 1) / kMinSpan;
  const long long blocks = (spans + kThreads / 32 - 1) / (kThreads / 32);
  const int grid = persistent_grid(per_sm, blocks);
  if (p.v_moved) {
    // Copy-on-write V rows by bulk copies, then the K rotation; both are
    // programmatic dependent launches (each waits for its predecessor).
    const int row_bytes = p.num_heads * p.head_dim * (int)sizeof(T);
    const int move_smem = kMoveWarps * kMoveSlots * row_bytes;
    if (cudaFuncSetAttribute(reposition_v_move_kernel,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, move_smem) != cudaSuccess)
      return AKV_ERR_CUDA;
    int move_per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&move_per_sm, reposition_v_move_kernel,
                                                      kMoveWarps * 32, move_smem) != cudaSuccess ||
        move_per_sm < 1)
      move_per_sm = 1;
    const int move_grid = persistent_grid(move_per_sm, (p.count + kMoveWarps - 1) / kMoveWarps);
    if (launch_pdl(reposition_v_move_kernel, move_grid, kMoveWarps * 32, move_smem, stream, p,
                   row_bytes) != cudaSuccess)
      return AKV_ERR_CUDA;
  }
  if (launch_pdl(kernel, grid, kThreads, smem, stream, p) != cudaSuccess) return AKV_ERR_CUDA;
  return launch_status();
}

template <typename T, typename C>
int dispatch_style(const RepositionParams& p, bool neox, bool vec, cudaStream_t s) {
  constexpr int VV = 16 / sizeof(T);
  if (vec) return neox ? launch<T, C, true, VV>(p, s) : launch<T, C, false, VV>(p, s);
  return neox ? launch<T, C, true, 1>(p, s) : launch<T, C, false, 1>(p, s);
}

template <typename T>
int dispatch_cache(const RepositionParams& p, int cache_dtype, bool cache_rows, bool neox,
                   bool vec, cudaStream_t s) {
  switch (cache_dtype) {
    case AKV_F32:
      if (cache_rows && vec) {
        constexpr int VV = 16 / sizeof(T);
        return neox ? launch<T, F32Rows, true, VV>(p, s) : launch<T, F32Rows, false, VV>(p, s);
      }
      return dispatch_style<T, float>(p, neox, vec, s);
    case AKV_BF16: return dispatch_style<T, __nv_bfloat16>(p, neox, vec, s);
    case AKV_F16: return dispatch_style<T, __half>(p, neox, vec, s);
  }
  return AKV_ERR_INVALID;
}

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

extern "C" int akv_reposition_kv_layers_ex(
    const void* k_data_ptrs, const void* v_data_ptrs, int32_t n_layers, int32_t kv_dtype,
    int32_t num_heads, int32_t head_dim, int32_t rotary_dim, int64_t k_stride_slot,
    int64_t k_stride_head, int64_t v_stride_slot, int64_t v_stride_head,
    const int32_t* source_slots, const int32_t* destination_slots,
    const int32_t* position_pairs, int64_t position_stride, int64_t count,
    const int32_t* count_device, const void* cos_sin_cache, int32_t cache_dtype,
    int64_t cache_stride, int32_t is_neox_style, int32_t skip_unmapped, int64_t num_slots,
    int64_t max_position, int32_t* error_flag, int32_t options, void* stream) {
  AKV_NVTX_RANGE("akv_reposition_kv_layers");
  using namespace akv;
  if (options & ~AKV_REPOSITION_BULK_V) return AKV_ERR_INVALID;
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
  p.one = 1.0f;
  p.v_moved = 0;
  const bool cache_rows = cache_dtype == AKV_F32 &&
                          (reinterpret_cast<uintptr_t>(cos_sin_cache) & 15) == 0 &&
                          cache_stride % 4 == 0 && p.half % 4 == 0;

  const int esize = kv_dtype == AKV_F32 ? 4 : 2;
  const int V = 16 / esize;
  // The 16-byte path needs every vector to start on a 16-byte boundary:
  // shapes and strides are checked here, each layer's base address in the
  // kernel (a misaligned layer sends the launch to element accesses).
  const bool vec = (p.half % V == 0) && (head_dim % V == 0) && (rotary_dim % V == 0) &&
                   (k_stride_slot % V == 0) && (k_stride_head % V == 0) &&
                   (v_stride_slot % V == 0) && (v_stride_head % V == 0);
  const bool neox = is_neox_style != 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // With AKV_REPOSITION_BULK_V, copy-on-write V rows go through the
  // bulk-copy move kernel when a token's V row over the local heads is one
  // contiguous run of 16-byte multiples and K has no tail to copy
  // (rotary_dim == head_dim); otherwise the main kernel moves them.
  const long long v_row = (long long)num_heads * head_dim * esize;
  p.v_moved = (options & AKV_REPOSITION_BULK_V) && vec && esize == 2 &&
              rotary_dim == head_dim && v_stride_head == head_dim && v_row % 16 == 0 &&
              v_row <= kMaxMoveRow && v_stride_slot % 8 == 0;
  switch (kv_dtype) {
    case AKV_F32: return dispatch_cache<float>(p, cache_dtype, cache_rows, neox, vec, s);
    case AKV_BF16: return dispatch_cache<__nv_bfloat16>(p, cache_dtype, cache_rows, neox, vec, s);
    case AKV_F16: return dispatch_cache<__half>(p, cache_dtype, cache_rows, neox, vec, s);
  }
  return AKV_ERR_INVALID;
}

extern "C" int akv_reposition_kv_layers(
    const void* k_data_ptrs, const void* v_data_ptrs, int32_t n_layers, int32_t kv_dtype,
    int32_t num_heads, int32_t head_dim, int32_t rotary_dim, int64_t k_stride_slot,
    int64_t k_stride_head, int64_t v_stride_slot, int64_t v_stride_head,
    const int32_t* source_slots, const int32_t* destination_slots,
    const int32_t* position_pairs, int64_t position_stride, int64_t count,
    const int32_t* count_device, const void* cos_sin_cache, int32_t cache_dtype,
    int64_t cache_stride, int32_t is_neox_style, int32_t skip_unmapped, int64_t num_slots,
    int64_t max_position, int32_t* error_flag, void* stream) {
  return akv_reposition_kv_layers_ex(
      k_data_ptrs, v_data_ptrs, n_layers, kv_dtype, num_heads, head_dim, rotary_dim,
      k_stride_slot, k_stride_head, v_stride_slot, v_stride_head, source_slots,
      destination_slots, position_pairs, position_stride, count, count_device, cos_sin_cache,
      cache_dtype, cache_stride, is_neox_style, skip_unmapped, num_slots, max_position,
      error_flag, 0, stream);
}

extern "C" int akv_reposition_divide(const float* numerators, const float* denominators,
                                     float* quotients, int64_t count, int32_t method,
                                     void* stream) {
  AKV_NVTX_RANGE("akv_reposition_divide");
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
