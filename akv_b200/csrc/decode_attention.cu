// Paged GQA decode attention over the compacted cache, with learned sinks.
//
// Replaces the native decode kernels the reference calls over the registry's
// kv_indptr / kv_indices (FlashInfer BatchDecodeWithPagedKVCacheWrapper and
// FA3 flash_attn_with_kvcache, not vendored), together with AKV's sink
// correction o *= sigmoid(lse - sink) (akv/system/sglang.patch:2170-2183,
// srt/layers/attention/context_backend.py:254-272), which here is folded into
// the softmax denominator: out = sum_k e^{s_k} v_k / (sum_k e^{s_k} + e^{sink}).
// Sliding-window layers read only the window the metadata builder selected
// (context_page_table.py:7-31), so this kernel needs no position mask.
//
// Decode attention reads every key once (8 flop per byte for a GQA group of
// 8) -- an HBM-bound stream.  Layout of the work:
//  * one CTA = one (request, key range) work item, all KV heads of the
//    request; warp w owns KV head w and its GROUP = 8 query heads;
//  * a key's K row (and V row) for all local heads is one contiguous
//    Hkv*D*2-byte run in the [slot, head, dim] pool; NSTAGE stages of TK keys
//    are gathered into shared memory with 16-byte cp.async (zero-filled
//    past the range end), XOR-swizzled by key so ldmatrix is conflict-free;
//  * tensor cores (mma.sync m16n8k16 bf16, fp32 accumulate) with KEYS as the
//    M dimension: S^T[16 keys x 8 heads] = K[16 x D] . Q^T[D x 8], so the
//    8-head group fills N = 8 exactly and no MMA row is padding; then
//    O^T[D x 8] += V^T[D x 16] . P^T[16 x 8], with P^T produced from the S^T
//    accumulator fragment by movmatrix (an in-register 8x8 transpose);
//  * fp32 online softmax in base 2; per-head state lives in the lanes that
//    hold that head's O^T columns, so rescaling is thread-local;
//  * long requests are split into several items whose partial (m, l, acc)
//    a second kernel combines; single-item requests write bf16 directly.

#include "attention_common.cuh"

namespace akv {
namespace {

constexpr int kGroup = 8;  // query heads per KV head (the MMA N)

// 16-key stages, two of them, for every head count: 64 KiB of shared memory
// for 8 KV heads of 64 dims (three CTAs per SM), proportionally less -- and
// more CTAs per SM -- when tensor parallelism leaves fewer heads per GPU.
// Measured on the c4 full layer (random slots): 8 heads 0.578 ms; 4 heads
// 0.333 ms, 2 heads 0.190 ms and 1 head 0.130 ms with the row-wise gather
// (below); 32-key stages (0.744 ms at 4 heads with the per-key split) and
// 3 or 4 stages were no better.  Also slower for 8 heads: 2 CTAs x 3 stages,
// 1 CTA x 32-key stages, per-warp rings (a key's 1 KiB row then reaches
// DRAM as eight separate 128-byte requests) and a warp-specialised variant
// with one cp.async.bulk per row and an mbarrier ring.
constexpr int kTileKeys = 16;
constexpr int kStages = 2;

struct AttnParams {
  const __nv_bfloat16* q;
  long long q_sb, q_sh;  // strides of q [batch, q_heads, D] in elements
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  long long k_ss, k_sh, v_ss, v_sh;
  long long num_slots;
  const int* kv_indices;
  const float* sinks;  // [q_heads] natural-log logits, or null
  float scale_log2;    // sm_scale * log2(e)
  const int4* work;    // {request, kv_begin, kv_end, partial or -1}
  const int* cta_items;  // [ctas + 1] per-CTA item lists, or null (one item per CTA)
  float* part_acc;     // [partials, q_heads, D]
  float* part_ml;      // [partials, q_heads, 2] (max in base 2, sum)
  __nv_bfloat16* out;
  long long o_sb, o_sh;
  float* lse;          // [batch, q_heads] natural log, or null
  int num_q_heads;
  int* error_flag;
};

template <int D, int HKV, int TK, int NSTAGE>
struct Cfg {
  static constexpr int kThreads = 32 * HKV;
  static constexpr int kCph = D / 8;               // 16-byte chunks per head row
  static constexpr int kChunks = HKV * kCph;       // chunks per key row
  static constexpr int kRowBytes = kChunks * 16;
  static constexpr int kTileBytes = TK * kRowBytes;
  static constexpr int kStageBytes = 2 * kTileBytes;  // K then V
  static constexpr int kSmem = NSTAGE * kStageBytes;
};

// One work item: a key range of one request, all KV heads.  Called by every
// thread of the CTA; it leaves no copy in flight and ends on a barrier, so
// the next item may reuse the shared-memory stages at once.
template <int D, int HKV, int TK, int NSTAGE>
__device__ __forceinline__ void attend_item(const AttnParams& p, const int4 w,
                                            unsigned char* smem) {
  using C = Cfg<D, HKV, TK, NSTAGE>;
  static_assert(D % 16 == 0 && D >= 64, "head_dim must be a multiple of 16, at least 64");
  static_assert(TK % 16 == 0, "key tile is a whole number of 16-key MMA blocks");
  const int b = w.x, kv_begin = w.y, kv_end = w.z, partial = w.w;
  const int n_keys = kv_end - kv_begin;
  const int n_tiles = (n_keys + TK - 1) / TK;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;

  // Gather of a tile's K and V rows into shared memory, kCpt 16-byte chunks
  // per thread for each.  At eight local heads each thread copies chunks of
  // one key (16 threads, 256 contiguous bytes of its 1 KiB row per warp
  // request), so it needs one index per tile.  With fewer heads that split
  // would leave a warp request 32-128 bytes of each of 16 different rows;
  // there the chunks are dealt row-wise instead (consecutive threads take
  // consecutive chunks of one key, so a request covers whole 128-byte lines
  // and, at four heads, a key's whole 512-byte row) and each thread needs
  // the index of the kCpt keys it serves.  Either way the indices are
  // loaded a tile ahead, so the copies never wait on their own address.
  // Measured on random slots: 1 / 2 / 4 heads 0.310 / 0.347 / 0.380 ms per
  // c4 full layer with the per-key split, 0.130 / 0.190 / 0.333 row-wise.
  constexpr int kTpk = C::kThreads / TK;        // threads per key
  constexpr int kCpt = C::kChunks / kTpk;       // chunks per thread (K, and as many of V)
  static_assert(C::kThreads % TK == 0 && C::kChunks % kTpk == 0, "tile split");
  constexpr bool kRowWise = kTpk < 16;
  static_assert(!kRowWise || C::kThreads % C::kChunks == 0, "row-wise split");
  constexpr int kKpr = kRowWise ? C::kThreads / C::kChunks : 1;  // keys per row-wise round
  constexpr int kNS = kRowWise ? kCpt : 1;                         // indices per thread
  const int my_key = tid / kTpk, my_q = tid - my_key * kTpk;
  const int my_c = kRowWise ? tid % C::kChunks : 0;  // row-wise: this thread's chunk
  // Tile-local key of index i of this thread.
  auto key_of = [&](int i) { return kRowWise ? i * kKpr + tid / C::kChunks : my_key; };
  struct Slots { long long v[kNS]; };
  // Slots of this thread's keys in `tile`, -1 past the range end.
  auto fetch_slot = [&](int tile) {
    Slots r;
#pragma unroll
    for (int i = 0; i < kNS; ++i) {
      const int kk = kv_begin + tile * TK + key_of(i);
      long long slot = -1;
      if (tile < n_tiles && kk < kv_end) {
        slot = __ldg(p.kv_indices + kk);
        if (slot < 0 || slot >= p.num_slots) {  // never touch memory outside the pools
          if (p.error_flag) *p.error_flag = 1;
          slot = 0;
        }
      }
      r.v[i] = slot;
    }
    return r;
  };
  auto issue_tile = [&](int s, const Slots& slots) {
    const uint32_t kbase = smem_u32(smem + s * C::kStageBytes);
    const uint32_t vbase = kbase + C::kTileBytes;
#pragma unroll
    for (int i = 0; i < kCpt; ++i) {
      const long long slot = slots.v[kRowWise ? i : 0];
      const bool valid = slot >= 0;
      const long long sl = valid ? slot : 0;
      const int bytes = valid ? 16 : 0;  // zero-fill past the range end
      const int key = key_of(i);
      const int c = kRowWise ? my_c : my_q + kTpk * i;
      const int head = c / C::kCph, cc = c - head * C::kCph;
      const int phys = head * C::kCph + (cc ^ (key & 7));
      const uint32_t off = key * C::kRowBytes + phys * 16;
      cp_async16(kbase + off, p.k + sl * p.k_ss + head * p.k_sh + cc * 8, bytes);
      cp_async16(vbase + off, p.v + sl * p.v_ss + head * p.v_sh + cc * 8, bytes);
    }
  };

#pragma unroll
  for (int s = 0; s < NSTAGE - 1; ++s) {
    if (s < n_tiles) issue_tile(s, fetch_slot(s));
    cp_async_commit();
  }
  Slots next_slot = fetch_slot(NSTAGE - 1);

  // Q^T fragments of this warp's 8 query heads (B operand, k = dims).
  const int qh0 = warp * kGroup;
  uint32_t qf[D / 16][2];
  {
    const __nv_bfloat16* qrow = p.q + (long long)b * p.q_sb + (long long)(qh0 + g) * p.q_sh;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      qf[ks][0] = *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 2 * t);
      qf[ks][1] = *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 8 + 2 * t);
    }
  }

  float m[2] = {-INFINITY, -INFINITY};  // running max (base 2) of heads 2t, 2t+1
  float l[2] = {0.f, 0.f};              // this lane's share of the running sum
  float acc[D / 16][4];
#pragma unroll
  for (int mt = 0; mt < D / 16; ++mt)
#pragma unroll
    for (int r = 0; r < 4; ++r) acc[mt][r] = 0.f;

  for (int tile = 0; tile < n_tiles; ++tile) {
    const int nt = tile + NSTAGE - 1;
    if (nt < n_tiles) {
      issue_tile(nt % NSTAGE, next_slot);
      next_slot = fetch_slot(nt + 1);
    }
    cp_async_commit();
    cp_async_wait<NSTAGE - 1>();
    __syncthreads();

    const unsigned char* stage = smem + (tile % NSTAGE) * C::kStageBytes;
    const uint32_t kb = smem_u32(stage);
    const uint32_t vb = kb + C::kTileBytes;
    const int key0 = tile * TK;

#pragma unroll
    for (int blk = 0; blk < TK / 16; ++blk) {
      // ---- S^T = K . Q^T for 16 keys ----
      float s[4] = {0.f, 0.f, 0.f, 0.f};
      {
        const int key = blk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const int cc = ks * 2 + (lane >> 4);
          const uint32_t addr =
              kb + key * C::kRowBytes + (warp * C::kCph + (cc ^ (key & 7))) * 16;
          uint32_t a0, a1, a2, a3;
          ldmatrix_x4(addr, a0, a1, a2, a3);
          mma_bf16(s, a0, a1, a2, a3, qf[ks][0], qf[ks][1]);
        }
      }
      // keys g and g + 8 of this block; mask past the item's end
      const int kg0 = key0 + blk * 16 + g, kg1 = kg0 + 8;
      s[0] = kg0 < n_keys ? s[0] * p.scale_log2 : -INFINITY;
      s[1] = kg0 < n_keys ? s[1] * p.scale_log2 : -INFINITY;
      s[2] = kg1 < n_keys ? s[2] * p.scale_log2 : -INFINITY;
      s[3] = kg1 < n_keys ? s[3] * p.scale_log2 : -INFINITY;

      // ---- online softmax, heads 2t (s0, s2) and 2t+1 (s1, s3) ----
      float bm0 = fmaxf(s[0], s[2]), bm1 = fmaxf(s[1], s[3]);
#pragma unroll
      for (int x = 4; x < 32; x <<= 1) {
        bm0 = fmaxf(bm0, __shfl_xor_sync(0xffffffffu, bm0, x));
        bm1 = fmaxf(bm1, __shfl_xor_sync(0xffffffffu, bm1, x));
      }
      const float mn0 = fmaxf(m[0], bm0), mn1 = fmaxf(m[1], bm1);
      const float base0 = mn0 == -INFINITY ? 0.f : mn0;
      const float base1 = mn1 == -INFINITY ? 0.f : mn1;
      const float al0 = fast_exp2(m[0] - base0), al1 = fast_exp2(m[1] - base1);
      m[0] = mn0;
      m[1] = mn1;
      const float p0 = fast_exp2(s[0] - base0), p1 = fast_exp2(s[1] - base1);
      const float p2 = fast_exp2(s[2] - base0), p3 = fast_exp2(s[3] - base1);
      l[0] = l[0] * al0 + p0 + p2;
      l[1] = l[1] * al1 + p1 + p3;
#pragma unroll
      for (int mt = 0; mt < D / 16; ++mt) {
        acc[mt][0] *= al0;
        acc[mt][1] *= al1;
        acc[mt][2] *= al0;
        acc[mt][3] *= al1;
      }

      // ---- O^T += V^T . P^T ----
      const uint32_t pb0 = movmatrix_trans(pack_bf16(p0, p1));  // keys 0-7
      const uint32_t pb1 = movmatrix_trans(pack_bf16(p2, p3));  // keys 8-15
      {
        const int mj = lane >> 3;
        const int key = blk * 16 + (lane & 7) + ((mj >> 1) & 1) * 8;
#pragma unroll
        for (int mt = 0; mt < D / 16; ++mt) {
          const int cc = mt * 2 + (mj & 1);
          const uint32_t addr =
              vb + key * C::kRowBytes + (warp * C::kCph + (cc ^ (key & 7))) * 16;
          uint32_t a0, a1, a2, a3;
          ldmatrix_x4_trans(addr, a0, a1, a2, a3);
          mma_bf16(acc[mt], a0, a1, a2, a3, pb0, pb1);
        }
      }
    }
    __syncthreads();  // the stage is refilled NSTAGE - 1 tiles later
  }
  cp_async_wait<0>();

  // ---- epilogue ----
#pragma unroll
  for (int x = 4; x < 32; x <<= 1) {
    l[0] += __shfl_xor_sync(0xffffffffu, l[0], x);
    l[1] += __shfl_xor_sync(0xffffffffu, l[1], x);
  }
  const int h0 = qh0 + 2 * t, h1 = h0 + 1;
  if (partial >= 0) {
    float* pa = p.part_acc + (long long)partial * p.num_q_heads * D;
#pragma unroll
    for (int mt = 0; mt < D / 16; ++mt) {
      const int d0 = mt * 16 + g, d1 = d0 + 8;
      pa[(long long)h0 * D + d0] = acc[mt][0];
      pa[(long long)h1 * D + d0] = acc[mt][1];
      pa[(long long)h0 * D + d1] = acc[mt][2];
      pa[(long long)h1 * D + d1] = acc[mt][3];
    }
    if (g == 0) {
      float* pm = p.part_ml + (long long)partial * p.num_q_heads * 2;
      pm[2 * h0] = m[0];
      pm[2 * h0 + 1] = l[0];
      pm[2 * h1] = m[1];
      pm[2 * h1 + 1] = l[1];
    }
    return;
  }
  float den0 = l[0], den1 = l[1];
  const float mb0 = m[0] == -INFINITY ? 0.f : m[0];
  const float mb1 = m[1] == -INFINITY ? 0.f : m[1];
  if (p.sinks) {
    den0 += fast_exp2(p.sinks[h0] * kLog2e - mb0);
    den1 += fast_exp2(p.sinks[h1] * kLog2e - mb1);
  }
  const float inv0 = den0 > 0.f ? 1.f / den0 : 0.f;
  const float inv1 = den1 > 0.f ? 1.f / den1 : 0.f;
  __nv_bfloat16* o = p.out + (long long)b * p.o_sb;
#pragma unroll
  for (int mt = 0; mt < D / 16; ++mt) {
    const int d0 = mt * 16 + g, d1 = d0 + 8;
    o[(long long)h0 * p.o_sh + d0] = __float2bfloat16_rn(acc[mt][0] * inv0);
    o[(long long)h1 * p.o_sh + d0] = __float2bfloat16_rn(acc[mt][1] * inv1);
    o[(long long)h0 * p.o_sh + d1] = __float2bfloat16_rn(acc[mt][2] * inv0);
    o[(long long)h1 * p.o_sh + d1] = __float2bfloat16_rn(acc[mt][3] * inv1);
  }
  if (p.lse && g == 0) {
    // natural-log LSE of [scores | sink] (the sink-corrected value,
    // context_backend.py:269-271); -inf for an empty key set without sink.
    p.lse[(long long)b * p.num_q_heads + h0] = den0 > 0.f ? (mb0 + log2f(den0)) * kLn2 : -INFINITY;
    p.lse[(long long)b * p.num_q_heads + h1] = den1 > 0.f ? (mb1 + log2f(den1)) * kLn2 : -INFINITY;
  }
}

// One CTA per work item, or -- with cta_items -- a persistent CTA that runs
// its list of items [cta_items[c], cta_items[c+1]) one after another (the
// host balances the lists, so no CTA is left with a long tail).
template <int D, int HKV, int TK, int NSTAGE>
__global__ void __launch_bounds__(32 * HKV)
decode_attention_kernel(const AttnParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  if (p.cta_items == nullptr) {
    attend_item<D, HKV, TK, NSTAGE>(p, p.work[blockIdx.x], smem);
    return;
  }
  const int i1 = p.cta_items[blockIdx.x + 1];
  for (int i = p.cta_items[blockIdx.x]; i < i1; ++i)
    attend_item<D, HKV, TK, NSTAGE>(p, p.work[i], smem);
}

// Combine the partial results of split requests.  Block (request, head
// group): one warp per query head.  The warp first turns the splits' maxima
// into per-split weights 2^(m_i - M) (kept in shared memory) and the
// denominator, then each lane sums its D/32 output dims over the splits
// with loads that are contiguous across the warp.
constexpr int kCombineHeads = 8;     // warps (query heads) per block
constexpr int kCombineMaxSplits = 512;

template <int D>
__global__ void __launch_bounds__(32 * kCombineHeads)
decode_combine_kernel(const AttnParams p, const int2* merge, int batch) {
  __shared__ float weight[kCombineHeads][kCombineMaxSplits];
  const int b = blockIdx.x;
  const int2 mg = merge[b];  // {first partial, count}; count 0 = written directly
  if (mg.y == 0) return;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int h = blockIdx.y * kCombineHeads + w;
  if (h >= p.num_q_heads) return;
  const int n = mg.y;
  float mx = -INFINITY;
  for (int s = lane; s < n; s += 32)
    mx = fmaxf(mx, p.part_ml[((long long)(mg.x + s) * p.num_q_heads + h) * 2]);
#pragma unroll
  for (int x = 16; x > 0; x >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, x));
  const float base = mx == -INFINITY ? 0.f : mx;
  float den = 0.f;
  for (int s = lane; s < n; s += 32) {
    const long long q = (long long)(mg.x + s) * p.num_q_heads + h;
    const float f = fast_exp2(p.part_ml[2 * q] - base);
    weight[w][s] = f;
    den += p.part_ml[2 * q + 1] * f;
  }
#pragma unroll
  for (int x = 16; x > 0; x >>= 1) den += __shfl_xor_sync(0xffffffffu, den, x);
  __syncwarp();
  if (p.sinks) den += fast_exp2(p.sinks[h] * kLog2e - base);
  const float inv = den > 0.f ? 1.f / den : 0.f;
  constexpr int kPer = D / 32;
  float num[kPer];
#pragma unroll
  for (int k = 0; k < kPer; ++k) num[k] = 0.f;
  const float* acc = p.part_acc + ((long long)mg.x * p.num_q_heads + h) * D + lane;
  const long long split_stride = (long long)p.num_q_heads * D;
  for (int s = 0; s < n; ++s) {
    const float f = weight[w][s];
#pragma unroll
    for (int k = 0; k < kPer; ++k) num[k] += acc[s * split_stride + 32 * k] * f;
  }
  __nv_bfloat16* o = p.out + (long long)b * p.o_sb + (long long)h * p.o_sh + lane;
#pragma unroll
  for (int k = 0; k < kPer; ++k) o[32 * k] = __float2bfloat16_rn(num[k] * inv);
  if (p.lse && lane == 0)
    p.lse[(long long)b * p.num_q_heads + h] = den > 0.f ? (base + log2f(den)) * kLn2 : -INFINITY;
}

// Keys per stage and stages (see kTileKeys).
template <int D, int HKV> struct Pick {
  static constexpr int TK = kTileKeys;
  static constexpr int NSTAGE = kStages;
  using C = Cfg<D, HKV, TK, NSTAGE>;
};

// Resident CTAs per SM of the kernel for this shape (the persistent grid).
template <int D, int HKV>
int ctas_per_sm() {
  using P = Pick<D, HKV>;
  auto kernel = decode_attention_kernel<D, HKV, P::TK, P::NSTAGE>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, P::C::kSmem) !=
      cudaSuccess)
    return -AKV_ERR_CUDA;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, P::C::kThreads, P::C::kSmem) !=
      cudaSuccess)
    return -AKV_ERR_CUDA;
  return n;
}

template <int D, int HKV>
int launch_attention(const AttnParams& p, int n_items, int n_ctas, const int2* merge,
                     int batch, cudaStream_t s) {
  using P = Pick<D, HKV>;
  using C = typename P::C;
  auto kernel = decode_attention_kernel<D, HKV, P::TK, P::NSTAGE>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem) !=
      cudaSuccess)
    return AKV_ERR_CUDA;
  const int grid = p.cta_items != nullptr ? n_ctas : n_items;
  if (n_items > 0 && grid > 0) kernel<<<grid, C::kThreads, C::kSmem, s>>>(p);
  if (merge != nullptr && batch > 0) {
    const dim3 grid(batch, (p.num_q_heads + kCombineHeads - 1) / kCombineHeads);
    decode_combine_kernel<D><<<grid, 32 * kCombineHeads, 0, s>>>(p, merge, batch);
  }
  return launch_status();
}

template <int D>
int dispatch_heads(const AttnParams& p, int hkv, int n_items, int n_ctas, const int2* merge,
                   int batch, cudaStream_t s) {
  switch (hkv) {
    case 1: return launch_attention<D, 1>(p, n_items, n_ctas, merge, batch, s);
    case 2: return launch_attention<D, 2>(p, n_items, n_ctas, merge, batch, s);
    case 4: return launch_attention<D, 4>(p, n_items, n_ctas, merge, batch, s);
    case 8: return launch_attention<D, 8>(p, n_items, n_ctas, merge, batch, s);
  }
  return AKV_ERR_UNSUPPORTED;
}

}  // namespace
}  // namespace akv

extern "C" int akv_decode_attention(
    const void* q, int64_t q_stride_batch, int64_t q_stride_head, const void* k_pool,
    const void* v_pool, int64_t k_stride_slot, int64_t k_stride_head, int64_t v_stride_slot,
    int64_t v_stride_head, int64_t num_slots, const int32_t* kv_indices, const float* sinks,
    float sm_scale, int32_t batch, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
    const int32_t* work, int32_t n_items, const int32_t* cta_items, int32_t n_ctas,
    const int32_t* merge, float* partial_acc,
    float* partial_ml, void* out, int64_t out_stride_batch, int64_t out_stride_head, float* lse,
    int32_t* error_flag, void* stream) {
  AKV_NVTX_RANGE("akv_decode_attention");
  using namespace akv;
  if (batch < 0 || n_items < 0 || (cta_items != nullptr && n_ctas < 0) || num_kv_heads <= 0 ||
      num_q_heads != num_kv_heads * kGroup ||
      !q || !k_pool || !v_pool || !kv_indices || !work || !out || num_slots <= 0)
    return AKV_ERR_INVALID;
  if ((q_stride_head % 2) || (reinterpret_cast<uintptr_t>(q) & 3) ||
      (reinterpret_cast<uintptr_t>(k_pool) & 15) || (reinterpret_cast<uintptr_t>(v_pool) & 15) ||
      (k_stride_slot % 8) || (k_stride_head % 8) || (v_stride_slot % 8) || (v_stride_head % 8))
    return AKV_ERR_INVALID;  // 16-byte cp.async rows and 4-byte q pairs
  AttnParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.q_sb = q_stride_batch;
  p.q_sh = q_stride_head;
  p.k = static_cast<const __nv_bfloat16*>(k_pool);
  p.v = static_cast<const __nv_bfloat16*>(v_pool);
  p.k_ss = k_stride_slot;
  p.k_sh = k_stride_head;
  p.v_ss = v_stride_slot;
  p.v_sh = v_stride_head;
  p.num_slots = num_slots;
  p.kv_indices = kv_indices;
  p.sinks = sinks;
  p.scale_log2 = sm_scale * kLog2e;
  p.work = reinterpret_cast<const int4*>(work);
  p.cta_items = cta_items;
  p.part_acc = partial_acc;
  p.part_ml = partial_ml;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.o_sb = out_stride_batch;
  p.o_sh = out_stride_head;
  p.lse = lse;
  p.num_q_heads = num_q_heads;
  p.error_flag = error_flag;
  const int2* mg = reinterpret_cast<const int2*>(merge);
  if (mg != nullptr && (!partial_acc || !partial_ml)) return AKV_ERR_INVALID;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (head_dim) {
    case 64: return dispatch_heads<64>(p, num_kv_heads, n_items, n_ctas, mg, batch, s);
    case 128: return dispatch_heads<128>(p, num_kv_heads, n_items, n_ctas, mg, batch, s);
  }
  return AKV_ERR_UNSUPPORTED;
}

extern "C" int32_t akv_decode_attention_ctas_per_sm(int32_t num_kv_heads, int32_t head_dim) {
  using namespace akv;
  switch (head_dim * 16 + num_kv_heads) {
    case 64 * 16 + 1: return ctas_per_sm<64, 1>();
    case 64 * 16 + 2: return ctas_per_sm<64, 2>();
    case 64 * 16 + 4: return ctas_per_sm<64, 4>();
    case 64 * 16 + 8: return ctas_per_sm<64, 8>();
    case 128 * 16 + 1: return ctas_per_sm<128, 1>();
    case 128 * 16 + 2: return ctas_per_sm<128, 2>();
    case 128 * 16 + 4: return ctas_per_sm<128, 4>();
    case 128 * 16 + 8: return ctas_per_sm<128, 8>();
  }
  return -AKV_ERR_UNSUPPORTED;
}
