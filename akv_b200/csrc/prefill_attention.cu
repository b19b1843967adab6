// Ragged prefill (extend) attention over the compacted cache, with the
// context positions AKV keeps after Drop / Reposition.
//
// Replaces the native ragged prefill the reference runs after each layer's
// KV write and copy-on-write (ContextAttentionMetadata.forward and
// native_plan, srt/layers/attention/context_backend.py:184-241; the
// position-aware extend kernel of akv/system/sglang.patch:106-237), and the
// sink correction of flash_attention_with_sink (context_backend.py:244-272),
// folded into the softmax denominator.
//
// Request b has P_b prefix keys (surviving context tokens: slots
// kv_indices[kv_indptr[b] ..], positions kv_positions[..]) followed by its
// Q_b new tokens (slots birth_slots[qo_indptr[b] ..], positions
// q_positions[..]), whose K/V the caller has already written to the pool.
// Query i of the request sees prefix key j when q_pos - k_pos <= window
// (window < 0: always) and new-token key j when j <= i and the same window
// condition holds -- the reference's mask: causal over the new tokens,
// sliding window by position (patch :524-541, :725-741).  Positions may have
// holes (dropped tokens), so the window is a position test, not an index
// test, and no host gather is needed for gapped segments.
//
// Layout: a CTA owns 16 queries x the 8 query heads of one KV head
// (128 rows; warp w: queries 2w and 2w+1, rows = (query, head)), so every
// K/V tile loaded from HBM serves the whole GQA group.  Tensor cores:
// mma.sync m16n8k16 bf16 with fp32 accumulation, S = Q K^T then O += P V,
// P reused from the S accumulators in registers; online softmax in base 2.
// K/V rows of the KV head (head_dim * 2 bytes per key) are gathered by
// 16-byte cp.async into a 3-stage, XOR-swizzled shared-memory ring.

#include "attention_common.cuh"

namespace akv {
namespace {

constexpr int kGroupP = 8;    // query heads per KV head
constexpr int kQBlock = 16;   // queries per CTA
constexpr int kWarpsP = 8;    // 2 queries x 8 heads = 16 MMA rows per warp
constexpr int kThreadsP = 32 * kWarpsP;
constexpr int kTK = 64;       // keys per stage
constexpr int kStagesP = 3;

struct PrefillParams {
  const __nv_bfloat16* q;
  long long q_st, q_sh;  // strides of q [tokens, q_heads, D]
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  long long k_ss, k_sh, v_ss, v_sh;
  long long num_slots;
  const int* qo_indptr;     // [batch + 1]
  const int* kv_indptr;     // [batch + 1] prefix keys
  const int* kv_indices;    // prefix slots
  const int* birth_slots;   // [tokens] slots of the new tokens' K/V
  const int* q_positions;   // [tokens]
  const int* kv_positions;  // prefix positions
  const int4* work;         // {request, first query (request-local), key_lo, key_hi}
  const float* sinks;       // [q_heads] natural-log logits, or null
  float scale_log2;
  int window;               // < 0: no sliding window
  __nv_bfloat16* out;
  long long o_st, o_sh;
  float* lse;               // [tokens, q_heads] natural log, or null
  int num_q_heads;
  int* error_flag;
};

template <int D>
struct PCfg {
  static constexpr int kCph = D / 8;          // 16-byte chunks per key row (one KV head)
  static constexpr int kRowBytes = D * 2;
  static constexpr int kTileBytes = kTK * kRowBytes;
  static constexpr int kStageBytes = 2 * kTileBytes + kTK * 4;  // K, V, key positions
  static constexpr int kSmem = kStagesP * kStageBytes;
  static constexpr int kTpk = kThreadsP / kTK;  // threads per key
  static constexpr int kCpt = kCph / kTpk;      // chunks per thread (K, and as many of V)
};

template <int D>
__global__ void __launch_bounds__(kThreadsP, D <= 64 ? 2 : 1)  // head_dim 64: two CTAs per SM
prefill_attention_kernel(const PrefillParams p) {
  using C = PCfg<D>;
  static_assert(D % 16 == 0 && C::kCph % C::kTpk == 0, "head_dim split");
  extern __shared__ __align__(128) unsigned char smem[];
  const int4 w = p.work[blockIdx.x];
  const int hk = blockIdx.y;  // KV head
  const int b = w.x, qb0 = w.y, key_lo = w.z, key_hi = w.w;
  const int qo0 = p.qo_indptr[b], nq_req = p.qo_indptr[b + 1] - qo0;
  const int kv0 = p.kv_indptr[b], n_prefix = p.kv_indptr[b + 1] - kv0;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int n_keys = key_hi - key_lo;
  const int n_tiles = (n_keys + kTK - 1) / kTK;

  // Key j of the request: prefix first, then the new tokens.
  auto key_slot_pos = [&](int j, long long& slot, int& pos) {
    if (j < n_prefix) {
      slot = __ldg(p.kv_indices + kv0 + j);
      pos = __ldg(p.kv_positions + kv0 + j);
    } else {
      slot = __ldg(p.birth_slots + qo0 + (j - n_prefix));
      pos = __ldg(p.q_positions + qo0 + (j - n_prefix));
    }
    if (slot < 0 || slot >= p.num_slots) {  // never touch memory outside the pools
      if (p.error_flag) *p.error_flag = 1;
      slot = 0;
    }
  };
  // Each thread gathers kCpt chunks of one key per tile; that key's slot and
  // position are loaded a tile ahead, so the copies never wait on them.
  const int my_key = tid / C::kTpk, my_q = tid - my_key * C::kTpk;
  struct KeyRef {
    long long slot;
    int pos;  // INT_MAX past the range end
  };
  auto fetch = [&](int tile) -> KeyRef {
    KeyRef r{0, INT_MAX};
    const int j = key_lo + tile * kTK + my_key;
    if (tile < n_tiles && j < key_hi) key_slot_pos(j, r.slot, r.pos);
    return r;
  };
  auto issue_tile = [&](int stage, const KeyRef r) {
    unsigned char* st = smem + stage * C::kStageBytes;
    const uint32_t kbase = smem_u32(st), vbase = kbase + C::kTileBytes;
    int* kpos = reinterpret_cast<int*>(st + 2 * C::kTileBytes);
    const bool valid = r.pos != INT_MAX;
    const long long slot = r.slot;
    if (my_q == 0) kpos[my_key] = r.pos;
    const int bytes = valid ? 16 : 0;  // zero-fill past the range end
#pragma unroll
    for (int i = 0; i < C::kCpt; ++i) {
      const int c = my_q + C::kTpk * i;
      const uint32_t off = my_key * C::kRowBytes + ((c ^ (my_key & 7)) * 16);
      cp_async16(kbase + off, p.k + slot * p.k_ss + hk * p.k_sh + c * 8, bytes);
      cp_async16(vbase + off, p.v + slot * p.v_ss + hk * p.v_sh + c * 8, bytes);
    }
  };

#pragma unroll
  for (int s = 0; s < kStagesP - 1; ++s) {
    if (s < n_tiles) issue_tile(s, fetch(s));
    cp_async_commit();
  }
  KeyRef next = fetch(kStagesP - 1);

  // This warp's rows: query qa = qb0 + 2 * warp (row g = head g) and qa + 1
  // (row g + 8).  Q fragments straight from global memory.
  const int qa = qb0 + 2 * warp, qb = qa + 1;
  const bool va = qa < nq_req, vb = qb < nq_req;
  const int head = hk * kGroupP + g;
  uint32_t qf[D / 16][4];
  {
    const __nv_bfloat16* ra = p.q + (long long)(qo0 + (va ? qa : 0)) * p.q_st + head * p.q_sh;
    const __nv_bfloat16* rb = p.q + (long long)(qo0 + (vb ? qb : 0)) * p.q_st + head * p.q_sh;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      qf[ks][0] = va ? *reinterpret_cast<const uint32_t*>(ra + ks * 16 + 2 * t) : 0u;
      qf[ks][1] = vb ? *reinterpret_cast<const uint32_t*>(rb + ks * 16 + 2 * t) : 0u;
      qf[ks][2] = va ? *reinterpret_cast<const uint32_t*>(ra + ks * 16 + 8 + 2 * t) : 0u;
      qf[ks][3] = vb ? *reinterpret_cast<const uint32_t*>(rb + ks * 16 + 8 + 2 * t) : 0u;
    }
  }
  // Positions are non-negative int32, so q_pos - k_pos cannot overflow.
  const int pa = va ? __ldg(p.q_positions + qo0 + qa) : 0;
  const int pb = vb ? __ldg(p.q_positions + qo0 + qb) : 0;
  // Birth keys a query may see: indices up to its own (j - n_prefix <= q).
  const int ja = n_prefix + qa, jb = n_prefix + qb;
  // Position of the CTA's newest query (the window test of a whole tile).
  const int q_last_pos = __ldg(p.q_positions + qo0 + min(qb0 + kQBlock, nq_req) - 1);

  float m[2] = {-INFINITY, -INFINITY};  // rows g (query qa) and g + 8 (query qb)
  float l[2] = {0.f, 0.f};
  float acc[D / 8][4];
#pragma unroll
  for (int n = 0; n < D / 8; ++n)
#pragma unroll
    for (int r = 0; r < 4; ++r) acc[n][r] = 0.f;

  for (int tile = 0; tile < n_tiles; ++tile) {
    const int nt = tile + kStagesP - 1;
    if (nt < n_tiles) {
      issue_tile(nt % kStagesP, next);
      next = fetch(nt + 1);
    }
    cp_async_commit();
    cp_async_wait<kStagesP - 1>();
    __syncthreads();

    const unsigned char* st = smem + (tile % kStagesP) * C::kStageBytes;
    const uint32_t kb = smem_u32(st), vbs = kb + C::kTileBytes;
    const int* kpos = reinterpret_cast<const int*>(st + 2 * C::kTileBytes);
    const int j0 = key_lo + tile * kTK;

    // ---- S = Q K^T: 8 n-tiles of 8 keys ----
    float s[kTK / 8][4];
#pragma unroll
    for (int n = 0; n < kTK / 8; ++n)
#pragma unroll
      for (int r = 0; r < 4; ++r) s[n][r] = 0.f;
#pragma unroll
    for (int np = 0; np < kTK / 16; ++np) {  // pairs of n-tiles (16 keys)
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        const int mtx = lane >> 3;
        const int key = np * 16 + ((mtx >> 1) << 3) + (lane & 7);
        const int chunk = ks * 2 + (mtx & 1);
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4(kb + key * C::kRowBytes + ((chunk ^ (key & 7)) * 16), b0, b1, b2, b3);
        mma_bf16(s[2 * np], qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3], b0, b1);
        mma_bf16(s[2 * np + 1], qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3], b2, b3);
      }
    }

    // ---- mask, scale, online softmax (rows g: qa, g + 8: qb) ----
    // A tile whose every key is visible to every query of the CTA (all keys
    // live, none after the first query's own token, the oldest key inside
    // the newest query's window) skips the per-element mask.
    const bool tile_full = j0 + kTK <= key_hi && j0 + kTK - 1 <= n_prefix + qb0 &&
                           (p.window < 0 || q_last_pos - kpos[0] <= p.window);
    float bm0 = -INFINITY, bm1 = -INFINITY;
    if (tile_full) {
#pragma unroll
      for (int n = 0; n < kTK / 8; ++n) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          s[n][e] *= p.scale_log2;
          s[n][2 + e] *= p.scale_log2;
          bm0 = fmaxf(bm0, s[n][e]);
          bm1 = fmaxf(bm1, s[n][2 + e]);
        }
      }
    } else {
#pragma unroll
      for (int n = 0; n < kTK / 8; ++n) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int kk = n * 8 + 2 * t + e;
          const int j = j0 + kk;
          const int kp = kpos[kk];
          const bool live = j < key_hi;
          const bool ok_a = va && live && (j < n_prefix || j <= ja) &&
                            (p.window < 0 || pa - kp <= p.window);
          const bool ok_b = vb && live && (j < n_prefix || j <= jb) &&
                            (p.window < 0 || pb - kp <= p.window);
          s[n][e] = ok_a ? s[n][e] * p.scale_log2 : -INFINITY;
          s[n][2 + e] = ok_b ? s[n][2 + e] * p.scale_log2 : -INFINITY;
          bm0 = fmaxf(bm0, s[n][e]);
          bm1 = fmaxf(bm1, s[n][2 + e]);
        }
      }
    }
#pragma unroll
    for (int x = 1; x < 4; x <<= 1) {
      bm0 = fmaxf(bm0, __shfl_xor_sync(0xffffffffu, bm0, x));
      bm1 = fmaxf(bm1, __shfl_xor_sync(0xffffffffu, bm1, x));
    }
    const float mn0 = fmaxf(m[0], bm0), mn1 = fmaxf(m[1], bm1);
    const float base0 = mn0 == -INFINITY ? 0.f : mn0;
    const float base1 = mn1 == -INFINITY ? 0.f : mn1;
    const float al0 = fast_exp2(m[0] - base0), al1 = fast_exp2(m[1] - base1);
    m[0] = mn0;
    m[1] = mn1;
    float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
    for (int n = 0; n < kTK / 8; ++n) {
      s[n][0] = fast_exp2(s[n][0] - base0);
      s[n][1] = fast_exp2(s[n][1] - base0);
      s[n][2] = fast_exp2(s[n][2] - base1);
      s[n][3] = fast_exp2(s[n][3] - base1);
      rs0 += s[n][0] + s[n][1];
      rs1 += s[n][2] + s[n][3];
    }
    l[0] = l[0] * al0 + rs0;
    l[1] = l[1] * al1 + rs1;
#pragma unroll
    for (int n = 0; n < D / 8; ++n) {
      acc[n][0] *= al0;
      acc[n][1] *= al0;
      acc[n][2] *= al1;
      acc[n][3] *= al1;
    }

    // ---- O += P V: P from the S accumulators, V^T fragments by ldmatrix.trans ----
    // P goes in as two bf16 terms, hi = RN(P) and lo = RN(P - hi), so the
    // weights carry about 16 significant bits: with a short window a query
    // averages only a few values, and a single bf16 P would leave errors
    // near 2^-9 of |v| in the output.
#pragma unroll
    for (int kk = 0; kk < kTK / 16; ++kk) {
      uint32_t hi[4], lo[4];
      split_bf16(s[2 * kk][0], s[2 * kk][1], hi[0], lo[0]);
      split_bf16(s[2 * kk][2], s[2 * kk][3], hi[1], lo[1]);
      split_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1], hi[2], lo[2]);
      split_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3], hi[3], lo[3]);
#pragma unroll
      for (int dc = 0; dc < D / 16; ++dc) {  // pairs of 8-dim output tiles
        const int mtx = lane >> 3;
        const int key = kk * 16 + ((mtx & 1) << 3) + (lane & 7);
        const int chunk = dc * 2 + (mtx >> 1);
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(vbs + key * C::kRowBytes + ((chunk ^ (key & 7)) * 16), b0, b1, b2,
                          b3);
        mma_bf16(acc[2 * dc], hi[0], hi[1], hi[2], hi[3], b0, b1);
        mma_bf16(acc[2 * dc + 1], hi[0], hi[1], hi[2], hi[3], b2, b3);
        mma_bf16(acc[2 * dc], lo[0], lo[1], lo[2], lo[3], b0, b1);
        mma_bf16(acc[2 * dc + 1], lo[0], lo[1], lo[2], lo[3], b2, b3);
      }
    }
    __syncthreads();  // the stage is refilled kStagesP - 1 tiles later
  }
  cp_async_wait<0>();

  // ---- epilogue: quad sums, sinks, normalise, store ----
#pragma unroll
  for (int x = 1; x < 4; x <<= 1) {
    l[0] += __shfl_xor_sync(0xffffffffu, l[0], x);
    l[1] += __shfl_xor_sync(0xffffffffu, l[1], x);
  }
  float den0 = l[0], den1 = l[1];
  const float mb0 = m[0] == -INFINITY ? 0.f : m[0];
  const float mb1 = m[1] == -INFINITY ? 0.f : m[1];
  if (p.sinks) {
    const float sk = p.sinks[head] * kLog2e;
    den0 += fast_exp2(sk - mb0);
    den1 += fast_exp2(sk - mb1);
  }
  const float inv0 = den0 > 0.f ? 1.f / den0 : 0.f;
  const float inv1 = den1 > 0.f ? 1.f / den1 : 0.f;
  if (va) {
    __nv_bfloat16* o = p.out + (long long)(qo0 + qa) * p.o_st + head * p.o_sh;
#pragma unroll
    for (int n = 0; n < D / 8; ++n)
      *reinterpret_cast<uint32_t*>(o + n * 8 + 2 * t) =
          pack_bf16(acc[n][0] * inv0, acc[n][1] * inv0);
    if (p.lse && t == 0)
      p.lse[(long long)(qo0 + qa) * p.num_q_heads + head] =
          den0 > 0.f ? (mb0 + log2f(den0)) * kLn2 : -INFINITY;
  }
  if (vb) {
    __nv_bfloat16* o = p.out + (long long)(qo0 + qb) * p.o_st + head * p.o_sh;
#pragma unroll
    for (int n = 0; n < D / 8; ++n)
      *reinterpret_cast<uint32_t*>(o + n * 8 + 2 * t) =
          pack_bf16(acc[n][2] * inv1, acc[n][3] * inv1);
    if (p.lse && t == 0)
      p.lse[(long long)(qo0 + qb) * p.num_q_heads + head] =
          den1 > 0.f ? (mb1 + log2f(den1)) * kLn2 : -INFINITY;
  }
}

template <int D>
int launch_prefill(const PrefillParams& p, int n_items, int num_kv_heads, cudaStream_t s) {
  using C = PCfg<D>;
  auto kernel = prefill_attention_kernel<D>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem) !=
      cudaSuccess)
    return AKV_ERR_CUDA;
  if (n_items > 0) kernel<<<dim3(n_items, num_kv_heads), kThreadsP, C::kSmem, s>>>(p);
  return launch_status();
}

}  // namespace
}  // namespace akv

extern "C" int64_t akv_context_attention_query_block(void) { return akv::kQBlock; }

extern "C" int akv_context_attention(
    const void* q, int64_t q_stride_token, int64_t q_stride_head, const void* k_pool,
    const void* v_pool, int64_t k_stride_slot, int64_t k_stride_head, int64_t v_stride_slot,
    int64_t v_stride_head, int64_t num_slots, const int32_t* qo_indptr, const int32_t* kv_indptr,
    const int32_t* kv_indices, const int32_t* birth_slots, const int32_t* q_positions,
    const int32_t* kv_positions, const float* sinks, float sm_scale, int64_t window,
    int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, const int32_t* work,
    int32_t n_items, void* out, int64_t out_stride_token, int64_t out_stride_head, float* lse,
    int32_t* error_flag, void* stream) {
  using namespace akv;
  if (n_items < 0 || num_kv_heads <= 0 || num_q_heads != num_kv_heads * kGroupP ||
      num_kv_heads > 65535 || num_slots <= 0)
    return AKV_ERR_INVALID;
  if (n_items == 0) return AKV_OK;
  if (!q || !k_pool || !v_pool || !qo_indptr || !kv_indptr || !birth_slots || !q_positions ||
      !work || !out)
    return AKV_ERR_INVALID;
  if ((q_stride_token % 2) || (q_stride_head % 2) || (out_stride_token % 2) ||
      (out_stride_head % 2) || (reinterpret_cast<uintptr_t>(q) & 3) ||
      (reinterpret_cast<uintptr_t>(out) & 3) || (reinterpret_cast<uintptr_t>(k_pool) & 15) ||
      (reinterpret_cast<uintptr_t>(v_pool) & 15) || (k_stride_slot % 8) ||
      (k_stride_head % 8) || (v_stride_slot % 8) || (v_stride_head % 8))
    return AKV_ERR_INVALID;  // 16-byte cp.async rows, 4-byte q / out pairs
  PrefillParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.q_st = q_stride_token;
  p.q_sh = q_stride_head;
  p.k = static_cast<const __nv_bfloat16*>(k_pool);
  p.v = static_cast<const __nv_bfloat16*>(v_pool);
  p.k_ss = k_stride_slot;
  p.k_sh = k_stride_head;
  p.v_ss = v_stride_slot;
  p.v_sh = v_stride_head;
  p.num_slots = num_slots;
  p.qo_indptr = qo_indptr;
  p.kv_indptr = kv_indptr;
  p.kv_indices = kv_indices;
  p.birth_slots = birth_slots;
  p.q_positions = q_positions;
  p.kv_positions = kv_positions;
  p.work = reinterpret_cast<const int4*>(work);
  p.sinks = sinks;
  p.scale_log2 = sm_scale * kLog2e;
  p.window = window < 0 ? -1 : (window > INT_MAX ? INT_MAX : (int)window);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.o_st = out_stride_token;
  p.o_sh = out_stride_head;
  p.lse = lse;
  p.num_q_heads = num_q_heads;
  p.error_flag = error_flag;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (head_dim) {
    case 64: return launch_prefill<64>(p, n_items, num_kv_heads, s);
    case 128: return launch_prefill<128>(p, n_items, num_kv_heads, s);
  }
  return AKV_ERR_UNSUPPORTED;
}
