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
  if (w.x < 0) return;  // padding item of a query-tile pair
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
      if (p.error_flag) atomicOr(p.error_flag, 1);
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

// ---------------------------------------------------------------------------
// 5th-generation tensor cores (tcgen05) for head_dim 64.
//
// Same work split (a CTA = 16 queries x 8 heads = 128 rows of one KV head)
// and the same mask, with the two GEMMs on tcgen05.mma and the accumulators
// in tensor memory (TMEM): thread r of the 128-thread CTA owns row r, which
// is TMEM lane r, so the softmax needs no shuffles.
//   S = Q K^T      kind::f16, M=128 N=64 K=64: A = Q, B = the K tile, both
//                  from shared memory (K-major, 128-byte swizzle);
//   O += P V       A = P from TMEM (hi and lo bf16 terms, two MMAs), B = the
//                  V tile from shared memory (MN-major, 128-byte swizzle).
// One thread issues the MMAs; tcgen05.commit arrives on an mbarrier that the
// CTA waits on (bounded: a wait that runs out sets error_flag and the CTA
// frees its TMEM and returns).  The row max is kept stale unless a tile
// raises it by more than 2^8, so O is rescaled in TMEM only then.
// Shared-memory tiles use the XOR swizzle chunk ^ (row & 7) on 128-byte rows
// from 1024-byte aligned bases, which is the canonical SWIZZLE_128B layout.
// ---------------------------------------------------------------------------
constexpr int kTcThreads = 256;   // two warps per 32 rows: one per column half
constexpr int kTcKeys = 64;
constexpr int kTcStages = 5;        // K/V tiles in flight: loads run 4 tiles ahead
constexpr int kTcCols = 256;          // TMEM columns per CTA (2 CTAs per SM)
constexpr int kColS = 0, kColPHi = 128, kColPLo = 160, kColO = 192;  // S: two buffers
constexpr int kTcQBytes = 128 * 128;  // Q tile: 128 rows x 64 bf16
constexpr int kTcKVBytes = kTcKeys * 128;
constexpr int kTcStageBytes = 2 * kTcKVBytes;
constexpr int kTcPosOff = kTcQBytes + kTcStages * kTcStageBytes;
constexpr int kTcRowOff = kTcPosOff + kTcStages * kTcKeys * 4;  // half-row max / sum
constexpr int kTcBarOff = kTcRowOff + 4 * 128 * 4;
// + alignment slack; at least 80 KB so that no more than two CTAs share an
// SM, which is all the tensor memory (2 x 256 columns) holds.
constexpr int kTcSmemUsed = kTcBarOff + 64 + 1024;
constexpr int kTcSmem = kTcSmemUsed > 80 * 1024 ? kTcSmemUsed : 80 * 1024;
constexpr float kStaleMax = 8.f;      // log2 headroom before O is rescaled
constexpr unsigned long long kWaitNs = 100000000ull;  // 100 ms per mbarrier wait

// Shared-memory matrix descriptor, 128-byte swizzle (UMMA canonical layout):
// start address >> 4, leading offset 16 B (unused for these shapes), stride
// offset 1024 B between 8-row groups, version 1, layout SWIZZLE_128B.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr) {
  return (uint64_t)((smem_addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) |
         ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// The same for an MN-major operand wider than one 64-element swizzle atom:
// lbo_bytes is the distance between consecutive atoms along MN.
__device__ __forceinline__ uint64_t sw128_desc_mn(uint32_t smem_addr, uint32_t lbo_bytes) {
  return (uint64_t)((smem_addr >> 4) & 0x3FFF) | ((uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16) |
         ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor, kind::f16: fp32 accumulate, bf16 A and B, A
// K-major, B K-major (b_mn = 0) or MN-major (1), M = 128, N.
__host__ __device__ constexpr uint32_t f16_idesc(int n, int b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)b_mn << 16) |
         ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                       uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                       uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_init(uint32_t bar, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait on an mbarrier phase (kWaitNs of wall time); false when it
// ran out.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  while (!mbar_try_wait(bar, parity))
    if (global_ns() - t0 > kWaitNs) return false;
  return true;
}
// TMEM access: each tcgen05.ld / tcgen05.st shares one asm statement with its
// tcgen05.wait, so the compiler never sees a destination (or source)
// register as settled while the asynchronous access is still in flight --
// a register spilled or reused in between would otherwise be written (or
// read) late.
__device__ __forceinline__ void tmem_ld32_sync(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31},"
      " [%32];\n\ttcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st32_sync(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
      "%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
      "\n\ttcgen05.wait::st.sync.aligned;" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
// One store of 16 columns (P's hi words alone) and its wait.
__device__ __forceinline__ void tmem_st16_sync(uint32_t ta, const uint32_t* a) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,"
      "%8,%9,%10,%11,%12,%13,%14,%15,%16};"
      "\n\ttcgen05.wait::st.sync.aligned;" ::"r"(ta),
      "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(a[4]), "r"(a[5]), "r"(a[6]), "r"(a[7]),
      "r"(a[8]), "r"(a[9]), "r"(a[10]), "r"(a[11]), "r"(a[12]), "r"(a[13]), "r"(a[14]),
      "r"(a[15])
      : "memory");
}
// Two stores of 16 columns (P's hi and lo words) and their wait.
__device__ __forceinline__ void tmem_st16x2_sync(uint32_t ta, const uint32_t* a, uint32_t tb,
                                                 const uint32_t* b) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%2,%3,%4,%5,%6,%7,%8,"
      "%9,%10,%11,%12,%13,%14,%15,%16,%17};"
      "\n\ttcgen05.st.sync.aligned.32x32b.x16.b32 [%1], {%18,%19,%20,%21,%22,%23,%24,%25,%26,"
      "%27,%28,%29,%30,%31,%32,%33};"
      "\n\ttcgen05.wait::st.sync.aligned;" ::"r"(ta), "r"(tb),
      "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(a[4]), "r"(a[5]), "r"(a[6]), "r"(a[7]),
      "r"(a[8]), "r"(a[9]), "r"(a[10]), "r"(a[11]), "r"(a[12]), "r"(a[13]), "r"(a[14]),
      "r"(a[15]), "r"(b[0]), "r"(b[1]), "r"(b[2]), "r"(b[3]), "r"(b[4]), "r"(b[5]), "r"(b[6]),
      "r"(b[7]), "r"(b[8]), "r"(b[9]), "r"(b[10]), "r"(b[11]), "r"(b[12]), "r"(b[13]),
      "r"(b[14]), "r"(b[15])
      : "memory");
}

__global__ void __launch_bounds__(kTcThreads, 2) prefill_attention_tc_kernel(const PrefillParams p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  // 1024-byte aligned base for the swizzled tiles.
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  unsigned char* smem = smem_raw + (base - raw);
  const uint32_t sQ = base;
  const uint32_t bar_s0 = base + kTcBarOff, bar_o = bar_s0 + 16;  // bar_s0, bar_s0 + 8: S buffers
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kTcBarOff + 24);
  float* s_max = reinterpret_cast<float*>(smem + kTcRowOff);      // [2][128] half-row maxima
  float* s_sum = s_max + 2 * 128;                                  // [2][128] half-row sums
  __shared__ int s_abort;

  const int4 w = p.work[blockIdx.x];
  if (w.x < 0) return;  // padding item of a query-tile pair
  const int hk = blockIdx.y;
  const int b = w.x, qb0 = w.y, key_lo = w.z, key_hi = w.w;
  const int qo0 = p.qo_indptr[b], nq_req = p.qo_indptr[b + 1] - qo0;
  const int kv0 = p.kv_indptr[b], n_prefix = p.kv_indptr[b + 1] - kv0;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // Warp w serves TMEM lanes 32 * (w % 4) .. (its rows) and column half w / 4.
  const int row = ((warp & 3) << 5) | lane, half = warp >> 2;
  const int n_tiles = (key_hi - key_lo + kTcKeys - 1) / kTcKeys;
  // After a wait ran out anywhere in this launch, later CTAs do nothing.  One
  // thread reads the launch's abort word and the CTA leaves as a whole: the
  // TMEM allocation below is warp-collective and the barriers count every
  // thread.
  __shared__ int s_skip;
  if (tid == 0)
    s_skip = p.error_flag != nullptr && reinterpret_cast<volatile int*>(p.error_flag)[1] != 0;
  __syncthreads();
  if (s_skip) return;

  if (warp == 0) {  // TMEM: two S buffers, P (hi, lo) and O
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTcCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    mbar_init(bar_s0, 1);
    mbar_init(bar_s0 + 8, 1);
    mbar_init(bar_o, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_abort = 0;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t trow = tmem + ((uint32_t)((warp & 3) * 32) << 16);  // this warp's TMEM lanes

  // ---- key gather: four threads per key, two 16-byte chunks each of K and V ----
  auto key_slot_pos = [&](int j, long long& slot, int& pos) {
    if (j < n_prefix) {
      slot = __ldg(p.kv_indices + kv0 + j);
      pos = __ldg(p.kv_positions + kv0 + j);
    } else {
      slot = __ldg(p.birth_slots + qo0 + (j - n_prefix));
      pos = __ldg(p.q_positions + qo0 + (j - n_prefix));
    }
    if (slot < 0 || slot >= p.num_slots) {
      if (p.error_flag) atomicOr(p.error_flag, 1);
      slot = 0;
    }
  };
  const int my_key = tid >> 2, my_quarter = tid & 3;
  struct KeyRef {
    long long slot;
    int pos;
  };
  auto fetch = [&](int tile) -> KeyRef {
    KeyRef r{0, INT_MAX};
    const int j = key_lo + tile * kTcKeys + my_key;
    if (tile < n_tiles && j < key_hi) key_slot_pos(j, r.slot, r.pos);
    return r;
  };
  auto stage_k = [&](int tile) { return base + kTcQBytes + (tile % kTcStages) * kTcStageBytes; };
  auto issue_tile = [&](int tile, const KeyRef r) {
    const uint32_t kb = stage_k(tile), vb = kb + kTcKVBytes;
    int* kpos = reinterpret_cast<int*>(smem + kTcPosOff + (tile % kTcStages) * kTcKeys * 4);
    if (my_quarter == 0) kpos[my_key] = r.pos;
    const int bytes = r.pos != INT_MAX ? 16 : 0;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int c = my_quarter * 2 + i;
      const uint32_t off = my_key * 128 + ((c ^ (my_key & 7)) * 16);
      cp_async16(kb + off, p.k + r.slot * p.k_ss + hk * p.k_sh + c * 8, bytes);
      cp_async16(vb + off, p.v + r.slot * p.v_ss + hk * p.v_sh + c * 8, bytes);
    }
  };
  // S(t) = Q K(t)^T into S buffer t & 1 (called by one thread).
  auto issue_s = [&](int tile) {
    const uint32_t kb = stage_k(tile);
#pragma unroll
    for (int k = 0; k < 4; ++k)  // K = 64 dims in 4 steps of 16 (32 bytes)
      mma_ss(tmem + kColS + (tile & 1) * kTcKeys, sw128_desc(sQ + 32 * k),
             sw128_desc(kb + 32 * k), f16_idesc(kTcKeys, 0), k > 0);
    umma_commit(bar_s0 + 8 * (tile & 1));
  };

  // ---- Q: row r = (query r / 8, head r % 8); two threads per row, four chunks each ----
  const int q_local = qb0 + (row >> 3);
  const int head = hk * kGroupP + (row & 7);
  const bool row_valid = q_local < nq_req;
  {
    const __nv_bfloat16* src = p.q + (long long)(qo0 + (row_valid ? q_local : 0)) * p.q_st +
                               (long long)head * p.q_sh;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int c = half * 4 + i;
      cp_async16(sQ + row * 128 + ((c ^ (row & 7)) * 16), src + c * 8, row_valid ? 16 : 0);
    }
  }
  // Groups: Q + tile 0, then tiles 1 .. kTcStages - 2, one group each.
#pragma unroll
  for (int t = 0; t < kTcStages - 1; ++t) {
    if (t < n_tiles) issue_tile(t, fetch(t));
    cp_async_commit();
  }
  KeyRef next = fetch(kTcStages - 1);

  // O = 0 in TMEM (every P.V then accumulates); this warp's 32 columns.
  {
    uint32_t z[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) z[i] = 0u;
    tmem_st32_sync(trow + kColO + 32 * half, z);
  }
  // S(0) as soon as Q and tile 0 have landed.
  cp_async_wait<kTcStages - 2>();
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  if (tid == 0 && n_tiles > 0) {
    tc_fence_after();
    issue_s(0);
  }

  const int pq = row_valid ? __ldg(p.q_positions + qo0 + q_local) : 0;
  const int jq = n_prefix + q_local;
  const int q_last_pos = __ldg(p.q_positions + qo0 + min(qb0 + kQBlock, nq_req) - 1);
  float m_used = -INFINITY, l = 0.f;  // l: this thread's half of the row sum
  uint32_t phase_o = 0u;
  bool timed_out = false;
  constexpr int kHalf = kTcKeys / 2;

  for (int tile = 0; tile < n_tiles; ++tile) {
    // 1. S(t) done -> this thread's 32 values of its row.  S buffer t & 1
    //    completes for the (t >> 1)-th time: its phase parity is (t >> 1) & 1.
    timed_out |= !mbar_wait(bar_s0 + 8 * (tile & 1), (uint32_t)(tile >> 1) & 1u);
    tc_fence_after();
    float s[kHalf];
    tmem_ld32_sync(trow + kColS + (tile & 1) * kTcKeys + half * kHalf, s);

    // 2. Mask; half-row maximum of the raw scores (the scale is positive, so
    //    it is applied to the maximum only) to shared memory.  Rows past the
    //    block's last query have Q = 0 and finite scores; they are never
    //    written out.
    const int j0 = key_lo + tile * kTcKeys;
    const int* kpos =
        reinterpret_cast<const int*>(smem + kTcPosOff + (tile % kTcStages) * kTcKeys * 4);
    const bool tile_full = j0 + kTcKeys <= key_hi && j0 + kTcKeys - 1 <= n_prefix + qb0 &&
                           (p.window < 0 || q_last_pos - kpos[0] <= p.window);
    float hm = -INFINITY;
    if (tile_full) {
#pragma unroll
      for (int i = 0; i < kHalf; ++i) hm = fmaxf(hm, s[i]);
    } else {
#pragma unroll
      for (int i = 0; i < kHalf; ++i) {
        const int kk = half * kHalf + i, j = j0 + kk;
        const bool ok = j < key_hi && (j < n_prefix || j <= jq) &&
                        (p.window < 0 || pq - kpos[kk] <= p.window);
        s[i] = ok ? s[i] : -INFINITY;
        hm = fmaxf(hm, s[i]);
      }
    }
    s_max[half * 128 + row] = hm * p.scale_log2;

    // 3. Tile t+1 landed -> S(t+1) on the tensor cores during this softmax.
    if (tile + 1 < n_tiles) cp_async_wait<kTcStages - 3>();
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    if (tid == 0 && tile + 1 < n_tiles) {
      tc_fence_after();
      issue_s(tile + 1);
    }

    // 4. Exponentials against the row's base; the base only moves when the
    //    tile exceeds it by 2^8, and then O and l are rescaled.
    const float bm = fmaxf(s_max[row], s_max[128 + row]);
    float alpha = 1.f;
    bool rescale = false;
    if (bm > m_used + kStaleMax || (m_used == -INFINITY && bm != -INFINITY)) {
      alpha = m_used == -INFINITY ? 0.f : fast_exp2(m_used - bm);
      rescale = m_used != -INFINITY;
      m_used = bm;
    }
    const float base2 = m_used == -INFINITY ? 0.f : m_used;
    // Two elements per packed instruction: x = s * scale - base (one fma),
    // exponentials, the row sum, and P = hi + lo (hi = RN_bf16(e), lo =
    // RN_bf16(e - hi)).
    const f32x2 scale2 = f2_pack(p.scale_log2, p.scale_log2), nbase2 = f2_pack(-base2, -base2);
    uint32_t hi[kHalf / 2], lo[kHalf / 2];
    f32x2 rs2 = f2_pack(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < kHalf; i += 2) {
      float x0, x1;
      f2_unpack(f2_fma(f2_pack(s[i], s[i + 1]), scale2, nbase2), x0, x1);
      const float e0 = fast_exp2(x0), e1 = fast_exp2(x1);
      const f32x2 e = f2_pack(e0, e1);
      rs2 = f2_add(rs2, e);
      const uint32_t h = pack_bf16(e0, e1);
      float d0, d1;
      f2_unpack(f2_sub(e, f2_pack(__uint_as_float(h << 16), __uint_as_float(h & 0xffff0000u))),
                d0, d1);
      hi[i / 2] = h;
      lo[i / 2] = pack_bf16(d0, d1);
    }
    float rs0, rs1;
    f2_unpack(rs2, rs0, rs1);
    l = l * alpha + (rs0 + rs1);

    // 5. P(t-1).V done: P and O may be rewritten, the stage of tile t-1 refilled.
    if (tile > 0) {
      timed_out |= !mbar_wait(bar_o, phase_o);
      phase_o ^= 1u;
      tc_fence_after();
    }
    {
      const int nt = tile + kTcStages - 1;  // into the stage tile t-1 used
      if (nt < n_tiles) {
        issue_tile(nt, next);
        next = fetch(nt + 1);
      }
      cp_async_commit();
    }
    // 6. Rescale this warp's half of O, write its half of P (tcgen05.ld / st
    //    are warp-wide: a warp rescales when any of its rows must).
    if (__any_sync(0xffffffffu, rescale)) {
      float o[32];
      tmem_ld32_sync(trow + kColO + 32 * half, o);
      uint32_t r[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(o[i] * alpha);
      tmem_st32_sync(trow + kColO + 32 * half, r);
    }
    tmem_st16x2_sync(trow + kColPHi + half * (kHalf / 2), hi, trow + kColPLo + half * (kHalf / 2),
                     lo);
    tc_fence_before();
    if (__syncthreads_or(timed_out)) {
      if (tid == 0) s_abort = 1;
      break;
    }
    // 7. O += P(t) V(t).
    if (tid == 0) {
      tc_fence_after();
      const uint32_t vb = stage_k(tile) + kTcKVBytes;
#pragma unroll
      for (int k = 0; k < kTcKeys / 16; ++k) {  // 16 keys per step: 8 TMEM columns, 2 KiB of V
        mma_ts(tmem + kColO, tmem + kColPHi + 8 * k, sw128_desc(vb + 2048 * k),
               f16_idesc(64, 1), 1);
        mma_ts(tmem + kColO, tmem + kColPLo + 8 * k, sw128_desc(vb + 2048 * k),
               f16_idesc(64, 1), 1);
      }
      umma_commit(bar_o);
    }
  }
  cp_async_wait<0>();

  // ---- epilogue ----
  s_sum[half * 128 + row] = l;
  __syncthreads();
  if (!s_abort && n_tiles > 0) {
    timed_out |= !mbar_wait(bar_o, phase_o);
    tc_fence_after();
  }
  const bool failed = __syncthreads_or(timed_out || s_abort);  // uniform over the CTA
  if (failed && tid == 0 && p.error_flag) {
    atomicOr(p.error_flag, 2);
    reinterpret_cast<volatile int*>(p.error_flag)[1] = 1;  // later CTAs of this launch skip
  }
  if (!failed) {
    float o[32];
    tmem_ld32_sync(trow + kColO + 32 * half, o);  // every thread: the load is warp-wide
    float den = s_sum[row] + s_sum[128 + row];
    const float mb = m_used == -INFINITY ? 0.f : m_used;
    if (p.sinks) den += fast_exp2(p.sinks[head] * kLog2e - mb);
    const float inv = den > 0.f ? 1.f / den : 0.f;
    __nv_bfloat16* dst = p.out + (long long)(qo0 + q_local) * p.o_st + (long long)head * p.o_sh +
                         32 * half;
#pragma unroll
    for (int c = 0; c < 4 && row_valid; ++c) {
      uint4 v;
      v.x = pack_bf16(o[8 * c] * inv, o[8 * c + 1] * inv);
      v.y = pack_bf16(o[8 * c + 2] * inv, o[8 * c + 3] * inv);
      v.z = pack_bf16(o[8 * c + 4] * inv, o[8 * c + 5] * inv);
      v.w = pack_bf16(o[8 * c + 6] * inv, o[8 * c + 7] * inv);
      *reinterpret_cast<uint4*>(dst + 8 * c) = v;
    }
    if (p.lse && row_valid && half == 0)
      p.lse[(long long)(qo0 + q_local) * p.num_q_heads + head] =
          den > 0.f ? (mb + log2f(den)) * kLn2 : -INFINITY;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTcCols));
  }
}

int launch_prefill_tc(const PrefillParams& p, int n_items, int num_kv_heads, cudaStream_t s) {
  if (cudaFuncSetAttribute(prefill_attention_tc_kernel,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem) != cudaSuccess)
    return AKV_ERR_CUDA;
  if (n_items > 0)
    prefill_attention_tc_kernel<<<dim3(n_items, num_kv_heads), kTcThreads, kTcSmem, s>>>(p);
  return launch_status();
}

// ---------------------------------------------------------------------------
// Warp-specialised form of the tcgen05 kernel: the same tiles, mask and
// arithmetic, with mbarriers instead of block barriers so that warps drift
// instead of meeting every tile.  Warps 0-7 gather K/V and run the softmax
// (two warps per TMEM lane quadrant, one per column half); warp 8 issues the
// MMAs.  P(t) is written over S(t) in tensor memory (hi bf16 pairs in
// columns 0-31 of the buffer, lo in 32-63), so P is double-buffered with S
// and the softmax never waits for the previous P.V.  Per key tile t:
//   kv[t % S]  256 arrivals: every loader's copies of tile t have landed
//              (cp.async.wait_group, proxy fence, arrive);
//   s[t & 1]   tcgen05.commit of S(t) = Q K(t)^T;
//   p          8 arrivals: P(t) is in tensor memory (and O rescaled);
//   o          tcgen05.commit of O += P(t) V(t).
// The issuer issues S(t) once K(t) has landed and P(t-2).V(t-2) is done
// (buffer t & 1 then holds nothing live), and P(t-1).V(t-1) once every warp
// has stored P(t-1).  Because S(t) completes after P(t-2).V(t-2), a softmax
// warp that has seen S(t) may refill the stage of tile t-2 (loads run three
// tiles ahead) and no further wait is needed before it stores P(t); only a
// rescale of O waits for P(t-1).V(t-1).  The two warps of a lane quadrant
// exchange half-row maxima through shared memory (double-buffered by tile
// parity) and a 64-thread named barrier, which also orders their S loads
// before either overwrites the buffer with P.  Every mbarrier wait is
// bounded; once one runs out, the CTA's abort flag makes every later wait
// return at once and the issuer stops issuing, so all warps still reach
// each named barrier and the end, where the CTA sets *error_flag = 2 and
// frees its tensor memory.
// ---------------------------------------------------------------------------
// Shared-memory and TMEM layout per head_dim D and query tiles per CTA QT
// (one query tile = 16 queries x 8 heads = 128 rows).  Rows of D bf16 are
// stored as D / 64 swizzle atoms of 128 bytes (atom a of every row, then
// atom a + 1).  head_dim 64: 5 stages (loads three tiles ahead); head_dim
// 128: 4 stages (two ahead).  QT = 1: two CTAs per SM at head_dim 64, one at
// 128; QT = 2: one CTA per SM whose two query tiles share every K/V tile.
// TMEM per query tile: 256 columns, S / P buffers in columns 0-63 and
// 64-127, O in the top D columns.
template <int D, int QT>
struct WsCfg {
  static constexpr int kThreads = 32 * (8 * QT + 1);  // 8 softmax warps per tile + the MMA warp
  static constexpr int kLoaders = 256 * QT;           // softmax threads, which also load
  static constexpr int kStages = D == 64 ? 5 : 4;
  static constexpr int kAhead = kStages - 2;  // tiles loaded ahead of the one in the softmax
  static constexpr int kChunks = D / 8;       // 16-byte chunks per row
  static constexpr int kTpk = kLoaders / kTcKeys;     // loader threads per key
  static constexpr int kCpt = kChunks / kTpk;         // chunks of K (and of V) per loader thread
  static constexpr int kQBytes = 128 * D * 2;         // one query tile
  static constexpr int kKVBytes = kTcKeys * D * 2;
  static constexpr int kStageBytes = 2 * kKVBytes;
  static constexpr int kStageOff = QT * kQBytes;
  static constexpr int kPosOff = kStageOff + kStages * kStageBytes;
  static constexpr int kRowOff = kPosOff + kStages * kTcKeys * 4;
  static constexpr int kRowBytes = 6 * 128 * 4;       // per tile: [2][2][128] max, [2][128] sum
  static constexpr int kBarOff = kRowOff + QT * kRowBytes;
  static constexpr int kSmemUsed = kBarOff + 256 + 1024;
  static constexpr int kSmem = QT == 1 && D == 64 && kSmemUsed < 80 * 1024 ? 80 * 1024 : kSmemUsed;
  static constexpr int kCols = 256 * QT;              // TMEM columns allocated
  static constexpr int kColO = 256 - D;               // within a query tile's 256 columns
  static constexpr int kMinBlocks = QT == 1 && D == 64 ? 2 : 1;
  static_assert(kAhead >= 2, "the loop signals tile t+1 from copies issued a tile earlier");
  static_assert(kCpt >= 1 && kChunks % kTpk == 0, "K/V chunks split over the loaders");
};
// Byte offset of 16-byte chunk c of row r in a swizzled tile of `rows` rows.
__device__ __forceinline__ uint32_t sw_chunk(int rows, int r, int c) {
  return (uint32_t)((c >> 3) * rows * 128 + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// 64-thread named barrier 1 + q of the two warps of pair q (query tile
// q / 4, lane quadrant q % 4); immediate ids, so the kernel reserves only the
// barriers it uses.
__device__ __forceinline__ void pair_sync(int q) {
  switch (q) {
    case 0: asm volatile("bar.sync 1, 64;" ::: "memory"); break;
    case 1: asm volatile("bar.sync 2, 64;" ::: "memory"); break;
    case 2: asm volatile("bar.sync 3, 64;" ::: "memory"); break;
    case 3: asm volatile("bar.sync 4, 64;" ::: "memory"); break;
    case 4: asm volatile("bar.sync 5, 64;" ::: "memory"); break;
    case 5: asm volatile("bar.sync 6, 64;" ::: "memory"); break;
    case 6: asm volatile("bar.sync 7, 64;" ::: "memory"); break;
    default: asm volatile("bar.sync 8, 64;" ::: "memory"); break;
  }
}
// Bounded wait that gives up at once after the CTA aborted.
__device__ __forceinline__ bool ws_wait(uint32_t bar, uint32_t parity, volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (*abort) return false;
    if (global_ns() - t0 > kWaitNs) {
      *abort = 1;
      return false;
    }
  }
  return true;
}

// LO: P enters P.V as the bf16 pair hi + lo (two MMAs per key block, P to
// about 16 bits); without it, as hi = RN_bf16(P) alone (one MMA), the
// precision of FlashInfer's and most flash kernels' P.V.
template <int D, int QT, bool LO>
__global__ void __launch_bounds__(WsCfg<D, QT>::kThreads, WsCfg<D, QT>::kMinBlocks)
prefill_attention_tc_ws_kernel(const PrefillParams p) {
  using C = WsCfg<D, QT>;
  constexpr int kTcStages = C::kStages, kWsAhead = C::kAhead;
  constexpr int kTcKVBytes = C::kKVBytes, kTcStageBytes = C::kStageBytes;
  constexpr int kTcPosOff = C::kPosOff, kWsBarOff = C::kBarOff;
  constexpr int kColO = C::kColO, kOCols = D / 2;  // O columns per softmax warp
  constexpr int kIssuer = 8 * QT;                  // the MMA warp
  extern __shared__ __align__(128) unsigned char smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  unsigned char* smem = smem_raw + (base - raw);
  // Barriers: kv[S] (tile landed), then per query tile s[2] and p[2] (by
  // tile parity), o (every P.V) and done (the last P.V).  A waiter on a
  // phase parity must never be two phases behind the barrier: P(t) arrives
  // on p[t & 1] because a warp can store P(t) while the MMA warp still
  // waits for P(t-1), and the epilogue waits on `done`, whose only phase
  // completes with the last P.V, because o may be anywhere from two phases
  // behind that to complete when a warp gets there.
  const uint32_t bars = base + kWsBarOff;
  auto bar_s = [&](int qt, int buf) { return bars + 8u * (kTcStages + 2 * qt + buf); };
  auto bar_p = [&](int qt, int buf) { return bars + 8u * (kTcStages + 2 * QT + 2 * qt + buf); };
  auto bar_o = [&](int qt) { return bars + 8u * (kTcStages + 4 * QT + qt); };
  auto bar_done = [&](int qt) { return bars + 8u * (kTcStages + 5 * QT + qt); };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kWsBarOff + 8 * (kTcStages + 6 * QT));
  __shared__ int s_abort;
  volatile int* abort = &s_abort;
  auto bar_kv = [&](int tile) { return bars + 8u * (uint32_t)(tile % kTcStages); };
  auto kv_parity = [&](int tile) { return (uint32_t)(tile / kTcStages) & 1u; };

  // Work items: query tile q of this CTA takes item QT * blockIdx.x + q.  The
  // host pairs consecutive 16-query blocks of one request; a second item
  // with a negative request is padding (its rows are past the request's
  // queries).  The CTA walks the union of the items' key ranges.
  const int4 w0 = p.work[QT * blockIdx.x];
  if (w0.x < 0) return;
  const int hk = blockIdx.y;
  const int b = w0.x;
  int key_lo = w0.z, key_hi = w0.w;
#pragma unroll
  for (int q = 1; q < QT; ++q) {
    const int4 wq = p.work[QT * blockIdx.x + q];
    if (wq.x >= 0) {
      key_lo = min(key_lo, wq.z);
      key_hi = max(key_hi, wq.w);
    }
  }
  const int qo0 = p.qo_indptr[b], nq_req = p.qo_indptr[b + 1] - qo0;
  const int kv0 = p.kv_indptr[b], n_prefix = p.kv_indptr[b + 1] - kv0;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n_tiles = (key_hi - key_lo + kTcKeys - 1) / kTcKeys;
  // After a wait ran out anywhere in this launch, later CTAs do nothing.  One
  // thread reads the launch's abort word and the CTA leaves as a whole: the
  // TMEM allocation below is warp-collective and the barriers count every
  // thread.
  __shared__ int s_skip;
  if (tid == 0)
    s_skip = p.error_flag != nullptr && reinterpret_cast<volatile int*>(p.error_flag)[1] != 0;
  __syncthreads();
  if (s_skip) return;

  if (warp == 0) {  // TMEM: per query tile two S / P buffers and O
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(C::kCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (tid == 0) {
    for (int st = 0; st < kTcStages; ++st) mbar_init(bars + 8 * st, C::kLoaders);
    for (int q = 0; q < QT; ++q) {
      mbar_init(bar_s(q, 0), 1);
      mbar_init(bar_s(q, 1), 1);
      mbar_init(bar_p(q, 0), 8);
      mbar_init(bar_p(q, 1), 8);
      mbar_init(bar_o(q), 1);
      mbar_init(bar_done(q), 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_abort = 0;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto stage_k = [&](int tile) {
    return base + C::kStageOff + (tile % kTcStages) * kTcStageBytes;
  };

  if (warp == kIssuer) {
    // ---- MMA issuer (one thread) ----
    if (lane == 0) {
      for (int t = 0; t <= n_tiles; ++t) {
        if (t < n_tiles) {  // S(t): K(t) landed; buffers t & 1 free once every P(t-2).V(t-2) is done
          ws_wait(bar_kv(t), kv_parity(t), abort);
          if (t >= 2)
            for (int q = 0; q < QT; ++q) ws_wait(bar_o(q), (uint32_t)(t - 2) & 1u, abort);
          if (!*abort) {
            tc_fence_after();
            const uint32_t kb = stage_k(t);
#pragma unroll
            for (int q = 0; q < QT; ++q) {
              const uint32_t sq = base + q * C::kQBytes;
#pragma unroll
              for (int k = 0; k < D / 16; ++k) {  // 16 dims a step; atom k / 4, 32 bytes each
                const uint32_t off = (uint32_t)(32 * (k & 3));
                mma_ss(tmem + 256 * q + kColS + (t & 1) * kTcKeys,
                       sw128_desc(sq + (k >> 2) * 128 * 128 + off),
                       sw128_desc(kb + (k >> 2) * kTcKeys * 128 + off), f16_idesc(kTcKeys, 0),
                       k > 0);
              }
              umma_commit(bar_s(q, t & 1));
            }
          }
        }
        if (t >= 1) {  // O += P(t-1) V(t-1) once every warp of the tile has stored P(t-1)
          const int u = t - 1;
          const uint32_t vb = stage_k(u) + kTcKVBytes;
#pragma unroll
          for (int q = 0; q < QT; ++q) {
            ws_wait(bar_p(q, u & 1), (uint32_t)(u >> 1) & 1u, abort);
            if (*abort) continue;
            tc_fence_after();
            const uint32_t pb = tmem + 256 * q + kColS + (u & 1) * kTcKeys;
#pragma unroll
            for (int k = 0; k < kTcKeys / 16; ++k) {  // 16 keys: 8 P columns, 2 KiB of V
              // V is MN-major (dims contiguous): atoms of 64 dims, 8 KiB apart.
              const uint64_t vd = D == 64 ? sw128_desc(vb + 2048 * k)
                                          : sw128_desc_mn(vb + 2048 * k, kTcKeys * 128);
              mma_ts(tmem + 256 * q + kColO, pb + 8 * k, vd, f16_idesc(D, 1), 1);
              if constexpr (LO)
                mma_ts(tmem + 256 * q + kColO, pb + 32 + 8 * k, vd, f16_idesc(D, 1), 1);
            }
            umma_commit(bar_o(q));
            if (u == n_tiles - 1) umma_commit(bar_done(q));
          }
        }
      }
    }
    __syncwarp();
  } else {
    // ---- loaders + softmax: warp w serves query tile w / 8, TMEM lanes
    //      32 (w % 4) .. and column half (w / 4) % 2 ----
    const int qt = QT == 1 ? 0 : warp >> 3;
    const int row = ((warp & 3) << 5) | lane, half = (warp >> 2) & 1;
    const uint32_t trow = tmem + 256 * qt + ((uint32_t)((warp & 3) * 32) << 16);
    const uint32_t sQ = base + qt * C::kQBytes;
    float* s_max = reinterpret_cast<float*>(smem + C::kRowOff + qt * C::kRowBytes);  // [parity][half][128]
    float* s_sum = s_max + 4 * 128;                                                 // [half][128]
    // This tile's queries: its item, or the 16 after the first item when the
    // item is padding (all of those rows are past the request's queries).
    int qb0 = w0.y;
#pragma unroll
    for (int q = 1; q < QT; ++q)
      if (qt == q) {
        const int4 wq = p.work[QT * blockIdx.x + q];
        qb0 = wq.x >= 0 ? wq.y : w0.y + q * kQBlock;
      }
    auto key_slot_pos = [&](int j, long long& slot, int& pos) {
      if (j < n_prefix) {
        slot = __ldg(p.kv_indices + kv0 + j);
        pos = __ldg(p.kv_positions + kv0 + j);
      } else {
        slot = __ldg(p.birth_slots + qo0 + (j - n_prefix));
        pos = __ldg(p.q_positions + qo0 + (j - n_prefix));
      }
      if (slot < 0 || slot >= p.num_slots) {
        if (p.error_flag) atomicOr(p.error_flag, 1);
        slot = 0;
      }
    };
    const int my_key = tid / C::kTpk, my_quarter = tid % C::kTpk;
    struct KeyRef {
      long long slot;
      int pos;
    };
    auto fetch = [&](int tile) -> KeyRef {
      KeyRef r{0, INT_MAX};
      const int j = key_lo + tile * kTcKeys + my_key;
      if (tile < n_tiles && j < key_hi) key_slot_pos(j, r.slot, r.pos);
      return r;
    };
    auto issue_tile = [&](int tile, const KeyRef r) {
      const uint32_t kb = stage_k(tile), vb = kb + kTcKVBytes;
      int* kpos = reinterpret_cast<int*>(smem + kTcPosOff + (tile % kTcStages) * kTcKeys * 4);
      if (my_quarter == 0) kpos[my_key] = r.pos;
      const int bytes = r.pos != INT_MAX ? 16 : 0;
#pragma unroll
      for (int i = 0; i < C::kCpt; ++i) {
        const int c = my_quarter * C::kCpt + i;
        const uint32_t off = sw_chunk(kTcKeys, my_key, c);
        cp_async16(kb + off, p.k + r.slot * p.k_ss + hk * p.k_sh + c * 8, bytes);
        cp_async16(vb + off, p.v + r.slot * p.v_ss + hk * p.v_sh + c * 8, bytes);
      }
    };

    // Q: row r = (query r / 8, head r % 8); two threads per row, half the chunks each.
    const int q_local = qb0 + (row >> 3);
    const int head = hk * kGroupP + (row & 7);
    const bool row_valid = q_local < nq_req;
    {
      const __nv_bfloat16* src = p.q + (long long)(qo0 + (row_valid ? q_local : 0)) * p.q_st +
                                 (long long)head * p.q_sh;
#pragma unroll
      for (int i = 0; i < C::kChunks / 2; ++i) {
        const int c = half * (C::kChunks / 2) + i;
        cp_async16(sQ + sw_chunk(128, row, c), src + c * 8, row_valid ? 16 : 0);
      }
    }
    // Groups: Q + tile 0, then tiles 1 .. kWsAhead - 1, one group each.
#pragma unroll
    for (int t = 0; t < kWsAhead; ++t) {
      if (t < n_tiles) issue_tile(t, fetch(t));
      cp_async_commit();
    }
    KeyRef next = fetch(kWsAhead);
    {  // O = 0 (every P.V accumulates): this warp's D / 2 columns
      uint32_t z[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) z[i] = 0u;
#pragma unroll
      for (int c = 0; c < kOCols; c += 32) tmem_st32_sync(trow + kColO + kOCols * half + c, z);
    }
    if (n_tiles > 0) {  // Q and tile 0 landed
      cp_async_wait<kWsAhead - 1>();
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(bar_kv(0));
    }

    const int pq = row_valid ? __ldg(p.q_positions + qo0 + q_local) : 0;
    const int jq = n_prefix + q_local;
    const int q_last_pos = __ldg(p.q_positions + qo0 + min(qb0 + kQBlock, nq_req) - 1);
    float m_used = -INFINITY, l = 0.f;
    constexpr int kHalf = kTcKeys / 2;

    for (int tile = 0; tile < n_tiles; ++tile) {
      // 0. This thread's copies of tile t+1 have landed (groups committed:
      //    tiles 0 .. t + kWsAhead - 1; tile t+1 and older complete).
      if (tile + 1 < n_tiles) {
        cp_async_wait<kWsAhead - 2>();
        fence_async_smem();
        mbar_arrive(bar_kv(tile + 1));
      }
      // 1. S(t) -> this thread's 32 values of its row.
      ws_wait(bar_s(qt, tile & 1), (uint32_t)(tile >> 1) & 1u, abort);
      tc_fence_after();
      // Tile t + kWsAhead into the stage of tile t-2 (S(t) completed after
      // P(t-2).V(t-2), so that stage is no longer read).
      {
        const int nt = tile + kWsAhead;
        if (nt < n_tiles) {
          issue_tile(nt, next);
          next = fetch(nt + 1);
        }
        cp_async_commit();
      }
      const uint32_t sbuf = trow + kColS + (tile & 1) * kTcKeys;
      float s[kHalf];
      tmem_ld32_sync(sbuf + half * kHalf, s);

      // 2. Mask (key positions of tile t: acquired through its kv barrier);
      //    half-row maximum of the raw scores, four independent chains.
      ws_wait(bar_kv(tile), kv_parity(tile), abort);
      const int j0 = key_lo + tile * kTcKeys;
      const int* kpos =
          reinterpret_cast<const int*>(smem + kTcPosOff + (tile % kTcStages) * kTcKeys * 4);
      const bool tile_full = j0 + kTcKeys <= key_hi && j0 + kTcKeys - 1 <= n_prefix + qb0 &&
                             (p.window < 0 || q_last_pos - kpos[0] <= p.window);
      if (!tile_full) {
#pragma unroll
        for (int i = 0; i < kHalf; ++i) {
          const int kk = half * kHalf + i, j = j0 + kk;
          const bool ok = j < key_hi && (j < n_prefix || j <= jq) &&
                          (p.window < 0 || pq - kpos[kk] <= p.window);
          s[i] = ok ? s[i] : -INFINITY;
        }
      }
      float hm4[4] = {s[0], s[1], s[2], s[3]};
#pragma unroll
      for (int i = 4; i < kHalf; ++i) hm4[i & 3] = fmaxf(hm4[i & 3], s[i]);
      const float hm = fmaxf(fmaxf(hm4[0], hm4[1]), fmaxf(hm4[2], hm4[3]));
      float* mx = s_max + (tile & 1) * 256;
      mx[half * 128 + row] = hm * p.scale_log2;
      // Both warps of the quadrant have their maxima in place and have read
      // S(t), which P(t) overwrites below.
      tc_fence_before();
      pair_sync(warp & 3 | qt << 2);  // qt is 0 when QT == 1: barriers 1-4 only
      tc_fence_after();
      const float bm = fmaxf(mx[row], mx[128 + row]);

      // 3. Exponentials against the row's base (moved only when the tile
      //    exceeds it by 2^8; then O and l are rescaled).
      float alpha = 1.f;
      bool rescale = false;
      if (bm > m_used + kStaleMax || (m_used == -INFINITY && bm != -INFINITY)) {
        alpha = m_used == -INFINITY ? 0.f : fast_exp2(m_used - bm);
        rescale = m_used != -INFINITY;
        m_used = bm;
      }
      const float base2 = m_used == -INFINITY ? 0.f : m_used;
      const f32x2 scale2 = f2_pack(p.scale_log2, p.scale_log2),
                  nbase2 = f2_pack(-base2, -base2);
      uint32_t hi[kHalf / 2], lo[kHalf / 2];
      f32x2 rsa = f2_pack(0.f, 0.f), rsb = rsa;
#pragma unroll
      for (int i = 0; i < kHalf; i += 2) {
        float x0, x1;
        f2_unpack(f2_fma(f2_pack(s[i], s[i + 1]), scale2, nbase2), x0, x1);
        const float e0 = fast_exp2(x0), e1 = fast_exp2(x1);
        const f32x2 e = f2_pack(e0, e1);
        if (i & 2) rsb = f2_add(rsb, e);
        else rsa = f2_add(rsa, e);
        const uint32_t h = pack_bf16(e0, e1);
        hi[i / 2] = h;
        if constexpr (LO) {
          float d0, d1;
          f2_unpack(
              f2_sub(e, f2_pack(__uint_as_float(h << 16), __uint_as_float(h & 0xffff0000u))),
              d0, d1);
          lo[i / 2] = pack_bf16(d0, d1);
        }
      }
      float rs0, rs1;
      f2_unpack(f2_add(rsa, rsb), rs0, rs1);
      l = l * alpha + (rs0 + rs1);

      // 4. Rescale this warp's half of O after P(t-1).V(t-1) (warp-wide TMEM
      //    access), then P(t) over S(t): hi in columns 0-31, lo in 32-63.
      if (__any_sync(0xffffffffu, rescale)) {
        ws_wait(bar_o(qt), (uint32_t)(tile - 1) & 1u, abort);
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < kOCols; c += 32) {
          float o[32];
          tmem_ld32_sync(trow + kColO + kOCols * half + c, o);
          uint32_t r[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(o[i] * alpha);
          tmem_st32_sync(trow + kColO + kOCols * half + c, r);
        }
      }
      if constexpr (LO)
        tmem_st16x2_sync(sbuf + half * (kHalf / 2), hi, sbuf + 32 + half * (kHalf / 2), lo);
      else
        tmem_st16_sync(sbuf + half * (kHalf / 2), hi);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_p(qt, tile & 1));
    }
    cp_async_wait<0>();

    // ---- epilogue ----
    s_sum[half * 128 + row] = l;
    pair_sync(warp & 3 | qt << 2);
    if (n_tiles > 0) {  // O is final once the last P.V is done
      ws_wait(bar_done(qt), 0u, abort);
      tc_fence_after();
    }
    if (!__any_sync(0xffffffffu, *abort != 0)) {
      float den = s_sum[row] + s_sum[128 + row];
      const float mb = m_used == -INFINITY ? 0.f : m_used;
      if (p.sinks) den += fast_exp2(p.sinks[head] * kLog2e - mb);
      const float inv = den > 0.f ? 1.f / den : 0.f;
      __nv_bfloat16* dst = p.out + (long long)(qo0 + q_local) * p.o_st +
                           (long long)head * p.o_sh + kOCols * half;
#pragma unroll
      for (int cb = 0; cb < kOCols; cb += 32) {
        float o[32];
        tmem_ld32_sync(trow + kColO + kOCols * half + cb, o);  // every lane: warp-wide load
#pragma unroll
        for (int c = 0; c < 4 && row_valid; ++c) {
          uint4 v;
          v.x = pack_bf16(o[8 * c] * inv, o[8 * c + 1] * inv);
          v.y = pack_bf16(o[8 * c + 2] * inv, o[8 * c + 3] * inv);
          v.z = pack_bf16(o[8 * c + 4] * inv, o[8 * c + 5] * inv);
          v.w = pack_bf16(o[8 * c + 6] * inv, o[8 * c + 7] * inv);
          *reinterpret_cast<uint4*>(dst + cb + 8 * c) = v;
        }
      }
      if (p.lse && row_valid && half == 0)
        p.lse[(long long)(qo0 + q_local) * p.num_q_heads + head] =
            den > 0.f ? (mb + log2f(den)) * kLn2 : -INFINITY;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (tid == 0 && s_abort && p.error_flag) {
    atomicOr(p.error_flag, 2);
    reinterpret_cast<volatile int*>(p.error_flag)[1] = 1;  // later CTAs of this launch skip
  }
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(C::kCols));
  }
}

// n_items counts 16-query items; with QT = 2 they come in pairs (the host
// pads the list to an even length).
template <int D, int QT, bool LO = true>
int launch_prefill_tc_ws(const PrefillParams& p, int n_items, int num_kv_heads, cudaStream_t s) {
  using C = WsCfg<D, QT>;
  if (n_items % QT) return AKV_ERR_INVALID;
  if (cudaFuncSetAttribute(prefill_attention_tc_ws_kernel<D, QT, LO>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem) != cudaSuccess)
    return AKV_ERR_CUDA;
  if (n_items > 0)
    prefill_attention_tc_ws_kernel<D, QT, LO>
        <<<dim3(n_items / QT, num_kv_heads), C::kThreads, C::kSmem, s>>>(p);
  return launch_status();
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
    int32_t* error_flag, int32_t variant, void* stream) {
  AKV_NVTX_RANGE("akv_context_attention");
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
  // Word 1 of the flag is this launch's abort word: cleared here so that a
  // wait that ran out in an earlier launch does not stop this one.  Word 0
  // keeps the error bits until the caller clears it.
  if (error_flag != nullptr && cudaMemsetAsync(error_flag + 1, 0, sizeof(int32_t), s) != cudaSuccess)
    return AKV_ERR_CUDA;
  // tcgen05 path: head_dim 64 with 16-byte aligned q / out rows.
  const bool aligned16 = (reinterpret_cast<uintptr_t>(q) & 15) == 0 &&
                         (reinterpret_cast<uintptr_t>(out) & 15) == 0 && q_stride_token % 8 == 0 &&
                         q_stride_head % 8 == 0 && out_stride_token % 8 == 0 &&
                         out_stride_head % 8 == 0;
  if (variant < 0 || variant > 6) return AKV_ERR_INVALID;
  // The tcgen05 kernels take row maxima of unscaled scores: sm_scale > 0.
  const bool tc_ok = aligned16 && sm_scale > 0.f;
  if (variant == 2 && !(tc_ok && head_dim == 64)) return AKV_ERR_UNSUPPORTED;
  if (variant >= 3 && !(tc_ok && (head_dim == 64 || head_dim == 128))) return AKV_ERR_UNSUPPORTED;
  // Default: one query tile per CTA at head_dim 64 (two CTAs per SM), two
  // query tiles per CTA at head_dim 128 (one CTA per SM either way).
  if (variant == 0 && tc_ok && head_dim == 128 && n_items % 2 == 0)
    return launch_prefill_tc_ws<128, 2>(p, n_items, num_kv_heads, s);
  if (variant == 3 || (variant == 0 && tc_ok)) {
    if (head_dim == 64) return launch_prefill_tc_ws<64, 1>(p, n_items, num_kv_heads, s);
    if (head_dim == 128) return launch_prefill_tc_ws<128, 1>(p, n_items, num_kv_heads, s);
  }
  if (variant == 4) {
    if (head_dim == 64) return launch_prefill_tc_ws<64, 2>(p, n_items, num_kv_heads, s);
    if (head_dim == 128) return launch_prefill_tc_ws<128, 2>(p, n_items, num_kv_heads, s);
  }
  // 5, 6: the forms of 3 and 4 with P rounded to bf16 for P.V.
  if (variant == 5) {
    if (head_dim == 64) return launch_prefill_tc_ws<64, 1, false>(p, n_items, num_kv_heads, s);
    if (head_dim == 128) return launch_prefill_tc_ws<128, 1, false>(p, n_items, num_kv_heads, s);
  }
  if (variant == 6) {
    if (head_dim == 64) return launch_prefill_tc_ws<64, 2, false>(p, n_items, num_kv_heads, s);
    if (head_dim == 128) return launch_prefill_tc_ws<128, 2, false>(p, n_items, num_kv_heads, s);
  }
  if (variant == 2) return launch_prefill_tc(p, n_items, num_kv_heads, s);
  switch (head_dim) {
    case 64: return launch_prefill<64>(p, n_items, num_kv_heads, s);
    case 128: return launch_prefill<128>(p, n_items, num_kv_heads, s);
  }
  return AKV_ERR_UNSUPPORTED;
}
