// GQA flash attention for the Qwen3 stack on tcgen05 (sm_100a): softmax(Q K^T / sqrt(128) + mask) V
// for 16 query heads sharing 8 key/value heads of dimension 128 (R:torch_xdna/stack.py:43-57).
//
// A work item = 128 queries of the two query heads that share one key/value head (2g and 2g+1), so each
// K and V^T block is loaded once for both. The kernel is persistent: one CTA per SM walks its share of
// the items (heaviest causal items first, snake order), and its roles run across item boundaries, so
// the next item's Q, K and first S overlap the current item's last P.V and output. 320 threads:
//   warp 0      TMA: both heads' Q tiles per item, then K blocks of 128 keys into a 2-stage ring and V^T
//               blocks into a 1-stage slot (Q and K read from the q/k projection output [T, 3072] bf16,
//               V^T from [1024, T'] bf16, which the projection epilogue wrote transposed so that P.V
//               has a K-major B operand);
//   warp 1      TMEM (per head: S, 128 columns; O, 128 columns) and the MMAs, issued as
//               S_A(j), S_B(j), O_A += P_A(j-1) V(j-1), O_B += P_B(j-1) V(j-1), ... so that while one
//               head's softmax works on block j the tensor core computes the other head's S and the
//               previous block's P.V;
//   warps 2..5  softmax of head A, warps 6..9 of head B: thread i of a group owns query row i. S_j is
//               loaded from TMEM once into registers; p = 2^(s * scale * log2 e - m) is written as bf16
//               into the head's 128-byte-swizzled K-major P tile and summed. O stays in TMEM and the
//               MMA accumulates into it; the running max m is only raised (and O, l rescaled in place)
//               when a block's max exceeds it by more than 2^8, so p <= 256 and most blocks touch O not
//               at all. The output row is O / l in bf16 [T, 2048].
// Masks: causal, per-sequence prefix blocks (the reference's OmniVoice layout: the first n positions
// see each other, later ones only themselves), a general bool mask [B, 1|H, L, L], or none; blocks that
// no mask entry can touch (for causal: every block left of the diagonal) skip the masking entirely.
// Keys past the sequence end are always masked. Every mbarrier wait is bounded (sm100.cuh).
#include <algorithm>

#include "host_util.h"
#include "sm100.cuh"

namespace xdna {

enum MaskKind { MASK_CAUSAL = 0, MASK_PREFIX = 1, MASK_BOOL = 2, MASK_NONE = 3 };

struct AttnArgs {
  __nv_bfloat16* out;     // [T, 2048]
  int T, L;               // tokens in all, tokens per sequence
  int L8;                 // round_up(L, 8): V^T column pitch of a sequence
  int q_blocks;           // ceil(L / 128)
  int B;                  // sequences
  int n_items;            // q_blocks x B x 8 work items (query block, sequence, key/value head)
  float scale_log2;       // log2(e) / sqrt(128)
  const int32_t* lens;    // MASK_PREFIX: per-sequence length
  const uint8_t* mask;    // MASK_BOOL: [B, Hm, L, L]
  int mask_heads;         // Hm: 1 or 16
  int* err;
};

constexpr int kAttnThreads = 320;
constexpr int kTileBytes = 128 * 128;  // one 128-row x 128-byte operand k-block
constexpr int kKStages = 2;
constexpr int kAttnSmem = (2 * 2 /*Q, 2 heads*/ + 2 * kKStages /*K*/ + 2 /*V*/ + 2 * 2 /*P, 2 heads*/) * kTileBytes +
                          1024 + 256;
constexpr float kRescaleLog2 = 8.0f;   // lazy rescale threshold: p stays <= 2^8

__device__ __forceinline__ uint32_t pack2_bf16(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ bool key_allowed(int kind, const AttnArgs& a, int seq, int head, int q, int k) {
  if (k >= a.L) return false;
  switch (kind) {
    case MASK_CAUSAL:
      return k <= q;
    case MASK_PREFIX: {
      const int n = a.lens[seq];
      return q < n ? k < n : k == q;
    }
    case MASK_BOOL:
      return a.mask[((static_cast<int64_t>(seq) * a.mask_heads + (a.mask_heads > 1 ? head : 0)) * a.L + q) * a.L + k] != 0;
    default:
      return true;
  }
}

template <int KIND>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attention_kernel(const __grid_constant__ CUtensorMap tmQK, const __grid_constant__ CUtensorMap tmVt,
                     const AttnArgs args) {
  constexpr uint32_t IDESC = idesc_bf16(128, 128);
  constexpr uint32_t TX = 2 * kTileBytes;  // one head's Q tile, or one K block, or one V^T block
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smQ = smem;                              // [head][k-block]
  uint8_t* smK = smQ + 4 * kTileBytes;              // [stage][k-block]
  uint8_t* smV = smK + 2 * kKStages * kTileBytes;   // [k-block]
  uint8_t* smP = smV + 2 * kTileBytes;              // [head][k-block]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smP + 4 * kTileBytes);
  uint64_t* q_full = bars;
  uint64_t* q_empty = bars + 1;              // an item's S MMAs done: Q may be reloaded
  uint64_t* k_full = bars + 2;               // [kKStages]
  uint64_t* k_empty = k_full + kKStages;     // [kKStages]
  uint64_t* v_full = k_empty + kKStages;
  uint64_t* v_empty = v_full + 1;
  uint64_t* s_full = v_empty + 1;            // [head] S ready in TMEM
  uint64_t* s_empty = s_full + 2;            // [head] S loaded by the softmax: the next S may be computed
  uint64_t* p_full = s_empty + 2;            // [head] P written (and O rescaled): O += P V may run
  uint64_t* p_empty = p_full + 2;            // [head] O += P V done: P may be rewritten, O read
  uint64_t* drain = p_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id(), lane = lane_id();
  // Work items (query block, sequence, key/value head) with the query block slowest, so that for causal
  // masks the items with the most key blocks come first. Round k of the G = gridDim.x CTAs takes items
  // kG .. kG+G-1, in snake order (CTA c takes kG + c in even rounds, kG + G-1-c in odd ones): with the
  // heaviest items first this balances the CTAs' total key blocks like a longest-first greedy schedule.
  // Every role walks the same items and counts key blocks across them (g), which gives each barrier's
  // phase: one K stage / V slot / S / P round per key block, one Q load per item.
  const int cta = static_cast<int>(blockIdx.x), G = static_cast<int>(gridDim.x);
  auto item_index = [&](int k) { return k * G + ((k & 1) ? G - 1 - cta : cta); };
  auto item_of = [&](int idx, int& qb, int& seq, int& kvh) {
    const int per = args.B * 8;
    const int lev = idx / per;
    const int rem = idx - lev * per;
    qb = KIND == MASK_CAUSAL ? args.q_blocks - 1 - lev : lev;
    seq = rem >> 3;
    kvh = rem & 7;
  };
  auto blocks_of = [&](int qb) { return KIND == MASK_CAUSAL ? qb + 1 : (args.L + 127) / 128; };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < kKStages; ++s) {
      mbar_init(k_full + s, 1);
      mbar_init(k_empty + s, 1);
    }
    mbar_init(v_full, 1);
    mbar_init(v_empty, 1);
    for (int h = 0; h < 2; ++h) {
      mbar_init(s_full + h, 1);
      mbar_init(s_empty + h, 4);
      mbar_init(p_full + h, 4);
      mbar_init(p_empty + h, 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmQK);
    tma_prefetch_desc(&tmVt);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // per head: S at columns [256 h, 256 h + 128), O at [256 h + 128, 256 h + 256)

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------------ TMA
      int k_last[kKStages] = {-1, -1};
      int v_last = -1;
      int q_loads = 0;
      // item number n's Q tiles (both heads), once the previous item's S MMAs have read the old ones
      auto load_q = [&](int n, int seq, int kvh, int q0) -> bool {
        if (!mbar_wait(q_empty, (n & 1) ^ 1, abort_flag, args.err, 20)) return false;
        mbar_arrive_expect_tx(q_full, 2 * TX);
        for (int h = 0; h < 2; ++h)
          for (int kk = 0; kk < 2; ++kk)
            tma_load_2d(smQ + (h * 2 + kk) * kTileBytes, &tmQK, q_full, (2 * kvh + h) * 128 + kk * 64,
                        seq * args.L + q0);
        ++q_loads;
        return true;
      };
      // key block j of (seq, kvh) as global block gb
      auto load_k = [&](int gb, int seq, int kvh, int j) -> bool {
        const int st = gb % kKStages;
        const uint32_t ph = (gb / kKStages) & 1;
        if (!mbar_wait(k_empty + st, ph ^ 1, abort_flag, args.err, 21)) return false;
        mbar_arrive_expect_tx(k_full + st, TX);
        for (int kk = 0; kk < 2; ++kk)
          tma_load_2d(smK + (st * 2 + kk) * kTileBytes, &tmQK, k_full + st, 16 * 128 + kvh * 128 + kk * 64,
                      seq * args.L + j * 128);
        k_last[st] = static_cast<int>(ph);
        return true;
      };
      auto load_v = [&](int gb, int seq, int kvh, int j) -> bool {
        const uint32_t ph = gb & 1;
        if (!mbar_wait(v_empty, ph ^ 1, abort_flag, args.err, 22)) return false;
        mbar_arrive_expect_tx(v_full, TX);
        // V^T column = seq * L8 + key: a multiple of 8 elements, the 16-byte TMA alignment
        for (int kk = 0; kk < 2; ++kk)
          tma_load_2d(smV + kk * kTileBytes, &tmVt, v_full, seq * args.L8 + j * 128 + kk * 64, kvh * 128);
        v_last = static_cast<int>(ph);
        return true;
      };
      // K runs one block ahead of V (K_{g+1} is issued before V_g), across items too: after an item's
      // last V come the next item's Q and first K.
      bool ok = true;
      int g = 0;
      for (int n = 0; ok && item_index(n) < args.n_items; ++n) {
        int qb, seq, kvh;
        item_of(item_index(n), qb, seq, kvh);
        const int nb = blocks_of(qb);
        if (n == 0) ok = load_q(0, seq, kvh, qb * 128) && load_k(0, seq, kvh, 0);
        for (int j = 0; ok && j < nb; ++j, ++g) {
          if (j + 1 < nb) {
            ok = load_k(g + 1, seq, kvh, j + 1) && load_v(g, seq, kvh, j);
          } else {
            ok = load_v(g, seq, kvh, j);
            if (ok && item_index(n + 1) < args.n_items) {
              int qb2, seq2, kvh2;
              item_of(item_index(n + 1), qb2, seq2, kvh2);
              ok = load_q(n + 1, seq2, kvh2, qb2 * 128) && load_k(g + 1, seq2, kvh2, 0);
            }
          }
        }
      }
      // every load has landed before the CTA may exit
      volatile int never = 0;
      if (q_loads > 0) mbar_wait(q_full, static_cast<uint32_t>((q_loads - 1) & 1), &never, args.err, 23);
      for (int s = 0; s < kKStages; ++s)
        if (k_last[s] >= 0) mbar_wait(k_full + s, static_cast<uint32_t>(k_last[s]), &never, args.err, 23);
      if (v_last >= 0) mbar_wait(v_full, static_cast<uint32_t>(v_last), &never, args.err, 23);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------------ MMA
      bool ok = true;
      bool issued = false;
      // O_h += P_h V for global block gb; the first block of an item overwrites O (acc = 0)
      auto issue_pv = [&](int gb, bool item_start) -> bool {
        if (!mbar_wait(v_full, gb & 1, abort_flag, args.err, 25)) return false;
        for (int h = 0; h < 2; ++h) {
          if (!mbar_wait(p_full + h, gb & 1, abort_flag, args.err, 26)) return false;
          tc_fence_after();
          const uint32_t tO = tmem + 256 * h + 128;
          for (int kk = 0; kk < 2; ++kk) {
            const uint64_t dP = smem_desc_k_sw128(smem_u32(smP + (h * 2 + kk) * kTileBytes));
            const uint64_t dV = smem_desc_k_sw128(smem_u32(smV + kk * kTileBytes));
#pragma unroll
            for (int k = 0; k < 4; ++k) umma_f16(tO, dP + 2 * k, dV + 2 * k, IDESC, (!item_start || kk | k) != 0);
          }
          umma_commit(p_empty + h);
          issued = true;
        }
        umma_commit(v_empty);
        return true;
      };
      int g = 0;
      bool prev_start = false;  // block g - 1 is the first of its item
      for (int n = 0; ok && item_index(n) < args.n_items; ++n) {
        int qb, seq, kvh;
        item_of(item_index(n), qb, seq, kvh);
        const int nb = blocks_of(qb);
        if (!mbar_wait(q_full, n & 1, abort_flag, args.err, 24)) break;
        for (int j = 0; j < nb; ++j, ++g) {
          const int st = g % kKStages;
          if (!mbar_wait(k_full + st, (g / kKStages) & 1, abort_flag, args.err, 27)) {
            ok = false;
            break;
          }
          for (int h = 0; h < 2 && ok; ++h) {
            if (!mbar_wait(s_empty + h, (g & 1) ^ 1, abort_flag, args.err, 28)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t tS = tmem + 256 * h;
            for (int kk = 0; kk < 2; ++kk) {
              const uint64_t dQ = smem_desc_k_sw128(smem_u32(smQ + (h * 2 + kk) * kTileBytes));
              const uint64_t dK = smem_desc_k_sw128(smem_u32(smK + (st * 2 + kk) * kTileBytes));
#pragma unroll
              for (int k = 0; k < 4; ++k) umma_f16(tS, dQ + 2 * k, dK + 2 * k, IDESC, (kk | k) != 0);
            }
            umma_commit(s_full + h);
            issued = true;
          }
          if (!ok) break;
          if (j == nb - 1) umma_commit(q_empty);  // this item's Q has been read once these complete
          umma_commit(k_empty + st);
          if (g >= 1 && !issue_pv(g - 1, prev_start)) {
            ok = false;
            break;
          }
          prev_start = j == 0;
        }
      }
      if (ok && g > 0) issue_pv(g - 1, prev_start);
      if (issued) {
        umma_commit(drain);
        volatile int never = 0;
        mbar_wait(drain, 0, &never, args.err, 29);
      }
    }
  } else {
    // -------------------------------------------------------------------- softmax (warps 2..9)
    const int hg = (warp - 2) >> 2;          // 0: query head 2 kvh, 1: 2 kvh + 1
    const int qd = warp & 3;                 // TMEM lane quadrant = row block
    const int r = qd * 32 + lane;            // query row within the tile
    const uint32_t lane_off = static_cast<uint32_t>(qd * 32) << 16;
    const uint32_t tS = tmem + 256 * hg;
    const uint32_t tO = tS + 128;
    uint8_t* myP = smP + hg * 2 * kTileBytes;
    const float sc = args.scale_log2;
    bool ok = true;
    uint32_t v[128];                         // this row of S, loaded from TMEM once
    int g = 0;
    for (int n = 0; ok && item_index(n) < args.n_items; ++n) {
      int qb, seq, kvh;
      item_of(item_index(n), qb, seq, kvh);
      const int nb = blocks_of(qb);
      const int head = 2 * kvh + hg;
      const int q0 = qb * 128;               // first query position in the sequence
      const int qpos = q0 + r;               // this row's query position
      float m_use = -INFINITY;               // the max the probabilities and O are relative to (log2 units)
      float l = 0.f;
      for (int j = 0; j < nb; ++j, ++g) {
        const int k0 = j * 128;
        // warp-uniform: does any entry of this block need the mask?
        const bool masked = KIND == MASK_PREFIX || KIND == MASK_BOOL || k0 + 128 > args.L ||
                            (KIND == MASK_CAUSAL && k0 + 127 > q0);
        if (!mbar_wait(s_full + hg, g & 1, abort_flag, args.err, 31)) {
          ok = false;
          break;
        }
        tc_fence_after();
        __syncwarp();
#pragma unroll
        for (int c = 0; c < 4; ++c)
          tmem_ld_32x32b_x32(tS + lane_off + c * 32, *reinterpret_cast<uint32_t(*)[32]>(v + c * 32));
        tmem_ld_wait();
        // S is in registers: the MMA may compute the next S into these columns
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(s_empty + hg);
        if (masked) {
#pragma unroll
          for (int e = 0; e < 128; ++e)
            if (!key_allowed(KIND, args, seq, head, qpos, k0 + e)) v[e] = __float_as_uint(-INFINITY);
        }
        // the row max of the raw scores (scale > 0 commutes with max), as 8 independent partial maxima so
        // that the reduction is not one 128-long dependent chain
        // (three-input max.f32: two keys per instruction)
        float m8[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) m8[i] = __uint_as_float(v[i]);
#pragma unroll
        for (int e = 8; e + 16 <= 128; e += 16) {
#pragma unroll
          for (int i = 0; i < 8; ++i) m8[i] = fmax3(m8[i], __uint_as_float(v[e + i]), __uint_as_float(v[e + 8 + i]));
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) m8[i] = fmaxf(m8[i], __uint_as_float(v[120 + i]));
        const float mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])), fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
        const float m_blk = mx * sc;
        // raise the running max only when this block would push p above 2^8
        float alpha = 1.f;
        const bool raise = m_blk > m_use + kRescaleLog2;
        if (raise) {
          alpha = fast_exp2(m_use - m_blk);  // 0 while m_use is -inf
          m_use = m_blk;
        }
        // O += P V of the previous block has finished: O may be rescaled and the P tile rewritten (for an
        // item's first block the previous item's output pass already waited for it)
        if (j >= 1 && !mbar_wait(p_empty + hg, (g - 1) & 1, abort_flag, args.err, 32)) {
          ok = false;
          break;
        }
        if (j >= 1 && __any_sync(0xffffffffu, raise && l > 0.f)) {
          // rows that did not raise multiply by 1
          tc_fence_after();
          uint32_t o[32];
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            __syncwarp();
            tmem_ld_32x32b_x32(tO + lane_off + c * 32, o);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tmem_st_32x32b_x32(tO + lane_off + c * 32, o);
          }
          tmem_st_wait();
        }
        l *= alpha;
        // p = 2^(s * scale - m) as bf16 into the swizzled K-major P tile, and the row sum
        const float neg_m = m_use == -INFINITY ? 0.f : -m_use;
        const bool none = m_use == -INFINITY;  // every key so far masked
        // two keys per instruction where the f32x2 pipe allows (the softmax is issue-bound): packed
        // s * scale - m and packed partial row sums, the exponentials on the MUFU
        float2 rs4[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
        const float2 sc2 = make_float2(sc, sc), nm2 = make_float2(neg_m, neg_m);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t w[16];
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            const float2 x = __ffma2_rn(make_float2(__uint_as_float(v[c * 32 + e]), __uint_as_float(v[c * 32 + e + 1])),
                                        sc2, nm2);
            float2 pp = make_float2(fast_exp2(x.x), fast_exp2(x.y));
            if (none) pp = make_float2(0.f, 0.f);
            rs4[(e >> 1) & 3] = __fadd2_rn(rs4[(e >> 1) & 3], pp);
            w[e / 2] = pack2_bf16(pp.x, pp.y);
          }
          // 32 keys = 64 bytes = 4 chunks of 16 bytes in k-block c / 2, chunk offset (c % 2) * 4
          uint8_t* rowp = myP + (c >> 1) * kTileBytes + r * 128;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int chunk = (c & 1) * 4 + q;
            *reinterpret_cast<uint4*>(rowp + ((chunk ^ (r & 7)) * 16)) =
                make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
          }
        }
        l += ((rs4[0].x + rs4[0].y) + (rs4[1].x + rs4[1].y)) + ((rs4[2].x + rs4[2].y) + (rs4[3].x + rs4[3].y));
        // P (and the rescaled O) are ready for the MMA
        tc_fence_before();
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full + hg);
      }
      if (!ok || nb == 0) break;
      // the item's last O += P V, then O / l
      if (!mbar_wait(p_empty + hg, (g - 1) & 1, abort_flag, args.err, 34)) break;
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      uint4* dst = reinterpret_cast<uint4*>(args.out + static_cast<int64_t>(seq * args.L + qpos) * (16 * 128) + head * 128);
      uint32_t o[32];
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        __syncwarp();
        tmem_ld_32x32b_x32(tO + lane_off + c * 32, o);
        tmem_ld_wait();
        if (qpos < args.L) {
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            uint4 u;
            u.x = pack2_bf16(__uint_as_float(o[e]) * inv, __uint_as_float(o[e + 1]) * inv);
            u.y = pack2_bf16(__uint_as_float(o[e + 2]) * inv, __uint_as_float(o[e + 3]) * inv);
            u.z = pack2_bf16(__uint_as_float(o[e + 4]) * inv, __uint_as_float(o[e + 5]) * inv);
            u.w = pack2_bf16(__uint_as_float(o[e + 6]) * inv, __uint_as_float(o[e + 7]) * inv);
            dst[(c * 32 + e) / 8] = u;
          }
        }
      }
      // O has been read: the next item's first O = P V (issued after this warp's next P) may overwrite it
      tc_fence_before();
    }
  }
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

int run_attention(const __nv_bfloat16* qk, const __nv_bfloat16* vt, int64_t ldvt, __nv_bfloat16* out, int64_t B,
                  int64_t L, int mask_kind, const int32_t* lens, const uint8_t* mask, int mask_heads,
                  cudaStream_t stream) {
  int sms = 0;
  int rc = check_device(&sms);
  if (rc != XDNA_OK) return rc;
  XDNA_CHECK_ARG(B >= 1 && L >= 1 && (L + 127) / 128 * B * 8 < (1ll << 31), "attention: bad batch / length");
  XDNA_CHECK_ARG(qk && vt && out, "attention: null pointer");
  const int64_t T = B * L;
  const int64_t L8 = (L + 7) / 8 * 8;
  XDNA_CHECK_ARG(ldvt >= B * L8 && ldvt % 8 == 0,
                 "attention: V^T row pitch must cover B x round_up(L, 8) columns and be a multiple of 8");
  XDNA_CHECK_ARG(mask_kind >= MASK_CAUSAL && mask_kind <= MASK_NONE, "attention: unknown mask kind %d", mask_kind);
  XDNA_CHECK_ARG(mask_kind != MASK_PREFIX || lens != nullptr, "attention: prefix masks need lengths");
  XDNA_CHECK_ARG(mask_kind != MASK_BOOL || (mask != nullptr && (mask_heads == 1 || mask_heads == 16)),
                 "attention: bool masks need a [B, 1|16, L, L] mask");
  CUtensorMap tq, tv;
  {
    const uint64_t dims[2] = {3072, static_cast<uint64_t>(T)};
    const uint64_t strides[1] = {3072 * 2};
    const uint32_t box[2] = {64, 128};
    if ((rc = encode_tma(&tq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, qk, dims, strides, box, "attention q/k")) != XDNA_OK)
      return rc;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(B * L8), 1024};
    const uint64_t strides[1] = {static_cast<uint64_t>(ldvt * 2)};
    const uint32_t box[2] = {64, 128};
    if ((rc = encode_tma(&tv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, vt, dims, strides, box, "attention v^T")) != XDNA_OK)
      return rc;
  }
  AttnArgs a{};
  a.out = out;
  a.T = static_cast<int>(T);
  a.L = static_cast<int>(L);
  a.L8 = static_cast<int>(L8);
  a.q_blocks = static_cast<int>((L + 127) / 128);
  a.B = static_cast<int>(B);
  a.n_items = a.q_blocks * a.B * 8;
  a.scale_log2 = 1.4426950408889634f / sqrtf(128.f);
  a.lens = lens;
  a.mask = mask;
  a.mask_heads = mask_heads;
  a.err = device_error_word();
  // persistent: one CTA per SM (its shared memory allows no second), each walking its share of the items
  const int grid = std::min(a.n_items, sms);
  static std::atomic<bool> configured[4][64];  // setting the attribute twice from two threads is harmless
  int dev = 0;
  XDNA_CUDA(cudaGetDevice(&dev));
  void (*kern)(const CUtensorMap, const CUtensorMap, const AttnArgs) =
      mask_kind == MASK_CAUSAL   ? attention_kernel<MASK_CAUSAL>
      : mask_kind == MASK_PREFIX ? attention_kernel<MASK_PREFIX>
      : mask_kind == MASK_BOOL   ? attention_kernel<MASK_BOOL>
                                 : attention_kernel<MASK_NONE>;
  if (dev < 0 || dev >= 64 || !configured[mask_kind][dev].load(std::memory_order_acquire)) {
    XDNA_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmem));
    if (dev >= 0 && dev < 64) configured[mask_kind][dev].store(true, std::memory_order_release);
  }
  kern<<<grid, kAttnThreads, kAttnSmem, stream>>>(tq, tv, a);
  return check_launch("attention_kernel");
}

}  // namespace xdna
