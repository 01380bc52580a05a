// Persistent, warp-specialised tcgen05 GEMM for sm_100a, shared by the W8A8 linear and the
// implicit-GEMM conv3x3.
//
//   C[m, n] = sum_k A[m, k] * B[n, k]        (A and B K-major; int8 -> int32 or bf16 -> f32)
//
// One CTA per SM walks output tiles of 128 x BN. Roles (320 threads):
//   warp 0        TMA producer: a ring of STAGES shared-memory stages, each one 128-byte-wide
//                 K block of A (128 rows) and B (BN rows), written with 128-byte swizzle;
//   warp 1        TMEM allocator and MMA issuer: 4 tcgen05.mma (K = 32 bytes each) per stage into
//                 one of two TMEM accumulators (2 x BN columns), so the epilogue of tile i
//                 overlaps the MMAs of tile i+1;
//   warps 2..9    epilogue: warp w reads TMEM lanes 32*(w%4)..+31 (its 32 output rows) and one half
//                 of the tile's columns, 32 columns per tcgen05.ld, issued one chunk ahead of the
//                 arithmetic. Per-column factors arrive once per tile as one coalesced load per lane,
//                 then sit in the warp's shared memory (dequantising epilogues) or are broadcast with
//                 warp shuffles. GEMM outputs are staged in swizzled shared memory (2 KB slots) and
//                 written by TMA bulk-tensor stores (full lines, tails clipped by the tensor map); conv
//                 outputs are staged per pixel and written as whole lines with direct stores.
//
// The A operand is either a plain row-major matrix (LOAD_GEMM) or, for the conv, the
// zero-bordered NHWC activations viewed as a [pixels, Cp] matrix: the K loop runs over 9 taps x
// channel blocks and a tap is a constant row offset dy*(W+2)+dx into that matrix (LOAD_CONV);
// TMA's zero fill covers rows before the first / past the last pixel and channels past Cp.
#pragma once

#include "host_util.h"
#include "sm100.cuh"

namespace xdna {

// LOAD_CONV_RB: the conv with its weights resident in shared memory for the whole kernel (one channel
// block of <= 64 channels, one column tile of <= 128 output channels): each stage then holds only the
// activation rows, which halves the TMA row requests per stage when rows are 64 bytes.
// LOAD_CONV_WIN: LOAD_CONV_RB for a stride-1 3x3 conv whose stages each hold one window of kBM + 2 activation
// rows per ky: the ky's three kx taps read it at row offsets 0, 1 and 2 (their MMA descriptors start one or
// two 64-byte rows into the window), so each row is requested from TMA once per ky instead of once per tap.
// LOAD_CONV_WIN2: LOAD_CONV_WIN over an input whose images are interleaved in pairs ([N/2, H+2, W+2, 2 x 64]:
// each 128-byte row holds one pixel of images 2i and 2i+1), so a window row request brings 128 bytes where
// LOAD_CONV_WIN's brings 64: half the TMA row requests, the mainloop's bound for 64-channel convs. Each kx
// tap issues the MMAs of both images, reading K bytes 0..63 (image 2i) and 64..127 (image 2i+1) of the
// rows into two accumulators; the epilogue drains both (int8 codes out only).
// LOAD_CONV_WINB: the window for convs of 128-byte channel blocks whose weights do not stay resident: a stage
// holds one window of kBM + 2 rows of one channel block for one ky and the three kx taps' weight tiles of that
// block, so the A rows are requested once per ky instead of once per tap (B as before).
enum LoadMode { LOAD_GEMM = 0, LOAD_CONV = 1, LOAD_CONV_RB = 2, LOAD_CONV_WIN = 3, LOAD_CONV_WIN2 = 4, LOAD_CONV_WINB = 5 };

enum EpiMode {
  EPI_I32 = 0,         // int32 accumulators
  EPI_DEQ = 1,         // (float(acc) * sx[m]) * sw[n] (+ bias[n]) -> f32 / bf16 / f16
  EPI_CONV_Q = 2,      // requantised int8 / uint8, NCHW
  EPI_CONV_DEQ = 3,    // requantised then dequantised, NCHW
  EPI_CONV_CALIB = 4,  // max of the sums (of image 0) into one int32
  // bf16 GEMMs of the Qwen3 stack (f32 accumulators)
  EPI_F32ACC = 5,      // acc (+ bias[n]) -> f32 / bf16 / f16 (the head; precision="bf16" linears)
  EPI_RESID = 6,       // resid_f32[m, n] += acc (o-proj and down-proj into the residual stream; with TSTORE
                       // a TMA reduce-add over tmC, which then maps the residual)
  EPI_SWIGLU = 7,      // columns come as 32 gate / 32 up pairs: act = silu(gate) * up -> bf16
  EPI_QKV = 8,         // q / k heads: RMSNorm over the head + weight + RoPE -> bf16; v heads -> bf16 V^T
  EPI_CONV_QNHWC = 9,  // requantised int8 / uint8, channels-last [N, H, W, Co]
};

// Geometry of the fused q/k/v projection (Qwen3-0.6B): 16 q heads, 8 k heads, 8 v heads of 128.
constexpr int kHeadDim = 128;
constexpr int kQCols = 16 * kHeadDim;
constexpr int kKCols = 8 * kHeadDim;

// n / d for 32-bit n and a divisor d >= 2 fixed at launch: t = umulhi(n, m), n / d = (t + ((n - t) >> 1))
// >> (l - 1), with l = ceil(log2 d) and m = floor(2^32 (2^l - d) / d) + 1 (Granlund and Montgomery,
// "Division by invariant integers using multiplication", 1994, section 4).
struct FastDiv {
  uint32_t d, m, l;
};
inline FastDiv make_fastdiv(uint32_t d) {
  uint32_t l = 0;
  while ((uint64_t(1) << l) < d) ++l;
  const uint64_t m = ((uint64_t(1) << 32) * ((uint64_t(1) << l) - d)) / d + 1;
  return FastDiv{d, static_cast<uint32_t>(m), l};
}
__device__ __forceinline__ uint32_t fast_div(uint32_t n, const FastDiv& f) {
  const uint32_t t = __umulhi(n, f.m);
  return (t + ((n - t) >> 1)) >> (f.l - 1);
}

struct GemmArgs {
  int M, N;            // output rows (GEMM rows, or bordered pixels for the conv) and columns
  int num_kb;          // 128-byte K blocks per tile
  int m_tiles, n_tiles;
  // conv geometry
  int cblocks;         // 128-channel blocks per tap
  int ntaps;           // taps of the stencil: 9 (3x3), or 1 (a 1x1 conv over the bordered layout, or taps
                       // packed into channels)
  int tap_off[9];      // per tap, the row offset of its input pixel from the output pixel's row in the [pixels,
                       // Cp] activation matrix: (ky-1)(W+2) + (kx-1) for a stride-1 3x3 conv; for a stride-2
                       // conv, whose input is split into phase planes, the plane's first row plus the offset
  int Wp, HWp;         // W + 2, (H + 2) * (W + 2) of the output's bordered geometry
  int H, W;
  FastDiv div_wp, div_hwp;
  // epilogue
  void* out;
  int64_t ldo;         // leading dimension of `out` in elements (GEMM modes)
  int out_dtype;
  int vec_ok;          // `out` rows allow 16-byte vector stores (direct-store path)
  const float* sx;
  const float* sw;     // per-column weight scale (GEMM) / requantise scale (conv)
  const void* bias;
  int bias_dtype;
  int shift, relu;     // relu: ReLU in the requantise (uint8 saturation)
  int post_relu;       // EPI_CONV_DEQ: max(y, 0) after the bias
  int* acc_max;
  // EPI_CONV_QNHWC with the next layer's maxima (XDNA_CONV_NEXT_AMAX): per image, the bit pattern of the max
  // |y| of the values the codes stand for, y = float(q) * (sw[c] * sx[n]) (+ bias[c]) (then max(y, 0) with
  // next_relu), over output rows < next_h and columns < next_w (a 2x2 pool's region); nullptr: not wanted
  uint32_t* next_amax;
  int next_relu, next_h, next_w;
  const int32_t* bias_i32;  // XDNA_CONV_BIAS_INT32: [N images, Co], added to the sums before the requantise
  int* err;
  // stack epilogues
  float* resid;        // EPI_RESID: [M, ldr] f32, updated in place
  int64_t ldr;
  __nv_bfloat16* vt;   // EPI_QKV: V^T [8 * 128, ldvt] bf16 (row = v head * 128 + d; column = sequence *
                       // round_up(seq_len, 8) + position)
  int64_t ldvt;
  const float* rope_cos;  // EPI_QKV: [seq_len, 64] f32 tables for positions 0..seq_len-1
  const float* rope_sin;
  const float* q_norm;    // EPI_QKV: [128] f32 per-head RMSNorm weights
  const float* k_norm;
  int seq_len;         // token m sits at position m % seq_len of its sequence
  float eps;
  int vt_tma;          // EPI_QKV: V^T through TMA stores (seq_len % 32 == 0)
  // LOAD_GEMM with the A rows split over several buffers (e.g. every rank's hidden states, read over
  // NVLink from the GPU that holds them): tensor maps in global memory, rows [i * a_rows, (i + 1) *
  // a_rows) of A from a_maps[i]; nullptr: A is tmA
  const CUtensorMap* a_maps;
  int a_rows;
};

constexpr int kBM = 128;
constexpr int kBKBytes = 128;  // one 128-byte swizzle row per operand row per stage (64 for convs of <= 64
                               // input channels, whose rows are 64 bytes)
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kStageOutBytes = 4096;  // per epilogue warp: two 2 KB TMA-store slots (or one 4 KB scratch)
constexpr int kStageSlotBytes = 2048; // 32 rows x 64 bytes
constexpr int kGroupM = 8;     // tile raster: GROUP_M m-tiles share a column of n-tiles (L2 reuse)
constexpr unsigned kFull = 0xffffffffu;

__host__ __device__ constexpr uint32_t tmem_cols_for(int cols) {
  return cols <= 32 ? 32 : cols <= 64 ? 64 : cols <= 128 ? 128 : cols <= 256 ? 256 : 512;
}

// RB: 0 -- A and B per stage; 1 -- conv weights resident (9 taps), A per stage; 2 -- resident weights and a
// window of kBM + 2 A rows per stage that serves a ky's three kx taps, stored in whole 8-row swizzle atoms;
// 3 -- the same with rows of two K blocks (an image pair, LOAD_CONV_WIN2); 4 -- a window and three taps' B
// tiles per stage, nothing resident (LOAD_CONV_WINB).
__host__ __device__ constexpr int a_stage_rows(int RB) { return RB >= 2 ? kBM + 8 : kBM; }

// Operand bytes per stage (RB: A only, the weights are resident) and of the resident weights (9 taps).
template <int BN, int KB, int RB>
__host__ __device__ constexpr int stage_bytes() {
  return RB == 4 ? (a_stage_rows(RB) + 3 * BN) * KB : (a_stage_rows(RB) * (RB == 3 ? 2 : 1) + (RB ? 0 : BN)) * KB;
}
template <int BN, int KB, int RB>
__host__ __device__ constexpr int resident_bytes() {
  return RB && RB != 4 ? 9 * BN * KB : 0;
}

// Operand stages in 224 KB less the epilogue's staging (8 x OUTB) and any resident weights, at most 12:
// with 4 KB per epilogue warp 4 / 6 / 8 stages for BN = 256 / 128 / 64 and 128-byte K blocks.
template <int BN, int KB = kBKBytes, int OUTB = kStageOutBytes, int RB = 0>
__host__ __device__ constexpr int stages_for() {
  return (224 * 1024 - kEpiWarps * OUTB - resident_bytes<BN, KB, RB>()) / stage_bytes<BN, KB, RB>() < 12
             ? (224 * 1024 - kEpiWarps * OUTB - resident_bytes<BN, KB, RB>()) / stage_bytes<BN, KB, RB>()
             : 12;
}

template <int BN, int KB = kBKBytes, int OUTB = kStageOutBytes, int RB = 0>
__host__ __device__ constexpr int smem_bytes_for() {
  return stages_for<BN, KB, OUTB, RB>() * stage_bytes<BN, KB, RB>() + resident_bytes<BN, KB, RB>() + kEpiWarps * OUTB +
         1024 /*align*/ + 256 /*barriers*/;
}

// Shared memory per epilogue warp: 8 KB where the epilogue keeps the tile's column factors (for the conv
// also its pixels' output offsets; for the q/k/v projection the head's RMSNorm weights) beside two
// staging slots, as long as the operand ring keeps at least 5 stages; 4 KB otherwise (one slot, or
// factors by warp shuffles).
template <int BROWS, int KB, int EPI, bool PAIR, int RB = 0>
__host__ __device__ constexpr int stage_out_bytes() {
  return ((EPI == EPI_CONV_DEQ || (PAIR && (EPI == EPI_DEQ || EPI == EPI_QKV))) && stages_for<BROWS, KB, 8192, RB>() >= 5)
             ? 8192
             : kStageOutBytes;
}

// Tiles of M rows per CTA (pair) and whether a GEMM of m_tiles128 128-row tiles x n_tiles 256-column
// tiles runs on CTA pairs: 256 x 256 tiles halve each CTA's share of B and cut its operand traffic by a
// third, worth it once the pairs still cover every SM.
inline bool use_pairs(int bn, int64_t m_tiles128, int64_t n_tiles, int sms) {
  return bn == 256 && ((m_tiles128 + 1) / 2) * n_tiles >= sms / 2;
}

__device__ __forceinline__ void tile_coords(int t, int m_tiles, int n_tiles, int& mb, int& nb) {
  const int per_group = kGroupM * n_tiles;
  const int g = t / per_group;
  const int first = g * kGroupM;
  const int gm = min(kGroupM, m_tiles - first);
  const int r = t - g * per_group;
  mb = first + r % gm;
  nb = r / gm;
}

__device__ __forceinline__ float load_as_float(const void* p, int dtype, int i) {
  if (dtype == XDNA_F32) return static_cast<const float*>(p)[i];
  if (dtype == XDNA_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(static_cast<const __half*>(p)[i]);
}

__device__ __forceinline__ uint32_t pack2(float a, float b, int dtype) {
  if (dtype == XDNA_BF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void store_one(void* out, int dtype, int64_t off, float v) {
  if (dtype == XDNA_F32)
    static_cast<float*>(out)[off] = v;
  else if (dtype == XDNA_BF16)
    static_cast<__nv_bfloat16*>(out)[off] = __float2bfloat16_rn(v);
  else
    static_cast<__half*>(out)[off] = __float2half_rn(v);
}

// The requantise of the conv: round half up by an arithmetic shift, then saturate.
__device__ __forceinline__ int requant(int acc, int shift, int relu) {
  const int q = (acc + (1 << (shift - 1))) >> shift;
  return relu ? min(max(q, 0), 255) : min(max(q, -128), 127);
}

// Four requantised codes in one word (byte i = code of acc[i]): the arithmetic shift of requant, the
// saturation to [-128, 127] (or [0, 255] with relu) done by cvt.pack.sat, which converts two s32 to 8 bits
// each into the word's low 16 bits (the first operand above the second) and copies its third operand's low
// 16 bits above them.
template <bool RELU>
__device__ __forceinline__ uint32_t requant_pack4(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, int rnd,
                                                  int shift) {
  const int q0 = (static_cast<int>(a0) + rnd) >> shift, q1 = (static_cast<int>(a1) + rnd) >> shift;
  const int q2 = (static_cast<int>(a2) + rnd) >> shift, q3 = (static_cast<int>(a3) + rnd) >> shift;
  uint32_t hi, w;
  if constexpr (RELU) {
    asm("cvt.pack.sat.u8.s32.b32 %0, %1, %2, 0;" : "=r"(hi) : "r"(q3), "r"(q2));
    asm("cvt.pack.sat.u8.s32.b32 %0, %1, %2, %3;" : "=r"(w) : "r"(q1), "r"(q0), "r"(hi));
  } else {
    asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, 0;" : "=r"(hi) : "r"(q3), "r"(q2));
    asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(w) : "r"(q1), "r"(q0), "r"(hi));
  }
  return w;
}

// 32 accumulators of one row -> 32 dequantised floats. Column factors: lane j holds column j's.
__device__ __forceinline__ void dequant32(const uint32_t (&r)[32], float srow, float sw_lane, float b_lane,
                                          bool has_bias, float (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const float w = __shfl_sync(kFull, sw_lane, j);
    v[j] = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[j])), srow), w);
  }
  if (has_bias) {  // warp-uniform
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(v[j], __shfl_sync(kFull, b_lane, j));
  }
}

// Per-warp staging for TMA stores: two 2 KB slots used in turn, so that the shared-memory writes of
// one block overlap the TMA store still reading the previous one. Lane 0 issues and commits every
// store of the warp (one bulk group each), so "at most one group still reading" frees the older slot.
struct StageRing {
  uint8_t* base;
  int slot;
  int nslots;  // 2, or 1 where the second 2 KB holds the warp's column factors (EPI_DEQ)
  __device__ __forceinline__ uint8_t* acquire() {
    if (lane_id() == 0) {
      if (nslots == 2)
        bulk_wait_read_one();
      else
        bulk_wait_read_all();
    }
    __syncwarp();
    uint8_t* b = base + slot * kStageSlotBytes;
    if (nslots == 2) slot ^= 1;
    return b;
  }
};

// The same with the column factors in this warp's shared memory (sw, and bias as f32, for the 32
// columns of the chunk; every lane reads the same 16 bytes, a broadcast) and packed f32x2 products:
// per value one conversion, one packed multiply by sx and one by sw, each rounded as __fmul_rn, then
// the bias added as __fadd_rn. Cheaper than 32 shuffles per chunk.
__device__ __forceinline__ void dequant32_smem(const uint32_t (&r)[32], float srow, const float* sw, const float* bias,
                                               bool has_bias, float (&v)[32]) {
  const float4* sw4 = reinterpret_cast<const float4*>(sw);
  const float2 sx2 = make_float2(srow, srow);
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float4 f = sw4[q];
    float2 a0 = make_float2(__int2float_rn(static_cast<int>(r[4 * q])), __int2float_rn(static_cast<int>(r[4 * q + 1])));
    float2 a1 = make_float2(__int2float_rn(static_cast<int>(r[4 * q + 2])), __int2float_rn(static_cast<int>(r[4 * q + 3])));
    a0 = __fmul2_rn(__fmul2_rn(a0, sx2), make_float2(f.x, f.y));
    a1 = __fmul2_rn(__fmul2_rn(a1, sx2), make_float2(f.z, f.w));
    if (has_bias) {  // warp-uniform
      const float4 b = reinterpret_cast<const float4*>(bias)[q];
      a0 = __fadd2_rn(a0, make_float2(b.x, b.y));
      a1 = __fadd2_rn(a1, make_float2(b.z, b.w));
    }
    v[4 * q] = a0.x;
    v[4 * q + 1] = a0.y;
    v[4 * q + 2] = a1.x;
    v[4 * q + 3] = a1.y;
  }
}

// Writes this warp's 32 rows x 32 columns through 64-byte-swizzled staging and TMA stores. `words`
// holds this lane's row: 16 words (2-byte outputs: one 32-column block) or 32 words (4-byte outputs:
// two 16-column blocks). Every block is 32 rows x 64 bytes; the tensor map's box matches.
// REDUCE: the block is added to the destination (TMA reduce-add, f32) instead of stored.
template <int NWORDS, bool REDUCE = false>
__device__ __forceinline__ void stage_and_store(StageRing& ring, const uint32_t (&words)[NWORDS],
                                                const CUtensorMap* tmC, int x, int y) {
  static_assert(NWORDS == 16 || NWORDS == 32, "2-byte or 4-byte outputs");
  const int lane = lane_id();
  const int sw = (lane >> 1) & 3;  // TMA 64-byte swizzle: 16-byte chunk ^ address bits 7..8
#pragma unroll
  for (int h = 0; h < NWORDS / 16; ++h) {
    uint8_t* buf = ring.acquire();
    uint8_t* row = buf + lane * 64;
#pragma unroll
    for (int k = 0; k < 4; ++k)
      *reinterpret_cast<uint4*>(row + ((k ^ sw) * 16)) =
          make_uint4(words[16 * h + 4 * k], words[16 * h + 4 * k + 1], words[16 * h + 4 * k + 2],
                     words[16 * h + 4 * k + 3]);
    fence_async_smem();
    __syncwarp();
    if (lane == 0) {
      if constexpr (REDUCE)
        tma_reduce_add_2d(tmC, buf, x + h * 16, y);
      else
        tma_store_2d(tmC, buf, x + h * 16, y);
      bulk_commit();
    }
  }
}

// 2-byte outputs on CTA-pair tiles: two consecutive 32-column chunks form one 32-row x 128-byte block of the
// warp's staging (128-byte swizzle: 16-byte chunk j of row r at position j ^ (r & 7), conflict-free), written
// by one TMA store once both halves are in -- or after the left half alone when the right one lies past the
// output's last column (the tensor map clips it). Half the store rows of 64-byte blocks: the TMA unit that
// issues every operand load of the mainloop spends its time per row, and the output's rows were most of it.
// buf: 4 KB, 1024-byte aligned; the tensor map's box is 32 rows x 128 bytes with SWIZZLE_128B.
__device__ __forceinline__ void stage_wide(uint8_t* buf, const uint32_t (&w)[16], int half, bool flush,
                                           const CUtensorMap* tmC, int x0, int y) {
  const int lane = lane_id();
  if (half == 0) {  // the previous block's store has finished reading the staging
    if (lane == 0) bulk_wait_read_all();
    __syncwarp();
  }
#pragma unroll
  for (int k = 0; k < 4; ++k)
    *reinterpret_cast<uint4*>(buf + lane * 128 + (((4 * half + k) ^ (lane & 7)) * 16)) =
        make_uint4(w[4 * k], w[4 * k + 1], w[4 * k + 2], w[4 * k + 3]);
  if (flush) {
    fence_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(tmC, buf, x0, y);
      bulk_commit();
    }
  }
}

// Whether an epilogue stores through 32 x 128-byte blocks (stage_wide): CTA pairs, 2-byte outputs, and 4 KB of
// the warp's staging free of column factors. The host encodes the output's tensor map to match
// (wide_store_map).
template <int EPI, int ODT, bool PAIR, int OUTB>
__host__ __device__ constexpr bool wide_store() {
  return PAIR && ODT != XDNA_F32 && ODT != XDNA_I32 &&
         ((EPI == EPI_DEQ && OUTB == 8192) || EPI == EPI_F32ACC);
}
// The host side of the same choice (pair tiles of 256 columns, 2-byte output elements).
inline bool wide_store_map(int epi, bool pair, int out_bytes) {
  return pair && out_bytes == 2 && (epi == EPI_DEQ || epi == EPI_F32ACC);
}

// Direct (non-TMA) stores of one row's 32 values, for outputs TMA cannot address.
template <int EPI>
__device__ __forceinline__ void store_direct(const GemmArgs& a, int row, int n0, const uint32_t (&r)[32],
                                             const float (&v)[32]) {
  if (row >= a.M) return;
  const int valid = min(32, a.N - n0);
  const int64_t off = static_cast<int64_t>(row) * a.ldo + n0;
  if constexpr (EPI == EPI_I32) {
    int32_t* o = static_cast<int32_t*>(a.out) + off;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < valid) o[j] = static_cast<int>(r[j]);
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < valid) store_one(a.out, a.out_dtype, off + j, v[j]);
  }
}

// Where an epilogue thread's bordered pixel sits: image, bordered row and column, whether it is an
// output pixel (not on the border), and the image's activation scale (dequantise only). Computed
// before the thread waits for the accumulator, so the division and the scale load are off the
// critical path.
struct ConvPixel {
  int img, yp, xp;
  bool valid;
  float s;
};

template <int EPI>
__device__ __forceinline__ ConvPixel conv_pixel(const GemmArgs& a, int p) {
  ConvPixel px;
  const uint32_t up = static_cast<uint32_t>(p);
  px.img = static_cast<int>(fast_div(up, a.div_hwp));
  const uint32_t rem = up - static_cast<uint32_t>(px.img) * static_cast<uint32_t>(a.HWp);
  px.yp = static_cast<int>(fast_div(rem, a.div_wp));
  px.xp = static_cast<int>(rem) - px.yp * a.Wp;
  px.valid = p < a.M && px.yp >= 1 && px.yp <= a.H && px.xp >= 1 && px.xp <= a.W;
  px.s = 0.f;
  if constexpr (EPI == EPI_CONV_DEQ) {
    if (px.valid) px.s = __ldg(a.sx + px.img);
  }
  return px;
}

// Whether every value the codes stand for is >= 0 (a ReLU after the bias, or one in the requantise of a conv
// without a float bias), so that the largest code of a channel gives its largest |y|.
__device__ __forceinline__ bool next_nonneg(const GemmArgs& a) {
  return a.next_relu || (a.relu && a.bias == nullptr);
}

// The next conv's per-image max from this conv's codes (XDNA_CONV_NEXT_AMAX). The value a code stands for,
// y(q) = fl(fl(q) * fl(scale[c] * sx[n])) (+ bias[c]) (then max(y, 0)) -- the next layer's quantise rebuilds it
// with exactly these f32 operations -- never decreases as q grows, so per channel only the largest code of the
// warp's pixels (and the smallest, for values that may be negative) decides max |y|: one warp max per channel,
// then lane c evaluates y for channel n0 + c alone, and one atomicMax on the bit pattern per image the warp
// holds. qv: this pixel's requantised codes. The whole warp calls it.
__device__ __forceinline__ void conv_next_amax(const GemmArgs& a, const ConvPixel& px, int nvalid, const int (&qv)[32],
                                               float scale_lane, float bias_lane) {
  const bool in = px.valid && px.yp - 1 < a.next_h && px.xp - 1 < a.next_w;
  const bool nonneg = next_nonneg(a);  // y >= 0: the largest code gives the largest |y|
  const int img = in ? px.img : -1;
  // the warp's pixels may span several images (a tile crossing an image's end): one pass per image
  const int lo = __reduce_min_sync(kFull, in ? img : INT_MAX);
  const int hi = __reduce_max_sync(kFull, img);
  const int lane = lane_id();
  for (int i = lo; i <= hi; ++i) {  // warp-uniform; no pass when no pixel counts (hi < 0)
    const bool mine = img == i;
    int qmax = INT_MIN, qmin = INT_MAX;  // of channel n0 + lane over this warp's pixels of image i
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int mx = __reduce_max_sync(kFull, mine ? qv[j] : INT_MIN);
      qmax = lane == j ? mx : qmax;
      if (!nonneg) {  // warp-uniform
        const int mn = __reduce_min_sync(kFull, mine ? qv[j] : INT_MAX);
        qmin = lane == j ? mn : qmin;
      }
    }
    uint32_t m = 0;  // max |y| of channel n0 + lane, as bits (non-negative floats order like their bit patterns)
    if (lane < nvalid && qmax != INT_MIN) {
      const float t = __fmul_rn(scale_lane, __ldg(a.sx + i));
      auto abs_y = [&](int q) {
        float y = __fmul_rn(static_cast<float>(q), t);
        if (a.bias != nullptr) y = __fadd_rn(y, bias_lane);
        if (a.next_relu) y = y > 0.f ? y : 0.f;
        return __float_as_uint(y) & 0x7FFFFFFFu;
      };
      m = abs_y(qmax);
      if (!nonneg) m = max(m, abs_y(qmin));
    }
    const uint32_t mi = __reduce_max_sync(kFull, m);
    if (lane == 0 && mi != 0u) atomicMax(a.next_amax + i, mi);
  }
}

// XDNA_CONV_NEXT_AMAX for values >= 0 (next_nonneg), accumulated across tiles: each epilogue lane keeps, per
// channel of its chunks, the largest code of its pixels over the tiles it drains of one image and one column
// tile (in unsigned order: a signed code is stored as code + 128; with at most two chunks per warp two codes
// per word as 16-bit lanes -- word 2k holding channels 4k and 4k + 2, word 2k + 1 channels 4k + 1 and 4k + 3 --
// so that the merge is the packed 16-bit max; with four chunks, where registers are short, four codes per
// word and __vmaxu4), and the warp combines
// them and evaluates y once per channel when the image or the column tile changes and after the last tile --
// instead of a warp reduction per channel per tile. img < 0: nothing held. sc / bi: this lane's channel
// scale and bias for each chunk; sx: the image's scale.
template <int NCH>
struct NextMax {
  static constexpr int kWords = NCH <= 2 ? 16 : 8;  // per chunk: 16-bit lanes, or 8-bit lanes
  int img, nb;
  float sx;
  uint32_t w[NCH][kWords];
  float sc[NCH], bi[NCH];
};

// Combine a NextMax over the warp and raise the image's max (the whole warp calls it). col0: the first
// column of the warp's chunks in the held column tile.
template <int NCH>
__device__ __forceinline__ void next_max_flush(const GemmArgs& a, const NextMax<NCH>& nm, int col0) {
  const int lane = lane_id();
  uint32_t best = 0;  // max |y| over this lane's channels, as bits (non-negative floats order like them)
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    const int n0 = col0 + c * 32;
    if (n0 < a.N) {  // warp-uniform
      constexpr int W = NextMax<NCH>::kWords;
      uint32_t w[W];
#pragma unroll
      for (int k = 0; k < W; ++k) w[k] = nm.w[c][k];
#pragma unroll
      for (int s = 16; s >= 1; s >>= 1) {
#pragma unroll
        for (int k = 0; k < W; ++k)
          w[k] = W == 16 ? __vmaxu2(w[k], __shfl_xor_sync(kFull, w[k], s)) : __vmaxu4(w[k], __shfl_xor_sync(kFull, w[k], s));
      }
      // every lane holds the 32 channels' largest codes; lane j takes channel n0 + j: 16-bit lanes: word
      // 2 (j / 4) + j % 2, lane (j % 4) / 2; 8-bit lanes: word j / 4, byte j % 4
      const int sel = W == 16 ? 2 * (lane >> 2) + (lane & 1) : lane >> 2;
      uint32_t word = w[0];
#pragma unroll
      for (int k = 1; k < W; ++k) word = sel == k ? w[k] : word;
      const int u = static_cast<int>((word >> (W == 16 ? 16 * ((lane >> 1) & 1) : 8 * (lane & 3))) & 0xFFu);
      const int q = a.relu ? u : u - 128;
      if (lane < a.N - n0) {
        float y = __fmul_rn(static_cast<float>(q), __fmul_rn(nm.sc[c], nm.sx));
        if (a.bias != nullptr) y = __fadd_rn(y, nm.bi[c]);
        if (a.next_relu) y = y > 0.f ? y : 0.f;
        best = max(best, __float_as_uint(y) & 0x7FFFFFFFu);
      }
    }
  }
  best = __reduce_max_sync(kFull, best);
  if (lane == 0 && best != 0u) atomicMax(a.next_amax + nm.img, best);
}

// Per tile (the whole warp): how the next layer's maxima of this warp's pixels are taken -- *mode 1: folded
// into nm (flushed first when nm holds another image or column tile), 2: reduced at once (pixels of two
// images, or values that may be negative), 0: no pixel counts -- and whether this lane's pixel counts (*in).
// col_base_held: the first column of the warp's chunks in the column tile nm holds; sc / bi: this lane's
// channel factors in column tile nb.
template <int NCH>
__device__ __forceinline__ void next_max_prepare(const GemmArgs& a, const ConvPixel& px, NextMax<NCH>& nm, int nb,
                                                 int col_base_held, const float (&sc)[NCH], const float (&bi)[NCH],
                                                 int* mode, bool* in) {
  *mode = 0;
  *in = px.valid && px.yp - 1 < a.next_h && px.xp - 1 < a.next_w;
  if (!next_nonneg(a)) {
    *mode = 2;
    return;
  }
  const int img = *in ? px.img : -1;
  const int lo = __reduce_min_sync(kFull, *in ? img : INT_MAX);
  const int hi = __reduce_max_sync(kFull, img);
  if (hi < 0) return;  // no pixel of this warp counts
  if (nm.img >= 0 && (lo != nm.img || hi != nm.img || nb != nm.nb)) {
    next_max_flush(a, nm, col_base_held);
    nm.img = -1;
  }
  if (lo != hi) {
    *mode = 2;  // the warp's pixels span two images
    return;
  }
  if (nm.img < 0) {
    nm.img = lo;
    nm.nb = nb;
    nm.sx = __ldg(a.sx + lo);
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      nm.sc[c] = sc[c];
      nm.bi[c] = bi[c];
#pragma unroll
      for (int k = 0; k < NextMax<NCH>::kWords; ++k) nm.w[c][k] = 0u;
    }
  }
  *mode = 1;
}

// XDNA_CONV_BIAS_INT32: the sums of this lane's pixel, channels n0..n0+31, plus the image's int32 bias row.
__device__ __forceinline__ void add_bias_i32(const GemmArgs& a, const ConvPixel& px, int n0, uint32_t (&r)[32]) {
  if (!px.valid) return;
  const int32_t* b = a.bias_i32 + static_cast<int64_t>(px.img) * a.N + n0;
  if (n0 + 32 <= a.N && (a.N & 3) == 0) {  // 16-byte aligned rows
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      const int4 v = __ldg(reinterpret_cast<const int4*>(b + j));
      r[j] += static_cast<uint32_t>(v.x);
      r[j + 1] += static_cast<uint32_t>(v.y);
      r[j + 2] += static_cast<uint32_t>(v.z);
      r[j + 3] += static_cast<uint32_t>(v.w);
    }
  } else {
    const int nvalid = min(32, a.N - n0);
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < nvalid) r[j] += static_cast<uint32_t>(__ldg(b + j));
  }
}

// Conv epilogues: one thread, one bordered pixel, channels n0..n0+31 in r[].
// nm_mode (EPI_CONV_QNHWC with XDNA_CONV_NEXT_AMAX): 1 fold the codes of the pixels in the next layer's
// region (nm_in) into nm_acc (NextMax), 2 reduce this chunk's maxima at once (conv_next_amax), 0 neither.
template <int EPI, int NW>
__device__ __forceinline__ void conv_chunk(const GemmArgs& a, const ConvPixel& px, int n0, const uint32_t (&r)[32],
                                           float scale_lane, float bias_lane, uint8_t* stage, int nm_mode,
                                           bool nm_in, uint32_t (&nm_acc)[NW]) {
  const int img = px.img;
  const int yp = px.yp;
  const int xp = px.xp;
  const bool valid = px.valid;
  const int nvalid = min(32, a.N - n0);
  if constexpr (EPI == EPI_CONV_CALIB) {
    int best = 0;
    if (valid) {
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (j < nvalid) {
          const int acc = static_cast<int>(r[j]);
          best = max(best, a.relu ? acc : abs(acc));
        }
      }
    }
    best = __reduce_max_sync(kFull, best);
    if (lane_id() == 0 && best > 0) atomicMax(a.acc_max, best);
  } else if constexpr (EPI == EPI_CONV_QNHWC) {
    uint32_t w[8];  // this pixel's codes, four per word
    const int rnd = 1 << (a.shift - 1);
    if (a.relu) {  // warp-uniform
#pragma unroll
      for (int k = 0; k < 8; ++k) w[k] = requant_pack4<true>(r[4 * k], r[4 * k + 1], r[4 * k + 2], r[4 * k + 3], rnd, a.shift);
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) w[k] = requant_pack4<false>(r[4 * k], r[4 * k + 1], r[4 * k + 2], r[4 * k + 3], rnd, a.shift);
    }
    if (nm_mode == 1) {  // warp-uniform
      const uint32_t flip = a.relu ? 0u : 0x80808080u;  // signed codes in unsigned order
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t x = nm_in ? (w[k] ^ flip) : 0u;
        if constexpr (NW == 16) {
          nm_acc[2 * k] = __vmaxu2(nm_acc[2 * k], __byte_perm(x, 0u, 0x4240));          // bytes 0 and 2
          nm_acc[2 * k + 1] = __vmaxu2(nm_acc[2 * k + 1], __byte_perm(x, 0u, 0x4341));  // bytes 1 and 3
        } else {
          nm_acc[k] = __vmaxu4(nm_acc[k], x);
        }
      }
    } else if (nm_mode == 2) {
      int qv[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) qv[j] = requant(static_cast<int>(r[j]), a.shift, a.relu);
      conv_next_amax(a, px, nvalid, qv, scale_lane, bias_lane);
    }
    if (!valid) return;
    // out[img, yp-1, xp-1, n0 ..]: this pixel's 32 codes are 32 contiguous bytes
    uint8_t* o = static_cast<uint8_t*>(a.out) + ((static_cast<int64_t>(img) * a.H + (yp - 1)) * a.W + (xp - 1)) * a.N + n0;
    if (nvalid == 32 && a.vec_ok) {
      reinterpret_cast<uint4*>(o)[0] = make_uint4(w[0], w[1], w[2], w[3]);
      reinterpret_cast<uint4*>(o)[1] = make_uint4(w[4], w[5], w[6], w[7]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < nvalid) o[j] = static_cast<uint8_t>(w[j >> 2] >> (8 * (j & 3)));
    }
  } else if constexpr (EPI == EPI_CONV_Q) {
    if (!valid) return;
    const int64_t HW = static_cast<int64_t>(a.H) * a.W;
    const int64_t base = (static_cast<int64_t>(img) * a.N + n0) * HW + static_cast<int64_t>(yp - 1) * a.W + (xp - 1);
    if (a.relu) {
      uint8_t* o = static_cast<uint8_t*>(a.out) + base;
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < nvalid) o[j * HW] = static_cast<uint8_t>(requant(static_cast<int>(r[j]), a.shift, 1));
    } else {
      int8_t* o = static_cast<int8_t*>(a.out) + base;
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < nvalid) o[j * HW] = static_cast<int8_t>(requant(static_cast<int>(r[j]), a.shift, 0));
    }
  } else {  // EPI_CONV_DEQ: q.float() * (scale[co] * sx[img]) (+ bias[co]), channels-last output
    const float s = px.s;
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int q = requant(static_cast<int>(r[j]), a.shift, a.relu);
      v[j] = __fmul_rn(static_cast<float>(q), __fmul_rn(__shfl_sync(kFull, scale_lane, j), s));
    }
    if (a.bias != nullptr) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(v[j], __shfl_sync(kFull, bias_lane, j));
    }
    if (a.post_relu) {  // after the bias; rounding to the output dtype keeps the order (monotone, 0 -> 0)
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = v[j] > 0.f ? v[j] : 0.f;
    }
    // out[img, yp-1, xp-1, co]: the 32 channels of this pixel are contiguous
    const int64_t base = ((static_cast<int64_t>(img) * a.H + (yp - 1)) * a.W + (xp - 1)) * a.N + n0;
    if (nvalid == 32 && a.vec_ok && stage != nullptr) {
      // through shared memory, so that each store instruction writes whole 128-byte lines: lane i first
      // parks its pixel's 32 values (row i, 16-byte chunks swizzled by i), then the warp writes 4 (f32)
      // or 8 (2-byte) pixels per instruction, one 16-byte chunk per lane
      const int lane = lane_id();
      const bool f32 = a.out_dtype == XDNA_F32;
      const int chunks = f32 ? 8 : 4;               // 16-byte chunks per pixel
      uint4* row = reinterpret_cast<uint4*>(stage) + lane * 8;
      if (f32) {
#pragma unroll
        for (int j = 0; j < 8; ++j)
          row[j ^ (lane & 7)] = make_uint4(__float_as_uint(v[4 * j]), __float_as_uint(v[4 * j + 1]),
                                           __float_as_uint(v[4 * j + 2]), __float_as_uint(v[4 * j + 3]));
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          row[j ^ (lane & 7)] = make_uint4(pack2(v[8 * j], v[8 * j + 1], a.out_dtype), pack2(v[8 * j + 2], v[8 * j + 3], a.out_dtype),
                                           pack2(v[8 * j + 4], v[8 * j + 5], a.out_dtype), pack2(v[8 * j + 6], v[8 * j + 7], a.out_dtype));
      }
      __syncwarp();
      const int per = 32 / chunks;                  // pixels per store instruction
      const int es = f32 ? 4 : 2;
#pragma unroll
      for (int it = 0; it < 8; ++it) {
        if (it < chunks) {                          // warp-uniform
          const int pi = it * per + lane / chunks;  // which of the warp's 32 pixels this lane writes
          const int ch = lane % chunks;
          const int64_t pbase = __shfl_sync(kFull, static_cast<long long>(base), pi);
          const bool pvalid = __shfl_sync(kFull, valid ? 1 : 0, pi) != 0;
          const uint4 val = reinterpret_cast<const uint4*>(stage)[pi * 8 + (ch ^ (pi & 7))];
          if (pvalid) *reinterpret_cast<uint4*>(static_cast<uint8_t*>(a.out) + pbase * es + ch * 16) = val;
        }
      }
      __syncwarp();
      return;
    }
    if (!valid) return;
    if (nvalid == 32 && a.vec_ok) {
      if (a.out_dtype == XDNA_F32) {
        float4* o = reinterpret_cast<float4*>(static_cast<float*>(a.out) + base);
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
      } else {
        uint4* o = reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.out) + base);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          o[j] = make_uint4(pack2(v[8 * j], v[8 * j + 1], a.out_dtype), pack2(v[8 * j + 2], v[8 * j + 3], a.out_dtype),
                            pack2(v[8 * j + 4], v[8 * j + 5], a.out_dtype), pack2(v[8 * j + 6], v[8 * j + 7], a.out_dtype));
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < nvalid) store_one(a.out, a.out_dtype, base + j, v[j]);
    }
  }
}

// EPI_CONV_DEQ for a full chunk of 32 channels (one pixel per lane), with the tile's channel scales
// and biases in this warp's shared memory (every lane reads the same 16 bytes, a broadcast). The
// requantise runs in integers; the int -> float conversion of q (|q| <= 255) is exact through the
// 1.5 * 2^23 bias: the bit pattern 0x4B400000 + q is the float 12582912 + q, from which 12582912 is
// subtracted exactly. Products and sums are packed f32x2 with the rounding of __fmul_rn / __fadd_rn:
// y = q * (scale[co] * s) (+ bias[co]) (then y > 0 ? y : 0), as conv_chunk computes.
// The 32 values are staged per pixel in swizzled rows, then the warp writes whole 128-byte lines with
// 16-byte stores, each pixel's output offset (-1: a border pixel) read from the tile's table.
__device__ __forceinline__ void conv_deq_smem(const GemmArgs& a, float s, int n0, const uint32_t (&r)[32],
                                              const float* scale, const float* bias, const long long* pix_off,
                                              uint8_t* stage) {
  const int lane = lane_id();
  const int shift = a.shift;
  const int rnd = 1 << (shift - 1);
  const int lo = a.relu ? 0 : -128;
  const int hi = a.relu ? 255 : 127;
  const float2 s2 = make_float2(s, s);
  const float2 unbias = make_float2(-12582912.f, -12582912.f);
  const bool has_bias = a.bias != nullptr;
  const bool relu_after = a.post_relu != 0;
  // four values (channels 4g .. 4g+3) at a time, staged as soon as they are done
  auto dq4 = [&](int g) {
    const float4 f = reinterpret_cast<const float4*>(scale)[g];
    int t[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      t[i] = min(max((static_cast<int>(r[4 * g + i]) + rnd) >> shift, lo), hi) + 0x4B400000;
    float2 a0 = __fadd2_rn(make_float2(__int_as_float(t[0]), __int_as_float(t[1])), unbias);
    float2 a1 = __fadd2_rn(make_float2(__int_as_float(t[2]), __int_as_float(t[3])), unbias);
    a0 = __fmul2_rn(a0, __fmul2_rn(make_float2(f.x, f.y), s2));
    a1 = __fmul2_rn(a1, __fmul2_rn(make_float2(f.z, f.w), s2));
    if (has_bias) {  // warp-uniform
      const float4 b = reinterpret_cast<const float4*>(bias)[g];
      a0 = __fadd2_rn(a0, make_float2(b.x, b.y));
      a1 = __fadd2_rn(a1, make_float2(b.z, b.w));
    }
    float4 o = make_float4(a0.x, a0.y, a1.x, a1.y);
    if (relu_after) {  // y > 0 ? y : 0 on the bits: positive floats are positive integers
      o.x = __int_as_float(max(__float_as_int(o.x), 0));
      o.y = __int_as_float(max(__float_as_int(o.y), 0));
      o.z = __int_as_float(max(__float_as_int(o.z), 0));
      o.w = __int_as_float(max(__float_as_int(o.w), 0));
    }
    return o;
  };
  const bool f32 = a.out_dtype == XDNA_F32;
  uint4* row = reinterpret_cast<uint4*>(stage) + lane * 8;
  if (f32) {
#pragma unroll
    for (int g = 0; g < 8; ++g) {
      const float4 o = dq4(g);
      row[g ^ (lane & 7)] = make_uint4(__float_as_uint(o.x), __float_as_uint(o.y), __float_as_uint(o.z), __float_as_uint(o.w));
    }
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 o0 = dq4(2 * j);
      const float4 o1 = dq4(2 * j + 1);
      row[j ^ (lane & 7)] = make_uint4(pack2(o0.x, o0.y, a.out_dtype), pack2(o0.z, o0.w, a.out_dtype),
                                       pack2(o1.x, o1.y, a.out_dtype), pack2(o1.z, o1.w, a.out_dtype));
    }
  }
  __syncwarp();
  const int lg = f32 ? 3 : 2;  // log2 of the 16-byte chunks per pixel
  const int es = f32 ? 4 : 2;
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    if (it < (1 << lg)) {  // warp-uniform
      const int pi = (it << (5 - lg)) + (lane >> lg);  // the pixel whose chunk this lane writes
      const int ch = lane & ((1 << lg) - 1);
      const long long off = pix_off[pi];
      const uint4 val = reinterpret_cast<const uint4*>(stage)[pi * 8 + (ch ^ (pi & 7))];
      if (off >= 0) *reinterpret_cast<uint4*>(static_cast<uint8_t*>(a.out) + (off + n0) * es + ch * 16) = val;
    }
  }
  __syncwarp();
}

// --------------------------------------------------------------------------- stack epilogues (bf16)
__device__ __forceinline__ float f32_of(uint32_t u) { return __uint_as_float(u); }

// One warp's half-tile of the fused q/k/v projection: exactly one head (128 columns) of its 32 rows.
// q and k heads (R:torch_xdna/stack.py:43-57; transformers' Qwen3 attention): per-head RMSNorm in f32
// (x * rsqrt(mean(x^2) + eps)) times the norm weight, then RoPE with the half rotation
// (out[d] = x[d] cos - x[d+64] sin, out[d+64] = x[d+64] cos + x[d] sin), stored bf16 through TMA.
// v heads are written transposed, V^T[head * 128 + d][token], the K-major operand of P.V.
__device__ __forceinline__ void qkv_tile(const GemmArgs& a, uint32_t taddr, int row0, int col0, StageRing& ring,
                                         const CUtensorMap* tmC, const CUtensorMap* tmD, float* wsm) {
  const int lane = lane_id();
  const int row = row0 + lane;
  if (row0 >= a.M) return;  // warp-uniform: no rows of this warp exist
  uint32_t x1[32], x2[32];
  if (col0 >= kQCols + kKCols) {  // a v head (warp-uniform)
    const int vh = (col0 - kQCols - kKCols) / kHeadDim;
    // V^T columns: each sequence starts at a multiple of 8 tokens (TMA reads them as 16-byte aligned boxes)
    const int l8 = (a.seq_len + 7) / 8 * 8;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      __syncwarp();
      tmem_ld_32x32b_x32(taddr + c * 32, x1);
      tmem_ld_wait();
      if (a.vt_tma) {
        // 32 dims x 32 tokens, transposed through shared memory, one TMA store; the warp's 32 rows are
        // consecutive positions of one sequence, so their V^T columns are row0 .. row0 + 31
        uint8_t* buf = ring.acquire();
        __nv_bfloat16* t = reinterpret_cast<__nv_bfloat16*>(buf);
#pragma unroll
        for (int j = 0; j < 32; ++j) t[j * 32 + lane] = __float2bfloat16_rn(f32_of(x1[j]));
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(tmD, buf, row0, vh * kHeadDim + c * 32);
          bulk_commit();
        }
      } else if (row < a.M) {
        const int64_t vcol = static_cast<int64_t>(row / a.seq_len) * l8 + row % a.seq_len;
        __nv_bfloat16* dst = a.vt + static_cast<int64_t>(vh * kHeadDim + c * 32) * a.ldvt + vcol;
#pragma unroll
        for (int j = 0; j < 32; ++j) dst[static_cast<int64_t>(j) * a.ldvt] = __float2bfloat16_rn(f32_of(x1[j]));
      }
    }
    return;
  }
  // pass 1: sum of squares over the head's 128 values (two packed partial sums)
  float2 ss2 = make_float2(0.f, 0.f);
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    __syncwarp();
    tmem_ld_32x32b_x32(taddr + c * 32, x1);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
      const float2 xv = make_float2(f32_of(x1[j]), f32_of(x1[j + 1]));
      ss2 = __ffma2_rn(xv, xv, ss2);
    }
  }
  const float rstd = rsqrtf((ss2.x + ss2.y) * (1.0f / kHeadDim) + a.eps);
  // the head's norm weights into this warp's shared memory: read back 4 at a time as a broadcast
  const float* nw = col0 < kQCols ? a.q_norm : a.k_norm;
  __syncwarp();  // this warp's reads of the previous head's weights are done
#pragma unroll
  for (int i = 0; i < 4; ++i) wsm[i * 32 + lane] = __ldg(nw + i * 32 + lane);
  __syncwarp();
  const float4* w4 = reinterpret_cast<const float4*>(wsm);
  const int pos = (row < a.M ? row : 0) % a.seq_len;
  // this row's RoPE table entries: the tables are [16][seq_len] float4 (four frequencies per vector,
  // positions fastest), so the warp's consecutive positions read consecutive 16-byte vectors
  const float4* cs4 = reinterpret_cast<const float4*>(a.rope_cos) + pos;
  const float4* sn4 = reinterpret_cast<const float4*>(a.rope_sin) + pos;
  const int64_t qstride = a.seq_len;  // float4s between one group of four frequencies and the next
  const float2 r2 = make_float2(rstd, rstd);
  // pass 2: columns d and d + 64 together (the RoPE pairs), 32 at a time, two neighbouring d per packed
  // f32x2 operation: u = x_d w_d rstd, v = x_{d+64} w_{d+64} rstd, out_d = u cos - v sin,
  // out_{d+64} = v cos + u sin
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    __syncwarp();
    tmem_ld_32x32b_x32(taddr + c * 32, x1);
    tmem_ld_32x32b_x32(taddr + 64 + c * 32, x2);
    tmem_ld_wait();
    uint32_t lo[16], hi[16];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 cv = __ldg(cs4 + (c * 8 + q) * qstride);
      const float4 sv = __ldg(sn4 + (c * 8 + q) * qstride);
      const float4 wa = w4[c * 8 + q];       // w[d .. d+3], d = 32 c + 4 q
      const float4 wb = w4[16 + c * 8 + q];  // w[d+64 .. d+67]
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int j = 4 * q + 2 * h;
        const float2 c2 = h ? make_float2(cv.z, cv.w) : make_float2(cv.x, cv.y);
        const float2 s2 = h ? make_float2(sv.z, sv.w) : make_float2(sv.x, sv.y);
        const float2 u = __fmul2_rn(__fmul2_rn(make_float2(f32_of(x1[j]), f32_of(x1[j + 1])),
                                               h ? make_float2(wa.z, wa.w) : make_float2(wa.x, wa.y)),
                                    r2);
        const float2 v = __fmul2_rn(__fmul2_rn(make_float2(f32_of(x2[j]), f32_of(x2[j + 1])),
                                               h ? make_float2(wb.z, wb.w) : make_float2(wb.x, wb.y)),
                                    r2);
        const float2 o_lo = __ffma2_rn(v, make_float2(-s2.x, -s2.y), __fmul2_rn(u, c2));
        const float2 o_hi = __ffma2_rn(u, s2, __fmul2_rn(v, c2));
        lo[q * 2 + h] = pack2(o_lo.x, o_lo.y, XDNA_BF16);
        hi[q * 2 + h] = pack2(o_hi.x, o_hi.y, XDNA_BF16);
      }
    }
    stage_and_store<16>(ring, lo, tmC, col0 + c * 32, row0);
    stage_and_store<16>(ring, hi, tmC, col0 + 64 + c * 32, row0);
  }
}

// One warp's half-tile of the fused gate/up projection. The packed weight interleaves 32 gate rows
// and the matching 32 up rows, so accumulator chunks 2p and 2p+1 are gate and up of the same 32
// output columns: act = silu(gate) * up (f32), stored bf16 at act column col0 / 2 + 32 p.
template <int NCH>
__device__ __forceinline__ void swiglu_tile(const GemmArgs& a, uint32_t taddr, int row0, int col0, StageRing& ring,
                                            const CUtensorMap* tmC) {
  uint32_t g[32], u[32];
#pragma unroll 1
  for (int p = 0; p < NCH / 2; ++p) {
    __syncwarp();
    tmem_ld_32x32b_x32(taddr + p * 64, g);
    tmem_ld_32x32b_x32(taddr + p * 64 + 32, u);
    tmem_ld_wait();
    uint32_t w[16];
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
      const float g0 = f32_of(g[j]), g1 = f32_of(g[j + 1]);
      const float a0 = g0 / (1.0f + expf(-g0)) * f32_of(u[j]);
      const float a1 = g1 / (1.0f + expf(-g1)) * f32_of(u[j + 1]);
      w[j / 2] = pack2(a0, a1, XDNA_BF16);
    }
    if (col0 / 2 + p * 32 < a.N / 2) stage_and_store<16>(ring, w, tmC, col0 / 2 + p * 32, row0);
  }
}

// --------------------------------------------------------------------------- the kernel
// ODT: the output element type of the GEMM epilogues, fixed at compile time (XDNA_I32 for EPI_I32).
template <int BN, int LOAD, int EPI, bool BF16, bool TSTORE, int ODT, int KB = kBKBytes, bool PAIR = false>
__global__ void __launch_bounds__(kThreads, 1)
    umma_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmD,
                     const __grid_constant__ GemmArgs args) {
  static_assert(KB == 128 || KB == 64, "K blocks of 128 or 64 bytes");
  static_assert(!PAIR || (BN == 256 && KB == 128), "CTA pairs: 256 x 256 tiles of 128-byte K blocks");
  constexpr int RBM = LOAD == LOAD_CONV_WINB ? 4 : LOAD == LOAD_CONV_WIN2 ? 3 : LOAD == LOAD_CONV_WIN ? 2
                    : LOAD == LOAD_CONV_RB ? 1 : 0;
  constexpr bool RB = RBM != 0 && RBM != 4;   // conv weights resident in shared memory
  constexpr bool WIN = RBM >= 2;              // one A window per ky serves its three kx taps
  constexpr bool WINB = RBM == 4;             // ... with the three taps' B tiles in the stage
  constexpr bool PIMG = RBM == 3;             // image pairs: two accumulators per tile
  constexpr int A_ROW = PIMG ? 2 * KB : KB;   // bytes of one A row in shared memory
  static_assert(!PIMG || (EPI == EPI_CONV_QNHWC && KB == 64 && !PAIR), "image pairs: 64-channel convs, codes out");
  static_assert(!WINB || (KB == 128 && (PAIR ? BN / 2 : BN) <= 128), "windows of 128-byte blocks, <= 128 B rows");
  constexpr bool kConv = LOAD != LOAD_GEMM;
  static_assert(!RB || (!PAIR && KB == 64 && BN <= 128), "resident conv weights: one 64-byte channel block, BN <= 128");
  constexpr int BROWS = PAIR ? BN / 2 : BN;  // B rows (tile columns) this CTA loads
  constexpr int OUTB = stage_out_bytes<BROWS, KB, EPI, PAIR, RBM>();
  constexpr int STAGES = stages_for<BROWS, KB, OUTB, RBM>();
  constexpr int A_BYTES = a_stage_rows(RBM) * A_ROW;  // WIN: kBM + 2 rows used, whole swizzle atoms kept
  constexpr int B_BYTES = BROWS * KB;        // one K block of B (one tap, for the conv)
  constexpr int B_STAGE = RB ? 0 : WINB ? 3 * B_BYTES : B_BYTES;  // B bytes in each ring stage
  // a pair's stage: both CTAs' bytes; WIN: the window's kBM + 2 rows
  constexpr uint32_t STAGE_TX = WINB ? (PAIR ? 2 : 1) * ((kBM + 2) * KB + B_STAGE)
                                : WIN ? (kBM + 2) * A_ROW : (PAIR ? 2 : 1) * (A_BYTES + B_STAGE);
  static_assert(!WIN || (A_BYTES % (8 * A_ROW) == 0), "window stages in whole swizzle atoms");
  constexpr int NACC = 2;  // accumulator buffers (four for 64-column pair tiles measured no faster)
  constexpr uint32_t TMEM_COLS = tmem_cols_for(NACC * BN * (PIMG ? 2 : 1));
  constexpr int MMA_M = PAIR ? 2 * kBM : kBM;
  constexpr uint32_t IDESC = BF16 ? idesc_bf16(MMA_M, BN) : idesc_i8(MMA_M, BN);
  constexpr int KSTEPS = KB / 32;  // one MMA consumes 32 bytes of K (32 int8 or 16 bf16)
  constexpr int K_ELEMS = BF16 ? KB / 2 : KB;
  // Epilogue groups: for the conv with resident weights, 64 output channels and int8 codes out (the first
  // layers of an image net: a tile is one or a few K blocks, so the epilogue sets the pace), warps 2-5 and
  // 6-9 drain alternate tiles, each group its own accumulator (group g: buffer g) and each warp all 64
  // columns of its 32 rows, so two tiles' epilogues overlap; an accumulator is released by four warps.
  constexpr bool kGroups = EPI == EPI_CONV_QNHWC && RBM == 1 && BN == 64 && !PAIR;
  constexpr int WCOLS = kGroups ? BN : BN / 2;  // columns per epilogue warp
  constexpr int NCH = WCOLS / 32;               // 32-column chunks per epilogue warp
  static_assert(NCH >= 1 && NCH <= 4, "BN must be 64, 128 or 256");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smem + STAGES * A_BYTES;
  uint8_t* smRes = smB + STAGES * B_STAGE;  // RB: the 9 taps' weights, B_BYTES each
  uint8_t* smOut = smRes + resident_bytes<BROWS, KB, RBM>();  // kEpiWarps x OUTB (1024-aligned unless WIN)
  uint64_t* full = reinterpret_cast<uint64_t*>(smOut + kEpiWarps * OUTB);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + NACC;
  uint64_t* drain = tempty + NACC;
  uint64_t* bres = drain + 1;  // RB: the resident weights have landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bres + 1);
  static_assert((2 * STAGES + 2 * NACC + 2) * 8 + 8 <= 256, "barrier area");
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  // CTA pairs: the even CTA (rank 0) issues the MMAs of a 256 x 256 tile whose rows 0..127 are its own
  // and rows 128..255 the odd CTA's; each CTA loads its own A rows and half of the B rows.
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  const int t_first = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int t_step = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  auto tile_row0 = [&](int mb) { return PAIR ? (2 * mb + static_cast<int>(rank)) * kBM : mb * kBM; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < NACC; ++b) {
      mbar_init(tfull + b, 1);
      mbar_init(tempty + b, PAIR ? 2 * kEpiWarps : kGroups ? kEpiWarps / 2 : kEpiWarps);  // a pair: both CTAs' warps
    }
    mbar_init(drain, 1);
    mbar_init(bres, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, TMEM_COLS);
      tmem_relinquish();
    }
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if constexpr (LOAD == LOAD_GEMM) {
      if (args.a_maps != nullptr)
        for (int i = 0; i * args.a_rows < args.M; ++i) tensormap_acquire(args.a_maps + i);
    }
    if constexpr (TSTORE) tma_prefetch_desc(&tmC);
  }
  tc_fence_before();
  if constexpr (PAIR)
    cluster_sync();  // both CTAs' barriers initialised and TMEM allocated before any cross-CTA arrival
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int total = args.m_tiles * args.n_tiles;
  // Convs walk one contiguous range of tiles per CTA (pair), so that an epilogue warp's consecutive tiles lie
  // in one image (the next layer's maxima are then combined once per image, not per tile); GEMMs interleave
  // the CTAs' tiles (t_first, t_first + t_step, ...).
  const int t_begin = kConv ? static_cast<int>(static_cast<int64_t>(t_first) * total / t_step) : t_first;
  const int t_end = kConv ? static_cast<int>(static_cast<int64_t>(t_first + 1) * total / t_step) : total;
  const int t_inc = kConv ? 1 : t_step;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------------- TMA producer
      int stage = 0;
      uint32_t phase = 0;
      int last_parity[STAGES];
#pragma unroll
      for (int s = 0; s < STAGES; ++s) last_parity[s] = -1;
      bool ok = true;
      if constexpr (RB) {  // the weights of all taps, once
        if (t_begin < t_end) {
          const int ntaps = args.ntaps;
          mbar_arrive_expect_tx(bres, ntaps * B_BYTES);
          for (int tap = 0; tap < ntaps; ++tap) tma_load_3d(smRes + tap * B_BYTES, &tmB, bres, 0, tap, 0);
        }
      }
      for (int t = t_begin; t < t_end && ok; t += t_inc) {
        int mb, nb;
        tile_coords(t, args.m_tiles, args.n_tiles, mb, nb);
        for (int kb = 0; kb < args.num_kb; ++kb) {
          if (!mbar_wait<PAIR>(empty + stage, phase ^ 1, abort_flag, args.err, 1)) {
            ok = false;
            break;
          }
          if constexpr (PAIR) {
            // both CTAs' bytes complete on the even CTA's barrier, which only it arms
            if (leader) mbar_arrive_expect_tx(full + stage, STAGE_TX);
            const uint32_t fb = cluster_addr(full + stage, 0);
            const int b_row = nb * BN + static_cast<int>(rank) * BROWS;  // this CTA's half of the B rows
            if constexpr (LOAD == LOAD_GEMM) {
              const int ar = tile_row0(mb);
              if (args.a_maps != nullptr)
                tma_load_2d_pair(smA + stage * A_BYTES, args.a_maps + ar / args.a_rows, fb, kb * K_ELEMS, ar % args.a_rows);
              else
                tma_load_2d_pair(smA + stage * A_BYTES, &tmA, fb, kb * K_ELEMS, ar);
              tma_load_2d_pair(smB + stage * B_BYTES, &tmB, fb, kb * K_ELEMS, b_row);
            } else if constexpr (WINB) {
              // K block kb: ky = kb / cblocks and channel block cb; the window from the row of tap (ky, 0),
              // the weights of taps 3 ky + 0, 1, 2
              const int ky = kb / args.cblocks;
              const int cb = kb - ky * args.cblocks;
              tma_load_2d_pair(smA + stage * A_BYTES, &tmA, fb, cb * K_ELEMS, tile_row0(mb) + args.tap_off[3 * ky]);
#pragma unroll
              for (int kx = 0; kx < 3; ++kx)
                tma_load_3d_pair(smB + stage * B_STAGE + kx * B_BYTES, &tmB, fb, cb * K_ELEMS, 3 * ky + kx, b_row);
            } else {
              const int tap = kb / args.cblocks;
              const int cb = kb - tap * args.cblocks;
              const int off = args.tap_off[tap];
              tma_load_2d_pair(smA + stage * A_BYTES, &tmA, fb, cb * K_ELEMS, tile_row0(mb) + off);
              tma_load_3d_pair(smB + stage * B_BYTES, &tmB, fb, cb * K_ELEMS, tap, b_row);
            }
          } else if constexpr (LOAD == LOAD_GEMM) {
            mbar_arrive_expect_tx(full + stage, STAGE_TX);
            if (args.a_maps != nullptr)
              tma_load_2d(smA + stage * A_BYTES, args.a_maps + (mb * kBM) / args.a_rows, full + stage, kb * K_ELEMS,
                          (mb * kBM) % args.a_rows);
            else
              tma_load_2d(smA + stage * A_BYTES, &tmA, full + stage, kb * K_ELEMS, mb * kBM);
            tma_load_2d(smB + stage * B_BYTES, &tmB, full + stage, kb * K_ELEMS, nb * BN);
          } else if constexpr (WINB) {
            mbar_arrive_expect_tx(full + stage, STAGE_TX);
            const int ky = kb / args.cblocks;
            const int cb = kb - ky * args.cblocks;
            tma_load_2d(smA + stage * A_BYTES, &tmA, full + stage, cb * K_ELEMS, mb * kBM + args.tap_off[3 * ky]);
#pragma unroll
            for (int kx = 0; kx < 3; ++kx)
              tma_load_3d(smB + stage * B_STAGE + kx * B_BYTES, &tmB, full + stage, cb * K_ELEMS, 3 * ky + kx, nb * BN);
          } else {
            mbar_arrive_expect_tx(full + stage, STAGE_TX);
            // WIN: K block kb is ky = kb, its window starting at the row of tap (ky, kx = 0)
            const int tap = WIN ? 3 * kb : kb / args.cblocks;
            const int cb = WIN ? 0 : kb - tap * args.cblocks;
            tma_load_2d(smA + stage * A_BYTES, &tmA, full + stage, cb * K_ELEMS, mb * kBM + args.tap_off[tap]);
            if constexpr (!RB) tma_load_3d(smB + stage * B_BYTES, &tmB, full + stage, cb * K_ELEMS, tap, nb * BN);
          }
          last_parity[stage] = static_cast<int>(phase);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Drain: the last load of every stage has landed before the CTA may exit (a no-op on the
      // normal path, where the MMA warp consumed them all). A pair's loads complete on the even CTA's
      // barriers, so the even CTA drains for both.
      for (int s = 0; s < STAGES; ++s)
        if (last_parity[s] >= 0 && leader) {
          volatile int never = 0;
          mbar_wait(full + s, static_cast<uint32_t>(last_parity[s]), &never, args.err, 2);
        }
      if constexpr (RB) {
        if (t_begin < t_end) {
          volatile int never = 0;
          mbar_wait(bres, 0, &never, args.err, 2);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------------------------------------------------------- MMA issuer
      int stage = 0;
      uint32_t phase = 0;
      int buf = 0;
      uint32_t bphase = 0;
      bool issued = false;
      bool ok = true;
      if constexpr (RB) {
        if (t_begin < t_end && !mbar_wait(bres, 0, abort_flag, args.err, 4)) ok = false;
      }
      for (int t = t_begin; t < t_end && ok; t += t_inc) {
        if (!mbar_wait<PAIR>(tempty + buf, bphase ^ 1, abort_flag, args.err, 3)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(buf * BN * (PIMG ? 2 : 1));
        for (int kb = 0; kb < args.num_kb; ++kb) {
          if (!mbar_wait<PAIR>(full + stage, phase, abort_flag, args.err, 4)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if constexpr (WINB) {
            // the three kx taps read the window from row kx on (128-byte rows) with their own weight tiles
#pragma unroll
            for (int kx = 0; kx < 3; ++kx) {
              const uint64_t da = smem_desc_k_sw128_at(smem_u32(smA + stage * A_BYTES + kx * KB));
              const uint64_t db = smem_desc_k_sw128(smem_u32(smB + stage * B_STAGE + kx * B_BYTES));
#pragma unroll
              for (int k = 0; k < KSTEPS; ++k) {
                const uint32_t acc = (kb | kx | k) != 0;
                if constexpr (PAIR)
                  umma_i8_pair(d, da + 2 * k, db + 2 * k, IDESC, acc);
                else
                  umma_i8(d, da + 2 * k, db + 2 * k, IDESC, acc);
              }
            }
          } else if constexpr (WIN) {
            // K block kb is ky = kb; its three kx taps read the window from row kx on (64-byte rows, so the
            // descriptor starts kx rows into the stage) and weights of tap 3 ky + kx
#pragma unroll
            for (int kx = 0; kx < 3; ++kx) {
              const uint64_t db = smem_desc_k_sw64(smem_u32(smRes + (3 * kb + kx) * B_BYTES));
              if constexpr (PIMG) {
                // 128-byte rows (128-byte swizzle): image 2i's K bytes 0..63, then image 2i+1's 64..127
                const uint64_t da = smem_desc_k_sw128_at(smem_u32(smA + stage * A_BYTES + kx * A_ROW));
#pragma unroll
                for (int w = 0; w < 2; ++w)
#pragma unroll
                  for (int k = 0; k < KSTEPS; ++k)
                    umma_i8(d + w * BN, da + 4 * w + 2 * k, db + 2 * k, IDESC, (kb | kx | k) != 0);
              } else {
                const uint64_t da = smem_desc_k_sw64_at(smem_u32(smA + stage * A_BYTES + kx * KB));
#pragma unroll
                for (int k = 0; k < KSTEPS; ++k) umma_i8(d, da + 2 * k, db + 2 * k, IDESC, (kb | kx | k) != 0);
              }
            }
          } else {
          const uint64_t da = KB == 128 ? smem_desc_k_sw128(smem_u32(smA + stage * A_BYTES))
                                        : smem_desc_k_sw64(smem_u32(smA + stage * A_BYTES));
          // RB: one channel block, so K block kb is tap kb
          uint8_t* const b_src = RB ? smRes + kb * B_BYTES : smB + stage * B_BYTES;
          const uint64_t db = KB == 128 ? smem_desc_k_sw128(smem_u32(b_src)) : smem_desc_k_sw64(smem_u32(b_src));
#pragma unroll
          for (int k = 0; k < KSTEPS; ++k) {
            const uint32_t acc = (kb | k) != 0;
            if constexpr (PAIR && BF16)
              umma_f16_pair(d, da + 2 * k, db + 2 * k, IDESC, acc);
            else if constexpr (PAIR)
              umma_i8_pair(d, da + 2 * k, db + 2 * k, IDESC, acc);
            else if constexpr (BF16)
              umma_f16(d, da + 2 * k, db + 2 * k, IDESC, acc);
            else
              umma_i8(d, da + 2 * k, db + 2 * k, IDESC, acc);
          }
          }
          if constexpr (PAIR)
            umma_commit_pair(empty + stage, 0x3);  // frees the stage in both CTAs
          else
            umma_commit(empty + stage);
          issued = true;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        if constexpr (PAIR)
          umma_commit_pair(tfull + buf, 0x3);
        else
          umma_commit(tfull + buf);
        if (++buf == NACC) {
          buf = 0;
          bphase ^= 1;
        }
      }
      // Drain: every MMA this thread issued has completed before TMEM is freed.
      if (issued) {
        if constexpr (PAIR)
          umma_commit_pair(drain, 0x1);
        else
          umma_commit(drain);
        volatile int never = 0;
        mbar_wait(drain, 0, &never, args.err, 5);
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2..9)
    const int ew = warp - 2;
    const int q = warp & 3;          // the TMEM lane quadrant this warp may read
    const int half = kGroups ? 0 : ew >> 2;   // which half of the tile's columns
    const int group = kGroups ? ew >> 2 : 0;  // with epilogue groups: which of the alternate tiles
    const int t_first_e = t_begin + group * t_inc;
    const int t_next = (kGroups ? 2 : 1) * t_inc;
    uint8_t* obuf = smOut + ew * OUTB;
    // The tile's column factors in shared memory: EPI_DEQ through TMA (with 4 KB per warp one staging
    // slot and the factors in the second 2 KB; with 8 KB two slots and the factors behind them) and
    // EPI_CONV_DEQ with 8 KB (4 KB of staging, the factors, then the 32 pixels' output offsets).
    constexpr bool kConvRows = EPI == EPI_CONV_DEQ && OUTB == 8192;
    constexpr bool kSmemFactors = (EPI == EPI_DEQ && TSTORE) || kConvRows;
    constexpr int kFactorOff = OUTB == 8192 ? 4096 : kStageSlotBytes;
    // 32 x 128-byte output blocks (stage_wide): the first 4 KB of the warp's area, factors behind them
    constexpr bool kWide = TSTORE && wide_store<EPI, ODT, PAIR, OUTB>();
    static_assert(!(TSTORE && PAIR && EPI == EPI_DEQ && ODT != XDNA_F32 && ODT != XDNA_I32) || kWide,
                  "the host encodes 32 x 128-byte output blocks for every pair tile with 2-byte outputs");
    static_assert(!kWide || (NCH % 2 == 0 && (!kSmemFactors || kFactorOff >= 4096)), "wide blocks: 4 KB of staging");
    // (EPI_QKV: the head's norm weights where the factors would be; with 4 KB, one staging slot)
    StageRing ring{obuf, 0, ((EPI == EPI_DEQ && TSTORE) || EPI == EPI_QKV) && OUTB == kStageOutBytes ? 1 : 2};
    float* col_sw = reinterpret_cast<float*>(obuf + kFactorOff);          // [WCOLS]
    float* col_bias = col_sw + WCOLS;                                      // [WCOLS]
    long long* pix_off = reinterpret_cast<long long*>(col_bias + WCOLS);  // kConvRows: [32]
    static_assert(!kSmemFactors || kFactorOff + 2 * WCOLS * 4 + 32 * 8 <= OUTB, "factor area");
    // hand an accumulator back to the MMA issuer (in a pair: the even CTA's, for both CTAs' warps)
    auto release_accumulator = [](uint64_t* bar) {
      if constexpr (PAIR)
        mbar_arrive_remote(cluster_addr(bar, 0));
      else
        mbar_arrive(bar);
    };
    const bool has_bias = args.bias != nullptr;
    int buf = group;
    uint32_t bphase = 0;
    // Per-row and per-column factors of a tile (and, for the conv, where its pixel sits). Loaded one
    // tile ahead: right after this warp's accumulator for tile t is ready, the loads for the next
    // tile are issued, and their latency passes while tile t is drained.
    struct Factors {
      float srow;
      float fcol[NCH], bcol[NCH];
      ConvPixel px;
    };
    auto load_factors = [&](int t) {
      Factors f{};
      int mb, nb;
      tile_coords(t, args.m_tiles, args.n_tiles, mb, nb);
      const int row = tile_row0(mb) + q * 32 + lane;
      const int col0 = nb * BN + half * WCOLS;
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        const int n = col0 + c * 32 + lane;
        f.fcol[c] = 0.f;
        f.bcol[c] = 0.f;
        if constexpr (EPI == EPI_DEQ || EPI == EPI_CONV_DEQ || EPI == EPI_CONV_QNHWC) {
          if (n < args.N && (EPI != EPI_CONV_QNHWC || args.next_amax != nullptr)) {
            f.fcol[c] = __ldg(args.sw + n);
            if (has_bias) f.bcol[c] = load_as_float(args.bias, args.bias_dtype, n);
          }
        }
        if constexpr (EPI == EPI_F32ACC) {
          if (n < args.N && has_bias) f.bcol[c] = load_as_float(args.bias, args.bias_dtype, n);
        }
      }
      if constexpr (EPI == EPI_DEQ) f.srow = row < args.M ? __ldg(args.sx + row) : 0.f;
      if constexpr (kConv) f.px = conv_pixel<EPI>(args, row);
      return f;
    };
    Factors fac{};
    if (t_first_e < t_end) fac = load_factors(t_first_e);
    NextMax<NCH> nm;  // EPI_CONV_QNHWC with XDNA_CONV_NEXT_AMAX
    nm.img = -1;
    nm.nb = 0;
    NextMax<NCH> nm1;  // PIMG: the odd images' maxima (nm: the even images')
    nm1.img = -1;
    nm1.nb = 0;
    for (int t = t_first_e; t < t_end; t += t_next) {
      int mb, nb;
      tile_coords(t, args.m_tiles, args.n_tiles, mb, nb);
      const int row0 = tile_row0(mb) + q * 32;
      const int row = row0 + lane;
      const int col0 = nb * BN + half * WCOLS;
      const float srow = fac.srow;
      float fcol[NCH], bcol[NCH];
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        fcol[c] = fac.fcol[c];
        bcol[c] = fac.bcol[c];
      }
      const ConvPixel px = fac.px;
      int nm_mode = 0;
      bool nm_in = false;
      if constexpr (EPI == EPI_CONV_QNHWC && !PIMG) {
        if (args.next_amax != nullptr)  // warp-uniform
          next_max_prepare(args, px, nm, nb, nm.nb * BN + half * WCOLS, fcol, bcol, &nm_mode, &nm_in);
      }
      if constexpr (kSmemFactors) {
        __syncwarp();  // this warp is done reading the previous tile's factors
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
          col_sw[c * 32 + lane] = fcol[c];
          col_bias[c * 32 + lane] = bcol[c];
        }
        if constexpr (kConvRows)  // out[img, yp-1, xp-1, 0] of this lane's pixel (channels-last), -1: border
          pix_off[lane] = px.valid ? ((static_cast<long long>(px.img) * args.H + (px.yp - 1)) * args.W + (px.xp - 1)) *
                                         args.N
                                   : -1ll;
        __syncwarp();
      }

      if (!mbar_wait<PAIR>(tfull + buf, bphase, abort_flag, args.err, 6)) break;
      tc_fence_after();
      if (t + t_next < t_end) fac = load_factors(t + t_next);
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(buf * BN + half * WCOLS);
      if constexpr (EPI == EPI_QKV || EPI == EPI_SWIGLU) {
        if (col0 < args.N) {  // warp-uniform
          if constexpr (EPI == EPI_QKV)
            qkv_tile(args, taddr, row0, col0, ring, &tmC, &tmD, col_sw);
          else
            swiglu_tile<NCH>(args, taddr, row0, col0, ring, &tmC);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) release_accumulator(tempty + buf);
      } else if constexpr (PIMG) {
        // two accumulators: the tile's pixels of image 2i (columns buf * 2BN ..) and of image 2i + 1 (+ BN)
#pragma unroll
        for (int w = 0; w < 2; ++w) {
          ConvPixel pw = px;
          pw.img = 2 * px.img + w;
          NextMax<NCH>& st = w == 0 ? nm : nm1;
          int mode = 0;
          bool in = false;
          if (args.next_amax != nullptr)  // warp-uniform
            next_max_prepare(args, pw, st, nb, st.nb * BN + half * WCOLS, fcol, bcol, &mode, &in);
#pragma unroll
          for (int c = 0; c < NCH; ++c) {
            uint32_t r[32];
            __syncwarp();
            tmem_ld_32x32b_x32(taddr + buf * BN + w * BN + c * 32, r);
            tmem_ld_wait();
            if (w == 1 && c + 1 == NCH) {  // every column of both accumulators is in registers
              tc_fence_before();
              __syncwarp();
              if (lane == 0) release_accumulator(tempty + buf);
            }
            const int n0 = col0 + c * 32;
            if (n0 < args.N) {  // warp-uniform
              if (args.bias_i32 != nullptr) add_bias_i32(args, pw, n0, r);
              conv_chunk<EPI>(args, pw, n0, r, fcol[c], bcol[c], obuf, mode, in, st.w[c]);
            }
          }
        }
      } else {
      uint32_t r[2][32];
      __syncwarp();
      tmem_ld_32x32b_x32(taddr, r[0]);
      tmem_ld_wait();
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        if (c + 1 < NCH) {
          __syncwarp();
          tmem_ld_32x32b_x32(taddr + (c + 1) * 32, r[(c + 1) & 1]);
        } else {
          // every column of this tile is in registers: hand the accumulator back to the MMA warp
          tc_fence_before();
          __syncwarp();
          if (lane == 0) release_accumulator(tempty + buf);
        }
        const int n0 = col0 + c * 32;
        // warp-uniform: this chunk has columns in range (and, for GEMM outputs, rows in range)
        if (n0 < args.N && (kConv || row0 < args.M)) {
          if constexpr (kConv) {
            if (args.bias_i32 != nullptr) add_bias_i32(args, px, n0, r[c & 1]);  // warp-uniform
          }
          const uint32_t(&rc)[32] = r[c & 1];
          if constexpr (EPI == EPI_I32 || EPI == EPI_DEQ) {
            if constexpr (TSTORE) {
              if constexpr (EPI == EPI_I32) {
                stage_and_store<32>(ring, rc, &tmC, n0, row0);
              } else {
                float v[32];
                if constexpr (kSmemFactors)
                  dequant32_smem(rc, srow, col_sw + c * 32, col_bias + c * 32, has_bias, v);
                else
                  dequant32(rc, srow, fcol[c], bcol[c], has_bias, v);
                if constexpr (ODT == XDNA_F32) {
                  uint32_t w[32];
#pragma unroll
                  for (int j = 0; j < 32; ++j) w[j] = __float_as_uint(v[j]);
                  stage_and_store<32>(ring, w, &tmC, n0, row0);
                } else {
                  uint32_t w[16];
#pragma unroll
                  for (int j = 0; j < 16; ++j) w[j] = pack2(v[2 * j], v[2 * j + 1], ODT);
                  if constexpr (kWide)
                    stage_wide(obuf, w, c & 1, (c & 1) || c + 1 == NCH || n0 + 32 >= args.N, &tmC,
                               n0 - 32 * (c & 1), row0);
                  else
                    stage_and_store<16>(ring, w, &tmC, n0, row0);
                }
              }
            } else {
              float v[32];
              if constexpr (EPI == EPI_DEQ) dequant32(rc, srow, fcol[c], bcol[c], has_bias, v);
              store_direct<EPI>(args, row, n0, rc, v);
            }
          } else if constexpr (EPI == EPI_F32ACC) {
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = f32_of(rc[j]);
            if (has_bias) {
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(v[j], __shfl_sync(kFull, bcol[c], j));
            }
            if constexpr (TSTORE) {
              if constexpr (ODT == XDNA_F32) {
                uint32_t w[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) w[j] = __float_as_uint(v[j]);
                stage_and_store<32>(ring, w, &tmC, n0, row0);
              } else {
                uint32_t w[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) w[j] = pack2(v[2 * j], v[2 * j + 1], ODT);
                if constexpr (kWide)
                  stage_wide(obuf, w, c & 1, (c & 1) || c + 1 == NCH || n0 + 32 >= args.N, &tmC,
                             n0 - 32 * (c & 1), row0);
                else
                  stage_and_store<16>(ring, w, &tmC, n0, row0);
              }
            } else {
              store_direct<EPI>(args, row, n0, rc, v);
            }
          } else if constexpr (EPI == EPI_RESID && TSTORE) {
            // resid[rows, n0..n0+31] += acc by a TMA reduce-add of the staged block (one f32 add per
            // element, in L2; rows and columns past the residual's extent are clipped)
            stage_and_store<32, true>(ring, rc, &tmC, n0, row0);
          } else if constexpr (EPI == EPI_RESID) {
            // resid[row, n0..n0+31] += acc: 128 contiguous bytes per thread
            if (row < args.M) {
              float* res = args.resid + static_cast<int64_t>(row) * args.ldr + n0;
              if (n0 + 32 <= args.N) {
#pragma unroll
                for (int j = 0; j < 32; j += 4) {
                  float4 o = *reinterpret_cast<float4*>(res + j);
                  o.x += f32_of(rc[j]);
                  o.y += f32_of(rc[j + 1]);
                  o.z += f32_of(rc[j + 2]);
                  o.w += f32_of(rc[j + 3]);
                  *reinterpret_cast<float4*>(res + j) = o;
                }
              } else {
                const int nv = args.N - n0;
#pragma unroll
                for (int j = 0; j < 32; ++j)
                  if (j < nv) res[j] += f32_of(rc[j]);
              }
            }
          } else if constexpr (kConvRows) {
            if (n0 + 32 <= args.N && args.vec_ok)  // warp-uniform
              conv_deq_smem(args, px.s, n0, rc, col_sw + c * 32, col_bias + c * 32, pix_off, obuf);
            else
              conv_chunk<EPI>(args, px, n0, rc, col_sw[c * 32 + lane], col_bias[c * 32 + lane], nullptr, 0, false,
                              nm.w[c]);
          } else {
            conv_chunk<EPI>(args, px, n0, rc, fcol[c], bcol[c], obuf, nm_mode, nm_in, nm.w[c]);
          }
        }
        if (c + 1 < NCH) tmem_ld_wait();
      }
      }  // generic chunk loop
      if constexpr (kGroups) {
        bphase ^= 1;  // this group's accumulator comes back every other tile
      } else if (++buf == NACC) {
        buf = 0;
        bphase ^= 1;
      }
    }
    if constexpr (EPI == EPI_CONV_QNHWC) {
      if (nm.img >= 0) next_max_flush(args, nm, nm.nb * BN + half * WCOLS);
      if constexpr (PIMG) {
        if (nm1.img >= 0) next_max_flush(args, nm1, nm1.nb * BN + half * WCOLS);
      }
    }
    if constexpr (TSTORE) {
      if (lane == 0) bulk_wait_all();
      __syncwarp();
    }
  }

  __syncthreads();
  // A pair: the even CTA's MMAs read this CTA's shared memory and write its TMEM, and this CTA's
  // warps arrive on the even CTA's barriers; neither may free or exit before both are done.
  if constexpr (PAIR) cluster_sync();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem_base, TMEM_COLS);
    else
      tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ----------------------------------------------------------------------------- host launcher
// Persistent grid: one CTA per SM, or (PAIR) as many 2-CTA clusters as can be resident at once, and
// never more CTAs (pairs) than tiles. args.m_tiles counts 256-row tiles for pairs.
// (static: its per-instantiation caches stay private to each translation unit and to this library)
template <int BN, int LOAD, int EPI, bool BF16, bool TSTORE, int ODT, int KB, bool PAIR>
static int launch_gemm_kernel(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                              const CUtensorMap& td, const GemmArgs& args, int sms, cudaStream_t stream) {
  constexpr int RB = LOAD == LOAD_CONV_WINB ? 4 : LOAD == LOAD_CONV_WIN2 ? 3 : LOAD == LOAD_CONV_WIN ? 2
                   : LOAD == LOAD_CONV_RB ? 1 : 0;
  constexpr int smem = smem_bytes_for<PAIR ? BN / 2 : BN, KB, stage_out_bytes<PAIR ? BN / 2 : BN, KB, EPI, PAIR, RB>(), RB>();
  auto kern = umma_gemm_kernel<BN, LOAD, EPI, BF16, TSTORE, ODT, KB, PAIR>;
  // per instantiation and device: resident pairs once the kernel is configured (0 = not yet). Two threads
  // configuring at once both set the same attribute and store the same count.
  static std::atomic<int> max_pairs[64];
  int dev = 0;
  XDNA_CUDA(cudaGetDevice(&dev));
  const int cached_pairs = dev >= 0 && dev < 64 ? max_pairs[dev].load(std::memory_order_acquire) : 0;
  int pairs_resident = sms / 2;
  if (cached_pairs == 0) {
    XDNA_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    if constexpr (PAIR) {
      cudaLaunchConfig_t cfg{};
      cudaLaunchAttribute attr{};
      attr.id = cudaLaunchAttributeClusterDimension;
      attr.val.clusterDim.x = 2;
      attr.val.clusterDim.y = 1;
      attr.val.clusterDim.z = 1;
      cfg.gridDim = dim3(static_cast<unsigned>(sms & ~1));
      cfg.blockDim = dim3(kThreads);
      cfg.dynamicSmemBytes = smem;
      cfg.attrs = &attr;
      cfg.numAttrs = 1;
      int n = 0;
      XDNA_CUDA(cudaOccupancyMaxActiveClusters(&n, kern, &cfg));
      pairs_resident = n > 0 ? n : 1;
    }
    if (dev >= 0 && dev < 64) max_pairs[dev].store(pairs_resident, std::memory_order_release);
  } else {
    pairs_resident = cached_pairs;
  }
  const int tiles = args.m_tiles * args.n_tiles;
  if constexpr (PAIR) {
    const int pairs = std::max(1, std::min(tiles, pairs_resident));
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr{};
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    XDNA_CUDA(cudaLaunchKernelEx(&cfg, kern, ta, tb, tc, td, args));
  } else {
    kern<<<std::max(1, std::min(tiles, sms)), kThreads, smem, stream>>>(ta, tb, tc, td, args);
  }
  return check_launch("umma_gemm_kernel");
}

}  // namespace xdna
