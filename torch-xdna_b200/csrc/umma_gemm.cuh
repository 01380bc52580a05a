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
//                 arithmetic. Per-column factors arrive once per tile as one coalesced load per lane
//                 and are broadcast with warp shuffles. GEMM outputs are staged in swizzled shared
//                 memory (4 KB per warp) and written by TMA bulk-tensor stores (full lines, tails
//                 clipped by the tensor map); conv outputs (NCHW scatter) use direct stores.
//
// The A operand is either a plain row-major matrix (LOAD_GEMM) or, for the conv, the
// zero-bordered NHWC activations viewed as a [pixels, Cp] matrix: the K loop runs over 9 taps x
// channel blocks and a tap is a constant row offset dy*(W+2)+dx into that matrix (LOAD_CONV);
// TMA's zero fill covers rows before the first / past the last pixel and channels past Cp.
#pragma once

#include "sm100.cuh"

namespace xdna {

enum LoadMode { LOAD_GEMM = 0, LOAD_CONV = 1 };

enum EpiMode {
  EPI_I32 = 0,         // int32 accumulators
  EPI_DEQ = 1,         // (float(acc) * sx[m]) * sw[n] (+ bias[n]) -> f32 / bf16 / f16
  EPI_CONV_Q = 2,      // requantised int8 / uint8, NCHW
  EPI_CONV_DEQ = 3,    // requantised then dequantised, NCHW
  EPI_CONV_CALIB = 4,  // max of the sums (of image 0) into one int32
  // bf16 GEMMs of the Qwen3 stack (f32 accumulators)
  EPI_F32ACC = 5,      // acc (+ bias[n]) -> f32 / bf16 / f16 (the head; precision="bf16" linears)
  EPI_RESID = 6,       // resid_f32[m, n] += acc (o-proj and down-proj into the residual stream)
  EPI_SWIGLU = 7,      // columns come as 32 gate / 32 up pairs: act = silu(gate) * up -> bf16
  EPI_QKV = 8,         // q / k heads: RMSNorm over the head + weight + RoPE -> bf16; v heads -> bf16 V^T
};

// Geometry of the fused q/k/v projection (Qwen3-0.6B): 16 q heads, 8 k heads, 8 v heads of 128.
constexpr int kHeadDim = 128;
constexpr int kQCols = 16 * kHeadDim;
constexpr int kKCols = 8 * kHeadDim;

struct GemmArgs {
  int M, N;            // output rows (GEMM rows, or bordered pixels for the conv) and columns
  int num_kb;          // 128-byte K blocks per tile
  int m_tiles, n_tiles;
  // conv geometry
  int cblocks;         // 128-channel blocks per tap
  int Wp, HWp;         // W + 2, (H + 2) * (W + 2)
  int H, W;
  // epilogue
  void* out;
  int64_t ldo;         // leading dimension of `out` in elements (GEMM modes)
  int out_dtype;
  int vec_ok;          // `out` rows allow 16-byte vector stores (direct-store path)
  const float* sx;
  const float* sw;     // per-column weight scale (GEMM) / requantise scale (conv)
  const void* bias;
  int bias_dtype;
  int shift, relu;
  int* acc_max;
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
};

constexpr int kBM = 128;
constexpr int kBKBytes = 128;  // one 128-byte swizzle row per operand row per stage
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kStageOutBytes = 4096;  // per epilogue warp: 32 rows x 32 columns x <= 4 bytes
constexpr int kGroupM = 8;     // tile raster: GROUP_M m-tiles share a column of n-tiles (L2 reuse)
constexpr unsigned kFull = 0xffffffffu;

__host__ __device__ constexpr uint32_t tmem_cols_for(int cols) {
  return cols <= 32 ? 32 : cols <= 64 ? 64 : cols <= 128 ? 128 : cols <= 256 ? 256 : 512;
}

template <int BN>
__host__ __device__ constexpr int stages_for() {
  return BN >= 256 ? 4 : BN >= 128 ? 6 : 8;
}

template <int BN>
__host__ __device__ constexpr int smem_bytes_for() {
  return stages_for<BN>() * (kBM + BN) * kBKBytes + kEpiWarps * kStageOutBytes + 1024 /*align*/ +
         256 /*barriers*/;
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

// Writes one 32 x 32 output block (this warp's rows, 32 columns) through swizzled shared memory and
// a TMA store. `words` holds this lane's row: 16 words (2-byte outputs) or 32 words (4-byte outputs).
template <int NWORDS>
__device__ __forceinline__ void stage_and_store(uint8_t* buf, const uint32_t (&words)[NWORDS], const CUtensorMap* tmC,
                                                int x, int y) {
  const int lane = lane_id();
  if (lane == 0) bulk_wait_read_all();  // the previous store from this buffer has read it
  __syncwarp();
  constexpr int CHUNKS = NWORDS / 4;    // 16-byte chunks per row: 4 (64 B rows) or 8 (128 B rows)
  uint8_t* row = buf + lane * (CHUNKS * 16);
  const int sw = CHUNKS == 8 ? (lane & 7) : ((lane >> 1) & 3);  // TMA 128B / 64B swizzle pattern
#pragma unroll
  for (int k = 0; k < CHUNKS; ++k)
    *reinterpret_cast<uint4*>(row + ((k ^ sw) * 16)) =
        make_uint4(words[4 * k], words[4 * k + 1], words[4 * k + 2], words[4 * k + 3]);
  fence_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(tmC, buf, x, y);
    bulk_commit();
  }
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

// Conv epilogues: one thread, one bordered pixel `p`, channels n0..n0+31 in r[].
template <int EPI>
__device__ __forceinline__ void conv_chunk(const GemmArgs& a, int p, int n0, const uint32_t (&r)[32],
                                           float scale_lane, float bias_lane, uint8_t* stage) {
  const int img = p / a.HWp;
  const int rem = p - img * a.HWp;
  const int yp = rem / a.Wp;
  const int xp = rem - yp * a.Wp;
  const bool valid = p < a.M && yp >= 1 && yp <= a.H && xp >= 1 && xp <= a.W;
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
    const float s = valid ? a.sx[img] : 0.f;
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
#pragma unroll 1
      for (int it = 0; it < chunks; ++it) {
        const int px = it * per + lane / chunks;    // which of the warp's 32 pixels this lane writes
        const int ch = lane % chunks;
        const int64_t pbase = __shfl_sync(kFull, static_cast<long long>(base), px);
        const bool pvalid = __shfl_sync(kFull, valid ? 1 : 0, px) != 0;
        const uint4 val = reinterpret_cast<const uint4*>(stage)[px * 8 + (ch ^ (px & 7))];
        if (pvalid) *reinterpret_cast<uint4*>(static_cast<uint8_t*>(a.out) + pbase * es + ch * 16) = val;
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

// --------------------------------------------------------------------------- stack epilogues (bf16)
__device__ __forceinline__ float f32_of(uint32_t u) { return __uint_as_float(u); }

// One warp's half-tile of the fused q/k/v projection: exactly one head (128 columns) of its 32 rows.
// q and k heads (R:torch_xdna/stack.py:43-57; transformers' Qwen3 attention): per-head RMSNorm in f32
// (x * rsqrt(mean(x^2) + eps)) times the norm weight, then RoPE with the half rotation
// (out[d] = x[d] cos - x[d+64] sin, out[d+64] = x[d+64] cos + x[d] sin), stored bf16 through TMA.
// v heads are written transposed, V^T[head * 128 + d][token], the K-major operand of P.V.
__device__ __forceinline__ void qkv_tile(const GemmArgs& a, uint32_t taddr, int row0, int col0, uint8_t* obuf,
                                         const CUtensorMap* tmC, const CUtensorMap* tmD) {
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
        if (lane == 0) bulk_wait_read_all();
        __syncwarp();
        __nv_bfloat16* t = reinterpret_cast<__nv_bfloat16*>(obuf);
#pragma unroll
        for (int j = 0; j < 32; ++j) t[j * 32 + lane] = __float2bfloat16_rn(f32_of(x1[j]));
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(tmD, obuf, row0, vh * kHeadDim + c * 32);
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
  // pass 1: sum of squares over the head's 128 values
  float ss = 0.f;
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    __syncwarp();
    tmem_ld_32x32b_x32(taddr + c * 32, x1);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 32; ++j) ss = fmaf(f32_of(x1[j]), f32_of(x1[j]), ss);
  }
  const float rstd = rsqrtf(ss * (1.0f / kHeadDim) + a.eps);
  const float* nw = col0 < kQCols ? a.q_norm : a.k_norm;
  const float w_lane[4] = {nw[lane], nw[32 + lane], nw[64 + lane], nw[96 + lane]};
  const int pos = (row < a.M ? row : 0) % a.seq_len;
  // this row's RoPE table entries, 16 bytes at a time (rows are 256-byte aligned)
  const float4* cs4 = reinterpret_cast<const float4*>(a.rope_cos + static_cast<int64_t>(pos) * (kHeadDim / 2));
  const float4* sn4 = reinterpret_cast<const float4*>(a.rope_sin + static_cast<int64_t>(pos) * (kHeadDim / 2));
  // pass 2: columns d and d + 64 together (the RoPE pairs), 32 at a time
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    __syncwarp();
    tmem_ld_32x32b_x32(taddr + c * 32, x1);
    tmem_ld_32x32b_x32(taddr + 64 + c * 32, x2);
    tmem_ld_wait();
    uint32_t lo[16], hi[16];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 cv = __ldg(cs4 + c * 8 + q);
      const float4 sv = __ldg(sn4 + c * 8 + q);
      const float co[4] = {cv.x, cv.y, cv.z, cv.w};
      const float si[4] = {sv.x, sv.y, sv.z, sv.w};
      float o[4][2];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int j = q * 4 + e;
        const float u = f32_of(x1[j]) * rstd * __shfl_sync(kFull, w_lane[c], j);
        const float v = f32_of(x2[j]) * rstd * __shfl_sync(kFull, w_lane[c + 2], j);
        o[e][0] = u * co[e] - v * si[e];
        o[e][1] = v * co[e] + u * si[e];
      }
      lo[q * 2] = pack2(o[0][0], o[1][0], XDNA_BF16);
      lo[q * 2 + 1] = pack2(o[2][0], o[3][0], XDNA_BF16);
      hi[q * 2] = pack2(o[0][1], o[1][1], XDNA_BF16);
      hi[q * 2 + 1] = pack2(o[2][1], o[3][1], XDNA_BF16);
    }
    stage_and_store<16>(obuf, lo, tmC, col0 + c * 32, row0);
    stage_and_store<16>(obuf, hi, tmC, col0 + 64 + c * 32, row0);
  }
}

// One warp's half-tile of the fused gate/up projection. The packed weight interleaves 32 gate rows
// and the matching 32 up rows, so accumulator chunks 2p and 2p+1 are gate and up of the same 32
// output columns: act = silu(gate) * up (f32), stored bf16 at act column col0 / 2 + 32 p.
template <int NCH>
__device__ __forceinline__ void swiglu_tile(const GemmArgs& a, uint32_t taddr, int row0, int col0, uint8_t* obuf,
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
    if (col0 / 2 + p * 32 < a.N / 2) stage_and_store<16>(obuf, w, tmC, col0 / 2 + p * 32, row0);
  }
}

// --------------------------------------------------------------------------- the kernel
// ODT: the output element type of the GEMM epilogues, fixed at compile time (XDNA_I32 for EPI_I32).
template <int BN, int LOAD, int EPI, bool BF16, bool TSTORE, int ODT>
__global__ void __launch_bounds__(kThreads, 1)
    umma_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmD,
                     const GemmArgs args) {
  constexpr int STAGES = stages_for<BN>();
  constexpr int A_BYTES = kBM * kBKBytes;
  constexpr int B_BYTES = BN * kBKBytes;
  constexpr uint32_t STAGE_TX = A_BYTES + B_BYTES;
  constexpr uint32_t TMEM_COLS = tmem_cols_for(2 * BN);
  constexpr uint32_t IDESC = BF16 ? idesc_bf16(kBM, BN) : idesc_i8(kBM, BN);
  constexpr int KSTEPS = kBKBytes / 32;  // one MMA consumes 32 bytes of K (32 int8 or 16 bf16)
  constexpr int K_ELEMS = BF16 ? kBKBytes / 2 : kBKBytes;
  constexpr int WCOLS = BN / 2;          // columns per epilogue warp
  constexpr int NCH = WCOLS / 32;        // 32-column chunks per epilogue warp
  static_assert(NCH >= 1 && NCH <= 4, "BN must be 64, 128 or 256");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smem + STAGES * A_BYTES;
  uint8_t* smOut = smB + STAGES * B_BYTES;  // kEpiWarps x kStageOutBytes, 1024-aligned
  uint64_t* full = reinterpret_cast<uint64_t*>(smOut + kEpiWarps * kStageOutBytes);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull + b, 1);
      mbar_init(tempty + b, kEpiWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if constexpr (TSTORE) tma_prefetch_desc(&tmC);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int total = args.m_tiles * args.n_tiles;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------------- TMA producer
      int stage = 0;
      uint32_t phase = 0;
      int last_parity[STAGES];
#pragma unroll
      for (int s = 0; s < STAGES; ++s) last_parity[s] = -1;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        int mb, nb;
        tile_coords(t, args.m_tiles, args.n_tiles, mb, nb);
        for (int kb = 0; kb < args.num_kb; ++kb) {
          if (!mbar_wait(empty + stage, phase ^ 1, abort_flag, args.err, 1)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full + stage, STAGE_TX);
          if constexpr (LOAD == LOAD_GEMM) {
            tma_load_2d(smA + stage * A_BYTES, &tmA, full + stage, kb * K_ELEMS, mb * kBM);
            tma_load_2d(smB + stage * B_BYTES, &tmB, full + stage, kb * K_ELEMS, nb * BN);
          } else {
            const int tap = kb / args.cblocks;
            const int cb = kb - tap * args.cblocks;
            const int dy = tap / 3 - 1;
            const int dx = tap % 3 - 1;
            tma_load_2d(smA + stage * A_BYTES, &tmA, full + stage, cb * K_ELEMS, mb * kBM + dy * args.Wp + dx);
            tma_load_3d(smB + stage * B_BYTES, &tmB, full + stage, cb * K_ELEMS, tap, nb * BN);
          }
          last_parity[stage] = static_cast<int>(phase);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Drain: the last load of every stage has landed before the CTA may exit (a no-op on the
      // normal path, where the MMA warp consumed them all).
      for (int s = 0; s < STAGES; ++s)
        if (last_parity[s] >= 0) {
          volatile int never = 0;
          mbar_wait(full + s, static_cast<uint32_t>(last_parity[s]), &never, args.err, 2);
        }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------------- MMA issuer
      int stage = 0;
      uint32_t phase = 0;
      int buf = 0;
      uint32_t bphase = 0;
      bool issued = false;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        if (!mbar_wait(tempty + buf, bphase ^ 1, abort_flag, args.err, 3)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(buf * BN);
        for (int kb = 0; kb < args.num_kb; ++kb) {
          if (!mbar_wait(full + stage, phase, abort_flag, args.err, 4)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = smem_desc_k_sw128(smem_u32(smA + stage * A_BYTES));
          const uint64_t db = smem_desc_k_sw128(smem_u32(smB + stage * B_BYTES));
#pragma unroll
          for (int k = 0; k < KSTEPS; ++k) {
            const uint32_t acc = (kb | k) != 0;
            if constexpr (BF16)
              umma_f16(d, da + 2 * k, db + 2 * k, IDESC, acc);
            else
              umma_i8(d, da + 2 * k, db + 2 * k, IDESC, acc);
          }
          umma_commit(empty + stage);
          issued = true;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(tfull + buf);
        if (++buf == 2) {
          buf = 0;
          bphase ^= 1;
        }
      }
      // Drain: every MMA this thread issued has completed before TMEM is freed.
      if (issued) {
        umma_commit(drain);
        volatile int never = 0;
        mbar_wait(drain, 0, &never, args.err, 5);
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2..9)
    const int ew = warp - 2;
    const int q = warp & 3;          // the TMEM lane quadrant this warp may read
    const int half = ew >> 2;        // which half of the tile's columns
    uint8_t* obuf = smOut + ew * kStageOutBytes;
    const bool has_bias = args.bias != nullptr;
    int buf = 0;
    uint32_t bphase = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      int mb, nb;
      tile_coords(t, args.m_tiles, args.n_tiles, mb, nb);
      const int row0 = mb * kBM + q * 32;
      const int row = row0 + lane;
      const int col0 = nb * BN + half * WCOLS;
      // per-row and per-column factors, loaded before waiting for the accumulator
      float srow = 0.f;
      float fcol[NCH], bcol[NCH];
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        const int n = col0 + c * 32 + lane;
        fcol[c] = 0.f;
        bcol[c] = 0.f;
        if constexpr (EPI == EPI_DEQ || EPI == EPI_CONV_DEQ) {
          if (n < args.N) {
            fcol[c] = __ldg(args.sw + n);
            if (has_bias) bcol[c] = load_as_float(args.bias, args.bias_dtype, n);
          }
        }
        if constexpr (EPI == EPI_F32ACC) {
          if (n < args.N && has_bias) bcol[c] = load_as_float(args.bias, args.bias_dtype, n);
        }
      }
      if constexpr (EPI == EPI_DEQ) srow = row < args.M ? __ldg(args.sx + row) : 0.f;

      if (!mbar_wait(tfull + buf, bphase, abort_flag, args.err, 6)) break;
      tc_fence_after();
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(buf * BN + half * WCOLS);
      if constexpr (EPI == EPI_QKV || EPI == EPI_SWIGLU) {
        if (col0 < args.N) {  // warp-uniform
          if constexpr (EPI == EPI_QKV)
            qkv_tile(args, taddr, row0, col0, obuf, &tmC, &tmD);
          else
            swiglu_tile<NCH>(args, taddr, row0, col0, obuf, &tmC);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tempty + buf);
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
          if (lane == 0) mbar_arrive(tempty + buf);
        }
        const int n0 = col0 + c * 32;
        // warp-uniform: this chunk has columns in range (and, for GEMM outputs, rows in range)
        if (n0 < args.N && (LOAD == LOAD_CONV || row0 < args.M)) {
          const uint32_t(&rc)[32] = r[c & 1];
          if constexpr (EPI == EPI_I32 || EPI == EPI_DEQ) {
            if constexpr (TSTORE) {
              if constexpr (EPI == EPI_I32) {
                stage_and_store<32>(obuf, rc, &tmC, n0, row0);
              } else {
                float v[32];
                dequant32(rc, srow, fcol[c], bcol[c], has_bias, v);
                if constexpr (ODT == XDNA_F32) {
                  uint32_t w[32];
#pragma unroll
                  for (int j = 0; j < 32; ++j) w[j] = __float_as_uint(v[j]);
                  stage_and_store<32>(obuf, w, &tmC, n0, row0);
                } else {
                  uint32_t w[16];
#pragma unroll
                  for (int j = 0; j < 16; ++j) w[j] = pack2(v[2 * j], v[2 * j + 1], ODT);
                  stage_and_store<16>(obuf, w, &tmC, n0, row0);
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
                stage_and_store<32>(obuf, w, &tmC, n0, row0);
              } else {
                uint32_t w[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) w[j] = pack2(v[2 * j], v[2 * j + 1], ODT);
                stage_and_store<16>(obuf, w, &tmC, n0, row0);
              }
            } else {
              store_direct<EPI>(args, row, n0, rc, v);
            }
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
          } else {
            conv_chunk<EPI>(args, row, n0, rc, fcol[c], bcol[c], obuf);
          }
        }
        if (c + 1 < NCH) tmem_ld_wait();
      }
      }  // generic chunk loop
      if (++buf == 2) {
        buf = 0;
        bphase ^= 1;
      }
    }
    if constexpr (TSTORE) {
      if (lane == 0) bulk_wait_all();
      __syncwarp();
    }
  }

  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace xdna
