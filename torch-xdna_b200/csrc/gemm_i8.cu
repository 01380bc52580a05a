// xdna_gemm_i8 and xdna_conv3x3_i8: host side of the tcgen05 int8 GEMM (umma_gemm.cuh).
#include <algorithm>
#include <cstdlib>

#include "host_util.h"
#include "umma_gemm.cuh"

namespace xdna {

template <int BN, int LOAD, int EPI, bool TSTORE, int ODT, int KB>
static int launch_umma(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const GemmArgs& args,
                       int sms, cudaStream_t stream) {
  return launch_gemm_kernel<BN, LOAD, EPI, false, TSTORE, ODT, KB, false>(ta, tb, tc, ta, args, sms, stream);
}

template <int LOAD, int EPI, bool TSTORE, int ODT, int KB = kBKBytes>
static int dispatch_bn(int bn, bool pair, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                       const GemmArgs& args, int sms, cudaStream_t stream) {
  switch (bn) {
    case 256:
      if constexpr (KB == 128) {
        if (pair) return launch_gemm_kernel<256, LOAD, EPI, false, TSTORE, ODT, KB, true>(ta, tb, tc, ta, args, sms, stream);
      }
      return launch_umma<256, LOAD, EPI, TSTORE, ODT, KB>(ta, tb, tc, args, sms, stream);
    case 128:
      return launch_umma<128, LOAD, EPI, TSTORE, ODT, KB>(ta, tb, tc, args, sms, stream);
    default:
      return launch_umma<64, LOAD, EPI, TSTORE, ODT, KB>(ta, tb, tc, args, sms, stream);
  }
}

// The conv's kernel for one mode, with 64-byte K blocks when the input has at most 64 channels (a
// 128-byte block would be half zero fill).
template <int EPI, int ODT>
static int dispatch_conv(int kb, int bn, bool pair, bool win, bool winb, const CUtensorMap& ta, const CUtensorMap& tb,
                         const GemmArgs& args, int sms, cudaStream_t stream) {
  if (winb) {  // 128-byte channel blocks: one window per (ky, block) with its three taps' weights (LOAD_CONV_WINB)
    if (pair) return launch_gemm_kernel<256, LOAD_CONV_WINB, EPI, false, false, ODT, 128, true>(ta, tb, ta, ta, args, sms, stream);
    if (bn == 128) return launch_umma<128, LOAD_CONV_WINB, EPI, false, ODT, 128>(ta, tb, ta, args, sms, stream);
    return launch_umma<64, LOAD_CONV_WINB, EPI, false, ODT, 128>(ta, tb, ta, args, sms, stream);
  }
  if (win) {  // resident weights, one window of 130 activation rows per ky (conv_window)
    if (bn == 128) return launch_umma<128, LOAD_CONV_WIN, EPI, false, ODT, 64>(ta, tb, ta, args, sms, stream);
    return launch_umma<64, LOAD_CONV_WIN, EPI, false, ODT, 64>(ta, tb, ta, args, sms, stream);
  }
  if (kb == 64) {
    // one column tile of <= 128 output channels: the 9 taps' weights stay in shared memory
    if (args.n_tiles == 1 && args.cblocks == 1 && bn <= 128) {
      if (bn == 128) return launch_umma<128, LOAD_CONV_RB, EPI, false, ODT, 64>(ta, tb, ta, args, sms, stream);
      return launch_umma<64, LOAD_CONV_RB, EPI, false, ODT, 64>(ta, tb, ta, args, sms, stream);
    }
    return dispatch_bn<LOAD_CONV, EPI, false, ODT, 64>(bn, false, ta, tb, ta, args, sms, stream);
  }
  return dispatch_bn<LOAD_CONV, EPI, false, ODT, 128>(bn, pair, ta, tb, ta, args, sms, stream);
}

// Whether stride-1 3x3 convs use the window loads (LOAD_CONV_WIN, LOAD_CONV_WIN2, LOAD_CONV_WINB);
// XDNA_CONV_WINDOW=0 in the environment turns them off (per-tap loads), e.g. to compare the two; image pairs
// (XDNA_CONV_PAIRS), which only the window reads, are then refused.
static bool conv_window() {
  static const bool on = [] {
    const char* e = std::getenv("XDNA_CONV_WINDOW");
    return e == nullptr || e[0] != '0';
  }();
  return on;
}

// ------------------------------------------------------------------ a few rows: dp4a dot products
// For M <= kGemvMaxM rows the 128-row tensor-core tiles leave most SMs idle and stream the weights at a
// fraction of HBM bandwidth. Here each warp owns CPW output columns: per step every lane reads 16
// contiguous weight bytes of each of its columns (512 bytes per column and warp, coalesced) and the MR
// activation rows' matching 16 bytes (from L1: every warp reads the same rows), and accumulates exact int32
// sums with __dp4a, two steps' loads in flight. No byte past K of a row is read (the padding may hold
// anything, or not exist for the last row). The warp then adds its lanes' partial sums (exact in int32) and lane
// c * MR + m writes y[m, column c]: the sum itself (int32 out) or the GEMM epilogue's arithmetic,
// fl(fl(float(acc) * sx[m]) * sw[n]) (+ bias[n]), rounded once to the output type.
// (up to 8 rows: at 8 it matches the tensor path's time at 128 rows, at 32 it takes 2.8x as long)
constexpr int kGemvMaxM = 8;

// 16 bytes of a row from byte k: a vector load, or for the row's last partial chunk (k + 16 > K) the
// bytes before K one by one and zeros after them (nothing past byte K of the row is read).
__device__ __forceinline__ uint4 load_row16(const int8_t* row, int k, int K) {
  if (k + 16 <= K) return __ldg(reinterpret_cast<const uint4*>(row + k));
  uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
  for (int i = 0; i < 16; ++i)
    if (k + i < K) w[i >> 2] |= static_cast<uint32_t>(static_cast<uint8_t>(__ldg(row + k + i))) << (8 * (i & 3));
  return make_uint4(w[0], w[1], w[2], w[3]);
}

template <int MR, int CPW>
__global__ void __launch_bounds__(256) gemv_i8_kernel(const int8_t* __restrict__ xq, int64_t ldx,
                                                      const int8_t* __restrict__ wq, int64_t ldw, int M, int N, int K,
                                                      const float* __restrict__ sx, const float* __restrict__ sw,
                                                      const void* __restrict__ bias, int bias_dtype,
                                                      void* __restrict__ y, int y_dtype, int64_t ldy) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = (blockIdx.x * 8 + warp) * CPW;
  const int m0 = blockIdx.y * MR;
  if (n0 >= N) return;  // the whole warp
  int acc[CPW][MR];
#pragma unroll
  for (int c = 0; c < CPW; ++c)
#pragma unroll
    for (int m = 0; m < MR; ++m) acc[c][m] = 0;
  auto step = [&](const uint4 (&wv)[CPW], int k) {
    uint4 xv[MR];
#pragma unroll
    for (int m = 0; m < MR; ++m) {
      xv[m] = m0 + m < M ? load_row16(xq + static_cast<int64_t>(m0 + m) * ldx, k, K) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int c = 0; c < CPW; ++c)
#pragma unroll
      for (int m = 0; m < MR; ++m) {
        int s = acc[c][m];
        s = __dp4a(static_cast<int>(xv[m].x), static_cast<int>(wv[c].x), s);
        s = __dp4a(static_cast<int>(xv[m].y), static_cast<int>(wv[c].y), s);
        s = __dp4a(static_cast<int>(xv[m].z), static_cast<int>(wv[c].z), s);
        s = __dp4a(static_cast<int>(xv[m].w), static_cast<int>(wv[c].w), s);
        acc[c][m] = s;
      }
  };
  auto load_w = [&](uint4 (&wv)[CPW], int k) {
#pragma unroll
    for (int c = 0; c < CPW; ++c)
      wv[c] = (k < K && n0 + c < N) ? load_row16(wq + static_cast<int64_t>(n0 + c) * ldw, k, K)
                                    : make_uint4(0u, 0u, 0u, 0u);
  };
  for (int k = lane * 16; k < K; k += 1024) {
    uint4 wa[CPW], wb[CPW];
    load_w(wa, k);
    load_w(wb, k + 512);
    step(wa, k);
    if (k + 512 < K) step(wb, k + 512);
  }
#pragma unroll
  for (int c = 0; c < CPW; ++c)
#pragma unroll
    for (int m = 0; m < MR; ++m)
#pragma unroll
      for (int s = 16; s >= 1; s >>= 1) acc[c][m] += __shfl_xor_sync(kFull, acc[c][m], s);
  int mine = 0;
#pragma unroll
  for (int c = 0; c < CPW; ++c)
#pragma unroll
    for (int m = 0; m < MR; ++m) mine = lane == c * MR + m ? acc[c][m] : mine;
  const int c = lane / MR, m = lane % MR;
  const int n = n0 + c, row = m0 + m;
  if (c >= CPW || n >= N || row >= M) return;
  const int64_t off = static_cast<int64_t>(row) * ldy + n;
  if (y_dtype == XDNA_I32) {
    static_cast<int32_t*>(y)[off] = mine;
    return;
  }
  float v = __fmul_rn(__fmul_rn(__int2float_rn(mine), __ldg(sx + row)), __ldg(sw + n));
  if (bias != nullptr) v = __fadd_rn(v, load_as_float(bias, bias_dtype, n));
  store_one(y, y_dtype, off, v);
}

template <int MR>
static int launch_gemv_mr(const int8_t* xq, int64_t ldx, const int8_t* wq, int64_t ldw, int M, int N, int K,
                          const float* sx, const float* sw, const void* bias, int bias_dtype, void* y, int y_dtype,
                          int64_t ldy, int sms, cudaStream_t s) {
  const int passes = (M + MR - 1) / MR;
  auto blocks = [&](int cpw) { return (N + 8 * cpw - 1) / (8 * cpw); };
  // as many columns per warp as still fill the GPU (more loads in flight per lane)
  // (at most 2 for 8 rows: 4 x 8 sums and their operands spill)
  const int cpw = MR < 8 && static_cast<int64_t>(blocks(4)) * passes >= sms ? 4
                  : static_cast<int64_t>(blocks(2)) * passes >= sms ? 2 : 1;
  const dim3 grid(blocks(cpw), passes);
  if constexpr (MR < 8) {
    if (cpw == 4) {
      gemv_i8_kernel<MR, 4><<<grid, 256, 0, s>>>(xq, ldx, wq, ldw, M, N, K, sx, sw, bias, bias_dtype, y, y_dtype, ldy);
      return check_launch("gemv_i8_kernel");
    }
  }
  if (cpw == 2)
    gemv_i8_kernel<MR, 2><<<grid, 256, 0, s>>>(xq, ldx, wq, ldw, M, N, K, sx, sw, bias, bias_dtype, y, y_dtype, ldy);
  else
    gemv_i8_kernel<MR, 1><<<grid, 256, 0, s>>>(xq, ldx, wq, ldw, M, N, K, sx, sw, bias, bias_dtype, y, y_dtype, ldy);
  return check_launch("gemv_i8_kernel");
}

static int launch_gemv(const int8_t* xq, int64_t ldx, const int8_t* wq, int64_t ldw, int M, int N, int K,
                       const float* sx, const float* sw, const void* bias, int bias_dtype, void* y, int y_dtype,
                       int64_t ldy, int sms, cudaStream_t s) {
  if (M <= 1) return launch_gemv_mr<1>(xq, ldx, wq, ldw, M, N, K, sx, sw, bias, bias_dtype, y, y_dtype, ldy, sms, s);
  if (M <= 2) return launch_gemv_mr<2>(xq, ldx, wq, ldw, M, N, K, sx, sw, bias, bias_dtype, y, y_dtype, ldy, sms, s);
  if (M <= 4) return launch_gemv_mr<4>(xq, ldx, wq, ldw, M, N, K, sx, sw, bias, bias_dtype, y, y_dtype, ldy, sms, s);
  return launch_gemv_mr<8>(xq, ldx, wq, ldw, M, N, K, sx, sw, bias, bias_dtype, y, y_dtype, ldy, sms, s);
}

// Widest tile that still gives every SM work; 64 for narrow outputs.
static int choose_bn(int64_t m_tiles, int64_t N, int sms) {
  if (N <= 64) return 64;
  if (N <= 128) return 128;
  if (m_tiles * ((N + 255) / 256) >= sms) return 256;
  if (m_tiles * ((N + 127) / 128) >= sms) return 128;
  return N >= 1024 ? 64 : 128;
}

}  // namespace xdna

using namespace xdna;

extern "C" {

int xdna_gemm_i8(const int8_t* xq, int64_t ldx, const int8_t* wq, int64_t ldw, int64_t M, int64_t N, int64_t K,
                 const float* sx, const float* sw, const void* bias, int bias_dtype, void* y, int y_dtype,
                 int64_t ldy, void* stream) {
  int sms = 0;
  int rc = check_device(&sms);
  if (rc != XDNA_OK) return rc;
  XDNA_CHECK_ARG(M >= 0 && N >= 0 && K >= 0, "gemm_i8: negative size");
  XDNA_CHECK_ARG(M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), "gemm_i8: size exceeds 2^31");
  XDNA_CHECK_ARG(ldx >= K && ldw >= K && ldy >= N, "gemm_i8: leading dimension smaller than the row");
  XDNA_CHECK_ARG(y_dtype == XDNA_I32 || is_float_dtype(y_dtype), "gemm_i8: y_dtype %d unsupported", y_dtype);
  if (M == 0 || N == 0) return XDNA_OK;
  XDNA_CHECK_ARG(xq && wq && y, "gemm_i8: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (K == 0) {  // empty sum: zeros (dequantised zeros are bias)
    if (y_dtype == XDNA_I32 && ldy == N) {
      XDNA_CUDA(cudaMemsetAsync(y, 0, M * N * sizeof(int32_t), s));
      return XDNA_OK;
    }
    return fail(XDNA_ERR_UNSUPPORTED, "gemm_i8: K == 0 is only supported for a dense int32 output");
  }
  if (y_dtype != XDNA_I32) {
    XDNA_CHECK_ARG(sx && sw, "gemm_i8: dequantised output needs sx and sw");
    XDNA_CHECK_ARG(bias == nullptr || is_float_dtype(bias_dtype), "gemm_i8: bias dtype %d", bias_dtype);
  }
  XDNA_CHECK_ARG(ldx % 16 == 0 && ldw % 16 == 0, "gemm_i8: int8 row pitch must be a multiple of 16 bytes");
  if (M <= kGemvMaxM && aligned16(xq) && aligned16(wq))
    return launch_gemv(xq, ldx, wq, ldw, static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), sx, sw, bias,
                       bias_dtype, y, y_dtype, ldy, sms, s);

  GemmArgs a{};
  a.M = static_cast<int>(M);
  a.N = static_cast<int>(N);
  a.num_kb = static_cast<int>((K + kBKBytes - 1) / kBKBytes);
  a.m_tiles = static_cast<int>((M + kBM - 1) / kBM);
  const int bn = choose_bn(a.m_tiles, N, sms);
  a.n_tiles = static_cast<int>((N + bn - 1) / bn);
  const bool pair = use_pairs(bn, a.m_tiles, a.n_tiles, sms);
  if (pair) a.m_tiles = static_cast<int>((M + 2 * kBM - 1) / (2 * kBM));
  a.out = y;
  a.ldo = ldy;
  a.out_dtype = y_dtype;
  const int es = dtype_size(y_dtype);
  a.vec_ok = aligned16(y) && (ldy * es) % 16 == 0;
  a.sx = sx;
  a.sw = sw;
  a.bias = bias;
  a.bias_dtype = bias_dtype;
  a.err = device_error_word();

  CUtensorMap ta, tb, tc;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
    const uint64_t strides[1] = {static_cast<uint64_t>(ldx)};
    const uint32_t box[2] = {kBKBytes, kBM};
    rc = encode_tma(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, xq, dims, strides, box, "gemm_i8 activations");
    if (rc != XDNA_OK) return rc;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(N)};
    const uint64_t strides[1] = {static_cast<uint64_t>(ldw)};
    const uint32_t box[2] = {kBKBytes, static_cast<uint32_t>(pair ? bn / 2 : bn)};  // a pair: each CTA half of B
    rc = encode_tma(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, wq, dims, strides, box, "gemm_i8 weights");
    if (rc != XDNA_OK) return rc;
  }
  // Output through TMA stores when the rows are 16-byte addressable (box: 32 rows x 64 bytes, i.e. 32
  // columns of a 2-byte type or 16 of a 4-byte type, 64-byte swizzle).
  const bool tstore = a.vec_ok != 0;
  if (tstore) {
    const uint64_t dims[2] = {static_cast<uint64_t>(N), static_cast<uint64_t>(M)};
    const uint64_t strides[1] = {static_cast<uint64_t>(ldy * es)};
    // pair tiles with 2-byte outputs store 32 x 128-byte blocks (stage_wide), the rest 32 x 64-byte ones
    const bool wide = y_dtype != XDNA_I32 && wide_store_map(EPI_DEQ, pair, es);
    const uint32_t box[2] = {static_cast<uint32_t>((wide ? 128 : 64) / es), 32};
    const CUtensorMapDataType dt = es == 4 ? CU_TENSOR_MAP_DATA_TYPE_INT32
                                   : y_dtype == XDNA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                          : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    rc = encode_tma(&tc, dt, 2, y, dims, strides, box, "gemm_i8 output",
                    wide ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
    if (rc != XDNA_OK) return rc;
  } else {
    tc = ta;  // unused
  }
  if (!tstore) {  // rows TMA cannot address: direct stores (any output type)
    if (y_dtype == XDNA_I32) return dispatch_bn<LOAD_GEMM, EPI_I32, false, XDNA_I32>(bn, pair, ta, tb, tc, a, sms, s);
    return dispatch_bn<LOAD_GEMM, EPI_DEQ, false, XDNA_F32>(bn, pair, ta, tb, tc, a, sms, s);
  }
  switch (y_dtype) {
    case XDNA_I32:
      return dispatch_bn<LOAD_GEMM, EPI_I32, true, XDNA_I32>(bn, pair, ta, tb, tc, a, sms, s);
    case XDNA_F32:
      return dispatch_bn<LOAD_GEMM, EPI_DEQ, true, XDNA_F32>(bn, pair, ta, tb, tc, a, sms, s);
    case XDNA_BF16:
      return dispatch_bn<LOAD_GEMM, EPI_DEQ, true, XDNA_BF16>(bn, pair, ta, tb, tc, a, sms, s);
    default:
      return dispatch_bn<LOAD_GEMM, EPI_DEQ, true, XDNA_F16>(bn, pair, ta, tb, tc, a, sms, s);
  }
}

int xdna_gemm_i8_config(int64_t M, int64_t N, int* tile_n, int* pair) {
  int sms = 0;
  int rc = check_device(&sms);
  if (rc != XDNA_OK) return rc;
  XDNA_CHECK_ARG(M >= 0 && N >= 0 && M < (1ll << 31) && N < (1ll << 31) && tile_n && pair, "gemm_i8_config: bad args");
  const int64_t m_tiles = (M + kBM - 1) / kBM;
  const int bn = choose_bn(m_tiles, N, sms);  // the calls xdna_gemm_i8 makes
  *tile_n = bn;
  *pair = use_pairs(bn, m_tiles, (N + bn - 1) / bn, sms) ? 1 : 0;
  return XDNA_OK;
}

int xdna_conv3x3_i8(const int8_t* xp, const int8_t* wp, int64_t N, int64_t Ci, int64_t Cp, int64_t Co, int64_t H,
                    int64_t W, int mode, int shift, int relu, const float* scale, const float* sx, const void* bias,
                    int bias_dtype, void* out, int out_dtype, int32_t* acc_max, void* stream) {
  int sms = 0;
  int rc = check_device(&sms);
  if (rc != XDNA_OK) return rc;
  XDNA_CHECK_ARG(N >= 0 && Ci >= 1 && Co >= 1 && H >= 1 && W >= 1, "conv3x3: bad shape");
  XDNA_CHECK_ARG(Cp >= Ci && Cp % 16 == 0, "conv3x3: Cp must be >= Ci and a multiple of 16");
  const bool single_tap = (mode & XDNA_CONV_SINGLE_TAP) != 0;
  const bool stride2 = (mode & XDNA_CONV_STRIDE2) != 0;
  const bool next_amax = (mode & XDNA_CONV_NEXT_AMAX) != 0;
  const bool next_relu = (mode & XDNA_CONV_NEXT_RELU) != 0;
  const bool next_pool = (mode & XDNA_CONV_NEXT_POOL) != 0;
  const bool bias_i32 = (mode & XDNA_CONV_BIAS_INT32) != 0;
  const bool pimg = (mode & XDNA_CONV_PAIRS) != 0;
  mode &= ~(XDNA_CONV_SINGLE_TAP | XDNA_CONV_STRIDE2 | XDNA_CONV_NEXT_AMAX | XDNA_CONV_NEXT_RELU | XDNA_CONV_NEXT_POOL |
            XDNA_CONV_BIAS_INT32 | XDNA_CONV_PAIRS);
  XDNA_CHECK_ARG(!pimg || (mode == XDNA_CONV_Q_NHWC && Cp == 64 && N % 2 == 0 && !single_tap && !stride2 && Co <= 128 &&
                           conv_window()),
                 "conv3x3: XDNA_CONV_PAIRS needs XDNA_CONV_Q_NHWC, Cp = 64, an even N, a stride-1 3x3 conv and "
                 "Co <= 128");
  XDNA_CHECK_ARG(!bias_i32 || (bias != nullptr && bias_dtype == XDNA_I32),
                 "conv3x3: XDNA_CONV_BIAS_INT32 needs an int32 bias [N, Co]");
  XDNA_CHECK_ARG(bias_i32 || bias == nullptr || is_float_dtype(bias_dtype), "conv3x3: a float bias (or XDNA_CONV_BIAS_INT32)");
  if (bias_i32) XDNA_CHECK_ARG(aligned16(bias), "conv3x3: int32 bias not 16-byte aligned");
  XDNA_CHECK_ARG(!next_amax || (mode == XDNA_CONV_Q_NHWC && scale != nullptr && sx != nullptr && acc_max != nullptr),
                 "conv3x3: XDNA_CONV_NEXT_AMAX needs XDNA_CONV_Q_NHWC, scale, sx and acc_max (N words)");
  XDNA_CHECK_ARG(!next_amax || !next_pool || next_relu || (relu == 1 && (bias == nullptr || bias_i32)),
                 "conv3x3: pooled maxima need non-negative values (XDNA_CONV_NEXT_RELU, or a fused ReLU and no float bias)");
  XDNA_CHECK_ARG(!next_amax || bias_i32 || bias == nullptr || bias_dtype == XDNA_F32,
                 "conv3x3: next maxima need an f32 bias");
  XDNA_CHECK_ARG(mode == XDNA_CONV_Q || mode == XDNA_CONV_DEQUANT || mode == XDNA_CONV_CALIBRATE ||
                     mode == XDNA_CONV_Q_NHWC,
                 "conv3x3: unknown mode %d", mode);
  XDNA_CHECK_ARG(relu == 0 || relu == 1 || (relu == XDNA_RELU_AFTER_BIAS && mode == XDNA_CONV_DEQUANT),
                 "conv3x3: relu %d (0, 1, or XDNA_RELU_AFTER_BIAS with XDNA_CONV_DEQUANT)", relu);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t n_in = N;  // images in xp (a stride-2 input's phase planes are n_in images apart)
  if (mode == XDNA_CONV_CALIBRATE) {
    XDNA_CHECK_ARG(acc_max != nullptr, "conv3x3: calibration needs acc_max");
    XDNA_CUDA(cudaMemsetAsync(acc_max, 0, sizeof(int32_t), s));
    if (N == 0) return XDNA_OK;
    N = 1;  // the shift is fixed from the first image's sums
  } else {
    XDNA_CHECK_ARG(shift >= 1 && shift <= 31, "conv3x3: shift %d outside [1, 31]", shift);
    XDNA_CHECK_ARG(scale != nullptr || mode == XDNA_CONV_Q || mode == XDNA_CONV_Q_NHWC, "conv3x3: dequantise needs scale");
    if (mode == XDNA_CONV_Q || mode == XDNA_CONV_Q_NHWC)
      XDNA_CHECK_ARG(out_dtype == (relu ? XDNA_U8 : XDNA_I8), "conv3x3: requantised output is %s",
                     relu ? "uint8 with relu" : "int8 without relu");
    else
      XDNA_CHECK_ARG(is_float_dtype(out_dtype) && sx != nullptr, "conv3x3: dequantise needs a float out and sx");
    if (N == 0) return XDNA_OK;
    XDNA_CHECK_ARG(out != nullptr, "conv3x3: null output");
  }
  XDNA_CHECK_ARG(xp && wp, "conv3x3: null pointer");
  const int64_t Wp = W + 2, HWp = (H + 2) * (W + 2);
  const int64_t NP = N * HWp;
  // rows of the activation matrix: one bordered image per image, or for a stride-2 conv the phase planes
  // (4, or the even-even plane alone for the 1x1 conv), each n_in bordered images of the output's geometry
  const int planes = stride2 ? (single_tap ? 1 : 4) : 1;
  const int64_t a_rows = stride2 ? planes * n_in * HWp : pimg ? NP / 2 : NP;  // pairs: one row per two images
  XDNA_CHECK_ARG(a_rows < (1ll << 31) && Co * Cp * 9 < (1ll << 31), "conv3x3: problem exceeds 2^31 elements");

  GemmArgs a{};
  a.M = static_cast<int>(pimg ? NP / 2 : NP);  // pairs: the tiles run over pair rows, each two images' pixel
  a.N = static_cast<int>(Co);
  const int kb = Cp <= 64 ? 64 : kBKBytes;  // K block bytes (= channels) per tap
  a.cblocks = static_cast<int>((Cp + kb - 1) / kb);
  a.ntaps = single_tap ? 1 : 9;
  for (int t = 0; t < a.ntaps; ++t) {
    const int ky = single_tap ? 1 : t / 3, kx = single_tap ? 1 : t % 3;
    if (stride2) {
      // input row 2y + ky - 1 is row y - 1 (ky = 0) or y (ky = 2) of the odd phase, row y of the even one (ky = 1)
      const int ry = ky == 1 ? 0 : 1, rx = kx == 1 ? 0 : 1;
      const int dy = ky == 0 ? -1 : 0, dx = kx == 0 ? -1 : 0;
      a.tap_off[t] = static_cast<int>((2 * ry + rx) * n_in * HWp + dy * Wp + dx);
    } else {
      a.tap_off[t] = static_cast<int>((ky - 1) * Wp + (kx - 1));
    }
  }
  a.num_kb = a.ntaps * a.cblocks;
  // a stride-1 3x3 conv on the resident-weight path (<= 64 input channels, one column tile of <= 128 output
  // channels) loads one window of kBM + 2 rows per ky, which its three kx taps share (LOAD_CONV_WIN)
  const bool win = conv_window() && kb == 64 && a.cblocks == 1 && a.ntaps == 9 && !stride2 && Co <= 128;
  if (win) a.num_kb = 3;
  a.m_tiles = static_cast<int>((a.M + kBM - 1) / kBM);
  int bn = choose_bn(a.m_tiles, Co, sms);
  // a small conv of 128-byte channel blocks (a few images per GPU, deep layers): 64-column tiles while
  // 128-column ones leave SMs idle (not for <= 64 input channels, whose resident-weight paths take one
  // column tile of all the output channels)
  if (kb == 128 && bn == 128 && Co > 64 && a.m_tiles * ((Co + 127) / 128) < sms) bn = 64;
  a.n_tiles = static_cast<int>((Co + bn - 1) / bn);
  // 256 x 256 tiles on CTA pairs for wide convs (not the calibration, which runs one image)
  const bool pair = kb == 128 && mode != XDNA_CONV_CALIBRATE && use_pairs(bn, a.m_tiles, a.n_tiles, sms);
  if (pair) a.m_tiles = static_cast<int>((NP + 2 * kBM - 1) / (2 * kBM));
  // stride-1 3x3 convs of 128-byte channel blocks: one window per (ky, channel block) serving three taps, when
  // a CTA's B tiles are at most 128 rows (three of them share the stage with the window); not for the
  // dequantise, whose staged whole-line stores need the shared memory the window's stages take
  const bool winb = conv_window() && kb == 128 && a.ntaps == 9 && !stride2 && (pair ? bn / 2 : bn) <= 128 &&
                    mode != XDNA_CONV_DEQUANT;
  if (winb) a.num_kb = 3 * a.cblocks;
  a.Wp = static_cast<int>(Wp);
  a.HWp = static_cast<int>(HWp);
  a.H = static_cast<int>(H);
  a.W = static_cast<int>(W);
  a.div_wp = make_fastdiv(static_cast<uint32_t>(Wp));
  a.div_hwp = make_fastdiv(static_cast<uint32_t>(HWp));
  a.out = out;
  a.out_dtype = out_dtype;
  // XDNA_CONV_DEQUANT writes channels-last: 32 channels of a pixel as 16-byte vectors when aligned
  a.vec_ok = mode == XDNA_CONV_DEQUANT ? (aligned16(out) && (Co * dtype_size(out_dtype)) % 16 == 0)
            : mode == XDNA_CONV_Q_NHWC ? (aligned16(out) && Co % 16 == 0) : 0;
  a.sx = sx;
  a.sw = scale;
  a.bias = bias_i32 ? nullptr : bias;
  a.bias_dtype = bias_i32 ? XDNA_F32 : bias_dtype;
  a.bias_i32 = bias_i32 ? static_cast<const int32_t*>(bias) : nullptr;
  a.shift = shift;
  a.relu = relu == 1 ? 1 : 0;
  a.post_relu = relu == XDNA_RELU_AFTER_BIAS ? 1 : 0;
  a.acc_max = acc_max;
  if (next_amax) {
    XDNA_CUDA(cudaMemsetAsync(acc_max, 0, N * sizeof(uint32_t), s));
    a.next_amax = reinterpret_cast<uint32_t*>(acc_max);
    a.next_relu = next_relu ? 1 : 0;
    a.next_h = static_cast<int>(next_pool ? H & ~1ll : H);
    a.next_w = static_cast<int>(next_pool ? W & ~1ll : W);
  }
  a.err = device_error_word();

  CUtensorMap ta, tb;
  {
    // pairs: rows of 128 bytes, images 2i and 2i + 1 side by side
    const uint64_t row_bytes = pimg ? 2 * Cp : Cp;
    const uint64_t dims[2] = {row_bytes, static_cast<uint64_t>(a_rows)};
    const uint64_t strides[1] = {row_bytes};
    const uint32_t box[2] = {static_cast<uint32_t>(pimg ? 128 : kb), static_cast<uint32_t>(win || winb ? kBM + 2 : kBM)};
    rc = encode_tma(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, xp, dims, strides, box, "conv3x3 activations",
                    kb == 64 && !pimg ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != XDNA_OK) return rc;
  }
  {
    const uint64_t taps = single_tap ? 1 : 9;
    const uint64_t dims[3] = {static_cast<uint64_t>(Cp), taps, static_cast<uint64_t>(Co)};
    const uint64_t strides[2] = {static_cast<uint64_t>(Cp), static_cast<uint64_t>(taps * Cp)};
    const uint32_t box[3] = {static_cast<uint32_t>(kb), 1, static_cast<uint32_t>(pair ? bn / 2 : bn)};
    rc = encode_tma(&tb, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, wp, dims, strides, box, "conv3x3 weights",
                    kb == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != XDNA_OK) return rc;
  }
  switch (mode) {
    case XDNA_CONV_Q:
      return dispatch_conv<EPI_CONV_Q, XDNA_I8>(kb, bn, pair, win, winb, ta, tb, a, sms, s);
    case XDNA_CONV_DEQUANT:
      return dispatch_conv<EPI_CONV_DEQ, XDNA_F32>(kb, bn, pair, win, winb, ta, tb, a, sms, s);
    case XDNA_CONV_Q_NHWC:
      if (pimg) {
        if (bn == 128) return launch_umma<128, LOAD_CONV_WIN2, EPI_CONV_QNHWC, false, XDNA_I8, 64>(ta, tb, ta, a, sms, s);
        return launch_umma<64, LOAD_CONV_WIN2, EPI_CONV_QNHWC, false, XDNA_I8, 64>(ta, tb, ta, a, sms, s);
      }
      return dispatch_conv<EPI_CONV_QNHWC, XDNA_I8>(kb, bn, pair, win, winb, ta, tb, a, sms, s);
    default:
      return dispatch_conv<EPI_CONV_CALIB, XDNA_I32>(kb, bn, false, win, winb, ta, tb, a, sms, s);
  }
}

}  // extern "C"
