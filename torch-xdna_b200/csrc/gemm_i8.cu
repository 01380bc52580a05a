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
static int dispatch_conv(int kb, int bn, bool pair, bool win, const CUtensorMap& ta, const CUtensorMap& tb,
                         const GemmArgs& args, int sms, cudaStream_t stream) {
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

// Whether stride-1 3x3 convs of <= 64 input channels use the window load (LOAD_CONV_WIN); XDNA_CONV_WINDOW=0
// in the environment turns it off (the per-tap loads of LOAD_CONV_RB), e.g. to compare the two.
static bool conv_window() {
  static const bool on = [] {
    const char* e = std::getenv("XDNA_CONV_WINDOW");
    return e == nullptr || e[0] != '0';
  }();
  return on;
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
  mode &= ~(XDNA_CONV_SINGLE_TAP | XDNA_CONV_STRIDE2 | XDNA_CONV_NEXT_AMAX | XDNA_CONV_NEXT_RELU | XDNA_CONV_NEXT_POOL |
            XDNA_CONV_BIAS_INT32);
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
  const int64_t a_rows = stride2 ? planes * n_in * HWp : NP;
  XDNA_CHECK_ARG(a_rows < (1ll << 31) && Co * Cp * 9 < (1ll << 31), "conv3x3: problem exceeds 2^31 elements");

  GemmArgs a{};
  a.M = static_cast<int>(NP);
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
  a.m_tiles = static_cast<int>((NP + kBM - 1) / kBM);
  const int bn = choose_bn(a.m_tiles, Co, sms);
  a.n_tiles = static_cast<int>((Co + bn - 1) / bn);
  // 256 x 256 tiles on CTA pairs for wide convs (not the calibration, which runs one image)
  const bool pair = kb == 128 && mode != XDNA_CONV_CALIBRATE && use_pairs(bn, a.m_tiles, a.n_tiles, sms);
  if (pair) a.m_tiles = static_cast<int>((NP + 2 * kBM - 1) / (2 * kBM));
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
    const uint64_t dims[2] = {static_cast<uint64_t>(Cp), static_cast<uint64_t>(a_rows)};
    const uint64_t strides[1] = {static_cast<uint64_t>(Cp)};
    const uint32_t box[2] = {static_cast<uint32_t>(kb), win ? kBM + 2 : kBM};
    rc = encode_tma(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, xp, dims, strides, box, "conv3x3 activations",
                    kb == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B);
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
      return dispatch_conv<EPI_CONV_Q, XDNA_I8>(kb, bn, pair, win, ta, tb, a, sms, s);
    case XDNA_CONV_DEQUANT:
      return dispatch_conv<EPI_CONV_DEQ, XDNA_F32>(kb, bn, pair, win, ta, tb, a, sms, s);
    case XDNA_CONV_Q_NHWC:
      return dispatch_conv<EPI_CONV_QNHWC, XDNA_I8>(kb, bn, pair, win, ta, tb, a, sms, s);
    default:
      return dispatch_conv<EPI_CONV_CALIB, XDNA_I32>(kb, bn, false, win, ta, tb, a, sms, s);
  }
}

}  // extern "C"
