// Symmetric int8 quantisation kernels (HBM-bound):
//   - per row (activations of the W8A8 linear, and every weight matrix once);
//   - per image, fused with the NCHW -> zero-bordered NHWC layout the implicit-GEMM conv reads;
//   - int8 NCHW -> bordered NHWC (the xdna::conv3x3 op's own input), and the conv weight packing.
//
// Arithmetic follows the reference exactly: the max of |x| is taken in x's dtype (exact), widened
// to f32, clamped below by 1e-8 and divided by 127 (IEEE division); each value is x / scale with
// IEEE division, rounded half to even, clamped to [-127, 127]. No FMA contraction is involved.
#include <algorithm>

#include "host_util.h"
#include "sm100.cuh"

namespace xdna {

template <typename T>
struct Vec16;  // 16 bytes of T
template <>
struct Vec16<float> {
  static constexpr int N = 4;
};
template <>
struct Vec16<__nv_bfloat16> {
  static constexpr int N = 8;
};
template <>
struct Vec16<__half> {
  static constexpr int N = 8;
};

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f32(int8_t v) { return static_cast<float>(v); }

__device__ __forceinline__ int8_t quant1(float v, float s) {
  const float q = rintf(__fdiv_rn(v, s));
  return static_cast<int8_t>(static_cast<int>(fminf(fmaxf(q, -127.f), 127.f)));
}

__device__ __forceinline__ float scale_from_amax(float amax) { return __fdiv_rn(fmaxf(amax, 1e-8f), 127.f); }

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// One warp per row. VEC: 16-byte loads when the row allows them.
template <typename T, bool VEC>
__global__ void __launch_bounds__(256) quant_rows_kernel(const T* __restrict__ x, int64_t rows, int64_t cols,
                                                         int64_t ldx, int8_t* __restrict__ xq, int64_t ldq,
                                                         float* __restrict__ scale) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int lane = threadIdx.x & 31;
  const T* xr = x + row * ldx;
  int8_t* qr = xq + row * ldq;
  float amax = 0.f;
  if constexpr (VEC) {
    constexpr int V = Vec16<T>::N;
    for (int64_t c = static_cast<int64_t>(lane) * V; c < cols; c += 32 * V) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(xr + c));
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int j = 0; j < V; ++j) amax = fmaxf(amax, fabsf(to_f32(e[j])));
    }
  } else {
    for (int64_t c = lane; c < cols; c += 32) amax = fmaxf(amax, fabsf(to_f32(xr[c])));
  }
  amax = warp_max(amax);
  const float s = scale_from_amax(amax);
  if (lane == 0) scale[row] = s;
  if constexpr (VEC) {
    constexpr int V = Vec16<T>::N;
    for (int64_t c = static_cast<int64_t>(lane) * V; c < cols; c += 32 * V) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(xr + c));
      const T* e = reinterpret_cast<const T*>(&u);
      int8_t q[V];
#pragma unroll
      for (int j = 0; j < V; ++j) q[j] = quant1(to_f32(e[j]), s);
      if constexpr (V == 4)
        *reinterpret_cast<uint32_t*>(qr + c) = *reinterpret_cast<uint32_t*>(q);
      else
        *reinterpret_cast<uint2*>(qr + c) = *reinterpret_cast<uint2*>(q);
    }
  } else {
    for (int64_t c = lane; c < cols; c += 32) qr[c] = quant1(to_f32(xr[c]), s);
  }
}

template <typename T>
static int launch_quant_rows(const void* x, int64_t rows, int64_t cols, int64_t ldx, int8_t* xq, int64_t ldq,
                             float* scale, cudaStream_t stream) {
  constexpr int V = Vec16<T>::N;
  const bool vec = cols % V == 0 && ldx % V == 0 && ldq % V == 0 && aligned16(x) &&
                   (reinterpret_cast<uintptr_t>(xq) % V) == 0;
  const int rows_per_block = 8;
  const int64_t blocks = (rows + rows_per_block - 1) / rows_per_block;
  if (blocks > 0x7fffffff) return fail(XDNA_ERR_INVALID, "quant_rows: too many rows");
  if (vec)
    quant_rows_kernel<T, true><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
        static_cast<const T*>(x), rows, cols, ldx, xq, ldq, scale);
  else
    quant_rows_kernel<T, false><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
        static_cast<const T*>(x), rows, cols, ldx, xq, ldq, scale);
  return check_launch("quant_rows_kernel");
}

// ---------------------------------------------------------------------------- per-image amax
// grid (chunks, N). Non-negative floats order like their bit patterns, so the image's max |x|
// is an atomicMax over uint32 bits.
template <typename T>
__global__ void __launch_bounds__(256) image_amax_kernel(const T* __restrict__ x, int64_t per_image,
                                                         uint32_t* __restrict__ amax) {
  const int64_t n = blockIdx.y;
  const T* xi = x + n * per_image;
  float m = 0.f;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < per_image; i += stride)
    m = fmaxf(m, fabsf(to_f32(xi[i])));
  m = warp_max(m);
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_max(v);
    if (threadIdx.x == 0) atomicMax(amax + n, __float_as_uint(v));
  }
}

// ---------------------------------------------------------------------------- NCHW -> bordered NHWC
// Block: 32 bordered pixels of one bordered row (x), 64 channels. grid (ceil((W+2)/32), H+2, N*cgroups).
// Reads are coalesced along W (NCHW), writes along C (NHWC) through a shared-memory transpose.
// QUANT: T is a float type, values are quantised with the image's scale; otherwise T is int8
// copied as is. Border pixels and channels >= C are written as zeros.
template <typename T, bool QUANT>
__global__ void __launch_bounds__(256) to_bordered_nhwc_kernel(const T* __restrict__ x, int C, int H, int W,
                                                               int Cp, int cgroups, const uint32_t* __restrict__ amax,
                                                               int8_t* __restrict__ xp, float* __restrict__ sx) {
  __shared__ int8_t tile[64][33];
  const int xb0 = blockIdx.x * 32;  // bordered x of the block's first pixel
  const int yb = blockIdx.y;        // bordered y
  const int n = blockIdx.z / cgroups;
  const int c0 = (blockIdx.z - n * cgroups) * 64;
  const int Wp = W + 2;
  float s = 1.f;
  if constexpr (QUANT) {
    s = scale_from_amax(__uint_as_float(amax[n]));
    if (blockIdx.x == 0 && blockIdx.y == 0 && c0 == 0 && threadIdx.x == 0) sx[n] = s;
  }
  const int y = yb - 1;
  // load: thread (tx = lane, ty = warp) reads channels c0+ty, +8, ... at x = xb0 + tx - 1
  const int tx = threadIdx.x & 31;
  const int ty = threadIdx.x >> 5;
  const int xin = xb0 + tx - 1;
  const bool in_row = y >= 0 && y < H && xin >= 0 && xin < W;
  for (int cc = ty; cc < 64; cc += 8) {
    const int c = c0 + cc;
    int8_t q = 0;
    if (in_row && c < C) {
      const T v = x[((static_cast<int64_t>(n) * C + c) * H + y) * W + xin];
      if constexpr (QUANT)
        q = quant1(to_f32(v), s);
      else
        q = static_cast<int8_t>(v);
    }
    tile[cc][tx] = q;
  }
  __syncthreads();
  // store: 32 pixels x 64 channels; thread writes 8 consecutive channels of one pixel
  const int pix = threadIdx.x >> 3;       // 0..31
  const int cseg = (threadIdx.x & 7) * 8;  // 0..56
  const int xb = xb0 + pix;
  if (xb < Wp) {
    int8_t* dst = xp + ((static_cast<int64_t>(n) * (H + 2) + yb) * Wp + xb) * Cp + c0 + cseg;
    const int cmax = Cp - (c0 + cseg);
    if (cmax >= 8 && (reinterpret_cast<uintptr_t>(dst) & 7) == 0) {
      uint2 u;
      int8_t* b = reinterpret_cast<int8_t*>(&u);
#pragma unroll
      for (int j = 0; j < 8; ++j) b[j] = tile[cseg + j][pix];
      *reinterpret_cast<uint2*>(dst) = u;
    } else {
      for (int j = 0; j < 8 && j < cmax; ++j) dst[j] = tile[cseg + j][pix];
    }
  }
}

// wq [Co, Ci, 3, 3] -> wp [Co, 9, Cp], pad channels zero.
__global__ void pack_weight_kernel(const int8_t* __restrict__ wq, int64_t Co, int64_t Ci, int8_t* __restrict__ wp,
                                   int64_t Cp) {
  const int64_t total = Co * 9 * Cp;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t c = i % Cp;
    const int64_t tap = (i / Cp) % 9;
    const int64_t co = i / (9 * Cp);
    wp[i] = c < Ci ? wq[(co * Ci + c) * 9 + tap] : static_cast<int8_t>(0);
  }
}

}  // namespace xdna

using namespace xdna;

extern "C" {

int xdna_quant_rows_i8(const void* x, int x_dtype, int64_t rows, int64_t cols, int64_t ldx, int8_t* xq,
                       int64_t ldq, float* scale, void* stream) {
  int rc = check_device(nullptr);
  if (rc != XDNA_OK) return rc;
  XDNA_CHECK_ARG(rows >= 0 && cols >= 0, "quant_rows: negative size");
  XDNA_CHECK_ARG(ldx >= cols && ldq >= cols, "quant_rows: leading dimension smaller than cols");
  if (rows == 0) return XDNA_OK;
  XDNA_CHECK_ARG(x != nullptr && xq != nullptr && scale != nullptr, "quant_rows: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (x_dtype) {
    case XDNA_F32:
      return launch_quant_rows<float>(x, rows, cols, ldx, xq, ldq, scale, s);
    case XDNA_BF16:
      return launch_quant_rows<__nv_bfloat16>(x, rows, cols, ldx, xq, ldq, scale, s);
    case XDNA_F16:
      return launch_quant_rows<__half>(x, rows, cols, ldx, xq, ldq, scale, s);
    default:
      return fail(XDNA_ERR_INVALID, "quant_rows: x_dtype %d is not f32/bf16/f16", x_dtype);
  }
}

int xdna_conv_quant_nhwc(const void* x, int x_dtype, int64_t N, int64_t C, int64_t H, int64_t W, int8_t* xp,
                         int64_t Cp, float* sx, uint32_t* amax_scratch, void* stream) {
  int rc = check_device(nullptr);
  if (rc != XDNA_OK) return rc;
  XDNA_CHECK_ARG(N >= 0 && C >= 1 && H >= 1 && W >= 1, "conv_quant: bad shape");
  XDNA_CHECK_ARG(Cp >= C && Cp % 16 == 0, "conv_quant: Cp must be >= C and a multiple of 16");
  XDNA_CHECK_ARG(H + 2 <= 65535, "conv_quant: H too large");
  if (N == 0) return XDNA_OK;
  XDNA_CHECK_ARG(N * ((C + 63) / 64) <= 65535, "conv_quant: N * channel groups too large");
  XDNA_CHECK_ARG(x && xp && sx && amax_scratch, "conv_quant: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  XDNA_CUDA(cudaMemsetAsync(amax_scratch, 0, N * sizeof(uint32_t), s));
  const int64_t per_image = C * H * W;
  const int chunks = static_cast<int>(std::min<int64_t>((per_image + 256 * 16 - 1) / (256 * 16), 1024));
  const int cgroups = static_cast<int>((Cp + 63) / 64);
  dim3 g_amax(chunks, static_cast<unsigned>(N));
  dim3 g_tr(static_cast<unsigned>((W + 2 + 31) / 32), static_cast<unsigned>(H + 2), static_cast<unsigned>(N * cgroups));
  switch (x_dtype) {
    case XDNA_F32:
      image_amax_kernel<float><<<g_amax, 256, 0, s>>>(static_cast<const float*>(x), per_image, amax_scratch);
      to_bordered_nhwc_kernel<float, true><<<g_tr, 256, 0, s>>>(static_cast<const float*>(x), (int)C, (int)H, (int)W,
                                                                (int)Cp, cgroups, amax_scratch, xp, sx);
      break;
    case XDNA_BF16:
      image_amax_kernel<__nv_bfloat16>
          <<<g_amax, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), per_image, amax_scratch);
      to_bordered_nhwc_kernel<__nv_bfloat16, true><<<g_tr, 256, 0, s>>>(
          static_cast<const __nv_bfloat16*>(x), (int)C, (int)H, (int)W, (int)Cp, cgroups, amax_scratch, xp, sx);
      break;
    case XDNA_F16:
      image_amax_kernel<__half><<<g_amax, 256, 0, s>>>(static_cast<const __half*>(x), per_image, amax_scratch);
      to_bordered_nhwc_kernel<__half, true><<<g_tr, 256, 0, s>>>(static_cast<const __half*>(x), (int)C, (int)H,
                                                                 (int)W, (int)Cp, cgroups, amax_scratch, xp, sx);
      break;
    default:
      return fail(XDNA_ERR_INVALID, "conv_quant: x_dtype %d is not f32/bf16/f16", x_dtype);
  }
  return check_launch("conv quantise");
}

int xdna_conv_pack_input(const int8_t* xq, int64_t N, int64_t C, int64_t H, int64_t W, int8_t* xp, int64_t Cp,
                         void* stream) {
  int rc = check_device(nullptr);
  if (rc != XDNA_OK) return rc;
  XDNA_CHECK_ARG(N >= 0 && C >= 1 && H >= 1 && W >= 1, "conv_pack_input: bad shape");
  XDNA_CHECK_ARG(Cp >= C && Cp % 16 == 0, "conv_pack_input: Cp must be >= C and a multiple of 16");
  XDNA_CHECK_ARG(H + 2 <= 65535, "conv_pack_input: H too large");
  if (N == 0) return XDNA_OK;
  XDNA_CHECK_ARG(N * ((C + 63) / 64) <= 65535, "conv_pack_input: N * channel groups too large");
  XDNA_CHECK_ARG(xq && xp, "conv_pack_input: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int cgroups = static_cast<int>((Cp + 63) / 64);
  dim3 g(static_cast<unsigned>((W + 2 + 31) / 32), static_cast<unsigned>(H + 2), static_cast<unsigned>(N * cgroups));
  to_bordered_nhwc_kernel<int8_t, false>
      <<<g, 256, 0, s>>>(xq, (int)C, (int)H, (int)W, (int)Cp, cgroups, nullptr, xp, nullptr);
  return check_launch("conv pack input");
}

int xdna_conv_pack_weight(const int8_t* wq, int64_t Co, int64_t Ci, int8_t* wp, int64_t Cp, void* stream) {
  int rc = check_device(nullptr);
  if (rc != XDNA_OK) return rc;
  XDNA_CHECK_ARG(Co >= 1 && Ci >= 1 && Cp >= Ci && Cp % 16 == 0, "conv_pack_weight: bad shape");
  XDNA_CHECK_ARG(wq && wp, "conv_pack_weight: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t total = Co * 9 * Cp;
  const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 4096));
  pack_weight_kernel<<<blocks, 256, 0, s>>>(wq, Co, Ci, wp, Cp);
  return check_launch("conv pack weight");
}

}  // extern "C"
