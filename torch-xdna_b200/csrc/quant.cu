// Symmetric int8 quantisation kernels (HBM-bound):
//   - per row (activations of the W8A8 linear, and every weight matrix once);
//   - per image, fused with the NCHW -> zero-bordered NHWC layout the implicit-GEMM conv reads;
//   - int8 NCHW -> bordered NHWC (the xdna::conv3x3 op's own input), and the conv weight packing.
//
// Results equal the reference's bit for bit: the max of |x| is taken in x's dtype (exact), widened
// to f32, clamped below by 1e-8 and divided by 127 (IEEE division); each value becomes
// clamp(round_half_even(fl(x / scale)), -127, 127).
//
// The per-value division needs no divide instruction: with r = RN(1/scale), y = RN(x * r) is within
// an ulp of x / scale, and one FMA correction step, q = RN(y + r * RN(x - y * scale)), is the
// correctly rounded quotient fl(x / scale). This is the correction theorem of P. Markstein,
// "Computation of elementary functions on the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1),
// 1990 (Theorem 1: if y is within an ulp of a/b and r = RN(1/b), then RN(y + r * (a - b y)) = RN(a/b),
// the residual a - b y being exact in one FMA), as restated for FMA hardware by M. Cornea, J. Harrison
// and P. T. P. Tang, "Scientific Computing on Itanium-based Systems", Intel Press, 2002, ch. 8. Where the
// residual underflows, |x / scale| is far below 0.5 and both round to 0. The construction was checked
// against IEEE division on the final int8, exhaustively for every bf16 and every f16 (x, amax) pair with
// |x| <= amax and on 8.8e8 random f32 pairs: no difference; tests/test_linear_gpu.py compares it with
// numpy's IEEE division at edge scales (amax below the 1e-8 clamp, subnormal and huge values).
#include <algorithm>
#include <atomic>
#include <mutex>

#include "host_util.h"
#include "sm100.cuh"

namespace xdna {

template <typename T>
struct Vec16;  // elements of T in 16 bytes
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

// 1.5 * 2^23: adding it to |y| < 2^22 rounds y to an integer (ties to even) held in the low
// mantissa bits, two's complement in the low byte for -128 <= y <= 127.
constexpr float kRoundMagic = 12582912.0f;

// round_half_even(fl(v / s)) as the low byte of the returned float's bit pattern (two's complement
// for -128..127); r = RN(1 / s). |v| <= amax makes |v / s| <= 127 (scale = amax / 127): no clamp.
__device__ __forceinline__ float quant_t(float v, float s, float r) {
  const float y = __fmul_rn(v, r);
  const float q = __fmaf_rn(__fmaf_rn(-y, s, v), r, y);  // fl(v / s)
  return __fadd_rn(q, kRoundMagic);
}

__device__ __forceinline__ uint32_t quant_byte(float v, float s, float r) { return __float_as_uint(quant_t(v, s, r)); }

// Four int8 (the low bytes of t's bit patterns) in one word, byte i = value i.
__device__ __forceinline__ uint32_t pack_bytes(float t0, float t1, float t2, float t3) {
  const uint32_t lo = __byte_perm(__float_as_uint(t0), __float_as_uint(t1), 0x0040);
  const uint32_t hi = __byte_perm(__float_as_uint(t2), __float_as_uint(t3), 0x0040);
  return __byte_perm(lo, hi, 0x5410);
}

// Four values -> four int8 in one word (byte i = value i).
__device__ __forceinline__ uint32_t quant4(float a, float b, float c, float d, float s, float r) {
  return pack_bytes(quant_t(a, s, r), quant_t(b, s, r), quant_t(c, s, r), quant_t(d, s, r));
}

// max |x| over the 16 bytes of `u`, in x's own encoding: non-negative IEEE values order like their
// bit patterns, so the max is taken on integers with the sign bits cleared.
template <typename T>
__device__ __forceinline__ float amax16(const uint4& u);
template <>
__device__ __forceinline__ float amax16<float>(const uint4& u) {
  const uint32_t m = max(max(u.x & 0x7FFFFFFFu, u.y & 0x7FFFFFFFu), max(u.z & 0x7FFFFFFFu, u.w & 0x7FFFFFFFu));
  return __uint_as_float(m);
}
template <>
__device__ __forceinline__ float amax16<__nv_bfloat16>(const uint4& u) {
  uint32_t m = __vmaxu2(__vmaxu2(u.x & 0x7FFF7FFFu, u.y & 0x7FFF7FFFu), __vmaxu2(u.z & 0x7FFF7FFFu, u.w & 0x7FFF7FFFu));
  m = max(m & 0xFFFFu, m >> 16);
  return __uint_as_float(m << 16);  // bf16 bits are the top half of the f32 bits
}
template <>
__device__ __forceinline__ float amax16<__half>(const uint4& u) {
  uint32_t m = __vmaxu2(__vmaxu2(u.x & 0x7FFF7FFFu, u.y & 0x7FFF7FFFu), __vmaxu2(u.z & 0x7FFF7FFFu, u.w & 0x7FFF7FFFu));
  m = max(m & 0xFFFFu, m >> 16);
  return __half2float(__ushort_as_half(static_cast<unsigned short>(m)));
}

// 16 bytes of T as floats (4 or 8 values).
template <typename T>
struct Unpack16;
template <>
struct Unpack16<float> {
  static constexpr int N = 4;
  __device__ __forceinline__ static void get(const uint4& u, float (&v)[4]) {
    v[0] = __uint_as_float(u.x);
    v[1] = __uint_as_float(u.y);
    v[2] = __uint_as_float(u.z);
    v[3] = __uint_as_float(u.w);
  }
};
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
template <>
struct Unpack16<__nv_bfloat16> {
  static constexpr int N = 8;
  __device__ __forceinline__ static void get(const uint4& u, float (&v)[8]) {
    v[0] = bf16_lo(u.x), v[1] = bf16_hi(u.x), v[2] = bf16_lo(u.y), v[3] = bf16_hi(u.y);
    v[4] = bf16_lo(u.z), v[5] = bf16_hi(u.z), v[6] = bf16_lo(u.w), v[7] = bf16_hi(u.w);
  }
};
__device__ __forceinline__ float f16_lo(uint32_t w) { return __half2float(__ushort_as_half(static_cast<unsigned short>(w))); }
__device__ __forceinline__ float f16_hi(uint32_t w) { return __half2float(__ushort_as_half(static_cast<unsigned short>(w >> 16))); }
template <>
struct Unpack16<__half> {
  static constexpr int N = 8;
  __device__ __forceinline__ static void get(const uint4& u, float (&v)[8]) {
    v[0] = f16_lo(u.x), v[1] = f16_hi(u.x), v[2] = f16_lo(u.y), v[3] = f16_hi(u.y);
    v[4] = f16_lo(u.z), v[5] = f16_hi(u.z), v[6] = f16_lo(u.w), v[7] = f16_hi(u.w);
  }
};

// 16 bytes of T -> their int8 (4 or 8 bytes, as 1 or 2 words).
template <typename T>
__device__ __forceinline__ void quant16(const uint4& u, float s, float r, uint32_t (&out)[2]) {
  constexpr int N = Unpack16<T>::N;
  float v[N];
  Unpack16<T>::get(u, v);
  out[0] = quant4(v[0], v[1], v[2], v[3], s, r);
  out[1] = N == 8 ? quant4(v[N - 4], v[N - 3], v[N - 2], v[N - 1], s, r) : 0u;
}

// clamp(round_half_even(fl(v / s)), -127, 127) for one value (scalar paths); r = 1 / s.
__device__ __forceinline__ int8_t quant1(float v, float s, float r) {
  return static_cast<int8_t>(quant_byte(v, s, r) & 0xFFu);
}

// max(amax, 1e-8) / 127 as torch's clamp(min=1e-8) then / 127: a NaN amax stays NaN.
__device__ __forceinline__ float scale_from_amax(float amax) {
  return __fdiv_rn(amax < 1e-8f ? 1e-8f : amax, 127.f);
}

// The max of two absolute values (non-negative floats or NaN) by their bit patterns: non-negative floats
// order like their bits and every NaN pattern with the sign cleared sorts above +inf, so a NaN anywhere
// makes the max NaN, as torch's amax does (fmaxf would drop it).
__device__ __forceinline__ float amax_max(float a, float b) {
  return __uint_as_float(max(__float_as_uint(a), __float_as_uint(b)));
}

__device__ __forceinline__ float warp_max(float v) {
  return __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(v)));
}


// A warp's row in registers (NV lane-interleaved vectors per lane; vectors past the row are zeros)
// -> the row's scale and int8.
template <typename T, int NV>
__device__ __forceinline__ void quant_row_share(const uint4 (&buf)[NV], int64_t cols, int lane, float* scale_out,
                                                int8_t* qr) {
  constexpr int V = Vec16<T>::N;
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) amax = amax_max(amax, amax16<T>(buf[i]));
  amax = warp_max(amax);
  const float s = scale_from_amax(amax);
  const float r = __frcp_rn(s);
  if (lane == 0) *scale_out = s;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int64_t c = (static_cast<int64_t>(i) * 32 + lane) * V;
    if (c < cols) {
      uint32_t w[2];
      quant16<T>(buf[i], s, r, w);
      if constexpr (V == 4)
        *reinterpret_cast<uint32_t*>(qr + c) = w[0];
      else
        *reinterpret_cast<uint2*>(qr + c) = make_uint2(w[0], w[1]);
    }
  }
}

// One warp per row, the row held in registers: NV 16-byte vectors per lane, lane-interleaved so
// every load and store instruction of the warp is contiguous. One read of x, one write of xq.
template <typename T, int NV>
__global__ void __launch_bounds__(256, 3) quant_rows_reg_kernel(const T* __restrict__ x, int64_t rows, int64_t cols,
                                                             int64_t ldx, int8_t* __restrict__ xq, int64_t ldq,
                                                             float* __restrict__ scale) {
  constexpr int V = Vec16<T>::N;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int lane = threadIdx.x & 31;
  const T* xr = x + row * ldx;
  uint4 buf[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int64_t c = (static_cast<int64_t>(i) * 32 + lane) * V;
    buf[i] = c < cols ? __ldg(reinterpret_cast<const uint4*>(xr + c)) : make_uint4(0, 0, 0, 0);
  }
  quant_row_share<T, NV>(buf, cols, lane, scale + row, xq + row * ldq);
}

// Rows too long for registers, or not 16-byte addressable: two passes over the row.
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
      for (int j = 0; j < V; ++j) amax = amax_max(amax, fabsf(to_f32(e[j])));
    }
  } else {
    for (int64_t c = lane; c < cols; c += 32) amax = amax_max(amax, fabsf(to_f32(xr[c])));
  }
  amax = warp_max(amax);
  const float s = scale_from_amax(amax);
  const float r = __frcp_rn(s);
  if (lane == 0) scale[row] = s;
  if constexpr (VEC) {
    constexpr int V = Vec16<T>::N;
    for (int64_t c = static_cast<int64_t>(lane) * V; c < cols; c += 32 * V) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(xr + c));
      const T* e = reinterpret_cast<const T*>(&u);
      int8_t q[V];
#pragma unroll
      for (int j = 0; j < V; ++j) q[j] = quant1(to_f32(e[j]), s, r);
      if constexpr (V == 4)
        *reinterpret_cast<uint32_t*>(qr + c) = *reinterpret_cast<uint32_t*>(q);
      else
        *reinterpret_cast<uint2*>(qr + c) = *reinterpret_cast<uint2*>(q);
    }
  } else {
    for (int64_t c = lane; c < cols; c += 32) qr[c] = quant1(to_f32(xr[c]), s, r);
  }
}

template <typename T, int NV>
static int launch_rows(const T* x, int64_t rows, int64_t cols, int64_t ldx, int8_t* xq, int64_t ldq, float* scale,
                       unsigned grid, cudaStream_t stream) {
  quant_rows_reg_kernel<T, NV><<<grid, 256, 0, stream>>>(x, rows, cols, ldx, xq, ldq, scale);
  return check_launch("quant_rows_reg_kernel");
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
  const unsigned g = static_cast<unsigned>(blocks);
  const T* xt = static_cast<const T*>(x);
  const int64_t nv = (cols + 32 * V - 1) / (32 * V);  // 16-byte vectors per lane
  if (vec && nv <= 16) {
    if (nv <= 1) return launch_rows<T, 1>(xt, rows, cols, ldx, xq, ldq, scale, g, stream);
    if (nv <= 2) return launch_rows<T, 2>(xt, rows, cols, ldx, xq, ldq, scale, g, stream);
    if (nv <= 4) return launch_rows<T, 4>(xt, rows, cols, ldx, xq, ldq, scale, g, stream);
    if (nv <= 8) return launch_rows<T, 8>(xt, rows, cols, ldx, xq, ldq, scale, g, stream);
    if (nv <= 12) return launch_rows<T, 12>(xt, rows, cols, ldx, xq, ldq, scale, g, stream);
    return launch_rows<T, 16>(xt, rows, cols, ldx, xq, ldq, scale, g, stream);
  } else if (vec) {
    quant_rows_kernel<T, true><<<g, 256, 0, stream>>>(xt, rows, cols, ldx, xq, ldq, scale);
  } else {
    quant_rows_kernel<T, false><<<g, 256, 0, stream>>>(xt, rows, cols, ldx, xq, ldq, scale);
  }
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
    m = amax_max(m, fabsf(to_f32(xi[i])));
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
  float s = 1.f, r = 1.f;
  if constexpr (QUANT) {
    s = scale_from_amax(__uint_as_float(amax[n]));
    r = __frcp_rn(s);
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
        q = static_cast<int8_t>(quant_byte(to_f32(v), s, r) & 0xFFu);
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

// ---------------------------------------------------------------------------- channels-last -> bordered NHWC
// x is [N, H, W, C] in memory (torch's channels_last): no transpose, each bordered row is a stream of
// 4-channel words. grid (H + 2, N); border rows, border pixels and channels >= C are zeros.
template <typename T>
__global__ void __launch_bounds__(256) cl_to_bordered_kernel(const T* __restrict__ x, int C, int H, int W, int Cp,
                                                             const uint32_t* __restrict__ amax,
                                                             int8_t* __restrict__ xp, float* __restrict__ sx) {
  const int yb = blockIdx.x;
  const int n = blockIdx.y;
  const int Wp = W + 2;
  const float s = scale_from_amax(__uint_as_float(amax[n]));
  const float r = __frcp_rn(s);
  if (yb == 0 && threadIdx.x == 0) sx[n] = s;
  uint32_t* dst = reinterpret_cast<uint32_t*>(xp + (static_cast<int64_t>(n) * (H + 2) + yb) * Wp * Cp);
  const int words = Wp * Cp / 4;
  const bool border_row = yb == 0 || yb == H + 1;
  const int y = yb - 1;
  for (int e = threadIdx.x; e < words; e += blockDim.x) {
    const int xb = (e * 4) / Cp;
    const int c = e * 4 - xb * Cp;
    uint32_t word = 0;
    if (!border_row && xb >= 1 && xb <= W && c < C) {
      const T* src = x + ((static_cast<int64_t>(n) * H + y) * W + (xb - 1)) * C + c;
      float f[4];
      if (c + 4 <= C && (C & 3) == 0) {
        if constexpr (sizeof(T) == 4) {
          const float4 u = __ldg(reinterpret_cast<const float4*>(src));
          f[0] = u.x, f[1] = u.y, f[2] = u.z, f[3] = u.w;
        } else {
          const uint2 u = __ldg(reinterpret_cast<const uint2*>(src));
          const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
          for (int k = 0; k < 4; ++k) f[k] = to_f32(h[k]);
        }
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) f[k] = c + k < C ? to_f32(src[k]) : 0.f;
      }
      word = quant4(f[0], f[1], f[2], f[3], s, r);
      if (c + 4 > C) word &= 0xFFFFFFFFu >> (8 * (c + 4 - C));  // channels >= C stay zero
    }
    dst[e] = word;
  }
}

// ---------------------------------------------------------------------------- stride phases of a stride-2 conv
// xp [planes, N, Ho+2, Wo+2, Cp]: plane 2 ry + rx at bordered pixel (Y, X) holds the quantised input pixel
// (2 (Y - 1) + ry, 2 (X - 1) + rx), zeros on the border, past the input and for channels >= C. One block per
// bordered row of one plane of one image, grid (Ho + 2, planes * N), each thread a stream of 4-channel words as
// cl_to_bordered_kernel. CL: x is channels-last [N, H, W, C] (VEC: 4-channel vector loads), else NCHW.
template <typename T, bool CL, bool VEC>
__global__ void __launch_bounds__(256) to_phases_kernel(const T* __restrict__ x, int N, int C, int H, int W, int Ho,
                                                        int Wo, int Cp, const uint32_t* __restrict__ amax,
                                                        int8_t* __restrict__ xp, float* __restrict__ sx) {
  const int Yb = blockIdx.x;
  const int plane = blockIdx.y / N;
  const int n = blockIdx.y - plane * N;
  const int ry = plane >> 1, rx = plane & 1;
  const int Wp = Wo + 2;
  const float s = scale_from_amax(__uint_as_float(amax[n]));
  const float r = __frcp_rn(s);
  if (plane == 0 && Yb == 0 && threadIdx.x == 0) sx[n] = s;
  uint32_t* dst = reinterpret_cast<uint32_t*>(xp + ((static_cast<int64_t>(plane) * N + n) * (Ho + 2) + Yb) * Wp * Cp);
  const int words = Wp * Cp / 4;
  const int y = 2 * (Yb - 1) + ry;
  const bool row_ok = Yb >= 1 && Yb <= Ho && y < H;
  for (int e = threadIdx.x; e < words; e += blockDim.x) {
    const int Xb = (e * 4) / Cp;
    const int c = e * 4 - Xb * Cp;
    const int xx = 2 * (Xb - 1) + rx;
    uint32_t word = 0;
    if (row_ok && Xb >= 1 && Xb <= Wo && xx < W && c < C) {
      float f[4];
      if constexpr (CL) {
        const T* src = x + ((static_cast<int64_t>(n) * H + y) * W + xx) * C + c;
        if (VEC && c + 4 <= C) {
          if constexpr (sizeof(T) == 4) {
            const float4 u = __ldg(reinterpret_cast<const float4*>(src));
            f[0] = u.x, f[1] = u.y, f[2] = u.z, f[3] = u.w;
          } else {
            const uint2 u = __ldg(reinterpret_cast<const uint2*>(src));
            const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
            for (int k = 0; k < 4; ++k) f[k] = to_f32(h[k]);
          }
        } else {
#pragma unroll
          for (int k = 0; k < 4; ++k) f[k] = c + k < C ? to_f32(src[k]) : 0.f;
        }
      } else {
        const int64_t hw = static_cast<int64_t>(H) * W;
        const T* src = x + (static_cast<int64_t>(n) * C + c) * hw + static_cast<int64_t>(y) * W + xx;
#pragma unroll
        for (int k = 0; k < 4; ++k) f[k] = c + k < C ? to_f32(src[k * hw]) : 0.f;
      }
      word = quant4(f[0], f[1], f[2], f[3], s, r);
      if (c + 4 > C) word &= 0xFFFFFFFFu >> (8 * (c + 4 - C));  // channels >= C stay zero
    }
    dst[e] = word;
  }
}

// ---------------------------------------------------------------------------- NCHW -> tap-packed bordered
// One thread per bordered pixel (yb, xb), i.e. output pixel (yb - 1, xb - 1): the 3x3 stencil's taps of
// C <= 7 channels as 9 C quantised bytes of its Kp-byte row, tap t = 3 dy + dx reading input pixel
// (yb - 2 + dy, xb - 2 + dx); zeros outside the image and past byte 9 C. grid (ceil((H+2)(W+2) / 256), N).
// C is a template parameter, so the tap and channel loops unroll and the row's words stay in registers.
template <typename T, int C>
__global__ void __launch_bounds__(256) to_taps_kernel(const T* __restrict__ x, int H, int W,
                                                      const uint32_t* __restrict__ amax, int8_t* __restrict__ xp,
                                                      float* __restrict__ sx) {
  constexpr int Kp = (9 * C + 15) / 16 * 16;
  const int n = blockIdx.y;
  const int Wp = W + 2, HWp = (H + 2) * Wp;
  const int p = blockIdx.x * blockDim.x + threadIdx.x;
  const float s = scale_from_amax(__uint_as_float(amax[n]));
  const float r = __frcp_rn(s);
  if (blockIdx.x == 0 && threadIdx.x == 0) sx[n] = s;
  if (p >= HWp) return;
  const int yb = p / Wp, xb = p - yb * Wp;
  uint32_t words[Kp / 4];
#pragma unroll
  for (int i = 0; i < Kp / 4; ++i) words[i] = 0;
#pragma unroll
  for (int t = 0; t < 9; ++t) {
    const int y = yb - 2 + t / 3, xx = xb - 2 + t % 3;
    const bool in = y >= 0 && y < H && xx >= 0 && xx < W;
#pragma unroll
    for (int c = 0; c < C; ++c) {
      const uint32_t q =
          in ? quant_byte(to_f32(x[((static_cast<int64_t>(n) * C + c) * H + y) * W + xx]), s, r) & 0xFFu : 0u;
      const int k = t * C + c;
      words[k >> 2] |= q << (8 * (k & 3));
    }
  }
  uint4* dst = reinterpret_cast<uint4*>(xp + (static_cast<int64_t>(n) * HWp + p) * Kp);
#pragma unroll
  for (int i = 0; i < Kp / 16; ++i) dst[i] = make_uint4(words[4 * i], words[4 * i + 1], words[4 * i + 2], words[4 * i + 3]);
}

// ---------------------------------------------------------------------------- int8 codes -> bordered NHWC
// The next conv's input from a conv's channels-last codes q [N, H, W, C] (C % 4 == 0), read as words of 4
// channels. A code stands for y = float(q) * (scale[c] * sx[n]) (+ bias[c]) (then max(y, 0)), the same
// f32 operations as the conv's dequantising epilogue; y grows with q (scale, sx > 0), so a 2x2 max-pool
// of y is y of the bytewise max of the codes. amax pass: grid (chunks, N), one word per thread; quantise
// pass: grid (H' + 2, N) as cl_to_bordered_kernel.
template <bool POOL, bool USGN>
__device__ __forceinline__ uint32_t codes_word(const uint32_t* __restrict__ q, int n, int yo, int xo, int c4, int H, int W,
                                               int C4) {
  if constexpr (!POOL) {
    return __ldg(q + ((static_cast<int64_t>(n) * H + yo) * W + xo) * C4 + c4);
  } else {
    const uint32_t* p = q + ((static_cast<int64_t>(n) * H + 2 * yo) * W + 2 * xo) * C4 + c4;
    const uint32_t a = __ldg(p), b = __ldg(p + C4), c = __ldg(p + static_cast<int64_t>(W) * C4),
                   d = __ldg(p + static_cast<int64_t>(W) * C4 + C4);
    return USGN ? __vmaxu4(__vmaxu4(a, b), __vmaxu4(c, d)) : __vmaxs4(__vmaxs4(a, b), __vmaxs4(c, d));
  }
}

template <bool USGN>
__device__ __forceinline__ void codes_values(uint32_t word, int c, float t, const float* __restrict__ scale,
                                             const float* __restrict__ bias, bool relu_after, float (&v)[4]) {
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    const uint32_t byte = (word >> (8 * b)) & 0xFFu;
    const int qv = USGN ? static_cast<int>(byte) : static_cast<int>(static_cast<int8_t>(byte));
    float y = __fmul_rn(static_cast<float>(qv), __fmul_rn(__ldg(scale + c + b), t));
    if (bias != nullptr) y = __fadd_rn(y, __ldg(bias + c + b));
    if (relu_after) y = y > 0.f ? y : 0.f;
    v[b] = y;
  }
}

template <bool POOL, bool USGN>
__global__ void __launch_bounds__(256) codes_amax_kernel(const uint32_t* __restrict__ q, int H, int W, int C4,
                                                         const float* __restrict__ scale, const float* __restrict__ sx,
                                                         const float* __restrict__ bias, int relu_after,
                                                         uint32_t* __restrict__ amax) {
  const int n = blockIdx.y;
  const int Ho = POOL ? H / 2 : H, Wo = POOL ? W / 2 : W;
  const int64_t per = static_cast<int64_t>(Ho) * Wo * C4;
  const float t = __ldg(sx + n);
  float m = 0.f;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < per; i += stride) {
    const int c4 = static_cast<int>(i % C4);
    const int64_t pix = i / C4;
    const int xo = static_cast<int>(pix % Wo), yo = static_cast<int>(pix / Wo);
    float v[4];
    codes_values<USGN>(codes_word<POOL, USGN>(q, n, yo, xo, c4, H, W, C4), 4 * c4, t, scale, bias, relu_after != 0, v);
    m = fmaxf(m, fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3]))));
  }
  m = warp_max(m);
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float u = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    u = warp_max(u);
    if (threadIdx.x == 0) atomicMax(amax + n, __float_as_uint(u));
  }
}

template <bool POOL, bool USGN>
__global__ void __launch_bounds__(256) codes_to_bordered_kernel(const uint32_t* __restrict__ q, int H, int W, int C4,
                                                                const float* __restrict__ scale,
                                                                const float* __restrict__ sx_in,
                                                                const float* __restrict__ bias, int relu_after, int Cp,
                                                                const uint32_t* __restrict__ amax,
                                                                int8_t* __restrict__ xp, float* __restrict__ sx_out) {
  const int yb = blockIdx.x;
  const int n = blockIdx.y;
  const int Ho = POOL ? H / 2 : H, Wo = POOL ? W / 2 : W;
  const int Wp = Wo + 2;
  const float s = scale_from_amax(__uint_as_float(amax[n]));
  const float r = __frcp_rn(s);
  const float t = __ldg(sx_in + n);
  if (yb == 0 && threadIdx.x == 0) sx_out[n] = s;
  uint32_t* dst = reinterpret_cast<uint32_t*>(xp + (static_cast<int64_t>(n) * (Ho + 2) + yb) * Wp * Cp);
  const int words = Wp * Cp / 4;
  const bool border_row = yb == 0 || yb == Ho + 1;
  for (int e = threadIdx.x; e < words; e += blockDim.x) {
    const int xb = (e * 4) / Cp;
    const int c = e * 4 - xb * Cp;
    uint32_t word = 0;
    if (!border_row && xb >= 1 && xb <= Wo && c < 4 * C4) {
      float v[4];
      codes_values<USGN>(codes_word<POOL, USGN>(q, n, yb - 1, xb - 1, c / 4, H, W, C4), c, t, scale, bias,
                         relu_after != 0, v);
      word = quant4(v[0], v[1], v[2], v[3], s, r);
    }
    dst[e] = word;
  }
}

// The same quantise, 16 bytes per thread, for C = Cp a power of two (16 .. 4096) and 16-byte aligned
// tensors: a thread always handles the same 16 channels (256 threads x 16 bytes is a whole number of
// pixels), so their factors t[c] = fl(scale[c] * sx_in[n]) and biases stay in registers, and a block
// walks several bordered rows of one image. A code becomes a float exactly through the 2^23 bias (the
// bit pattern 0x4B000000 + u is 2^23 + u; a signed code is stored as u = code + 128 first); then
// y = fl(q * t[c]) + b[c] (+0 without a bias: the same quantised byte), the ReLU, round(y / s) as quant_t.
// PAIRS: xp holds the images in pairs, [N/2, Ho+2, Wo+2, 2 x C] (XDNA_CONV_PAIRS): image n's bytes of a pixel
// are the (n % 2)-th C of the pair row.
template <bool POOL, bool USGN, bool PAIRS = false>
__global__ void __launch_bounds__(256) codes_to_bordered16_kernel(const uint4* __restrict__ q, int H, int W, int C,
                                                                  const float* __restrict__ scale,
                                                                  const float* __restrict__ sx_in,
                                                                  const float* __restrict__ bias, int relu_after,
                                                                  const uint32_t* __restrict__ amax,
                                                                  uint4* __restrict__ xp, float* __restrict__ sx_out) {
  const int n = blockIdx.y;
  const int Ho = POOL ? H / 2 : H, Wo = POOL ? W / 2 : W;
  const int Wp = Wo + 2;
  const int C16 = C / 16;  // 16-byte chunks per pixel (a power of two <= 256)
  const float s = scale_from_amax(__uint_as_float(amax[n]));
  const float r = __frcp_rn(s);
  if (blockIdx.x == 0 && threadIdx.x == 0) sx_out[n] = s;
  const int chunk = threadIdx.x & (C16 - 1);
  const float sxn = __ldg(sx_in + n);
  float t[16], b[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int c = chunk * 16 + j;
    t[j] = __fmul_rn(__ldg(scale + c), sxn);
    b[j] = bias != nullptr ? __ldg(bias + c) : 0.f;
  }
  const float unbias = USGN ? 8388608.f : 8388736.f;  // 2^23 (+ 128: signed codes stored as code + 128)
  const uint32_t flip = USGN ? 0u : 0x80808080u;
  const int per_row = Wp * C16;
  auto load = [&](int yb, int xb) {  // the pixel's 16 codes, signed ones as code + 128 (pooled: the 2x2 max)
    if constexpr (!POOL) {
      const uint4 u = __ldg(q + ((static_cast<int64_t>(n) * H + (yb - 1)) * W + (xb - 1)) * C16 + chunk);
      return make_uint4(u.x ^ flip, u.y ^ flip, u.z ^ flip, u.w ^ flip);
    } else {
      const int64_t p0 = ((static_cast<int64_t>(n) * H + 2 * (yb - 1)) * W + 2 * (xb - 1)) * C16 + chunk;
      const int64_t row = static_cast<int64_t>(W) * C16;
      const uint4 a = __ldg(q + p0), bq = __ldg(q + p0 + C16), c = __ldg(q + p0 + row), d = __ldg(q + p0 + row + C16);
      auto mx = [&](uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3) {
        return __vmaxu4(__vmaxu4(w0 ^ flip, w1 ^ flip), __vmaxu4(w2 ^ flip, w3 ^ flip));
      };
      return make_uint4(mx(a.x, bq.x, c.x, d.x), mx(a.y, bq.y, c.y, d.y), mx(a.z, bq.z, c.z, d.z),
                        mx(a.w, bq.w, c.w, d.w));
    }
  };
  auto convert = [&](const uint4& u) {
    const uint32_t wi[4] = {u.x, u.y, u.z, u.w};
    uint32_t wo[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float v[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float qf = __fsub_rn(__uint_as_float(__byte_perm(wi[k], 0x4B000000u, 0x7540u + i)), unbias);
        float y = __fadd_rn(__fmul_rn(qf, t[4 * k + i]), b[4 * k + i]);
        if (relu_after) y = y > 0.f ? y : 0.f;
        v[i] = quant_t(y, s, r);
      }
      wo[k] = pack_bytes(v[0], v[1], v[2], v[3]);
    }
    return make_uint4(wo[0], wo[1], wo[2], wo[3]);
  };
  constexpr int U = POOL ? 2 : 4;  // 16-byte vectors per thread in flight (a pooled one is four loads)
  for (int yb = blockIdx.x; yb < Ho + 2; yb += gridDim.x) {
    // this image's row: plain, or every other C bytes of its pair's row
    uint4* dst = PAIRS ? xp + (static_cast<int64_t>(n >> 1) * (Ho + 2) + yb) * 2 * per_row + (n & 1) * C16
                       : xp + (static_cast<int64_t>(n) * (Ho + 2) + yb) * per_row;
    const bool border_row = yb == 0 || yb == Ho + 1;
    for (int e0 = threadIdx.x; e0 < per_row; e0 += U * blockDim.x) {
      uint4 u[U];
      bool in[U];
#pragma unroll
      for (int j = 0; j < U; ++j) {  // all loads first
        const int e = e0 + j * blockDim.x;
        const int xb = e / C16;  // C16 a power of two: a shift
        in[j] = e < per_row && !border_row && xb >= 1 && xb <= Wo;
        u[j] = in[j] ? load(yb, xb) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int j = 0; j < U; ++j) {
        const int e = e0 + j * blockDim.x;
        if (e < per_row) dst[PAIRS ? e + (e / C16) * C16 : e] = in[j] ? convert(u[j]) : make_uint4(0u, 0u, 0u, 0u);
      }
    }
  }
}

__device__ __forceinline__ void cp_async16(uint32_t smem, const void* gmem, bool fill) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem), "l"(gmem), "r"(fill ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// The same quantise through a table, for C a multiple of 64: within one image a code's next-layer byte
// depends only on the code's byte u (signed codes stored as code + 128) and its channel c, so a block
// first evaluates byte(c, u) for its 64 channels (grid z: the channel slice) and all 256 u into 16 KB of
// shared memory, with the arithmetic of codes_to_bordered16_kernel operation for operation (so the bytes
// are the same), then maps each code with one byte permute and one shared-memory byte load instead of
// ~11 floating-point operations. Row c of the table holds u at column u ^ (32 * (c / 16)): the four
// 16-channel chunks a warp reads at once start 8 banks apart, and the XOR is applied to a whole word of
// codes before the bytes are taken out. A block covers a contiguous range of bordered rows, flattened
// into (row, pixel, chunk) elements; the row of an element comes from a multiply-high by wp_magic =
// ceil(2^32 / Wp), exact while (rows x Wp) x (Wp - 1) < 2^32 (checked by the host).
// The codes are prefetched into shared memory, not registers: each thread owns a ring of kRingStages x 4
// sixteen-byte slots (slot (stage, v) of thread t at [(stage * 4 + v) * 256 + t], so a warp's slot reads
// are conflict-free) and fills them with cp.async, zero-filling what lies outside the image; two stages
// are in flight while it converts the third, the first two while the block builds its table. A thread
// reads only its own slots and waits only on its own copies (cp.async.wait_group), so the ring needs no
// barrier; a slot is refilled one iteration after it was read, once the stores that used its codes have
// issued. Pooled, a stage holds the four codes vectors of one output vector. Dynamic shared memory: the
// 16 KB table, then the 48 KB ring (three blocks per SM).
constexpr int kRingStages = 3;
constexpr size_t kRingSmem = 64 * 256 + static_cast<size_t>(kRingStages) * 4 * 256 * 16;

template <bool POOL, bool USGN, bool PAIRS = false>
__global__ void __launch_bounds__(256, 3) codes_lut_kernel(const uint4* __restrict__ q, int H, int W, int C,
                                                           const float* __restrict__ scale,
                                                           const float* __restrict__ sx_in,
                                                           const float* __restrict__ bias, int relu_after,
                                                           const uint32_t* __restrict__ amax, uint4* __restrict__ xp,
                                                           float* __restrict__ sx_out, uint32_t wp_magic) {
  extern __shared__ __align__(16) uint8_t ring_sm[];
  uint8_t* tbl = ring_sm;
  uint4* ring = reinterpret_cast<uint4*>(ring_sm + 64 * 256);
  const int n = blockIdx.y, sl = blockIdx.z;
  const int Ho = POOL ? H / 2 : H, Wo = POOL ? W / 2 : W;
  const int Wp = Wo + 2;
  const int C16 = C / 16;
  const float s = scale_from_amax(__uint_as_float(amax[n]));
  const float r = __frcp_rn(s);
  if (blockIdx.x == 0 && sl == 0 && threadIdx.x == 0) sx_out[n] = s;
  const int chunk = threadIdx.x & 3;
  const uint32_t flip = USGN ? 0u : 0x80808080u;
  const uint32_t swz = 0x20202020u * static_cast<uint32_t>(chunk);
  const uint32_t rowb = static_cast<uint32_t>(chunk) << 12;
  const int col = sl * 4 + chunk;
  const int rows = Ho + 2;
  const int y0 = static_cast<int>(static_cast<int64_t>(blockIdx.x) * rows / gridDim.x);
  const int y1 = static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * rows / gridDim.x);
  const int total = (y1 - y0) * Wp * 4;
  constexpr int U = POOL ? 1 : 4;  // output vectors per stage (a pooled one reads four)
  const int step = U * static_cast<int>(blockDim.x);
  auto pixel = [&](int g, int& yb, int& xb, bool& in) {
    const uint32_t px = static_cast<uint32_t>(g) >> 2;
    const int yl = static_cast<int>(__umulhi(px, wp_magic));
    xb = static_cast<int>(px) - yl * Wp;
    yb = y0 + yl;
    in = g < total && yb >= 1 && yb <= Ho && xb >= 1 && xb <= Wo;
  };
  const uint32_t ring_base = static_cast<uint32_t>(__cvta_generic_to_shared(ring)) + threadIdx.x * 16;
  auto issue = [&](int g0, int stage) {  // the codes of elements g0, g0 + 256, ... into the stage's slots
#pragma unroll
    for (int j = 0; j < U; ++j) {
      int yb, xb;
      bool in;
      pixel(g0 + j * static_cast<int>(blockDim.x), yb, xb, in);
      if constexpr (!POOL) {
        const uint4* src = in ? q + ((static_cast<int64_t>(n) * H + (yb - 1)) * W + (xb - 1)) * C16 + col : q;
        cp_async16(ring_base + (stage * 4 + j) * 256 * 16, src, in);
      } else {
        const int64_t p0 = in ? ((static_cast<int64_t>(n) * H + 2 * (yb - 1)) * W + 2 * (xb - 1)) * C16 + col : 0;
        const int64_t row = in ? static_cast<int64_t>(W) * C16 : 0;
        const int64_t off[4] = {p0, p0 + (in ? C16 : 0), p0 + row, p0 + row + (in ? C16 : 0)};
#pragma unroll
        for (int v = 0; v < 4; ++v) cp_async16(ring_base + (stage * 4 + v) * 256 * 16, q + off[v], in);
      }
    }
    cp_async_commit();
  };
  // the first stages' copies are in flight while the block builds its table
  int g_issue = threadIdx.x;
#pragma unroll
  for (int st = 0; st < kRingStages - 1; ++st, g_issue += step) issue(g_issue, st);

  const float sxn = __ldg(sx_in + n);
  const float unbias = USGN ? 8388608.f : 8388736.f;
  for (int e = threadIdx.x; e < 64 * 64; e += 256) {
    const int c = e >> 6, u0 = (e & 63) * 4;
    const float t = __fmul_rn(__ldg(scale + sl * 64 + c), sxn);
    const float b = bias != nullptr ? __ldg(bias + sl * 64 + c) : 0.f;
    float v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float qf = __fsub_rn(__uint_as_float(0x4B000000u | static_cast<uint32_t>(u0 + i)), unbias);
      float y = __fadd_rn(__fmul_rn(qf, t), b);
      if (relu_after) y = y > 0.f ? y : 0.f;
      v[i] = quant_t(y, s, r);
    }
    *reinterpret_cast<uint32_t*>(tbl + c * 256 + (u0 ^ ((c >> 4) << 5))) = pack_bytes(v[0], v[1], v[2], v[3]);
  }
  __syncthreads();

  auto convert = [&](const uint4& u) {
    const uint32_t wi[4] = {u.x ^ swz, u.y ^ swz, u.z ^ swz, u.w ^ swz};
    uint32_t wo[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) o[i] = tbl[__byte_perm(wi[k], rowb, 0x7650u + i) + (4 * k + i) * 256];
      wo[k] = __byte_perm(__byte_perm(o[0], o[1], 0x0040), __byte_perm(o[2], o[3], 0x0040), 0x5410);
    }
    return make_uint4(wo[0], wo[1], wo[2], wo[3]);
  };
  int stage = 0;
  for (int g0 = threadIdx.x; g0 < total; g0 += step) {
    cp_async_wait<kRingStages - 2>();  // this stage's group has landed
    uint4 u[U];
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const uint4* slot = ring + (stage * 4 + j) * 256 + threadIdx.x;
      if constexpr (!POOL) {
        const uint4 a = slot[0];
        u[j] = make_uint4(a.x ^ flip, a.y ^ flip, a.z ^ flip, a.w ^ flip);
      } else {
        const uint4 a = slot[0], b = slot[256], c = slot[512], d = slot[768];
        auto mx = [&](uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3) {
          return __vmaxu4(__vmaxu4(w0 ^ flip, w1 ^ flip), __vmaxu4(w2 ^ flip, w3 ^ flip));
        };
        u[j] = make_uint4(mx(a.x, b.x, c.x, d.x), mx(a.y, b.y, c.y, d.y), mx(a.z, b.z, c.z, d.z), mx(a.w, b.w, c.w, d.w));
      }
    }
    // refill the slots read one iteration ago (an empty group past the end keeps the count uniform)
    issue(g_issue, (stage + kRingStages - 1) % kRingStages);
    g_issue += step;
#pragma unroll
    for (int j = 0; j < U; ++j) {
      const int g = g0 + j * static_cast<int>(blockDim.x);
      int yb, xb;
      bool in;
      pixel(g, yb, xb, in);
      if (g < total) {
        const int64_t at = PAIRS ? ((static_cast<int64_t>(n >> 1) * rows + yb) * Wp + xb) * 2 * C16 + (n & 1) * C16 + col
                                 : ((static_cast<int64_t>(n) * rows + yb) * Wp + xb) * C16 + col;
        xp[at] = in ? convert(u[j]) : make_uint4(0u, 0u, 0u, 0u);
      }
    }
    stage = stage + 1 == kRingStages ? 0 : stage + 1;
  }
  cp_async_wait<0>();  // no copy outlives the block
}

// XDNA_CODES_LUT: 0 = never the table kernel, 2 = wherever it applies, else (default) where it pays.
static int codes_lut() {
  static const int mode = [] {
    const char* e = std::getenv("XDNA_CODES_LUT");
    return e == nullptr ? 1 : e[0] == '0' ? 0 : e[0] == '2' ? 2 : 1;
  }();
  return mode;
}

template <bool POOL, bool USGN>
static void launch_codes(const uint32_t* q, int N, int H, int W, int C4, const float* scale, const float* sx_in,
                         const float* bias, int relu_after, int Cp, uint32_t* amax, int8_t* xp, float* sx_out,
                         cudaStream_t s, bool amax_given = false, bool pairs = false) {
  const int Ho = POOL ? H / 2 : H;
  const int64_t per = static_cast<int64_t>(Ho) * (POOL ? W / 2 : W) * C4;
  const int chunks = static_cast<int>(std::min<int64_t>((per + 256 * 8 - 1) / (256 * 8), 1024));
  if (!amax_given)
    codes_amax_kernel<POOL, USGN><<<dim3(chunks, N), 256, 0, s>>>(q, H, W, C4, scale, sx_in, bias, relu_after, amax);
  const int C = 4 * C4;
  const bool pow2 = C >= 16 && C <= 4096 && (C & (C - 1)) == 0;
  const bool al16 = reinterpret_cast<uintptr_t>(q) % 16 == 0 && reinterpret_cast<uintptr_t>(xp) % 16 == 0;
  const int Wp = (POOL ? W / 2 : W) + 2;
  const int slices = C / 64;
  // the table kernel: three blocks per SM (64 KB of shared memory each) over all (image, slice) pairs. It
  // pays where a block maps at least one table's worth of codes, or where many (image, slice) pairs leave
  // each block few rows (the direct kernel is then worse still); a small batch of large images keeps the
  // direct kernel.
  const int pairs_ns = N * std::max(slices, 1);
  const int parts = std::max(1, std::min(Ho + 2, 148 * 3 / std::max(pairs_ns, 1)));
  const int64_t codes_per_block = static_cast<int64_t>(Ho) * (Wp - 2) * 64 / parts;
  if (codes_lut() != 0 && C % 64 == 0 && slices <= 65535 && Cp == C && al16 &&
      (codes_lut() == 2 || codes_per_block >= 16384 || pairs_ns >= 128) &&
      static_cast<int64_t>(Ho + 2) * Wp * (Wp - 1) < (int64_t{1} << 32)) {
    const uint32_t magic = static_cast<uint32_t>(((uint64_t{1} << 32) + Wp - 1) / Wp);
    const dim3 grid(parts, N, slices);
    static const bool attr = [] {  // 64 KB of dynamic shared memory
      cudaFuncSetAttribute(codes_lut_kernel<POOL, USGN, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(kRingSmem));
      cudaFuncSetAttribute(codes_lut_kernel<POOL, USGN, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(kRingSmem));
      return true;
    }();
    (void)attr;
    if (pairs)
      codes_lut_kernel<POOL, USGN, true><<<grid, 256, kRingSmem, s>>>(reinterpret_cast<const uint4*>(q), H, W, C,
                                                                     scale, sx_in, bias, relu_after, amax,
                                                                     reinterpret_cast<uint4*>(xp), sx_out, magic);
    else
      codes_lut_kernel<POOL, USGN><<<grid, 256, kRingSmem, s>>>(reinterpret_cast<const uint4*>(q), H, W, C, scale,
                                                               sx_in, bias, relu_after, amax,
                                                               reinterpret_cast<uint4*>(xp), sx_out, magic);
  } else if (pow2 && Cp == C && al16) {
    // one wave: three resident blocks per SM over all images, each walking several rows
    const int blocks = std::max(1, std::min(Ho + 2, 148 * 3 / std::max(N, 1)));
    if (pairs)
      codes_to_bordered16_kernel<POOL, USGN, true><<<dim3(blocks, N), 256, 0, s>>>(
          reinterpret_cast<const uint4*>(q), H, W, C, scale, sx_in, bias, relu_after, amax,
          reinterpret_cast<uint4*>(xp), sx_out);
    else
      codes_to_bordered16_kernel<POOL, USGN><<<dim3(blocks, N), 256, 0, s>>>(
          reinterpret_cast<const uint4*>(q), H, W, C, scale, sx_in, bias, relu_after, amax,
          reinterpret_cast<uint4*>(xp), sx_out);
  } else {
    codes_to_bordered_kernel<POOL, USGN>
        <<<dim3(Ho + 2, N), 256, 0, s>>>(q, H, W, C4, scale, sx_in, bias, relu_after, Cp, amax, xp, sx_out);
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

template <typename T>
static void launch_phases(const void* x, bool cl, bool vec, int N, int C, int H, int W, int Ho, int Wo, int Cp,
                          dim3 grid, const uint32_t* amax, int8_t* xp, float* sx, cudaStream_t s) {
  const T* xt = static_cast<const T*>(x);
  if (!cl)
    to_phases_kernel<T, false, false><<<grid, 256, 0, s>>>(xt, N, C, H, W, Ho, Wo, Cp, amax, xp, sx);
  else if (vec)
    to_phases_kernel<T, true, true><<<grid, 256, 0, s>>>(xt, N, C, H, W, Ho, Wo, Cp, amax, xp, sx);
  else
    to_phases_kernel<T, true, false><<<grid, 256, 0, s>>>(xt, N, C, H, W, Ho, Wo, Cp, amax, xp, sx);
}

// out[n][co] = rint(bias[co] / (sw[co] * sx[n])), clamped to [-2^29, 2^29], NaN -> 0 (XDNA_CONV_BIAS_INT32).
template <typename T>
__global__ void __launch_bounds__(256) bias_int32_kernel(const T* __restrict__ bias, const float* __restrict__ sw,
                                                         const float* __restrict__ sx, int N, int Co,
                                                         int32_t* __restrict__ out) {
  const int64_t total = static_cast<int64_t>(N) * Co;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int n = static_cast<int>(i / Co), c = static_cast<int>(i - static_cast<int64_t>(n) * Co);
    const float v = rintf(__fdiv_rn(to_f32(bias[c]), __fmul_rn(sw[c], sx[n])));
    const float lim = 536870912.f;  // 2^29
    out[i] = v != v ? 0 : static_cast<int32_t>(fminf(fmaxf(v, -lim), lim));
  }
}

// The same taps, one block per bordered row yb for C <= 4: the three input rows yb - 2 .. yb that the row's
// stencils read are quantised once into shared memory, one word per pixel (channel c in byte c, zero
// outside the image; columns -2 .. W + 1), and each pixel's 9 C bytes are assembled from nine of those
// words with constant shifts. An input value is quantised three times (once per row block reading it)
// instead of nine, and loaded as one coalesced row instead of per stencil. grid (H + 2, N), shared memory
// 3 (W + 4) words.
template <typename T, int C>
__global__ void __launch_bounds__(256) to_taps_rows_kernel(const T* __restrict__ x, int H, int W,
                                                           const uint32_t* __restrict__ amax,
                                                           int8_t* __restrict__ xp, float* __restrict__ sx) {
  static_assert(C >= 1 && C <= 4, "one word per pixel");
  constexpr int Kp = (9 * C + 15) / 16 * 16;
  extern __shared__ uint32_t rows_sm[];  // [3][W + 4]
  const int n = blockIdx.y, yb = blockIdx.x;
  const int Wp = W + 2, Ws = W + 4;
  const float s = scale_from_amax(__uint_as_float(amax[n]));
  const float r = __frcp_rn(s);
  if (yb == 0 && threadIdx.x == 0) sx[n] = s;
  for (int e = threadIdx.x; e < 3 * Ws; e += blockDim.x) {
    const int dy = e / Ws, xi = e - dy * Ws;
    const int y = yb - 2 + dy, xx = xi - 2;
    uint32_t word = 0;
    if (y >= 0 && y < H && xx >= 0 && xx < W) {
#pragma unroll
      for (int c = 0; c < C; ++c)
        word |= (quant_byte(to_f32(x[((static_cast<int64_t>(n) * C + c) * H + y) * W + xx]), s, r) & 0xFFu) << (8 * c);
    }
    rows_sm[e] = word;
  }
  __syncthreads();
  for (int xb = threadIdx.x; xb < Wp; xb += blockDim.x) {
    uint32_t words[Kp / 4];
#pragma unroll
    for (int i = 0; i < Kp / 4; ++i) words[i] = 0;
#pragma unroll
    for (int t = 0; t < 9; ++t) {  // tap t's C bytes at byte C t of the row: input column xb - 2 + t % 3
      const uint32_t p = rows_sm[(t / 3) * Ws + xb + t % 3];
      constexpr int kBits = 8 * C;
      const int bit = kBits * t, i = bit >> 5, sh = bit & 31;
      words[i] |= p << sh;
      if (sh + kBits > 32) words[i + 1] |= p >> (32 - sh);
    }
    uint4* dst = reinterpret_cast<uint4*>(xp + (static_cast<int64_t>(n) * (H + 2) * Wp + static_cast<int64_t>(yb) * Wp + xb) * Kp);
#pragma unroll
    for (int i = 0; i < Kp / 16; ++i) dst[i] = make_uint4(words[4 * i], words[4 * i + 1], words[4 * i + 2], words[4 * i + 3]);
  }
}

template <typename T>
static void launch_taps(const T* x, int C, int H, int W, dim3 g, const uint32_t* amax, int8_t* xp, float* sx,
                        cudaStream_t s) {
  const size_t rows_smem = static_cast<size_t>(3) * (W + 4) * sizeof(uint32_t);
  if (C <= 4 && rows_smem <= 48 * 1024 && H + 2 <= 2147483647) {
    const dim3 gr(static_cast<unsigned>(H + 2), g.y);
    switch (C) {
      case 1: to_taps_rows_kernel<T, 1><<<gr, 256, rows_smem, s>>>(x, H, W, amax, xp, sx); break;
      case 2: to_taps_rows_kernel<T, 2><<<gr, 256, rows_smem, s>>>(x, H, W, amax, xp, sx); break;
      case 3: to_taps_rows_kernel<T, 3><<<gr, 256, rows_smem, s>>>(x, H, W, amax, xp, sx); break;
      default: to_taps_rows_kernel<T, 4><<<gr, 256, rows_smem, s>>>(x, H, W, amax, xp, sx); break;
    }
    return;
  }
  switch (C) {
    case 1: to_taps_kernel<T, 1><<<g, 256, 0, s>>>(x, H, W, amax, xp, sx); break;
    case 2: to_taps_kernel<T, 2><<<g, 256, 0, s>>>(x, H, W, amax, xp, sx); break;
    case 3: to_taps_kernel<T, 3><<<g, 256, 0, s>>>(x, H, W, amax, xp, sx); break;
    case 4: to_taps_kernel<T, 4><<<g, 256, 0, s>>>(x, H, W, amax, xp, sx); break;
    case 5: to_taps_kernel<T, 5><<<g, 256, 0, s>>>(x, H, W, amax, xp, sx); break;
    case 6: to_taps_kernel<T, 6><<<g, 256, 0, s>>>(x, H, W, amax, xp, sx); break;
    default: to_taps_kernel<T, 7><<<g, 256, 0, s>>>(x, H, W, amax, xp, sx); break;
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

int xdna_conv_quant_phases(const void* x, int x_dtype, int x_channels_last, int64_t N, int64_t C, int64_t H,
                           int64_t W, int planes, int8_t* xp, int64_t Cp, float* sx, uint32_t* amax_scratch,
                           void* stream) {
  int rc = check_device(nullptr);
  if (rc != XDNA_OK) return rc;
  XDNA_CHECK_ARG(N >= 0 && C >= 1 && H >= 1 && W >= 1, "conv_quant_phases: bad shape");
  XDNA_CHECK_ARG(planes == 1 || planes == 4, "conv_quant_phases: planes must be 1 or 4");
  XDNA_CHECK_ARG(Cp >= C && Cp % 16 == 0, "conv_quant_phases: Cp must be >= C and a multiple of 16");
  const int64_t Ho = (H + 1) / 2, Wo = (W + 1) / 2;
  XDNA_CHECK_ARG(Ho + 2 <= 65535 && N * planes <= 65535, "conv_quant_phases: image or batch too large");
  XDNA_CHECK_ARG(N * C * H * W < (1ll << 40) && (Wo + 2) * Cp < (1ll << 31), "conv_quant_phases: too large");
  if (N == 0) return XDNA_OK;
  XDNA_CHECK_ARG(x && xp && sx && amax_scratch, "conv_quant_phases: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  XDNA_CUDA(cudaMemsetAsync(amax_scratch, 0, N * sizeof(uint32_t), s));
  const int64_t per_image = C * H * W;  // an image is contiguous in either layout
  const int chunks = static_cast<int>(std::min<int64_t>((per_image + 256 * 16 - 1) / (256 * 16), 1024));
  const dim3 g_amax(chunks, static_cast<unsigned>(N));
  const dim3 g_ph(static_cast<unsigned>(Ho + 2), static_cast<unsigned>(N * planes));
  const bool cl = x_channels_last != 0;
  const bool vec = cl && C % 4 == 0 && aligned16(x);
  switch (x_dtype) {
    case XDNA_F32:
      image_amax_kernel<float><<<g_amax, 256, 0, s>>>(static_cast<const float*>(x), per_image, amax_scratch);
      launch_phases<float>(x, cl, vec, (int)N, (int)C, (int)H, (int)W, (int)Ho, (int)Wo, (int)Cp, g_ph, amax_scratch,
                           xp, sx, s);
      break;
    case XDNA_BF16:
      image_amax_kernel<__nv_bfloat16>
          <<<g_amax, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), per_image, amax_scratch);
      launch_phases<__nv_bfloat16>(x, cl, vec, (int)N, (int)C, (int)H, (int)W, (int)Ho, (int)Wo, (int)Cp, g_ph,
                                   amax_scratch, xp, sx, s);
      break;
    case XDNA_F16:
      image_amax_kernel<__half><<<g_amax, 256, 0, s>>>(static_cast<const __half*>(x), per_image, amax_scratch);
      launch_phases<__half>(x, cl, vec, (int)N, (int)C, (int)H, (int)W, (int)Ho, (int)Wo, (int)Cp, g_ph, amax_scratch,
                            xp, sx, s);
      break;
    default:
      return fail(XDNA_ERR_INVALID, "conv_quant_phases: x_dtype %d is not f32/bf16/f16", x_dtype);
  }
  return check_launch("conv quantise (stride phases)");
}

int xdna_conv_quant_taps(const void* x, int x_dtype, int64_t N, int64_t C, int64_t H, int64_t W, int8_t* xp,
                         int64_t Kp, float* sx, uint32_t* amax_scratch, void* stream) {
  int rc = check_device(nullptr);
  if (rc != XDNA_OK) return rc;
  XDNA_CHECK_ARG(N >= 0 && C >= 1 && C <= 7 && H >= 1 && W >= 1, "conv_quant_taps: bad shape (1 <= C <= 7)");
  XDNA_CHECK_ARG(Kp == (9 * C + 15) / 16 * 16, "conv_quant_taps: Kp must be 9 C rounded up to a multiple of 16");
  XDNA_CHECK_ARG(N <= 65535 && (H + 2) * (W + 2) < (1ll << 31), "conv_quant_taps: too large");
  if (N == 0) return XDNA_OK;
  XDNA_CHECK_ARG(x && xp && sx && amax_scratch, "conv_quant_taps: null pointer");
  XDNA_CHECK_ARG(aligned16(xp), "conv_quant_taps: xp must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  XDNA_CUDA(cudaMemsetAsync(amax_scratch, 0, N * sizeof(uint32_t), s));
  const int64_t per_image = C * H * W;
  const int chunks = static_cast<int>(std::min<int64_t>((per_image + 256 * 16 - 1) / (256 * 16), 1024));
  dim3 g_amax(chunks, static_cast<unsigned>(N));
  dim3 g(static_cast<unsigned>(((H + 2) * (W + 2) + 255) / 256), static_cast<unsigned>(N));
  const int c = static_cast<int>(C), h = static_cast<int>(H), w = static_cast<int>(W), kp = static_cast<int>(Kp);
  (void)kp;
  switch (x_dtype) {
    case XDNA_F32:
      image_amax_kernel<float><<<g_amax, 256, 0, s>>>(static_cast<const float*>(x), per_image, amax_scratch);
      launch_taps<float>(static_cast<const float*>(x), c, h, w, g, amax_scratch, xp, sx, s);
      break;
    case XDNA_BF16:
      image_amax_kernel<__nv_bfloat16>
          <<<g_amax, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), per_image, amax_scratch);
      launch_taps<__nv_bfloat16>(static_cast<const __nv_bfloat16*>(x), c, h, w, g, amax_scratch, xp, sx, s);
      break;
    case XDNA_F16:
      image_amax_kernel<__half><<<g_amax, 256, 0, s>>>(static_cast<const __half*>(x), per_image, amax_scratch);
      launch_taps<__half>(static_cast<const __half*>(x), c, h, w, g, amax_scratch, xp, sx, s);
      break;
    default:
      return fail(XDNA_ERR_INVALID, "conv_quant_taps: x_dtype %d is not f32/bf16/f16", x_dtype);
  }
  return check_launch("conv quantise (taps packed)");
}

int xdna_conv_quant_codes(const void* q, int q_unsigned, int64_t N, int64_t C, int64_t H, int64_t W,
                          const float* scale, const float* sx_in, const float* bias, int relu_after, int pool,
                          int8_t* xp, int64_t Cp, float* sx_out, uint32_t* amax_scratch, void* stream) {
  int rc = check_device(nullptr);
  if (rc != XDNA_OK) return rc;
  XDNA_CHECK_ARG(N >= 0 && C >= 4 && C % 4 == 0 && H >= 1 && W >= 1,
                 "conv_quant_codes: bad shape (C must be a positive multiple of 4)");
  XDNA_CHECK_ARG(!pool || (H >= 2 && W >= 2), "conv_quant_codes: a 2x2 pool needs H, W >= 2");
  XDNA_CHECK_ARG(Cp >= C && Cp % 16 == 0, "conv_quant_codes: Cp must be >= C and a multiple of 16");
  XDNA_CHECK_ARG(N <= 65535 && H + 2 <= 65535 && N * H * W * C < (1ll << 40), "conv_quant_codes: too large");
  if (N == 0) return XDNA_OK;
  XDNA_CHECK_ARG(q && scale && sx_in && xp && sx_out && amax_scratch, "conv_quant_codes: null pointer");
  XDNA_CHECK_ARG(reinterpret_cast<uintptr_t>(q) % 4 == 0 && aligned16(xp), "conv_quant_codes: q must be 4-byte and "
                 "xp 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  XDNA_CUDA(cudaMemsetAsync(amax_scratch, 0, N * sizeof(uint32_t), s));
  const uint32_t* qw = static_cast<const uint32_t*>(q);
  const int n = static_cast<int>(N), h = static_cast<int>(H), w = static_cast<int>(W), c4 = static_cast<int>(C / 4);
  const int cp = static_cast<int>(Cp), ra = relu_after ? 1 : 0;
  if (pool) {
    if (q_unsigned)
      launch_codes<true, true>(qw, n, h, w, c4, scale, sx_in, bias, ra, cp, amax_scratch, xp, sx_out, s);
    else
      launch_codes<true, false>(qw, n, h, w, c4, scale, sx_in, bias, ra, cp, amax_scratch, xp, sx_out, s);
  } else {
    if (q_unsigned)
      launch_codes<false, true>(qw, n, h, w, c4, scale, sx_in, bias, ra, cp, amax_scratch, xp, sx_out, s);
    else
      launch_codes<false, false>(qw, n, h, w, c4, scale, sx_in, bias, ra, cp, amax_scratch, xp, sx_out, s);
  }
  return check_launch("conv quantise (int8 codes)");
}

int xdna_conv_quant_codes_given_amax(const void* q, int q_unsigned, int64_t N, int64_t C, int64_t H, int64_t W,
                                     const float* scale, const float* sx_in, const float* bias, int relu_after,
                                     int pool, int8_t* xp, int64_t Cp, float* sx_out, const uint32_t* amax,
                                     void* stream) {
  int rc = check_device(nullptr);
  if (rc != XDNA_OK) return rc;
  XDNA_CHECK_ARG(N >= 0 && C >= 4 && C % 4 == 0 && H >= 1 && W >= 1,
                 "conv_quant_codes_given_amax: bad shape (C must be a positive multiple of 4)");
  XDNA_CHECK_ARG(!pool || (H >= 2 && W >= 2), "conv_quant_codes_given_amax: a 2x2 pool needs H, W >= 2");
  XDNA_CHECK_ARG(Cp >= C && Cp % 16 == 0, "conv_quant_codes_given_amax: Cp must be >= C and a multiple of 16");
  XDNA_CHECK_ARG(N <= 65535 && H + 2 <= 65535 && N * H * W * C < (1ll << 40), "conv_quant_codes_given_amax: too large");
  if (N == 0) return XDNA_OK;
  XDNA_CHECK_ARG(q && scale && sx_in && xp && sx_out && amax, "conv_quant_codes_given_amax: null pointer");
  XDNA_CHECK_ARG(reinterpret_cast<uintptr_t>(q) % 4 == 0 && aligned16(xp),
                 "conv_quant_codes_given_amax: q must be 4-byte and xp 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint32_t* qw = static_cast<const uint32_t*>(q);
  uint32_t* am = const_cast<uint32_t*>(amax);  // only read: the max pass is skipped
  const int n = static_cast<int>(N), h = static_cast<int>(H), w = static_cast<int>(W), c4 = static_cast<int>(C / 4);
  const int cp = static_cast<int>(Cp), ra = relu_after ? 1 : 0;
  if (pool) {
    if (q_unsigned)
      launch_codes<true, true>(qw, n, h, w, c4, scale, sx_in, bias, ra, cp, am, xp, sx_out, s, true);
    else
      launch_codes<true, false>(qw, n, h, w, c4, scale, sx_in, bias, ra, cp, am, xp, sx_out, s, true);
  } else {
    if (q_unsigned)
      launch_codes<false, true>(qw, n, h, w, c4, scale, sx_in, bias, ra, cp, am, xp, sx_out, s, true);
    else
      launch_codes<false, false>(qw, n, h, w, c4, scale, sx_in, bias, ra, cp, am, xp, sx_out, s, true);
  }
  return check_launch("conv quantise (int8 codes, given maxima)");
}

int xdna_conv_bias_int32(const void* bias, int bias_dtype, const float* sw, const float* sx, int64_t N, int64_t Co,
                         int32_t* out, void* stream) {
  int rc = check_device(nullptr);
  if (rc != XDNA_OK) return rc;
  XDNA_CHECK_ARG(N >= 0 && Co >= 1 && N * Co < (1ll << 31), "conv_bias_int32: bad shape");
  if (N == 0) return XDNA_OK;
  XDNA_CHECK_ARG(bias && sw && sx && out, "conv_bias_int32: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int n = static_cast<int>(N), co = static_cast<int>(Co);
  const int blocks = static_cast<int>(std::min<int64_t>((N * Co + 255) / 256, 1024));
  switch (bias_dtype) {
    case XDNA_F32:
      bias_int32_kernel<float><<<blocks, 256, 0, s>>>(static_cast<const float*>(bias), sw, sx, n, co, out);
      break;
    case XDNA_BF16:
      bias_int32_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(bias), sw, sx, n, co, out);
      break;
    case XDNA_F16:
      bias_int32_kernel<__half><<<blocks, 256, 0, s>>>(static_cast<const __half*>(bias), sw, sx, n, co, out);
      break;
    default:
      return fail(XDNA_ERR_INVALID, "conv_bias_int32: bias_dtype %d is not f32/bf16/f16", bias_dtype);
  }
  return check_launch("conv bias to int32");
}

int xdna_conv_quant_codes_pairs(const void* q, int q_unsigned, int64_t N, int64_t C, int64_t H, int64_t W,
                                const float* scale, const float* sx_in, const float* bias, int relu_after, int pool,
                                int8_t* xp, float* sx_out, uint32_t* amax, int amax_given, void* stream) {
  int rc = check_device(nullptr);
  if (rc != XDNA_OK) return rc;
  XDNA_CHECK_ARG(N >= 0 && N % 2 == 0 && C == 64 && H >= 1 && W >= 1,
                 "conv_quant_codes_pairs: bad shape (64 channels, an even number of images)");
  XDNA_CHECK_ARG(!pool || (H >= 2 && W >= 2), "conv_quant_codes_pairs: a 2x2 pool needs H, W >= 2");
  XDNA_CHECK_ARG(N <= 65535 && H + 2 <= 65535 && N * H * W * C < (1ll << 40), "conv_quant_codes_pairs: too large");
  if (N == 0) return XDNA_OK;
  XDNA_CHECK_ARG(q && scale && sx_in && xp && sx_out && amax, "conv_quant_codes_pairs: null pointer");
  XDNA_CHECK_ARG(aligned16(q) && aligned16(xp), "conv_quant_codes_pairs: q and xp must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint32_t* qw = static_cast<const uint32_t*>(q);
  const int n = static_cast<int>(N), h = static_cast<int>(H), w = static_cast<int>(W), c4 = 16;
  const int ra = relu_after ? 1 : 0;
  const bool given = amax_given != 0;
  if (!given) XDNA_CUDA(cudaMemsetAsync(amax, 0, N * sizeof(uint32_t), s));
  if (pool) {
    if (q_unsigned)
      launch_codes<true, true>(qw, n, h, w, c4, scale, sx_in, bias, ra, 64, amax, xp, sx_out, s, given, true);
    else
      launch_codes<true, false>(qw, n, h, w, c4, scale, sx_in, bias, ra, 64, amax, xp, sx_out, s, given, true);
  } else {
    if (q_unsigned)
      launch_codes<false, true>(qw, n, h, w, c4, scale, sx_in, bias, ra, 64, amax, xp, sx_out, s, given, true);
    else
      launch_codes<false, false>(qw, n, h, w, c4, scale, sx_in, bias, ra, 64, amax, xp, sx_out, s, given, true);
  }
  return check_launch("conv quantise (int8 codes, image pairs)");
}

int xdna_conv_quant_channels_last(const void* x, int x_dtype, int64_t N, int64_t C, int64_t H, int64_t W,
                                  int8_t* xp, int64_t Cp, float* sx, uint32_t* amax_scratch, void* stream) {
  int rc = check_device(nullptr);
  if (rc != XDNA_OK) return rc;
  XDNA_CHECK_ARG(N >= 0 && C >= 1 && H >= 1 && W >= 1, "conv_quant_cl: bad shape");
  XDNA_CHECK_ARG(Cp >= C && Cp % 16 == 0, "conv_quant_cl: Cp must be >= C and a multiple of 16");
  XDNA_CHECK_ARG(H + 2 <= 2147483647 && N <= 65535, "conv_quant_cl: too many images");
  if (N == 0) return XDNA_OK;
  XDNA_CHECK_ARG(x && xp && sx && amax_scratch, "conv_quant_cl: null pointer");
  XDNA_CHECK_ARG(aligned16(x) && aligned16(xp), "conv_quant_cl: x and xp must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  XDNA_CUDA(cudaMemsetAsync(amax_scratch, 0, N * sizeof(uint32_t), s));
  const int64_t per_image = C * H * W;
  const int chunks = static_cast<int>(std::min<int64_t>((per_image + 256 * 16 - 1) / (256 * 16), 1024));
  dim3 g_amax(chunks, static_cast<unsigned>(N));
  dim3 g(static_cast<unsigned>(H + 2), static_cast<unsigned>(N));
  switch (x_dtype) {
    case XDNA_F32:
      image_amax_kernel<float><<<g_amax, 256, 0, s>>>(static_cast<const float*>(x), per_image, amax_scratch);
      cl_to_bordered_kernel<float><<<g, 256, 0, s>>>(static_cast<const float*>(x), (int)C, (int)H, (int)W, (int)Cp,
                                                     amax_scratch, xp, sx);
      break;
    case XDNA_BF16:
      image_amax_kernel<__nv_bfloat16>
          <<<g_amax, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), per_image, amax_scratch);
      cl_to_bordered_kernel<__nv_bfloat16><<<g, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), (int)C, (int)H,
                                                             (int)W, (int)Cp, amax_scratch, xp, sx);
      break;
    case XDNA_F16:
      image_amax_kernel<__half><<<g_amax, 256, 0, s>>>(static_cast<const __half*>(x), per_image, amax_scratch);
      cl_to_bordered_kernel<__half><<<g, 256, 0, s>>>(static_cast<const __half*>(x), (int)C, (int)H, (int)W, (int)Cp,
                                                      amax_scratch, xp, sx);
      break;
    default:
      return fail(XDNA_ERR_INVALID, "conv_quant_cl: x_dtype %d is not f32/bf16/f16", x_dtype);
  }
  return check_launch("conv quantise (channels-last)");
}

int xdna_conv_image_amax(const void* x, int x_dtype, int64_t N, int64_t per_image, uint32_t* amax, void* stream) {
  int rc = check_device(nullptr);
  if (rc != XDNA_OK) return rc;
  XDNA_CHECK_ARG(N >= 0 && N <= 65535 && per_image >= 1, "conv_image_amax: bad shape");
  if (N == 0) return XDNA_OK;
  XDNA_CHECK_ARG(x && amax, "conv_image_amax: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  XDNA_CUDA(cudaMemsetAsync(amax, 0, N * sizeof(uint32_t), s));
  const int chunks = static_cast<int>(std::min<int64_t>((per_image + 256 * 16 - 1) / (256 * 16), 1024));
  const dim3 g(chunks, static_cast<unsigned>(N));
  switch (x_dtype) {
    case XDNA_F32:
      image_amax_kernel<float><<<g, 256, 0, s>>>(static_cast<const float*>(x), per_image, amax);
      break;
    case XDNA_BF16:
      image_amax_kernel<__nv_bfloat16><<<g, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), per_image, amax);
      break;
    case XDNA_F16:
      image_amax_kernel<__half><<<g, 256, 0, s>>>(static_cast<const __half*>(x), per_image, amax);
      break;
    default:
      return fail(XDNA_ERR_INVALID, "conv_image_amax: x_dtype %d is not f32/bf16/f16", x_dtype);
  }
  return check_launch("image_amax_kernel");
}

int xdna_conv_quant_given_amax(const void* x, int x_dtype, int x_channels_last, int64_t N, int64_t C, int64_t H,
                               int64_t W, int8_t* xp, int64_t Cp, float* sx, const uint32_t* amax, void* stream) {
  int rc = check_device(nullptr);
  if (rc != XDNA_OK) return rc;
  XDNA_CHECK_ARG(N >= 0 && C >= 1 && H >= 1 && W >= 1, "conv_quant_given_amax: bad shape");
  XDNA_CHECK_ARG(Cp >= C && Cp % 16 == 0, "conv_quant_given_amax: Cp must be >= C and a multiple of 16");
  XDNA_CHECK_ARG(H + 2 <= 65535 && N * ((Cp + 63) / 64) <= 65535, "conv_quant_given_amax: too large");
  if (N == 0) return XDNA_OK;
  XDNA_CHECK_ARG(x && xp && sx && amax, "conv_quant_given_amax: null pointer");
  const bool cl = x_channels_last != 0;
  if (cl) XDNA_CHECK_ARG(aligned16(x) && aligned16(xp), "conv_quant_given_amax: x and xp must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int cgroups = static_cast<int>((Cp + 63) / 64);
  const dim3 g_tr(static_cast<unsigned>((W + 2 + 31) / 32), static_cast<unsigned>(H + 2),
                  static_cast<unsigned>(N * cgroups));
  const dim3 g_cl(static_cast<unsigned>(H + 2), static_cast<unsigned>(N));
  switch (x_dtype) {
    case XDNA_F32:
      if (cl)
        cl_to_bordered_kernel<float><<<g_cl, 256, 0, s>>>(static_cast<const float*>(x), (int)C, (int)H, (int)W,
                                                          (int)Cp, amax, xp, sx);
      else
        to_bordered_nhwc_kernel<float, true><<<g_tr, 256, 0, s>>>(static_cast<const float*>(x), (int)C, (int)H,
                                                                  (int)W, (int)Cp, cgroups, amax, xp, sx);
      break;
    case XDNA_BF16:
      if (cl)
        cl_to_bordered_kernel<__nv_bfloat16><<<g_cl, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), (int)C,
                                                                  (int)H, (int)W, (int)Cp, amax, xp, sx);
      else
        to_bordered_nhwc_kernel<__nv_bfloat16, true><<<g_tr, 256, 0, s>>>(
            static_cast<const __nv_bfloat16*>(x), (int)C, (int)H, (int)W, (int)Cp, cgroups, amax, xp, sx);
      break;
    case XDNA_F16:
      if (cl)
        cl_to_bordered_kernel<__half><<<g_cl, 256, 0, s>>>(static_cast<const __half*>(x), (int)C, (int)H, (int)W,
                                                           (int)Cp, amax, xp, sx);
      else
        to_bordered_nhwc_kernel<__half, true><<<g_tr, 256, 0, s>>>(static_cast<const __half*>(x), (int)C, (int)H,
                                                                   (int)W, (int)Cp, cgroups, amax, xp, sx);
      break;
    default:
      return fail(XDNA_ERR_INVALID, "conv_quant_given_amax: x_dtype %d is not f32/bf16/f16", x_dtype);
  }
  return check_launch("conv quantise (given maxima)");
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

// ---------------------------------------------------------------------------- no-allocation variant
// xdna_conv_quant_nhwc needs N words of scratch (the per-image max) that its caller allocates. Some
// callers cannot allocate: a host framework that hands a plugin all of its device memory when the
// plugin is loaded and forbids allocation while requests are served, or a serving loop that must not
// call cudaMalloc because it may synchronise the whole device and stall every other stream. For them
// this variant keeps its scratch in the file-scope array below, which every GPU that loads the library
// holds until the process exits.
namespace xdna {

constexpr int64_t kStaticScratchImages = 4096;  // 16 KB per device
static __device__ __align__(256) uint32_t g_conv_amax_scratch[kStaticScratchImages];

constexpr int kMaxStaticDevices = 64;
// its device address, per device (published with release order once looked up)
static std::atomic<uint32_t*> g_conv_amax_scratch_ptr[kMaxStaticDevices];
static std::mutex g_conv_amax_scratch_mutex;

// The device address of g_conv_amax_scratch on the current device. In host code the array's name is
// only a host-side stand-in, never a device address, so it is looked up once per device (with that
// device current) and cached. The cached address belongs to the device's primary context: the library
// must not be used across a cudaDeviceReset of that device.
static int conv_amax_scratch(uint32_t** out) {
  int dev = 0;
  XDNA_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxStaticDevices) return fail(XDNA_ERR_DEVICE, "device ordinal %d out of range", dev);
  uint32_t* ptr = g_conv_amax_scratch_ptr[dev].load(std::memory_order_acquire);
  if (ptr == nullptr) {
    std::lock_guard<std::mutex> lock(g_conv_amax_scratch_mutex);
    ptr = g_conv_amax_scratch_ptr[dev].load(std::memory_order_relaxed);
    if (ptr == nullptr) {
      void* p = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&p, g_conv_amax_scratch);
      if (e != cudaSuccess)
        return fail(XDNA_ERR_CUDA, "conv_quant_static: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      ptr = static_cast<uint32_t*>(p);
      g_conv_amax_scratch_ptr[dev].store(ptr, std::memory_order_release);
    }
  }
  *out = ptr;
  return XDNA_OK;
}

}  // namespace xdna

extern "C" int xdna_conv_quant_nhwc_static(const void* x, int x_dtype, int64_t N, int64_t C, int64_t H, int64_t W,
                                           int8_t* xp, int64_t Cp, float* sx, void* stream) {
  int rc = check_device(nullptr);
  if (rc != XDNA_OK) return rc;
  if (N > kStaticScratchImages)
    return fail(XDNA_ERR_INVALID, "conv_quant_static: %lld images; the static scratch holds at most %lld",
                static_cast<long long>(N), static_cast<long long>(kStaticScratchImages));
  uint32_t* scratch = nullptr;
  rc = conv_amax_scratch(&scratch);
  if (rc != XDNA_OK) return rc;
  // the allocating entry point clears the N words it uses before the max kernel runs
  return xdna_conv_quant_nhwc(x, x_dtype, N, C, H, W, xp, Cp, sx, scratch, stream);
}
