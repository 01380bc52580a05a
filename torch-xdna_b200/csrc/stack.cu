// The Qwen3-0.6B stack on the B200: RMSNorm and embedding-gather kernels, the bf16 tcgen05 GEMM
// launcher (umma_gemm.cuh in kind::f16 mode with the stack epilogues), the attention launcher
// (attention.cu) and xdna_qwen3_stack, the native driver that runs every layer, the final norm and the
// head on one stream with no host synchronisation.
//
// Per layer (R:torch_xdna/stack.py:43-57 shapes; transformers' Qwen3 decoder layer math):
//   h    = bf16(rmsnorm(x) * input_norm)                  rmsnorm_kernel           (HBM)
//   q,k  = rope(rmsnorm_head(h Wq^T | h Wk^T) * q/k_norm)  GEMM, EPI_QKV             (tensor)
//   v^T  = (h Wv^T)^T                                       (same GEMM)
//   o    = softmax(q k^T / sqrt(128) + mask) v              attention_kernel          (tensor)
//   x   += o Wo^T                                           GEMM, EPI_RESID          (tensor)
//   h    = bf16(rmsnorm(x) * post_norm)                     rmsnorm_kernel
//   a    = silu(h Wgate^T) * (h Wup^T)                      GEMM, EPI_SWIGLU         (tensor)
//   x   += a Wdown^T                                        GEMM, EPI_RESID
// then h = bf16(rmsnorm(x) * final_norm) and out = h Whead^T (+ bias) (GEMM, EPI_F32ACC).
// The residual stream x stays f32 for the whole stack.
#include <algorithm>
#include <vector>

#include "host_util.h"
#include "umma_gemm.cuh"
#include "xdna_b200.h"

namespace xdna {

// ---------------------------------------------------------------------------- RMSNorm
// One warp per row of D = 32 * 4 * NV floats: y = bf16(x * rsqrt(mean(x^2) + eps) * w).
template <int NV>
__global__ void __launch_bounds__(256) rmsnorm_kernel(const float* __restrict__ x, int64_t rows, int D,
                                                      const float* __restrict__ w, float eps,
                                                      __nv_bfloat16* __restrict__ y) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int lane = threadIdx.x & 31;
  const float4* xr = reinterpret_cast<const float4*>(x + row * D);
  float4 v[NV];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    v[i] = xr[i * 32 + lane];
    ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float rstd = rsqrtf(ss / static_cast<float>(D) + eps);
  const float4* wr = reinterpret_cast<const float4*>(w);
  uint2* yr = reinterpret_cast<uint2*>(y + row * D);
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const float4 g = wr[i * 32 + lane];
    const __nv_bfloat162 a = __floats2bfloat162_rn(v[i].x * rstd * g.x, v[i].y * rstd * g.y);
    const __nv_bfloat162 b = __floats2bfloat162_rn(v[i].z * rstd * g.z, v[i].w * rstd * g.w);
    yr[i * 32 + lane] = make_uint2(*reinterpret_cast<const uint32_t*>(&a), *reinterpret_cast<const uint32_t*>(&b));
  }
}

// ---------------------------------------------------------------------------- embedding gather
// x[t, :] = float(table[ids[t], :]) for a bf16 or f32 table; one warp per token (HBM-bound).
template <typename T>
__global__ void __launch_bounds__(256) embed_kernel(const int64_t* __restrict__ ids, int64_t tokens, int D,
                                                    const T* __restrict__ table, int64_t vocab,
                                                    float* __restrict__ x, int* err) {
  const int64_t t = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (t >= tokens) return;
  const int lane = threadIdx.x & 31;
  const int64_t id = ids[t];
  float* xr = x + t * D;
  if (id < 0 || id >= vocab) {  // out-of-range id: zeros, and an error the host can read
    if (lane == 0 && err != nullptr) atomicCAS(err, 0, XDNA_ERR_INVALID);
    for (int d = lane; d < D; d += 32) xr[d] = 0.f;
    return;
  }
  const T* src = table + id * D;
  for (int d = lane; d < D; d += 32) {
    if constexpr (sizeof(T) == 2)
      xr[d] = __bfloat162float(src[d]);
    else
      xr[d] = src[d];
  }
}

// ---------------------------------------------------------------------------- bf16 GEMM launch
template <int BN, int EPI, int ODT>
static int launch_bf16(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const GemmArgs& a,
                       int sms, bool pair, cudaStream_t stream, const CUtensorMap* td = nullptr) {
  constexpr bool TSTORE = (EPI == EPI_F32ACC || EPI == EPI_QKV || EPI == EPI_SWIGLU || EPI == EPI_RESID);
  if constexpr (BN == 256) {
    if (pair)
      return launch_gemm_kernel<BN, LOAD_GEMM, EPI, true, TSTORE, ODT, kBKBytes, true>(ta, tb, tc, td ? *td : ta, a, sms,
                                                                                       stream);
  }
  return launch_gemm_kernel<BN, LOAD_GEMM, EPI, true, TSTORE, ODT, kBKBytes, false>(ta, tb, tc, td ? *td : ta, a, sms,
                                                                                    stream);
}

static int bf16_map(CUtensorMap* m, const void* p, int64_t rows, int64_t cols, int64_t ld, uint32_t box_rows,
                    const char* what) {
  const uint64_t dims[2] = {static_cast<uint64_t>(cols), static_cast<uint64_t>(rows)};
  const uint64_t strides[1] = {static_cast<uint64_t>(ld * 2)};
  const uint32_t box[2] = {64, box_rows};
  return encode_tma(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p, dims, strides, box, what);
}

static int out_map(CUtensorMap* m, const void* p, int64_t rows, int64_t cols, int64_t ld, int dtype,
                   const char* what, bool wide = false) {
  const int es = dtype_size(dtype);
  const uint64_t dims[2] = {static_cast<uint64_t>(cols), static_cast<uint64_t>(rows)};
  const uint64_t strides[1] = {static_cast<uint64_t>(ld * es)};
  // 32 rows x 64 bytes (the epilogue's staging blocks), or 32 x 128 bytes for stage_wide's blocks
  const uint32_t box[2] = {static_cast<uint32_t>((wide ? 128 : 64) / es), 32};
  const CUtensorMapDataType dt = dtype == XDNA_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : dtype == XDNA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                      : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return encode_tma(m, dt, 2, p, dims, strides, box, what, wide ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
}

// C[M, N] = A[M, K] . B[N, K]^T (bf16, f32 accumulate) with one of the stack epilogues.
struct Bf16Gemm {
  const void* a;  // (with a_maps: the first row block, used only to type the unused tmA)
  int64_t lda;
  const void* b;
  int64_t ldb;
  int64_t M, N, K;
  int mode;  // XDNA_GEMM_*
  void* out;
  int out_dtype;
  int64_t ldo;
  const void* bias;
  int bias_dtype;
  float* resid;
  int64_t ldr;
  __nv_bfloat16* vt;
  int64_t ldvt;
  const float *rope_cos, *rope_sin, *q_norm, *k_norm;
  int seq_len;
  float eps;
  const CUtensorMap* a_maps = nullptr;  // A split by rows over several buffers (xdna_gemm_bf16_gather)
  int a_rows = 0;
};

static int run_bf16_gemm(const Bf16Gemm& g, cudaStream_t s) {
  int sms = 0;
  int rc = check_device(&sms);
  if (rc != XDNA_OK) return rc;
  XDNA_CHECK_ARG(g.M >= 0 && g.N > 0 && g.K > 0 && g.M < (1ll << 31) && g.N < (1ll << 31), "gemm_bf16: bad sizes");
  if (g.M == 0) return XDNA_OK;
  XDNA_CHECK_ARG(g.a && g.b, "gemm_bf16: null operand");
  XDNA_CHECK_ARG(g.lda % 8 == 0 && g.ldb % 8 == 0 && g.lda >= g.K && g.ldb >= g.K,
                 "gemm_bf16: operand row pitch must cover K and be a multiple of 8 elements");
  GemmArgs a{};
  a.M = static_cast<int>(g.M);
  a.N = static_cast<int>(g.N);
  a.num_kb = static_cast<int>((g.K + 63) / 64);
  a.m_tiles = static_cast<int>((g.M + kBM - 1) / kBM);
  // 256-column tiles, or 128 when 256 would leave SMs idle (F32ACC / RESID; the fused q/k/v and SwiGLU
  // epilogues need the 256-column tile)
  int bn = 256;
  if ((g.mode == XDNA_GEMM_F32ACC || g.mode == XDNA_GEMM_RESID) &&
      (g.N <= 128 || a.m_tiles * ((g.N + 255) / 256) < sms))
    bn = 128;
  a.n_tiles = static_cast<int>((g.N + bn - 1) / bn);
  const bool pair = use_pairs(bn, a.m_tiles, a.n_tiles, sms);
  if (pair) a.m_tiles = static_cast<int>((g.M + 2 * kBM - 1) / (2 * kBM));
  a.out = g.out;
  a.ldo = g.ldo;
  a.out_dtype = g.out_dtype;
  a.bias = g.bias;
  a.bias_dtype = g.bias_dtype;
  a.resid = g.resid;
  a.ldr = g.ldr;
  a.vt = g.vt;
  a.ldvt = g.ldvt;
  a.rope_cos = g.rope_cos;
  a.rope_sin = g.rope_sin;
  a.q_norm = g.q_norm;
  a.k_norm = g.k_norm;
  a.seq_len = g.seq_len;
  a.eps = g.eps;
  a.err = device_error_word();
  a.a_maps = g.a_maps;
  a.a_rows = g.a_rows;
  CUtensorMap ta, tb, tc;
  if ((rc = bf16_map(&ta, g.a, g.a_maps ? g.a_rows : g.M, g.K, g.lda, kBM, "gemm_bf16 A")) != XDNA_OK) return rc;
  if ((rc = bf16_map(&tb, g.b, g.N, g.K, g.ldb, static_cast<uint32_t>(pair ? bn / 2 : bn), "gemm_bf16 B")) != XDNA_OK)
    return rc;
  switch (g.mode) {
    case XDNA_GEMM_F32ACC: {
      XDNA_CHECK_ARG(g.out && is_float_dtype(g.out_dtype) && g.ldo >= g.N, "gemm_bf16: bad output");
      XDNA_CHECK_ARG(g.bias == nullptr || is_float_dtype(g.bias_dtype), "gemm_bf16: bad bias dtype");
      a.vec_ok = aligned16(g.out) && (g.ldo * dtype_size(g.out_dtype)) % 16 == 0;
      XDNA_CHECK_ARG(a.vec_ok, "gemm_bf16: output rows must be 16-byte aligned (base and row pitch)");
      if ((rc = out_map(&tc, g.out, g.M, g.N, g.ldo, g.out_dtype, "gemm_bf16 out",
                        wide_store_map(EPI_F32ACC, pair && bn == 256, dtype_size(g.out_dtype)))) != XDNA_OK)
        return rc;
      if (g.out_dtype == XDNA_F32)
        return bn == 256 ? launch_bf16<256, EPI_F32ACC, XDNA_F32>(ta, tb, tc, a, sms, pair, s)
                         : launch_bf16<128, EPI_F32ACC, XDNA_F32>(ta, tb, tc, a, sms, pair, s);
      if (g.out_dtype == XDNA_BF16)
        return bn == 256 ? launch_bf16<256, EPI_F32ACC, XDNA_BF16>(ta, tb, tc, a, sms, pair, s)
                         : launch_bf16<128, EPI_F32ACC, XDNA_BF16>(ta, tb, tc, a, sms, pair, s);
      return bn == 256 ? launch_bf16<256, EPI_F32ACC, XDNA_F16>(ta, tb, tc, a, sms, pair, s)
                       : launch_bf16<128, EPI_F32ACC, XDNA_F16>(ta, tb, tc, a, sms, pair, s);
    }
    case XDNA_GEMM_RESID:
      XDNA_CHECK_ARG(g.resid && g.ldr >= g.N && g.ldr % 4 == 0 && aligned16(g.resid), "gemm_bf16: bad residual");
      if ((rc = out_map(&tc, g.resid, g.M, g.N, g.ldr, XDNA_F32, "gemm_bf16 residual")) != XDNA_OK) return rc;
      return bn == 256 ? launch_bf16<256, EPI_RESID, XDNA_F32>(ta, tb, tc, a, sms, pair, s)
                       : launch_bf16<128, EPI_RESID, XDNA_F32>(ta, tb, tc, a, sms, pair, s);
    case XDNA_GEMM_SWIGLU:
      XDNA_CHECK_ARG(g.N % 64 == 0 && g.out && g.ldo >= g.N / 2, "gemm_bf16: swiglu needs N % 64 == 0 and an output");
      if ((rc = out_map(&tc, g.out, g.M, g.N / 2, g.ldo, XDNA_BF16, "gemm_bf16 swiglu out")) != XDNA_OK) return rc;
      return launch_bf16<256, EPI_SWIGLU, XDNA_BF16>(ta, tb, tc, a, sms, pair, s);
    case XDNA_GEMM_QKV:
      XDNA_CHECK_ARG(g.N == kQCols + 2 * kKCols && g.out && g.vt && g.rope_cos && g.rope_sin && g.q_norm && g.k_norm &&
                         g.seq_len > 0 && g.ldvt % 8 == 0 &&
                         g.ldvt >= (g.M + g.seq_len - 1) / g.seq_len * ((g.seq_len + 7) / 8 * 8),
                     "gemm_bf16: qkv needs N = 4096, q/k output, V^T (pitch >= sequences x round_up(L, 8)), "
                     "rope tables and norms");
      if ((rc = out_map(&tc, g.out, g.M, kQCols + kKCols, g.ldo, XDNA_BF16, "gemm_bf16 qk out")) != XDNA_OK) return rc;
      {
        // V^T written by TMA (32 tokens x 32 dims per store) when every 32-row block lies in one sequence
        CUtensorMap td = ta;
        a.vt_tma = g.seq_len % 32 == 0 && aligned16(g.vt);
        if (a.vt_tma) {
          const uint64_t dims[2] = {static_cast<uint64_t>(g.ldvt), 1024};
          const uint64_t strides[1] = {static_cast<uint64_t>(g.ldvt * 2)};
          const uint32_t box[2] = {32, 32};
          if ((rc = encode_tma(&td, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, g.vt, dims, strides, box, "gemm_bf16 v^T",
                               CU_TENSOR_MAP_SWIZZLE_NONE)) != XDNA_OK)
            return rc;
        }
        return launch_bf16<256, EPI_QKV, XDNA_BF16>(ta, tb, tc, a, sms, pair, s, &td);
      }
    default:
      return fail(XDNA_ERR_INVALID, "gemm_bf16: unknown mode %d", g.mode);
  }
}

}  // namespace xdna

// attention (attention.cu)
namespace xdna {
int run_attention(const __nv_bfloat16* qk, const __nv_bfloat16* vt, int64_t ldvt, __nv_bfloat16* out, int64_t B,
                  int64_t L, int mask_kind, const int32_t* lens, const uint8_t* mask, int mask_heads,
                  cudaStream_t stream);
}

using namespace xdna;

extern "C" {

int xdna_rmsnorm_bf16(const float* x, int64_t rows, int64_t D, const float* w, float eps, void* y, void* stream) {
  int rc = check_device(nullptr);
  if (rc != XDNA_OK) return rc;
  XDNA_CHECK_ARG(rows >= 0 && (D == 1024 || D == 512 || D == 128), "rmsnorm: D must be 128, 512 or 1024");
  if (rows == 0) return XDNA_OK;
  XDNA_CHECK_ARG(x && w && y && aligned16(x) && aligned16(w) && aligned16(y), "rmsnorm: null or unaligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const unsigned g = static_cast<unsigned>((rows + 7) / 8);
  auto* yb = static_cast<__nv_bfloat16*>(y);
  if (D == 1024)
    rmsnorm_kernel<8><<<g, 256, 0, s>>>(x, rows, 1024, w, eps, yb);
  else if (D == 512)
    rmsnorm_kernel<4><<<g, 256, 0, s>>>(x, rows, 512, w, eps, yb);
  else
    rmsnorm_kernel<1><<<g, 256, 0, s>>>(x, rows, 128, w, eps, yb);
  return check_launch("rmsnorm_kernel");
}

int xdna_embed(const int64_t* ids, int64_t tokens, const void* table, int table_dtype, int64_t vocab, int64_t D,
               float* x, void* stream) {
  int rc = check_device(nullptr);
  if (rc != XDNA_OK) return rc;
  XDNA_CHECK_ARG(tokens >= 0 && vocab > 0 && D > 0, "embed: bad sizes");
  if (tokens == 0) return XDNA_OK;
  XDNA_CHECK_ARG(ids && table && x, "embed: null pointer");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const unsigned g = static_cast<unsigned>((tokens + 7) / 8);
  if (table_dtype == XDNA_BF16)
    embed_kernel<__nv_bfloat16><<<g, 256, 0, s>>>(ids, tokens, (int)D, static_cast<const __nv_bfloat16*>(table), vocab,
                                                  x, device_error_word());
  else if (table_dtype == XDNA_F32)
    embed_kernel<float><<<g, 256, 0, s>>>(ids, tokens, (int)D, static_cast<const float*>(table), vocab, x,
                                          device_error_word());
  else
    return fail(XDNA_ERR_INVALID, "embed: table dtype %d", table_dtype);
  return check_launch("embed_kernel");
}

int xdna_gemm_bf16(const void* a, int64_t lda, const void* b, int64_t ldb, int64_t M, int64_t N, int64_t K, int mode,
                   void* out, int out_dtype, int64_t ldo, const void* bias, int bias_dtype, float* resid, int64_t ldr,
                   void* vt, int64_t ldvt, const float* rope_cos, const float* rope_sin, const float* q_norm,
                   const float* k_norm, int64_t seq_len, float eps, void* stream) {
  Bf16Gemm g{a, lda, b, ldb, M, N, K, mode, out, out_dtype, ldo, bias, bias_dtype, resid, ldr,
             static_cast<__nv_bfloat16*>(vt), ldvt, rope_cos, rope_sin, q_norm, k_norm, static_cast<int>(seq_len), eps};
  return run_bf16_gemm(g, static_cast<cudaStream_t>(stream));
}

int xdna_gemm_bf16_gather(const void* const* a_parts, int n_parts, int64_t rows_per_part, int64_t lda, const void* b,
                          int64_t ldb, int64_t N, int64_t K, void* out, int out_dtype, int64_t ldo, const void* bias,
                          int bias_dtype, void* maps, void* stream) {
  int rc = check_device(nullptr);
  if (rc != XDNA_OK) return rc;
  XDNA_CHECK_ARG(a_parts != nullptr && n_parts >= 1 && n_parts <= 64, "gemm_bf16_gather: 1..64 parts");
  XDNA_CHECK_ARG(rows_per_part >= kBM && rows_per_part % kBM == 0 && rows_per_part < (1ll << 31) / n_parts,
                 "gemm_bf16_gather: rows per part must be a positive multiple of %d", kBM);
  XDNA_CHECK_ARG(maps != nullptr && reinterpret_cast<uintptr_t>(maps) % 64 == 0,
                 "gemm_bf16_gather: the tensor-map buffer must be 64-byte aligned device memory");
  std::vector<CUtensorMap> host(static_cast<size_t>(n_parts));
  for (int i = 0; i < n_parts; ++i) {
    XDNA_CHECK_ARG(a_parts[i] != nullptr, "gemm_bf16_gather: part %d is null", i);
    if ((rc = bf16_map(&host[i], a_parts[i], rows_per_part, K, lda, kBM, "gemm_bf16_gather part")) != XDNA_OK)
      return rc;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // pageable source: staged before the call returns, ordered on the stream before the GEMM reads it
  XDNA_CUDA(cudaMemcpyAsync(maps, host.data(), host.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice, s));
  Bf16Gemm g{a_parts[0], lda, b, ldb, n_parts * rows_per_part, N, K, XDNA_GEMM_F32ACC, out, out_dtype, ldo, bias,
             bias_dtype, nullptr, 0, nullptr, 0, nullptr, nullptr, nullptr, nullptr, 0, 0.f};
  g.a_maps = static_cast<const CUtensorMap*>(maps);
  g.a_rows = static_cast<int>(rows_per_part);
  return run_bf16_gemm(g, s);
}

int xdna_attention(const void* qk, const void* vt, int64_t ldvt, void* out, int64_t B, int64_t L, int mask_kind,
                   const int32_t* lens, const uint8_t* mask, int mask_heads, void* stream) {
  return run_attention(static_cast<const __nv_bfloat16*>(qk), static_cast<const __nv_bfloat16*>(vt), ldvt,
                       static_cast<__nv_bfloat16*>(out), B, L, mask_kind, lens, mask, mask_heads,
                       static_cast<cudaStream_t>(stream));
}

size_t xdna_qwen3_stack_workspace(int64_t B, int64_t L) {
  const int64_t T = B * L;
  const int64_t T8 = B * ((L + 7) / 8 * 8);  // V^T columns: sequences start at multiples of 8
  auto up = [](int64_t v) { return (v + 255) / 256 * 256; };
  return static_cast<size_t>(up(T * 1024 * 2) + up(T * 3072 * 2) + up(1024 * T8 * 2) + up(T * 2048 * 2) +
                             up(T * 3072 * 2));
}

int xdna_qwen3_stack(const xdna_qwen3_layer* layers, int n_layers, const float* final_norm, const void* head_w,
                     int64_t head_n, const void* head_bias, int head_bias_dtype, const float* rope_cos,
                     const float* rope_sin, float eps, float* x, int64_t B, int64_t L, int mask_kind,
                     const int32_t* lens, const uint8_t* mask, int mask_heads, void* out, int out_dtype, int64_t ldo,
                     void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_device(nullptr);
  if (rc != XDNA_OK) return rc;
  XDNA_CHECK_ARG(layers && n_layers >= 1 && final_norm && head_w && head_n >= 1 && rope_cos && rope_sin && x,
                 "qwen3_stack: missing weights or input");
  XDNA_CHECK_ARG(B >= 1 && L >= 1, "qwen3_stack: bad batch / length");
  XDNA_CHECK_ARG(workspace && workspace_bytes >= xdna_qwen3_stack_workspace(B, L),
                 "qwen3_stack: workspace of %zu bytes, need %zu", workspace_bytes, xdna_qwen3_stack_workspace(B, L));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t T = B * L;
  const int64_t T8 = B * ((L + 7) / 8 * 8);
  auto up = [](int64_t v) { return (v + 255) / 256 * 256; };
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  auto* h = reinterpret_cast<__nv_bfloat16*>(ws);
  ws += up(T * 1024 * 2);
  auto* qk = reinterpret_cast<__nv_bfloat16*>(ws);
  ws += up(T * 3072 * 2);
  auto* vt = reinterpret_cast<__nv_bfloat16*>(ws);
  ws += up(1024 * T8 * 2);
  auto* o = reinterpret_cast<__nv_bfloat16*>(ws);
  ws += up(T * 2048 * 2);
  auto* act = reinterpret_cast<__nv_bfloat16*>(ws);
  // V^T's padding columns (between sequences when L % 8 != 0) are read under the mask: keep them zero
  if (L % 8 != 0) XDNA_CUDA(cudaMemsetAsync(vt, 0, 1024 * T8 * 2, s));

  for (int i = 0; i < n_layers; ++i) {
    const xdna_qwen3_layer& w = layers[i];
    if ((rc = xdna_rmsnorm_bf16(x, T, 1024, w.input_norm, eps, h, stream)) != XDNA_OK) return rc;
    Bf16Gemm qkv{h, 1024, w.w_qkv, 1024, T, 4096, 1024, XDNA_GEMM_QKV, qk, XDNA_BF16, 3072, nullptr, 0, nullptr, 0,
                 vt, T8, rope_cos, rope_sin, w.q_norm, w.k_norm, static_cast<int>(L), eps};
    if ((rc = run_bf16_gemm(qkv, s)) != XDNA_OK) return rc;
    if ((rc = run_attention(qk, vt, T8, o, B, L, mask_kind, lens, mask, mask_heads, s)) != XDNA_OK) return rc;
    Bf16Gemm op{o, 2048, w.w_o, 2048, T, 1024, 2048, XDNA_GEMM_RESID, nullptr, 0, 0, nullptr, 0, x, 1024,
                nullptr, 0, nullptr, nullptr, nullptr, nullptr, 0, eps};
    if ((rc = run_bf16_gemm(op, s)) != XDNA_OK) return rc;
    if ((rc = xdna_rmsnorm_bf16(x, T, 1024, w.post_norm, eps, h, stream)) != XDNA_OK) return rc;
    Bf16Gemm gu{h, 1024, w.w_gu, 1024, T, 6144, 1024, XDNA_GEMM_SWIGLU, act, XDNA_BF16, 3072, nullptr, 0, nullptr, 0,
                nullptr, 0, nullptr, nullptr, nullptr, nullptr, 0, eps};
    if ((rc = run_bf16_gemm(gu, s)) != XDNA_OK) return rc;
    Bf16Gemm dn{act, 3072, w.w_down, 3072, T, 1024, 3072, XDNA_GEMM_RESID, nullptr, 0, 0, nullptr, 0, x, 1024,
                nullptr, 0, nullptr, nullptr, nullptr, nullptr, 0, eps};
    if ((rc = run_bf16_gemm(dn, s)) != XDNA_OK) return rc;
  }
  if ((rc = xdna_rmsnorm_bf16(x, T, 1024, final_norm, eps, h, stream)) != XDNA_OK) return rc;
  if (out == nullptr) return XDNA_OK;  // hidden states only (the head runs elsewhere, e.g. column-parallel)
  Bf16Gemm hd{h, 1024, head_w, 1024, T, head_n, 1024, XDNA_GEMM_F32ACC, out, out_dtype, ldo, head_bias,
              head_bias_dtype, nullptr, 0, nullptr, 0, nullptr, nullptr, nullptr, nullptr, 0, eps};
  return run_bf16_gemm(hd, s);
}

}  // extern "C"
