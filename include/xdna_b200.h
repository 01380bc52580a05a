/* xdna_b200.h -- C ABI of libxdna_b200.so, the B200 (sm_100a) kernels behind torch_xdna's custom ops.
 *
 * Conventions (every entry point):
 *   - returns XDNA_OK (0) or a negative XDNA_ERR_* code; xdna_last_error() then describes the
 *     failure (thread-local, valid until the next call on the same thread);
 *   - every pointer is caller-owned device memory on the current CUDA device, except where a
 *     comment says "host";
 *   - `stream` is a cudaStream_t (NULL = legacy default stream); calls only enqueue work and
 *     never synchronise, except xdna_take_device_error();
 *   - no entry point allocates device memory except xdna_ipc_alloc (the shareable buffer a caller
 *     asks for); scratch is passed in by the caller;
 *   - leading dimensions (`ld*`) are in elements; int8 operands read by TMA need their row
 *     pitch in bytes to be a multiple of 16 and their base 16-byte aligned;
 *   - the library caches, per device, the device addresses of its own globals (the error word,
 *     the no-allocation scratch) on first use: it must not be used on a device after a
 *     cudaDeviceReset of that device (the cached addresses would point into the destroyed
 *     context); load the library again in a new process instead.
 *
 * The reference (AyaSakura-comp/torch-xdna) reaches its device through Python calls into
 * Triton-XDNA; each entry point below names the reference call it replaces.
 */
#ifndef XDNA_B200_H
#define XDNA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status codes */
#define XDNA_OK 0
#define XDNA_ERR_INVALID (-1)     /* bad argument: shape, stride, alignment, dtype, mode */
#define XDNA_ERR_UNSUPPORTED (-2) /* a valid request this build does not implement */
#define XDNA_ERR_CUDA (-3)        /* a CUDA runtime or driver call failed */
#define XDNA_ERR_TIMEOUT (-4)     /* a bounded device-side wait gave up; the kernel returned early */
#define XDNA_ERR_DEVICE (-5)      /* the current device is not an sm_100 (B200-class) GPU */

/* ------------------------------------------------------------------ element types */
#define XDNA_F32 0
#define XDNA_BF16 1
#define XDNA_F16 2
#define XDNA_I32 3
#define XDNA_I8 4
#define XDNA_U8 5

/* ------------------------------------------------------------------ conv3x3 modes */
#define XDNA_CONV_Q 0         /* q = sat((acc + 2^(shift-1)) >> shift) as int8, or uint8 [0,255] with relu, NCHW */
#define XDNA_CONV_DEQUANT 1   /* y = float(q) * (scale[co] * sx[n]) (+ bias[co]) in out_dtype, channels-last
                                 memory [N, H, W, Co] (torch's channels_last layout of an [N, Co, H, W] tensor) */
#define XDNA_CONV_CALIBRATE 2 /* *acc_max = max over the sums of image 0 of (relu ? max(acc,0) : |acc|) */
#define XDNA_CONV_Q_NHWC 3    /* q as XDNA_CONV_Q, written channels-last [N, H, W, Co]: the int8 form in which
                                 one conv's output feeds the next (xdna_conv_quant_codes) */
/* Or'ed into a mode: one tap at offset 0 instead of the 3x3 stencil's nine, i.e. a 1x1 conv over the
 * bordered input with weights wp [Co, 1, Cp]. With the input from xdna_conv_quant_taps (the nine taps of
 * a few channels packed into each pixel's row) and the weights packed the same way, it is the 3x3 conv
 * of a layer with <= 7 input channels in one K block instead of nine. */
#define XDNA_CONV_SINGLE_TAP 16
/* Or'ed into a mode: a stride-2 conv (3x3 with padding 1, or with XDNA_CONV_SINGLE_TAP the 1x1 conv with no
 * padding). xp is then the input split into its stride phases by xdna_conv_quant_phases,
 * [planes, N, Ho+2, Wo+2, Cp] with planes = 4 (3x3) or 1 (1x1), and H, W are the OUTPUT's height and width
 * (Ho = ceil(H_in / 2), Wo = ceil(W_in / 2)). Plane 2 * ry + rx at bordered pixel (Y, X) holds input pixel
 * (2 (Y - 1) + ry, 2 (X - 1) + rx), zero outside the input; tap (ky, kx) of output pixel (y, x) reads plane
 * ((ky != 1), (kx != 1)) at bordered row y + (ky != 0), column x + (kx != 0), so every tap is a constant row
 * offset as in the stride-1 conv. Extends the reference's conv route (which offloads only 3x3 stride-1 convs,
 * R:torch_xdna/backend.py:130-174) to the ResNet-style layers it lists as missing
 * (R:results/conv3x3_cascade.md:222-223): same quantise, calibration and requantise. */
#define XDNA_CONV_STRIDE2 32
/* Or'ed into XDNA_CONV_Q_NHWC: the next layer's per-image maxima, so that its quantise from these codes
 * (xdna_conv_quant_codes_given_amax) needs no pass of its own over them. acc_max then holds N words, cleared by
 * this call, that receive per image the f32 bit pattern of max |y| over the output pixels, where
 * y = float(q) * (scale[c] * sx[n]) (+ bias[c], f32) is computed with the f32 operations of
 * xdna_conv_quant_codes; with XDNA_CONV_NEXT_RELU y is max(y, 0) first; with XDNA_CONV_NEXT_POOL only the
 * rows and columns a 2x2 / stride-2 pool keeps (an odd last one is left out) count, which is the pooled
 * image's max when y >= 0 (so it needs XDNA_CONV_NEXT_RELU, or relu = 1 and no bias). Needs scale, sx
 * (this conv's input scales) and bias (f32 or NULL; with XDNA_CONV_BIAS_INT32 the bias is in the codes and y
 * has no float bias term). */
#define XDNA_CONV_NEXT_AMAX 64
#define XDNA_CONV_NEXT_RELU 128
#define XDNA_CONV_NEXT_POOL 256
/* Or'ed into any conv mode: the bias inside the int32 sums, before the requantise (an option the reference
 * names as future work; its own route adds the bias to the dequantised floats, R:results/conv3x3_cascade.md:224).
 * `bias` is then int32 [N, Co] (bias_dtype XDNA_I32, one row per image: the units of the sums depend on the
 * image's sx), from xdna_conv_bias_int32; the sums become acc + bias[n][co] in every mode (the calibration's
 * max included), and DEQUANT adds no float bias. |acc| must stay below 2^31 - 3 * 2^29 (K * 127^2 < 5.3e8). */
#define XDNA_CONV_BIAS_INT32 512
/* Or'ed into XDNA_CONV_Q_NHWC for a stride-1 3x3 conv with Cp = 64, Co <= 128 and an even N: xp holds the
 * images in pairs, [N/2, H+2, W+2, 128] (bytes 0..63 of a row: image 2i's channels, 64..127: image 2i+1's;
 * xdna_conv_quant_codes_pairs writes it), which halves the TMA row requests of the conv's loads. */
#define XDNA_CONV_PAIRS 1024
/* `relu` of xdna_conv3x3_i8: 0 none; 1 fused into the requantise ([0,255] uint8, the reference's ReLU of
 * a bias-free conv); XDNA_RELU_AFTER_BIAS (DEQUANT only) applied to the dequantised output after the
 * bias, the requantise saturating to int8 — the same values as torch.relu on the DEQUANT output. */
#define XDNA_RELU_AFTER_BIAS 2

/* Last error of this thread, as text. */
const char* xdna_last_error(void);

/* ABI version of this library (bumped when a signature changes). */
int xdna_abi_version(void);

/* XDNA_OK when `device` is an sm_100 GPU this library's kernels run on. */
int xdna_device_check(int device);

/* Reads and clears the device-side error word that bounded waits write (code, site). Synchronises
 * `stream`. *code is XDNA_OK when no kernel recorded an error since the last call. */
int xdna_take_device_error(int* code, int* site, void* stream);

/* Self-test of the bounded device waits (no reference counterpart): launches one block whose wait on an
 * mbarrier that nothing arrives at gives up after limit_ns (1 us .. 2 s) of device time, exactly as the
 * waits inside every kernel of the library do, records XDNA_ERR_TIMEOUT at site 99 in the device error word
 * and returns; xdna_take_device_error then reports it. The GPU context stays usable. */
int xdna_selftest_wait_timeout(uint64_t limit_ns, void* stream);

/* ------------------------------------------------------------------ W8A8 linear
 * Per-row symmetric int8 quantisation: for each row r of x [rows, cols] (leading dim ldx, dtype
 * f32 / bf16 / f16): scale[r] = max(max_c |x[r,c]|, 1e-8) / 127 (the max taken in x's dtype),
 * xq[r,c] = clamp(round_half_even(float(x[r,c]) / scale[r]), -127, 127). IEEE division, no FMA.
 * Replaces R:torch_xdna/runtime.py:145-148 (_quant_rows), the quantise ops of
 * R:torch_xdna/runtime.py:366-368 (linear_int8) and the weight quantisation of QWeight
 * R:torch_xdna/runtime.py:59-66 (a weight is quantised as rows of [N, K]). */
int xdna_quant_rows_i8(const void* x, int x_dtype, int64_t rows, int64_t cols, int64_t ldx, int8_t* xq,
                       int64_t ldq, float* scale, void* stream);

/* acc[M,N] = xq[M,K] . wq[N,K]^T in int32 on the tcgen05 tensor cores (both operands K-major).
 * y_dtype XDNA_I32: y receives acc (sx, sw, bias ignored).
 * y_dtype XDNA_F32 / XDNA_BF16 / XDNA_F16: y = (float(acc) * sx[m]) * sw[n] (+ float(bias[n])),
 *   rounded once to y_dtype (round to nearest even) -- the reference's dequantise order.
 * bias may be NULL; bias_dtype is its element type.
 * Replaces kernels.mm_i8 R:torch_xdna/kernels.py:172-192 as called by _npu_acc
 * R:torch_xdna/runtime.py:191-209 (and the CPU route torch._int_mm, R:torch_xdna/runtime.py:162-163),
 * fused with the dequantisation of R:torch_xdna/runtime.py:350-353, :370-374 and :429-432. */
int xdna_gemm_i8(const int8_t* xq, int64_t ldx, const int8_t* wq, int64_t ldw, int64_t M, int64_t N, int64_t K,
                 const float* sx, const float* sw, const void* bias, int bias_dtype, void* y, int y_dtype,
                 int64_t ldy, void* stream);

/* The kernel configuration xdna_gemm_i8 launches for an M x N output on the current device: *tile_n output
 * columns per tile (64, 128 or 256) and *pair = 1 when 256 x 256 tiles run on CTA pairs. Callers that
 * verify one launch per configuration (the reference's verify="first", R:torch_xdna/runtime.py:191-209)
 * key their checks with it. */
int xdna_gemm_i8_config(int64_t M, int64_t N, int* tile_n, int* pair);

/* ------------------------------------------------------------------ conv3x3
 * The implicit-GEMM conv reads activations as a zero-bordered NHWC int8 tensor
 * xp [N, H+2, W+2, Cp] (Cp = channels rounded up to a multiple of 16, pad channels zero), and
 * weights as wp [Co, 9, Cp] int8 (tap = 3*ky + kx, pad channels zero). */

/* Per-image quantisation fused with the layout change: for image n of x [N, C, H, W] (NCHW,
 * contiguous, f32 / bf16 / f16): sx[n] = max(max |x[n]|, 1e-8) / 127, and xp gets
 * clamp(round_half_even(float(x) / sx[n]), -127, 127) inside a zero border.
 * amax_scratch: N uint32 words of scratch this call clears and uses.
 * Replaces the quantise ops of conv3x3_int8, R:torch_xdna/conv.py:45-46, and the host-side
 * NCHW -> NPU layout packing of Triton-XDNA's conv3x3 host code. */
int xdna_conv_quant_nhwc(const void* x, int x_dtype, int64_t N, int64_t C, int64_t H, int64_t W, int8_t* xp,
                         int64_t Cp, float* sx, uint32_t* amax_scratch, void* stream);

/* The same quantisation for x in channels-last memory ([N, H, W, C], torch's channels_last layout of
 * an [N, C, H, W] tensor; 16-byte aligned): a streaming copy with no transpose. This is the layout the
 * XDNA_CONV_DEQUANT epilogue writes, so one conv's output feeds the next conv's quantise directly. */
int xdna_conv_quant_channels_last(const void* x, int x_dtype, int64_t N, int64_t C, int64_t H, int64_t W,
                                  int8_t* xp, int64_t Cp, float* sx, uint32_t* amax_scratch, void* stream);

/* The next conv's input straight from a conv's int8 output, with no float tensor in between: q [N, H, W, C]
 * (XDNA_CONV_Q_NHWC; uint8 when q_unsigned, else int8; C a multiple of 4) stands for the dequantised
 * y = float(q) * (scale[c] * sx_in[n]) (+ bias[c]) (then max(y, 0) when relu_after), computed with the
 * same f32 roundings as XDNA_CONV_DEQUANT. With pool, y is max-pooled 2x2 / stride 2 first (output
 * H / 2 x W / 2, rounded down: torch's max_pool2d(2)); pooling the codes is exact because y grows with q.
 * Then y is quantised per image exactly as xdna_conv_quant_nhwc does (sx_out[n] = max(amax, 1e-8) / 127,
 * round half even, saturate to +-127) into the bordered xp [N, H'+2, W'+2, Cp]. amax_scratch: N words.
 * Replaces the dequantise at the end of conv3x3_int8 R:torch_xdna/conv.py:47-50, the graph's relu and
 * max_pool2d, and the next conv3x3_int8's quantise R:torch_xdna/conv.py:45-46, for a chain of convs whose
 * intermediate activations have no other use (the int8 NHWC chaining the reference names as its largest
 * remaining cost). */
/* xdna_conv_quant_nhwc for a layer of C <= 7 input channels with the 3x3 stencil's taps packed into each
 * pixel's row: xp [N, H+2, W+2, Kp] (Kp = round_up(9 C, 16)), byte t * C + c of bordered pixel (yb, xb) is
 * the quantised x[n, c, yb - 2 + t / 3, xb - 2 + t % 3] (0 outside the image), the rest zeros. The same
 * per-image scale and quantised values as xdna_conv_quant_nhwc; the conv then runs with
 * XDNA_CONV_SINGLE_TAP and weights wp [Co, 1, Kp], byte t * C + c of row co = wq[co, c, t / 3, t % 3]. */
int xdna_conv_quant_taps(const void* x, int x_dtype, int64_t N, int64_t C, int64_t H, int64_t W, int8_t* xp,
                         int64_t Kp, float* sx, uint32_t* amax_scratch, void* stream);

/* The per-image quantisation of xdna_conv_quant_nhwc (same sx, same values) written as the stride phases a
 * stride-2 conv reads (XDNA_CONV_STRIDE2): xp [planes, N, Ho+2, Wo+2, Cp], Ho = ceil(H / 2), Wo = ceil(W / 2),
 * planes 4 (all phases, for the 3x3 conv) or 1 (the even-even phase, for the 1x1 conv). x [N, C, H, W] in
 * NCHW memory (x_channels_last 0) or channels-last memory (1). Every byte of xp is written (borders and pixels
 * past the input are zeros). amax_scratch: N words. */
int xdna_conv_quant_phases(const void* x, int x_dtype, int x_channels_last, int64_t N, int64_t C, int64_t H,
                           int64_t W, int planes, int8_t* xp, int64_t Cp, float* sx, uint32_t* amax_scratch,
                           void* stream);

/* The two halves of xdna_conv_quant_nhwc / xdna_conv_quant_channels_last, for an image split into strips of
 * rows over several GPUs, whose scale needs the max over every strip (combined between the two calls, e.g.
 * by an all-reduce of the words): xdna_conv_image_amax writes each image's max |x| as its f32 bit pattern
 * (amax [N], cleared first; per_image = C * H * W contiguous elements, NaN propagates); xdna_conv_quant_given_amax
 * quantises x [N, C, H, W] (NCHW, or channels-last memory with x_channels_last) into the bordered xp with
 * sx[n] = max(amax[n], 1e-8) / 127 from the given words. A strip's border rows are written as zeros: the
 * halo rows from its neighbours are copied over them afterwards. No reference counterpart (the reference
 * runs on one device); the arithmetic is that of R:torch_xdna/conv.py:45-46. */
int xdna_conv_image_amax(const void* x, int x_dtype, int64_t N, int64_t per_image, uint32_t* amax, void* stream);
int xdna_conv_quant_given_amax(const void* x, int x_dtype, int x_channels_last, int64_t N, int64_t C, int64_t H,
                               int64_t W, int8_t* xp, int64_t Cp, float* sx, const uint32_t* amax, void* stream);

int xdna_conv_quant_codes(const void* q, int q_unsigned, int64_t N, int64_t C, int64_t H, int64_t W,
                          const float* scale, const float* sx_in, const float* bias, int relu_after, int pool,
                          int8_t* xp, int64_t Cp, float* sx_out, uint32_t* amax_scratch, void* stream);

/* xdna_conv_quant_codes with the per-image maxima already known (amax [N], the bit patterns the producing
 * conv wrote with XDNA_CONV_NEXT_AMAX, XDNA_CONV_NEXT_POOL iff pool): one pass over the codes instead of two. */
/* xdna_conv_quant_codes into the image-pair layout XDNA_CONV_PAIRS reads: xp [N/2, H'+2, W'+2, 128], image n's
 * channels at bytes 64 * (n % 2) .. of each pair row. C = 64, N even. amax: N words; with amax_given the
 * per-image maxima the producing conv wrote (XDNA_CONV_NEXT_AMAX), else scratch this call fills. */
int xdna_conv_quant_codes_pairs(const void* q, int q_unsigned, int64_t N, int64_t C, int64_t H, int64_t W,
                                const float* scale, const float* sx_in, const float* bias, int relu_after, int pool,
                                int8_t* xp, float* sx_out, uint32_t* amax, int amax_given, void* stream);

/* The int32 bias of XDNA_CONV_BIAS_INT32: out[n][co] = rint(bias[co] / (sw[co] * sx[n])) in f32 (the product
 * and the quotient correctly rounded, rint to nearest even), clamped to [-2^29, 2^29], NaN -> 0. bias: Co
 * values of bias_dtype (f32 / bf16 / f16); sw: the layer's weight scales [Co]; sx: the images' scales [N]. */
int xdna_conv_bias_int32(const void* bias, int bias_dtype, const float* sw, const float* sx, int64_t N, int64_t Co,
                         int32_t* out, void* stream);

int xdna_conv_quant_codes_given_amax(const void* q, int q_unsigned, int64_t N, int64_t C, int64_t H, int64_t W,
                                     const float* scale, const float* sx_in, const float* bias, int relu_after,
                                     int pool, int8_t* xp, int64_t Cp, float* sx_out, const uint32_t* amax,
                                     void* stream);

/* xdna_conv_quant_nhwc without caller-provided scratch: the same inputs, outputs and results, but the
 * per-image max lives in a 16 KB array inside the library, so the call allocates nothing and takes no
 * scratch pointer. It has no counterpart in the reference (whose quantise runs on the CPU).
 * It is for callers that must not allocate device memory: plugins whose host framework hands them all
 * of their memory up front and forbids allocation while serving, and latency-bound serving loops that
 * cannot afford cudaMalloc's device-wide synchronisation.
 * Limits and behaviour:
 *   - at most 4096 images per call; more returns XDNA_ERR_INVALID with a message;
 *   - the first call on each device looks up the array's device address (cudaGetSymbolAddress, with
 *     that device current) and caches it; make that first call before any stream capture;
 *   - every call on a device shares the one array and clears the words it uses first; calls that
 *     overlap on the GPU (other streams, or other threads) race on it and must be serialised;
 *   - the array stays allocated on every GPU that loaded the library until the process exits. */
int xdna_conv_quant_nhwc_static(const void* x, int x_dtype, int64_t N, int64_t C, int64_t H, int64_t W, int8_t* xp,
                                int64_t Cp, float* sx, void* stream);

/* NCHW int8 xq [N, C, H, W] (the xdna::conv3x3 op's input) -> bordered NHWC xp as above. */
int xdna_conv_pack_input(const int8_t* xq, int64_t N, int64_t C, int64_t H, int64_t W, int8_t* xp, int64_t Cp,
                         void* stream);

/* int8 weights wq [Co, Ci, 3, 3] (contiguous) -> wp [Co, 9, Cp]. */
int xdna_conv_pack_weight(const int8_t* wq, int64_t Co, int64_t Ci, int8_t* wp, int64_t Cp, void* stream);

/* 3x3 / stride 1 / padding 1 conv of xp by wp on the int8 tensor cores, int32 sums, and one of the
 * epilogues XDNA_CONV_Q / XDNA_CONV_DEQUANT / XDNA_CONV_CALIBRATE (see above). Rounding of the
 * requantise is round half up via an arithmetic shift, then saturation: [-128,127] int8, or
 * [0,255] uint8 when relu != 0. Output `out`: NCHW [N, Co, H, W] XDNA_I8 / XDNA_U8 for XDNA_CONV_Q;
 * channels-last [N, H, W, Co] XDNA_F32 / XDNA_BF16 / XDNA_F16 for XDNA_CONV_DEQUANT. For XDNA_CONV_CALIBRATE
 * only image 0 is computed and acc_max (one int32, cleared by this call) receives the maximum.
 * XDNA_CONV_Q_NHWC writes the same q as XDNA_CONV_Q, channels-last [N, H, W, Co] (XDNA_I8 / XDNA_U8).
 * Replaces tl.extra.npu.conv3x3.Conv3x3(...)(xq) as used by ConvLayer.npu
 * R:torch_xdna/conv.py:78-84,94-103, the CPU integers ConvLayer.cpu R:torch_xdna/conv.py:86-92,
 * the calibration sums of ConvLayer.calibrate R:torch_xdna/conv.py:71-76, and (DEQUANT) the
 * dequantise ops of conv3x3_int8 R:torch_xdna/conv.py:47-50. */
int xdna_conv3x3_i8(const int8_t* xp, const int8_t* wp, int64_t N, int64_t Ci, int64_t Cp, int64_t Co, int64_t H,
                    int64_t W, int mode, int shift, int relu, const float* scale, const float* sx, const void* bias,
                    int bias_dtype, void* out, int out_dtype, int32_t* acc_max, void* stream);

/* ------------------------------------------------------------------ the Qwen3 stack (bf16)
 * Replaces tl.extra.npu.qwen3_stack.Qwen3Stack(...)(x0, x1), the one-launch NPU program called by
 * stack.run R:torch_xdna/stack.py:360-389, for Qwen3-0.6B's shapes (hidden 1024, 16 query / 8 kv heads
 * of 128, MLP 3072), any depth, and extends it to causal and general masks and any length. */

/* epilogues of xdna_gemm_bf16 */
#define XDNA_GEMM_F32ACC 0 /* out = acc (+ bias[n]) in out_dtype */
#define XDNA_GEMM_RESID 1  /* resid[m, n] += acc (f32, in place) */
#define XDNA_GEMM_SWIGLU 2 /* B rows interleave 32 gate / 32 up rows: out[m, j] = bf16(silu(gate) * up), N/2 columns */
#define XDNA_GEMM_QKV 3    /* N = 4096 = q 2048 | k 1024 | v 1024 columns: out [M, 3072] bf16 gets q and k after the
                              per-head RMSNorm (q_norm / k_norm) and RoPE at position m % seq_len; vt [1024, ldvt]
                              bf16 gets v transposed */

/* attention masks */
#define XDNA_MASK_CAUSAL 0 /* key <= query */
#define XDNA_MASK_PREFIX 1 /* lens[b]: the first n positions see each other, later ones only themselves */
#define XDNA_MASK_BOOL 2   /* mask [B, 1|16, L, L] bytes, nonzero = may attend */
#define XDNA_MASK_NONE 3

/* One decoder layer's weights, bf16 matrices (row-major [out, in]) and f32 norm weights. */
typedef struct {
  const void* w_qkv;        /* [4096, 1024]: q_proj (2048 rows), k_proj (1024), v_proj (1024) */
  const void* w_o;          /* [1024, 2048] */
  const void* w_gu;         /* [6144, 1024]: gate_proj / up_proj interleaved in blocks of 32 rows */
  const void* w_down;       /* [1024, 3072] */
  const float* input_norm;  /* [1024] */
  const float* post_norm;   /* [1024] */
  const float* q_norm;      /* [128] */
  const float* k_norm;      /* [128] */
} xdna_qwen3_layer;

/* y [rows, D] bf16 = x * rsqrt(mean(x^2) + eps) * w, x f32 (D = 128, 512 or 1024). */
int xdna_rmsnorm_bf16(const float* x, int64_t rows, int64_t D, const float* w, float eps, void* y, void* stream);

/* x [tokens, D] f32 = table[ids] (bf16 or f32 table [vocab, D]); ids outside [0, vocab) give zeros and
 * record XDNA_ERR_INVALID in the device error word. Replaces the embed_tokens lookup of the model. */
int xdna_embed(const int64_t* ids, int64_t tokens, const void* table, int table_dtype, int64_t vocab, int64_t D,
               float* x, void* stream);

/* C [M, N] = A [M, K] . B [N, K]^T, bf16 operands (row pitches lda / ldb in elements, multiples of 8),
 * f32 accumulation on the tcgen05 tensor cores, with one of the XDNA_GEMM_* epilogues. XDNA_GEMM_QKV's
 * rope_cos / rope_sin: f32 tables of the model's inverse frequencies at positions 0..seq_len-1 in the layout
 * [16, seq_len, 4]: frequency d of position p at index (d / 4) * seq_len * 4 + p * 4 + d % 4. */
int xdna_gemm_bf16(const void* a, int64_t lda, const void* b, int64_t ldb, int64_t M, int64_t N, int64_t K, int mode,
                   void* out, int out_dtype, int64_t ldo, const void* bias, int bias_dtype, float* resid, int64_t ldr,
                   void* vt, int64_t ldvt, const float* rope_cos, const float* rope_sin, const float* q_norm,
                   const float* k_norm, int64_t seq_len, float eps, void* stream);

/* The head GEMM of a column-parallel stack, fused with the all-gather of its input: out [n_parts *
 * rows_per_part, N] = A . b^T (+ bias) with the XDNA_GEMM_F32ACC epilogue, where rows [i * rows_per_part,
 * (i + 1) * rows_per_part) of A are a_parts[i] ([rows_per_part, K] bf16, pitch lda) — device pointers
 * that may belong to other GPUs of the box (peer memory opened with xdna_ipc_open), read by the GEMM's
 * TMA producer over NVLink while the tensor cores run, instead of a separate all-gather. rows_per_part
 * must be a multiple of 256. maps: device memory for n_parts tensor maps (128 bytes each, 64-byte
 * aligned), written by this call (stream-ordered). The caller orders the parts' writes before this call
 * on every GPU (e.g. a barrier collective). Replaces the all-gather followed by the head GEMM of the
 * column-parallel head on several GPUs, which the reference (one device) does not have. */
int xdna_gemm_bf16_gather(const void* const* a_parts, int n_parts, int64_t rows_per_part, int64_t lda, const void* b,
                          int64_t ldb, int64_t N, int64_t K, void* out, int out_dtype, int64_t ldo, const void* bias,
                          int bias_dtype, void* maps, void* stream);

/* CUDA IPC for xdna_gemm_bf16_gather's peer parts (no reference counterpart; the only entry points
 * that allocate): a dedicated device allocation that can be shared, its release; the 64-byte handle of
 * such an allocation; the device pointer of another process's allocation on this box (NVLink peer
 * access enabled) and its release. */
int xdna_ipc_alloc(size_t bytes, void** dev_ptr);
int xdna_ipc_free(void* dev_ptr);
int xdna_ipc_handle(const void* dev_ptr, void* handle64);
int xdna_ipc_open(const void* handle64, void** dev_ptr);
int xdna_ipc_close(void* dev_ptr);

/* out [B*L, 2048] bf16 = softmax(q k^T / sqrt(128) + mask) v for 16 query heads over 8 kv heads (GQA),
 * q and k read from qk [B*L, 3072] (the XDNA_GEMM_QKV output), v from vt [1024, ldvt]. */
int xdna_attention(const void* qk, const void* vt, int64_t ldvt, void* out, int64_t B, int64_t L, int mask_kind,
                   const int32_t* lens, const uint8_t* mask, int mask_heads, void* stream);

/* Bytes of workspace xdna_qwen3_stack needs for B sequences of L tokens. */
size_t xdna_qwen3_stack_workspace(int64_t B, int64_t L);

/* The whole stack: x [B*L, 1024] f32 (the hidden states, updated in place as the residual stream)
 * through n_layers decoder layers, the final RMSNorm and the head: out [B*L, head_n] (row pitch ldo)
 * = h Whead^T (+ bias) in out_dtype. rope_cos / rope_sin: f32 tables of the model's inverse frequencies
 * at positions 0..L-1, laid out [16, L, 4] as for xdna_gemm_bf16. With out == NULL the head is skipped and the final-normed hidden
 * states [B*L, 1024] bf16 are left at the start of the workspace. */
int xdna_qwen3_stack(const xdna_qwen3_layer* layers, int n_layers, const float* final_norm, const void* head_w,
                     int64_t head_n, const void* head_bias, int head_bias_dtype, const float* rope_cos,
                     const float* rope_sin, float eps, float* x, int64_t B, int64_t L, int mask_kind,
                     const int32_t* lens, const uint8_t* mask, int mask_heads, void* out, int out_dtype, int64_t ldo,
                     void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* XDNA_B200_H */
