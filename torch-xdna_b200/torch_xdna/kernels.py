"""The device side: libxdna_b200.so, hand-written sm_100a kernels behind a C ABI (include/xdna_b200.h).

Replaces the reference's Triton-XDNA driver module (R:torch_xdna/kernels.py): `available()`,
`unavailable_reason()` and `mark_broken()` keep their meaning; the launch functions below replace
`mm_i8` (R:torch_xdna/kernels.py:172-192) and the Triton-XDNA conv3x3 / qwen3_stack calls.

The library is loaded from this package (lib/libxdna_b200.so, built in-tree by
__graft_entry__.build() or `make -C torch-xdna_b200/csrc`). There is no CPU fallback: without the
library or without an sm_100 GPU, every op raises XdnaUnavailable with the reason.
"""

import ctypes
import os
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libxdna_b200.so"
ABI_VERSION = 1

# element types (XDNA_F32 ...)
F32, BF16, F16, I32, I8, U8 = 0, 1, 2, 3, 4, 5
DTYPE_CODES = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16, torch.int32: I32, torch.int8: I8,
               torch.uint8: U8}
# conv3x3 modes
CONV_Q, CONV_DEQUANT, CONV_CALIBRATE, CONV_Q_NHWC = 0, 1, 2, 3
CONV_SINGLE_TAP = 16  # or'ed into a conv mode: one tap at offset 0 (a 1x1 conv, or taps packed into channels)
CONV_STRIDE2 = 32     # or'ed into a conv mode: stride 2, the input split into phase planes (conv_quant_phases)
# or'ed into CONV_Q_NHWC: the next layer's per-image maxima into acc_max (with its ReLU / 2x2 pool region)
CONV_NEXT_AMAX, CONV_NEXT_RELU, CONV_NEXT_POOL = 64, 128, 256
CONV_BIAS_INT32 = 512  # or'ed into any conv mode: `bias` is int32 [N, Co] (conv_bias_int32), added to the sums
CONV_PAIRS = 1024      # or'ed into CONV_Q_NHWC: the input holds the images in pairs (conv_quant_codes_pairs)
# status codes
ERR_TIMEOUT = -4

_lock = threading.RLock()
_state = {"lib": None, "ok": None, "error": None}


class XdnaUnavailable(RuntimeError):
    """No B200 or no library: the xdna ops cannot run in this process."""


class XdnaError(RuntimeError):
    """A library call returned an error status."""

    def __init__(self, name, status, message):
        super().__init__(f"{name} failed ({status}): {message}")
        self.status = status


def _load():
    if not LIB_PATH.exists():
        raise XdnaUnavailable(f"{LIB_PATH} is not built (run __graft_entry__.build() or make -C torch-xdna_b200/csrc)")
    lib = ctypes.CDLL(str(LIB_PATH))
    P, I64, I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    sig = {
        "xdna_last_error": ([], ctypes.c_char_p),
        "xdna_abi_version": ([], I),
        "xdna_device_check": ([I], I),
        "xdna_take_device_error": ([P, P, P], I),
        "xdna_quant_rows_i8": ([P, I, I64, I64, I64, P, I64, P, P], I),
        "xdna_gemm_i8": ([P, I64, P, I64, I64, I64, I64, P, P, P, I, P, I, I64, P], I),
        "xdna_gemm_i8_config": ([I64, I64, P, P], I),
        "xdna_selftest_wait_timeout": ([ctypes.c_uint64, P], I),
        "xdna_conv_quant_nhwc": ([P, I, I64, I64, I64, I64, P, I64, P, P, P], I),
        "xdna_conv_quant_channels_last": ([P, I, I64, I64, I64, I64, P, I64, P, P, P], I),
        "xdna_conv_quant_codes": ([P, I, I64, I64, I64, I64, P, P, P, I, I, P, I64, P, P, P], I),
        "xdna_conv_quant_codes_given_amax": ([P, I, I64, I64, I64, I64, P, P, P, I, I, P, I64, P, P, P], I),
        "xdna_conv_bias_int32": ([P, I, P, P, I64, I64, P, P], I),
        "xdna_conv_quant_codes_pairs": ([P, I, I64, I64, I64, I64, P, P, P, I, I, P, P, P, I, P], I),
        "xdna_conv_quant_taps": ([P, I, I64, I64, I64, I64, P, I64, P, P, P], I),
        "xdna_conv_quant_phases": ([P, I, I, I64, I64, I64, I64, I, P, I64, P, P, P], I),
        "xdna_conv_image_amax": ([P, I, I64, I64, P, P], I),
        "xdna_conv_quant_given_amax": ([P, I, I, I64, I64, I64, I64, P, I64, P, P, P], I),
        "xdna_conv_pack_input": ([P, I64, I64, I64, I64, P, I64, P], I),
        "xdna_conv_pack_weight": ([P, I64, I64, P, I64, P], I),
        "xdna_conv3x3_i8": ([P, P, I64, I64, I64, I64, I64, I64, I, I, I, P, P, P, I, P, I, P, P], I),
        "xdna_rmsnorm_bf16": ([P, I64, I64, P, ctypes.c_float, P, P], I),
        "xdna_embed": ([P, I64, P, I, I64, I64, P, P], I),
        "xdna_gemm_bf16": ([P, I64, P, I64, I64, I64, I64, I, P, I, I64, P, I, P, I64, P, I64, P, P, P, P, I64,
                            ctypes.c_float, P], I),
        "xdna_gemm_bf16_gather": ([P, I, I64, I64, P, I64, I64, I64, P, I, I64, P, I, P, P], I),
        "xdna_ipc_alloc": ([ctypes.c_size_t, P], I),
        "xdna_ipc_free": ([P], I),
        "xdna_ipc_handle": ([P, P], I),
        "xdna_ipc_open": ([P, P], I),
        "xdna_ipc_close": ([P], I),
        "xdna_attention": ([P, P, I64, P, I64, I64, I, P, P, I, P], I),
        "xdna_qwen3_stack_workspace": ([I64, I64], ctypes.c_size_t),
        "xdna_qwen3_stack": ([P, I, P, P, I64, P, I, P, P, ctypes.c_float, P, I64, I64, I, P, P, I, P, I, I64, P,
                              ctypes.c_size_t, P], I),
    }
    for name, (args, res) in sig.items():
        fn = getattr(lib, name)
        fn.argtypes, fn.restype = args, res
    if lib.xdna_abi_version() != ABI_VERSION:
        raise XdnaUnavailable(f"{LIB_PATH} has ABI {lib.xdna_abi_version()}, this package needs {ABI_VERSION}")
    return lib


def lib():
    """The loaded library; raises XdnaUnavailable (loudly) when it cannot be used."""
    with _lock:
        if _state["lib"] is None:
            try:
                _state["lib"] = _load()
            except XdnaUnavailable:
                raise
            except OSError as e:
                raise XdnaUnavailable(f"cannot load {LIB_PATH}: {e}") from e
        return _state["lib"]


def available() -> bool:
    """True if the xdna ops can run here: the library loads and CUDA device 0 is an sm_100 GPU."""
    with _lock:
        if _state["ok"] is None:
            try:
                if os.environ.get("TORCH_XDNA_DISABLE_GPU") == "1":
                    raise XdnaUnavailable("disabled by TORCH_XDNA_DISABLE_GPU=1")
                if not torch.cuda.is_available():
                    raise XdnaUnavailable("no CUDA device")
                L = lib()
                rc = L.xdna_device_check(torch.cuda.current_device())
                if rc != 0:
                    raise XdnaUnavailable(L.xdna_last_error().decode())
                _state["ok"] = True
            except Exception as e:  # any missing piece: the ops raise with this reason
                _state["ok"], _state["error"] = False, f"{type(e).__name__}: {e}"
        return _state["ok"]


def unavailable_reason():
    return _state["error"]


def mark_broken(err: BaseException):
    """A launch failed unrecoverably: stop accepting calls for the rest of the process."""
    with _lock:
        _state["ok"], _state["error"] = False, f"{type(err).__name__}: {err}"


def require():
    if not available():
        raise XdnaUnavailable(f"torch_xdna needs a B200 (sm_100) and libxdna_b200.so: {unavailable_reason()}")
    return lib()


def device_name() -> str:
    if not available():
        return "none"
    return torch.cuda.get_device_name(torch.cuda.current_device())


# ---------------------------------------------------------------- call helpers
def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _check(name, rc):
    if rc != 0:
        raise XdnaError(name, rc, lib().xdna_last_error().decode())


def _cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise XdnaUnavailable("torch_xdna ops run on CUDA tensors; move the model and inputs to the B200")


def take_device_error():
    """(code, site) recorded by a bounded device wait since the last call; (0, 0) when none. Synchronises."""
    L = require()
    code, site = ctypes.c_int(0), ctypes.c_int(0)
    _check("xdna_take_device_error", L.xdna_take_device_error(ctypes.byref(code), ctypes.byref(site), _stream()))
    return code.value, site.value


def selftest_wait_timeout(limit_ns=1_000_000):
    """Launch the bounded-wait self-test (a wait that nothing completes, limit_ns of device time); read the
    result with take_device_error(): (ERR_TIMEOUT, 99)."""
    _check("xdna_selftest_wait_timeout", require().xdna_selftest_wait_timeout(limit_ns, _stream()))


def gemm_i8_config(M, N):
    """(columns per tile, on CTA pairs) of the kernel xdna_gemm_i8 launches for an M x N output here."""
    tile_n, pair = ctypes.c_int(0), ctypes.c_int(0)
    _check("xdna_gemm_i8_config", require().xdna_gemm_i8_config(M, N, ctypes.byref(tile_n), ctypes.byref(pair)))
    return tile_n.value, bool(pair.value)


def round_up(x, m):
    return -(-x // m) * m


def quant_rows(x2d, xq, scale):
    """xq[:, :K] / scale[:] = per-row int8 of x2d [R, K] (f32/bf16/f16; unit column stride)."""
    L = require()
    _cuda(x2d, xq, scale)
    R, K = x2d.shape
    assert x2d.stride(1) == 1 or K <= 1, "rows must be contiguous"
    _check("xdna_quant_rows_i8", L.xdna_quant_rows_i8(_p(x2d), DTYPE_CODES[x2d.dtype], R, K, max(x2d.stride(0), K),
                                                      _p(xq), xq.stride(0), _p(scale), _stream()))


def gemm_i8(xq, wq, K, y, sx=None, sw=None, bias=None):
    """y [M, N] = xq[:, :K] . wq[:, :K]^T (int32 y), or its dequantisation in y's float dtype."""
    L = require()
    _cuda(xq, wq, y, sx, sw, bias)
    M, N = y.shape
    _check("xdna_gemm_i8", L.xdna_gemm_i8(_p(xq), xq.stride(0), _p(wq), wq.stride(0), M, N, K, _p(sx), _p(sw),
                                          _p(bias), DTYPE_CODES[bias.dtype] if bias is not None else F32,
                                          _p(y), DTYPE_CODES[y.dtype], y.stride(0), _stream()))


def conv_quant(x, xp, sx, scratch):
    L = require()
    _cuda(x, xp, sx, scratch)
    N, C, H, W = x.shape
    _check("xdna_conv_quant_nhwc", L.xdna_conv_quant_nhwc(_p(x), DTYPE_CODES[x.dtype], N, C, H, W, _p(xp),
                                                          xp.shape[-1], _p(sx), _p(scratch), _stream()))


def conv_quant_channels_last(x, xp, sx, scratch):
    """conv_quant for x [N, C, H, W] stored channels-last (x.is_contiguous(memory_format=channels_last))."""
    L = require()
    _cuda(x, xp, sx, scratch)
    N, C, H, W = x.shape
    _check("xdna_conv_quant_channels_last", L.xdna_conv_quant_channels_last(
        _p(x), DTYPE_CODES[x.dtype], N, C, H, W, _p(xp), xp.shape[-1], _p(sx), _p(scratch), _stream()))


def conv_quant_taps(x, xp, sx, scratch):
    """conv_quant for x [N, C <= 7, H, W] (NCHW contiguous) with the 3x3 stencil's taps packed into each
    pixel's row of xp [N, H+2, W+2, Kp] (xdna_conv_quant_taps)."""
    L = require()
    _cuda(x, xp, sx, scratch)
    N, C, H, W = x.shape
    _check("xdna_conv_quant_taps", L.xdna_conv_quant_taps(_p(x), DTYPE_CODES[x.dtype], N, C, H, W, _p(xp),
                                                          xp.shape[-1], _p(sx), _p(scratch), _stream()))


def conv_image_amax(x, amax):
    """amax [N] int32 = the bit patterns of each image's max |x| (x [N, ...], each image contiguous)."""
    L = require()
    _cuda(x, amax)
    N = x.shape[0]
    _check("xdna_conv_image_amax", L.xdna_conv_image_amax(_p(x), DTYPE_CODES[x.dtype], N, x.numel() // max(N, 1),
                                                          _p(amax), _stream()))


def conv_quant_given_amax(x, xp, sx, amax, channels_last):
    """The bordered quantise of x [N, C, H, W] (NCHW, or channels-last memory) with the per-image maxima given
    as bit patterns in amax [N] (e.g. combined over an image's strips)."""
    L = require()
    _cuda(x, xp, sx, amax)
    N, C, H, W = x.shape
    _check("xdna_conv_quant_given_amax", L.xdna_conv_quant_given_amax(
        _p(x), DTYPE_CODES[x.dtype], int(channels_last), N, C, H, W, _p(xp), xp.shape[-1], _p(sx), _p(amax),
        _stream()))


def conv_quant_phases(x, xp, sx, scratch, channels_last):
    """The per-image quantise of x [N, C, H, W] (NCHW or, with channels_last, channels-last memory) written as
    the stride phases of a stride-2 conv: xp [planes, N, ceil(H/2)+2, ceil(W/2)+2, Cp], planes 4 (3x3 conv) or
    1 (1x1 conv) (xdna_conv_quant_phases)."""
    L = require()
    _cuda(x, xp, sx, scratch)
    N, C, H, W = x.shape
    _check("xdna_conv_quant_phases", L.xdna_conv_quant_phases(
        _p(x), DTYPE_CODES[x.dtype], int(channels_last), N, C, H, W, xp.shape[0], _p(xp), xp.shape[-1], _p(sx),
        _p(scratch), _stream()))


def conv_quant_codes(q, scale, sx_in, bias, relu_after, pool, xp, sx, scratch):
    """The next conv's bordered input xp from a conv's channels-last codes q [N, H, W, C] (uint8 / int8):
    y = float(q) * (scale * sx_in) (+ bias) (then max(y, 0)), 2x2 max-pooled when `pool`, quantised per
    image (xdna_conv_quant_codes)."""
    L = require()
    _cuda(q, scale, sx_in, bias, xp, sx, scratch)
    N, H, W, C = q.shape
    _check("xdna_conv_quant_codes", L.xdna_conv_quant_codes(
        _p(q), int(q.dtype == torch.uint8), N, C, H, W, _p(scale), _p(sx_in), _p(bias), int(relu_after), int(pool),
        _p(xp), xp.shape[-1], _p(sx), _p(scratch), _stream()))


def conv_quant_codes_given_amax(q, scale, sx_in, bias, relu_after, pool, xp, sx, amax):
    """conv_quant_codes with each image's max already known (amax [N] int32 bit patterns written by the
    producing conv with CONV_NEXT_AMAX): one pass over the codes."""
    L = require()
    _cuda(q, scale, sx_in, bias, xp, sx, amax)
    N, H, W, C = q.shape
    _check("xdna_conv_quant_codes_given_amax", L.xdna_conv_quant_codes_given_amax(
        _p(q), int(q.dtype == torch.uint8), N, C, H, W, _p(scale), _p(sx_in), _p(bias), int(relu_after), int(pool),
        _p(xp), xp.shape[-1], _p(sx), _p(amax), _stream()))


def conv_quant_codes_pairs(q, scale, sx_in, bias, relu_after, pool, xp2, sx, amax, amax_given):
    """conv_quant_codes into the image-pair layout xp2 [N/2, H'+2, W'+2, 128] (64 channels): amax holds the
    producing conv's maxima when amax_given, else it is scratch."""
    L = require()
    _cuda(q, scale, sx_in, bias, xp2, sx, amax)
    N, H, W, C = q.shape
    _check("xdna_conv_quant_codes_pairs", L.xdna_conv_quant_codes_pairs(
        _p(q), int(q.dtype == torch.uint8), N, C, H, W, _p(scale), _p(sx_in), _p(bias), int(relu_after), int(pool),
        _p(xp2), _p(sx), _p(amax), int(amax_given), _stream()))


def conv_bias_int32(bias, sw, sx, out):
    """out [N, Co] int32 = rint(bias / (sw * sx)) per image (xdna_conv_bias_int32)."""
    L = require()
    _cuda(bias, sw, sx, out)
    _check("xdna_conv_bias_int32", L.xdna_conv_bias_int32(_p(bias), DTYPE_CODES[bias.dtype], _p(sw), _p(sx),
                                                          sx.numel(), sw.numel(), _p(out), _stream()))


def conv_pack_input(xq, xp):
    L = require()
    _cuda(xq, xp)
    N, C, H, W = xq.shape
    _check("xdna_conv_pack_input", L.xdna_conv_pack_input(_p(xq), N, C, H, W, _p(xp), xp.shape[-1], _stream()))


def conv_pack_weight(wq, wp):
    L = require()
    _cuda(wq, wp)
    Co, Ci = wq.shape[:2]
    _check("xdna_conv_pack_weight", L.xdna_conv_pack_weight(_p(wq), Co, Ci, _p(wp), wp.shape[-1], _stream()))


RELU_AFTER_BIAS = 2  # conv3x3 relu mode: max(y, 0) after the dequantise and the bias (XDNA_RELU_AFTER_BIAS)


def conv3x3(xp, wp, N, Ci, Co, H, W, mode, shift=1, relu=False, scale=None, sx=None, bias=None, out=None,
            acc_max=None):
    L = require()
    _cuda(xp, wp, scale, sx, bias, out, acc_max)
    Cp = wp.shape[-1]
    _check("xdna_conv3x3_i8", L.xdna_conv3x3_i8(
        _p(xp), _p(wp), N, Ci, Cp, Co, H, W, mode, shift, int(relu), _p(scale), _p(sx), _p(bias),
        DTYPE_CODES[bias.dtype] if bias is not None else F32, _p(out),
        DTYPE_CODES[out.dtype] if out is not None else I8, _p(acc_max), _stream()))


# ---------------------------------------------------------------- the Qwen3 stack (bf16)
GEMM_F32ACC, GEMM_RESID, GEMM_SWIGLU, GEMM_QKV = 0, 1, 2, 3
MASK_CAUSAL, MASK_PREFIX, MASK_BOOL, MASK_NONE = 0, 1, 2, 3


class Qwen3Layer(ctypes.Structure):
    """xdna_qwen3_layer: one decoder layer's device pointers."""

    _fields_ = [(n, ctypes.c_void_p) for n in ("w_qkv", "w_o", "w_gu", "w_down", "input_norm", "post_norm", "q_norm",
                                                 "k_norm")]


def rmsnorm_bf16(x, w, eps, y):
    L = require()
    _cuda(x, w, y)
    rows, D = x.shape
    _check("xdna_rmsnorm_bf16", L.xdna_rmsnorm_bf16(_p(x), rows, D, _p(w), eps, _p(y), _stream()))


def embed(ids, table, x):
    L = require()
    _cuda(ids, table, x)
    _check("xdna_embed", L.xdna_embed(_p(ids), ids.numel(), _p(table), DTYPE_CODES[table.dtype], table.shape[0],
                                      table.shape[1], _p(x), _stream()))


def rope_layout(table):
    """A RoPE table [L, 64] (position, frequency) f32 in the layout the q/k/v epilogue reads, [16, L, 4]:
    four frequencies per 16-byte vector, positions fastest, so that the 32 consecutive positions of a warp's
    rows are one coalesced 512-byte load."""
    L = table.shape[0]
    return table.reshape(L, 16, 4).transpose(0, 1).contiguous()


def gemm_bf16(a, b, mode, out=None, bias=None, resid=None, vt=None, rope_cos=None, rope_sin=None, q_norm=None,
              k_norm=None, seq_len=0, eps=1e-6, M=None):
    """C = a[:, :K] . b[:, :K]^T (bf16) with the epilogue `mode` (GEMM_*); see include/xdna_b200.h."""
    L = require()
    _cuda(a, b, out, bias, resid, vt, rope_cos, rope_sin, q_norm, k_norm)
    M = a.shape[0] if M is None else M
    N, K = b.shape[0], a.shape[1]
    _check("xdna_gemm_bf16", L.xdna_gemm_bf16(
        _p(a), a.stride(0), _p(b), b.stride(0), M, N, K, mode, _p(out),
        DTYPE_CODES[out.dtype] if out is not None else BF16, out.stride(0) if out is not None else 0,
        _p(bias), DTYPE_CODES[bias.dtype] if bias is not None else F32, _p(resid),
        resid.stride(0) if resid is not None else 0, _p(vt), vt.stride(0) if vt is not None else 0,
        _p(rope_cos), _p(rope_sin), _p(q_norm), _p(k_norm), seq_len, eps, _stream()))


def gemm_bf16_gather(parts, rows_per_part, lda, b, out, maps, bias=None):
    """out = A . b^T with the head epilogue, A the row-concatenation of `parts` (device pointers, possibly
    on peer GPUs, each [rows_per_part, K] bf16 with row pitch lda); maps: a device buffer of at least
    128 * len(parts) bytes, 64-byte aligned (xdna_gemm_bf16_gather)."""
    L = require()
    _cuda(b, out, maps, bias)
    arr = (ctypes.c_void_p * len(parts))(*[p if isinstance(p, int) else p.data_ptr() for p in parts])
    N, K = b.shape
    _check("xdna_gemm_bf16_gather", L.xdna_gemm_bf16_gather(
        ctypes.cast(arr, ctypes.c_void_p), len(parts), rows_per_part, lda, _p(b), b.stride(0), N, K, _p(out),
        DTYPE_CODES[out.dtype], out.stride(0), _p(bias), DTYPE_CODES[bias.dtype] if bias is not None else F32,
        _p(maps), _stream()))


class _CudaArray:
    """A zero-copy view of raw device memory for torch.as_tensor (__cuda_array_interface__)."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": tuple(shape), "typestr": typestr,
                                         "version": 3}


def ipc_alloc(shape, device):
    """A bf16 tensor on `device` in its own shareable allocation (xdna_ipc_alloc); free with ipc_free."""
    L = require()
    ptr = ctypes.c_void_p()
    numel = 1
    for d in shape:
        numel *= d
    with torch.cuda.device(device):
        _check("xdna_ipc_alloc", L.xdna_ipc_alloc(numel * 2, ctypes.byref(ptr)))
    return device_view(ptr.value, shape, device), ptr.value


def device_view(ptr, shape, device):
    """A bf16 tensor over existing device memory at `ptr` (e.g. a peer GPU's buffer opened with ipc_open)."""
    with torch.cuda.device(device):
        return torch.as_tensor(_CudaArray(ptr, shape, "<i2"), device=device).view(torch.bfloat16)


def ipc_free(ptr):
    _check("xdna_ipc_free", require().xdna_ipc_free(ctypes.c_void_p(ptr)))


def ipc_handle(ptr) -> bytes:
    buf = ctypes.create_string_buffer(64)
    _check("xdna_ipc_handle", require().xdna_ipc_handle(ctypes.c_void_p(ptr), buf))
    return buf.raw


def ipc_open(handle: bytes) -> int:
    ptr = ctypes.c_void_p()
    _check("xdna_ipc_open", require().xdna_ipc_open(ctypes.create_string_buffer(handle, 64), ctypes.byref(ptr)))
    return ptr.value


def ipc_close(ptr):
    _check("xdna_ipc_close", require().xdna_ipc_close(ctypes.c_void_p(ptr)))


def attention(qk, vt, out, B, L_, mask_kind, lens=None, mask=None):
    L = require()
    _cuda(qk, vt, out, lens, mask)
    mh = mask.shape[1] if mask is not None else 1
    _check("xdna_attention", L.xdna_attention(_p(qk), _p(vt), vt.stride(0), _p(out), B, L_, mask_kind, _p(lens),
                                              _p(mask), mh, _stream()))


def qwen3_stack_workspace(B, L_):
    return int(require().xdna_qwen3_stack_workspace(B, L_))


def qwen3_stack(layers, final_norm, head_w, head_bias, rope_cos, rope_sin, eps, x, B, L_, mask_kind, lens, mask,
                out, workspace):
    """The whole stack through xdna_qwen3_stack. layers: a ctypes array of Qwen3Layer."""
    L = require()
    _cuda(final_norm, head_w, head_bias, rope_cos, rope_sin, x, lens, mask, out, workspace)
    mh = mask.shape[1] if mask is not None else 1
    _check("xdna_qwen3_stack", L.xdna_qwen3_stack(
        ctypes.cast(layers, ctypes.c_void_p), len(layers), _p(final_norm), _p(head_w), head_w.shape[0],
        _p(head_bias), DTYPE_CODES[head_bias.dtype] if head_bias is not None else F32, _p(rope_cos), _p(rope_sin),
        eps, _p(x), B, L_, mask_kind, _p(lens), _p(mask), mh, _p(out),
        DTYPE_CODES[out.dtype] if out is not None else F32, out.stride(0) if out is not None else 0,
        _p(workspace), workspace.numel() * workspace.element_size(), _stream()))
