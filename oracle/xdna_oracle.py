"""CPU oracle for the torch_xdna B200 build -- TEST INFRASTRUCTURE, NOT PRODUCT CODE.

A numpy restatement of the reference's (AyaSakura-comp/torch-xdna) CPU arithmetic for the three
offloaded ops, used only as the checker. Only tests/, __graft_entry__.smoke() and bench.py's
cpu_baseline / --impl reference leg may import this module; the product package never does, and
the product fails loudly when its CUDA library is missing instead of falling back to anything here.

Pinned against the reference: tests/test_oracle.py checks every function below against the golden
vectors that tests/golden/make_golden.py recorded by running the unmodified reference on the CPU
(bit-exact for the integer and dequantised outputs; within 1e-5 relative for the fp32 stack).

Each function cites the reference file:line it restates ("R:" = path inside the reference).
Integer sums are computed exactly as float64 matrix products: every product of two int8 values is at
most 2^14 in magnitude, so sums stay exact far beyond any K used here (< 2^53 / 2^14).
"""

import numpy as np

F32 = np.float32


# ---------------------------------------------------------------- dtype helpers
def bf16_round(x):
    """float32 -> nearest-even bfloat16, returned as float32 values (torch's .to(torch.bfloat16))."""
    x = np.ascontiguousarray(x, dtype=F32)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = (r & 0xFFFFFFFF).astype(np.uint32).view(F32)
    return np.where(np.isnan(x), x, out).astype(F32)


def f16_round(x):
    return np.asarray(x, dtype=F32).astype(np.float16).astype(F32)


def cast(y, dtype):
    """y (float32) rounded to `dtype` ("float32" | "bfloat16" | "float16"), kept as float32 values."""
    if dtype == "float32":
        return np.asarray(y, dtype=F32)
    if dtype == "bfloat16":
        return bf16_round(y)
    if dtype == "float16":
        return f16_round(y)
    raise ValueError(dtype)


# ---------------------------------------------------------------- W8A8 linear
def quant_rows(x):
    """Per-row int8: R:torch_xdna/runtime.py:145-148 (_quant_rows) and the graph form :366-368.

    x holds the row values as float32 (for a bf16 input: the exactly widened bf16 values; the
    reference takes the max in bf16, which is exact, then widens). Returns (xq int8, scale f32 [R]).
    """
    x = np.asarray(x, dtype=F32)
    amax = np.abs(x).max(axis=1) if x.shape[1] else np.zeros(x.shape[0], F32)
    s = (np.maximum(amax, F32(1e-8)) / F32(127)).astype(F32)
    q = np.clip(np.rint(x / s[:, None]), -127, 127).astype(np.int8)
    return q, s


def quant_weight(w, transposed=False):
    """QWeight, R:torch_xdna/runtime.py:59-66: per output channel. Returns (wq [N, K] int8, sw [N])."""
    w = np.asarray(w, dtype=F32)
    if transposed:
        w = w.T
    return quant_rows(w)


def int_mm(xq, wq):
    """acc [M, N] int32 = xq [M, K] . wq [N, K]^T -- torch._int_mm(xq, w_kn), R:torch_xdna/runtime.py:162-163."""
    acc = np.asarray(xq, dtype=np.float64) @ np.asarray(wq, dtype=np.float64).T
    return acc.astype(np.int64).astype(np.int32)


def dequant(acc, sx, sw, bias=None, out_dtype="float32"):
    """R:torch_xdna/runtime.py:370-374 / :350-353 / :429-432: (acc.float() * sx) * sw, + bias.float(),
    rounded once to the input dtype. Returned as float32 values of that dtype."""
    y = (np.asarray(acc, dtype=np.int64).astype(F32) * np.asarray(sx, F32)[:, None]) * np.asarray(sw, F32)[None, :]
    if bias is not None:
        y = y + np.asarray(bias, dtype=F32)[None, :]
    return cast(y.astype(F32), out_dtype)


def linear(x, weights, biases=None, transposed=False, x_dtype="float32"):
    """y = cat_i(x @ W_i^T + b_i) through W8A8, exactly as runtime.linear_int8 / linear_cat compute it
    (R:torch_xdna/runtime.py:358-374, :402-434). x, weights in float32 holding values of x_dtype /
    the weights' dtype. Returns (y, acc, sx, sw)."""
    x = np.asarray(x, dtype=F32)
    if not isinstance(weights, (list, tuple)):
        weights, biases = [weights], [biases]
    biases = biases if biases is not None else [None] * len(weights)
    x2 = x.reshape(-1, x.shape[-1])
    ws = [np.asarray(w, F32) for w in weights]
    w = ws[0] if len(ws) == 1 else np.concatenate(ws, axis=0)
    wq, sw = quant_weight(w, transposed)
    xq, sx = quant_rows(x2)
    acc = int_mm(xq, wq)
    bias = None
    if any(b is not None for b in biases):
        sizes = [(wi.shape[1] if transposed else wi.shape[0]) for wi in ws]
        bias = np.concatenate([np.asarray(b, F32) if b is not None else np.zeros(n, F32) for b, n in zip(biases, sizes)])
    y = dequant(acc, sx, sw, bias, x_dtype)
    return y.reshape(*x.shape[:-1], y.shape[-1]), acc, sx, sw


# ---------------------------------------------------------------- conv3x3
def conv_quant(x):
    """Per-image int8 of conv3x3_int8, R:torch_xdna/conv.py:45-46. x [N, C, H, W] f32 -> (xq, sx [N])."""
    x = np.asarray(x, dtype=F32)
    amax = np.abs(x).reshape(x.shape[0], -1).max(axis=1)
    s = (np.maximum(amax, F32(1e-8)) / F32(127)).astype(F32)
    q = np.clip(np.rint(x / s[:, None, None, None]), -127, 127).astype(np.int8)
    return q, s


def conv_weight(w):
    """ConvLayer int8 weights, R:torch_xdna/conv.py:58-60. w [Co, Ci, 3, 3] -> (wq, sw [Co])."""
    w = np.asarray(w, dtype=F32)
    sw = (np.maximum(np.abs(w).reshape(w.shape[0], -1).max(axis=1), F32(1e-8)) / F32(127)).astype(F32)
    wq = np.clip(np.rint(w / sw[:, None, None, None]), -127, 127).astype(np.int8)
    return wq, sw


def conv_acc(xq, wq, stride=1):
    """Exact int32 sums of the conv of the integers, R:torch_xdna/conv.py:86-87 (F.conv2d(xq, wq, padding=1)
    for the reference's 3x3 convs). A [Co, Ci, 1, 1] wq is a 1x1 conv with no padding, and stride 2 takes
    every second output row and column -- F.conv2d(xq, wq, stride, padding=k // 2), the same call applied to
    the 1x1 / stride-2 convs the reference lists as missing (R:results/conv3x3_cascade.md:222-223)."""
    xq = np.asarray(xq, dtype=np.float64)
    wq = np.asarray(wq, dtype=np.float64)
    n, ci, h, w = xq.shape
    co, k = wq.shape[0], wq.shape[-1]
    p = k // 2
    ho, wo = (h + 2 * p - k) // stride + 1, (w + 2 * p - k) // stride + 1
    xp = np.zeros((n, ci, h + 2 * p, w + 2 * p), np.float64)
    xp[:, :, p:p + h, p:p + w] = xq
    acc = np.zeros((n, co, ho, wo), np.float64)
    for ky in range(k):
        for kx in range(k):
            win = xp[:, :, ky:ky + stride * (ho - 1) + 1:stride, kx:kx + stride * (wo - 1) + 1:stride]
            acc += np.einsum("nchw,oc->nohw", win, wq[:, :, ky, kx], optimize=True)
    return acc.astype(np.int64).astype(np.int32)


def calibrate_shift(acc0, relu):
    """ConvLayer.calibrate, R:torch_xdna/conv.py:71-76 (acc0: the sums of the first image)."""
    import math

    acc0 = np.asarray(acc0, dtype=np.int64)
    top = float(np.maximum(acc0, 0).max()) if relu else float(np.abs(acc0).max())
    return min(31, max(1, math.ceil(math.log2(max(top * 1.25, 1.0) / (255 if relu else 127)))))


def requant(acc, shift, relu):
    """ConvLayer.cpu, R:torch_xdna/conv.py:89-92: round half up by an arithmetic shift, saturate."""
    q = (np.asarray(acc, dtype=np.int32) + np.int32(1 << (shift - 1))) >> np.int32(shift)
    return np.clip(q, 0, 255).astype(np.uint8) if relu else np.clip(q, -128, 127).astype(np.int8)


def conv_bias_int32(bias, sw, sx):
    """The optional bias inside the int32 sums (R:results/conv3x3_cascade.md:224-225 names it as future work;
    the reference has no code for it, so this restates the definition the B200 build adopts):
    b[n, co] = rint(bias[co] / (sw[co] * sx[n])) in f32 -- product and quotient correctly rounded, rint to
    nearest even -- clamped to [-2^29, 2^29], NaN -> 0."""
    b = np.asarray(bias, F32)
    t = (np.asarray(sx, F32)[:, None] * np.asarray(sw, F32)[None, :]).astype(F32)
    with np.errstate(all="ignore"):
        v = np.rint((b[None, :] / t).astype(F32))
    lim = F32(2.0 ** 29)
    v = np.where(np.isnan(v), F32(0), np.clip(v, -lim, lim))
    return v.astype(np.int32)


def conv3x3_int8(x, w, bias=None, relu=False, shift=None, x_dtype="float32", stride=1, bias_int32=False):
    """conv3x3_int8 + xdna::conv3x3 on the CPU route, R:torch_xdna/conv.py:43-51,164-189 (and, for a 1x1 w or
    stride 2, the same route on that conv's sums, conv_acc). Returns dict(y, q, scale, shift, xq, sx, wq, sw).
    bias_int32 (a biased conv): the bias joins the sums as conv_bias_int32 before the calibration and the
    requantise, relu is then the ReLU after the bias, and y has no float bias term."""
    xq, sx = conv_quant(x)
    wq, sw = conv_weight(w)
    acc = conv_acc(xq, wq, stride)
    bint = None
    if bias_int32 and bias is not None:
        bint = conv_bias_int32(bias, sw, sx)
        acc = (acc.astype(np.int64) + bint[:, :, None, None]).astype(np.int32)
    if shift is None:
        shift = calibrate_shift(acc[0], relu)
    q = requant(acc, shift, relu)
    scale = (sw * F32(2.0 ** shift)).astype(F32)
    y = q.astype(F32) * (scale[None, :, None, None] * sx[:, None, None, None])
    if bias is not None and bint is None:
        y = y + np.asarray(bias, F32)[None, :, None, None]
    return dict(y=cast(y.astype(F32), x_dtype), q=q, scale=scale, shift=shift, xq=xq, sx=sx, wq=wq, sw=sw, acc=acc,
                bint=bint)


# ---------------------------------------------------------------- Qwen3 stack (fp64)
QWEN3 = dict(D=1024, NH=16, NKV=8, DH=128, INTER=3072, EPS=1e-6, THETA=1e6)


def _rms(x, w, eps):
    var = np.mean(x * x, axis=-1, keepdims=True)
    return (x / np.sqrt(var + eps)) * w


def _silu(x):
    return x / (1.0 + np.exp(-x))


def qwen3_stack(layers, final_norm, head, head_bias, x, mask, theta=1e6, eps=1e-6):
    """The fp32-eager model the reference checks its fused stack against (R:torch_xdna/stack.py:444-460):
    transformers' Qwen3Model decoder layers on inputs_embeds x [B, L, D] under a 4-D bool mask
    [B, 1|H, L, L] (True = may attend), the final RMSNorm and the linear head. Computed in float64.
    Layer math per R:torch_xdna/stack.py:43-57 shapes: pre-norm, fused q/k/v, per-head q/k RMSNorm,
    RoPE (half rotation, positions 0..L-1), GQA softmax attention scaled by head_dim^-0.5,
    o-proj + residual, pre-norm, SwiGLU MLP + residual."""
    D, NH, NKV, DH = QWEN3["D"], QWEN3["NH"], QWEN3["NKV"], QWEN3["DH"]
    h = np.asarray(x, np.float64)
    B, L, _ = h.shape
    mask = np.asarray(mask, bool)
    inv_freq = 1.0 / (theta ** (np.arange(0, DH, 2, dtype=np.float64) / DH))
    pos = np.arange(L, dtype=np.float64)
    freqs = np.outer(pos, inv_freq)
    emb = np.concatenate([freqs, freqs], axis=-1)
    cos, sin = np.cos(emb), np.sin(emb)

    def rope(t):  # t [B, H, L, DH]
        t1, t2 = t[..., :DH // 2], t[..., DH // 2:]
        rot = np.concatenate([-t2, t1], axis=-1)
        return t * cos + rot * sin

    for lw in layers:
        W = {k: np.asarray(v, np.float64) for k, v in lw.items()}
        a = _rms(h, W["input_norm"], eps)
        q = (a @ W["q"].T).reshape(B, L, NH, DH)
        k = (a @ W["k"].T).reshape(B, L, NKV, DH)
        v = (a @ W["v"].T).reshape(B, L, NKV, DH)
        q = _rms(q, W["q_norm"], eps).transpose(0, 2, 1, 3)
        k = _rms(k, W["k_norm"], eps).transpose(0, 2, 1, 3)
        v = v.transpose(0, 2, 1, 3)
        q, k = rope(q), rope(k)
        rep = NH // NKV
        k = np.repeat(k, rep, axis=1)
        v = np.repeat(v, rep, axis=1)
        s = (q @ k.transpose(0, 1, 3, 2)) * (DH ** -0.5)
        s = np.where(mask, s, -np.inf)
        s = s - s.max(axis=-1, keepdims=True)
        p = np.exp(s)
        p = p / p.sum(axis=-1, keepdims=True)
        o = (p @ v).transpose(0, 2, 1, 3).reshape(B, L, NH * DH)
        h = h + o @ W["o"].T
        a = _rms(h, W["post_norm"], eps)
        h = h + (_silu(a @ W["gate"].T) * (a @ W["up"].T)) @ W["down"].T
    h = _rms(h, np.asarray(final_norm, np.float64), eps)
    out = h @ np.asarray(head, np.float64).T
    if head_bias is not None:
        out = out + np.asarray(head_bias, np.float64)
    return out


def mask_lengths(mask):
    """stack.lengths, R:torch_xdna/stack.py:328-352: per-sequence n when the 4-D mask is a prefix block
    (first n positions see exactly those n; later positions see only themselves or nothing), else None."""
    m = np.asarray(mask)
    if m.ndim != 4 or m.shape[-1] != m.shape[-2]:
        return None
    if m.dtype == bool:
        allowed = m
    elif np.issubdtype(m.dtype, np.floating):
        allowed = m == 0
        if not np.all(allowed | (m <= -1e4)):
            return None
    else:
        return None
    if allowed.shape[1] > 1 and not np.all(allowed == allowed[:, :1]):
        return None
    a = allowed[:, 0]
    n = a[:, 0].sum(-1)
    ar = np.arange(a.shape[-1])
    want = ar[None, None, :] < n[:, None, None]
    rows = ar[None, :, None] < n[:, None, None]
    eye = ar[:, None] == ar[None, :]
    pad = (a == eye[None]) | ~a.any(-1, keepdims=True)
    if not np.all(np.where(rows, a == want, pad)):
        return None
    return [int(v) for v in n]
