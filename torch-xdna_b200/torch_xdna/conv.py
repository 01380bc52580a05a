"""xdna::conv3x3: 3x3 / stride-1 / padding-1 convolutions of a parameter weight, int8 on the B200.

The math is the reference's (R:torch_xdna/conv.py:1-19):

  weights     int8 per output channel, quantised once
  activations int8 per image (sx)
  sums        int32 on the int8 tensor cores (implicit GEMM: K = 9 taps x input channels),
              requantised in the epilogue by one shift: round half up, saturate to int8, or to
              [0, 255] with a fused ReLU. The shift is fixed on the layer's first call from the
              first image's sums with 25% headroom (R:torch_xdna/conv.py:71-76).
  output      q * sw[co] * 2^shift * sx (+ bias)

Data layout on the device: activations are quantised straight into a zero-bordered NHWC int8
tensor [N, H+2, W+2, Cp] (Cp = channels rounded up to 16), so each of the 9 taps is a constant row
offset into a [pixels, Cp] matrix that TMA streams into shared memory; weights are packed once as
[Co, 9, Cp]. Three kernels per conv3x3_int8 call: per-image max, quantise + layout, and the
conv with the dequantise (or requantise) in its epilogue.
"""

import logging
import math
import os
import threading
import time
import weakref

import torch

from . import kernels, parallel
from .runtime import DEVICE, XdnaResultMismatch, stats

log = logging.getLogger("torch_xdna")
_lock = threading.RLock()
_layers = {}            # (id(weight), H, W, relu) -> (weakref to weight, ConvLayer)


def supported(ci, co, h, w):
    """Shapes the B200 conv takes: any channel counts and image size (R:torch_xdna/conv.py:38-40 capped
    input channels at 512 for the NPU op; kept here so the pass rewrites the same convs)."""
    return 1 <= ci <= 512 and co >= 1 and h >= 1 and w >= 1


def conv3x3_int8(x, weight, bias, relu: bool, cfg_id: int, post_relu: bool = False):
    """relu?(conv2d(x, weight, bias, padding=1)) through int8: what the backend puts in the graph
    (R:torch_xdna/conv.py:43-51). One custom op: quantise, conv and dequantise run as B200 kernels.
    post_relu: torch.relu of the result, applied in the epilogue after the bias (for biased convs, whose
    ReLU the reference leaves in the graph; same values)."""
    return torch.ops.xdna.conv3x3_fused(x, weight, bias, relu, cfg_id, post_relu)


def conv3x3_strip(cfg, x, weight, bias, relu, post_relu=False, group=None):
    """conv3x3_int8 (R:torch_xdna/conv.py:43-51) of images split into strips of rows over the ranks of
    `group` (parallel.strip_rows): x [N, Ci, rows, W] holds this rank's rows, the result this rank's rows of
    the output -- the same values one GPU computes for the whole images. Each image's max |x| and the
    calibration's max of the sums are combined over the ranks (all-reduce max) and every strip's bordered
    input gets the neighbouring strips' edge rows (parallel.exchange_halo) before the conv."""
    assert not (relu and post_relu), "relu fuses into the requantise, post_relu after the bias: one of them"
    kernels._cuda(x, weight, bias)
    n, ci, rows, w = x.shape
    co = weight.shape[0]
    t0 = time.perf_counter()
    with _lock:
        layer = _layer(weight, rows, w, relu, strips=True)
        xc = x if x.dtype in (torch.float32, torch.bfloat16, torch.float16) else x.float()
        cl = _channels_last(xc)
        xc = xc if cl else xc.contiguous()
        amax = torch.empty((n,), dtype=torch.int32, device=x.device)
        kernels.conv_image_amax(xc, amax)
        parallel.all_max_(amax, group)
        xp = _bordered(n, rows, w, layer.cp, x.device)
        sx = torch.empty((n,), dtype=torch.float32, device=x.device)
        kernels.conv_quant_given_amax(xc, xp, sx, amax, cl)
        parallel.exchange_halo(xp, group)
        stats.launches += 2
        if layer.shift is None:
            layer.calibrate(xp, strips=group if group is not None else True)
        y = layer.dequant(xp, n, sx, bias, x.dtype, post_relu)
    stats.calls[DEVICE] += 1
    stats.seconds[DEVICE] += time.perf_counter() - t0
    stats.macs[DEVICE] += n * co * ci * rows * w * 9
    return y


def conv_ext_int8(x, weight, bias, stride: int, relu: bool, cfg_id: int, post_relu: bool = False):
    """A 1x1 conv (stride 1 or 2) or a stride-2 3x3 conv through int8 (xdna::conv_int8): what the backend
    puts in the graph for the convs Config(conv_ext=True) offloads."""
    return torch.ops.xdna.conv_int8(x, weight, bias, stride, relu, cfg_id, post_relu)


def conv3x3_chain_int8(x, xmeta, weight, bias, relu: bool, cfg_id: int, post_relu: bool, in_mode: int,
                       in_relu_after: bool, out_q: bool, out_pool: bool = False):
    """One conv of a chain whose activations between convs stay int8 (xdna::conv3x3_chain)."""
    return torch.ops.xdna.conv3x3_chain(x, xmeta, weight, bias, relu, cfg_id, post_relu, in_mode, in_relu_after,
                                        out_q, out_pool)


def channels_padded(c):
    return kernels.round_up(c, 16)


class ConvLayer:
    """One conv weight at one input size: int8 weights packed for the implicit GEMM, the shift.
    taps: a layer of <= 7 input channels whose float input is quantised with the stencil's 9 taps packed
    into each pixel's row (conv_quant_taps): its conv is one K block of a single tap instead of nine.
    A [Co, Ci, 1, 1] weight is a 1x1 conv (one tap); stride 2 reads the input's stride phases
    (conv_quant_phases). h, w: the input's size; self.h, self.w: the output's."""

    def __init__(self, weight, h, w, relu, taps=False, stride=1, bint=False):
        kernels._cuda(weight)
        co, ci, k = weight.shape[0], weight.shape[1], weight.shape[-1]
        assert k in (1, 3) and stride in (1, 2) and (k == 3 or not taps) and (stride == 1 or not taps)
        wf = weight.detach()
        if wf.dtype not in (torch.float32, torch.bfloat16, torch.float16):
            wf = wf.float()
        rows = wf.reshape(co, ci * k * k).contiguous()
        self.wq = torch.empty((co, kernels.round_up(ci * k * k, 16)), dtype=torch.int8, device=weight.device)
        self.sw = torch.empty((co,), dtype=torch.float32, device=weight.device)
        kernels.quant_rows(rows, self.wq, self.sw)           # R:torch_xdna/conv.py:58-60
        self.ci, self.co, self.cp, self.k, self.stride = ci, co, channels_padded(ci), k, stride
        wq4 = self.wq[:, :ci * k * k].contiguous().view(co, ci, k, k)
        self.wq4 = wq4
        self.taps = bool(taps) and ci <= 7
        if self.taps:
            # byte (3 ky + kx) C + c of row co = wq[co, c, ky, kx]: the order conv_quant_taps packs the input in
            self.cp = channels_padded(9 * ci)
            self.wp = torch.zeros((co, 1, self.cp), dtype=torch.int8, device=weight.device)
            self.wp[:, 0, :9 * ci] = wq4.permute(0, 2, 3, 1).reshape(co, 9 * ci)
            self.mode_flag, self.ci_k = kernels.CONV_SINGLE_TAP, 9 * ci
        elif k == 1:
            self.wp = torch.zeros((co, 1, self.cp), dtype=torch.int8, device=weight.device)
            self.wp[:, 0, :ci] = wq4[:, :, 0, 0]
            self.mode_flag, self.ci_k = kernels.CONV_SINGLE_TAP, ci
        else:
            self.wp = torch.empty((co, 9, self.cp), dtype=torch.int8, device=weight.device)
            kernels.conv_pack_weight(wq4, self.wp)
            self.mode_flag, self.ci_k = 0, ci
        if stride == 2:
            self.mode_flag |= kernels.CONV_STRIDE2
        self.hi, self.wi = h, w
        self.h, self.w = (h + 1) // 2 if stride == 2 else h, (w + 1) // 2 if stride == 2 else w
        self.relu = relu
        self.bint = bool(bint)  # the bias inside the int32 sums (Config(conv_bias_int32=True))
        self.shift = self.scale = None
        self.checked = False
        kind = "conv3x3" if k == 3 else "conv1x1"
        self.name = (f"{kind}{' stride 2' if stride == 2 else ''} {ci}->{co} {h}x{w}" + (" relu" if relu else "")
                     + (" int32-bias" if bint else ""))

    def quantise(self, xc, n):
        """(xp, sx) of the float input xc [n, Ci, h, w]: the per-image quantise into the layout this layer's
        conv reads (bordered, tap-packed, or the stride-2 phase planes)."""
        sx = torch.empty((n,), dtype=torch.float32, device=xc.device)
        scratch = torch.empty((n,), dtype=torch.int32, device=xc.device)
        if self.stride == 2:
            xp = torch.empty((1 if self.k == 1 else 4, n, self.h + 2, self.w + 2, self.cp), dtype=torch.int8,
                             device=xc.device)
            cl = _channels_last(xc)
            kernels.conv_quant_phases(xc if cl else xc.contiguous(), xp, sx, scratch, cl)
        else:
            xp = _bordered(n, self.h, self.w, self.cp, xc.device)
            _quantise_float(self, xc, xp, sx, scratch)
        stats.launches += 2
        return xp, sx

    def calibrate(self, xp, n=1, strips=None, bint=None):
        """Fix the shift from the first image's integer sums (R:torch_xdna/conv.py:71-76). n: the images in xp
        (a stride-2 input's phase planes are n images apart). strips: the process group over whose ranks the
        image is split into strips of rows; the max of the sums is then the max over every rank's strip.
        bint: the int32 bias [n, Co] (bias_int32), part of the sums the shift must hold."""
        acc_max = torch.empty((1,), dtype=torch.int32, device=xp.device)
        kernels.conv3x3(xp, self.wp, n, self.ci_k, self.co, self.h, self.w,
                        kernels.CONV_CALIBRATE | self.flags(bint), relu=self.relu, bias=bint, acc_max=acc_max)
        stats.launches += 1
        if strips is not None:
            parallel.all_max_(acc_max, None if strips is True else strips)
        top = float(int(acc_max.item()))
        shift = min(31, max(1, math.ceil(math.log2(max(top * 1.25, 1.0) / (255 if self.relu else 127)))))
        # data parallel: every rank adopts the shift of rank 0, which holds global image 0 (strips: every rank
        # computed the same shift from the combined max)
        self.shift = parallel.broadcast_shift(shift, xp.device) if strips is None else shift
        self.scale = self.sw * 2.0 ** self.shift

    def flags(self, bint=None):
        return self.mode_flag | (kernels.CONV_BIAS_INT32 if bint is not None else 0)

    def bias_int32(self, bias, sx):
        """The int32 bias [n, Co] of Config(conv_bias_int32=True): rint(bias / (sw * sx)) per image, the units
        of the integer sums (xdna_conv_bias_int32)."""
        out = torch.empty((sx.numel(), self.co), dtype=torch.int32, device=sx.device)
        kernels.conv_bias_int32(bias, self.sw, sx, out)
        stats.launches += 1
        return out

    def q(self, xp, n, bint=None):
        out = torch.empty((n, self.co, self.h, self.w), dtype=torch.uint8 if self.relu else torch.int8,
                          device=xp.device)
        kernels.conv3x3(xp, self.wp, n, self.ci_k, self.co, self.h, self.w, kernels.CONV_Q | self.flags(bint),
                        shift=self.shift, relu=self.relu, bias=bint, out=out)
        stats.launches += 1
        return out

    def dequant(self, xp, n, sx, bias, dtype, post_relu=False, bint=None):
        # channels-last: the epilogue writes each pixel's channels contiguously (same values and shape as
        # the reference's NCHW tensor; torch ops downstream keep the layout)
        out = torch.empty((n, self.co, self.h, self.w), dtype=dtype, device=xp.device,
                          memory_format=torch.channels_last)
        relu = kernels.RELU_AFTER_BIAS if post_relu else self.relu
        kernels.conv3x3(xp, self.wp, n, self.ci_k, self.co, self.h, self.w, kernels.CONV_DEQUANT | self.flags(bint),
                        shift=self.shift, relu=relu, scale=self.scale, sx=sx, bias=bint if bint is not None else bias,
                        out=out)
        stats.launches += 1
        return out

    def cpu_integers(self, xq_nchw_cpu, bint=None):
        """The reference's CPU integers for the same layer and shift (ConvLayer.cpu,
        R:torch_xdna/conv.py:86-92), used only to verify launches; with bint [N, Co], added to the sums
        before the shift."""
        dt = torch.float32 if 127 * float(self.wq4.abs().sum(dim=(1, 2, 3)).max()) < 2 ** 24 else torch.float64
        acc = torch.nn.functional.conv2d(xq_nchw_cpu.to(dt), self.wq4.cpu().to(dt), stride=self.stride,
                                         padding=self.k // 2).to(torch.int32)
        if bint is not None:
            acc = acc + bint.cpu()[:, :, None, None]
        q = (acc + (1 << (self.shift - 1))) >> self.shift
        return q.clamp_(0, 255).to(torch.uint8) if self.relu else q.clamp_(-128, 127).to(torch.int8)


def _layer(weight, h, w, relu, taps=False, stride=1, strips=False, bint=False):
    # strips: a layer of a strip-split image keeps its own (combined) shift, apart from a same-size whole image;
    # bint: the int32-bias route calibrates on the sums with the bias in them
    key = (id(weight), h, w, relu, bool(taps), stride, strips, bool(bint))
    hit = _layers.get(key)
    if hit is not None and hit[0]() is weight:
        return hit[1]
    layer = ConvLayer(weight, h, w, relu, taps, stride, bint)
    _layers[key] = (weakref.ref(weight), layer)
    return layer


def _channels_last(t):
    """True when t [N, C, H, W] is stored channels-last and not also plain contiguous."""
    return (t.is_contiguous(memory_format=torch.channels_last) and not t.is_contiguous()
            and t.data_ptr() % 16 == 0)


def _quantise_float(layer, xc, xp, sx, scratch):
    """The per-image quantise of a float input into layer's bordered layout: taps packed for a layer of
    few channels, a streaming pass for a channels-last input (e.g. the previous conv's output), else the
    NCHW transpose."""
    if layer.taps:
        kernels.conv_quant_taps(xc.contiguous(), xp, sx, scratch)
    elif _channels_last(xc):
        kernels.conv_quant_channels_last(xc, xp, sx, scratch)
    else:
        kernels.conv_quant(xc.contiguous(), xp, sx, scratch)


def _bordered(n, h, w, cp, device):
    return torch.empty((n, h + 2, w + 2, cp), dtype=torch.int8, device=device)


def int32_bias(cfg, bias):
    """Whether this conv adds its bias inside the int32 sums (Config(conv_bias_int32=True), biased convs)."""
    return bool(getattr(cfg, "conv_bias_int32", False)) and bias is not None


def effective_relu(cfg, relu, bias, post_relu):
    """(ReLU fused into the requantise, ReLU after the float bias) of a conv: with the bias inside the int32
    sums, a ReLU after the bias is the requantise's [0, 255] saturation."""
    if int32_bias(cfg, bias):
        return bool(relu or post_relu), False
    return relu, post_relu


def _verify(cfg, layer, xp, xq_cpu_fn, n=None, bint=None):
    if cfg.verify == "off" or (cfg.verify == "first" and layer.checked):
        return
    n = xp.shape[0] if n is None else n
    got = layer.q(xp, n, bint).cpu()
    want = layer.cpu_integers(xq_cpu_fn(), bint)
    if not torch.equal(got, want):
        raise XdnaResultMismatch(f"{layer.name} disagrees with the CPU integers: "
                                 f"{int((got != want).sum())} of {want.numel()} values differ")
    layer.checked = True
    stats.checks.append((layer.name, "bitwise equal to the CPU integers"))


def conv3x3(cfg, xq, weight, relu):
    """(q, scale) of xdna::conv3x3 for int8 xq [N, Ci, H, W] (R:torch_xdna/conv.py:164-189)."""
    kernels._cuda(xq, weight)
    n, ci, h, w = xq.shape
    co = weight.shape[0]
    t0 = time.perf_counter()
    with _lock:
        layer = _layer(weight, h, w, relu)
        xp = _bordered(n, h, w, layer.cp, xq.device)
        kernels.conv_pack_input(xq.contiguous(), xp)
        stats.launches += 1
        if layer.shift is None:
            layer.calibrate(xp)
        _verify(cfg, layer, xp, lambda: xq.cpu())
        q = layer.q(xp, n)
    stats.calls[DEVICE] += 1
    stats.seconds[DEVICE] += time.perf_counter() - t0
    stats.macs[DEVICE] += n * co * ci * h * w * 9
    # a fresh tensor: Inductor may reuse an extern op's output buffer once it is dead
    return q, layer.scale.clone()


def conv3x3_fused(cfg, x, weight, bias, relu, post_relu=False):
    """conv3x3_int8 in three kernels: per-image max, quantise into the bordered NHWC layout, and the
    conv whose epilogue requantises and dequantises (q * (scale * sx) + bias, then max(., 0) when
    post_relu) straight to x.dtype."""
    assert not (relu and post_relu), "relu fuses into the requantise, post_relu after the bias: one of them"
    kernels._cuda(x, weight, bias)
    n, ci, h, w = x.shape
    co = weight.shape[0]
    bint_mode = int32_bias(cfg, bias)
    relu, post_relu = effective_relu(cfg, relu, bias, post_relu)
    t0 = time.perf_counter()
    with _lock:
        layer = _layer(weight, h, w, relu, taps=ci <= 7, bint=bint_mode)
        xc = x if x.dtype in (torch.float32, torch.bfloat16, torch.float16) else x.float()
        xp = _bordered(n, h, w, layer.cp, x.device)
        sx = torch.empty((n,), dtype=torch.float32, device=x.device)
        scratch = torch.empty((n,), dtype=torch.int32, device=x.device)
        _quantise_float(layer, xc, xp, sx, scratch)
        stats.launches += 2
        bint = layer.bias_int32(bias, sx) if bint_mode else None
        if layer.shift is None:
            layer.calibrate(xp, bint=bint)

        def xq_cpu():
            xf = xc.float().cpu()
            s = xf.abs().amax(dim=(1, 2, 3), keepdim=True).clamp(min=1e-8) / 127
            return torch.round(xf / s).clamp(-127, 127).to(torch.int8)

        _verify(cfg, layer, xp, xq_cpu, bint=bint)
        y = layer.dequant(xp, n, sx, bias, x.dtype, post_relu, bint)
    stats.calls[DEVICE] += 1
    stats.seconds[DEVICE] += time.perf_counter() - t0
    stats.macs[DEVICE] += n * co * ci * h * w * 9
    return y


def conv_int8(cfg, x, weight, bias, stride, relu, post_relu=False):
    """The reference's conv route (R:torch_xdna/conv.py:43-51: per-image quantise, int8 weights per output
    channel, exact int32 sums, the 25 %-headroom shift fixed from image 0, requantise, dequantise + bias)
    applied to the ResNet-style convs the reference lists as missing (R:results/conv3x3_cascade.md:222-223):
    a 1x1 conv (stride 1 or 2, no padding) or a 3x3 conv with stride 2 and padding 1. The integer sums are
    those of F.conv2d on the integers with the conv's own stride and padding (ConvLayer.cpu_integers).
    Output channels-last, x.dtype; post_relu as conv3x3_fused."""
    assert not (relu and post_relu), "relu fuses into the requantise, post_relu after the bias: one of them"
    kernels._cuda(x, weight, bias)
    k = weight.shape[-1]
    if k == 3 and stride == 1:
        return conv3x3_fused(cfg, x, weight, bias, relu, post_relu)
    n, ci, h, w = x.shape
    co = weight.shape[0]
    bint_mode = int32_bias(cfg, bias)
    relu, post_relu = effective_relu(cfg, relu, bias, post_relu)
    t0 = time.perf_counter()
    with _lock:
        layer = _layer(weight, h, w, relu, stride=stride, bint=bint_mode)
        xc = x if x.dtype in (torch.float32, torch.bfloat16, torch.float16) else x.float()
        xp, sx = layer.quantise(xc, n)
        bint = layer.bias_int32(bias, sx) if bint_mode else None
        if layer.shift is None:
            layer.calibrate(xp, n, bint=bint)

        def xq_cpu():
            xf = xc.float().cpu()
            s = xf.abs().amax(dim=(1, 2, 3), keepdim=True).clamp(min=1e-8) / 127
            return torch.round(xf / s).clamp(-127, 127).to(torch.int8)

        _verify(cfg, layer, xp, xq_cpu, n, bint=bint)
        y = layer.dequant(xp, n, sx, bias, x.dtype, post_relu, bint)
    stats.calls[DEVICE] += 1
    stats.seconds[DEVICE] += time.perf_counter() - t0
    stats.macs[DEVICE] += n * co * ci * layer.h * layer.w * k * k
    return y


# int8 chaining: IN_FLOAT takes a float input; IN_CODES / IN_CODES_POOL take the previous conv's codes
IN_FLOAT, IN_CODES, IN_CODES_POOL = 0, 1, 2


def codes_meta(sx, scale, bias, co, amax=False, pool=False):
    """The float data that turns a conv's codes back into its output: sx [N], scale [Co], bias [Co]; with
    amax, N more words for the next layer's per-image maxima (bit patterns, written by the producing conv's
    epilogue), and one word more when they cover a 2x2 pool's region -- the consumer reads which from the
    length alone, so it needs no device read."""
    b = bias.float() if bias is not None else torch.zeros((co,), dtype=torch.float32, device=scale.device)
    parts = [sx, scale, b]
    if amax:
        parts.append(torch.empty((sx.numel() + (1 if pool else 0),), dtype=torch.float32, device=sx.device))
    return torch.cat(parts)


def next_amax_ok(relu, bias, post_relu, pool):
    """Whether a chain producer can compute the next layer's per-image maxima in its epilogue: always without
    a pool; with a 2x2 max-pool only for non-negative values (the pooled image's max is then the max over the
    pool's region), i.e. a ReLU after the bias, or a ReLU fused into a bias-free conv's requantise."""
    return (not pool) or bool(post_relu) or (bool(relu) and bias is None)


def codes_to_float(q, meta, relu_after, pool):
    """The float activation a chain's codes stand for, on the CPU with torch's f32 ops in the epilogue's
    order (float(q) * (scale * sx) + bias, max(., 0), 2x2 max-pool), NCHW: the reference's own tensor."""
    n, h, w, c = q.shape
    m = meta.cpu()
    sx, scale, bias = m[:n], m[n:n + c], m[n + c:n + 2 * c]
    t = scale[None, :] * sx[:, None]                                  # [N, C], rounded as scale * sx
    y = q.cpu().to(torch.int32).float() * t[:, None, None, :] + bias  # NHWC
    if relu_after:
        y = torch.relu(y)
    y = y.permute(0, 3, 1, 2)
    return torch.nn.functional.max_pool2d(y, 2) if pool else y


def conv3x3_chain(cfg, x, xmeta, weight, bias, relu, post_relu, in_mode, in_relu_after, out_q, out_pool=False):
    """A conv of a chain (R:torch_xdna/conv.py:43-51 applied layer after layer, with the graph's ReLU and
    2x2 max-pool between): the activations between convs stay int8 codes [N, H, W, C] with their float
    factors, and the next conv's quantise rebuilds the float values the reference would have (same f32
    operations), pools them on the codes (exact: the value grows with the code) and quantises per image.
    x: the float input [N, Ci, H, W] (IN_FLOAT), or the previous conv's codes [N, H, W, Ci] with
    xmeta = codes_meta(...) (IN_CODES; IN_CODES_POOL: 2x2 max-pooled first). in_relu_after: the previous
    conv's ReLU applies after its bias. Returns (codes [N, H, W, Co], their meta) when out_q, else (the
    float output [N, Co, H, W] channels-last, an empty tensor). out_pool: the next conv pools these codes
    first; with out_q the epilogue then also writes the next layer's per-image maxima (over the pool's
    region), so the next quantise makes one pass over the codes instead of two."""
    assert not (relu and post_relu), "relu fuses into the requantise, post_relu after the bias: one of them"
    kernels._cuda(x, xmeta, weight, bias)
    if in_mode == IN_FLOAT:
        n, ci, h, w = x.shape
    else:
        n, hq, wq, ci = x.shape
        h, w = (hq // 2, wq // 2) if in_mode == IN_CODES_POOL else (hq, wq)
    co = weight.shape[0]
    bint_mode = int32_bias(cfg, bias)
    relu, post_relu = effective_relu(cfg, relu, bias, post_relu)
    fbias = None if bint_mode else bias   # the bias added to the floats (none when it is in the sums)
    t0 = time.perf_counter()
    with _lock:
        layer = _layer(weight, h, w, relu, taps=in_mode == IN_FLOAT and ci <= 7, bint=bint_mode)
        # image pairs (XDNA_CONV_PAIRS): a 64-channel input from codes, written two images per 128-byte row (they
        # read through the window loads, which XDNA_CONV_WINDOW=0 turns off for comparisons)
        pairs = (in_mode != IN_FLOAT and out_q and ci == 64 and layer.cp == 64 and n % 2 == 0 and co <= 128
                 and os.environ.get("XDNA_CONV_WINDOW", "1") != "0")
        xp = None if pairs else _bordered(n, h, w, layer.cp, x.device)
        sx = torch.empty((n,), dtype=torch.float32, device=x.device)
        scratch = torch.empty((n,), dtype=torch.int32, device=x.device)
        if pairs:
            xq = x.contiguous()
            in_pool = in_mode == IN_CODES_POOL
            xp2 = torch.empty((n // 2, h + 2, w + 2, 128), dtype=torch.int8, device=x.device)
            given = xmeta.numel() == 2 * n + 2 * ci + (1 if in_pool else 0)
            kernels.conv_quant_codes_pairs(xq, xmeta[n:n + ci], xmeta[:n], xmeta[n + ci:n + 2 * ci], in_relu_after,
                                           in_pool, xp2, sx,
                                           xmeta[n + 2 * ci:2 * n + 2 * ci].view(torch.int32) if given else scratch,
                                           given)
            float_in = lambda: codes_to_float(xq, xmeta, in_relu_after, in_pool)  # noqa: E731
            if layer.shift is None or (cfg.verify != "off" and not (cfg.verify == "first" and layer.checked)):
                # the plain layout, for the calibration and the CPU check (first calls)
                xp = xp2.view(n // 2, h + 2, w + 2, 2, 64).permute(0, 3, 1, 2, 4).reshape(n, h + 2, w + 2, 64)
        elif in_mode == IN_FLOAT:
            xc = x if x.dtype in (torch.float32, torch.bfloat16, torch.float16) else x.float()
            _quantise_float(layer, xc, xp, sx, scratch)
            float_in = lambda: xc.float().cpu()  # noqa: E731
        else:
            xq = x.contiguous()
            in_pool = in_mode == IN_CODES_POOL
            if xmeta.numel() == 2 * n + 2 * ci + (1 if in_pool else 0):   # maxima from the producing conv
                kernels.conv_quant_codes_given_amax(xq, xmeta[n:n + ci], xmeta[:n], xmeta[n + ci:n + 2 * ci],
                                                    in_relu_after, in_pool, xp, sx,
                                                    xmeta[n + 2 * ci:2 * n + 2 * ci].view(torch.int32))
            else:
                kernels.conv_quant_codes(xq, xmeta[n:n + ci], xmeta[:n], xmeta[n + ci:n + 2 * ci], in_relu_after,
                                         in_pool, xp, sx, scratch)
            float_in = lambda: codes_to_float(xq, xmeta, in_relu_after, in_mode == IN_CODES_POOL)  # noqa: E731
        stats.launches += 1 if pairs else 2
        bint = layer.bias_int32(bias, sx) if bint_mode else None
        if layer.shift is None:
            layer.calibrate(xp, bint=bint)

        def xq_cpu():
            xf = float_in()
            s = xf.abs().amax(dim=(1, 2, 3), keepdim=True).clamp(min=1e-8) / 127
            return torch.round(xf / s).clamp(-127, 127).to(torch.int8)

        _verify(cfg, layer, xp, xq_cpu, bint=bint)
        if out_q:
            q = torch.empty((n, h, w, co), dtype=torch.uint8 if relu else torch.int8, device=x.device)
            if next_amax_ok(relu, fbias, post_relu, out_pool):
                meta = codes_meta(sx, layer.scale, fbias, co, amax=True, pool=out_pool)
                mode = (kernels.CONV_Q_NHWC | layer.flags(bint) | kernels.CONV_NEXT_AMAX
                        | (kernels.CONV_NEXT_RELU if post_relu else 0) | (kernels.CONV_NEXT_POOL if out_pool else 0)
                        | (kernels.CONV_PAIRS if pairs else 0))
                kb = bint if bint is not None else (meta[n + co:n + 2 * co] if bias is not None else None)
                kernels.conv3x3(xp2 if pairs else xp, layer.wp, n, layer.ci_k, co, h, w, mode, shift=layer.shift,
                                relu=relu,
                                scale=meta[n:n + co], sx=sx, bias=kb, out=q,
                                acc_max=meta[n + 2 * co:2 * n + 2 * co].view(torch.int32))
                out = (q, meta)
            else:
                kernels.conv3x3(xp2 if pairs else xp, layer.wp, n, layer.ci_k, co, h, w,
                                kernels.CONV_Q_NHWC | layer.flags(bint) | (kernels.CONV_PAIRS if pairs else 0),
                                shift=layer.shift, relu=relu, bias=bint, out=q)
                out = (q, codes_meta(sx, layer.scale, fbias, co))
            stats.launches += 1
        else:
            dtype = x.dtype if in_mode == IN_FLOAT else torch.float32
            out = (layer.dequant(xp, n, sx, bias, dtype, post_relu, bint), sx.new_empty((0,)))
    stats.calls[DEVICE] += 1
    stats.seconds[DEVICE] += time.perf_counter() - t0
    stats.macs[DEVICE] += n * co * ci * h * w * 9
    return out
