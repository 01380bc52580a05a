"""Runtime of the xdna::linear ops on the B200: weight cache, the W8A8 launches, verification, stats.

Every offloaded GEMM is W8A8 as in the reference (R:torch_xdna/runtime.py:1-7): weights int8 per
output channel, activations int8 per row, int8 x int8 -> int32 on the tensor cores, dequantised in
fp32. A call is two kernels of libxdna_b200.so:

  quant_rows   x [R, K] -> xq [R, K16] int8 + sx [R]          (HBM-bound, one pass over x)
  gemm_i8      tcgen05 int8 GEMM; its epilogue computes (float(acc) * sx) * sw (+ bias) and writes
               the input dtype -- the reference's dequantise, in its operation order, never leaving
               registers.

There is no CPU route: "verify" compares a launch with the CPU integers (torch._int_mm, the
reference's own CPU kernel) and raises XdnaResultMismatch on any difference.
"""

import logging
import threading
import time
import weakref
from collections import defaultdict

import torch

from . import kernels

log = logging.getLogger("torch_xdna")
_lock = threading.RLock()

DEVICE = "gpu"  # the device name stats use for B200 work


# ------------------------------------------------------------------ stats
class Stats:
    """Where the offloaded work went (R:torch_xdna/runtime.py:24-48)."""

    def __init__(self):
        self.reset()

    def reset(self):
        self.calls = defaultdict(int)       # device -> op calls (GEMMs, convs, stacks)
        self.seconds = defaultdict(float)   # device -> host seconds inside the op (enqueue time; launches are async)
        self.macs = defaultdict(int)        # device -> multiply-accumulates
        self.launches = 0                   # kernel launches of libxdna_b200
        self.fallbacks = []                 # (what, error) of ops that raised (the build never falls back)
        self.stacks = defaultdict(int)      # (stack, "gpu" fused / "plain" graph) -> graph calls
        self.checks = []                    # (what, result) of verification

    def as_dict(self):
        return dict(calls=dict(self.calls), seconds={k: round(v, 4) for k, v in self.seconds.items()},
                    gmacs={k: round(v / 1e9, 3) for k, v in self.macs.items()},
                    gpu_launches=self.launches, npu_launches=self.launches, fallbacks=list(self.fallbacks),
                    stacks={f"{k[0]} on {k[1]}": v for k, v in self.stacks.items()}, checks=list(self.checks),
                    decisions={}, gpu_available=kernels.available(), npu_available=kernels.available(),
                    gpu_unavailable_reason=kernels.unavailable_reason(),
                    npu_unavailable_reason=kernels.unavailable_reason(), device=kernels.device_name())


stats = Stats()


class XdnaResultMismatch(RuntimeError):
    """A kernel returned something the CPU integers (or the fp32 model) disagree with."""


NPUResultMismatch = XdnaResultMismatch  # the reference's name for the same failure


def _account(t0, rows, n, k, launches):
    stats.calls[DEVICE] += 1
    stats.seconds[DEVICE] += time.perf_counter() - t0
    stats.macs[DEVICE] += rows * n * k
    stats.launches += launches


# ------------------------------------------------------------------ weights
class QWeight:
    """One weight (or several concatenated on the output dim), quantised once on the B200:
    wq [N, K16] int8 (K-major, rows padded to 16 bytes for TMA), sw [N] f32 per output channel
    (R:torch_xdna/runtime.py:56-69)."""

    def __init__(self, w: torch.Tensor, transposed: bool):
        kernels._cuda(w)
        wf = w.detach()
        if transposed:          # given as [K, N] (x @ W): per output channel = per column
            wf = wf.t()
        if wf.dtype not in (torch.float32, torch.bfloat16, torch.float16):
            wf = wf.float()
        wf = wf.contiguous()
        self.N, self.K = wf.shape
        self.K16 = kernels.round_up(max(self.K, 1), 16)
        self.wq = torch.zeros((self.N, self.K16), dtype=torch.int8, device=wf.device)
        self.sw = torch.empty((self.N,), dtype=torch.float32, device=wf.device)
        if self.N and self.K:
            kernels.quant_rows(wf, self.wq, self.sw)
        else:
            self.sw.fill_(1e-8 / 127)
        self.w_fp = wf          # [N, K] in the weight's own dtype (precision "bf16")
        self._w_bf16 = None

    def bf16(self):
        if self._w_bf16 is None:
            w = self.w_fp.to(torch.bfloat16)
            K8 = kernels.round_up(max(self.K, 1), 8)
            if K8 != self.K:
                w = torch.nn.functional.pad(w, (0, K8 - self.K))
            self._w_bf16 = w.contiguous()
        return self._w_bf16


_weights = {}  # key -> (weakrefs to the source tensors, QWeight)


def _ref(t):
    try:
        return weakref.ref(t)
    except TypeError:
        return lambda: t


def qweight(ws, transposed: bool = False) -> QWeight:
    """The cached QWeight of one weight, or of several concatenated (fused linears); keyed like the
    reference by (data_ptr, shape, _version) and validated through weak references
    (R:torch_xdna/runtime.py:99-110)."""
    ws = list(ws) if isinstance(ws, (list, tuple)) else [ws]
    key = (tuple((w.data_ptr(), tuple(w.shape), w._version) for w in ws), transposed)
    with _lock:
        hit = _weights.get(key)
        if hit is not None and all(r() is w for r, w in zip(hit[0], ws)):
            return hit[1]
        src = ws[0] if len(ws) == 1 else torch.cat([w.detach() for w in ws])
        qw = QWeight(src, transposed)
        _weights[key] = ([_ref(w) for w in ws], qw)
        return qw


_biases = {}  # concatenated biases of fused linears


def _cat_bias(weights, biases):
    if not any(b is not None for b in biases):
        return None
    if len(biases) == 1:
        return biases[0]
    key = tuple((b.data_ptr(), b._version) if b is not None else (None, w.shape[0]) for w, b in zip(weights, biases))
    with _lock:
        hit = _biases.get(key)
        if hit is not None and all(r() is b for r, b in zip(hit[0], biases) if b is not None):
            return hit[1]
        dt = next(b.dtype for b in biases if b is not None)
        cat = torch.cat([b.to(dt) if b is not None else w.new_zeros(w.shape[0], dtype=dt)
                         for w, b in zip(weights, biases)])
        _biases[key] = ([_ref(b) for b in biases if b is not None], cat)
        return cat


# ------------------------------------------------------------------ verification
_verified = set()


def _bn_for(rows, n):
    """The kernel configuration libxdna_b200 launches for a GEMM, as the library reports it
    (xdna_gemm_i8_config), for verify keys: the tile width, and "pair" when 256 x 256 tiles run on CTA
    pairs. A new configuration is verified on its first launch."""
    tile_n, pair = kernels.gemm_i8_config(rows, n)
    return f"{tile_n} pair" if pair else tile_n


def _want_check(cfg, key):
    if cfg.verify == "off":
        return False
    return cfg.verify == "always" or key not in _verified


def _check_linear(cfg, key, x2d, xq, sx, qw, bias, y):
    """The launch vs the reference's CPU arithmetic (torch._int_mm + the dequantise ops), bit for bit."""
    xc = x2d.detach().float().cpu()
    s_ref = xc.abs().amax(dim=1, keepdim=True).clamp(min=1e-8) / 127
    xq_ref = torch.round(xc / s_ref).clamp(-127, 127).to(torch.int8)
    K = qw.K
    got_xq = xq[:, :K].cpu()
    if not torch.equal(got_xq, xq_ref) or not torch.equal(sx.cpu().view(-1, 1), s_ref):
        raise XdnaResultMismatch(f"quant_rows {key} disagrees with the CPU: "
                                 f"{int((got_xq != xq_ref).sum())} of {xq_ref.numel()} values differ")
    acc = torch._int_mm(xq_ref, qw.wq[:, :K].cpu().t().contiguous())
    if y.dtype == torch.int32:
        want = acc
    else:
        want = acc.float() * s_ref * qw.sw.cpu()[None, :]
        if bias is not None:
            want = want + bias.float().cpu()
        want = want.to(y.dtype)
    got = y.cpu()
    if not torch.equal(got, want):
        raise XdnaResultMismatch(f"gemm_i8 {key} disagrees with the CPU: "
                                 f"{int((got != want).sum())} of {want.numel()} values differ")
    _verified.add(key)
    stats.checks.append((f"gemm_i8 {key}", "bitwise equal to the CPU integers"))


# ------------------------------------------------------------------ the ops
def _quant(x2d):
    R, K = x2d.shape
    if x2d.stride(-1) != 1 or x2d.dtype not in (torch.float32, torch.bfloat16, torch.float16):
        x2d = x2d.contiguous() if x2d.dtype in (torch.float32, torch.bfloat16, torch.float16) else x2d.float()
    xq = torch.empty((R, kernels.round_up(max(K, 1), 16)), dtype=torch.int8, device=x2d.device)
    sx = torch.empty((R,), dtype=torch.float32, device=x2d.device)
    kernels.quant_rows(x2d, xq, sx)
    return xq, sx, x2d


def _w8a8(cfg, x2d, qw, bias, out_dtype):
    """y [R, N] in out_dtype through quant_rows + gemm_i8 (dequantising epilogue)."""
    xq, sx, x2d = _quant(x2d)
    y = torch.empty((x2d.shape[0], qw.N), dtype=out_dtype, device=x2d.device)
    kernels.gemm_i8(xq, qw.wq, qw.K, y, sx, qw.sw, bias)
    key = ("w8a8", qw.N, qw.K, str(out_dtype), bias is not None, _bn_for(x2d.shape[0], qw.N),
           x2d.shape[0] % 128 != 0)
    if _want_check(cfg, key):
        _check_linear(cfg, key, x2d, xq, sx, qw, bias, y)
    return y


def _bf16(cfg, x2d, qw, bias, out_dtype):
    """y [R, N] = x @ W^T (+ bias) with bf16 operands and f32 accumulation on the bf16 tensor cores: one
    gemm_bf16 whose epilogue adds the bias in f32 and rounds once to out_dtype. The reference runs the
    same product on the NPU (bfp16 MACs) and adds bias.float() on the host (R:torch_xdna/runtime.py:218-237,
    :299-313, :340-345)."""
    R, K = x2d.shape
    w = qw.bf16()                                       # [N, K8] bf16, K zero-padded to 8
    K8 = w.shape[1]
    if (x2d.dtype == torch.bfloat16 and K == K8 and x2d.stride(1) == 1 and x2d.stride(0) % 8 == 0
            and x2d.data_ptr() % 16 == 0):
        a = x2d
    else:                                               # TMA wants 16-byte rows: stage a padded bf16 copy
        a = torch.zeros((R, K8), dtype=torch.bfloat16, device=x2d.device)
        a[:, :K].copy_(x2d)
    per16 = 16 // torch.empty((), dtype=out_dtype).element_size()
    Np = kernels.round_up(qw.N, per16)
    y = torch.empty((R, Np), dtype=out_dtype, device=x2d.device)
    kernels.gemm_bf16(a, w, kernels.GEMM_F32ACC, out=y, bias=bias)
    if Np != qw.N:
        y = y[:, :qw.N].contiguous()
    key = ("bf16", qw.N, qw.K, str(out_dtype), bias is not None, R % 128 != 0)
    if _want_check(cfg, key):
        _check_bf16(key, a, w, bias, y)
    return y


def _check_bf16(key, a, w, bias, y):
    """The launch vs the f32 product of the same bf16 operands, with the reference's tolerance for its
    bf16 route (norm-relative error below 5e-2, all finite; R:torch_xdna/runtime.py:174-188)."""
    want = a.float().cpu() @ w.float().cpu().t()
    if bias is not None:
        want = want + bias.float().cpu()
    got = y.float().cpu()
    err = float((got - want).norm() / want.norm().clamp(min=1e-30))
    if not bool(torch.isfinite(got).all()) or err >= 5e-2:
        raise XdnaResultMismatch(f"gemm_bf16 {key} disagrees with the f32 product: rel err {err:.3g}")
    _verified.add(key)
    stats.checks.append((f"gemm_bf16 {key}", f"rel err {err:.2e} vs the f32 product of the bf16 operands"))


def linear(cfg, x, weight, bias, transposed):
    """y = x @ W^T + b (or x @ W when transposed) through W8A8 on the B200 (R:torch_xdna/runtime.py:326-355)."""
    shape = x.shape[:-1]
    K = x.shape[-1]
    N = weight.shape[1] if transposed else weight.shape[0]
    x2d = x.reshape(-1, K)
    if x2d.shape[0] == 0:
        return x.new_zeros(*shape, N)
    t0 = time.perf_counter()
    qw = qweight(weight, transposed)
    fn = _bf16 if cfg.precision == "bf16" else _w8a8
    y = fn(cfg, x2d, qw, bias, x.dtype)
    _account(t0, x2d.shape[0], qw.N, qw.K, 2)
    return y.reshape(*shape, N)


def linear_cat(cfg, x, weights, biases):
    """torch.cat([F.linear(x, w, b) ...], -1) as one W8A8 GEMM (R:torch_xdna/runtime.py:402-434)."""
    shape = x.shape[:-1]
    N = sum(w.shape[0] for w in weights)
    x2d = x.reshape(-1, x.shape[-1])
    if x2d.shape[0] == 0:
        return x.new_zeros(*shape, N)
    t0 = time.perf_counter()
    qw = qweight(list(weights))
    bias = _cat_bias(list(weights), list(biases))
    fn = _bf16 if cfg.precision == "bf16" else _w8a8
    y = fn(cfg, x2d, qw, bias, x.dtype)
    _account(t0, x2d.shape[0], qw.N, qw.K, 2)
    return y.reshape(*shape, N)


def linear_i8(cfg, xq, weights, transposed):
    """(int32 acc [R, N], weight scales [N]) of xdna::linear_i8 (R:torch_xdna/runtime.py:377-399)."""
    t0 = time.perf_counter()
    qw = qweight(weights[0] if len(weights) == 1 else list(weights), transposed)
    R, K = xq.shape
    assert K == qw.K, f"xq has {K} columns, the weights {qw.K}"
    if R == 0:
        return xq.new_zeros((0, qw.N), dtype=torch.int32), qw.sw.clone()
    kernels._cuda(xq)
    K16 = kernels.round_up(max(K, 1), 16)
    if xq.stride(-1) != 1 or xq.stride(0) % 16 or K16 != K or xq.data_ptr() % 16:
        staged = torch.zeros((R, K16), dtype=torch.int8, device=xq.device)
        staged[:, :K].copy_(xq)
    else:
        staged = xq
    acc = torch.empty((R, qw.N), dtype=torch.int32, device=xq.device)
    kernels.gemm_i8(staged, qw.wq, K, acc)
    key = ("i8", qw.N, qw.K, _bn_for(R, qw.N), R % 128 != 0)
    if _want_check(cfg, key):
        want = torch._int_mm(xq.cpu(), qw.wq[:, :K].cpu().t().contiguous())
        got = acc.cpu()
        if not torch.equal(got, want):
            raise XdnaResultMismatch(f"gemm_i8 {key} disagrees with the CPU: {int((got != want).sum())} values differ")
        _verified.add(key)
        stats.checks.append((f"gemm_i8 {key}", "bitwise equal to the CPU integers"))
    _account(t0, R, qw.N, qw.K, 1)
    # fresh tensors: Inductor may reuse an extern op's output buffer once it is dead
    return acc, qw.sw.clone()


def linear_int8(x, weights, biases, transposed: bool, cfg_id: int):
    """torch.cat([F.linear(x, w, b) ...], -1) through W8A8 (R:torch_xdna/runtime.py:358-374).

    The reference spells quantise / xdna::linear_i8 / dequantise as graph ops for Inductor to fuse on
    the CPU. On the B200 the quantise is its own kernel and the dequantise is the GEMM's epilogue, so
    this is the fused op; the result is bitwise the same.
    """
    if len(weights) == 1:
        return torch.ops.xdna.linear(x, weights[0], biases[0], transposed, cfg_id)
    assert not transposed, "fused linears are never transposed"
    return torch.ops.xdna.linear_cat(x, list(weights), list(biases), cfg_id)
