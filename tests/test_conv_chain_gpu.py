"""int8 chaining between convs (xdna::conv3x3_chain): the activations between convs stay int8 codes and
the next conv's quantise rebuilds the float values. The results must be bit-identical to running the
same convs one by one with conv3x3_fused and torch's max-pool in between, which the conv tests pin to
the oracle and to the reference's goldens."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _inference():
    with torch.no_grad():
        yield


def _cid(**kw):
    import torch_xdna

    return torch_xdna.ops.config_id(torch_xdna.Config(**kw))


def _weights(dev, g, shapes, biased):
    out = []
    for (co, ci), b in zip(shapes, biased):
        w = torch.nn.Parameter(torch.randn(co, ci, 3, 3, device=dev, generator=g) * (2.0 / (ci * 9)) ** 0.5)
        out.append((w, (torch.randn(co, device=dev, generator=g) * 0.05) if b else None))
    return out


# (channels per conv, bias per conv, pool before conv i, H, W, images)
CASES = [
    ([(64, 3), (64, 64), (128, 64), (128, 128)], [True, True, True, False], [False, False, True, False], 32, 48, 3),
    # odd sizes: the pool rounds down (15 x 17 -> 7 x 8); 20 channels: scalar stores of the codes
    ([(20, 8), (32, 20), (16, 32)], [True, False, True], [False, True, False], 15, 17, 3),
    # an even batch: the 64-channel convs read their input in image pairs (XDNA_CONV_PAIRS), pooled or not
    ([(64, 3), (64, 64), (128, 64), (64, 128), (64, 64)], [True, True, True, False, True],
     [False, False, True, False, True], 30, 26, 4),
    # ~420 tiles of the first conv (taps packed, codes out) over 148 SMs: two or three per CTA, so both of
    # its epilogue warp groups drain tiles, unevenly, and images change inside a CTA's range
    ([(64, 3), (64, 64)], [True, True], [False, False], 80, 80, 8),
]


@pytest.mark.parametrize("case", range(len(CASES)))
@pytest.mark.parametrize("verify", ["off", "always"])
@pytest.mark.parametrize("hint", [True, False])
@pytest.mark.parametrize("bint", [False, True])
def test_chain_equals_unchained(cuda, case, verify, hint, bint):
    """hint: each conv is told whether the next one pools its codes, so its epilogue writes the next
    layer's per-image maxima (over the pool's region); without, a pooling consumer finds maxima of the
    unpooled image and makes its own two passes. bint: Config(conv_bias_int32=True) on both routes."""
    from torch_xdna.conv import IN_CODES, IN_CODES_POOL, IN_FLOAT

    shapes, biased, pools, H, W, nimg = CASES[case]
    g = torch.Generator(device=cuda).manual_seed(7 + case)
    layers = _weights(cuda, g, shapes, biased)
    x = torch.randn(nimg, shapes[0][1], H, W, device=cuda, generator=g)
    cid = _cid(verify=verify, conv_bias_int32=bint)
    # one by one: a biased conv's ReLU after its bias, a bias-free conv's ReLU in the requantise
    y = x
    for i, (w, b) in enumerate(layers):
        if pools[i]:
            y = torch.nn.functional.max_pool2d(y, 2)
        y = torch.ops.xdna.conv3x3_fused(y, w, b, b is None, cid, b is not None)
    want = y
    # chained: codes between the convs, the pools taken into the next conv's quantise
    q, meta, ra = x, None, False
    for i, (w, b) in enumerate(layers):
        last = i == len(layers) - 1
        mode = IN_FLOAT if i == 0 else (IN_CODES_POOL if pools[i] else IN_CODES)
        out_pool = hint and not last and pools[i + 1]
        q, meta = torch.ops.xdna.conv3x3_chain(q, meta, w, b, b is None, cid, b is not None, mode, ra, not last,
                                               out_pool)
        if not last:
            assert q.dtype == (torch.uint8 if b is None or bint else torch.int8) and q.shape[-1] == w.shape[0]
        ra = b is not None
    got = q
    assert got.shape == want.shape and got.dtype == want.dtype
    assert torch.equal(got, want), f"{int((got != want).sum())} of {want.numel()} values differ"


KINDS = ["relu_after_bias", "fused_relu", "signed"]


@pytest.mark.parametrize("shape", [(3, 40, 64, 15, 17), (2, 64, 128, 30, 22), (9, 16, 32, 3, 4), (2, 32, 320, 9, 11),
                                   (2, 128, 512, 20, 20)])
@pytest.mark.parametrize("kind", KINDS)
@pytest.mark.parametrize("pool", [False, True])
def test_next_layer_maxima_from_the_producer(cuda, shape, kind, pool):
    """A conv with XDNA_CONV_NEXT_AMAX writes, per image, the max |y| of the float values its codes stand for
    (y = float(q) * (scale * sx) + bias, then the ReLU after the bias; over the 2x2 pool's region when the
    next conv pools): the same bits the two-pass quantise of those codes finds, so the one-pass quantise
    from them gives the same input bytes and factors."""
    from torch_xdna import conv as xconv
    from torch_xdna import kernels

    if pool and kind == "signed":
        pytest.skip("pooled maxima need non-negative values")
    n, ci, co, h, w = shape
    g = torch.Generator(device=cuda).manual_seed(sum(shape) + KINDS.index(kind) + 10 * pool)
    wt = torch.randn(co, ci, 3, 3, device=cuda, generator=g) * (2.0 / (ci * 9)) ** 0.5
    fused = kind == "fused_relu"
    bias = None if fused else torch.randn(co, device=cuda, generator=g) * 0.05
    layer = xconv.ConvLayer(wt, h, w, fused)
    xp, sx = layer.quantise(torch.randn(n, ci, h, w, device=cuda, generator=g), n)
    layer.calibrate(xp)
    relu_after = kind == "relu_after_bias"
    q = torch.empty((n, h, w, co), dtype=torch.uint8 if fused else torch.int8, device=cuda)
    meta = xconv.codes_meta(sx, layer.scale, bias, co, amax=True, pool=pool)
    mode = (kernels.CONV_Q_NHWC | kernels.CONV_NEXT_AMAX | (kernels.CONV_NEXT_RELU if relu_after else 0)
            | (kernels.CONV_NEXT_POOL if pool else 0))
    amax = meta[n + 2 * co:2 * n + 2 * co].view(torch.int32)
    kernels.conv3x3(xp, layer.wp, n, ci, co, h, w, mode, shift=layer.shift, relu=fused, scale=meta[n:n + co],
                    sx=sx, bias=meta[n + co:n + 2 * co] if bias is not None else None, out=q, acc_max=amax)
    # the codes are those of the plain requantise
    q0 = torch.empty_like(q)
    kernels.conv3x3(xp, layer.wp, n, ci, co, h, w, kernels.CONV_Q_NHWC, shift=layer.shift, relu=fused, out=q0)
    assert torch.equal(q, q0)
    # the maxima: max |y| over each image (pooled) on the CPU with the epilogue's f32 operations
    y = xconv.codes_to_float(q, meta, relu_after, pool)
    want = y.abs().amax(dim=(1, 2, 3))
    assert torch.equal(amax.cpu().view(torch.float32), want)
    # the next conv's input from them equals the two-pass one
    hn, wn = (h // 2, w // 2) if pool else (h, w)
    cp = xconv.channels_padded(co)
    xa, xb = (torch.full((n, hn + 2, wn + 2, cp), 77, dtype=torch.int8, device=cuda) for _ in range(2))
    sa, sb = torch.empty(n, device=cuda), torch.empty(n, device=cuda)
    scratch = torch.empty(n, dtype=torch.int32, device=cuda)
    args = (q, meta[n:n + co], meta[:n], meta[n + co:n + 2 * co], relu_after, pool)
    kernels.conv_quant_codes(*args, xa, sa, scratch)
    kernels.conv_quant_codes_given_amax(*args, xb, sb, amax)
    assert torch.equal(sa, sb) and torch.equal(xa, xb)


@pytest.mark.parametrize("shape", [(2, 64, 15, 17), (4, 128, 30, 22), (6, 64, 3, 4), (2, 128, 112, 112)])
@pytest.mark.parametrize("kind", ["relu_after_bias", "fused_relu", "signed"])
def test_image_pairs_equal_the_plain_layout(cuda, shape, kind):
    """XDNA_CONV_PAIRS: the same conv over the input interleaved two images per 128-byte row gives the same
    codes and the same next-layer maxima as over the plain layout; conv_quant_codes_pairs writes exactly the
    interleave of conv_quant_codes' output."""
    from torch_xdna import conv as xconv
    from torch_xdna import kernels

    n, co, h, w = shape
    g = torch.Generator(device=cuda).manual_seed(n + co + h + len(kind))
    wt = torch.randn(co, 64, 3, 3, device=cuda, generator=g) * (2.0 / (64 * 9)) ** 0.5
    fused = kind == "fused_relu"
    bias = None if fused else torch.randn(co, device=cuda, generator=g) * 0.05
    relu_after = kind == "relu_after_bias"
    # the input: a previous conv's codes, quantised both ways
    qin = torch.randint(0 if fused else -128, 256 if fused else 128, (n, h, w, 64), device=cuda, generator=g)
    qin = qin.to(torch.uint8 if fused else torch.int8)
    scale_in = torch.rand(64, device=cuda, generator=g) * 1e-3 + 1e-4
    sx_in = torch.rand(n, device=cuda, generator=g) + 0.5
    b_in = torch.randn(64, device=cuda, generator=g) * 0.05
    xp = torch.empty(n, h + 2, w + 2, 64, dtype=torch.int8, device=cuda)
    sx = torch.empty(n, device=cuda)
    kernels.conv_quant_codes(qin, scale_in, sx_in, b_in, True, False, xp, sx, torch.empty(n, dtype=torch.int32,
                                                                                           device=cuda))
    xp2 = torch.empty(n // 2, h + 2, w + 2, 128, dtype=torch.int8, device=cuda)
    sx2 = torch.empty(n, device=cuda)
    kernels.conv_quant_codes_pairs(qin, scale_in, sx_in, b_in, True, False, xp2, sx2,
                                   torch.empty(n, dtype=torch.int32, device=cuda), False)
    assert torch.equal(sx, sx2)
    assert torch.equal(xp2.view(n // 2, h + 2, w + 2, 2, 64).permute(0, 3, 1, 2, 4).reshape(xp.shape), xp)
    layer = xconv.ConvLayer(wt, h, w, fused)
    layer.calibrate(xp)
    mode = kernels.CONV_Q_NHWC
    if kind != "signed":
        mode |= kernels.CONV_NEXT_AMAX | (kernels.CONV_NEXT_RELU if relu_after else 0)
    outs = []
    for src, extra in ((xp, 0), (xp2, kernels.CONV_PAIRS)):
        q = torch.empty((n, h, w, co), dtype=torch.uint8 if fused else torch.int8, device=cuda)
        amax = torch.zeros(n, dtype=torch.int32, device=cuda)
        kernels.conv3x3(src, layer.wp, n, 64, co, h, w, mode | extra, shift=layer.shift, relu=fused,
                        scale=layer.scale, sx=sx, bias=bias, out=q, acc_max=amax if kind != "signed" else None)
        outs.append((q, amax))
    assert torch.equal(outs[0][0], outs[1][0]), f"{int((outs[0][0] != outs[1][0]).sum())} codes differ"
    assert torch.equal(outs[0][1], outs[1][1])


@pytest.mark.parametrize("c", [64, 256])
@pytest.mark.parametrize("pool", [False, True])
@pytest.mark.parametrize("relu_after", [True, False])
@pytest.mark.parametrize("pairs", [False, True])
def test_quantise_from_codes_matches_the_cpu(cuda, c, pool, relu_after, pairs):
    """The quantise from codes on millions of values against the CPU: y rebuilt with torch's f32 operations
    in the epilogue's order (codes_to_float), the per-image max, and round(y / s) by IEEE division -- bit
    for bit. Large enough that a rounding difference of a few codes in 10^5 shows."""
    from torch_xdna import conv as xconv
    from torch_xdna import kernels

    if pairs and c != 64:
        pytest.skip("image pairs are 64-channel layouts")
    n, h, w = 4, 96, 104
    g = torch.Generator(device=cuda).manual_seed(3 + pool + 2 * relu_after + 4 * pairs + c)
    q = torch.randint(-128, 128, (n, h, w, c), device=cuda, generator=g).to(torch.int8)
    scale = torch.rand(c, device=cuda, generator=g) * 1e-3 + 1e-4
    sx_in = torch.rand(n, device=cuda, generator=g) + 0.5
    bias = torch.randn(c, device=cuda, generator=g) * 0.02
    meta = xconv.codes_meta(sx_in, scale, bias, c)
    ho, wo = (h // 2, w // 2) if pool else (h, w)
    sx = torch.empty(n, device=cuda)
    scratch = torch.empty(n, dtype=torch.int32, device=cuda)
    if pairs:
        xp2 = torch.empty(n // 2, ho + 2, wo + 2, 128, dtype=torch.int8, device=cuda)
        kernels.conv_quant_codes_pairs(q, scale, sx_in, bias, relu_after, pool, xp2, sx, scratch, False)
        xp = xp2.view(n // 2, ho + 2, wo + 2, 2, 64).permute(0, 3, 1, 2, 4).reshape(n, ho + 2, wo + 2, 64)
    else:
        xp = torch.empty(n, ho + 2, wo + 2, c, dtype=torch.int8, device=cuda)
        kernels.conv_quant_codes(q, scale, sx_in, bias, relu_after, pool, xp, sx, scratch)
    y = xconv.codes_to_float(q, meta, relu_after, pool)                    # CPU, NCHW
    s = (y.abs().amax(dim=(1, 2, 3)).clamp(min=1e-8) / 127).float()
    want = torch.round(y / s[:, None, None, None]).clamp(-127, 127).to(torch.int8).permute(0, 2, 3, 1)
    assert torch.equal(sx.cpu(), s)
    got = xp[:, 1:ho + 1, 1:wo + 1].cpu()
    bad = int((got != want).sum())
    assert bad == 0, f"{bad} of {want.numel()} quantised values differ"
    assert int(xp[:, 0].abs().sum()) == 0 and int(xp[:, :, 0].abs().sum()) == 0   # the zero border


def test_quantise_through_the_table():
    """The table kernel for the quantise from codes (chosen by size: large batches of large images) run
    wherever it applies (XDNA_CODES_LUT=2, a fresh process since the library reads it once) through this
    file's bit-exact tests of the quantise, the image pairs, the producers' maxima and the chain; and the
    direct kernel alone (XDNA_CODES_LUT=0) through the quantise test."""
    import os
    import subprocess
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    for mode, sel in (("2", "quantise_from_codes or image_pairs or next_layer_maxima or chain_equals_unchained"),
                      ("0", "quantise_from_codes")):
        env = dict(os.environ, XDNA_CODES_LUT=mode)
        out = subprocess.run([sys.executable, "-m", "pytest", "-x", "-q", "-p", "no:cacheprovider", "-m", "gpu",
                              "-k", sel, os.path.join(here, "test_conv_chain_gpu.py")],
                             env=env, capture_output=True, text=True, timeout=900)
        assert out.returncode == 0, f"XDNA_CODES_LUT={mode}:\n{out.stdout[-3000:]}\n{out.stderr[-2000:]}"


def test_compiled_vgg_block_chained_equals_unchained(cuda):
    """torch.compile(backend="xdna"): the chained graph (default) and the unchained one (fuse=False, ReLU
    and max-pool left to torch) give identical outputs."""
    import torch_xdna  # noqa: F401

    class Net(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.c1 = torch.nn.Conv2d(3, 64, 3, padding=1)
            self.c2 = torch.nn.Conv2d(64, 64, 3, padding=1)
            self.c3 = torch.nn.Conv2d(64, 128, 3, padding=1)
            self.pool = torch.nn.MaxPool2d(2)

        def forward(self, x):
            h = torch.relu(self.c2(torch.relu(self.c1(x))))
            return torch.relu(self.c3(self.pool(h)))

    net = Net().to(cuda).eval()
    x = torch.randn(2, 3, 40, 56, device=cuda)
    outs = []
    for fuse in (True, False):
        torch._dynamo.reset()
        m = torch.compile(net, backend="xdna", options={"fuse": fuse, "verify": "off"})
        outs.append(m(x))
    assert torch.equal(outs[0], outs[1]), f"{int((outs[0] != outs[1]).sum())} values differ"
    ref = net(x)
    assert (outs[0] - ref).abs().max() / ref.abs().max() < 0.05  # int8 vs fp32: the quantisation error only
