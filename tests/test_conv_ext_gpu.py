"""The ResNet-style convs the reference has no kernel for (R:results/conv3x3_cascade.md:222-223), offloaded
with Config(conv_ext=True): 1x1 convs (stride 1 and 2) and stride-2 3x3 convs, through the reference's int8
conv arithmetic (per-image quantise, int8 weights per output channel, exact sums, the shift fixed from
image 0, requantise, dequantise + bias). Bit-exact against the oracle, whose sums are F.conv2d of the
integers with the conv's own stride and padding; and a compiled bottleneck block against the oracle."""

import numpy as np
import pytest
import torch

import make_golden as mg
from oracle import xdna_oracle as orc

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _inference(request):
    from torch_xdna import kernels

    if "cuda" in request.fixturenames:
        kernels.take_device_error()
    with torch.no_grad():
        yield
    if "cuda" in request.fixturenames:
        assert kernels.take_device_error() == (0, 0), "a kernel recorded a device-side error"


def _cid(**kw):
    import torch_xdna

    return torch_xdna.ops.config_id(torch_xdna.Config(**kw))


CASES = [  # (k, stride, n, ci, co, h, w)
    (1, 1, 2, 64, 256, 56, 56), (1, 1, 3, 256, 64, 14, 14), (1, 1, 1, 3, 20, 9, 5), (1, 1, 2, 512, 2048, 7, 7),
    (1, 2, 2, 256, 512, 56, 56), (1, 2, 2, 40, 24, 13, 11), (1, 2, 1, 1024, 2048, 14, 14),
    (3, 2, 2, 64, 64, 56, 56), (3, 2, 1, 128, 128, 29, 31), (3, 2, 3, 7, 20, 9, 10), (3, 2, 2, 256, 300, 28, 28),
    (3, 2, 2, 512, 512, 14, 14),
]


@pytest.mark.parametrize("layout", ["nchw", "channels_last"])
@pytest.mark.parametrize("k,stride,n,ci,co,h,w", CASES)
def test_conv_ext_bitexact_vs_oracle(cuda, k, stride, n, ci, co, h, w, layout):
    """Biased conv with the ReLU after the bias (post_relu), f32: y equals the oracle's bit for bit; the
    op's first-launch verify compares the requantised integers with F.conv2d on the CPU."""
    x, _, b = mg.conv_inputs(k * 100 + stride * 10 + ci + co + h, n, ci, co, h, w, bias=True)
    g = mg.rng(ci * 7 + co)
    wt = (g.standard_normal((co, ci, k, k)) * np.sqrt(2.0 / (ci * k * k))).astype(np.float32)
    want = orc.conv3x3_int8(x, wt, b, relu=False, stride=stride)
    weight = torch.nn.Parameter(torch.from_numpy(wt).to(cuda))
    xt = torch.from_numpy(x).to(cuda)
    if layout == "channels_last":
        xt = xt.contiguous(memory_format=torch.channels_last)
    y = torch.ops.xdna.conv_int8(xt, weight, torch.from_numpy(b).to(cuda), stride, False, _cid(verify="first"), True)
    assert tuple(y.shape) == want["y"].shape
    got = y.cpu().numpy()
    ref = np.maximum(want["y"], np.float32(0))
    bad = int((got != ref).sum())
    assert bad == 0, f"{bad} of {got.size} values differ"
    from torch_xdna import conv as xconv

    assert xconv._layer(weight, h, w, False, stride=stride).shift == want["shift"]


@pytest.mark.parametrize("k,stride", [(1, 1), (1, 2), (3, 2)])
def test_conv_ext_fused_relu_bf16(cuda, k, stride):
    """Bias-free conv with its ReLU fused into the requantise (uint8 saturation), bf16 in and out."""
    n, ci, co, h, w = 2, 96, 80, 30, 27
    x, _, _ = mg.conv_inputs(9 + k + stride, n, ci, co, h, w)
    xb = orc.cast(x, "bfloat16")
    g = mg.rng(k * 3 + stride)
    wt = (g.standard_normal((co, ci, k, k)) * np.sqrt(2.0 / (ci * k * k))).astype(np.float32)
    want = orc.conv3x3_int8(xb, wt, None, relu=True, stride=stride, x_dtype="bfloat16")
    weight = torch.nn.Parameter(torch.from_numpy(wt).to(cuda))
    y = torch.ops.xdna.conv_int8(torch.from_numpy(xb).to(cuda, torch.bfloat16), weight, None, stride, True,
                                 _cid(verify="first"), False)
    assert np.array_equal(y.float().cpu().numpy(), want["y"])


def test_conv_quant_phases_layout(cuda):
    """The stride phases: plane 2 ry + rx at bordered (Y, X) = the quantised input pixel (2(Y-1)+ry, 2(X-1)+rx),
    zeros elsewhere; the same codes and scale from NCHW and channels-last input."""
    from torch_xdna import kernels

    n, c, h, w = 2, 20, 9, 12
    x, _, _ = mg.conv_inputs(3, n, c, 4, h, w)
    xq, sx_ref = orc.conv_quant(x)
    ho, wo = (h + 1) // 2, (w + 1) // 2
    want = np.zeros((4, n, ho + 2, wo + 2, 32), np.int8)
    for ry in range(2):
        for rx in range(2):
            for Y in range(1, ho + 1):
                for X in range(1, wo + 1):
                    yy, xx = 2 * (Y - 1) + ry, 2 * (X - 1) + rx
                    if yy < h and xx < w:
                        want[2 * ry + rx, :, Y, X, :c] = xq[:, :, yy, xx]
    for cl in (False, True):
        xt = torch.from_numpy(x).to(cuda)
        if cl:
            xt = xt.contiguous(memory_format=torch.channels_last)
        xp = torch.full((4, n, ho + 2, wo + 2, 32), 99, dtype=torch.int8, device=cuda)
        sx = torch.empty(n, device=cuda)
        kernels.conv_quant_phases(xt, xp, sx, torch.empty(n, dtype=torch.int32, device=cuda), cl)
        assert np.array_equal(sx.cpu().numpy(), sx_ref)
        assert np.array_equal(xp.cpu().numpy(), want)


class Bottleneck(torch.nn.Module):
    """A ResNet-50 bottleneck with a stride-2 downsample (no batch norm: folded into the convs' weights and
    biases at inference)."""

    def __init__(self, cin, mid, cout, g):
        super().__init__()
        self.c1 = torch.nn.Conv2d(cin, mid, 1)
        self.c2 = torch.nn.Conv2d(mid, mid, 3, stride=2, padding=1)
        self.c3 = torch.nn.Conv2d(mid, cout, 1)
        self.down = torch.nn.Conv2d(cin, cout, 1, stride=2)
        for c in (self.c1, self.c2, self.c3, self.down):
            fan = c.weight[0].numel()
            c.weight.data = torch.randn(c.weight.shape, generator=g) * (2.0 / fan) ** 0.5
            c.bias.data = torch.randn(c.bias.shape, generator=g) * 0.01

    def forward(self, x):
        h = torch.relu(self.c1(x))
        h = torch.relu(self.c2(h))
        return torch.relu(self.c3(h) + self.down(x))


@pytest.mark.parametrize("bint", [False, True])
def test_compiled_bottleneck_vs_oracle(cuda, bint):
    """bint: Config(conv_bias_int32=True), every conv's bias inside its int32 sums and the sole-user ReLUs
    in the requantise."""
    import torch_xdna

    g = torch.Generator().manual_seed(3)
    net = Bottleneck(256, 128, 512, g).eval()
    x = torch.randn(2, 256, 28, 28, generator=torch.Generator().manual_seed(4))

    def oc(h, c, stride, relu_next=False):
        return orc.conv3x3_int8(h, c.weight.detach().numpy(), c.bias.detach().numpy(), relu=bint and relu_next,
                                stride=stride, bias_int32=bint)["y"]

    relu = lambda a: np.maximum(a, np.float32(0))  # noqa: E731
    xn = x.numpy()
    h = relu(oc(xn, net.c1, 1, True))
    h = relu(oc(h, net.c2, 2, True))
    want = relu((oc(h, net.c3, 1) + oc(xn, net.down, 2)).astype(np.float32))
    torch._dynamo.reset()
    torch_xdna.stats.reset()
    comp = torch.compile(net.to(cuda), backend="xdna",
                         options={"fallback": "eager", "conv_ext": True, "conv_bias_int32": bint})
    y = comp(x.to(cuda))
    assert torch_xdna.stats.as_dict()["calls"]["gpu"] == 4
    assert len(torch_xdna.stats.checks) == 4      # every conv's first launch verified against the CPU integers
    got = y.cpu().numpy()
    assert np.array_equal(got, want), f"{int((got != want).sum())} of {want.size} values differ"


def test_conv_bias_int32_kernel_vs_oracle(cuda):
    """xdna_conv_bias_int32: rint(bias / (sw * sx)) in f32 per image, ties to even, clamped, NaN -> 0; f32 and
    bf16 biases."""
    from torch_xdna import kernels

    g = mg.rng(31)
    co, n = 300, 5
    bias = (g.standard_normal(co) * 0.3).astype(np.float32)
    bias[:6] = [1.25, -0.375, 1e12, -np.inf, np.nan, 2.5]
    sw = (np.abs(g.standard_normal(co)) * 1e-2 + 1e-6).astype(np.float32)
    sw[:6] = [0.5, 0.25, 1.0, 2.0, 1.0, 1.0]
    sx = (np.abs(g.standard_normal(n)) * 0.02 + 1e-4).astype(np.float32)
    sx[0] = 1.0
    for dtype in ("float32", "bfloat16"):
        b = orc.cast(bias, dtype)
        want = orc.conv_bias_int32(b, sw, sx)
        out = torch.empty((n, co), dtype=torch.int32, device=cuda)
        bt = torch.from_numpy(b).to(cuda, torch.float32 if dtype == "float32" else torch.bfloat16)
        kernels.conv_bias_int32(bt, torch.from_numpy(sw).to(cuda), torch.from_numpy(sx).to(cuda), out)
        got = out.cpu().numpy()
        assert np.array_equal(got, want), f"{dtype}: {int((got != want).sum())} of {want.size} differ"
    assert want[0, :6].tolist()[:3] == [2, -2, 2 ** 29] and want[0, 4] == 0


BINT_CASES = [  # (k, stride, n, ci, co, h, w)
    (3, 1, 2, 64, 64, 30, 22), (3, 1, 3, 3, 30, 17, 19), (3, 1, 2, 256, 300, 14, 14), (1, 1, 2, 64, 256, 14, 14),
    (1, 2, 2, 40, 24, 13, 11), (3, 2, 2, 64, 64, 28, 28),
]


@pytest.mark.parametrize("relu", [True, False])
@pytest.mark.parametrize("k,stride,n,ci,co,h,w", BINT_CASES)
def test_bias_int32_bitexact_vs_oracle(cuda, k, stride, n, ci, co, h, w, relu):
    """Config(conv_bias_int32=True): the bias inside the int32 sums (calibration included), the ReLU after the
    bias as the requantise's saturation; f32 y bit for bit against the oracle's route, the shift the same."""
    from torch_xdna import conv as xconv

    x, _, b = mg.conv_inputs(k * 100 + stride * 10 + ci + co + h + relu, n, ci, co, h, w, bias=True, bias_std=0.5)
    g = mg.rng(ci * 5 + co + k)
    wt = (g.standard_normal((co, ci, k, k)) * np.sqrt(2.0 / (ci * k * k))).astype(np.float32)
    want = orc.conv3x3_int8(x, wt, b, relu=relu, stride=stride, bias_int32=True)
    weight = torch.nn.Parameter(torch.from_numpy(wt).to(cuda))
    cid = _cid(verify="first", conv_ext=True, conv_bias_int32=True)
    y = torch.ops.xdna.conv_int8(torch.from_numpy(x).to(cuda), weight, torch.from_numpy(b).to(cuda), stride, False,
                                 cid, relu)
    got = y.cpu().numpy()
    bad = int((got != want["y"]).sum())
    assert bad == 0, f"{bad} of {got.size} values differ"
    if k == 3 and stride == 1:
        layer = xconv._layer(weight, h, w, relu, taps=ci <= 7, bint=True)
    else:
        layer = xconv._layer(weight, h, w, relu, stride=stride, bint=True)
    assert layer.shift == want["shift"] and layer.checked
