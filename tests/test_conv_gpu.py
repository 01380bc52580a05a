"""int8 conv3x3 on the B200 vs the oracle (bit-exact): calibration shift, requantised integers (int8 /
uint8 with ReLU), the fused quantise -> conv -> dequantise, the backend's conv pass, and the golden
digests recorded from the reference's CPU integers."""

import numpy as np
import pytest
import torch

import make_golden as mg
from oracle import xdna_oracle as orc

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _inference():
    """The xdna ops are inference-only (no autograd formula, as in the reference): run under no_grad."""
    with torch.no_grad():
        yield


def t(a, dev, dtype=None):
    x = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return x.to(dtype) if dtype is not None else x


def _cid(**kw):
    import torch_xdna

    return torch_xdna.ops.config_id(torch_xdna.Config(**kw))


@pytest.mark.parametrize("name", [c[0] for c in mg.CONV_CASES])
def test_conv_op_matches_reference_digests(cuda, golden, name):
    manifest, _ = golden
    ent = manifest["conv"][name]
    x, w, b = mg.conv_inputs(ent["seed"], ent["N"], ent["Ci"], ent["Co"], ent["H"], ent["W"], bias=ent["bias"])
    xq, sx = orc.conv_quant(x)
    weight = torch.nn.Parameter(t(w, cuda))
    q, scale = torch.ops.xdna.conv3x3(t(xq, cuda), weight, ent["relu"], _cid(verify="off"))
    from torch_xdna import conv as xconv

    layer = xconv._layer(weight, ent["H"], ent["W"], ent["relu"])
    assert layer.shift == ent["shift"], (layer.shift, ent["shift"])
    assert mg.sha(q.cpu().numpy()) == ent["q_sha"], "requantised integers differ from the reference's"
    assert mg.sha(scale.cpu().numpy()) == ent["scale_sha"]
    # the fused path (quantise + conv + dequantise) on the same layer
    y = torch.ops.xdna.conv3x3_fused(t(x, cuda), weight, t(b, cuda) if b is not None else None, ent["relu"],
                                     _cid(verify="off"))
    assert mg.sha(y.cpu().numpy()) == ent["y_sha"], "dequantised output differs from the reference's"


@pytest.mark.parametrize("relu", [False, True])
@pytest.mark.parametrize("n,ci,co,h,w", [(1, 256, 256, 64, 64), (2, 3, 64, 13, 37), (2, 64, 48, 13, 37),
                                         (1, 16, 16, 1, 1), (3, 130, 20, 7, 129), (1, 512, 512, 14, 14),
                                         (2, 64, 64, 224, 224), (2, 40, 128, 17, 23), (1, 64, 200, 16, 16),
                                         # 256 x 256 tiles on CTA pairs (the second: ragged Co and channel block)
                                         (8, 128, 256, 56, 56), (5, 160, 300, 40, 52)])
def test_conv_q_bitexact_vs_oracle(cuda, relu, n, ci, co, h, w):
    x, wt, _ = mg.conv_inputs(n * 1000 + ci + co + h, n, ci, co, h, w)
    want = orc.conv3x3_int8(x, wt, None, relu=relu)
    weight = torch.nn.Parameter(t(wt, cuda))
    q, scale = torch.ops.xdna.conv3x3(t(want["xq"], cuda), weight, relu, _cid(verify="off"))
    from torch_xdna import conv as xconv

    assert xconv._layer(weight, h, w, relu).shift == want["shift"]
    got = q.cpu().numpy()
    bad = int((got != want["q"]).sum())
    assert bad == 0, f"{bad} of {got.size} requantised values differ"
    assert np.array_equal(scale.cpu().numpy(), want["scale"])


@pytest.mark.parametrize("post_relu", [False, True])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
# (2, 64, 64, ...) and (3, 40, 128, ...): weights resident in shared memory; (5, 160, 300, ...): CTA pairs;
# (2, 3, 64, ...) and (1, 7, 20, ...): <= 7 input channels, the stencil's taps packed into the channels
@pytest.mark.parametrize("n,ci,co,h,w", [(2, 96, 80, 30, 50), (5, 160, 300, 40, 52), (2, 64, 64, 30, 50),
                                         (3, 40, 128, 21, 19), (2, 3, 64, 33, 47), (1, 7, 20, 9, 5)])
def test_conv_fused_dequant_bitexact(cuda, dtype, post_relu, n, ci, co, h, w):
    """The dequantise (+ bias) to x.dtype, bit for bit; post_relu equals torch.relu of it."""
    x, wt, b = mg.conv_inputs(5, n, ci, co, h, w, bias=True)
    xd = orc.cast(x, "bfloat16") if dtype == torch.bfloat16 else x
    want = orc.conv3x3_int8(xd, wt, b, relu=False, x_dtype="bfloat16" if dtype == torch.bfloat16 else "float32")
    weight = torch.nn.Parameter(t(wt, cuda))
    y = torch.ops.xdna.conv3x3_fused(t(xd, cuda, dtype), weight, t(b, cuda), False, _cid(verify="off"), post_relu)
    w = np.maximum(want["y"], 0) if post_relu else want["y"]
    assert np.array_equal(y.float().cpu().numpy(), w)


@pytest.mark.parametrize("layout", ["nchw", "channels_last"])
def test_conv_quant_nan_image_scale(cuda, layout):
    """An image holding a NaN gets a NaN scale, as the reference's x.abs().amax(...).clamp(min=1e-8)
    (R:torch_xdna/conv.py:45) does; the other images' scales and codes stay bit-exact. The codes of the NaN
    image are outside the parity claim (the reference's int8 cast of NaN is platform-defined)."""
    from torch_xdna import kernels

    n, c, h, w = 4, 32, 9, 11
    x, _, _ = mg.conv_inputs(71, n, c, 8, h, w)
    x[2, 5, 3, 4] = np.nan
    xt = t(x, cuda)
    if layout == "channels_last":
        xt = xt.contiguous(memory_format=torch.channels_last)
    xp = torch.empty((n, h + 2, w + 2, 32), dtype=torch.int8, device=cuda)
    sx = torch.empty((n,), dtype=torch.float32, device=cuda)
    scratch = torch.empty((n,), dtype=torch.int32, device=cuda)
    (kernels.conv_quant_channels_last if layout == "channels_last" else kernels.conv_quant)(xt, xp, sx, scratch)
    got = sx.cpu().numpy()
    assert np.isnan(got[2]) and not np.isnan(got[[0, 1, 3]]).any()
    q_ref, s_ref = orc.conv_quant(x[[0, 1, 3]])
    assert np.array_equal(got[[0, 1, 3]], s_ref)
    inner = xp[[0, 1, 3], 1:h + 1, 1:w + 1, :c].permute(0, 3, 1, 2).cpu().numpy()
    assert np.array_equal(inner, q_ref)


def test_cfg3_chain_matches_reference(cuda, golden):
    """4 x (conv3x3 256->256 + fused ReLU) on 1x256x64x64; shifts and every layer's
    integers equal the reference's."""
    manifest, _ = golden
    ent = manifest["conv"]["cfg3_chain"]
    g = mg.rng(ent["seed"])
    x = g.standard_normal((1, 256, 64, 64), dtype=np.float32)
    ws = [g.standard_normal((256, 256, 3, 3), dtype=np.float32) * np.float32(np.sqrt(2.0 / (256 * 9)))
          for _ in range(4)]
    from torch_xdna import conv as xconv

    h = t(x, cuda)
    cid = _cid(verify="off")
    for i, w in enumerate(ws):
        weight = torch.nn.Parameter(t(w, cuda))
        h = torch.ops.xdna.conv3x3_fused(h, weight, None, True, cid)
        assert xconv._layer(weight, 64, 64, True).shift == ent["shifts"][i]
    assert mg.sha(h.cpu().numpy()) == ent["y_sha"]


def test_conv_verify_first(cuda):
    import torch_xdna

    torch_xdna.stats.reset()
    x, wt, _ = mg.conv_inputs(9, 1, 32, 32, 20, 20)
    weight = torch.nn.Parameter(t(wt, cuda))
    cid = _cid(verify="first")
    torch.ops.xdna.conv3x3_fused(t(x, cuda), weight, None, True, cid)
    torch.ops.xdna.conv3x3_fused(t(x, cuda), weight, None, True, cid)
    checks = torch_xdna.stats.as_dict()["checks"]
    assert len(checks) == 1 and "bitwise" in checks[0][1]


class CNN(torch.nn.Module):
    """R:tests/test_backend.py:203-217: bias + ReLU, bias-free + ReLU (fused), "same", a stride-2 conv."""

    def __init__(self):
        super().__init__()
        self.c1 = torch.nn.Conv2d(64, 128, 3, padding=1)
        self.c2 = torch.nn.Conv2d(128, 128, 3, padding=1, bias=False)
        self.c3 = torch.nn.Conv2d(128, 32, 3, padding="same")
        self.down = torch.nn.Conv2d(32, 32, 3, stride=2, padding=1)

    def forward(self, x):
        h = torch.relu(self.c1(x))
        h = torch.relu(self.c2(h))
        return self.down(self.c3(h))


def test_compiled_cnn(cuda):
    """3 of 4 convs on the B200 (the stride-2 one stays), close to fp32; each layer's integers equal the
    oracle's on the same quantised input."""
    import torch_xdna

    torch.manual_seed(0)
    net = CNN().eval().to(cuda)
    x = torch.randn(2, 64, 32, 64, device=cuda)
    torch._dynamo.reset()
    torch_xdna.stats.reset()
    m = torch.compile(net, backend="xdna", options={"fallback": "eager"})
    with torch.no_grad():
        y, ref = m(x), net(x)
    s = torch_xdna.stats.as_dict()
    assert s["calls"] == {"gpu": 3}, s
    err = ((y - ref).norm() / ref.norm()).item()
    assert err < 0.05, err
    # layer by layer against the oracle (c1 with bias, its ReLU separate; c2 ReLU fused; c3 plain)
    xs = x.cpu().numpy()
    r1 = orc.conv3x3_int8(xs, net.c1.weight.detach().cpu().numpy(), net.c1.bias.detach().cpu().numpy(), relu=False)
    h = np.maximum(r1["y"], 0)
    r2 = orc.conv3x3_int8(h, net.c2.weight.detach().cpu().numpy(), None, relu=True)
    r3 = orc.conv3x3_int8(r2["y"], net.c3.weight.detach().cpu().numpy(), net.c3.bias.detach().cpu().numpy(),
                          relu=False)
    with torch.no_grad():
        want = net.down(torch.from_numpy(r3["y"]).to(cuda))
    assert torch.equal(y, want)


@pytest.mark.parametrize("c", [1, 2, 3, 4, 5, 7])
@pytest.mark.parametrize("n,h,w", [(2, 9, 13), (3, 33, 47), (1, 4, 300)])
def test_quant_taps_layout(cuda, c, n, h, w):
    """The first layer's input with the 3x3 stencil's taps packed into each bordered pixel's row, byte for
    byte: row (yb, xb) holds, for tap t = 3 dy + dx and channel ch, the oracle's int8 of input pixel
    (yb - 2 + dy, xb - 2 + dx) at byte C t + ch (zero outside the image and past byte 9 C). C <= 4 takes
    the row-per-block kernel, C >= 5 the pixel-per-thread one."""
    from torch_xdna import kernels

    x, _, _ = mg.conv_inputs(300 + c + h, n, c, 8, h, w)
    kp = (9 * c + 15) // 16 * 16
    xp = torch.full((n, h + 2, w + 2, kp), 77, dtype=torch.int8, device=cuda)
    sx = torch.empty((n,), dtype=torch.float32, device=cuda)
    scratch = torch.empty((n,), dtype=torch.int32, device=cuda)
    kernels.conv_quant_taps(t(x, cuda), xp, sx, scratch)
    q, s = orc.conv_quant(x)
    assert np.array_equal(sx.cpu().numpy(), s)
    pad = np.zeros((n, c, h + 4, w + 4), dtype=np.int8)     # input pixel (y, x) at (y + 2, x + 2)
    pad[:, :, 2:h + 2, 2:w + 2] = q
    want = np.zeros((n, h + 2, w + 2, kp), dtype=np.int8)
    for tap in range(9):
        dy, dx = divmod(tap, 3)
        # bordered pixel (yb, xb) reads input (yb - 2 + dy, xb - 2 + dx) = pad[yb + dy, xb + dx]
        want[..., tap * c:(tap + 1) * c] = pad[:, :, dy:dy + h + 2, dx:dx + w + 2].transpose(0, 2, 3, 1)
    got = xp.cpu().numpy()
    bad = int((got != want).sum())
    assert bad == 0, f"{bad} of {got.size} bytes differ"
