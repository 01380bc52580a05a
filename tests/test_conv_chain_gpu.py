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


# (channels per conv, bias per conv, pool before conv i, H, W)
CASES = [
    ([(64, 3), (64, 64), (128, 64), (128, 128)], [True, True, True, False], [False, False, True, False], 32, 48),
    # odd sizes: the pool rounds down (15 x 17 -> 7 x 8); 20 channels: scalar stores of the codes
    ([(20, 8), (32, 20), (16, 32)], [True, False, True], [False, True, False], 15, 17),
]


@pytest.mark.parametrize("case", range(len(CASES)))
@pytest.mark.parametrize("verify", ["off", "always"])
def test_chain_equals_unchained(cuda, case, verify):
    from torch_xdna.conv import IN_CODES, IN_CODES_POOL, IN_FLOAT

    shapes, biased, pools, H, W = CASES[case]
    g = torch.Generator(device=cuda).manual_seed(7 + case)
    layers = _weights(cuda, g, shapes, biased)
    x = torch.randn(3, shapes[0][1], H, W, device=cuda, generator=g)
    cid = _cid(verify=verify)
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
        q, meta = torch.ops.xdna.conv3x3_chain(q, meta, w, b, b is None, cid, b is not None, mode, ra, not last)
        if not last:
            assert q.dtype == (torch.uint8 if b is None else torch.int8) and q.shape[-1] == w.shape[0]
        ra = b is not None
    got = q
    assert got.shape == want.shape and got.dtype == want.dtype
    assert torch.equal(got, want), f"{int((got != want).sum())} of {want.numel()} values differ"


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
