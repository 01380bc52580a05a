"""Parity at BASELINE.json's stated configurations, not scaled-down ones.

- config 5: the whole Qwen3-0.6B stack at 16 sequences x 1024 tokens, 28 layers, causal mask, the
  151936-wide head, token ids embedded by xdna_embed -- the logits of two full sequences (every column,
  the ragged last column tile included) against the fp32 model the reference checks its stack against
  (R:torch_xdna/stack.py:444-460), within the bf16 tolerance max|got - ref| <= 2e-2 * max|ref|;
- xdna_embed: the token-id gather, bit for bit, ids at both ends of the vocabulary;
- config 4: VGG16's 13 biased conv3x3 layers with ReLU and 2x2 max-pools on 2 images of 224 x 224,
  compiled by the backend (int8 codes chained between convs), against the oracle applied layer by layer
  (R:torch_xdna/conv.py:43-51 per conv, torch's ReLU and max-pool between): bit-exact.
"""

import numpy as np
import pytest
import torch

from oracle import xdna_oracle as orc

pytestmark = pytest.mark.gpu
VOCAB = 151936


@pytest.fixture(autouse=True)
def _inference(request):
    from torch_xdna import kernels

    if "cuda" in request.fixturenames:
        kernels.take_device_error()
    with torch.no_grad():
        yield
    if "cuda" in request.fixturenames:
        assert kernels.take_device_error() == (0, 0), "a kernel recorded a device-side error"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_embed_gather_bitexact(cuda, dtype):
    from torch_xdna import kernels

    g = torch.Generator(device=cuda).manual_seed(21)
    table = torch.randn(VOCAB, 1024, device=cuda, generator=g).to(dtype)
    ids = torch.randint(0, VOCAB, (4099,), device=cuda, generator=g)
    ids[:7] = torch.tensor([0, 1, VOCAB - 1, VOCAB - 2, VOCAB - 3, 151935, 75968], device=cuda)
    x = torch.full((ids.numel(), 1024), float("nan"), device=cuda)
    kernels.embed(ids, table, x)
    assert torch.equal(x, table[ids].float())


def test_embed_out_of_range_ids_give_zeros_and_an_error(cuda):
    from torch_xdna import kernels

    table = torch.randn(1000, 1024, device=cuda).to(torch.bfloat16)
    ids = torch.tensor([5, -1, 999, 1000, 7], device=cuda)
    x = torch.full((5, 1024), 3.0, device=cuda)
    kernels.embed(ids, table, x)
    code, _ = kernels.take_device_error()
    assert code == -1, code                        # XDNA_ERR_INVALID recorded for the host to read
    assert not x[1].any() and not x[3].any()
    assert torch.equal(x[[0, 2, 4]], table[ids[[0, 2, 4]]].float())
    assert kernels.take_device_error() == (0, 0)   # read and cleared


def test_cfg5_full_stack_vs_fp32_model(cuda):
    """BASELINE config 5 at its stated size, through xdna_embed and xdna_qwen3_stack (the kernels the op runs),
    with non-trivial norm weights; sequences 0 and 15 against the fp32 model on the same bf16 weights."""
    from oracle import reference_cpu as rc
    from torch_xdna import kernels
    from torch_xdna import stack as xstack

    torch.backends.cuda.matmul.allow_tf32 = False
    B, L, NL = 16, 1024, 28
    g = torch.Generator(device=cuda).manual_seed(5)

    def w(*s):   # bf16 weights, kept as their exact f32 values for the reference
        return (torch.randn(*s, device=cuda, generator=g) * 0.02).to(torch.bfloat16).float()

    def norm(n):
        return 1 + 0.1 * torch.randn(n, device=cuda, generator=g)

    ts, ls = [], []
    for _ in range(NL):
        lw = dict(q=w(2048, 1024), k=w(1024, 1024), v=w(1024, 1024), o=w(1024, 2048), gate=w(3072, 1024),
                  up=w(3072, 1024), down=w(1024, 3072), input_norm=norm(1024), post_norm=norm(1024), q_norm=norm(128),
                  k_norm=norm(128))
        ls.append(lw)
        ts += [lw[k] for k in xstack.LAYER_KEYS]
    final, head = norm(1024), w(VOCAB, 1024)
    inv_freq = 1.0 / (1e6 ** (torch.arange(0, 128, 2, dtype=torch.float32, device=cuda) / 128))
    pk = xstack.Packed(ts + [final, head, inv_freq], NL, None)
    table = (torch.randn(VOCAB, 1024, device=cuda, generator=g) * 0.5).to(torch.bfloat16)
    ids = torch.randint(0, VOCAB, (B * L,), device=cuda, generator=g)
    ids[L - 3:L] = torch.tensor([VOCAB - 1, 0, VOCAB - 2], device=cuda)
    x = torch.empty(B * L, 1024, device=cuda)
    kernels.embed(ids, table, x)
    seqs = [0, B - 1]
    x_ref = torch.stack([table[ids[s * L:(s + 1) * L]].float() for s in seqs])
    assert torch.equal(x.view(B, L, 1024)[seqs], x_ref)
    cos, sin = pk.rope(L)
    out = torch.empty(B * L, VOCAB, dtype=torch.bfloat16, device=cuda)
    ws = torch.empty(kernels.qwen3_stack_workspace(B, L), dtype=torch.uint8, device=cuda)
    kernels.qwen3_stack(pk.table, pk.final_norm, pk.head, None, cos, sin, 1e-6, x, B, L, kernels.MASK_CAUSAL, None,
                        None, out, ws)
    got = out.view(B, L, VOCAB)[seqs].float()
    del out, ws
    mask = torch.ones(L, L, dtype=torch.bool, device=cuda).tril()[None, None].expand(len(seqs), 1, L, L)
    want = rc.qwen3_stack(ls, final, head, None, x_ref, mask)
    assert torch.isfinite(got).all()
    rel = float((got - want).abs().max() / want.abs().max())
    assert rel < 2e-2, rel
    # the ragged last column tile (151936 = 593 x 256 + 128) on its own
    tail = slice(VOCAB - 128, VOCAB)
    rel_tail = float((got[..., tail] - want[..., tail]).abs().max() / want.abs().max())
    assert rel_tail < 2e-2, rel_tail


VGG16 = [64, 64, "M", 128, 128, "M", 256, 256, 256, "M", 512, 512, 512, "M", 512, 512, 512, "M"]


class VGG16Features(torch.nn.Module):
    """The conv part of VGG16: 3x3 convs with bias, each followed by ReLU, 2x2 max-pools."""

    def __init__(self, g):
        super().__init__()
        mods, ci = [], 3
        for v in VGG16:
            if v == "M":
                mods.append(torch.nn.MaxPool2d(2))
                continue
            c = torch.nn.Conv2d(ci, v, 3, padding=1)
            c.weight.data = torch.randn(v, ci, 3, 3, generator=g) * (2.0 / (ci * 9)) ** 0.5
            c.bias.data = torch.randn(v, generator=g) * 0.01
            mods += [c, torch.nn.ReLU()]
            ci = v
        self.features = torch.nn.Sequential(*mods)

    def forward(self, x):
        return self.features(x)


def _maxpool2(h):
    n, c, hh, ww = h.shape
    return h[:, :, :hh // 2 * 2, :ww // 2 * 2].reshape(n, c, hh // 2, 2, ww // 2, 2).max(axis=(3, 5))


def test_cfg4_vgg16_compiled_chain_vs_oracle(cuda):
    """Two 224 x 224 images through the compiled VGG16 conv stack: the backend offloads all 13 convs and
    chains them on int8 codes through ReLU and the max-pools; the output equals the oracle's layer-by-layer
    result bit for bit (every layer's shift fixed from image 0, as the reference does)."""
    import torch_xdna

    g = torch.Generator().manual_seed(7)
    net = VGG16Features(g).eval()
    x = torch.randn(2, 3, 224, 224, generator=torch.Generator().manual_seed(8))
    h = x.numpy()
    for m in net.features:
        if isinstance(m, torch.nn.Conv2d):
            r = orc.conv3x3_int8(h, m.weight.detach().numpy(), m.bias.detach().numpy(), relu=False)
            h = r["y"]
        elif isinstance(m, torch.nn.ReLU):
            h = np.maximum(h, np.float32(0))
        else:
            h = _maxpool2(h)
    torch._dynamo.reset()
    torch_xdna.stats.reset()
    comp = torch.compile(net.to(cuda), backend="xdna", options={"fallback": "eager", "verify": "off"})
    y = comp(x.to(cuda))
    s = torch_xdna.stats.as_dict()
    assert s["calls"]["gpu"] == 13, s["calls"]
    assert np.array_equal(y.cpu().numpy(), h), f"{int((y.cpu().numpy() != h).sum())} of {h.size} values differ"
