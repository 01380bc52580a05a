"""Host-side layouts and rebuilds that the kernels rely on, checked on the CPU: the RoPE table layout the
q/k/v epilogue reads, the float activation a chain of convs' int8 codes stands for (the verify path's
CPU rebuild, against a numpy restatement of the conv epilogue's arithmetic and against the oracle's conv
outputs), and which max-pools the conv chaining pass takes into a chain."""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from torch_xdna import backend, conv, kernels


def test_rope_layout_index():
    """Frequency d of position p sits at (d / 4) * L * 4 + p * 4 + d % 4 (the header's layout)."""
    L = 37
    t = torch.arange(L * 64, dtype=torch.float32).reshape(L, 64)
    flat = kernels.rope_layout(t).reshape(-1)
    assert flat.shape[0] == L * 64
    for p in (0, 1, 17, L - 1):
        for d in (0, 3, 4, 31, 63):
            assert flat[(d // 4) * L * 4 + p * 4 + d % 4] == t[p, d]


def _epilogue_f32(q, scale, sx, bias, relu_after):
    """numpy f32 restatement of the dequantising epilogue: float(q) * (scale[c] * sx[n]) + bias[c], each
    operation rounded to f32, then max(y, 0)."""
    n, h, w, c = q.shape
    t = (scale[None, :].astype(np.float32) * sx[:, None].astype(np.float32)).astype(np.float32)
    y = (q.astype(np.float32) * t[:, None, None, :]).astype(np.float32)
    y = (y + bias[None, None, None, :].astype(np.float32)).astype(np.float32)
    if relu_after:
        y = np.maximum(y, np.float32(0))
    return y


@pytest.mark.parametrize("unsigned,relu_after,pool", [(False, True, False), (False, True, True),
                                                      (False, False, True), (True, False, True)])
def test_codes_to_float_matches_epilogue_arithmetic(unsigned, relu_after, pool):
    g = np.random.default_rng(3)
    n, h, w, c = 2, 7, 9, 12
    q = (g.integers(0, 256, (n, h, w, c)) if unsigned else g.integers(-128, 128, (n, h, w, c)))
    q = q.astype(np.uint8 if unsigned else np.int8)
    sx = g.random(n, dtype=np.float32) * np.float32(0.1) + np.float32(1e-3)
    scale = g.random(c, dtype=np.float32) * np.float32(0.05) + np.float32(1e-4)
    bias = np.zeros(c, np.float32) if unsigned else (g.standard_normal(c).astype(np.float32) * np.float32(0.1))
    meta = torch.from_numpy(np.concatenate([sx, scale, bias]))
    got = conv.codes_to_float(torch.from_numpy(q), meta, relu_after, pool).numpy()
    y = _epilogue_f32(q, scale, sx, bias, relu_after)            # NHWC
    if pool:  # 2x2, stride 2, rounding the size down
        hh, ww = h // 2, w // 2
        y = y[:, :2 * hh, :2 * ww].reshape(n, hh, 2, ww, 2, c).max(axis=(2, 4))
    want = y.transpose(0, 3, 1, 2)
    assert got.shape == want.shape
    assert np.array_equal(got, want)
    # pooling the codes first gives the same values: the value grows with the code
    if pool:
        qp = q[:, :2 * (h // 2), :2 * (w // 2)].reshape(n, h // 2, 2, w // 2, 2, c).max(axis=(2, 4))
        assert np.array_equal(_epilogue_f32(qp, scale, sx, bias, relu_after).transpose(0, 3, 1, 2), want)


def _pool_node(*args, **kwargs):
    g = torch.fx.Graph()
    x = g.placeholder("x")
    return g.call_function(F.max_pool2d, (x, *args), kwargs)


@pytest.mark.parametrize("args,kwargs,ok", [
    ((2,), {}, True), ((2, 2), {}, True), (((2, 2), (2, 2), 0, 1), {}, True), ((2,), {"stride": None}, True),
    ((3,), {}, False), ((2, 1), {}, False), ((2, 2, 1), {}, False), ((2,), {"ceil_mode": True}, False),
    ((2,), {"dilation": 2}, False), ((2,), {"return_indices": True}, False),
])
def test_maxpool_pattern(args, kwargs, ok):
    assert backend._is_maxpool_2x2(_pool_node(*args, **kwargs)) is ok


@pytest.mark.parametrize("bias,relu,pool", [(True, False, False), (True, False, True), (False, True, True)])
def test_codes_rebuild_the_oracle_conv_output(bias, relu, pool):
    """A conv's codes and factors, as the chain passes them, rebuild exactly the float output the oracle
    (the reference's CPU route, pinned to its goldens) computes, after the graph's ReLU and max-pool."""
    from oracle import xdna_oracle as orc

    g = np.random.default_rng(5)
    x = g.standard_normal((2, 12, 10, 14)).astype(np.float32)
    w = (g.standard_normal((16, 12, 3, 3)) * 0.15).astype(np.float32)
    b = (g.standard_normal(16) * 0.1).astype(np.float32) if bias else None
    r = orc.conv3x3_int8(x, w, b, relu=relu)
    y = torch.from_numpy(np.asarray(r["y"], np.float32))
    if bias:                       # a biased conv's ReLU stays in the graph after it
        y = torch.relu(y)
    if pool:
        y = F.max_pool2d(y, 2)
    q = torch.from_numpy(np.ascontiguousarray(np.asarray(r["q"]).transpose(0, 2, 3, 1)))   # NHWC codes
    meta = conv.codes_meta(torch.from_numpy(r["sx"].astype(np.float32)), torch.from_numpy(r["scale"]),
                           torch.from_numpy(b) if bias else None, 16)
    got = conv.codes_to_float(q, meta, relu_after=bias, pool=pool)
    assert got.dtype == torch.float32 and torch.equal(got, y)


@pytest.mark.parametrize("bint", [False, True])
@pytest.mark.parametrize("out_pool", [False, True])
@pytest.mark.parametrize("kind", ["relu_after_bias", "fused_relu", "signed_biased"])
def test_chain_fake_matches_the_op(kind, out_pool, bint):
    """xdna::conv3x3_chain's shape function (what torch.compile traces with) gives the codes' dtype and the
    meta vector's length the op produces: [sx, scale, bias] plus the next layer's maxima (one word more when
    the next conv pools) exactly when the producer can compute them (conv.next_amax_ok), the int32-bias
    option turning a ReLU after the bias into uint8 codes."""
    import torch_xdna
    from torch._subclasses.fake_tensor import FakeTensorMode

    n, ci, co, h, w = 2, 64, 32, 10, 12
    relu, post_relu = (False, True) if kind == "relu_after_bias" else (True, False) if kind == "fused_relu" \
        else (False, False)
    has_bias = kind != "fused_relu"
    cid = torch_xdna.ops.config_id(torch_xdna.Config(conv_bias_int32=bint))
    cfg = torch_xdna.ops._configs[cid]
    with FakeTensorMode():
        x = torch.empty((n, h, w, ci), dtype=torch.int8)
        xmeta = torch.empty((n + 2 * ci,), dtype=torch.float32)
        wt = torch.empty((co, ci, 3, 3))
        b = torch.empty((co,)) if has_bias else None
        q, meta = torch.ops.xdna.conv3x3_chain(x, xmeta, wt, b, relu, cid, post_relu, conv.IN_CODES, True, True,
                                               out_pool)
    erelu, epost = conv.effective_relu(cfg, relu, b, post_relu)
    fbias = None if conv.int32_bias(cfg, b) else b
    assert q.shape == (n, h, w, co) and q.dtype == (torch.uint8 if erelu else torch.int8)
    extra = n + (1 if out_pool else 0) if conv.next_amax_ok(erelu, fbias, epost, out_pool) else 0
    assert meta.numel() == n + 2 * co + extra
    # the consumer tells from the length alone whether the maxima are there (and cover a pool's region)
    assert (meta.numel() == 2 * n + 2 * co + (1 if out_pool else 0)) == bool(extra)
