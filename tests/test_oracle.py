"""Pins the oracle (oracle/xdna_oracle.py) to the reference: every function against the golden vectors
that tests/golden/make_golden.py recorded by running the unmodified reference on the CPU.
Bit-exact (SHA-256 of the arrays) for quantised values, int32 sums, scales and dequantised outputs;
1e-5 relative for the fp32 stack logits (the oracle runs in float64). No GPU needed."""

import numpy as np
import pytest

import make_golden as mg
from oracle import xdna_oracle as orc


def _linear_case(ent):
    x, w, b = mg.linear_inputs(ent["seed"], ent["rows"], ent["K"], ent["N"], bias=ent["bias"])
    assert mg.sha(x) == ent["x_sha"] and mg.sha(w) == ent["w_sha"], "inputs did not regenerate"
    xdt = ent["x_dtype"]
    xv = orc.cast(x, xdt)
    wv = orc.cast(w, ent["w_model_dtype"])       # a bf16 module holds bf16 weights
    bv = orc.cast(b, ent["w_model_dtype"]) if b is not None else None
    if ent["transposed"]:
        return orc.linear(xv, [wv.T.copy()], [bv], transposed=True, x_dtype=xdt)
    return orc.linear(xv, [wv], [bv], transposed=False, x_dtype=xdt)


@pytest.mark.parametrize("name", [c[0] for c in mg.LINEAR_CASES])
def test_linear_oracle_matches_reference(golden, name):
    manifest, arrays = golden
    ent = manifest["linear"][name]
    y, acc, sx, sw = _linear_case(ent)
    xq, _ = orc.quant_rows(orc.cast(mg.linear_inputs(ent["seed"], ent["rows"], ent["K"], ent["N"],
                                                     bias=ent["bias"])[0], ent["x_dtype"]))
    assert mg.sha(xq) == ent["xq_sha"]
    assert mg.sha(sx) == ent["sx_sha"]
    assert mg.sha(sw) == ent["sw_sha"]
    assert mg.sha(acc) == ent["acc_sha"]
    assert mg.sha(y.astype(np.float32)) == ent["y_sha"], "dequantised output differs from the reference's"
    if f"linear/{name}/acc" in arrays:
        assert np.array_equal(arrays[f"linear/{name}/acc"], acc)
        assert np.array_equal(arrays[f"linear/{name}/y"], y)


@pytest.mark.parametrize("name", [c[0] for c in mg.CONV_CASES])
def test_conv_oracle_matches_reference(golden, name):
    manifest, arrays = golden
    ent = manifest["conv"][name]
    x, w, b = mg.conv_inputs(ent["seed"], ent["N"], ent["Ci"], ent["Co"], ent["H"], ent["W"], bias=ent["bias"])
    assert mg.sha(x) == ent["x_sha"] and mg.sha(w) == ent["w_sha"]
    r = orc.conv3x3_int8(x, w, b, relu=ent["relu"])
    assert r["shift"] == ent["shift"]
    assert mg.sha(r["xq"]) == ent["xq_sha"] and mg.sha(r["sx"]) == ent["sx_sha"]
    assert mg.sha(r["wq"]) == ent["wq_sha"] and mg.sha(r["sw"]) == ent["sw_sha"]
    assert str(r["q"].dtype) == ent["q_dtype"]
    assert mg.sha(r["q"]) == ent["q_sha"], "requantised integers differ from the reference's CPU integers"
    assert mg.sha(r["scale"]) == ent["scale_sha"]
    assert mg.sha(r["y"]) == ent["y_sha"]
    if f"conv/{name}/q" in arrays:
        assert np.array_equal(arrays[f"conv/{name}/q"], r["q"])


def test_conv_chain_cfg3(golden):
    """BASELINE config 3 as the reference's example runs it: 4 x (conv3x3 256->256 + ReLU), 1x256x64x64."""
    manifest, _ = golden
    ent = manifest["conv"]["cfg3_chain"]
    g = mg.rng(ent["seed"])
    x = g.standard_normal((1, 256, 64, 64), dtype=np.float32)
    ws = [g.standard_normal((256, 256, 3, 3), dtype=np.float32) * np.float32(np.sqrt(2.0 / (256 * 9)))
          for _ in range(4)]
    assert mg.sha(x) == ent["x_sha"]
    h = x
    for i, w in enumerate(ws):
        r = orc.conv3x3_int8(h, w, None, relu=True)
        assert r["shift"] == ent["shifts"][i]
        assert mg.sha(r["q"]) == ent["q_shas"][i]
        h = r["y"]
    assert mg.sha(h) == ent["y_sha"]


@pytest.mark.parametrize("name", [c[0] for c in mg.STACK_CASES])
def test_stack_oracle_matches_fp32_model(golden, name):
    manifest, arrays = golden
    ent = manifest["stack"][name]
    ls, final, head, head_b, x = mg.stack_inputs(ent["seed"], ent["layers"], ent["head_n"], ent["batch"], ent["seq"])
    assert mg.sha(x) == ent["x_sha"]
    mask = mg.causal_mask(ent["batch"], ent["seq"]) if ent["mask"] == "causal" else mg.prefix_mask(ent["lens"], ent["seq"])
    got = orc.qwen3_stack(ls, final, head, head_b, x, mask)
    want = arrays[f"stack/{name}/logits"].astype(np.float64)
    err = np.abs(got - want).max() / np.abs(want).max()
    assert err < 1e-5, err


def test_mask_lengths_restates_reference_classifier():
    """stack.lengths semantics (R:torch_xdna/stack.py:328-352): prefix blocks -> lengths; causal -> None."""
    assert orc.mask_lengths(mg.prefix_mask([40, 29, 17], 40)) == [40, 29, 17]
    assert orc.mask_lengths(mg.causal_mask(2, 16)) is None
    m = mg.prefix_mask([5, 3], 8).astype(np.float32)
    f = np.where(m, 0.0, -1e9).astype(np.float32)
    assert orc.mask_lengths(f) == [5, 3]
    f[0, 0, 0, 7] = -1.0            # neither 0 nor a large negative: not a mask the classifier accepts
    assert orc.mask_lengths(f) is None


def test_bf16_round_half_even():
    v = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -2.5, 65504.0], np.float32)
    r = orc.bf16_round(v)
    assert r[0] == 1.0 and r[1] == 1.0 and r[2] == np.float32(1.0 + 2 ** -6) and r[3] == -2.5


def test_oracle_nan_scale_follows_torch():
    """Non-finite inputs: the reference's scale is torch's x.abs().amax().float().clamp(min=1e-8) / 127
    (R:torch_xdna/runtime.py:146, R:torch_xdna/conv.py:45), which propagates NaN, and so do the oracle's
    per-row and per-image scales (the GPU kernels are checked against them by the -m gpu NaN tests); finite
    rows keep their scales."""
    import torch

    g = mg.rng(5)
    x = g.standard_normal((6, 40)).astype(np.float32)
    x[1, 7] = np.nan
    x[4, 0] = np.inf
    with np.errstate(invalid="ignore"):
        _, s = orc.quant_rows(x)
        _, si = orc.conv_quant(x.reshape(3, 2, 4, 10))
    xt = torch.from_numpy(x)
    want = (xt.abs().amax(dim=1).float().clamp(min=1e-8) / 127).numpy()
    want_img = (xt.view(3, 80).abs().amax(dim=1).float().clamp(min=1e-8) / 127).numpy()
    assert np.isnan(s[1]) and np.isinf(s[4])
    assert np.array_equal(s, want, equal_nan=True)
    assert np.array_equal(si, want_img, equal_nan=True)


@pytest.mark.parametrize("k,stride,h,w", [(3, 1, 9, 11), (1, 1, 7, 5), (1, 2, 7, 6), (3, 2, 9, 10), (3, 2, 8, 8)])
def test_conv_acc_is_the_references_conv2d_call(k, stride, h, w):
    """The oracle's exact sums are the reference's F.conv2d(xq, wq, padding=1) (R:torch_xdna/conv.py:86-87),
    and for the 1x1 / stride-2 extension the same call with the conv's own stride and padding k // 2."""
    import torch

    g = mg.rng(k * 10 + stride)
    xq = g.integers(-127, 128, (2, 5, h, w)).astype(np.int8)
    wq = g.integers(-127, 128, (4, 5, k, k)).astype(np.int8)
    want = torch.nn.functional.conv2d(torch.from_numpy(xq).double(), torch.from_numpy(wq).double(), stride=stride,
                                      padding=k // 2).to(torch.int32).numpy()
    assert np.array_equal(orc.conv_acc(xq, wq, stride), want)


def test_conv_bias_int32_definition():
    """The int32 bias of the optional bias-inside-the-sums route: f32 quotient, ties to even, clamp, NaN -> 0;
    with a zero bias the route gives the reference's values."""
    sw = np.array([0.5, 0.25, 1.0, 2.0, 1.0, 1.0], np.float32)
    sx = np.array([1.0, 0.5], np.float32)
    bias = np.array([1.25, -0.375, 1e12, -1e12, np.nan, 2.5], np.float32)
    b = orc.conv_bias_int32(bias, sw, sx)
    assert b.dtype == np.int32 and b.shape == (2, 6)
    # 1.25 / 0.5 = 2.5 -> 2 (even); -0.375 / 0.25 = -1.5 -> -2; the clamps; NaN -> 0; 2.5 / 1 -> 2
    assert b[0].tolist() == [2, -2, 2 ** 29, -2 ** 29, 0, 2]
    # image 1 (sx 0.5): 1.25 / 0.25 = 5; -0.375 / 0.125 = -3; 2.5 / 0.5 = 5
    assert b[1].tolist() == [5, -3, 2 ** 29, -2 ** 29, 0, 5]
    g = mg.rng(5)
    x = g.standard_normal((2, 6, 7, 5)).astype(np.float32)
    w = (g.standard_normal((4, 6, 3, 3)) * 0.2).astype(np.float32)
    plain = orc.conv3x3_int8(x, w, None, relu=True)
    zero = orc.conv3x3_int8(x, w, np.zeros(4, np.float32), relu=True, bias_int32=True)
    assert np.array_equal(plain["y"], zero["y"]) and plain["shift"] == zero["shift"]
    # the int32 route's values approximate relu(conv + bias) within its rounding
    bias = (g.standard_normal(4) * 0.5).astype(np.float32)
    bi = orc.conv3x3_int8(x, w, bias, relu=True, bias_int32=True)
    fl = orc.conv3x3_int8(x, w, bias, relu=False)
    ref = np.maximum(fl["y"], 0)
    assert np.abs(bi["y"] - ref).max() <= 2 * float((bi["scale"][:, None] * bi["sx"][None, :]).max())


def test_requant_rounds_half_up_and_saturates():
    acc = np.array([[-5, -4, -3, 3, 4, 5, 10 ** 6, -10 ** 6]], np.int32)
    assert orc.requant(acc, 1, False).tolist() == [[-2, -2, -1, 2, 2, 3, 127, -128]]
    assert orc.requant(acc, 1, True).tolist() == [[0, 0, 0, 2, 2, 3, 255, 0]]


# ---------------------------------------------------------------- the torch-CPU port (baseline arm)
@pytest.mark.parametrize("name", ["cfg1", "odd_k200_n300", "qkv_m128", "down_m512"])
def test_reference_cpu_port_linear(golden, name):
    import torch

    from oracle import reference_cpu as rc

    manifest, _ = golden
    ent = manifest["linear"][name]
    x, w, b = mg.linear_inputs(ent["seed"], ent["rows"], ent["K"], ent["N"], bias=ent["bias"])
    xt = torch.from_numpy(x).to(getattr(torch, ent["x_dtype"]))
    wt = torch.from_numpy(w).to(getattr(torch, ent["w_model_dtype"]))
    w_kn, sw = rc.quant_weight(wt)
    bt = torch.from_numpy(b).to(wt.dtype) if b is not None else None
    y = rc.linear_int8(xt, w_kn, sw, bt)
    assert mg.sha(y.float().numpy()) == ent["y_sha"]


@pytest.mark.parametrize("name", [c[0] for c in mg.STACK_CASES])
def test_reference_cpu_port_stack(golden, name):
    import torch

    from oracle import reference_cpu as rc

    manifest, arrays = golden
    ent = manifest["stack"][name]
    ls, final, head, head_b, x = mg.stack_inputs(ent["seed"], ent["layers"], ent["head_n"], ent["batch"], ent["seq"])
    mask = mg.causal_mask(ent["batch"], ent["seq"]) if ent["mask"] == "causal" else mg.prefix_mask(ent["lens"], ent["seq"])
    layers = [{k: torch.from_numpy(v) for k, v in L.items()} for L in ls]
    with torch.no_grad():
        got = rc.qwen3_stack(layers, torch.from_numpy(final), torch.from_numpy(head), torch.from_numpy(head_b),
                             torch.from_numpy(x), torch.from_numpy(mask))
    want = torch.from_numpy(arrays[f"stack/{name}/logits"])
    assert float((got - want).abs().max() / want.abs().max()) < 1e-4


@pytest.mark.parametrize("name", ["odd_3_64_13x37", "odd_64_48_relu"])
def test_reference_cpu_port_conv(golden, name):
    import torch

    from oracle import reference_cpu as rc

    manifest, _ = golden
    ent = manifest["conv"][name]
    x, w, b = mg.conv_inputs(ent["seed"], ent["N"], ent["Ci"], ent["Co"], ent["H"], ent["W"], bias=ent["bias"])
    layer = rc.conv_layer(torch.from_numpy(w), ent["relu"])
    y = rc.conv3x3_int8(torch.from_numpy(x), layer, torch.from_numpy(b) if b is not None else None)
    assert layer["shift"] == ent["shift"]
    assert mg.sha(y.numpy()) == ent["y_sha"]
