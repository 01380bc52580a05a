"""W8A8 linear on the B200 vs the oracle (bit-exact): the quantise kernel, the tcgen05 int8 GEMM with
int32 output and with the dequantising epilogue, the xdna:: ops, torch.compile(backend="xdna"),
and the golden digests recorded from the reference itself."""

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

TORCH_DT = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16}


def t(a, dev, dtype=None):
    x = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return x.to(dtype) if dtype is not None else x


def quant_gpu(x):
    from torch_xdna import kernels

    R, K = x.shape
    xq = torch.zeros((R, kernels.round_up(max(K, 1), 16)), dtype=torch.int8, device=x.device)
    sx = torch.empty((R,), dtype=torch.float32, device=x.device)
    kernels.quant_rows(x, xq, sx)
    return xq, sx


@pytest.mark.parametrize("dtype", ["float32", "bfloat16", "float16"])
@pytest.mark.parametrize("rows,k", [(1, 1024), (37, 200), (699, 300), (513, 3072), (3, 7)])
def test_quant_rows_bitexact(cuda, dtype, rows, k):
    g = mg.rng(rows * 7 + k)
    x = g.standard_normal((rows, k), dtype=np.float32) * np.float32(3.0)
    x[0, : min(k, 4)] = [0.0, -0.0, 1e-9, -7.5][: min(k, 4)]
    if rows > 2:
        x[2] = 0.0          # an all-zero row: scale = 1e-8 / 127, all zeros
    xv = orc.cast(x, dtype)
    xq, sx = quant_gpu(t(xv, cuda, TORCH_DT[dtype]))
    q_ref, s_ref = orc.quant_rows(xv)
    torch.cuda.synchronize()
    assert np.array_equal(sx.cpu().numpy(), s_ref)
    assert np.array_equal(xq[:, :k].cpu().numpy(), q_ref)


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_quant_rows_half_integer_boundaries(cuda, dtype):
    """Values at, and one ulp either side of, (k + 0.5) * scale: where round-half-even of the IEEE
    quotient decides, and where a quotient computed any other way would round differently."""
    g = mg.rng(4242)
    rows, k = 256, 1024
    amax = (g.uniform(0.1, 50.0, rows)).astype(np.float32)
    x = np.zeros((rows, k), np.float32)
    x[:, 0] = amax                                   # fixes each row's scale
    s = (np.maximum(amax, np.float32(1e-8)) / np.float32(127)).astype(np.float32)
    kk = g.integers(-126, 126, (rows, k - 1)).astype(np.float32) + np.float32(0.5)
    base = (kk * s[:, None]).astype(np.float32)
    which = g.integers(0, 3, (rows, k - 1))
    x[:, 1:] = np.where(which == 0, np.nextafter(base, np.float32(-np.inf)),
                        np.where(which == 1, base, np.nextafter(base, np.float32(np.inf))))
    x = np.clip(x, -amax[:, None], amax[:, None])
    xv = orc.cast(x, dtype)
    xq, sx = quant_gpu(t(xv, cuda, TORCH_DT[dtype]))
    q_ref, s_ref = orc.quant_rows(xv)
    assert np.array_equal(sx.cpu().numpy(), s_ref)
    bad = int((xq[:, :k].cpu().numpy() != q_ref).sum())
    assert bad == 0, f"{bad} boundary values rounded differently"


@pytest.mark.parametrize("dtype", ["float32", "bfloat16", "float16"])
def test_quant_rows_edge_scales(cuda, dtype):
    """The division-free quotient against numpy's IEEE division at the scales where a reciprocal product
    is most fragile: rows whose max is below the 1e-8 clamp (scale 1e-8 / 127, so quotients of tiny values),
    subnormal values, values near the type's largest, and rows of one repeated value."""
    g = mg.rng(777)
    rows, k = 64, 512
    x = g.standard_normal((rows, k)).astype(np.float32)
    mag = {"float32": [1e-12, 1e-9, 3e-39, 1e-30, 1e30, 3e38], "bfloat16": [1e-12, 1e-9, 1e-30, 1e30, 3e38],
           "float16": [1e-7, 6e-8, 1e-4, 6e4]}[dtype]
    for i in range(rows):   # each row's max |x| is exactly its magnitude (no overflow to inf)
        x[i] = (x[i] / np.abs(x[i]).max()).astype(np.float32) * np.float32(mag[i % len(mag)])
    x[-1] = np.float32(mag[0])          # every value equal: each quotient is exactly 127
    xv = orc.cast(x, dtype)
    xq, sx = quant_gpu(t(xv, cuda, TORCH_DT[dtype]))
    q_ref, s_ref = orc.quant_rows(xv)
    assert np.array_equal(sx.cpu().numpy(), s_ref)
    assert np.array_equal(xq[:, :k].cpu().numpy(), q_ref)


def test_quant_rows_nan_scale(cuda):
    """A NaN in a row makes that row's scale NaN, as the reference's abs().amax().clamp(min=1e-8) does
    (R:torch_xdna/runtime.py:146); the other rows are unaffected and bit-exact. The int8 codes of a NaN row
    are outside the parity claim (the reference's cast of NaN to int8 is platform-defined)."""
    g = mg.rng(31)
    x = g.standard_normal((48, 1024)).astype(np.float32)
    nan_rows = [3, 17, 40]
    for r in nan_rows:
        x[r, (r * 37) % 1024] = np.nan
    for dtype in ("float32", "bfloat16"):
        xv = orc.cast(x, dtype)
        xq, sx = quant_gpu(t(xv, cuda, TORCH_DT[dtype]))
        got = sx.cpu().numpy()
        assert np.isnan(got[nan_rows]).all()
        keep = [r for r in range(48) if r not in nan_rows]
        q_ref, s_ref = orc.quant_rows(xv[keep])
        assert np.array_equal(got[keep], s_ref)
        assert np.array_equal(xq[keep, :1024].cpu().numpy(), q_ref)


def test_quant_rows_strided_rows(cuda):
    x = torch.randn(64, 2048, device=cuda)[:, :1000]     # ldx 2048, K 1000
    xq, sx = quant_gpu(x)
    q_ref, s_ref = orc.quant_rows(x.cpu().numpy())
    assert np.array_equal(xq[:, :1000].cpu().numpy(), q_ref) and np.array_equal(sx.cpu().numpy(), s_ref)


def gemm_gpu(xq, wq, K, out_dtype, sx=None, sw=None, bias=None):
    from torch_xdna import kernels

    y = torch.empty((xq.shape[0], wq.shape[0]), dtype=out_dtype, device=xq.device)
    kernels.gemm_i8(xq, wq, K, y, sx, sw, bias)
    return y


GEMM_SHAPES = [
    (1, 4096, 1024), (37, 300, 200), (128, 64, 128), (129, 200, 1040), (512, 3072, 1024), (300, 520, 1024),
    (1000, 1000, 1000), (2048, 6144, 1024), (512, 1024, 3072), (4096, 4096, 4096),
    # 256 x 256 tiles on CTA pairs, with a ragged last pair (odd CTA partly / wholly past M)
    (2300, 6144, 1024), (1100, 8192, 512),
    # CTA pairs with a ragged last column tile (columns 3840..3999 of its 256)
    (4096, 4000, 384),
]


@pytest.mark.parametrize("M,N,K", GEMM_SHAPES)
def test_gemm_int32_bitexact(cuda, M, N, K):
    g = mg.rng(M + N + K)
    xq = g.integers(-127, 128, (M, K), dtype=np.int8)
    wq = g.integers(-127, 128, (N, K), dtype=np.int8)
    K16 = -(-K // 16) * 16
    xp = np.zeros((M, K16), np.int8)
    xp[:, :K] = xq
    wp = np.zeros((N, K16), np.int8)
    wp[:, :K] = wq
    acc = gemm_gpu(t(xp, cuda), t(wp, cuda), K, torch.int32)
    want = orc.int_mm(xq, wq)
    got = acc.cpu().numpy()
    bad = int((got != want).sum())
    assert bad == 0, f"{bad} of {want.size} sums differ"


def test_gemm_int32_extremes(cuda):
    """All +-127 operands: the largest sums in magnitude (127*127*K), both signs."""
    M, N, K = 256, 384, 4096
    xq = np.full((M, K), 127, np.int8)
    xq[::2] = -127
    wq = np.full((N, K), 127, np.int8)
    wq[:, ::3] = -127
    acc = gemm_gpu(t(xq, cuda), t(wq, cuda), K, torch.int32).cpu().numpy()
    assert np.array_equal(acc, orc.int_mm(xq, wq))


@pytest.mark.parametrize("out", ["float32", "bfloat16", "float16"])
@pytest.mark.parametrize("bias", [False, True])
@pytest.mark.parametrize("M,N,K", [(37, 300, 200), (512, 3072, 1024), (257, 136, 64), (1100, 8192, 512),
                                   (4096, 4000, 384)])
def test_gemm_dequant_bitexact(cuda, out, bias, M, N, K):
    x, w, b = mg.linear_inputs(M * 3 + N, M, K, N, bias=True)
    xq, sx = orc.quant_rows(x)
    wq, sw = orc.quant_rows(w)
    bias_v = orc.cast(b, out) if bias else None
    K16 = -(-K // 16) * 16
    xp = np.zeros((M, K16), np.int8)
    xp[:, :K] = xq
    wp = np.zeros((N, K16), np.int8)
    wp[:, :K] = wq
    y = gemm_gpu(t(xp, cuda), t(wp, cuda), K, TORCH_DT[out], t(sx, cuda), t(sw, cuda),
                 t(bias_v, cuda, TORCH_DT[out]) if bias else None)
    want = orc.dequant(orc.int_mm(xq, wq), sx, sw, bias_v, out)
    got = y.float().cpu().numpy()
    bad = int((got != want).sum())
    assert bad == 0, f"{bad} of {want.size} dequantised values differ (max abs diff {np.abs(got - want).max()})"


SMALL_M = [(1, 6144, 1024), (1, 1024, 3072), (2, 300, 200), (3, 4096, 1024), (5, 7, 7), (8, 1024, 3072),
           (9, 33, 1040), (17, 520, 1000), (32, 6144, 1024), (31, 100, 16)]


@pytest.mark.parametrize("out", ["int32", "float32", "bfloat16", "float16"])
@pytest.mark.parametrize("M,N,K", SMALL_M)
def test_small_m_gemm_bitexact(cuda, out, M, N, K):
    """M <= 8 rows take the dp4a path of xdna_gemm_i8 (larger M the tensor path): the same sums and the same
    dequantise either way, bit for bit against the oracle. The rows' padding past K holds random bytes, which
    must not count."""
    x, w, b = mg.linear_inputs(M * 7 + N + K, M, K, N, bias=True)
    xq, sx = orc.quant_rows(x)
    wq, sw = orc.quant_rows(w)
    g = mg.rng(M + 3 * N)
    K16 = -(-K // 16) * 16
    xp = g.integers(-128, 128, (M, K16), dtype=np.int8)
    xp[:, :K] = xq
    wp = g.integers(-128, 128, (N, K16), dtype=np.int8)
    wp[:, :K] = wq
    if out == "int32":
        got = gemm_gpu(t(xp, cuda), t(wp, cuda), K, torch.int32).cpu().numpy()
        want = orc.int_mm(xq, wq)
    else:
        bias_v = orc.cast(b, out) if M % 2 else None
        y = gemm_gpu(t(xp, cuda), t(wp, cuda), K, TORCH_DT[out], t(sx, cuda), t(sw, cuda),
                     t(bias_v, cuda, TORCH_DT[out]) if bias_v is not None else None)
        got = y.float().cpu().numpy()
        want = orc.dequant(orc.int_mm(xq, wq), sx, sw, bias_v, out)
    bad = int((got != want).sum())
    assert bad == 0, f"{bad} of {want.size} values differ"


def test_small_m_extremes(cuda):
    """All +-127 operands at M = 4: the largest sums in magnitude through dp4a."""
    M, N, K = 4, 96, 4096
    xq = np.full((M, K), 127, np.int8)
    xq[::2] = -127
    wq = np.full((N, K), 127, np.int8)
    wq[:, ::3] = -127
    acc = gemm_gpu(t(xq, cuda), t(wq, cuda), K, torch.int32).cpu().numpy()
    assert np.array_equal(acc, orc.int_mm(xq, wq))


@pytest.mark.parametrize("name", [c[0] for c in mg.LINEAR_CASES])
def test_reference_golden_digests(cuda, golden, name):
    """The GPU's int32 sums and dequantised outputs hash to exactly what the reference produced."""
    import torch_xdna

    manifest, _ = golden
    ent = manifest["linear"][name]
    x, w, b = mg.linear_inputs(ent["seed"], ent["rows"], ent["K"], ent["N"], bias=ent["bias"])
    assert mg.sha(x) == ent["x_sha"]
    xdt, wdt = TORCH_DT[ent["x_dtype"]], TORCH_DT[ent["w_model_dtype"]]
    xt = t(x, cuda, xdt)
    wt = t(w.T.copy() if ent["transposed"] else w, cuda, wdt)
    bt = t(b, cuda, wdt) if b is not None else None
    cid = torch_xdna.ops.config_id(torch_xdna.Config(verify="off"))
    y = torch.ops.xdna.linear(xt, wt, bt, ent["transposed"], cid)
    xq, sx = quant_gpu(xt)
    acc, sw = torch.ops.xdna.linear_i8(xq[:, : ent["K"]].contiguous(), [wt], ent["transposed"], cid)
    assert mg.sha(xq[:, : ent["K"]].cpu().numpy()) == ent["xq_sha"]
    assert mg.sha(sx.cpu().numpy()) == ent["sx_sha"]
    assert mg.sha(sw.cpu().numpy()) == ent["sw_sha"]
    assert mg.sha(acc.cpu().numpy()) == ent["acc_sha"]
    assert mg.sha(y.float().cpu().numpy()) == ent["y_sha"]


def test_row_sum_property_full_size(cuda):
    """Size-independent check at BASELINE config 2's largest shape (M=8192, gate/up N=6144): the column
    sums of acc equal (column sums of xq) . wq^T exactly (int64)."""
    g = torch.Generator(device=cuda).manual_seed(0)
    M, N, K = 8192, 6144, 1024
    xq = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=cuda, generator=g)
    wq = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=cuda, generator=g)
    acc = gemm_gpu(xq, wq, K, torch.int32)
    lhs = acc.to(torch.int64).sum(0)
    rhs = (xq.to(torch.int64).sum(0)[None, :] * wq.to(torch.int64)).sum(1)
    assert torch.equal(lhs, rhs)
    # and one full row / column against the oracle
    r = 4321
    want_row = orc.int_mm(xq[r:r + 1].cpu().numpy(), wq.cpu().numpy())
    assert np.array_equal(acc[r:r + 1].cpu().numpy(), want_row)


class Net(torch.nn.Module):
    """Odd shapes on purpose (R:tests/test_backend.py:19-31): K=200, N=300, a third GEMM via h @ self.w."""

    def __init__(self):
        super().__init__()
        self.a = torch.nn.Linear(200, 300)
        self.b = torch.nn.Linear(300, 1024, bias=False)
        self.w = torch.nn.Parameter(torch.randn(1024, 520) * 0.03)

    def forward(self, x):
        h = torch.nn.functional.gelu(self.a(x))
        h = torch.nn.functional.silu(self.b(h))
        return h @ self.w


def _run(net, x, **opts):
    import torch_xdna

    torch._dynamo.reset()
    torch_xdna.stats.reset()
    m = torch.compile(net, backend="xdna", options=opts)
    with torch.no_grad():
        return m(x)


@pytest.mark.parametrize("fallback", ["eager", "inductor"])
@pytest.mark.parametrize("rows", [37, 300, 699])
def test_compiled_net_matches_oracle(cuda, rows, fallback):
    """3 GEMMs offloaded; each equals the oracle's W8A8 on the same input, bit for bit; close to fp32."""
    import torch_xdna

    torch.manual_seed(0)
    net = Net().eval().to(cuda)
    x = torch.randn(rows, 200, device=cuda)
    y = _run(net, x, fallback=fallback)
    s = torch_xdna.stats.as_dict()
    assert s["calls"] == {"gpu": 3}, s["calls"]
    with torch.no_grad():
        ref = net(x)
    err = ((y - ref).norm() / ref.norm()).item()
    assert err < 0.03, err
    # oracle chain on the same weights
    a_w, a_b = net.a.weight.detach().cpu().numpy(), net.a.bias.detach().cpu().numpy()
    h, *_ = orc.linear(x.cpu().numpy(), [a_w], [a_b])
    h = torch.nn.functional.gelu(torch.from_numpy(h).to(cuda))
    h2, *_ = orc.linear(h.cpu().numpy(), [net.b.weight.detach().cpu().numpy()], [None])
    h2 = torch.nn.functional.silu(torch.from_numpy(h2).to(cuda))
    want, *_ = orc.linear(h2.cpu().numpy(), [net.w.detach().cpu().numpy()], [None], transposed=True)
    if fallback == "eager":
        assert np.array_equal(y.cpu().numpy(), want)
    else:   # Inductor's own gelu/silu may differ in the last bit from eager's: compare closely
        assert np.abs(y.cpu().numpy() - want).max() <= 1e-3 * np.abs(want).max()


class Attn(torch.nn.Module):
    """q/k/v read the same input -> one fused GEMM; o reads another (R:tests/test_backend.py:97-109)."""

    def __init__(self):
        super().__init__()
        self.q = torch.nn.Linear(256, 256)
        self.k = torch.nn.Linear(256, 128, bias=False)
        self.v = torch.nn.Linear(256, 128)
        self.o = torch.nn.Linear(256, 256)

    def forward(self, x):
        q, k, v = self.q(x), self.k(x), self.v(x)
        return self.o(q * torch.cat([k, v], -1).sigmoid())


def test_fusion_counts_and_bits(cuda):
    import torch_xdna

    torch.manual_seed(0)
    net = Attn().eval().to(cuda)
    x = torch.randn(200, 256, device=cuda)
    with torch.no_grad():
        ref = net(x)
    y = _run(net, x, fallback="eager")
    fused = torch_xdna.stats.as_dict()["calls"]
    y2 = _run(net, x, fallback="eager", fuse=False)
    unfused = torch_xdna.stats.as_dict()["calls"]
    assert fused == {"gpu": 2} and unfused == {"gpu": 4}, (fused, unfused)
    assert torch.equal(y, y2), "one fused GEMM and three separate ones give different bits"
    assert ((y - ref).norm() / ref.norm()).item() < 0.03


def test_bf16_linear_cat_projection_set(cuda):
    """BASELINE config 2 shapes through xdna::linear_cat (qkv 16x128 + 2x8x128, gate/up), bf16, M=512."""
    import torch_xdna

    cid = torch_xdna.ops.config_id(torch_xdna.Config(verify="off"))
    g = mg.rng(77)
    x = g.standard_normal((512, 1024), dtype=np.float32)
    ws = [g.standard_normal((n, 1024), dtype=np.float32) * np.float32(0.02) for n in (2048, 1024, 1024)]
    xb = orc.bf16_round(x)
    wb = [orc.bf16_round(w) for w in ws]
    y = torch.ops.xdna.linear_cat(t(xb, cuda, torch.bfloat16), [t(w, cuda, torch.bfloat16) for w in wb],
                                  [None, None, None], cid)
    want, *_ = orc.linear(xb, wb, None, x_dtype="bfloat16")
    assert np.array_equal(y.float().cpu().numpy(), want)


@pytest.mark.parametrize("dtype", ["float32", "bfloat16", "float16"])
@pytest.mark.parametrize("rows,n,k,bias", [(512, 4096, 1024, False), (300, 1000, 333, True), (1, 6, 7, True),
                                           (129, 3072, 1024, True)])
def test_precision_bf16_linear(cuda, dtype, rows, n, k, bias):
    """precision="bf16": bf16 operands, f32 accumulate, bias in f32, one rounding to x.dtype — against the
    f32 product of the same bf16-rounded operands (bf16 out: within its half-ulp; f32/f16: 1e-5 / 1e-3)."""
    import torch_xdna

    cid = torch_xdna.ops.config_id(torch_xdna.Config(precision="bf16", verify="first"))
    g = torch.Generator(device=cuda).manual_seed(rows * n + k)
    dt = TORCH_DT[dtype]
    x = torch.randn(rows, k, device=cuda, generator=g).to(dt)
    w = (torch.randn(n, k, device=cuda, generator=g) * 0.05).to(dt)
    b = torch.randn(n, device=cuda, generator=g).to(dt) if bias else None
    y = torch.ops.xdna.linear(x, w, b, False, cid)
    assert y.dtype == dt and y.shape == (rows, n) and y.is_contiguous()
    want = x.bfloat16().double() @ w.bfloat16().double().t()
    if b is not None:
        want = want + b.double()
    err = ((y.double() - want).abs().max() / want.abs().max()).item()
    assert err < {"bfloat16": 8e-3, "float16": 1e-3, "float32": 1e-5}[dtype], err
    yt = torch.ops.xdna.linear(x, w.t().contiguous(), b, True, cid)       # x @ W with W [K, N]
    assert torch.equal(yt, y)


def test_precision_bf16_linear_cat_and_compile(cuda):
    """precision="bf16" through torch.compile: the fused q/k/v GEMM equals three separate bf16 GEMMs."""
    import torch_xdna

    torch.manual_seed(1)
    net = Attn().eval().to(cuda)
    x = torch.randn(200, 256, device=cuda)
    with torch.no_grad():
        ref = net(x)
    y = _run(net, x, precision="bf16")
    assert torch_xdna.stats.as_dict()["calls"] == {"gpu": 2}
    assert ((y - ref).norm() / ref.norm()).item() < 1e-2


def test_verify_first_passes_and_records(cuda):
    import torch_xdna
    from torch_xdna import runtime

    runtime._verified.clear()
    torch_xdna.stats.reset()
    cid = torch_xdna.ops.config_id(torch_xdna.Config(verify="first"))
    x = torch.randn(77, 333, device=cuda)
    w = torch.randn(100, 333, device=cuda) * 0.05
    torch.ops.xdna.linear(x, w, None, False, cid)
    torch.ops.xdna.linear(x, w, None, False, cid)
    checks = torch_xdna.stats.as_dict()["checks"]
    assert len(checks) == 1 and "bitwise" in checks[0][1], checks


def test_empty_rows(cuda):
    import torch_xdna

    cid = torch_xdna.ops.config_id(torch_xdna.Config())
    y = torch.ops.xdna.linear(torch.empty(0, 64, device=cuda), torch.randn(32, 64, device=cuda), None, False, cid)
    assert y.shape == (0, 32)
    acc, sw = torch.ops.xdna.linear_i8(torch.empty(0, 64, dtype=torch.int8, device=cuda),
                                       [torch.randn(32, 64, device=cuda)], False, cid)
    assert acc.shape == (0, 32) and acc.dtype == torch.int32 and sw.shape == (32,)


def test_no_device_error_recorded(cuda):
    from torch_xdna import kernels

    assert kernels.take_device_error() == (0, 0)
