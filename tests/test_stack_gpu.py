"""The Qwen3 stack on the B200: each bf16 kernel against an fp32 torch restatement of the same op, and the
whole compiled stack against the golden logits of the reference's fp32 model check (the bf16 tolerance
of BASELINE config 5: max |got - ref| <= 2e-2 * max |ref|)."""

import numpy as np
import pytest
import torch

import make_golden as mg

pytestmark = pytest.mark.gpu
TOL = 2e-2   # logits: max-abs relative to the fp32 model


@pytest.fixture(autouse=True)
def _inference(request):
    """Inference only; each test starts with a clear device error word and must leave it clear."""
    from torch_xdna import kernels

    if "cuda" in request.fixturenames:
        kernels.take_device_error()
    with torch.no_grad():
        yield
    if "cuda" in request.fixturenames:
        assert kernels.take_device_error() == (0, 0), "a kernel recorded a device-side timeout"


def rel_max(got, want):
    return float((got.float() - want.float()).abs().max() / want.float().abs().max())


def bf(t):
    return t.to(torch.bfloat16)


def test_rmsnorm(cuda):
    from torch_xdna import kernels

    x = torch.randn(301, 1024, device=cuda) * 3
    w = 1 + 0.1 * torch.randn(1024, device=cuda)
    y = torch.empty(301, 1024, dtype=torch.bfloat16, device=cuda)
    kernels.rmsnorm_bf16(x, w, 1e-6, y)
    want = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * w
    assert rel_max(y, want) < 8e-3


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("M,N,K", [(333, 520, 1000), (128, 64, 64), (1, 4096, 1024), (1030, 1024, 3072),
                                   (2300, 8192, 1024)])  # the last: 256 x 256 tiles on CTA pairs
def test_gemm_bf16_f32acc(cuda, out_dtype, M, N, K):
    from torch_xdna import kernels

    a = bf(torch.randn(M, K, device=cuda))
    b = bf(torch.randn(N, K, device=cuda) * 0.05)
    bias = torch.randn(N, device=cuda) * 0.1
    out = torch.empty(M, N, dtype=out_dtype, device=cuda)
    kernels.gemm_bf16(a, b, kernels.GEMM_F32ACC, out=out, bias=bias)
    want = a.float() @ b.float().t() + bias
    assert rel_max(out, want) < (1e-4 if out_dtype == torch.float32 else 8e-3)


@pytest.mark.parametrize("parts,rows,N", [(1, 256, 1024), (2, 1024, 2048), (3, 2048, 4096), (2, 128, 520)])
def test_gemm_bf16_gather(cuda, parts, rows, N):
    """The head GEMM over A split by rows into several buffers (the fused all-gather of the column-parallel
    head; here every part is on this GPU): equals one GEMM over the concatenated rows."""
    from torch_xdna import kernels

    g = torch.Generator(device=cuda).manual_seed(parts * rows + N)
    bufs = [bf(torch.randn(rows, 1024, device=cuda, generator=g)) for _ in range(parts)]
    w = bf(torch.randn(N, 1024, device=cuda, generator=g) * 0.03)
    out = torch.empty(parts * rows, N, dtype=torch.bfloat16, device=cuda)
    maps = torch.empty(parts * 128, dtype=torch.uint8, device=cuda)
    kernels.gemm_bf16_gather(bufs, rows, 1024, w, out, maps)
    want = torch.empty_like(out)
    kernels.gemm_bf16(torch.cat(bufs), w, kernels.GEMM_F32ACC, out=want)
    assert torch.equal(out, want)
    assert rel_max(out, torch.cat(bufs).float() @ w.float().t()) < 8e-3


def test_ipc_allocation_and_handle(cuda):
    """The shareable allocation of the fused head's parts: usable as a tensor, a 64-byte handle, freed."""
    from torch_xdna import kernels

    t, ptr = kernels.ipc_alloc((256, 1024), cuda)
    t.copy_(torch.ones(256, 1024, dtype=torch.bfloat16, device=cuda))
    assert t.data_ptr() == ptr and float(t.float().sum()) == 256 * 1024
    h = kernels.ipc_handle(ptr)
    assert len(h) == 64 and any(h)
    del t
    kernels.ipc_free(ptr)


@pytest.mark.parametrize("M", [700, 8300])  # 8300: CTA pairs
def test_gemm_bf16_residual(cuda, M):
    from torch_xdna import kernels

    a = bf(torch.randn(M, 2048, device=cuda))
    b = bf(torch.randn(1024, 2048, device=cuda) * 0.02)
    resid = torch.randn(M, 1024, device=cuda)
    want = resid + a.float() @ b.float().t()
    kernels.gemm_bf16(a, b, kernels.GEMM_RESID, resid=resid)
    assert rel_max(resid, want) < 1e-5


@pytest.mark.parametrize("M", [500, 1000])  # 1000: CTA pairs
def test_gemm_bf16_swiglu(cuda, M):
    from torch_xdna import kernels

    h = bf(torch.randn(M, 1024, device=cuda))
    gate = bf(torch.randn(3072, 1024, device=cuda) * 0.03)
    up = bf(torch.randn(3072, 1024, device=cuda) * 0.03)
    gu = torch.stack([gate.reshape(96, 32, 1024), up.reshape(96, 32, 1024)], dim=1).reshape(6144, 1024).contiguous()
    act = torch.empty(M, 3072, dtype=torch.bfloat16, device=cuda)
    kernels.gemm_bf16(h, gu, kernels.GEMM_SWIGLU, out=act)
    g, u = h.float() @ gate.float().t(), h.float() @ up.float().t()
    want = torch.nn.functional.silu(g) * u
    assert rel_max(act, want) < 1e-2


def _rope_tables(L, dev, theta=1e6):
    inv = 1.0 / (theta ** (torch.arange(0, 128, 2, dtype=torch.float32, device=dev) / 128))
    f = torch.arange(L, dtype=torch.float32, device=dev)[:, None] * inv[None, :]
    return f.cos().contiguous(), f.sin().contiguous()


def _qkv_ref(h, wq, wk, wv, qn, kn, cos, sin, L, eps=1e-6):
    """transformers' Qwen3 q/k/v: per-head RMSNorm of q and k, then RoPE (half rotation)."""
    T = h.shape[0]
    q = (h.float() @ wq.float().t()).view(T, 16, 128)
    k = (h.float() @ wk.float().t()).view(T, 8, 128)
    v = (h.float() @ wv.float().t()).view(T, 8, 128)
    q = q * torch.rsqrt(q.pow(2).mean(-1, keepdim=True) + eps) * qn
    k = k * torch.rsqrt(k.pow(2).mean(-1, keepdim=True) + eps) * kn
    pos = torch.arange(T, device=h.device) % L
    c = torch.cat([cos, cos], -1)[pos][:, None, :]
    s = torch.cat([sin, sin], -1)[pos][:, None, :]

    def rot(t):
        return torch.cat([-t[..., 64:], t[..., :64]], -1)

    return q * c + rot(q) * s, k * c + rot(k) * s, v


def _project(h, L, dev, g):
    wq = bf(torch.randn(2048, 1024, device=dev, generator=g) * 0.02)
    wk = bf(torch.randn(1024, 1024, device=dev, generator=g) * 0.02)
    wv = bf(torch.randn(1024, 1024, device=dev, generator=g) * 0.02)
    qn = 1 + 0.1 * torch.randn(128, device=dev, generator=g)
    kn = 1 + 0.1 * torch.randn(128, device=dev, generator=g)
    return wq, wk, wv, qn, kn


@pytest.mark.parametrize("B,L", [(3, 100), (5, 256), (13, 100)])  # the last two: CTA pairs (V^T by TMA / direct)
def test_gemm_bf16_qkv_norm_rope(cuda, B, L):
    from torch_xdna import kernels

    g = torch.Generator(device=cuda).manual_seed(3)
    T = B * L
    h = bf(torch.randn(T, 1024, device=cuda, generator=g))
    wq, wk, wv, qn, kn = _project(h, L, cuda, g)
    cos, sin = _rope_tables(L, cuda)
    qk = torch.empty(T, 3072, dtype=torch.bfloat16, device=cuda)
    L8 = -(-L // 8) * 8           # V^T: every sequence starts at a multiple of 8 columns
    vt = torch.zeros(1024, B * L8, dtype=torch.bfloat16, device=cuda)
    kernels.gemm_bf16(h, torch.cat([wq, wk, wv]).contiguous(), kernels.GEMM_QKV, out=qk, vt=vt,
                      rope_cos=kernels.rope_layout(cos), rope_sin=kernels.rope_layout(sin), q_norm=qn, k_norm=kn,
                      seq_len=L)
    q, k, v = _qkv_ref(h, wq, wk, wv, qn, kn, cos, sin, L)
    assert rel_max(qk[:, :2048].view(T, 16, 128), q) < 1e-2
    assert rel_max(qk[:, 2048:].view(T, 8, 128), k) < 1e-2
    v_got = vt.view(1024, B, L8)[:, :, :L].reshape(1024, T).t().reshape(T, 8, 128)
    assert rel_max(v_got, v) < 1e-2
    assert not vt.view(1024, B, L8)[:, :, L:].any(), "padding columns of V^T were written"


def _attention_ref(qk, vt, B, L, allowed):
    """fp32 SDPA on the same bf16 q / k / v (GQA: q head h reads kv head h // 2)."""
    T = B * L
    L8 = -(-L // 8) * 8
    q = qk[:, :2048].float().view(B, L, 16, 128).transpose(1, 2)
    k = qk[:, 2048:].float().view(B, L, 8, 128).transpose(1, 2).repeat_interleave(2, 1)
    v = vt.view(1024, B, L8)[:, :, :L].float().reshape(1024, T).t().reshape(B, L, 8, 128)
    v = v.transpose(1, 2).repeat_interleave(2, 1)
    o = torch.nn.functional.scaled_dot_product_attention(q, k, v, attn_mask=allowed)
    return o.transpose(1, 2).reshape(T, 2048)


@pytest.mark.parametrize("kind", ["causal", "prefix", "bool", "none"])
@pytest.mark.parametrize("B,L", [(2, 256), (3, 200), (1, 1024), (3, 100)])
def test_attention(cuda, kind, B, L):
    from torch_xdna import kernels

    g = torch.Generator(device=cuda).manual_seed(B * L)
    T = B * L
    L8 = -(-L // 8) * 8
    qk = bf(torch.randn(T, 3072, device=cuda, generator=g))
    vt = bf(torch.randn(1024, B * L8, device=cuda, generator=g))
    lens = mask = None
    if kind == "causal":
        allowed = torch.ones(L, L, dtype=torch.bool, device=cuda).tril()[None, None].expand(B, 1, L, L)
        mk = kernels.MASK_CAUSAL
    elif kind == "none":
        allowed = torch.ones(B, 1, L, L, dtype=torch.bool, device=cuda)
        mk = kernels.MASK_NONE
    elif kind == "prefix":
        ln = [L - 7 * b - 1 for b in range(B)]
        allowed = torch.from_numpy(mg.prefix_mask(ln, L)).to(cuda)
        lens = torch.tensor(ln, dtype=torch.int32, device=cuda)
        mk = kernels.MASK_PREFIX
    else:
        allowed = torch.rand(B, 1, L, L, device=cuda, generator=g) < 0.7
        allowed |= torch.eye(L, dtype=torch.bool, device=cuda)
        mask = allowed.to(torch.uint8).contiguous()
        mk = kernels.MASK_BOOL
    out = torch.empty(T, 2048, dtype=torch.bfloat16, device=cuda)
    kernels.attention(qk, vt, out, B, L, mk, lens=lens, mask=mask)
    want = _attention_ref(qk, vt, B, L, allowed)
    assert rel_max(out, want) < 2e-2
    assert kernels.take_device_error() == (0, 0)


class Stack(torch.nn.Module):
    """R:tests/test_backend.py:333-348: a Qwen3Model of Qwen3-0.6B's widths into a linear head, fed
    embeddings and a 4-D mask."""

    def __init__(self, layers=2, head_n=1000, bias=True):
        super().__init__()
        from transformers import Qwen3Config, Qwen3Model

        cfg = Qwen3Config(hidden_size=1024, intermediate_size=3072, num_hidden_layers=layers, num_attention_heads=16,
                          num_key_value_heads=8, head_dim=128, vocab_size=16, rms_norm_eps=1e-6,
                          rope_parameters={"rope_type": "default", "rope_theta": 1e6}, attn_implementation="sdpa")
        self.llm = Qwen3Model(cfg)
        self.head = torch.nn.Linear(1024, head_n, bias=bias)

    def forward(self, x, mask):
        return self.head(self.llm(inputs_embeds=x, attention_mask=mask)[0])


def _golden_model(ent, dev):
    ls, final, head, head_b, x = mg.stack_inputs(ent["seed"], ent["layers"], ent["head_n"], ent["batch"], ent["seq"])
    net = Stack(ent["layers"], ent["head_n"])
    for i, L in enumerate(ls):
        lay = net.llm.layers[i]
        lay.self_attn.q_proj.weight.data = torch.from_numpy(L["q"])
        lay.self_attn.k_proj.weight.data = torch.from_numpy(L["k"])
        lay.self_attn.v_proj.weight.data = torch.from_numpy(L["v"])
        lay.self_attn.o_proj.weight.data = torch.from_numpy(L["o"])
        lay.mlp.gate_proj.weight.data = torch.from_numpy(L["gate"])
        lay.mlp.up_proj.weight.data = torch.from_numpy(L["up"])
        lay.mlp.down_proj.weight.data = torch.from_numpy(L["down"])
        lay.input_layernorm.weight.data = torch.from_numpy(L["input_norm"])
        lay.post_attention_layernorm.weight.data = torch.from_numpy(L["post_norm"])
        lay.self_attn.q_norm.weight.data = torch.from_numpy(L["q_norm"])
        lay.self_attn.k_norm.weight.data = torch.from_numpy(L["k_norm"])
    net.llm.norm.weight.data = torch.from_numpy(final)
    net.head.weight.data = torch.from_numpy(head)
    net.head.bias.data = torch.from_numpy(head_b)
    mask = mg.causal_mask(ent["batch"], ent["seq"]) if ent["mask"] == "causal" else mg.prefix_mask(ent["lens"],
                                                                                                     ent["seq"])
    return net.eval().to(dev), torch.from_numpy(x).to(dev), torch.from_numpy(mask).to(dev)


@pytest.mark.parametrize("name", [c[0] for c in mg.STACK_CASES])
def test_compiled_stack_matches_reference_golden(cuda, golden, name):
    """torch.compile(backend="xdna") on the reference test's Stack model: one xdna::qwen3_stack call,
    logits within 2e-2 of the golden fp32 logits, padding rows zero, and the first-call check recorded."""
    import torch_xdna

    manifest, arrays = golden
    ent = manifest["stack"][name]
    net, x, mask = _golden_model(ent, cuda)
    torch._dynamo.reset()
    torch_xdna.stats.reset()
    m = torch.compile(net, backend="xdna", options={"fallback": "eager"})
    y = m(x, mask)
    s = torch_xdna.stats.as_dict()
    assert s["stacks"] == {f"qwen3 stack {ent['layers']} layers -> {ent['head_n']} on gpu": 1}, s["stacks"]
    assert len(s["checks"]) == 1, s["checks"]
    want = torch.from_numpy(arrays[f"stack/{name}/logits"]).to(cuda)
    if ent["mask"] == "prefix":
        for b, n in enumerate(ent["lens"]):
            assert not y[b, n:].any(), "padding rows are not zero"
            assert rel_max(y[b, :n], want[b, :n]) < TOL
    else:
        assert rel_max(y, want) < TOL


def test_stack_28_layers_causal_vs_fp32_model(cuda):
    """BASELINE config 5's depth (28 layers, Qwen3-0.6B widths) on 2 x 256 tokens under a causal mask,
    head 8192: the logits of the bf16 stack vs the fp32 model run eagerly on the GPU."""
    import torch_xdna

    torch.manual_seed(0)
    net = Stack(layers=28, head_n=8192, bias=False)
    for p in net.parameters():
        if p.dim() == 2:
            p.data.normal_(0, 0.02)
    net = net.eval().to(cuda)
    B, L = 2, 256
    x = torch.randn(B, L, 1024, device=cuda)
    mask = torch.ones(L, L, dtype=torch.bool, device=cuda).tril()[None, None].expand(B, 1, L, L).contiguous()
    want = net(x, mask)
    torch._dynamo.reset()
    y = torch.compile(net, backend="xdna", options={"fallback": "eager", "verify": "off"})(x, mask)
    assert rel_max(y, want) < TOL, rel_max(y, want)
