"""Host logic without a GPU: the FX pass (which nodes become which xdna:: op), shared-input fusion, the
conv pass and its ReLU fusion, Config validation, and the loud failure without a B200
(mirrors R:tests/test_backend.py case_fusion / case_conv_pass / case_no_npu, by graph inspection)."""

import copy

import pytest
import torch

import torch_xdna
from torch_xdna import kernels
from torch_xdna.conv import IN_CODES, IN_CODES_POOL, IN_FLOAT, conv3x3_chain_int8, conv3x3_int8


def capture_graphs(model, x, cfg):
    """Run Dynamo on `model` and return the rewritten FX graphs (the model itself runs eagerly)."""
    graphs = []

    def backend(gm, example_inputs):
        original = torch.fx.GraphModule(gm, copy.deepcopy(gm.graph))
        torch_xdna.offload_gemms(gm, example_inputs, cfg)
        graphs.append(gm)
        return original.forward

    torch._dynamo.reset()
    with torch.no_grad():
        torch.compile(model, backend=backend)(x)
    return graphs


def call_targets(gm):
    return [n.target for n in gm.graph.nodes if n.op == "call_function"]


class Net(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.a = torch.nn.Linear(200, 300)
        self.b = torch.nn.Linear(300, 1024, bias=False)
        self.w = torch.nn.Parameter(torch.randn(1024, 520) * 0.03)

    def forward(self, x):
        h = torch.nn.functional.gelu(self.a(x))
        h = torch.nn.functional.silu(self.b(h))
        return h @ self.w


class Attn(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.q = torch.nn.Linear(256, 256)
        self.k = torch.nn.Linear(256, 128, bias=False)
        self.v = torch.nn.Linear(256, 128)
        self.o = torch.nn.Linear(256, 256)

    def forward(self, x):
        q, k, v = self.q(x), self.k(x), self.v(x)
        return self.o(q * torch.cat([k, v], -1).sigmoid())


class CNN(torch.nn.Module):
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


class AddmmNet(torch.nn.Module):
    """HF Conv1D-style b + x @ W, plus a GEMM between two activations that must stay."""

    def __init__(self):
        super().__init__()
        self.w = torch.nn.Parameter(torch.randn(64, 96))
        self.b = torch.nn.Parameter(torch.randn(96))

    def forward(self, x):
        h = torch.addmm(self.b, x, self.w)
        return h @ h.t()


def test_linear_patterns_rewritten():
    (gm,) = capture_graphs(Net().eval(), torch.randn(37, 200), torch_xdna.Config())
    targets = call_targets(gm)
    lin = [n for n in gm.graph.nodes if n.op == "call_function" and n.target is torch.ops.xdna.linear.default]
    assert len(lin) == 3
    assert [n.args[3] for n in lin] == [False, False, True]      # F.linear, F.linear, h @ W
    assert torch.nn.functional.linear not in targets


def test_addmm_rewritten_activation_gemm_left():
    (gm,) = capture_graphs(AddmmNet(), torch.randn(8, 64), torch_xdna.Config())
    lin = [n for n in gm.graph.nodes if n.op == "call_function" and n.target is torch.ops.xdna.linear.default]
    assert len(lin) == 1 and lin[0].args[3] is True and lin[0].args[2] is not None
    remaining = [n for n in gm.graph.nodes if n.op in ("call_function", "call_method")
                 and (n.target in (torch.matmul, torch.mm) or n.target in ("matmul", "mm", "__matmul__")
                      or getattr(n.target, "__name__", "") == "matmul")]
    assert remaining, "the activation x activation GEMM must not be offloaded"


def test_shared_input_fusion():
    (gm,) = capture_graphs(Attn().eval(), torch.randn(20, 256), torch_xdna.Config())
    targets = call_targets(gm)
    assert targets.count(torch.ops.xdna.linear_cat.default) == 1
    assert targets.count(torch.ops.xdna.linear.default) == 1        # o
    assert targets.count(torch.narrow) == 3
    cat = next(n for n in gm.graph.nodes if n.target is torch.ops.xdna.linear_cat.default)
    assert len(cat.args[1]) == 3 and [b is None for b in cat.args[2]] == [False, True, False]
    (gm2,) = capture_graphs(Attn().eval(), torch.randn(20, 256), torch_xdna.Config(fuse=False))
    assert call_targets(gm2).count(torch.ops.xdna.linear.default) == 4


def test_conv_pass_which_convs_and_relu():
    """3 of 4 convs rewritten, stride 2 left alone (R:tests/test_backend.py:220-240); the bias-free conv's
    ReLU fused into the requantise as in the reference, the biased conv's ReLU after its bias. Without
    fusion the three stay separate conv3x3_int8 nodes with the ReLUs in the graph."""
    (gm2,) = capture_graphs(CNN().eval(), torch.randn(1, 64, 16, 64), torch_xdna.Config(policy="npu", fuse=False))
    nodes2 = [n for n in gm2.graph.nodes if n.op == "call_function"]
    assert sum(n.target is conv3x3_int8 for n in nodes2) == 3
    assert sum(n.target in (torch.relu, torch.nn.functional.relu) for n in nodes2) == 2
    assert sum(n.target is torch.conv2d for n in nodes2) == 1
    # with fusion the three consecutive convs also pass int8 codes between them (conv3x3_chain)
    (gm,) = capture_graphs(CNN().eval(), torch.randn(1, 64, 16, 64), torch_xdna.Config(policy="npu"))
    nodes = [n for n in gm.graph.nodes if n.op == "call_function"]
    chain = [n for n in nodes if n.target is conv3x3_chain_int8]
    # args: (x, xmeta, w, b, relu, cfg_id, post_relu, in_mode, in_relu_after, out_q)
    assert [n.args[4] for n in chain] == [False, True, False], [n.args for n in chain]
    assert [n.args[6] for n in chain] == [True, False, False]
    assert [n.args[7] for n in chain] == [IN_FLOAT, IN_CODES, IN_CODES]
    assert [n.args[8] for n in chain] == [False, True, False]   # the previous conv's ReLU after its bias
    assert [n.args[9] for n in chain] == [True, True, False]    # the last one feeds the stride-2 conv: float
    assert sum(n.target is conv3x3_int8 for n in nodes) == 0
    assert sum(n.target in (torch.relu, torch.nn.functional.relu) for n in nodes) == 0
    assert sum(n.target is torch.conv2d for n in nodes) == 1


class Bottleneck(torch.nn.Module):
    """A ResNet-50 bottleneck with a stride-2 downsample and a stride-1 3x3 in the middle block."""

    def __init__(self):
        super().__init__()
        self.c1 = torch.nn.Conv2d(256, 64, 1, bias=False)
        self.c2 = torch.nn.Conv2d(64, 64, 3, stride=2, padding=1)
        self.c3 = torch.nn.Conv2d(64, 256, 1)
        self.down = torch.nn.Conv2d(256, 256, 1, stride=2, bias=False)
        self.c4 = torch.nn.Conv2d(256, 64, 3, padding=1)
        self.c5 = torch.nn.Conv2d(64, 64, 5, padding=2)    # a 5x5 conv: never offloaded

    def forward(self, x):
        h = torch.relu(self.c1(x))
        h = torch.relu(self.c2(h))
        h = torch.relu(self.c3(h) + self.down(x))
        return self.c5(torch.relu(self.c4(h)))


def test_conv_ext_offloads_resnet_convs_only_when_asked():
    """By default the pass rewrites exactly the reference's convs (3x3 / stride 1 / padding 1: c4 here); with
    conv_ext also the 1x1 convs (stride 1 and 2) and the stride-2 3x3, each with its stride and the ReLU
    fusion rules of the 3x3 convs (bias-free: into the requantise; biased: after the bias)."""
    from torch_xdna.conv import conv_ext_int8

    x = torch.randn(1, 256, 16, 16)
    (gm,) = capture_graphs(Bottleneck().eval(), x, torch_xdna.Config(policy="npu"))
    nodes = [n for n in gm.graph.nodes if n.op == "call_function"]
    assert sum(n.target is conv_ext_int8 for n in nodes) == 0
    assert sum(n.target is torch.conv2d for n in nodes) == 5
    assert sum(n.target in (conv3x3_int8, conv3x3_chain_int8) for n in nodes) == 1
    (gm,) = capture_graphs(Bottleneck().eval(), x, torch_xdna.Config(policy="npu", conv_ext=True))
    nodes = [n for n in gm.graph.nodes if n.op == "call_function"]
    ext = [n for n in nodes if n.target is conv_ext_int8]
    # args: (x, w, b, stride, relu into the requantise, cfg_id, relu after the bias)
    assert [(n.args[3], n.args[4], n.args[6]) for n in ext] == [(1, True, False), (2, False, True), (1, False, False),
                                                                (2, False, False)]
    assert sum(n.target is torch.conv2d for n in nodes) == 1              # the 5x5 conv
    assert sum(n.target in (torch.relu, torch.nn.functional.relu) for n in nodes) == 1   # after the residual add


class VGGish(torch.nn.Module):
    """VGG-style blocks: conv, ReLU, conv, ReLU, 2x2 max-pool, ...; `tap` also returns an intermediate
    activation, which then must stay a float tensor."""

    def __init__(self, tap=False):
        super().__init__()
        self.c1 = torch.nn.Conv2d(3, 64, 3, padding=1)
        self.c2 = torch.nn.Conv2d(64, 64, 3, padding=1)
        self.c3 = torch.nn.Conv2d(64, 128, 3, padding=1)
        self.c4 = torch.nn.Conv2d(128, 128, 3, padding=1, bias=False)
        self.pool = torch.nn.MaxPool2d(2)
        self.tap = tap

    def forward(self, x):
        h = torch.relu(self.c1(x))
        a = torch.relu(self.c2(h))
        h = torch.relu(self.c3(self.pool(a)))
        h = self.pool(torch.relu(self.c4(h)))
        return (h, a) if self.tap else h


def test_conv_chain_through_max_pool():
    """The 2x2 max-pool between two convs is taken into the chain (pooled on the codes); the last pool,
    whose input is the graph's output, stays."""
    (gm,) = capture_graphs(VGGish().eval(), torch.randn(1, 3, 16, 16), torch_xdna.Config(policy="npu"))
    nodes = [n for n in gm.graph.nodes if n.op == "call_function"]
    chain = [n for n in nodes if n.target is conv3x3_chain_int8]
    assert [n.args[7] for n in chain] == [IN_FLOAT, IN_CODES, IN_CODES_POOL, IN_CODES]
    assert [n.args[9] for n in chain] == [True, True, True, False]
    assert [n.args[8] for n in chain] == [False, True, True, True]
    assert sum(n.target in (torch.nn.functional.max_pool2d, torch.max_pool2d) for n in nodes) == 1


def test_conv_chain_stops_at_other_uses_and_non_f32():
    """An activation with another user (here a graph output) is not chained across; bf16 activations are
    not chained at all."""
    (gm,) = capture_graphs(VGGish(tap=True).eval(), torch.randn(1, 3, 16, 16), torch_xdna.Config(policy="npu"))
    nodes = [n for n in gm.graph.nodes if n.op == "call_function"]
    chain = [n for n in nodes if n.target is conv3x3_chain_int8]
    # c1 -> c2 chained; c2's output is also returned, so c2 -> pool -> c3 is not; c3 -> c4 chained
    assert [(n.args[7], n.args[9]) for n in chain] == [(IN_FLOAT, True), (IN_CODES, False), (IN_FLOAT, True),
                                                       (IN_CODES, False)]
    (gmb,) = capture_graphs(VGGish().eval().to(torch.bfloat16), torch.randn(1, 3, 16, 16, dtype=torch.bfloat16),
                            torch_xdna.Config(policy="npu"))
    nodes = [n for n in gmb.graph.nodes if n.op == "call_function"]
    assert sum(n.target is conv3x3_chain_int8 for n in nodes) == 0
    assert sum(n.target is conv3x3_int8 for n in nodes) == 4


def test_policy_cpu_rewrites_nothing_and_runs():
    torch._dynamo.reset()
    net = Net().eval()
    x = torch.randn(5, 200)
    m = torch.compile(net, backend="xdna", options={"policy": "cpu", "fallback": "eager"})
    with torch.no_grad():
        assert torch.equal(m(x), net(x))


def test_config_validation():
    c = torch_xdna.Config().merged({"row_buckets": [512, 128], "policy": "npu"})
    assert c.row_buckets == (128, 512) and c.policy == "npu"
    with pytest.raises(AssertionError, match="unknown xdna options"):
        torch_xdna.Config().merged({"polcy": "npu"})
    with pytest.raises(AssertionError):
        torch_xdna.Config(policy="gpu")
    with pytest.raises(AssertionError):
        torch_xdna.Config(verify="sometimes")


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the behaviour without a GPU")
def test_no_gpu_fails_loudly():
    assert not torch_xdna.gpu_available()
    assert kernels.unavailable_reason()
    torch._dynamo.reset()
    m = torch.compile(Net().eval(), backend="xdna")
    with pytest.raises(Exception, match="B200|CUDA"):
        with torch.no_grad():
            m(torch.randn(4, 200))
    with pytest.raises(kernels.XdnaUnavailable):
        kernels.require()


def test_stack_found_in_qwen3_graph():
    """The FX search finds transformers' Qwen3Model + head (2 layers), its mask input and its head bias."""
    from transformers import Qwen3Config, Qwen3Model

    from torch_xdna import stack

    class Stack(torch.nn.Module):
        def __init__(self):
            super().__init__()
            cfg = Qwen3Config(hidden_size=1024, intermediate_size=3072, num_hidden_layers=2, num_attention_heads=16,
                              num_key_value_heads=8, head_dim=128, vocab_size=16, rms_norm_eps=1e-6,
                              rope_parameters={"rope_type": "default", "rope_theta": 1e6}, attn_implementation="sdpa")
            self.llm = Qwen3Model(cfg)
            self.head = torch.nn.Linear(1024, 1000)

        def forward(self, x, mask):
            return self.head(self.llm(inputs_embeds=x, attention_mask=mask)[0])

    plans = []

    def backend(gm, example_inputs):
        plans.append(stack.find(gm, example_inputs))
        return gm.forward

    torch._dynamo.reset()
    mask = torch.ones(24, 24, dtype=torch.bool).tril().expand(2, 1, 24, 24).contiguous()
    with torch.no_grad():
        torch.compile(Stack().eval(), backend=backend)(torch.randn(2, 24, 1024), mask)
    plan = plans[0]
    assert plan is not None and plan.layers == 2 and plan.out_features == 1000 and plan.bias is not None
    assert len(plan.tensors()) == 2 * 11 + 3


def test_stack_mask_classification():
    from torch_xdna import kernels, stack

    import make_golden as mg

    L = 40
    causal = torch.ones(L, L, dtype=torch.bool).tril().expand(3, 1, L, L)
    assert stack.classify(causal, 3, L)[0] == kernels.MASK_CAUSAL
    prefix = torch.from_numpy(mg.prefix_mask([40, 29, 17], L))
    kind, lens, _ = stack.classify(prefix, 3, L)
    assert kind == kernels.MASK_PREFIX and lens.tolist() == [40, 29, 17]
    assert stack.lengths(prefix) == [40, 29, 17]
    full = torch.zeros(3, 1, L, L)                       # float mask, all 0: attend everywhere
    assert stack.classify(full, 3, L)[0] == kernels.MASK_NONE
    other = causal.clone()
    other[0, 0, 5, 2] = False
    kind, _, m = stack.classify(other, 3, L)
    assert kind == kernels.MASK_BOOL and m.dtype == torch.uint8 and m.shape == (3, 1, L, L)
    bad = torch.zeros(3, 1, L, L)
    bad[0, 0, 0, 1] = -0.5                               # an additive bias, not a mask
    assert stack.classify(bad, 3, L) is None
    assert stack.classify(causal[:, :, :, :L - 1], 3, L) is None


def test_report_formats():
    torch_xdna.stats.reset()
    s = torch_xdna.report()
    assert s.startswith("B200 available:")
    assert '"calls"' in torch_xdna.report(as_json=True)
