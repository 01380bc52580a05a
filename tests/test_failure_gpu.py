"""Failure detection, with the failures made on the host (nothing here faults, traps or hangs a GPU):

- a bounded device wait that runs out: the self-test kernel waits, with a 2 ms limit, on an mbarrier that
  nothing arrives at, records XDNA_ERR_TIMEOUT in the device error word and returns; the host reads it and
  the context stays usable;
- the reference's failure-injection cases (R:tests/test_backend.py:131-176 a launch returning a wrong value
  and a launch that raises, :303-330 a wrong conv, :413-439 a stack output scaled by 1.5): the launch's
  output is perturbed, or the launch raises, in a host-side wrapper of the library call. The reference then
  falls back to its CPU route; this build has no CPU route, so the first-launch check raises
  XdnaResultMismatch and a failing launch raises its XdnaError -- a wrong value never reaches the output.
"""

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


def test_bounded_wait_runs_out_and_is_reported(cuda):
    from torch_xdna import kernels

    assert kernels.take_device_error() == (0, 0)
    kernels.selftest_wait_timeout(2_000_000)
    assert kernels.take_device_error() == (kernels.ERR_TIMEOUT, 99)
    assert kernels.take_device_error() == (0, 0)          # read and cleared
    # the context is still usable: a verified GEMM afterwards
    x = torch.randn(64, 96, device=cuda)
    w = torch.randn(48, 96, device=cuda) * 0.05
    y = torch.ops.xdna.linear(x, w, None, False, _cid(verify="always"))
    assert y.shape == (64, 48) and kernels.take_device_error() == (0, 0)


def test_gemm_config_comes_from_the_library(cuda):
    """The verify key's configuration is what the library reports for the shape (no Python mirror)."""
    from torch_xdna import kernels, runtime

    assert kernels.gemm_i8_config(8192, 6144) == (256, True)
    assert kernels.gemm_i8_config(37, 64)[0] == 64
    assert runtime._bn_for(8192, 6144) == "256 pair"


def test_wrong_gemm_value_is_caught_on_first_launch(cuda, monkeypatch):
    import torch_xdna
    from torch_xdna import kernels

    real = kernels.gemm_i8

    def corrupt(xq, wq, K, y, sx=None, sw=None, bias=None):
        real(xq, wq, K, y, sx, sw, bias)
        y.view(-1)[0] += 1      # one wrong value in a launch that otherwise ran

    monkeypatch.setattr(kernels, "gemm_i8", corrupt)
    x = torch.randn(300, 200, device=cuda)
    w = torch.randn(300, 200, device=cuda) * 0.05
    with pytest.raises(torch_xdna.XdnaResultMismatch, match="disagrees with the CPU"):
        torch.ops.xdna.linear(x, w, None, False, _cid(verify="always"))


def test_failing_launch_raises(cuda, monkeypatch):
    from torch_xdna import kernels

    def boom(*a, **k):
        raise kernels.XdnaError("xdna_gemm_i8", -3, "simulated launch failure")

    monkeypatch.setattr(kernels, "gemm_i8", boom)
    x = torch.randn(300, 200, device=cuda)
    w = torch.randn(300, 200, device=cuda) * 0.05
    with pytest.raises(kernels.XdnaError, match="simulated launch failure"):
        torch.ops.xdna.linear(x, w, None, False, _cid(verify="off"))


def test_wrong_conv_value_is_caught_on_first_launch(cuda, monkeypatch):
    import torch_xdna
    from torch_xdna import kernels

    real = kernels.conv3x3

    def corrupt(xp, wp, N, Ci, Co, H, W, mode, *a, **k):
        real(xp, wp, N, Ci, Co, H, W, mode, *a, **k)
        if (mode & 15) == kernels.CONV_Q:      # the integers the first-launch check compares
            out = k["out"]
            out.view(-1)[5] = out.view(-1)[5] ^ 1

    monkeypatch.setattr(kernels, "conv3x3", corrupt)
    x = torch.randn(2, 32, 12, 20, device=cuda)
    w = torch.nn.Parameter(torch.randn(48, 32, 3, 3, device=cuda) * 0.08)
    with pytest.raises(torch_xdna.XdnaResultMismatch, match="disagrees with the CPU integers"):
        torch.ops.xdna.conv3x3_fused(x, w, None, True, _cid(verify="always"))


class _Stack(torch.nn.Module):
    """A 2-layer Qwen3Model of Qwen3-0.6B's widths into a linear head (R:tests/test_backend.py:333-348)."""

    def __init__(self):
        super().__init__()
        from transformers import Qwen3Config, Qwen3Model

        cfg = Qwen3Config(hidden_size=1024, intermediate_size=3072, num_hidden_layers=2, num_attention_heads=16,
                          num_key_value_heads=8, head_dim=128, vocab_size=16, rms_norm_eps=1e-6,
                          rope_parameters={"rope_type": "default", "rope_theta": 1e6}, attn_implementation="sdpa")
        self.llm = Qwen3Model(cfg)
        self.head = torch.nn.Linear(1024, 1000)

    def forward(self, x, mask):
        return self.head(self.llm(inputs_embeds=x, attention_mask=mask)[0])


def test_wrong_stack_output_is_caught_on_first_call(cuda, monkeypatch):
    import torch_xdna
    from torch_xdna import kernels

    real = kernels.qwen3_stack

    def scaled(*a, **k):
        real(*a, **k)
        a[13].mul_(1.5)          # the head's output

    monkeypatch.setattr(kernels, "qwen3_stack", scaled)
    torch.manual_seed(0)
    net = _Stack().eval().to(cuda)
    x = torch.randn(2, 64, 1024, device=cuda)
    mask = torch.ones(64, 64, dtype=torch.bool, device=cuda).tril()[None, None].expand(2, 1, 64, 64).contiguous()
    torch._dynamo.reset()
    m = torch.compile(net, backend="xdna", options={"fallback": "eager", "verify": "first"})
    with pytest.raises(torch_xdna.XdnaResultMismatch, match="disagrees with the model"):
        m(x, mask)
