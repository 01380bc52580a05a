"""The custom ops the backend puts in place of offloadable GEMMs, convs and transformer stacks.

Schemas are the reference's, unchanged (R:torch_xdna/ops.py:25-89), so graphs and code that call
torch.ops.xdna.* keep working; the implementations call the B200 kernels. To the rest of
torch.compile each op is opaque with a shape function (the fake impl), and Inductor calls it as an
extern kernel. Two ops are new: xdna::conv3x3_fused, the whole quantise -> conv -> dequantise of
conv3x3_int8 as one op, because on the B200 those three steps are kernels of ours rather than
graph ops for the CPU compiler to fuse; xdna::conv3x3_chain, the same for a conv inside a chain of
convs whose activations between them stay int8 codes; and xdna::conv_int8, the same arithmetic for the
1x1 and stride-2 convs the reference has no kernel for (offloaded with Config(conv_ext=True)).
"""

from typing import Optional

import torch

from . import conv, runtime, stack

_configs = []  # cfg_id -> Config; op arguments must be plain values (R:torch_xdna/ops.py:14-22)


def config_id(cfg) -> int:
    for i, c in enumerate(_configs):
        if c == cfg:
            return i
    _configs.append(cfg)
    return len(_configs) - 1


@torch.library.custom_op("xdna::linear", mutates_args=())
def linear(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor],
           transposed: bool, cfg_id: int) -> torch.Tensor:
    return runtime.linear(_configs[cfg_id], x, weight, bias, transposed)


@linear.register_fake
def _(x, weight, bias, transposed, cfg_id):
    n = weight.shape[1] if transposed else weight.shape[0]
    return x.new_empty(*x.shape[:-1], n)


@torch.library.custom_op("xdna::linear_cat", mutates_args=())
def linear_cat(x: torch.Tensor, weights: list[torch.Tensor], biases: list[Optional[torch.Tensor]],
               cfg_id: int) -> torch.Tensor:
    """Linears that read the same input as one GEMM; outputs concatenated on the last dim."""
    return runtime.linear_cat(_configs[cfg_id], x, weights, biases)


@linear_cat.register_fake
def _(x, weights, biases, cfg_id):
    return x.new_empty(*x.shape[:-1], sum(w.shape[0] for w in weights))


@torch.library.custom_op("xdna::linear_i8", mutates_args=())
def linear_i8(xq: torch.Tensor, weights: list[torch.Tensor], transposed: bool,
              cfg_id: int) -> tuple[torch.Tensor, torch.Tensor]:
    """int8 xq [R, K] -> (acc [R, N] int32, sw [N] float32), x @ W^T ~= acc * sx[:, None] * sw."""
    return runtime.linear_i8(_configs[cfg_id], xq, weights, transposed)


@linear_i8.register_fake
def _(xq, weights, transposed, cfg_id):
    n = sum(w.shape[1] if transposed else w.shape[0] for w in weights)
    return xq.new_empty((xq.shape[0], n), dtype=torch.int32), xq.new_empty((n,), dtype=torch.float32)


@torch.library.custom_op("xdna::conv3x3", mutates_args=())
def conv3x3(xq: torch.Tensor, weight: torch.Tensor, relu: bool, cfg_id: int) -> tuple[torch.Tensor, torch.Tensor]:
    """int8 xq [N, Ci, H, W] -> (q [N, Co, H, W] int8 (uint8 with relu), scale [Co] float32),
    relu?(conv2d(x, weight, padding=1)) ~= q * scale[co] * sx."""
    return conv.conv3x3(_configs[cfg_id], xq, weight, relu)


@conv3x3.register_fake
def _(xq, weight, relu, cfg_id):
    q = xq.new_empty((xq.shape[0], weight.shape[0], xq.shape[2], xq.shape[3]),
                     dtype=torch.uint8 if relu else torch.int8)
    return q, weight.new_empty((weight.shape[0],), dtype=torch.float32)


@torch.library.custom_op("xdna::conv3x3_fused", mutates_args=())
def conv3x3_fused(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor], relu: bool,
                  cfg_id: int, post_relu: bool = False) -> torch.Tensor:
    """relu?(conv2d(x, weight, bias, padding=1)) through int8, as conv3x3_int8 defines it; post_relu:
    torch.relu of that result, applied in the epilogue after the bias."""
    return conv.conv3x3_fused(_configs[cfg_id], x, weight, bias, relu, post_relu)


@conv3x3_fused.register_fake
def _(x, weight, bias, relu, cfg_id, post_relu=False):
    # the kernel writes channels-last memory (see conv.ConvLayer.dequant)
    return torch.empty((x.shape[0], weight.shape[0], x.shape[2], x.shape[3]), dtype=x.dtype, device=x.device,
                       memory_format=torch.channels_last)


@torch.library.custom_op("xdna::conv_int8", mutates_args=())
def conv_int8(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor], stride: int, relu: bool,
              cfg_id: int, post_relu: bool = False) -> torch.Tensor:
    """A 1x1 conv (stride 1 or 2, padding 0) or a stride-2 3x3 conv (padding 1) through int8 with the
    arithmetic of conv3x3_int8 (conv.conv_int8); the ReLU options as conv3x3_fused."""
    return conv.conv_int8(_configs[cfg_id], x, weight, bias, stride, relu, post_relu)


@conv_int8.register_fake
def _(x, weight, bias, stride, relu, cfg_id, post_relu=False):
    h, w = x.shape[2], x.shape[3]
    if stride == 2:
        h, w = (h + 1) // 2, (w + 1) // 2
    return torch.empty((x.shape[0], weight.shape[0], h, w), dtype=x.dtype, device=x.device,
                       memory_format=torch.channels_last)


@torch.library.custom_op("xdna::conv3x3_chain", mutates_args=())
def conv3x3_chain(x: torch.Tensor, xmeta: Optional[torch.Tensor], weight: torch.Tensor, bias: Optional[torch.Tensor],
                  relu: bool, cfg_id: int, post_relu: bool, in_mode: int, in_relu_after: bool,
                  out_q: bool, out_pool: bool = False) -> tuple[torch.Tensor, torch.Tensor]:
    """One conv of a chain whose activations between convs stay int8 codes (conv.conv3x3_chain): the
    same values as conv3x3_fused layer after layer with the graph's ReLU and 2x2 max-pool between."""
    return conv.conv3x3_chain(_configs[cfg_id], x, xmeta, weight, bias, relu, post_relu, in_mode, in_relu_after,
                              out_q, out_pool)


@conv3x3_chain.register_fake
def _(x, xmeta, weight, bias, relu, cfg_id, post_relu, in_mode, in_relu_after, out_q, out_pool=False):
    n, co = x.shape[0], weight.shape[0]
    if in_mode == conv.IN_FLOAT:
        h, w = x.shape[2], x.shape[3]
    else:
        h, w = (x.shape[1] // 2, x.shape[2] // 2) if in_mode == conv.IN_CODES_POOL else (x.shape[1], x.shape[2])
    if out_q:
        cfg = _configs[cfg_id]
        fbias = None if conv.int32_bias(cfg, bias) else bias
        relu, post_relu = conv.effective_relu(cfg, relu, bias, post_relu)
        q = x.new_empty((n, h, w, co), dtype=torch.uint8 if relu else torch.int8)
        extra = n + (1 if out_pool else 0) if conv.next_amax_ok(relu, fbias, post_relu, out_pool) else 0
        return q, x.new_empty((n + 2 * co + extra,), dtype=torch.float32)
    dtype = x.dtype if in_mode == conv.IN_FLOAT else torch.float32
    y = torch.empty((n, co, h, w), dtype=dtype, device=x.device, memory_format=torch.channels_last)
    return y, x.new_empty((0,), dtype=torch.float32)


@torch.library.custom_op("xdna::qwen3_stack", mutates_args=())
def qwen3_stack(x: torch.Tensor, mask: torch.Tensor, stack_id: int, cfg_id: int) -> torch.Tensor:
    """A whole Qwen3-0.6B-sized stack with its final norm and linear head: hidden states x [B, L, 1024]
    under a 4-D attention mask -> the head's output [B, L, N]."""
    return stack.run(_configs[cfg_id], stack_id, x, mask)


@qwen3_stack.register_fake
def _(x, mask, stack_id, cfg_id):
    return x.new_empty(*x.shape[:-1], stack.out_features(stack_id))
