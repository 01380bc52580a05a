"""The reference's CPU route, restated with the same torch CPU calls -- TEST / BASELINE INFRASTRUCTURE.

Used as `bench.py --impl reference` and as the cpu_baseline leg: it times what the reference runs with
policy="cpu" on the host cores (torch._int_mm on oneDNN, eager quantise / dequantise ops; the conv's
exact fp conv of the integers), because the reference package itself is not present on the GPU box.
Only tests/, __graft_entry__.smoke() and bench.py's baseline legs may import this module.
Pinned against the reference's golden vectors by tests/test_oracle.py::test_reference_cpu_port_*.
"""

import math

import torch


def quant_rows(x2d):
    """R:torch_xdna/runtime.py:366-368."""
    sx = x2d.abs().amax(dim=1, keepdim=True).float().clamp(min=1e-8) / 127
    xq = torch.round(x2d.float() / sx).clamp(-127, 127).to(torch.int8)
    return xq, sx


def quant_weight(w):
    """QWeight, R:torch_xdna/runtime.py:59-66: (w_kn [K, N] int8 for torch._int_mm, sw [N])."""
    wf = w.detach().float()
    sw = wf.abs().amax(dim=1).clamp(min=1e-8) / 127
    q = torch.round(wf / sw[:, None]).clamp(-127, 127).to(torch.int8)
    return q.t().contiguous(), sw


def linear_int8(x, w_kn, sw, bias=None):
    """The W8A8 linear of R:torch_xdna/runtime.py:366-374 with a quantised weight."""
    x2 = x.reshape(-1, x.shape[-1])
    xq, sx = quant_rows(x2)
    acc = torch._int_mm(xq, w_kn)
    y = acc.float() * sx * sw
    if bias is not None:
        y = y + bias.float()
    return y.to(x.dtype).reshape(*x.shape[:-1], y.shape[-1])


def qwen3_stack(layers, final_norm, head, head_bias, x, allowed, theta=1e6, eps=1e-6):
    """The fp32 eager model the reference checks its fused stack against (R:torch_xdna/stack.py:444-460),
    restated with torch CPU ops: transformers' Qwen3 decoder layers on x [B, L, 1024] under a bool mask
    [B, 1, L, L], the final norm and the head. layers: list of dicts of float32 tensors (LAYER_KEYS).
    The same torch ops run on whatever device x is on (the full-size parity test runs them on the GPU in
    fp32, TF32 off)."""
    B, L, D = x.shape
    NH, NKV, DH = 16, 8, 128
    dev = x.device
    inv_freq = 1.0 / (theta ** (torch.arange(0, DH, 2, dtype=torch.float32, device=dev) / DH))
    freqs = torch.arange(L, dtype=torch.float32, device=dev)[:, None] * inv_freq[None, :]
    cos, sin = torch.cat([freqs, freqs], -1).cos(), torch.cat([freqs, freqs], -1).sin()

    def rms(t, w):
        return t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + eps) * w

    def rope(t):
        return t * cos + torch.cat([-t[..., DH // 2:], t[..., :DH // 2]], -1) * sin

    h = x.float()
    for w in layers:
        a = rms(h, w["input_norm"])
        q = rms((a @ w["q"].t()).view(B, L, NH, DH), w["q_norm"]).transpose(1, 2)
        k = rms((a @ w["k"].t()).view(B, L, NKV, DH), w["k_norm"]).transpose(1, 2)
        v = (a @ w["v"].t()).view(B, L, NKV, DH).transpose(1, 2)
        q, k = rope(q), rope(k)
        o = torch.nn.functional.scaled_dot_product_attention(q, k.repeat_interleave(NH // NKV, 1),
                                                             v.repeat_interleave(NH // NKV, 1), attn_mask=allowed)
        h = h + o.transpose(1, 2).reshape(B, L, NH * DH) @ w["o"].t()
        a = rms(h, w["post_norm"])
        h = h + (torch.nn.functional.silu(a @ w["gate"].t()) * (a @ w["up"].t())) @ w["down"].t()
    out = rms(h, final_norm) @ head.t()
    return out + head_bias if head_bias is not None else out


def conv_layer(weight, relu):
    """ConvLayer weights, R:torch_xdna/conv.py:58-63."""
    wf = weight.detach().float()
    sw = wf.abs().amax(dim=(1, 2, 3)).clamp(min=1e-8) / 127
    wq = torch.round(wf / sw[:, None, None, None]).clamp(-127, 127).to(torch.int8)
    dt = torch.float32 if 127 * float(wq.abs().sum(dim=(1, 2, 3)).max()) < 2 ** 24 else torch.float64
    return dict(wq=wq, sw=sw, dt=dt, relu=relu, shift=None)


def conv3x3_int8(x, layer, bias=None):
    """conv3x3_int8 on the CPU route, R:torch_xdna/conv.py:43-51,71-76,86-92."""
    sx = x.abs().amax(dim=(1, 2, 3), keepdim=True).float().clamp(min=1e-8) / 127
    xq = torch.round(x.float() / sx).clamp(-127, 127).to(torch.int8)
    acc = torch.nn.functional.conv2d(xq.to(layer["dt"]), layer["wq"].to(layer["dt"]), padding=1).to(torch.int32)
    if layer["shift"] is None:
        a0 = acc[0]
        top = float(a0.clamp(min=0).max()) if layer["relu"] else float(a0.abs().max())
        layer["shift"] = min(31, max(1, math.ceil(math.log2(max(top * 1.25, 1.0) / (255 if layer["relu"] else 127)))))
    s = layer["shift"]
    q = (acc + (1 << (s - 1))) >> s
    q = q.clamp_(0, 255).to(torch.uint8) if layer["relu"] else q.clamp_(-128, 127).to(torch.int8)
    scale = layer["sw"] * 2.0 ** s
    y = q.float() * (scale.view(1, -1, 1, 1) * sx)
    if bias is not None:
        y = y + bias.float().view(1, -1, 1, 1)
    return y.to(x.dtype)
