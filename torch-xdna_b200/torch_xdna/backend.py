"""torch.compile(model, backend="xdna"): GEMMs, 3x3 convs and Qwen3 stacks on the B200 kernels.

A pass over Dynamo's FX graph (the same patterns as R:torch_xdna/backend.py:59-256):

  F.linear(x, W, b), x @ W / torch.mm / torch.matmul / .mm / .matmul with a 2-D float parameter W,
  and torch.addmm(b, x, W) (alpha = beta = 1, 1-D parameter bias)   -> xdna::linear
  xdna::linear nodes (not transposed) that read the same x          -> one xdna::linear_cat + narrows
  conv2d of a [Co, Ci, 3, 3] parameter, stride 1, padding 1 / "same", dilation 1, groups 1
                                                                    -> conv3x3_int8 (xdna::conv3x3_fused)
  a ReLU that is the sole user of such a conv without bias          -> fused into the requantise
  a transformers Qwen3Model of Qwen3-0.6B's shapes into a linear head
                                                                    -> xdna::qwen3_stack (stack.py)

The rest of the graph goes to Inductor (fallback="inductor") or runs as written (fallback="eager").
GEMMs between two activations (attention scores) are not rewritten.

Where the reference decomposes each W8A8 linear into quantise / xdna::linear_i8 / dequantise graph
ops so that its CPU compiler can fuse them (R:torch_xdna/backend.py:206-226), the B200 build keeps
xdna::linear / linear_cat whole: the quantise is one HBM-bound kernel and the dequantise is the
GEMM's epilogue, with the same arithmetic and therefore the same bits.
"""

import logging
import operator

import torch
import torch.nn.functional as F

from . import config as _config
from . import kernels, ops

log = logging.getLogger("torch_xdna")

LINEAR = {torch._C._nn.linear, F.linear}
CONV2D = {torch.conv2d, F.conv2d}
RELU = {torch.relu, F.relu, torch.relu_}
MATMUL = {operator.matmul, torch.matmul}
FLOATS = (torch.float32, torch.bfloat16, torch.float16)


def _parameter_nodes(gm, example_inputs):
    """Placeholders that hold parameters or buffers: the weights worth quantising once."""
    placeholders = [n for n in gm.graph.nodes if n.op == "placeholder"]
    found = set()
    for node, value in zip(placeholders, example_inputs):
        if isinstance(value, torch.nn.Parameter) or "_parameters_" in node.name or "_buffers_" in node.name:
            found.add(node)
    return found


def _tensor_of(node, attr):
    if node.op == "get_attr":
        return attr(node.target)
    if node.op == "placeholder":
        return node.meta.get("example_value")
    return None


def offload_gemms(gm: torch.fx.GraphModule, example_inputs, cfg) -> int:
    """Rewrite offloadable GEMMs and 3x3 convs of `gm` in place; returns how many were rewritten."""
    params = _parameter_nodes(gm, example_inputs)

    def attr(target):
        obj = gm
        for part in target.split("."):
            obj = getattr(obj, part)
        return obj

    def is_static(n):
        return isinstance(n, torch.fx.Node) and (n in params or n.op == "get_attr")

    def is_weight(n):
        if not is_static(n):
            return False
        t = _tensor_of(n, attr)
        return isinstance(t, torch.Tensor) and t.dim() == 2 and t.dtype in FLOATS

    def is_bias_vector(n):
        t = n.meta.get("example_value") if isinstance(n, torch.fx.Node) else None
        return is_static(n) and isinstance(t, torch.Tensor) and t.dim() == 1

    cid = ops.config_id(cfg)
    count = 0
    for node in list(gm.graph.nodes):
        if node.op == "call_function" and node.target in LINEAR:
            x = node.args[0] if node.args else node.kwargs.get("input")
            w = node.args[1] if len(node.args) > 1 else node.kwargs.get("weight")
            b = node.args[2] if len(node.args) > 2 else node.kwargs.get("bias")
            transposed = False
        elif (((node.op == "call_function" and node.target in MATMUL | {torch.mm})
               or (node.op == "call_method" and node.target in ("matmul", "mm", "__matmul__")))
              and len(node.args) == 2 and not node.kwargs):
            x, w = node.args            # x @ W with W [K, N]
            b, transposed = None, True
        elif (node.op == "call_function" and node.target is torch.addmm and len(node.args) == 3
              and set(node.kwargs) <= {"beta", "alpha"}
              and all(node.kwargs.get(k, 1) == 1 for k in ("beta", "alpha"))):
            b, x, w = node.args         # b + x @ W (HF Conv1D)
            transposed = True
            if b is not None and not is_bias_vector(b):
                continue
        else:
            continue
        if not is_weight(w):
            continue
        with gm.graph.inserting_after(node):
            new = gm.graph.call_function(torch.ops.xdna.linear.default, (x, w, b, transposed, cid))
        new.meta.update(node.meta)
        node.replace_all_uses_with(new)
        gm.graph.erase_node(node)
        count += 1
    if cfg.fuse:
        _fuse_shared_input(gm, cid)
    count += _offload_convs(gm, params, cid, attr, cfg)
    if cfg.fuse:
        _chain_convs(gm)
    gm.graph.lint()
    gm.recompile()
    return count


def _conv_args(node):
    """(x, weight, bias, stride, padding, dilation, groups) of a conv2d call."""
    names = ("input", "weight", "bias", "stride", "padding", "dilation", "groups")
    defaults = dict(bias=None, stride=1, padding=0, dilation=1, groups=1)
    args = dict(zip(names, node.args), **node.kwargs)
    return [args.get(k, defaults.get(k)) for k in names]


def _pair(v):
    return tuple(v) if isinstance(v, (tuple, list)) else (v, v)


def _is_relu(n):
    return (n.op == "call_function" and n.target in RELU) or (n.op == "call_method" and n.target in ("relu", "relu_"))


def _offload_convs(gm, params, cid, attr, cfg):
    """3x3 / stride-1 / padding-1 / groups-1 convs of a parameter weight -> conv3x3_int8
    (R:torch_xdna/backend.py:130-174). A sole-user ReLU is fused: into the requantise for a bias-free conv
    (as the reference does), into the epilogue after the bias for a biased one. With cfg.conv_ext, also 1x1
    convs (stride 1 or 2, no padding) and 3x3 convs with stride 2 and padding 1 -> conv_ext_int8
    (xdna::conv_int8), the same arithmetic on the conv's own stride and padding."""
    from .conv import conv3x3_int8, conv_ext_int8, supported

    if not cfg.offload:
        return 0
    count = 0
    for node in list(gm.graph.nodes):
        if node.op != "call_function" or node.target not in CONV2D:
            continue
        x, w, b, stride, padding, dilation, groups = _conv_args(node)
        if _pair(dilation) != (1, 1) or groups != 1:
            continue
        if not (isinstance(w, torch.fx.Node) and (w in params or w.op == "get_attr")):
            continue
        wt = _tensor_of(w, attr)
        xt = x.meta.get("example_value") if isinstance(x, torch.fx.Node) else None
        if not (isinstance(wt, torch.Tensor) and wt.dim() == 4 and isinstance(xt, torch.Tensor) and xt.dim() == 4
                and xt.dtype in FLOATS):
            continue
        k, s = tuple(wt.shape[2:]), _pair(stride)
        pad = (0, 0) if padding == "valid" or (padding == "same" and k == (1, 1)) else \
            (1, 1) if (padding == "same" and k == (3, 3)) else _pair(padding)
        if k == (3, 3) and s == (1, 1) and pad == (1, 1):
            if not supported(int(wt.shape[1]), int(wt.shape[0]), int(xt.shape[2]), int(xt.shape[3])):
                continue
            ext = False
        elif cfg.conv_ext and ((k == (1, 1) and s in ((1, 1), (2, 2)) and pad == (0, 0))
                               or (k == (3, 3) and s == (2, 2) and pad == (1, 1))):
            ext = True
        else:
            continue
        users = list(node.users)
        relu = users[0] if (cfg.fuse and len(users) == 1 and _is_relu(users[0])) else None
        last = relu or node
        with gm.graph.inserting_after(last):
            # bias-free: the ReLU goes into the requantise (the reference's fusion); biased: it is applied
            # in the epilogue after the bias (the reference leaves it in the graph; the values are the same)
            fused, post = relu is not None and b is None, relu is not None and b is not None
            if ext:
                new = gm.graph.call_function(conv_ext_int8, (x, w, b, s[0], fused, cid, post))
            else:
                new = gm.graph.call_function(conv3x3_int8, (x, w, b, fused, cid, post))
        new.meta.update(last.meta)
        last.replace_all_uses_with(new)
        if relu is not None:
            gm.graph.erase_node(relu)
        gm.graph.erase_node(node)
        count += 1
    return count


MAXPOOL2D = {F.max_pool2d, torch.max_pool2d}


def _is_maxpool_2x2(n):
    """max_pool2d(x, 2) / (x, 2, 2): a 2x2 window, stride 2, no padding, dilation 1, floor, no indices."""
    if n.op != "call_function" or n.target not in MAXPOOL2D:
        return False
    names = ("input", "kernel_size", "stride", "padding", "dilation", "ceil_mode", "return_indices")
    a = dict(zip(names, n.args), **n.kwargs)
    stride = a.get("stride")
    return (_pair(a.get("kernel_size")) == (2, 2) and (stride in (None, []) or _pair(stride) == (2, 2))
            and _pair(a.get("padding", 0)) == (0, 0) and _pair(a.get("dilation", 1)) == (1, 1)
            and not a.get("ceil_mode", False) and not a.get("return_indices", False))


def _chain_convs(gm):
    """Offloaded convs feeding the next offloaded conv directly or through a 2x2 max-pool, with the
    activation in between used by nothing else, become xdna::conv3x3_chain nodes that pass int8 codes
    [N, H, W, C] (and their float factors) instead of a float tensor: the int8 NHWC chaining the reference
    names as its largest remaining conv cost (R:results/conv3x3_cascade.md:214-219). Same values: the next
    conv's quantise rebuilds the float activation with the epilogue's f32 operations. Only float32
    activations with a channel count divisible by 4 are chained."""
    from .conv import IN_CODES, IN_CODES_POOL, IN_FLOAT, conv3x3_chain_int8, conv3x3_int8

    def is_conv(n):
        return isinstance(n, torch.fx.Node) and n.op == "call_function" and n.target is conv3x3_int8

    def chainable(n):  # the activation n produces: f32, channels divisible by 4
        t = n.meta.get("example_value")
        return isinstance(t, torch.Tensor) and t.dtype == torch.float32 and t.dim() == 4 and t.shape[1] % 4 == 0

    link = {}  # producer conv -> (consumer conv, pool node or None)
    for c2 in gm.graph.nodes:
        if not is_conv(c2):
            continue
        src, pool = c2.args[0], None
        if isinstance(src, torch.fx.Node) and _is_maxpool_2x2(src) and len(src.users) == 1:
            pool, src = src, src.args[0]
        if is_conv(src) and len(src.users) == 1 and chainable(src) and src not in link:
            link[src] = (c2, pool)
    if not link:
        return 0
    fed = {c2: (c1, pool) for c1, (c2, pool) in link.items()}
    codes = {}  # producer -> (codes node, meta node, its ReLU applies after the bias)
    erase = []
    for n in list(gm.graph.nodes):
        if n not in link and n not in fed:
            continue
        x, w, b, relu, cid = n.args[:5]
        post_relu = n.args[5] if len(n.args) > 5 else False
        if n in fed:
            c1, pool = fed[n]
            xin, xmeta, in_ra = codes[c1]
            in_mode = IN_CODES_POOL if pool is not None else IN_CODES
            if pool is not None:
                erase.append(pool)
        else:
            xin, xmeta, in_mode, in_ra = x, None, IN_FLOAT, False
        out_q = n in link
        out_pool = out_q and link[n][1] is not None
        with gm.graph.inserting_after(n):
            call = gm.graph.call_function(conv3x3_chain_int8, (xin, xmeta, w, b, relu, cid, post_relu, in_mode, in_ra,
                                                               out_q, out_pool))
        with gm.graph.inserting_after(call):
            first = gm.graph.call_function(operator.getitem, (call, 0))
        with gm.graph.inserting_after(first):
            second = gm.graph.call_function(operator.getitem, (call, 1))
        if out_q:
            codes[n] = (first, second, post_relu)
        else:
            first.meta.update(n.meta)
            n.replace_all_uses_with(first)
        erase.append(n)
    for n in reversed(list(gm.graph.nodes)):  # consumers before producers
        if n in erase:
            gm.graph.erase_node(n)
    return len(link)


def _out_features(w):
    t = w.meta.get("example_value") if isinstance(w, torch.fx.Node) else None
    return int(t.shape[0]) if isinstance(t, torch.Tensor) else None


def _fuse_shared_input(gm, cid):
    """xdna::linear nodes reading the same input (q/k/v, gate/up) -> one xdna::linear_cat + narrows
    (R:torch_xdna/backend.py:177-203)."""
    groups = {}
    for node in gm.graph.nodes:
        if node.op == "call_function" and node.target is torch.ops.xdna.linear.default and not node.args[3]:
            groups.setdefault(node.args[0], []).append(node)
    for x, members in groups.items():
        if len(members) < 2:
            continue
        weights = [m.args[1] for m in members]
        sizes = [_out_features(w) for w in weights]
        if None in sizes:
            continue
        with gm.graph.inserting_before(members[0]):
            cat = gm.graph.call_function(torch.ops.xdna.linear_cat.default,
                                         (x, weights, [m.args[2] for m in members], cid))
            start = 0
            for m, n in zip(members, sizes):
                part = gm.graph.call_function(torch.narrow, (cat, -1, start, n))
                part.meta.update(m.meta)
                m.replace_all_uses_with(part)
                start += n
        for m in members:
            gm.graph.erase_node(m)


def _compile(gm, example_inputs, cfg):
    n = offload_gemms(gm, example_inputs, cfg) if cfg.offload else 0
    if cfg.verbose:
        log.warning("torch_xdna: %d GEMMs / convs offloaded in a graph of %d nodes (policy=%s, fallback=%s)",
                    n, len(gm.graph.nodes), cfg.policy, cfg.fallback)
    if cfg.fallback == "eager":
        return gm.forward
    from torch._inductor.compile_fx import compile_fx

    return compile_fx(gm, example_inputs)


def xdna_backend(gm: torch.fx.GraphModule, example_inputs, options=None, mode=None):
    """The torch.compile backend; `options` are torch_xdna.Config fields (R:torch_xdna/backend.py:246-256).

    Unlike the reference there is no CPU route: with offloading on (policy other than "cpu") and no
    usable B200, compiling raises XdnaUnavailable with the reason instead of falling back."""
    cfg = _config.config.merged(options)
    if cfg.offload:
        kernels.require()
        if cfg.stacks:
            from . import stack

            plan = stack.find(gm, example_inputs)
            if plan is not None:
                return stack.compile_fused(gm, example_inputs, cfg, ops.config_id(cfg), plan, _compile)
    return _compile(gm, example_inputs, cfg)
