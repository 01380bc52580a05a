"""xdna::qwen3_stack: a whole Qwen3-0.6B-sized transformer stack and its linear head on the B200.

The backend looks in Dynamo's graph for a transformers `Qwen3Model` whose last hidden states feed only
a linear layer, with Qwen3-0.6B's shapes, any depth, and attention under a 4-D mask that is a graph
input (the same search as R:torch_xdna/stack.py:111-240). Such a graph is compiled twice:

  fused  the stack and the head replaced by xdna::qwen3_stack, which runs libxdna_b200's
         xdna_qwen3_stack: every layer (bf16 tcgen05 GEMMs with fused q/k-norm + RoPE, SwiGLU and
         residual epilogues, GQA flash attention), the final norm and the head, on one stream;
  plain  the graph as the backend compiles any other (its linears offloaded as W8A8)

and Dispatch picks one per call from the mask: the fused graph for a causal mask, a prefix-block mask
(the reference's OmniVoice layout, rows past each length zero), a general bool mask, or a float mask of
0 / large negatives; the plain graph for anything else. Unlike the reference's NPU program (prefix
blocks of at most 384 positions) there is no length limit.

The first fused call of each mask kind and size is checked against the original graph run eagerly in
fp32 (relative norm <= 0.1 over the valid rows, R:torch_xdna/stack.py:444-460); a mismatch raises.
"""

import copy
import ctypes
import logging
import operator
import re
import threading
import time
import weakref

import torch
import torch.nn.functional as F

from . import kernels
from .runtime import DEVICE, XdnaResultMismatch, stats

log = logging.getLogger("torch_xdna")
_lock = threading.RLock()

LINEAR = {torch._C._nn.linear, F.linear}
SDPA = {torch._C._nn.scaled_dot_product_attention, F.scaled_dot_product_attention}
ADD = {operator.add, torch.add}
MUL = {operator.mul, torch.mul}
ROOTS = ("Qwen3Model",)
D, NH, NKV, DH, INTER, EPS = 1024, 16, 8, 128, 3072, 1e-6
LAYER_KEYS = ("q", "k", "v", "o", "gate", "up", "down", "input_norm", "post_norm", "q_norm", "k_norm")
SHAPES = dict(q=(NH * DH, D), k=(NKV * DH, D), v=(NKV * DH, D), o=(D, NH * DH), gate=(INTER, D), up=(INTER, D),
              down=(D, INTER), input_norm=(D,), post_norm=(D,), q_norm=(DH,), k_norm=(DH,))
VERIFY_TOL = 0.1

_PROJ = re.compile(r"layers\.(\d+)\.(?:self_attn\.(q|k|v|o)_proj|mlp\.(gate|up|down)_proj)")
_NORMS = {"input_layernorm": "input_norm", "post_attention_layernorm": "post_norm",
          "self_attn.q_norm": "q_norm", "self_attn.k_norm": "k_norm"}
_NORM = re.compile(r"layers\.(\d+)\.(" + "|".join(re.escape(k) for k in _NORMS) + ")")


# ------------------------------------------------------------------ finding a stack
class _NoStack(Exception):
    pass


class Plan:
    """A stack found in a graph; nodes kept by name so the plan applies to copies of the graph."""

    def __init__(self, region, x, mask, mask_index, head, weights, bias, layers, out_features):
        self.region, self.x, self.mask, self.mask_index, self.head = region, x, mask, mask_index, head
        self.weights, self.bias = weights, bias
        self.layers, self.out_features = layers, out_features

    def tensors(self):
        """Every weight in op order: per layer LAYER_KEYS, then the final norm, the head, inv_freq."""
        return [self.weights[(i, k)] for i in range(self.layers) for k in LAYER_KEYS] + \
            [self.weights["norm"], self.weights["head"], self.weights["inv_freq"]]


def _cls_name(c):
    return c.__name__ if isinstance(c, type) else str(c).rsplit(".", 1)[-1].strip("'>")


def _inner(n):
    path, cls = list(n.meta["nn_module_stack"].values())[-1]
    return path, _cls_name(cls)


def _linear_args(n):
    x = n.args[0] if n.args else n.kwargs.get("input")
    w = n.args[1] if len(n.args) > 1 else n.kwargs.get("weight")
    b = n.args[2] if len(n.args) > 2 else n.kwargs.get("bias")
    return x, w, b


def find(gm, example_inputs):
    """The first Qwen3 stack + linear head in `gm`, as a Plan, or None (R:torch_xdna/stack.py:111-131)."""
    placeholders = [n for n in gm.graph.nodes if n.op == "placeholder"]
    value = dict(zip(placeholders, example_inputs))
    roots = {}
    for n in gm.graph.nodes:
        if n.op not in ("call_function", "call_method", "call_module"):
            continue
        for path, cls in (n.meta.get("nn_module_stack") or {}).values():
            if _cls_name(cls) in ROOTS:
                roots.setdefault(path, []).append(n)
                break
    for root, region in roots.items():
        try:
            return _plan(root, region, value, placeholders)
        except _NoStack as e:
            log.info("torch_xdna: %s is not a stack xdna::qwen3_stack takes: %s", root, e)
    return None


def _plan(root, region, value, placeholders):
    """Checks a Qwen3Model region the way R:torch_xdna/stack.py:134-240 does and collects its weights."""
    inside = set(region)

    def static(n):
        return n.op == "placeholder" and (isinstance(value.get(n), torch.nn.Parameter)
                                          or "_parameters_" in n.name or "_buffers_" in n.name)

    weights, sdpa = {}, []

    def put(key, node):
        t = value.get(node)
        if not isinstance(t, torch.Tensor):
            raise _NoStack(f"{key}: no tensor")
        if weights.setdefault(key, t) is not t:
            raise _NoStack(f"two tensors for {key}")

    for n in region:
        path, cls = _inner(n)
        rel = "" if path == root else path[len(root) + 1:]
        others = n.all_input_nodes
        if n.op == "call_function" and n.target in LINEAR:
            _, w, b = _linear_args(n)
            m = _PROJ.fullmatch(rel)
            if m is None or b is not None or not static(w):
                raise _NoStack(f"a linear in {rel or 'the root'}")
            put((int(m[1]), m[2] or m[3]), w)
            others = [a for a in others if a is not w]
        elif n.op == "call_function" and n.target in SDPA:
            sdpa.append(n)
        for a in others:
            if not static(a):
                continue
            m = _NORM.fullmatch(rel)
            if m:
                put((int(m[1]), _NORMS[m[2]]), a)
            elif rel in ("norm", "rotary_emb"):
                put("norm" if rel == "norm" else "inv_freq", a)
            else:
                raise _NoStack(f"parameter {a.name} used in {rel or 'the root'}")
        consts = [a for a in n.args if isinstance(a, float)]
        if n.op == "call_function" and consts:
            if n.target in ADD and cls.endswith("RMSNorm") and any(abs(c - EPS) > 1e-12 for c in consts):
                raise _NoStack(f"RMSNorm eps {consts} (the kernels use {EPS})")
            if n.target in MUL and rel == "rotary_emb" and any(c != 1.0 for c in consts):
                raise _NoStack(f"RoPE attention scaling {consts}")

    layers = 1 + max((k[0] for k in weights if isinstance(k, tuple)), default=-1)
    if layers < 1:
        raise _NoStack("no layers")
    for i in range(layers):
        for k in LAYER_KEYS:
            t = weights.get((i, k))
            if t is None or tuple(t.shape) != SHAPES[k]:
                raise _NoStack(f"layer {i} {k}: {None if t is None else tuple(t.shape)}, need {SHAPES[k]}")
    if tuple(getattr(weights.get("norm"), "shape", ())) != (D,) or \
            tuple(getattr(weights.get("inv_freq"), "shape", ())) != (DH // 2,):
        raise _NoStack("final norm / RoPE frequencies")

    masks = set()
    for n in sdpa:
        kw = dict(zip(("query", "key", "value", "attn_mask", "dropout_p", "is_causal", "scale"), n.args))
        kw.update(n.kwargs)
        scale = kw.get("scale")
        if kw.get("dropout_p", 0.0) != 0.0 or kw.get("is_causal", False) or \
                (scale is not None and abs(scale - DH ** -0.5) > 1e-6):
            raise _NoStack("attention: dropout, is_causal or another scale")
        masks.add(kw.get("attn_mask"))
    if len(sdpa) != layers or len(masks) != 1:
        raise _NoStack(f"{len(sdpa)} attentions for {layers} layers, {len(masks)} masks")
    mask = masks.pop()
    mv = value.get(mask)
    if not isinstance(mask, torch.fx.Node) or mask.op != "placeholder" or not isinstance(mv, torch.Tensor) \
            or mv.dim() != 4 or not (mv.dtype == torch.bool or mv.is_floating_point()):
        raise _NoStack("the attention mask is not a 4-D input of the graph")

    ext = {}
    for n in region:
        for a in n.all_input_nodes:
            if a not in inside and a is not mask and not static(a):
                ext[a] = None
    rest = [a for a in ext if not (a.op == "placeholder" and isinstance(value.get(a), (int, torch.SymInt)))]
    if len(rest) != 1:
        raise _NoStack(f"inputs {[a.name for a in rest]}")
    x = rest[0]
    xv = x.meta.get("example_value")
    if not (isinstance(xv, torch.Tensor) and xv.dim() == 3 and xv.shape[-1] == D and xv.is_floating_point()):
        raise _NoStack("hidden states are not [B, L, 1024]")

    outs = [n for n in region if any(u not in inside for u in n.users)]
    if len(outs) != 1 or len(outs[0].users) != 1:
        raise _NoStack("the stack's output has other users than one head")
    head = next(iter(outs[0].users))
    if not (head.op == "call_function" and head.target in LINEAR):
        raise _NoStack(f"the stack's output goes to {head.target}")
    hx, hw, hb = _linear_args(head)
    W = value.get(hw) if static(hw) else None
    Bv = value.get(hb) if hb is not None and static(hb) else None
    if hx is not outs[0] or not isinstance(W, torch.Tensor) or W.dim() != 2 or W.shape[1] != D or \
            (hb is not None and not (isinstance(Bv, torch.Tensor) and tuple(Bv.shape) == (W.shape[0],))):
        raise _NoStack("the head is not a linear of a parameter [N, 1024]")
    weights["head"] = W
    return Plan([n.name for n in region], x.name, mask.name, placeholders.index(mask), head.name, weights, Bv,
                layers, int(W.shape[0]))


# ------------------------------------------------------------------ the fused graph
def copy_module(gm):
    """A new GraphModule with a copy of `gm`'s graph (same attributes, same node names)."""
    g = torch.fx.Graph()
    g._codegen = copy.deepcopy(gm.graph._codegen)
    g.output(g.graph_copy(gm.graph, {}))
    new = torch.fx.GraphModule(gm, g)
    new.meta.update(gm.meta)
    return new


def fuse(gm, plan, stack_id, cfg_id):
    """Replace the stack and its head in `gm` by xdna::qwen3_stack (R:torch_xdna/stack.py:254-267)."""
    by = {n.name: n for n in gm.graph.nodes}
    head = by[plan.head]
    with gm.graph.inserting_before(head):
        new = gm.graph.call_function(torch.ops.xdna.qwen3_stack.default, (by[plan.x], by[plan.mask], stack_id, cfg_id))
    new.meta.update(head.meta)
    head.replace_all_uses_with(new)
    gm.graph.erase_node(head)
    for name in reversed(plan.region):
        gm.graph.erase_node(by[name])
    gm.graph.lint()
    gm.recompile()


# ------------------------------------------------------------------ weights on the device
class Packed:
    """A stack's weights in the kernels' layout: bf16 matrices (q/k/v fused, gate/up interleaved in blocks
    of 32 rows), f32 norms, the bf16 head and its bias, and the per-layer pointer table."""

    def __init__(self, ts, layers, bias):
        n = len(LAYER_KEYS)
        dev = ts[0].device
        self.keep = []
        table = (kernels.Qwen3Layer * layers)()
        for i in range(layers):
            w = dict(zip(LAYER_KEYS, ts[i * n:(i + 1) * n]))
            bf = {k: w[k].detach().to(torch.bfloat16) for k in ("q", "k", "v", "o", "gate", "up", "down")}
            qkv = torch.cat([bf["q"], bf["k"], bf["v"]]).contiguous()
            gu = torch.stack([bf["gate"].reshape(INTER // 32, 32, D), bf["up"].reshape(INTER // 32, 32, D)],
                             dim=1).reshape(2 * INTER, D).contiguous()
            o, down = bf["o"].contiguous(), bf["down"].contiguous()
            norms = [w[k].detach().float().contiguous() for k in ("input_norm", "post_norm", "q_norm", "k_norm")]
            self.keep += [qkv, gu, o, down] + norms
            table[i] = kernels.Qwen3Layer(qkv.data_ptr(), o.data_ptr(), gu.data_ptr(), down.data_ptr(),
                                          *[t.data_ptr() for t in norms])
        norm, head, inv_freq = ts[layers * n:]
        self.final_norm = norm.detach().float().contiguous()
        self.head = head.detach().to(torch.bfloat16).contiguous()
        self.bias = bias.detach().float().contiguous() if bias is not None else None
        self.inv_freq = inv_freq.detach().float().to(dev)
        self.table = table
        self.layers = layers
        self._rope = {}

    def rope(self, L):
        """cos / sin at positions 0..L-1, as transformers computes them (f32 outer product), in the kernel's
        [16, L, 4] layout (kernels.rope_layout)."""
        if L not in self._rope:
            pos = torch.arange(L, device=self.inv_freq.device, dtype=torch.float32)
            freqs = pos[:, None] * self.inv_freq[None, :]
            self._rope[L] = (kernels.rope_layout(freqs.cos()), kernels.rope_layout(freqs.sin()))
        return self._rope[L]


class StackUnsupported(RuntimeError):
    pass


class _Stack:
    """One stack found by the backend: its weights (weakly), the packed copy, the checks done."""

    def __init__(self, plan):
        self.refs = [weakref.ref(t) for t in plan.tensors()]
        self.bias = weakref.ref(plan.bias) if plan.bias is not None else None
        self.layers, self.N = plan.layers, plan.out_features
        self.name = f"qwen3 stack {self.layers} layers -> {self.N}"
        self.verified = set()
        self.capture = False
        self.captured = None
        self._packed = None
        self._versions = None

    def packed(self):
        ts = [r() for r in self.refs]
        if any(t is None for t in ts):
            raise RuntimeError("the stack's weights are gone")
        versions = tuple(t._version for t in ts)
        if self._packed is None or versions != self._versions:
            self._packed = Packed(ts, self.layers, self.bias() if self.bias is not None else None)
            self._versions = versions
        return self._packed

    def macs(self, B, L, kind):
        per_token = self.layers * (D * (NH + 2 * NKV) * DH + NH * DH * D + 3 * D * INTER) + D * self.N
        keys = (L + 1) / 2 if kind == kernels.MASK_CAUSAL else L
        return int(per_token * B * L + self.layers * B * 2 * NH * DH * L * keys)


_stacks = []


def register(plan):
    with _lock:
        _stacks.append(_Stack(plan))
        return len(_stacks) - 1


def out_features(stack_id):
    return _stacks[stack_id].N


def lengths(mask):
    """Each sequence's length n when `mask` [B, H, L, L] is a prefix block per sequence (the first n positions
    see exactly those n, later positions only themselves or nothing), else None (R:torch_xdna/stack.py:328-352)."""
    if not isinstance(mask, torch.Tensor) or mask.dim() != 4 or mask.shape[-1] != mask.shape[-2]:
        return None
    allowed = _allowed(mask)
    if allowed is None:
        return None
    if allowed.shape[1] > 1 and not bool((allowed == allowed[:, :1]).all()):
        return None
    a = allowed[:, 0]
    n = a[:, 0].sum(-1)
    ar = torch.arange(a.shape[-1], device=a.device)
    want = ar[None, None, :] < n[:, None, None]
    rows = ar[None, :, None] < n[:, None, None]
    pad = (a == (ar[:, None] == ar[None, :])) | ~a.any(-1, keepdim=True)
    if not bool(torch.where(rows, a == want, pad).all()):
        return None
    return n.tolist()


def _allowed(mask):
    """The mask as bool (True = may attend), or None for float masks other than 0 / large negatives."""
    if mask.dtype == torch.bool:
        return mask
    if mask.is_floating_point():
        allowed = mask == 0
        if not bool((allowed | (mask <= -1e4)).all()):
            return None
        return allowed
    return None


def classify(mask, B, L):
    """(kind, lens tensor or None, bool mask or None) for the attention kernel, or None if unsupported."""
    if not isinstance(mask, torch.Tensor) or mask.dim() != 4 or tuple(mask.shape[-2:]) != (L, L) \
            or mask.shape[0] not in (1, B) or mask.shape[1] not in (1, NH):
        return None
    allowed = _allowed(mask)
    if allowed is None:
        return None
    causal = torch.ones(L, L, dtype=torch.bool, device=mask.device).tril_()
    if bool((allowed == causal).all()):
        return kernels.MASK_CAUSAL, None, None
    if bool(allowed.all()):
        return kernels.MASK_NONE, None, None
    lens = lengths(mask)
    if lens is not None:
        if len(lens) == 1 and B > 1:
            lens = lens * B
        return kernels.MASK_PREFIX, torch.tensor(lens, dtype=torch.int32, device=mask.device), None
    m = allowed.expand(B, allowed.shape[1], L, L).to(torch.uint8).contiguous()
    return kernels.MASK_BOOL, None, m


def run(cfg, stack_id, x, mask):
    """xdna::qwen3_stack: hidden states x [B, L, 1024] -> the head's output [B, L, N], on the B200."""
    kernels._cuda(x, mask)
    st = _stacks[stack_id]
    B, L = x.shape[:2]
    cls = classify(mask, B, L)
    if cls is None:
        raise StackUnsupported(f"{st.name}: the attention mask is not causal, prefix-block, bool or 0/-inf")
    kind, lens, m = cls
    t0 = time.perf_counter()
    with _lock:
        pk = st.packed()
        cos, sin = pk.rope(L)
        xs = x.detach().reshape(B * L, D).to(torch.float32).contiguous().clone()
        out = torch.empty((B * L, st.N), dtype=x.dtype if x.dtype in (torch.float32, torch.bfloat16, torch.float16)
                          else torch.float32, device=x.device)
        ws = torch.empty(kernels.qwen3_stack_workspace(B, L), dtype=torch.uint8, device=x.device)
        kernels.qwen3_stack(pk.table, pk.final_norm, pk.head, pk.bias, cos, sin, EPS, xs, B, L, kind, lens, m, out, ws)
        out = out.view(B, L, st.N)
        if kind == kernels.MASK_PREFIX:      # rows past each sequence's length are zeros (R:torch_xdna/stack.py:377-379)
            keep = torch.arange(L, device=x.device)[None, :] < lens.to(x.device)[:, None]
            out = out * keep[:, :, None].to(out.dtype)
        if st.capture:
            st.captured = out.float().clone()
        stats.launches += 7 * st.layers + 2
    stats.calls[DEVICE] += 1
    stats.seconds[DEVICE] += time.perf_counter() - t0
    stats.macs[DEVICE] += st.macs(B, L, kind)
    return out


class _Stop(Exception):
    pass


class _Until(torch.fx.Interpreter):
    """Runs a graph eagerly up to one node and keeps its value."""

    def __init__(self, gm, name):
        super().__init__(gm, garbage_collect_values=True)
        self.extra_traceback = False
        self.name, self.value = name, None

    def run_node(self, n):
        v = super().run_node(n)
        if n.name == self.name:
            self.value = v
            raise _Stop()
        return v


class Dispatch:
    """What the backend returns for a graph with a stack: the fused graph when the mask is one the kernels
    take, else the plain one; the first fused call of each (mask kind, B, L) is checked against the
    original graph run eagerly in fp32 (R:torch_xdna/stack.py:412-460)."""

    def __init__(self, plan, stack_id, cfg, fused, plain, orig):
        self.plan, self.stack_id, self.cfg = plan, stack_id, cfg
        self.fused, self.plain, self.orig = fused, plain, orig

    def __call__(self, *args):
        st = _stacks[self.stack_id]
        mask = args[self.plan.mask_index]
        shape = None
        for a in args:
            if isinstance(a, torch.Tensor) and a.dim() == 3 and a.shape[-1] == D and a.is_floating_point():
                shape = tuple(a.shape[:2])
                break
        cls = classify(mask, *shape) if shape is not None else None
        if cls is None:
            stats.stacks[(st.name, "plain")] += 1
            return self.plain(*args)
        key = (cls[0],) + shape
        check = self.cfg.verify == "always" or (self.cfg.verify == "first" and key not in st.verified)
        try:
            st.capture = check
            out = self.fused(*args)
            if check:
                self._check(st, args, mask, shape, cls, key)
        finally:
            st.capture, st.captured = False, None
        stats.stacks[(st.name, DEVICE)] += 1
        return out

    def _check(self, st, args, mask, shape, cls, key):
        """The fused call's stack output vs the original graph's, run eagerly in fp32."""
        it = _Until(self.orig, self.plan.head)
        with torch.no_grad():
            try:
                it.run(*[a.float() if isinstance(a, torch.Tensor) and a.is_floating_point() and a is not mask else a
                         for a in args])
            except _Stop:
                pass
        if it.value is None:
            raise RuntimeError(f"{self.plan.head} not reached")
        B, L = shape
        rows = torch.ones(B, L, dtype=torch.bool, device=it.value.device)
        if cls[0] == kernels.MASK_PREFIX:
            rows = torch.arange(L, device=rows.device)[None, :] < cls[1][:, None]
        got = st.captured[rows].double()
        want = it.value.float()[rows].double()
        err = float((got - want).norm() / want.norm().clamp(min=1e-30))
        stats.checks.append((f"{st.name}, mask kind {cls[0]}, {B}x{L}", f"rel err {err:.4f} vs the model in fp32"))
        if not bool(torch.isfinite(got).all()) or err > VERIFY_TOL:
            raise XdnaResultMismatch(f"{st.name} disagrees with the model: rel err {err:.3g}")
        st.verified.add(key)


def compile_fused(gm, example_inputs, cfg, cfg_id, plan, compile_graph):
    """The Dispatch over the fused and the plain compilation of `gm` (R:torch_xdna/stack.py:463-473)."""
    orig = copy_module(gm)
    fused = copy_module(gm)
    sid = register(plan)
    fuse(fused, plan, sid, cfg_id)
    if cfg.verbose:
        log.warning("torch_xdna: %s (%d nodes) -> xdna::qwen3_stack", _stacks[sid].name, len(plan.region) + 1)
    return Dispatch(plan, sid, cfg, compile_graph(fused, example_inputs, cfg), compile_graph(gm, example_inputs, cfg),
                    orig)
