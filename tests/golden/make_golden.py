"""Generate the golden vectors that pin the oracle to the reference (AyaSakura-comp/torch-xdna).

Runs the UNMODIFIED reference package on the CPU, in this container only:

    PYTHONPATH=<reference checkout> CXX=/usr/bin/g++ TORCH_XDNA_DISABLE_NPU=1 \
        python tests/golden/make_golden.py <reference checkout>

(the script re-executes itself with that environment when given the checkout path). Inputs are
drawn from numpy's PCG64 generator (bit-identical on every platform) so that a test can rebuild
every input from its seed; each case stores the SHA-256 of its inputs next to the reference's
outputs, so a test can tell a regenerated input apart from a different one.

What is recorded, per case (all through the reference's own public code):
  linear  torch.compile(backend="xdna", options={"policy": "cpu"}) outputs, and
          runtime.linear_i8 (int32 accumulators + weight scales) on the same quantised rows
          (R:torch_xdna/runtime.py:145-148,358-399);
  conv    conv.conv3x3_int8 with no NPU (ConvLayer.cpu integers: shift, q, scale, y),
          R:torch_xdna/conv.py:43-51,164-189;
  stack   the fp32 eager transformers Qwen3Model + linear head that the reference's first-call
          check compares the fused stack against, R:torch_xdna/stack.py:444-460.
Small cases keep every tensor; full-size cases keep digests of the outputs.
"""

import hashlib
import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def sha(a) -> str:
    a = np.ascontiguousarray(a)
    return hashlib.sha256(a.tobytes()).hexdigest()


def rng(seed):
    return np.random.Generator(np.random.PCG64(seed))


# ---------------------------------------------------------------- shared input builders
# (tests import these to rebuild inputs; they use numpy only)
def linear_inputs(seed, rows, k, n, x_std=1.0, w_std=0.02, bias=True):
    g = rng(seed)
    x = g.standard_normal((rows, k), dtype=np.float32) * np.float32(x_std)
    w = g.standard_normal((n, k), dtype=np.float32) * np.float32(w_std)
    b = (g.standard_normal((n,), dtype=np.float32) * np.float32(w_std)) if bias else None
    return x, w, b


def conv_inputs(seed, n, ci, co, h, w, bias=False, bias_std=0.01):
    g = rng(seed)
    x = g.standard_normal((n, ci, h, w), dtype=np.float32)
    # Kaiming-normal for ReLU: std = sqrt(2 / fan_in)
    wt = g.standard_normal((co, ci, 3, 3), dtype=np.float32) * np.float32(np.sqrt(2.0 / (ci * 9)))
    b = (g.standard_normal((co,), dtype=np.float32) * np.float32(bias_std)) if bias else None
    return x, wt, b


def stack_inputs(seed, layers, head_n, batch, seq, norm_jitter=0.1):
    """Qwen3-0.6B widths. Weights ~N(0, 0.02); norm weights 1 + jitter; x ~N(0, 1)."""
    g = rng(seed)
    D, NH, NKV, DH, INTER = 1024, 16, 8, 128, 3072

    def n(*shape, std=0.02):
        return g.standard_normal(shape, dtype=np.float32) * np.float32(std)

    def norm(d):
        return (1.0 + g.standard_normal((d,), dtype=np.float32) * np.float32(norm_jitter)).astype(np.float32)

    ls = []
    for _ in range(layers):
        ls.append(dict(q=n(NH * DH, D), k=n(NKV * DH, D), v=n(NKV * DH, D), o=n(D, NH * DH), gate=n(INTER, D),
                       up=n(INTER, D), down=n(D, INTER), input_norm=norm(D), post_norm=norm(D), q_norm=norm(DH),
                       k_norm=norm(DH)))
    final = norm(D)
    head = n(head_n, D)
    head_b = n(head_n)
    x = g.standard_normal((batch, seq, D), dtype=np.float32)
    return ls, final, head, head_b, x


def causal_mask(batch, seq):
    m = np.tril(np.ones((seq, seq), dtype=bool))
    return np.broadcast_to(m, (batch, 1, seq, seq)).copy()


def prefix_mask(lens, seq):
    """The reference test's OmniVoice mask: the first n positions see those n; padding sees itself."""
    m = np.zeros((len(lens), 1, seq, seq), dtype=bool)
    for b, n in enumerate(lens):
        m[b, :, :n, :n] = True
        i = np.arange(n, seq)
        m[b, :, i, i] = True
    return m


# ---------------------------------------------------------------- generation (needs the reference)
def _rel_err(y, x2, w, transposed, b):
    import torch

    wf = w.detach().float()
    ref = x2.float() @ (wf if transposed else wf.t())
    if b is not None:
        ref = ref + torch.from_numpy(b)
    return float(((y.float().reshape(ref.shape) - ref).norm() / ref.norm()).item())


LINEAR_CASES = [
    # name, seed, rows, K, N, bias, x dtype, keep tensors
    ("cfg1", 1, 512, 1024, 3072, True, "float32", False),
    ("odd_k200_n300", 2, 37, 200, 300, True, "float32", True),
    ("odd_3d_699", 3, 699, 200, 300, True, "float32", False),
    ("rows1", 4, 1, 1024, 4096, False, "bfloat16", True),
    ("qkv_m128", 5, 128, 1024, 4096, False, "bfloat16", False),
    ("down_m512", 6, 512, 3072, 1024, False, "bfloat16", False),
    ("gateup_m2048", 7, 2048, 1024, 6144, False, "bfloat16", False),
    ("transposed_k300_n520", 8, 300, 1024, 520, False, "float32", True),
]

CONV_CASES = [
    # name, seed, N, Ci, Co, H, W, bias, relu, keep
    ("cfg3_layer", 11, 1, 256, 256, 64, 64, False, True, False),
    ("odd_3_64_13x37", 12, 2, 3, 64, 13, 37, True, False, True),
    ("odd_64_48_relu", 13, 2, 64, 48, 13, 37, False, True, True),
    ("c128_32_same", 14, 1, 128, 32, 32, 64, False, False, True),
    ("noborder_16x16", 15, 3, 32, 16, 16, 16, False, True, True),
]

STACK_CASES = [
    # name, seed, layers, head N, batch, seq, mask kind, lens
    ("stack2_causal", 21, 2, 1000, 2, 48, "causal", None),
    ("stack2_prefix", 22, 2, 1000, 3, 40, "prefix", [40, 29, 17]),
]


def _generate(out_dir: Path):
    import torch

    torch.set_grad_enabled(False)
    import torch_xdna
    from torch_xdna import conv as xconv
    from torch_xdna import ops as xops
    from torch_xdna import runtime

    assert not torch_xdna.npu_available(), "golden vectors come from the reference's CPU route"
    manifest = {"reference": "AyaSakura-comp/torch-xdna (policy='cpu' / CPU-integer route)", "torch": torch.__version__,
                "linear": {}, "conv": {}, "stack": {}}
    arrays = {}

    # ------------------------------------------------------------ linear
    for name, seed, rows, k, n, bias, xdt, keep in LINEAR_CASES:
        x, w, b = linear_inputs(seed, rows, k, n, bias=bias)
        transposed = name.startswith("transposed")
        xt = torch.from_numpy(x).to(getattr(torch, xdt))
        if transposed:
            wt = torch.nn.Parameter(torch.from_numpy(np.ascontiguousarray(w.T)))   # [K, N], x @ W

            class M(torch.nn.Module):
                def __init__(self):
                    super().__init__()
                    self.w = wt

                def forward(self, h):
                    return h @ self.w
            mod = M()
        else:
            mod = torch.nn.Linear(k, n, bias=bias)
            mod.weight.data = torch.from_numpy(w)
            if bias:
                mod.bias.data = torch.from_numpy(b)
        mod = mod.to(getattr(torch, xdt)) if xdt != "float32" else mod
        torch._dynamo.reset()
        runtime.stats.reset()
        comp = torch.compile(mod, backend="xdna", options={"policy": "cpu"})
        y = comp(xt)
        calls = runtime.stats.as_dict()["calls"]
        # the integer half, through the op the graph uses
        cfg = torch_xdna.Config(policy="cpu")
        cid = xops.config_id(cfg)
        x2 = xt.reshape(-1, k)
        sx = x2.abs().amax(dim=1, keepdim=True).float().clamp(min=1e-8) / 127
        xq = torch.round(x2.float() / sx).clamp(-127, 127).to(torch.int8)
        wparam = mod.w if transposed else mod.weight
        acc, sw = torch.ops.xdna.linear_i8(xq, [wparam], transposed, cid)
        # bf16 weights are what the model holds when the module is bf16
        wq_src = wparam.detach()
        ent = dict(seed=seed, rows=rows, K=k, N=n, bias=bias, x_dtype=xdt, transposed=transposed,
                   calls=calls, x_sha=sha(x), w_sha=sha(w), b_sha=sha(b) if bias else None,
                   w_model_dtype=str(wq_src.dtype).replace("torch.", ""),
                   xq_sha=sha(xq.numpy()), sx_sha=sha(sx.numpy().reshape(-1)), acc_sha=sha(acc.numpy()),
                   sw_sha=sha(sw.numpy()), y_dtype=str(y.dtype).replace("torch.", ""),
                   y_sha=sha(y.float().numpy() if y.dtype == torch.bfloat16 else y.numpy()),
                   y_rel_err_vs_fp=_rel_err(y, x2, wparam, transposed, b))
        if keep:
            arrays[f"linear/{name}/acc"] = acc.numpy()
            arrays[f"linear/{name}/sw"] = sw.numpy()
            arrays[f"linear/{name}/sx"] = sx.numpy().reshape(-1)
            arrays[f"linear/{name}/y"] = y.float().numpy()
        manifest["linear"][name] = ent
        print("linear", name, calls, ent["acc_sha"][:12], flush=True)

    # ------------------------------------------------------------ conv (CPU integers)
    for name, seed, n, ci, co, h, wd, bias, relu, keep in CONV_CASES:
        x, wt, b = conv_inputs(seed, n, ci, co, h, wd, bias=bias)
        weight = torch.nn.Parameter(torch.from_numpy(wt))
        cfg = torch_xdna.Config(policy="npu")
        cid = xops.config_id(cfg)
        xt = torch.from_numpy(x)
        sx = xt.abs().amax(dim=(1, 2, 3), keepdim=True).float().clamp(min=1e-8) / 127
        xq = torch.round(xt.float() / sx).clamp(-127, 127).to(torch.int8)
        q, scale = torch.ops.xdna.conv3x3(xq, weight, relu, cid)
        layer = [lay for _, lay in xconv._layers.values() if lay.h == h and lay.w == wd and lay.relu == relu
                 and tuple(lay.wq.shape) == (co, ci, 3, 3)][-1]
        y = xconv.conv3x3_int8(xt, weight, torch.from_numpy(b) if bias else None, relu, cid)
        ent = dict(seed=seed, N=n, Ci=ci, Co=co, H=h, W=wd, bias=bias, relu=relu, shift=int(layer.shift),
                   x_sha=sha(x), w_sha=sha(wt), xq_sha=sha(xq.numpy()), sx_sha=sha(sx.numpy().reshape(-1)),
                   wq_sha=sha(layer.wq.numpy()), sw_sha=sha(layer.sw.numpy()), q_dtype=str(q.dtype).replace("torch.", ""),
                   q_sha=sha(q.numpy()), scale_sha=sha(scale.numpy()), y_sha=sha(y.numpy()))
        if keep:
            arrays[f"conv/{name}/q"] = q.numpy()
            arrays[f"conv/{name}/scale"] = scale.numpy()
            arrays[f"conv/{name}/y"] = y.numpy()
        manifest["conv"][name] = ent
        print("conv", name, "shift", layer.shift, ent["q_sha"][:12], flush=True)

    # cfg3 as the reference's example runs it: 4 x (conv3x3 256->256 + ReLU), 1x256x64x64, layer by layer
    g = rng(31)
    x = g.standard_normal((1, 256, 64, 64), dtype=np.float32)
    ws = [g.standard_normal((256, 256, 3, 3), dtype=np.float32) * np.float32(np.sqrt(2.0 / (256 * 9)))
          for _ in range(4)]
    cfg = torch_xdna.Config(policy="npu")
    cid = xops.config_id(cfg)
    h = torch.from_numpy(x)
    shifts, q_shas = [], []
    for i, wt in enumerate(ws):
        weight = torch.nn.Parameter(torch.from_numpy(wt))
        sx = h.abs().amax(dim=(1, 2, 3), keepdim=True).float().clamp(min=1e-8) / 127
        xq = torch.round(h.float() / sx).clamp(-127, 127).to(torch.int8)
        q, scale = torch.ops.xdna.conv3x3(xq, weight, True, cid)
        q_shas.append(sha(q.numpy()))
        h = xconv.conv3x3_int8(h, weight, None, True, cid)
        lay = [lay for _, lay in xconv._layers.values() if lay.wq.shape[0] == 256 and lay.h == 64][-1]
        shifts.append(int(lay.shift))
    manifest["conv"]["cfg3_chain"] = dict(seed=31, x_sha=sha(x), w_shas=[sha(w) for w in ws], shifts=shifts,
                                          q_shas=q_shas, y_sha=sha(h.numpy()))
    print("cfg3 chain shifts", shifts, flush=True)

    # ------------------------------------------------------------ stack (fp32 eager model)
    from transformers import Qwen3Config, Qwen3Model

    for name, seed, layers, head_n, batch, seq, kind, lens in STACK_CASES:
        ls, final, head, head_b, x = stack_inputs(seed, layers, head_n, batch, seq)
        qc = Qwen3Config(hidden_size=1024, intermediate_size=3072, num_hidden_layers=layers, num_attention_heads=16,
                         num_key_value_heads=8, head_dim=128, vocab_size=16, rms_norm_eps=1e-6,
                         rope_parameters={"rope_type": "default", "rope_theta": 1e6}, attn_implementation="sdpa")
        model = Qwen3Model(qc).eval()
        for i, L in enumerate(ls):
            lay = model.layers[i]
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
        model.norm.weight.data = torch.from_numpy(final)
        mask = causal_mask(batch, seq) if kind == "causal" else prefix_mask(lens, seq)
        hs = model(inputs_embeds=torch.from_numpy(x), attention_mask=torch.from_numpy(mask))[0]
        logits = hs @ torch.from_numpy(head).t() + torch.from_numpy(head_b)
        arrays[f"stack/{name}/logits"] = logits.numpy()
        manifest["stack"][name] = dict(seed=seed, layers=layers, head_n=head_n, batch=batch, seq=seq, mask=kind,
                                       lens=lens, x_sha=sha(x), logits_sha=sha(logits.numpy()))
        print("stack", name, tuple(logits.shape), flush=True)

    np.savez_compressed(out_dir / "golden.npz", **arrays)
    (out_dir / "golden.json").write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")
    print("wrote", out_dir / "golden.npz", out_dir / "golden.json")


if __name__ == "__main__":
    if len(sys.argv) > 1 and os.environ.get("XDNA_GOLDEN_CHILD") != "1":
        ref = str(Path(sys.argv[1]).resolve())
        env = dict(os.environ, PYTHONPATH=ref, CXX="/usr/bin/g++", TORCH_XDNA_DISABLE_NPU="1",
                   XDNA_GOLDEN_CHILD="1")
        sys.exit(subprocess.call([sys.executable, __file__], env=env, cwd="/tmp"))
    _generate(HERE)
