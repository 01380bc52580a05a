"""torch_xdna for B200: a torch.compile backend whose offloaded ops run hand-written sm_100a kernels.

    import torch, torch_xdna
    model = torch.compile(model.cuda(), backend="xdna")

A drop-in for AyaSakura-comp/torch-xdna's backend (same op schemas, options, FX patterns, weight
cache and report()): GEMMs against parameters run W8A8 on the int8 tensor cores (xdna::linear,
xdna::linear_cat, xdna::linear_i8), 3x3 stride-1 convs run as an int8 implicit GEMM with the
requantise and ReLU in the epilogue (xdna::conv3x3), and a Qwen3-0.6B-shaped stack with its head
runs as xdna::qwen3_stack. Integer results are bit-identical to the reference's CPU route.
There is no CPU fallback: without a B200 the backend raises with the reason.
"""

import json

from . import kernels, ops  # noqa: F401  (registers the xdna:: ops)
from .backend import offload_gemms, xdna_backend
from .config import Config, set_config
from .kernels import XdnaError, XdnaUnavailable
from .runtime import XdnaResultMismatch, stats

__all__ = ["Config", "set_config", "xdna_backend", "offload_gemms", "compile", "stats", "report",
           "npu_available", "gpu_available", "XdnaError", "XdnaUnavailable", "XdnaResultMismatch"]
__version__ = "0.1.0+b200"


def _register():
    from torch._dynamo.backends.registry import _BACKENDS, register_backend

    if "xdna" not in _BACKENDS:
        register_backend(xdna_backend, name="xdna")


_register()


def compile(model, **options):
    """torch.compile(model, backend="xdna", options=options)."""
    import torch

    return torch.compile(model, backend="xdna", options=options or None)


def gpu_available() -> bool:
    """True when the B200 kernels can run in this process."""
    return kernels.available()


npu_available = gpu_available  # the reference's name


def report(as_json=False):
    """Where the GEMMs, convs and stacks ran (calls, seconds, GMACs), launches, checks, failures."""
    d = stats.as_dict()
    if as_json:
        return json.dumps(d, indent=1)
    lines = [f"B200 available: {d['gpu_available']}" +
             (f" ({d['device']})" if d["gpu_available"] else f" ({d['gpu_unavailable_reason']})")]
    for dev in sorted(d["calls"]):
        lines.append(f"  {dev:4s}: {d['calls'][dev]} calls, {d['gmacs'][dev]} GMAC, {d['seconds'][dev]} s (host)")
    lines.append(f"  kernel launches: {d['gpu_launches']}")
    for k, v in d["stacks"].items():
        lines.append(f"  {k}: {v} calls")
    for k, res in d["checks"]:
        lines.append(f"  check {k}: {res}")
    for what, err in d["fallbacks"]:
        lines.append(f"  failed {what}: {err}")
    return "\n".join(lines)
