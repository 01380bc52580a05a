"""Options of the xdna backend: torch.compile(..., backend="xdna", options={...}) or torch_xdna.set_config.

The field names, values and validation are those of the reference's Config (R:torch_xdna/config.py:11-81),
so existing option dictionaries keep working. On the B200 build their meaning is:

  policy       "auto" / "npu": offloadable GEMMs, convs and stacks run on the B200 kernels.
               "cpu": nothing is offloaded; the graph compiles unchanged (no int8 CPU route exists
               in this build -- there is no CPU fallback).
  fallback     what compiles the rest of the graph: "inductor" (compile_fx) or "eager".
  precision    "int8": W8A8 on the int8 tensor cores. "bf16": bf16 operands, f32 accumulation
               on the bf16 tensor cores.
  cpu_kernel   accepted for compatibility; only meaningful with policy "cpu" in the reference.
  min_rows, row_buckets, min_macs, tuned_tilings
               NPU launch-size knobs; accepted and ignored (a B200 launch has no row buckets).
  fuse         linears that read the same input (q/k/v, gate/up) run as one GEMM; bias-free convs
               take their ReLU into the requantise.
  stacks       a Qwen3-0.6B-shaped transformers stack + linear head runs as xdna::qwen3_stack.
  verify       "first": the first launch of every kernel configuration is compared with the CPU
               integers (bit for bit) or the fp32 model (stack); a mismatch raises.
               "always": every launch. "off": never.
  verbose      log rewrites.

Two options are new in this build (off by default, so the default computes exactly the reference's values):
  conv_ext     also offload the ResNet-style convs the reference has no kernel for
               (R:results/conv3x3_cascade.md:222-223): 1x1 convs (stride 1 or 2, no padding) and 3x3
               convs with stride 2 and padding 1, through the same int8 arithmetic (xdna::conv_int8).
  conv_bias_int32
               a biased conv adds its bias inside the int32 sums, before the requantise, as
               rint(bias / (sw * sx)) per image (R:results/conv3x3_cascade.md:224-225 names this as future
               work); a ReLU after the bias becomes the requantise's [0, 255] saturation. Different numerics
               from the reference's route (the bias is rounded to the sums' units and shares their shift).
"""

from dataclasses import dataclass, fields, replace

POLICIES = ("auto", "npu", "cpu")
FALLBACKS = ("inductor", "eager")
CPU_KERNELS = ("int8", "fp")
PRECISIONS = ("int8", "bf16")
VERIFY = ("first", "always", "off")


@dataclass(frozen=True)
class Config:
    policy: str = "auto"
    fallback: str = "inductor"
    precision: str = "int8"
    cpu_kernel: str = "int8"
    min_rows: int = 16
    row_buckets: tuple = (128, 256, 512, 1024)
    min_macs: int = 2_000_000
    fuse: bool = True
    stacks: bool = True
    tuned_tilings: bool = True
    verify: str = "first"
    verbose: bool = False
    conv_ext: bool = False
    conv_bias_int32: bool = False

    def __post_init__(self):
        assert self.policy in POLICIES, f"policy must be one of {POLICIES}"
        assert self.fallback in FALLBACKS, f"fallback must be one of {FALLBACKS}"
        assert self.cpu_kernel in CPU_KERNELS, f"cpu_kernel must be one of {CPU_KERNELS}"
        assert self.precision in PRECISIONS, f"precision must be one of {PRECISIONS}"
        assert self.verify in VERIFY, f"verify must be one of {VERIFY}"
        assert all(b % 128 == 0 for b in self.row_buckets), "row buckets must be multiples of 128"

    @property
    def offload(self) -> bool:
        """Whether this configuration puts work on the B200 at all."""
        return self.policy != "cpu"

    def merged(self, options=None):
        """This config with `options` applied; unknown option names are an error."""
        if not options:
            return self
        names = {f.name for f in fields(self)}
        unknown = sorted(set(options) - names)
        assert not unknown, f"unknown xdna options {unknown}; known: {sorted(names)}"
        if "row_buckets" in options:
            options = dict(options, row_buckets=tuple(sorted(options["row_buckets"])))
        return replace(self, **options)


config = Config()


def set_config(**options):
    """Process-wide defaults; the options given to one torch.compile call override them."""
    global config
    config = config.merged(options)
    return config
