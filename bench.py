"""Benchmark of the three offloaded ops on B200: W8A8 linear, int8 conv3x3 and the Qwen3 stack.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl xdna|reference] [--workload all|cfg2|...]

The default run (--workload all) prints ONE JSON line whose top level is BASELINE config 2 and whose
sub-records carry the other headline metrics, so that every driver run measures all of them:

  top level  config 2: the Qwen3-0.6B projection set at M = 8192 bf16 rows, W8A8 -- xdna::linear_cat
             q/k/v (N = 2048+1024+1024, K = 1024), xdna::linear_cat gate/up (N = 2x3072, K = 1024),
             xdna::linear down (N = 1024, K = 3072), each our quantise kernel + tcgen05 int8 GEMM with the
             dequantising epilogue. Metric int8 TOPS = 2*M*sum(N*K) per step / step time, whole job;
  m_sweep    config 2 at M = 1, 128, 512, 2048 (N = 1 only): TOPS and, for M <= 128, where streaming the
             weights from HBM bounds the step, an HBM roofline;
  conv       config 4: the 13 VGG16 conv3x3 layers (bias + ReLU, 2x2 max-pools, int8 chained) on a batch of
             32 images 3x224x224, batch sharded over ranks; the single Ci = Co = 256 conv on a 1536x64 image;
             config 3: four 256-channel convs + ReLU on 1x256x64x64, in ms (device and end to end);
  stack      config 5: 28 layers + final norm + head 151936 on 16 x 1024 token ids under a causal mask;
             sequences sharded over ranks, the head column-parallel on N > 1 GPUs (every rank's hidden
             states exchanged over NVLink inside the head GEMM's pipeline), with a per-N breakdown.

Every record: value (device time, CUDA events on the launching stream, max over ranks), roofline of its
dominant kernel against MEASURED_PEAKS.json, clocks sampled during its timed region, and (rank 0, N = 1)
cpu_baseline = the reference's CPU route (oracle/reference_cpu.py, the same torch CPU calls the reference
makes with policy="cpu") on the host cores. e2e: the same work through the public API with host buffers.

--impl reference times the reference's CPU route for the same records on rank 0 (other ranks exit) and
prints one line with "impl": "reference".
Other workloads print their own line: cfg2, square (4096^3), msweep, conv, cfg3, stack.
--kernel NAME --shape a,b,c times one kernel (the commands the ncu summaries are captured with).
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "torch-xdna_b200"))
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

D, NQ, NKV, INTER = 1024, 2048, 1024, 3072
V_HEAD = 151936
L2_FLUSH_BYTES = 256 << 20
M_SWEEP = (1, 128, 512, 2048)
CFG2_METRIC = "int8 TOPS/GPU, W8A8 linear (BASELINE config 2 Qwen3-0.6B projection set)"
CONV_METRIC = "int8 TOPS/GPU, conv3x3 (BASELINE config 4: VGG16 int8, batch 32)"
STACK_METRIC = "Qwen3-0.6B stack tokens/s (BASELINE config 5)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="xdna", choices=["xdna", "reference"])
    ap.add_argument("--workload", default="all", choices=["all", "cfg2", "square", "msweep", "conv", "cfg3", "stack"],
                    help="all: config 2 with the m_sweep, conv and stack records (default)")
    ap.add_argument("--rows", type=int, default=8192)
    ap.add_argument("--seqs", type=int, default=16, help="stack: sequences in the global batch")
    ap.add_argument("--seq-len", type=int, default=1024, help="stack: tokens per sequence")
    ap.add_argument("--layers", type=int, default=28, help="stack: decoder layers")
    ap.add_argument("--images", type=int, default=32, help="conv: images in the global batch")
    ap.add_argument("--conv-unchained", action="store_true",
                    help="conv: float tensors between convs (conv3x3_fused + torch max-pool) instead of int8 codes")
    ap.add_argument("--head", default="column", choices=["column", "column-direct", "column-nccl", "dp"],
                    help="stack on N > 1 GPUs: head column-parallel with the all-gather pipelined into its GEMMs "
                         "(default: peer blocks copied over NVLink once, overlapping the GEMM), read by the GEMM's "
                         "TMA straight from peer memory, after an NCCL all-gather; or data-parallel with the sequences")
    ap.add_argument("--kernel", default=None,
                    choices=["gemm_i8", "quant_rows", "conv3x3", "conv3x3_chain", "conv_quant_codes", "attention",
                             "gemm_bf16", "gemm_bf16_qkv"],
                    help="time one kernel on --shape instead of a workload (profiling)")
    ap.add_argument("--shape", default="8192,6144,1024", help="--kernel shape, comma-separated")
    return ap.parse_args()


# ---------------------------------------------------------------- distributed plumbing
def dist_init(n):
    if n <= 1 and "RANK" not in os.environ:
        return 0, 1
    import datetime

    import torch.distributed as dist

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    return rank, world


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(v, world):
    if world == 1:
        return v
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def peaks():
    """(int8 TOPS, HBM GB/s, bf16 burst TFLOP/s, bf16 sustained TFLOP/s, source)."""
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return (2 * float(d["bf16_tflops"]), float(d["hbm_gbs"]), float(d["bf16_tflops"]),
                float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured (MEASURED_PEAKS.json)")
    return 2 * 1590.0, 6650.0, 1590.0, 1400.0, "fallback (6.65 TB/s, 1.59 PFLOP/s burst, 1.4 sustained)"


INT8_PEAK_NOTE = "int8 peak = 2 x the measured dense bf16 cuBLAS burst (B200's dense int8 rate is twice its bf16 rate)"


# DRAM bytes of one launch of the chained conv1_2 (32 images, 64 -> 64, 224 x 224), from an ncu capture of
# `bench.py --kernel conv3x3_chain --shape 32,64,224` (input in image pairs): reads 113.36 MB + writes 57.53 MB
# (the rest of the codes is still in L2 when the kernel ends)
CONV_CHAIN_DRAM_BYTES_32 = 113_359_360 + 57_533_952


def roof(bound, kernel, achieved, peak, unit, per_launch_ms, **extra):
    r = {"bound": bound, "kernel": kernel, "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": unit,
         "frac": round(achieved / peak, 4), "per_launch_ms": round(per_launch_ms, 4)}
    r.update(extra)
    return r


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples (every 20 ms) of this GPU's clocks and throttle reasons while running."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index, self.rows, self.proc = index, [], None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "20"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 8:
                self.rows.append(parts)

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        def num(v):
            try:
                return float(v)
            except ValueError:
                return None

        sm = [num(r[0]) for r in self.rows if num(r[0])]
        mx = [num(r[1]) for r in self.rows if num(r[1])]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in self.rows for n, v in zip(names, r[4:8]) if v.strip().lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


def time_graph(step, steps, world, dev, flush=None):
    """Capture one call of step() in a CUDA graph, replay it `steps` times between CUDA events on the current
    stream (a write of `flush` outside the events before each replay when given), with clocks sampled
    meanwhile. Returns (total seconds, max over ranks; per-step ms list; clocks summary)."""
    stream = torch.cuda.current_stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    graph.replay()
    barrier(world)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    with ClockSampler(dev.index) as clocks:
        barrier(world)
        for i in range(steps):
            if flush is not None:
                flush.fill_(i & 0xFF)
            starts[i].record(stream)
            graph.replay()
            ends[i].record(stream)
        barrier(world)
    ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    del graph
    return max_over_ranks(sum(ms) / 1e3, world), ms, clocks.summary()


def event_ms(fn, reps, flush=None, warm=2):
    """Median CUDA-event duration of fn() on the current stream (L2 flushed before each call when given)."""
    stream = torch.cuda.current_stream()
    for _ in range(warm):
        fn()
    ms = []
    for _ in range(reps):
        if flush is not None:
            flush.fill_(1)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        fn()
        e.record(stream)
        e.synchronize()
        ms.append(s.elapsed_time(e))
    return statistics.median(ms)


# ================================================================ BASELINE config 2: the W8A8 projection set
class ProjectionSet(torch.nn.Module):
    """The projections of one Qwen3-0.6B layer: q/k/v and gate/up share an input, down reads the MLP act."""

    def __init__(self):
        super().__init__()
        self.q = torch.nn.Linear(D, NQ, bias=False)
        self.k = torch.nn.Linear(D, NKV, bias=False)
        self.v = torch.nn.Linear(D, NKV, bias=False)
        self.gate = torch.nn.Linear(D, INTER, bias=False)
        self.up = torch.nn.Linear(D, INTER, bias=False)
        self.down = torch.nn.Linear(INTER, D, bias=False)

    def forward(self, x_attn, x_mlp, act):
        return (self.q(x_attn), self.k(x_attn), self.v(x_attn), self.gate(x_mlp), self.up(x_mlp),
                self.down(act))


def gemm_shapes(workload, rows):
    if workload == "square":
        return [(4096, 4096, 4096)]
    return [(rows, NQ + 2 * NKV, D), (rows, 2 * INTER, D), (rows, D, INTER)]


def make_model(dev):
    g = torch.Generator().manual_seed(0)
    m = ProjectionSet()
    for p in m.parameters():
        p.data = (torch.randn(p.shape, generator=g) * 0.02)
    return m.to(dev, torch.bfloat16).eval()


def cfg2_config(rows):
    return {"workload": f"cfg2 Qwen3-0.6B projection set, W8A8, M={rows} rows bf16: linear_cat qkv (N=4096,K=1024) "
                        f"+ linear_cat gate/up (N=6144,K=1024) + linear down (N=1024,K=3072)",
            "global_batch": rows, "parallelism": "replicas", "l2": "flushed between steps (256 MiB write)"}


# The DRAM and L2 -> SM bytes of one gemm_i8 launch per shape (bf16 out), from an earlier ncu capture of
# `bench.py --kernel gemm_i8 --shape M,N,K` (dram__bytes_read.sum + dram__bytes_write.sum;
# lts__t_sectors_srcunit_tex_op_read.sum x 32). Not measured by this run: DRAM writes still in L2 when the
# kernel ends are not counted in its DRAM bytes, so the L2 -> SM bytes show the on-chip re-reads instead.
PAST_CAPTURE = {(8192, 4096, 1024): (26222336, None), (8192, 6144, 1024): (61992960, 407.6e6),
                (8192, 1024, 3072): (28405248, None), (4096, 4096, 4096): (36336640, None)}


def gemm_roofline(shapes, dev, reps, flush):
    """The GEMM kernel alone: algorithmic int8 ops per launch / its CUDA-event duration, summed over the
    shapes (inputs pre-quantised, L2 flushed before every launch)."""
    from torch_xdna import kernels

    total_ms, total_ops = 0.0, 0
    for (m, n, k) in shapes:
        xq = torch.randint(-127, 128, (m, k), dtype=torch.int8, device=dev)
        wq = torch.randint(-127, 128, (n, k), dtype=torch.int8, device=dev)
        sx, sw = torch.rand(m, device=dev) * 0.01, torch.rand(n, device=dev) * 0.01
        y = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
        total_ms += event_ms(lambda: kernels.gemm_i8(xq, wq, k, y, sx, sw), max(5, reps), flush, warm=3)
        total_ops += 2 * m * n * k
    peak = peaks()[0]
    caps = [PAST_CAPTURE.get(tuple(s)) for s in shapes]
    traffic = round(sum(c[0] for c in caps) / len(caps)) if all(caps) else None
    return roof("tensor", "umma_gemm_kernel (gemm_i8, dequantising epilogue, bf16 out)",
                total_ops / (total_ms / 1e3) / 1e12, peak, "TOPS", total_ms / len(shapes),
                peak_source=INT8_PEAK_NOTE, traffic=traffic,
                traffic_source="earlier ncu capture of the same shapes (dram__bytes_read.sum + dram__bytes_write."
                               "sum per launch, averaged over the shapes), not measured by this run",
                l2_to_sm_bytes={f"{m}x{n}x{k}": c[1] for (m, n, k), c in zip(shapes, caps) if c and c[1]} or None)


def cfg2_records(args, rank, world, dev, flush):
    """Config 2 at args.rows (the top level) and its square 4096^3 case."""
    import torch_xdna
    from torch_xdna import kernels

    cid = torch_xdna.ops.config_id(torch_xdna.Config(verify="first", fallback="eager"))
    model = make_model(dev)
    R = args.rows
    square = args.workload == "square"
    g = torch.Generator(device=dev).manual_seed(0)
    if square:
        x = torch.randn(4096, 4096, device=dev, generator=g).to(torch.bfloat16)
        w_sq = (torch.randn(4096, 4096, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    else:
        x = torch.randn(R, D, device=dev, generator=g).to(torch.bfloat16)        # attention-norm output
    x2 = torch.randn(R, D, device=dev, generator=g).to(torch.bfloat16)           # MLP-norm output
    act = torch.randn(R, INTER, device=dev, generator=g).to(torch.bfloat16)      # silu(gate) * up
    shapes = gemm_shapes(args.workload, R)
    work = sum(2 * m * n * k for m, n, k in shapes)
    qkv = [model.q.weight, model.k.weight, model.v.weight]
    gu = [model.gate.weight, model.up.weight]

    def step():
        if square:
            return [torch.ops.xdna.linear(x, w_sq, None, False, cid)]
        return [torch.ops.xdna.linear_cat(x, qkv, [None] * 3, cid), torch.ops.xdna.linear_cat(x2, gu, [None] * 2, cid),
                torch.ops.xdna.linear(act, model.down.weight, None, False, cid)]

    with torch.no_grad():
        for _ in range(max(args.warmup, 3)):   # includes each kernel configuration's first-call verify
            step()
        torch.cuda.synchronize()
        torch_xdna.stats.reset()
        total_s, _, clocks = time_graph(step, args.steps, world, dev, flush)
        per_step = torch_xdna.stats.launches
    rec = {"value": round(world * work * args.steps / total_s / 1e12, 2), "unit": "TOPS",
           "ms_per_step": round(total_s * 1e3 / args.steps, 4), "gpu_launches": per_step * args.steps,
           "roofline": gemm_roofline(shapes, dev, args.steps, flush), "clocks": clocks}
    if not square:
        rec["roofline_square_4096"] = gemm_roofline([(4096, 4096, 4096)], dev, args.steps, flush)
        rec["e2e"] = cfg2_e2e(args, model, dev, world, work)
    if kernels.take_device_error() != (0, 0):
        raise SystemExit("a kernel recorded a device-side timeout")
    return rec


def cfg2_e2e(args, model, dev, world, work):
    """The step through torch.compile(backend="xdna"), fed from and drained to pinned host memory as a
    serving loop would: every step copies its three inputs host -> device and its six outputs device ->
    host, on their own streams (the copy engines work in both directions at once), double-buffered so
    that step i+1's inputs, step i's GEMMs and step i-1's outputs overlap; events order each step's
    copy-in, compute and copy-out. The timed region covers every step's copies."""
    import torch_xdna  # noqa: F401  (registers the backend)

    torch._dynamo.reset()
    comp = torch.compile(model, backend="xdna", options={"fallback": "eager", "verify": "off"})
    R = args.rows
    outs_n = [NQ, NKV, NKV, INTER, INTER, D]
    ins_n = [D, D, INTER]
    hin = [[torch.randn(R, n).to(torch.bfloat16).pin_memory() for n in ins_n] for _ in range(2)]
    hout = [[torch.empty(R, n, dtype=torch.bfloat16).pin_memory() for n in outs_n] for _ in range(2)]
    din = [[torch.empty(R, n, dtype=torch.bfloat16, device=dev) for n in ins_n] for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    s_comp = torch.cuda.current_stream()
    ev_in = [torch.cuda.Event() for _ in range(2)]     # inputs of buffer b on the device
    ev_used = [torch.cuda.Event() for _ in range(2)]   # compute done reading inputs of buffer b
    ev_comp = [torch.cuda.Event() for _ in range(2)]   # outputs of buffer b computed
    ev_out = [torch.cuda.Event() for _ in range(2)]    # outputs of buffer b on the host
    for b in range(2):                                  # nothing outstanding yet
        ev_used[b].record(s_comp)
        ev_out[b].record(s_comp)

    def step(i):
        b = i & 1
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_used[b])
            for d, h in zip(din[b], hin[b]):
                d.copy_(h, non_blocking=True)
            ev_in[b].record(s_in)
        s_comp.wait_event(ev_in[b])
        s_comp.wait_event(ev_out[b])                   # the host buffers of step i-2 were drained
        ys = comp(*din[b])
        ev_used[b].record(s_comp)
        ev_comp[b].record(s_comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_comp[b])
            for h, y in zip(hout[b], ys):
                y.record_stream(s_out)
                h.copy_(y, non_blocking=True)
            ev_out[b].record(s_out)

    with torch.no_grad():
        for i in range(4):
            step(i)
        torch.cuda.synchronize()
        barrier(world)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        steps = max(4, args.steps // 2)
        s.record(s_comp)
        s_in.wait_event(s)                              # the first copy-in starts inside the timed region
        for i in range(steps):
            step(i)
        s_comp.wait_stream(s_out)                      # the last outputs are on the host
        e.record(s_comp)
        e.synchronize()
        barrier(world)
    sec = max_over_ranks(s.elapsed_time(e) / 1e3, world)
    torch._dynamo.reset()
    return {"value": round(world * work * steps / sec / 1e12, 2), "unit": "TOPS",
            "h2d_bytes_per_step": sum(t.numel() for t in hin[0]) * 2,
            "d2h_bytes_per_step": sum(t.numel() for t in hout[0]) * 2,
            "api": "torch.compile(backend='xdna', fallback='eager')",
            "pipeline": "copy-in / compute / copy-out streams, double-buffered pinned host and device buffers"}


def gemm_hbm_bytes(m, n, k):
    """Algorithmic HBM bytes of one dequantising int8 GEMM launch: int8 weights and activations read once,
    bf16 output written once, the row and column scales."""
    return n * k + m * k + 2 * m * n + 4 * (m + n)


def msweep_record(args, dev, flush):
    """Config 2's row sweep: the projection set (quantise + GEMM per op, as the top level) at M = 1, 128,
    512, 2048. M <= 128: the step streams 13.6 MB of int8 weights and little else, so its roofline is HBM
    (algorithmic GEMM bytes / GEMM time against the measured copy bandwidth); larger M: the int8 peak."""
    import torch_xdna
    from torch_xdna import kernels

    cid = torch_xdna.ops.config_id(torch_xdna.Config(verify="first", fallback="eager"))
    model = make_model(dev)
    qkv = [model.q.weight, model.k.weight, model.v.weight]
    gu = [model.gate.weight, model.up.weight]
    int8_peak, hbm, _, _, src = peaks()
    out = {}
    g = torch.Generator(device=dev).manual_seed(2)
    for M in M_SWEEP:
        x = torch.randn(M, D, device=dev, generator=g).to(torch.bfloat16)
        x2 = torch.randn(M, D, device=dev, generator=g).to(torch.bfloat16)
        act = torch.randn(M, INTER, device=dev, generator=g).to(torch.bfloat16)

        def step():
            return [torch.ops.xdna.linear_cat(x, qkv, [None] * 3, cid),
                    torch.ops.xdna.linear_cat(x2, gu, [None] * 2, cid),
                    torch.ops.xdna.linear(act, model.down.weight, None, False, cid)]

        shapes = gemm_shapes("cfg2", M)
        work = sum(2 * m * n * k for m, n, k in shapes)
        with torch.no_grad():
            for _ in range(3):
                step()
            torch_xdna.stats.reset()
            total_s, _, clocks = time_graph(step, args.steps, 1, dev, flush)
            launches = torch_xdna.stats.launches
        # the GEMM kernels alone, L2 flushed before each (weights from HBM)
        gem_ms, gem_bytes = 0.0, 0
        for (m, n, k) in shapes:
            xq = torch.randint(-127, 128, (m, k), dtype=torch.int8, device=dev)
            wq = torch.randint(-127, 128, (n, k), dtype=torch.int8, device=dev)
            sx, sw = torch.rand(m, device=dev) * 0.01, torch.rand(n, device=dev) * 0.01
            y = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
            gem_ms += event_ms(lambda: kernels.gemm_i8(xq, wq, k, y, sx, sw), max(5, args.steps), flush, warm=3)
            gem_bytes += gemm_hbm_bytes(m, n, k)
        step_ms = total_s * 1e3 / args.steps
        rec = {"value": round(work * args.steps / total_s / 1e12, 3), "unit": "TOPS", "ms_per_step": round(step_ms, 4),
               "gpu_launches": launches * args.steps, "clocks": clocks}
        if M <= 128:
            rec["roofline"] = roof("hbm", "umma_gemm_kernel (gemm_i8, the three GEMMs of the set)",
                                   gem_bytes / (gem_ms / 1e3) / 1e9, hbm, "GB/s", gem_ms / 3,
                                   peak_source=src, bytes_per_step=gem_bytes,
                                   step_gbs=round(gem_bytes / (step_ms / 1e3) / 1e9, 1))
        else:
            rec["roofline"] = roof("tensor", "umma_gemm_kernel (gemm_i8, the three GEMMs of the set)",
                                   work / (gem_ms / 1e3) / 1e12, int8_peak, "TOPS", gem_ms / 3, peak_source=INT8_PEAK_NOTE)
        out[str(M)] = rec
    if kernels.take_device_error() != (0, 0):
        raise SystemExit("a kernel recorded a device-side timeout")
    return out


# ================================================================ BASELINE configs 3 and 4: int8 convs
VGG16 = [64, 64, "M", 128, 128, "M", 256, 256, 256, "M", 512, 512, 512, "M", 512, 512, 512]


def vgg_layers(dev, seed=7):
    g = torch.Generator(device=dev).manual_seed(seed)
    layers, ci = [], 3
    for v in VGG16:
        if v == "M":
            layers.append("M")
            continue
        w = torch.randn(v, ci, 3, 3, device=dev, generator=g) * (2.0 / (ci * 9)) ** 0.5   # Kaiming normal (ReLU)
        b = torch.randn(v, device=dev, generator=g) * 0.01
        layers.append((w, b))
        ci = v
    return layers


def vgg_macs(batch, hw=224):
    macs, ci, h = 0, 3, hw
    for v in VGG16:
        if v == "M":
            h //= 2
            continue
        macs += batch * h * h * ci * v * 9
        ci = v
    return macs


def cfg3_weights(dev, seed=3):
    g = torch.Generator(device=dev).manual_seed(seed)
    return [torch.randn(256, 256, 3, 3, device=dev, generator=g) * (2.0 / (256 * 9)) ** 0.5 for _ in range(4)]


CFG3_OPS = 4 * 2 * 64 * 64 * 256 * 256 * 9       # 19.3 G int8 ops


class Cfg3Net(torch.nn.Module):
    """BASELINE config 3 (R:examples/conv_xdna.py:20-82 shapes): four bias-free 3x3 convs 256 -> 256, each
    followed by ReLU."""

    def __init__(self, ws):
        super().__init__()
        self.convs = torch.nn.ModuleList(torch.nn.Conv2d(256, 256, 3, padding=1, bias=False) for _ in ws)
        for c, w in zip(self.convs, ws):
            c.weight.data = w

    def forward(self, x):
        for c in self.convs:
            x = torch.relu(c(x))
        return x


def single_conv_roofline(dev, peak, flush):
    """The conv kernel on BASELINE config 4's single Ci = Co = 256 conv of one 1536 x 64 image (dequantise
    epilogue with bias and ReLU), event-timed per launch with L2 flushed before each."""
    from torch_xdna import conv as xconv
    from torch_xdna import kernels

    g = torch.Generator(device=dev).manual_seed(7)
    w = torch.nn.Parameter(torch.randn(256, 256, 3, 3, device=dev, generator=g) * (2.0 / (256 * 9)) ** 0.5)
    b = torch.randn(256, device=dev, generator=g) * 0.01
    lay = xconv.ConvLayer(w, 1536, 64, False)
    xp = torch.randint(-127, 128, (1, 1538, 66, lay.cp), dtype=torch.int8, device=dev, generator=g)
    xp[:, 0].zero_(), xp[:, -1].zero_(), xp[:, :, 0].zero_(), xp[:, :, -1].zero_()
    lay.calibrate(xp)
    sx = torch.rand(1, device=dev)
    yo = torch.empty(1, 256, 1536, 64, device=dev, memory_format=torch.channels_last)
    ms = event_ms(lambda: kernels.conv3x3(xp, lay.wp, 1, 256, 256, 1536, 64, kernels.CONV_DEQUANT, shift=lay.shift,
                                          scale=lay.scale, sx=sx, bias=b, relu=kernels.RELU_AFTER_BIAS, out=yo),
                  6, flush)
    ops = 2 * 1536 * 64 * 256 * 256 * 9
    return roof("tensor", "umma_gemm_kernel LOAD_CONV (conv 256->256, 1 x 1536 x 64, bias + ReLU)",
                ops / ms / 1e9, peak, "TOPS", ms, peak_source=INT8_PEAK_NOTE)


def conv_record(args, rank, world, dev, flush):
    """Config 4: one step = the 13 int8 conv3x3 layers of VGG16 (bias + ReLU, 2x2 max-pool between blocks) on
    this rank's share of a batch of 32 images 3x224x224 (batch sharded over ranks, strong scaling), as the
    backend compiles it: xdna::conv3x3_chain, the activations between convs kept as int8 codes (the next
    conv's quantise rebuilds the float values and takes the 2x2 max-pool on the codes), the last conv's
    output dequantised with bias and ReLU in its epilogue and max-pooled by torch. --conv-unchained runs
    xdna::conv3x3_fused per conv with torch's max-pool between (same values). The requantise shift of every
    layer comes from global image 0 (rank 0), broadcast to the other ranks."""
    import torch_xdna
    from torch_xdna import conv as xconv
    from torch_xdna import kernels, parallel
    from torch_xdna.conv import IN_CODES, IN_CODES_POOL, IN_FLOAT

    if world > 1:
        parallel.enable_data_parallel()
    N_all = args.images
    assert N_all % world == 0, "images must divide over the ranks"
    N = N_all // world
    layers = vgg_layers(dev)
    params = [("M" if l == "M" else (torch.nn.Parameter(l[0]), l[1])) for l in layers]
    cid = torch_xdna.ops.config_id(torch_xdna.Config(verify="first"))
    g = torch.Generator(device=dev).manual_seed(99)
    x_all = torch.randn(N_all, 3, 224, 224, device=dev, generator=g)
    x = x_all[rank * N:(rank + 1) * N].contiguous()
    del x_all
    n_convs = sum(p != "M" for p in params)

    def step_unchained():
        h = x
        for p in params:
            if p == "M":
                h = torch.nn.functional.max_pool2d(h, 2)
            else:
                h = torch.ops.xdna.conv3x3_fused(h, p[0], p[1], False, cid, True)  # ReLU after the bias
        return h

    def step_chained():
        h, meta, k, pool = x, None, 0, False
        for i, p in enumerate(params):
            if p == "M":
                if k == n_convs:   # after the last conv: a float tensor
                    h = torch.nn.functional.max_pool2d(h, 2)
                else:
                    pool = True    # taken into the next conv's quantise
                continue
            mode = IN_FLOAT if k == 0 else (IN_CODES_POOL if pool else IN_CODES)
            k += 1
            out_pool = k < n_convs and i + 1 < len(params) and params[i + 1] == "M"
            h, meta = torch.ops.xdna.conv3x3_chain(h, meta, p[0], p[1], False, cid, True, mode, k > 1, k < n_convs,
                                                   out_pool)
            pool = False
        return h

    step = step_unchained if args.conv_unchained else step_chained
    with torch.no_grad():
        for _ in range(max(args.warmup, 3)):   # includes each layer's calibration and first-call verify
            step()
        torch.cuda.synchronize()
        torch_xdna.stats.reset()
        # replayed from a CUDA graph: with a half or quarter batch per GPU, per-op host work would pace the step
        total_s, _, clocks = time_graph(step, args.steps, world, dev)   # 400 MB of activations exceed L2
        per_step = torch_xdna.stats.launches
    if world > 1:
        parallel.disable_data_parallel()
    int8_peak = peaks()[0]
    # roofline: the conv kernel of the largest-work layer (conv 64->64 at 224x224, this rank's images) as the
    # chain runs it: int8 codes out, the next layer's per-image maxima over the 2x2 pool's region in the epilogue
    lay = xconv._layer(params[1][0], 224, 224, False)
    xp = torch.randint(-127, 128, (N, 226, 226, lay.cp), dtype=torch.int8, device=dev)
    xp2 = torch.randint(-127, 128, (N // 2, 226, 226, 128), dtype=torch.int8, device=dev) if N % 2 == 0 else None
    sx = torch.rand(N, device=dev) + 0.5
    bias = params[1][1].detach().float().contiguous()
    qo = torch.empty(N, 224, 224, 64, dtype=torch.int8, device=dev)
    amax = torch.empty(N, dtype=torch.int32, device=dev)
    # as the chain runs it: the input in image pairs when the rank holds an even number of images
    chain_mode = (kernels.CONV_Q_NHWC | kernels.CONV_NEXT_AMAX | kernels.CONV_NEXT_RELU | kernels.CONV_NEXT_POOL
                  | (kernels.CONV_PAIRS if xp2 is not None else 0))
    ms = event_ms(lambda: kernels.conv3x3(xp2 if xp2 is not None else xp, lay.wp, N, 64, 64, 224, 224,
                                          chain_mode | lay.mode_flag,
                                          shift=lay.shift, scale=lay.scale, sx=sx, bias=bias, out=qo, acc_max=amax), 5)
    yo = torch.empty(N, 64, 224, 224, device=dev, memory_format=torch.channels_last)
    ms_f32 = event_ms(lambda: kernels.conv3x3(xp, lay.wp, N, 64, 64, 224, 224, kernels.CONV_DEQUANT | lay.mode_flag,
                                              shift=lay.shift, scale=lay.scale, sx=sx, bias=params[1][1],
                                              relu=kernels.RELU_AFTER_BIAS, out=yo), 5)
    del xp, xp2, yo, qo
    conv_ops = 2 * N * 224 * 224 * 64 * 64 * 9
    rec = {"metric": CONV_METRIC, "value": round(2 * vgg_macs(N_all) * args.steps / total_s / 1e12, 2), "unit": "TOPS",
           "ms_per_step": round(total_s * 1e3 / args.steps, 3), "scaling": "strong", "dtype": "int8",
           "config": {"workload": "cfg4 VGG16 conv3x3 stack int8, 32x3x224x224, bias + ReLU, 2x2 max-pool",
                      "between_convs": "fp32 tensors, torch max-pool" if args.conv_unchained
                      else "int8 codes (pool on the codes)", "global_batch": N_all,
                      "parallelism": f"dp{world} (images)", "l2": "activations exceed L2"},
           "gpu_launches": per_step * args.steps,
           "roofline": roof("tensor", "umma_gemm_kernel conv (conv 64->64 224x224 as chained: image pairs in, int8 "
                            "codes out, next layer's pooled per-image maxima in the epilogue)", conv_ops / ms / 1e9,
                            int8_peak, "TOPS",
                            ms, peak_source=INT8_PEAK_NOTE, traffic=round(CONV_CHAIN_DRAM_BYTES_32 * N / 32),
                            traffic_source="ncu capture of bench.py --kernel conv3x3_chain --shape 32,64,224 "
                                           "(dram__bytes_read.sum + dram__bytes_write.sum, scaled to this rank's "
                                           "images), not measured by this run",
                            algorithmic_bytes=N * (226 * 226 * 64 + 224 * 224 * 64)),
           "roofline_dequant_f32": roof("tensor", "umma_gemm_kernel conv (conv 64->64 224x224, f32 out, dequantise "
                                        "epilogue, bias + ReLU)", conv_ops / ms_f32 / 1e9, int8_peak, "TOPS", ms_f32,
                                        peak_source=INT8_PEAK_NOTE, traffic=None),
           "step_frac": round(2 * vgg_macs(N_all) * args.steps / total_s / 1e12 / world / int8_peak, 4),
           "clocks": clocks}
    rec["single_conv_256x1536x64"] = single_conv_roofline(dev, int8_peak, flush)
    rec["cfg3"] = cfg3_record(args, rank, world, dev)
    if kernels.take_device_error() != (0, 0):
        raise SystemExit("a kernel recorded a device-side timeout")
    return rec


def cfg3_strips(args, rank, world, dev, ws, x):
    """Config 3 on N > 1 GPUs: the image split into strips of rows (64 / N per rank, parallel.strip_rows), each
    conv combining the image's max and the calibration max over the ranks and exchanging 1-row halos
    (conv.conv3x3_strip). Checked once, bit for bit, against the whole image run through the same four convs
    on this GPU alone."""
    import torch_xdna
    from torch_xdna import conv as xconv
    from torch_xdna import parallel

    cfg = torch_xdna.Config(verify="off")
    r0, r1 = parallel.strip_rows(64, rank, world)
    xl = x[:, :, r0:r1].contiguous()
    params = [torch.nn.Parameter(w) for w in ws]

    def step():
        h = xl
        for p in params:
            h = xconv.conv3x3_strip(cfg, h, p, None, True)
        return h

    with torch.no_grad():
        y = step()
        whole = x
        for w in ws:   # one GPU, the whole image (fresh weights: their own layers and shifts)
            whole = xconv.conv3x3_fused(cfg, whole, torch.nn.Parameter(w.clone()), None, True)
        exact = bool(torch.equal(y, whole[:, :, r0:r1]))
        all_exact = max_over_ranks(0.0 if exact else 1.0, world) == 0.0
        if not all_exact:
            raise SystemExit(f"rank {rank}: config 3 image strips differ from the whole image on one GPU")
        ms = max_over_ranks(event_ms(step, max(5, args.steps), warm=2), world)
    return {"ms_per_step": round(ms, 4), "tops": round(CFG3_OPS / ms / 1e9, 1),
            "parallelism": f"image strips: {world} x {64 // world} rows, 1-row halos over NCCL, image max and "
                           f"calibration max all-reduced", "rows_per_rank": r1 - r0,
            "strips_bit_exact_vs_one_gpu": all_exact,
            "reference_published_ms": {"inductor_fp32_cpu": 5.72, "xdna_npu_end_to_end": 1.68, "npu_launches": 0.80}}


def cfg3_record(args, rank, world, dev):
    """Config 3: four bias-free 256-channel convs + ReLU on one 1x256x64x64 image, compiled by the backend
    (which chains them on int8 codes). ms_per_step: device time of the compiled call replayed from a CUDA
    graph; e2e_ms: the compiled call with the input copied from pinned host memory and the output copied
    back, per call. On N > 1 GPUs the image is split into strips of rows over the ranks (cfg3_strips)."""
    import torch_xdna

    ws = cfg3_weights(dev)
    g = torch.Generator(device=dev).manual_seed(11)
    x = torch.randn(1, 256, 64, 64, device=dev, generator=g)
    if world > 1:
        return cfg3_strips(args, rank, world, dev, ws, x)
    net = Cfg3Net(ws).to(dev).eval()
    torch._dynamo.reset()
    comp = torch.compile(net, backend="xdna", options={"fallback": "eager", "verify": "first"})
    with torch.no_grad():
        for _ in range(max(args.warmup, 3)):
            comp(x)
        torch.cuda.synchronize()
        torch_xdna.stats.reset()
        total_s, _, clocks = time_graph(lambda: comp(x), args.steps, world, dev)
        per_call = torch_xdna.stats.launches
        hx = x.cpu().pin_memory()
        hy = torch.empty(1, 256, 64, 64, pin_memory=True)
        dx = torch.empty_like(x)
        stream = torch.cuda.current_stream()
        reps = max(5, args.steps)
        barrier(world)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        for _ in range(reps):
            dx.copy_(hx, non_blocking=True)
            hy.copy_(comp(dx), non_blocking=True)
        e.record(stream)
        e.synchronize()
        e2e_ms = max_over_ranks(s.elapsed_time(e) / reps, world)
    torch._dynamo.reset()
    ms = total_s * 1e3 / args.steps
    return {"ms_per_step": round(ms, 4), "tops": round(CFG3_OPS / ms / 1e9, 1), "gpu_launches": per_call * args.steps,
            "e2e_ms": round(e2e_ms, 4), "e2e_h2d_bytes": hx.numel() * 4, "e2e_d2h_bytes": hy.numel() * 4,
            "api": "torch.compile(backend='xdna') of 4 x (conv3x3 256->256 + ReLU)", "clocks": clocks,
            "parallelism": "one GPU",
            "reference_published_ms": {"inductor_fp32_cpu": 5.72, "xdna_npu_end_to_end": 1.68, "npu_launches": 0.80}}


# ================================================================ BASELINE config 5: the Qwen3 stack
def stack_flops(B, L, layers, vocab):
    """Algorithmic FLOPs of one step: the projections and head per token, causal attention (QK^T and PV over
    the keys each query sees)."""
    per_token = 2 * (layers * (D * 4096 + 2048 * D + D * 6144 + INTER * D) + D * vocab)
    attn = layers * B * 2 * 2 * 16 * 128 * (L * (L + 1) // 2)
    return B * L * per_token + attn


def stack_record(args, rank, world, dev):
    """Config 5: one step = embed the token ids of this rank's sequences and run xdna_qwen3_stack (28 layers,
    final norm, head over 151936) under a causal mask; the global batch is fixed (strong scaling). The layers
    are data-parallel over sequences (independent: no collective). The head, on more than one GPU, is
    column-parallel by default: each rank computes its 151936 / N vocabulary columns for every token of every
    rank, reading the other ranks' final hidden states over NVLink inside the head GEMM's pipeline."""
    from torch_xdna import kernels, parallel

    B_all, L, NL = args.seqs, args.seq_len, args.layers
    assert B_all % world == 0, "sequences must divide over the ranks"
    B = B_all // world
    g = torch.Generator(device=dev).manual_seed(1234)

    def w(*shape):
        return (torch.randn(*shape, device=dev, generator=g) * 0.02).to(torch.bfloat16)

    table = (kernels.Qwen3Layer * NL)()
    keep = []
    for i in range(NL):
        qkv, o, gu, down = w(4096, D), w(D, 2048), w(2 * INTER, D), w(D, INTER)
        norms = [torch.ones(D, device=dev), torch.ones(D, device=dev), torch.ones(128, device=dev),
                 torch.ones(128, device=dev)]
        keep += [qkv, o, gu, down] + norms
        table[i] = kernels.Qwen3Layer(qkv.data_ptr(), o.data_ptr(), gu.data_ptr(), down.data_ptr(),
                                      *[t.data_ptr() for t in norms])
    final = torch.ones(D, device=dev)
    head, embed = w(V_HEAD, D), w(V_HEAD, D)
    column = world > 1 and args.head in ("column", "column-direct", "column-nccl")
    fused = column and args.head != "column-nccl"  # the all-gather inside the head's GEMM pipeline
    n_cols = V_HEAD // world if column else V_HEAD       # 151936 = 2^7 x 1187: divides by 2, 4 and 8
    if column:
        head = head[rank * n_cols:(rank + 1) * n_cols].contiguous()
    inv = 1.0 / (1e6 ** (torch.arange(0, 128, 2, dtype=torch.float32, device=dev) / 128))
    f = torch.arange(L, dtype=torch.float32, device=dev)[:, None] * inv[None, :]
    cos, sin = kernels.rope_layout(f.cos()), kernels.rope_layout(f.sin())
    ids_all = torch.randint(0, V_HEAD, (B_all * L,), device=dev, generator=g)
    ids = ids_all[rank * B * L:(rank + 1) * B * L].contiguous()
    x = torch.empty(B * L, D, device=dev)
    out = torch.empty(B_all * L if column else B * L, n_cols, dtype=torch.bfloat16, device=dev)
    ws = torch.empty(kernels.qwen3_stack_workspace(B, L), dtype=torch.uint8, device=dev)
    hidden = ws[:B * L * D * 2].view(torch.bfloat16).view(B * L, D)   # the final-normed states (workspace head)
    h_all = torch.empty(B_all * L, D, dtype=torch.bfloat16, device=dev) if column and not fused else None
    rg = parallel.RowGather(B * L, D, dev, mode="direct" if args.head == "column-direct" else "pipelined") \
        if fused else None
    launches_per_step = 1 + 7 * NL + 2 + ((world - 1 if args.head == "column" else 0) if column else 0)

    def layers_only(ids_dev):
        kernels.embed(ids_dev, embed, x)
        kernels.qwen3_stack(table, final, head, None, cos, sin, 1e-6, x, B, L, kernels.MASK_CAUSAL, None, None,
                            None, ws)

    def head_part():
        if fused:
            rg.local.copy_(hidden)
            rg.gemm(head, out)
        else:
            parallel.gather_rows(hidden, h_all)
            kernels.gemm_bf16(h_all, head, kernels.GEMM_F32ACC, out=out)

    def step(ids_dev):
        if column:
            layers_only(ids_dev)
            head_part()
        else:
            kernels.embed(ids_dev, embed, x)
            kernels.qwen3_stack(table, final, head, None, cos, sin, 1e-6, x, B, L, kernels.MASK_CAUSAL, None, None,
                                out, ws)

    stream = torch.cuda.current_stream()
    for _ in range(max(args.warmup, 3)):
        step(ids)
    head_check = None
    if column:   # once, untimed: the pipelined head's logits against the 1-GPU head's for this rank's columns
        gathered = torch.empty(B_all * L, D, dtype=torch.bfloat16, device=dev)
        parallel.gather_rows(hidden, gathered)
        one_gpu = torch.empty_like(out)
        kernels.gemm_bf16(gathered, head, kernels.GEMM_F32ACC, out=one_gpu)   # one GEMM over all rows
        exact = bool(torch.equal(out, one_gpu))
        rows = torch.arange(0, B_all * L, 61, device=dev)
        ref = gathered[rows].float() @ head.float().t()
        err = float((out[rows].float() - ref).abs().max() / ref.abs().max())
        head_check = {"bit_exact_vs_one_gemm": exact, "max_rel_vs_f32_sampled_rows": round(err, 5),
                      "rows_checked": B_all * L}
        if not exact and not err < 2e-2:
            raise SystemExit(f"rank {rank}: column-parallel head disagrees with the one-GEMM head (rel {err:.3g})")
        del gathered, one_gpu
    barrier(world)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(dev.index) as clocks:
        barrier(world)
        for i in range(args.steps):          # weights (1.2 GB) and activations far exceed L2
            starts[i].record(stream)
            step(ids)
            ends[i].record(stream)
        barrier(world)
    total_s = max_over_ranks(sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / 1e3, world)
    tokens = B_all * L * args.steps
    flops = stack_flops(B_all, L, NL, V_HEAD)
    _, _, bf16_burst, bf16_sust, src = peaks()
    step_tflops = flops * args.steps / total_s / 1e12

    # breakdown: the layers alone, the head GEMM alone (all rows x this rank's columns, local operands), and
    # on N > 1 the exchange alone (every peer block copied over NVLink) and the overlapped head
    reps = max(3, min(args.steps, 10))
    layers_ms = max_over_ranks(event_ms(lambda: layers_only(ids), reps, warm=1), world)
    hn = torch.randn(out.shape[0], D, device=dev).to(torch.bfloat16)
    head_gemm_ms = event_ms(lambda: kernels.gemm_bf16(hn, head, kernels.GEMM_F32ACC, out=out), 5)
    head_flops = 2 * out.shape[0] * n_cols * D
    breakdown = {"layers_ms": round(layers_ms, 3), "head_gemm_ms": round(max_over_ranks(head_gemm_ms, world), 3)}
    if column:
        breakdown["head_total_ms"] = round(max_over_ranks(event_ms(head_part, reps, warm=1), world), 3)
        if fused and rg.mode == "pipelined":
            breakdown["exchange_ms"] = round(max_over_ranks(event_ms(rg.exchange, reps, warm=1), world), 3)
            breakdown["exchange_bytes_per_rank"] = (world - 1) * B * L * D * 2
        breakdown["exchange"] = ("peer blocks copied over NVLink by a copy engine while the GEMM runs"
                                 if args.head == "column" else "the GEMM's TMA reads peer rows" if fused
                                 else "NCCL all-gather, then the GEMM")
    rec = {"metric": STACK_METRIC, "value": round(tokens / total_s, 1), "unit": "tokens/s",
           "ms_per_step": round(total_s * 1e3 / args.steps, 3), "scaling": "strong", "dtype": "bf16",
           "config": {"workload": f"cfg5 Qwen3-0.6B stack: {NL} layers, {B_all} sequences x {L} tokens, causal "
                                  f"mask, head {V_HEAD}, bf16 with f32 accumulation", "global_batch": B_all,
                      "seq_len": L, "l2": "inputs exceed L2",
                      "parallelism": (f"dp{world} sequences; head column-parallel over {world}") if column
                      else f"dp{world} (sequences)"},
           "gpu_launches": launches_per_step * args.steps,
           "roofline": roof("tensor", "the whole step (bf16 tcgen05 GEMMs + attention), algorithmic FLOPs",
                            step_tflops / world, bf16_sust, "TFLOP/s", total_s * 1e3 / args.steps,
                            peak_source=f"dense bf16 cuBLAS sustained, {src}", traffic=None,
                            flops_per_step=flops),
           "head_roofline": roof("tensor", "umma_gemm_kernel bf16 (the head GEMM, EPI_F32ACC)",
                                 head_flops / head_gemm_ms / 1e9, bf16_burst, "TFLOP/s", head_gemm_ms,
                                 peak_source=f"dense bf16 cuBLAS burst, {src}"),
           "breakdown": breakdown, "clocks": clocks.summary()}
    if head_check is not None:
        rec["head_check"] = head_check

    # e2e: token ids from pinned host memory in, every logit back to pinned host memory
    h_ids = ids.cpu().pin_memory()
    h_out = torch.empty(out.shape, dtype=torch.bfloat16, pin_memory=True)
    d_ids = torch.empty_like(ids)
    e_steps = max(2, min(5, args.steps))
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    s.record(stream)
    for _ in range(e_steps):
        d_ids.copy_(h_ids, non_blocking=True)
        step(d_ids)
        h_out.copy_(out, non_blocking=True)
    e.record(stream)
    barrier(world)
    e2e_s = max_over_ranks(s.elapsed_time(e) / 1e3, world)
    rec["e2e"] = {"value": round(B_all * L * e_steps / e2e_s, 1), "unit": "tokens/s",
                  "h2d_bytes_per_step": h_ids.numel() * 8, "d2h_bytes_per_step": h_out.numel() * 2,
                  "api": "xdna_embed + xdna_qwen3_stack C ABI (torch_xdna.kernels)"}
    if rg is not None:
        rg.close()
    if kernels.take_device_error() != (0, 0):
        raise SystemExit("a kernel recorded a device-side timeout")
    return rec


# ================================================================ CPU baselines (the reference's CPU route)
def _threads():
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return n


def cpu_cfg2(rows, budget_s=8.0, min_passes=3):
    """The reference's CPU route for config 2 (torch._int_mm + its eager quantise / dequantise,
    oracle/reference_cpu.py) at `rows` rows, all host threads; (TOPS, passes, median seconds)."""
    from oracle import reference_cpu as rc

    threads = _threads()
    g = torch.Generator().manual_seed(1)
    ops = []
    for (m, n, k) in gemm_shapes("cfg2", rows):
        w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
        w_kn, sw = rc.quant_weight(w)
        ops.append((torch.randn(m, k, generator=g).to(torch.bfloat16), w_kn, sw))
    with torch.no_grad():
        for x, w_kn, sw in ops:           # warm-up
            rc.linear_int8(x, w_kn, sw)
        times = []
        t_end = time.perf_counter() + budget_s
        while time.perf_counter() < t_end or len(times) < min_passes:
            t0 = time.perf_counter()
            for x, w_kn, sw in ops:
                rc.linear_int8(x, w_kn, sw)
            times.append(time.perf_counter() - t0)
    step = statistics.median(times)
    work = sum(2 * m * n * k for m, n, k in gemm_shapes("cfg2", rows))
    return {"value": round(work / step / 1e12, 4), "unit": "TOPS", "cores": threads, "kind": "port",
            "sample": f"the whole cfg2 projection set at {rows} rows, median of {len(times)} passes; torch._int_mm + "
                      f"eager quantise/dequantise (the reference's policy='cpu' route)"}


def cpu_stack(layers, seqs=1, seq_len=1024):
    """The reference's parity route for the stack (the fp32 eager model) restated in torch CPU ops
    (oracle/reference_cpu.py) on a bounded sample: one sequence of the config's length, all host threads."""
    from oracle import reference_cpu as rc

    threads = _threads()
    g = torch.Generator().manual_seed(5)

    def w(*s):
        return torch.randn(*s, generator=g) * 0.02

    ls = [dict(q=w(2048, D), k=w(1024, D), v=w(1024, D), o=w(D, 2048), gate=w(INTER, D), up=w(INTER, D),
               down=w(D, INTER), input_norm=torch.ones(D), post_norm=torch.ones(D), q_norm=torch.ones(128),
               k_norm=torch.ones(128)) for _ in range(layers)]
    head = w(V_HEAD, D)
    x = torch.randn(seqs, seq_len, D, generator=g)
    mask = torch.ones(seq_len, seq_len, dtype=torch.bool).tril()[None, None].expand(seqs, 1, seq_len, seq_len)
    with torch.no_grad():
        rc.qwen3_stack(ls[:1], torch.ones(D), head[:1024], None, x[:, :64], mask[:, :, :64, :64])   # warm-up
        t0 = time.perf_counter()
        rc.qwen3_stack(ls, torch.ones(D), head, None, x, mask)
        dt = time.perf_counter() - t0
    return {"value": round(seqs * seq_len / dt, 1), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{seqs} sequence x {seq_len} tokens (causal) through {layers} layers + head {V_HEAD}, fp32 "
                      f"eager torch CPU (the reference's parity model), one pass of {dt:.1f} s"}


def cpu_vgg(images=2, budget_s=6.0):
    """The reference's CPU-integer conv route (oracle/reference_cpu.py: exact fp conv of the integers) through
    the VGG16 conv stack on a bounded sample of images, all host threads."""
    from oracle import reference_cpu as rc

    threads = _threads()
    layers = [("M" if l == "M" else (rc.conv_layer(l[0].cpu(), False), l[1].cpu())) for l in vgg_layers("cpu")]
    x = torch.randn(images, 3, 224, 224, generator=torch.Generator().manual_seed(3))

    def run():
        h = x
        for l in layers:
            h = torch.nn.functional.max_pool2d(h, 2) if l == "M" else torch.relu(rc.conv3x3_int8(h, l[0], l[1]))
        return h

    with torch.no_grad():
        run()
        times = []
        t_end = time.perf_counter() + budget_s
        while time.perf_counter() < t_end or len(times) < 2:
            t0 = time.perf_counter()
            run()
            times.append(time.perf_counter() - t0)
    dt = statistics.median(times)
    return {"value": round(2 * vgg_macs(images) / dt / 1e12, 4), "unit": "TOPS", "cores": threads, "kind": "port",
            "sample": f"{images} images 3x224x224 through the 13 VGG16 convs (CPU integers: quantise, fp conv of the "
                      f"integers, requantise, dequantise), median of {len(times)} passes"}


def cpu_cfg3(budget_s=3.0):
    """Config 3 on the reference's CPU-integer route (the whole config: one image, four convs + ReLU)."""
    from oracle import reference_cpu as rc

    threads = _threads()
    layers = [rc.conv_layer(w.cpu(), True) for w in cfg3_weights("cpu")]
    x = torch.randn(1, 256, 64, 64, generator=torch.Generator().manual_seed(11))

    def run():
        h = x
        for l in layers:
            h = rc.conv3x3_int8(h, l)
        return h

    with torch.no_grad():
        run()
        times = []
        t_end = time.perf_counter() + budget_s
        while time.perf_counter() < t_end or len(times) < 3:
            t0 = time.perf_counter()
            run()
            times.append(time.perf_counter() - t0)
    dt = statistics.median(times)
    return {"value": round(dt * 1e3, 3), "unit": "ms", "cores": threads, "kind": "port",
            "sample": f"the whole config (1x256x64x64, 4 convs + ReLU) on the CPU-integer route, median of "
                      f"{len(times)} passes"}


def cpu_msweep():
    return {str(M): cpu_cfg2(M, budget_s=1.5, min_passes=3) for M in M_SWEEP}


# ================================================================ the two arms
def base_line(args, world, metric, value, unit, dtype, config, scaling="weak"):
    return {"metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": max(args.warmup, 3), "higher_is_better": True, "scaling": scaling, "vs_baseline": None,
            "dtype": dtype, "data": "synthetic (seeded: N(0,1) activations and images, N(0,0.02) or Kaiming weights, "
                                    "uniform token ids)", "config": config}


def run_xdna(args, rank, world):
    import torch_xdna
    from torch_xdna import kernels

    if not torch_xdna.gpu_available():
        raise SystemExit(f"no usable B200: {kernels.unavailable_reason()}")
    dev = torch.device("cuda", torch.cuda.current_device())
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    wl = args.workload
    line = None
    if wl in ("all", "cfg2", "square"):
        rec = cfg2_records(args, rank, world, dev, flush)
        metric = CFG2_METRIC if wl != "square" else "int8 TOPS/GPU, W8A8 linear (BASELINE config 2 square 4096^3)"
        config = cfg2_config(args.rows) if wl != "square" else {
            "workload": "cfg2 square int8 GEMM M=N=K=4096 (quantise + GEMM + dequantise to bf16)", "l2": "flushed between steps"}
        line = base_line(args, world, metric, rec.pop("value"), "TOPS", "int8", config)
        line.update(rec)
    if wl in ("all", "msweep") and world == 1:
        ms = msweep_record(args, dev, flush)
        if line is None:
            line = base_line(args, world, "int8 TOPS/GPU, W8A8 linear (BASELINE config 2 row sweep)", None, "TOPS",
                             "int8", {"workload": f"cfg2 projection set at M = {list(M_SWEEP)}"})
        line["m_sweep"] = ms
    torch.cuda.empty_cache()
    if wl in ("all", "conv"):
        rec = conv_record(args, rank, world, dev, flush)
        if line is None:
            line = base_line(args, world, rec.pop("metric"), rec.pop("value"), "TOPS", "int8", rec.pop("config"),
                             "strong")
            line.update(rec)
        else:
            line["conv"] = rec
    elif wl == "cfg3":
        rec = cfg3_record(args, rank, world, dev)
        line = base_line(args, world, "ms per call, conv3x3 (BASELINE config 3: 4 x 256ch 64x64 + ReLU)",
                         rec.pop("ms_per_step"), "ms", "int8", {"workload": "cfg3 1x256x64x64, 4 convs + ReLU"})
        line["higher_is_better"] = False
        line.update(rec)
    torch.cuda.empty_cache()
    if wl in ("all", "stack"):
        rec = stack_record(args, rank, world, dev)
        if line is None:
            line = base_line(args, world, rec.pop("metric"), rec.pop("value"), "tokens/s", "bf16", rec.pop("config"),
                             "strong")
            line.update(rec)
        else:
            line["stack"] = rec
    del flush
    torch.cuda.synchronize()
    # CPU baselines last (rank 0, one GPU): host work after every GPU measurement
    if rank == 0 and world == 1:
        if wl in ("all", "cfg2"):
            line["cpu_baseline"] = cpu_cfg2(args.rows)
        if wl in ("all", "msweep"):
            for k, cb in cpu_msweep().items():
                line["m_sweep"][k]["cpu_baseline"] = cb
        conv = line.get("conv", line if wl == "conv" else None)
        if conv is not None:
            conv["cpu_baseline"] = cpu_vgg()
            conv["cfg3"]["cpu_baseline"] = cpu_cfg3()
        if wl == "cfg3":
            line["cpu_baseline"] = cpu_cfg3()
        stack = line.get("stack", line if wl == "stack" else None)
        if stack is not None:
            stack["cpu_baseline"] = cpu_stack(args.layers)
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU route for the same records on the host cores, rank 0 only. The
    top level is config 2 at the full row count, one pass of the whole projection set per step."""
    if rank != 0:
        return
    wl = args.workload
    if wl in ("all", "cfg2", "square"):
        rows = args.rows if wl != "square" else 4096
        cb = cpu_cfg2(rows, budget_s=0.0, min_passes=max(1, args.steps)) if wl != "square" else None
        if wl == "square":
            cb = cpu_square(max(1, args.steps))
        line = base_line(args, world, CFG2_METRIC if wl != "square" else
                         "int8 TOPS/GPU, W8A8 linear (BASELINE config 2 square 4096^3)", cb["value"], "TOPS", "int8",
                         cfg2_config(args.rows) if wl != "square" else {"workload": "cfg2 square int8 GEMM M=N=K=4096"})
    elif wl == "conv":
        cb = cpu_vgg()
        line = base_line(args, world, CONV_METRIC, cb["value"], "TOPS", "int8",
                         {"workload": "cfg4 VGG16 conv3x3 stack int8, 32x3x224x224", "global_batch": args.images},
                         "strong")
    elif wl == "cfg3":
        cb = cpu_cfg3()
        line = base_line(args, world, "ms per call, conv3x3 (BASELINE config 3: 4 x 256ch 64x64 + ReLU)", cb["value"],
                         "ms", "int8", {"workload": "cfg3 1x256x64x64, 4 convs + ReLU"})
        line["higher_is_better"] = False
    elif wl == "stack":
        cb = cpu_stack(args.layers)
        line = base_line(args, world, STACK_METRIC, cb["value"], "tokens/s", "fp32",
                         {"workload": f"cfg5 Qwen3-0.6B stack: {args.layers} layers, {args.seqs} sequences x "
                                      f"{args.seq_len} tokens, causal, head {V_HEAD}", "global_batch": args.seqs,
                          "seq_len": args.seq_len}, "strong")
    else:   # msweep
        ms = cpu_msweep()
        cb = ms[str(M_SWEEP[-1])]
        line = base_line(args, world, "int8 TOPS/GPU, W8A8 linear (BASELINE config 2 row sweep)", cb["value"], "TOPS",
                         "int8", {"workload": f"cfg2 projection set at M = {list(M_SWEEP)}"})
        line["m_sweep"] = {k: {"value": v["value"], "unit": "TOPS", "cpu_baseline": v} for k, v in ms.items()}
    line.update({"impl": "reference", "cpu_baseline": cb,
                 "e2e": {"value": cb["value"], "unit": cb["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})
    if wl == "all":
        ms = cpu_msweep()
        line["m_sweep"] = {k: {"value": v["value"], "unit": "TOPS", "cpu_baseline": v} for k, v in ms.items()}
        vgg, c3, st = cpu_vgg(), cpu_cfg3(), cpu_stack(args.layers)
        line["conv"] = {"metric": CONV_METRIC, "value": vgg["value"], "unit": "TOPS", "cpu_baseline": vgg,
                        "cfg3": {"ms_per_step": c3["value"], "cpu_baseline": c3}}
        line["stack"] = {"metric": STACK_METRIC, "value": st["value"], "unit": "tokens/s", "cpu_baseline": st}
    print(json.dumps(line), flush=True)


def cpu_square(passes):
    from oracle import reference_cpu as rc

    threads = _threads()
    g = torch.Generator().manual_seed(1)
    w_kn, sw = rc.quant_weight((torch.randn(4096, 4096, generator=g) * 0.02).to(torch.bfloat16))
    x = torch.randn(4096, 4096, generator=g).to(torch.bfloat16)
    with torch.no_grad():
        rc.linear_int8(x, w_kn, sw)
        times = []
        for _ in range(passes):
            t0 = time.perf_counter()
            rc.linear_int8(x, w_kn, sw)
            times.append(time.perf_counter() - t0)
    return {"value": round(2 * 4096 ** 3 / statistics.median(times) / 1e12, 4), "unit": "TOPS", "cores": threads,
            "kind": "port", "sample": f"the whole 4096^3 linear, median of {passes} passes"}


# ================================================================ one kernel (profiling)
def run_kernel(args):
    """--kernel NAME --shape a,b,c: one kernel of libxdna_b200 on one shape, warm-up then 20 launches replayed
    from a CUDA graph and timed with CUDA events (the command the ncu summaries are captured with;
    back-to-back launches on the same inputs, so operands may stay in L2 between them). Prints one JSON
    line."""
    from torch_xdna import conv as xconv
    from torch_xdna import kernels

    dev = torch.device("cuda", 0)
    shp = [int(v) for v in args.shape.split(",")]
    g = torch.Generator(device=dev).manual_seed(0)
    if args.kernel == "gemm_i8":                      # M, N, K: bf16 out through the dequantising epilogue
        M, N, K = shp
        xq = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=dev, generator=g)
        wq = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev, generator=g)
        sx, sw = torch.rand(M, device=dev) * 0.01, torch.rand(N, device=dev) * 0.01
        y = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
        fn, work, unit = (lambda: kernels.gemm_i8(xq, wq, K, y, sx, sw)), 2 * M * N * K, "TOPS"
    elif args.kernel == "quant_rows":                 # R, K: bf16 rows
        R, K = shp
        x = torch.randn(R, K, device=dev, generator=g).to(torch.bfloat16)
        xq, sx = torch.empty(R, K, dtype=torch.int8, device=dev), torch.empty(R, device=dev)
        fn, work, unit = (lambda: kernels.quant_rows(x, xq, sx)), 3 * R * K, "GB/s"
    elif args.kernel == "conv3x3":                    # N, C, H: C -> C channels on H x H, dequantise epilogue
        N, C, H = shp
        w = torch.nn.Parameter(torch.randn(C, C, 3, 3, device=dev, generator=g) * (2 / (C * 9)) ** 0.5)
        lay = xconv.ConvLayer(w, H, H, False)
        lay.shift, lay.scale = 10, lay.sw * 1024.0
        xp = torch.randint(-127, 128, (N, H + 2, H + 2, lay.cp), dtype=torch.int8, device=dev, generator=g)
        sx, b = torch.rand(N, device=dev), torch.randn(C, device=dev) * 0.01
        y = torch.empty(N, C, H, H, device=dev, memory_format=torch.channels_last)
        fn = lambda: kernels.conv3x3(xp, lay.wp, N, C, C, H, H, kernels.CONV_DEQUANT, shift=10, scale=lay.scale,  # noqa
                                     sx=sx, bias=b, out=y)
        work, unit = 2 * N * C * C * H * H * 9, "TOPS"
    elif args.kernel == "conv3x3_chain":              # N, C, H: C -> C on H x H as a chain runs it: int8 codes
        N, C, H = shp                                  # out, the next layer's pooled per-image maxima
        w = torch.nn.Parameter(torch.randn(C, C, 3, 3, device=dev, generator=g) * (2 / (C * 9)) ** 0.5)
        lay = xconv.ConvLayer(w, H, H, False)
        lay.shift, lay.scale = 10, lay.sw * 1024.0
        pairs = C == 64 and N % 2 == 0    # the chain's 64-channel input: two images per 128-byte row
        xp = (torch.randint(-127, 128, (N // 2, H + 2, H + 2, 128), dtype=torch.int8, device=dev, generator=g)
              if pairs else torch.randint(-127, 128, (N, H + 2, H + 2, lay.cp), dtype=torch.int8, device=dev,
                                          generator=g))
        sx, b = torch.rand(N, device=dev) + 0.5, torch.randn(C, device=dev) * 0.01
        q = torch.empty(N, H, H, C, dtype=torch.int8, device=dev)
        amax = torch.empty(N, dtype=torch.int32, device=dev)
        mode = (kernels.CONV_Q_NHWC | kernels.CONV_NEXT_AMAX | kernels.CONV_NEXT_RELU | kernels.CONV_NEXT_POOL
                | (kernels.CONV_PAIRS if pairs else 0))
        fn = lambda: kernels.conv3x3(xp, lay.wp, N, C, C, H, H, mode, shift=10, scale=lay.scale, sx=sx,  # noqa
                                     bias=b, out=q, acc_max=amax)
        work, unit = 2 * N * C * C * H * H * 9, "TOPS"
    elif args.kernel == "conv_quant_codes":           # N, C, H[, 1]: the chain's quantise from int8 codes [N, H, H, C]
        N, C, H = shp[:3]                              # (ReLU after the bias, maxima given); 1: 2x2 pool first
        pool = len(shp) > 3 and shp[3] == 1
        q = torch.randint(-128, 128, (N, H, H, C), dtype=torch.int8, device=dev, generator=g)
        scale = torch.rand(C, device=dev, generator=g) * 1e-3 + 1e-4
        sx_in = torch.rand(N, device=dev, generator=g) + 0.5
        b = torch.randn(C, device=dev, generator=g) * 0.05
        Ho = H // 2 if pool else H
        xp = torch.empty(N, Ho + 2, Ho + 2, xconv.channels_padded(C), dtype=torch.int8, device=dev)
        sx = torch.empty(N, device=dev)
        amax = torch.full((N,), 0x3F800000, dtype=torch.int32, device=dev)   # 1.0f
        fn = lambda: kernels.conv_quant_codes_given_amax(q, scale, sx_in, b, True, pool, xp, sx, amax)  # noqa
        work, unit = q.numel() + xp.numel(), "GB/s"
    elif args.kernel == "attention":                  # B, L: causal, 16 q heads / 8 kv heads of 128
        B, L = shp
        qk = torch.randn(B * L, 3072, device=dev, generator=g).to(torch.bfloat16)
        vt = torch.randn(1024, B * ((L + 7) // 8 * 8), device=dev, generator=g).to(torch.bfloat16)
        out = torch.empty(B * L, 2048, dtype=torch.bfloat16, device=dev)
        fn = lambda: kernels.attention(qk, vt, out, B, L, kernels.MASK_CAUSAL)  # noqa
        work, unit = B * 2 * 2 * 16 * 128 * (L * (L + 1) // 2), "TFLOP/s"
    elif args.kernel == "gemm_bf16":                  # M, N, K[, 1]: bf16 out (the head's epilogue); 1: residual add
        M, N, K = shp[:3]
        a = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
        b = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        if len(shp) > 3 and shp[3] == 1:
            resid = torch.zeros(M, N, device=dev)
            fn = lambda: kernels.gemm_bf16(a, b, kernels.GEMM_RESID, resid=resid)  # noqa
        else:
            y = torch.empty(M, N, dtype=torch.bfloat16, device=dev)
            fn = lambda: kernels.gemm_bf16(a, b, kernels.GEMM_F32ACC, out=y)  # noqa
        work, unit = 2 * M * N * K, "TFLOP/s"
    elif args.kernel == "gemm_bf16_qkv":             # B, L: the stack's fused q/k/v projection over B x L tokens
        B, L = shp
        T, L8 = B * L, (L + 7) // 8 * 8
        h = torch.randn(T, 1024, device=dev, generator=g).to(torch.bfloat16)
        w = (torch.randn(4096, 1024, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        inv = 1.0 / (1e6 ** (torch.arange(0, 128, 2, device=dev, dtype=torch.float32) / 128))
        ang = torch.arange(L, device=dev, dtype=torch.float32)[:, None] * inv[None, :]
        cos, sin = kernels.rope_layout(ang.cos()), kernels.rope_layout(ang.sin())
        qn, kn = torch.ones(128, device=dev), torch.ones(128, device=dev)
        qk = torch.empty(T, 3072, dtype=torch.bfloat16, device=dev)
        vt = torch.zeros(1024, B * L8, dtype=torch.bfloat16, device=dev)
        fn = lambda: kernels.gemm_bf16(h, w, kernels.GEMM_QKV, out=qk, vt=vt, rope_cos=cos, rope_sin=sin,  # noqa
                                       q_norm=qn, k_norm=kn, seq_len=L)
        work, unit = 2 * T * 4096 * 1024, "TFLOP/s"
    else:
        raise SystemExit(f"unknown kernel {args.kernel}")
    for _ in range(5):
        fn()
    torch.cuda.synchronize()
    # 20 launches captured in a CUDA graph: the replay times the kernels, not the host's launch path
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(20):
            fn()
    graph.replay()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    graph.replay()
    e.record()
    torch.cuda.synchronize()
    us = s.elapsed_time(e) / 20 * 1e3
    if kernels.take_device_error() != (0, 0):
        raise SystemExit("a kernel recorded a device-side timeout")
    print(json.dumps({"kernel": args.kernel, "shape": shp, "us_per_launch": round(us, 2),
                      "rate": round(work / us / 1e6 if unit != "GB/s" else work / us / 1e3, 1), "unit": unit}))


def main():
    args = parse()
    if args.kernel:
        run_kernel(args)
        return
    rank, world = dist_init(args.gpus)
    try:
        if args.impl == "reference":
            run_reference(args, rank, world)
        else:
            run_xdna(args, rank, world)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
