"""Benchmark: int8 TOPS of the W8A8 linear path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl xdna|reference] [--workload cfg2|square]

One step = one pass of the hot path over one batch: BASELINE config 2's Qwen3-0.6B projection set at
M = 8192 rows, bf16 activations, W8A8 -- xdna::linear_cat q/k/v (N = 2048+1024+1024, K = 1024),
xdna::linear_cat gate/up (N = 2x3072, K = 1024) and xdna::linear down (N = 1024, K = 3072). Each op is
our quantise kernel followed by our tcgen05 int8 GEMM with the dequantising epilogue. Metric: int8
TOPS = 2*M*sum(N*K) per step / step time, whole job (all ranks).

  value      device time of the K steps (CUDA events on the launching stream), inputs resident in HBM,
             L2 flushed (a 256 MiB write) between steps, outside the events;
  e2e        the same steps through the public API (torch.compile(backend="xdna")) with the inputs
             copied from pinned host memory and every output copied back, inside the timed region;
  roofline   the GEMM kernel alone: its algorithmic int8 ops per launch / its event-timed duration,
             against the int8 peak (2x the measured dense bf16 cuBLAS rate in MEASURED_PEAKS.json --
             B200's dense int8 rate is twice its bf16 rate);
  cpu_baseline  the reference's CPU route (torch._int_mm + its eager quantise / dequantise ops),
             restated in oracle/reference_cpu.py, on a bounded row sample, all host threads.

--impl reference times only that CPU route, on rank 0, and prints its own line.
Multi-GPU (torchrun): the linear does not shard (replicas only): every rank runs the whole workload,
value = ranks x units / max-over-ranks time.
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
L2_FLUSH_BYTES = 256 << 20


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="xdna", choices=["xdna", "reference"])
    ap.add_argument("--workload", default="cfg2", choices=["cfg2", "square", "stack", "conv"],
                    help="cfg2: W8A8 projection set (default); square: 4096^3 int8 GEMM; stack: BASELINE config 5; "
                         "conv: BASELINE config 4")
    ap.add_argument("--rows", type=int, default=8192)
    ap.add_argument("--cpu-rows", type=int, default=1024, help="row sample of the CPU baseline")
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
                    choices=["gemm_i8", "quant_rows", "conv3x3", "attention", "gemm_bf16", "gemm_bf16_qkv"],
                    help="time one kernel on --shape instead of a workload (profiling)")
    ap.add_argument("--shape", default="8192,6144,1024", help="--kernel shape, comma-separated")
    args = ap.parse_args()
    if args.workload in ("stack", "conv") and args.steps == 2000:
        args.steps = 10          # a step of these workloads is milliseconds, not microseconds
    return args


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


# ---------------------------------------------------------------- workload
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


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples (every 200 ms) of this GPU's clocks and throttle reasons while running."""

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


# ---------------------------------------------------------------- the CPU baseline (reference route)
def cpu_baseline(workload, rows_sample, budget_s=12.0):
    """The reference's CPU route on a bounded row sample (oracle/reference_cpu.py), all host threads."""
    from oracle import reference_cpu as rc

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(1)
    shapes = gemm_shapes(workload, rows_sample)
    ops = []
    for (m, n, k) in shapes:
        w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
        w_kn, sw = rc.quant_weight(w)
        x = torch.randn(m, k, generator=g).to(torch.bfloat16)
        ops.append((x, w_kn, sw))
    with torch.no_grad():
        for x, w_kn, sw in ops:           # warm-up
            rc.linear_int8(x, w_kn, sw)
        times = []
        t_end = time.perf_counter() + budget_s
        while time.perf_counter() < t_end or len(times) < 3:
            t0 = time.perf_counter()
            for x, w_kn, sw in ops:
                rc.linear_int8(x, w_kn, sw)
            times.append(time.perf_counter() - t0)
    step = statistics.median(times)
    work = sum(2 * m * n * k for m, n, k in shapes)
    return {"value": round(work / step / 1e12, 4), "unit": "TOPS", "cores": threads, "kind": "port",
            "sample": f"{workload} projection set at {rows_sample} rows (of the workload's rows), "
                      f"median of {len(times)} passes; torch._int_mm + eager quantise/dequantise (reference route)"}


def run_reference(args, rank, world):
    if rank != 0:
        return
    rows = args.cpu_rows if args.workload == "cfg2" else 4096
    cb = cpu_baseline(args.workload, rows, budget_s=12.0)   # a bounded sample: ~12 s of CPU work
    line = {"impl": "reference", "metric": metric_name(args.workload), "value": cb["value"], "unit": "TOPS",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
            "config": config_of(args), "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def metric_name(workload):
    return "int8 TOPS/GPU, W8A8 linear (BASELINE config 2" + (" square 4096^3)" if workload == "square" else
                                                               " Qwen3-0.6B projection set)")


def config_of(args):
    if args.workload == "square":
        return {"workload": "cfg2 square int8 GEMM M=N=K=4096 (quantise + GEMM + dequantise to bf16)",
                "l2": "flushed between steps"}
    return {"workload": f"cfg2 Qwen3-0.6B projection set, W8A8, M={args.rows} rows bf16: linear_cat qkv "
                        f"(N=4096,K=1024) + linear_cat gate/up (N=6144,K=1024) + linear down (N=1024,K=3072)",
            "global_batch": args.rows, "parallelism": "replicas", "l2": "flushed between steps (256 MiB write)"}


# ---------------------------------------------------------------- the B200 arm
def run_xdna(args, rank, world):
    import torch_xdna
    from torch_xdna import kernels

    dev = torch.device("cuda", torch.cuda.current_device())
    if not torch_xdna.gpu_available():
        raise SystemExit(f"no usable B200: {kernels.unavailable_reason()}")
    torch.manual_seed(0)
    cfg = torch_xdna.Config(verify="first", fallback="eager")
    cid = torch_xdna.ops.config_id(cfg)
    model = make_model(dev)
    R = args.rows
    x = torch.randn(R, D, device=dev).to(torch.bfloat16)          # attention-norm output
    x2 = torch.randn(R, D, device=dev).to(torch.bfloat16)         # MLP-norm output
    act = torch.randn(R, INTER, device=dev).to(torch.bfloat16)    # silu(gate) * up
    if args.workload == "square":
        w_sq = (torch.randn(4096, 4096, device=dev) * 0.02).to(torch.bfloat16)
        x = torch.randn(4096, 4096, device=dev).to(torch.bfloat16)
    shapes = gemm_shapes(args.workload, R)
    work = sum(2 * m * n * k for m, n, k in shapes)

    qkv = [model.q.weight, model.k.weight, model.v.weight]
    gu = [model.gate.weight, model.up.weight]

    def step():
        if args.workload == "square":
            return [torch.ops.xdna.linear(x, w_sq, None, False, cid)]
        return [torch.ops.xdna.linear_cat(x, qkv, [None] * 3, cid), torch.ops.xdna.linear_cat(x2, gu, [None] * 2, cid),
                torch.ops.xdna.linear(act, model.down.weight, None, False, cid)]

    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    with torch.no_grad():
        for _ in range(max(args.warmup, 3)):   # includes each kernel configuration's first-call verify
            step()
        torch.cuda.synchronize()
        # One step captured as a CUDA graph (the same kernels, launched without Python in between):
        # the timed region measures device work, not host launch overhead.
        torch_xdna.stats.reset()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        per_step = torch_xdna.stats.launches
        graph.replay()
        barrier(world)
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        with ClockSampler(dev.index) as clocks:
            barrier(world)
            for i in range(args.steps):
                flush.fill_(i & 0xFF)
                starts[i].record(stream)
                graph.replay()
                ends[i].record(stream)
            barrier(world)
        launches = per_step * args.steps
        step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
        del graph
    total_s = max_over_ranks(sum(step_ms) / 1e3, world)
    value = world * work * args.steps / total_s / 1e12

    # ---- roofline: the GEMM kernel alone (same shapes, same stream), event-timed per launch
    roof = gemm_roofline(shapes, dev, args.steps, flush)
    # config 2's square M = N = K = 4096 GEMM, the case the >= 70 %-of-peak target is stated on
    roof_sq = gemm_roofline([(4096, 4096, 4096)], dev, args.steps, flush) if args.workload == "cfg2" else None
    # ---- e2e through torch.compile(backend="xdna") with host buffers
    e2e = e2e_measure(args, model, dev, world, work)
    # ---- CPU baseline (rank 0, one GPU only)
    cb = cpu_baseline(args.workload, args.cpu_rows if args.workload == "cfg2" else 1024) \
        if (rank == 0 and world == 1) else None
    if kernels.take_device_error() != (0, 0):
        raise SystemExit("a kernel recorded a device-side timeout")
    if rank == 0:
        line = {"metric": metric_name(args.workload), "value": round(value, 2), "unit": "TOPS", "n_gpus": world,
                "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": round(total_s * 1e3 / args.steps, 4),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
                "data": "synthetic (seeded N(0,1) activations, N(0,0.02) weights)", "config": config_of(args),
                "gpu_launches": launches, "roofline": roof, "e2e": e2e, "clocks": clocks.summary()}
        if roof_sq is not None:
            line["roofline_square_4096"] = roof_sq
        if cb is not None:
            line["cpu_baseline"] = cb
        print(json.dumps(line), flush=True)


def int8_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return 2 * float(d["bf16_tflops"]), "2x measured dense bf16 cuBLAS burst (MEASURED_PEAKS.json)"
    return 2 * 1590.0, "2x fallback dense bf16 1.59 PFLOP/s"


# DRAM bytes (read + write) of one gemm_i8 launch per shape, from one ncu capture each
# (profiles/gemm_i8_dram_traffic.md has the command).
PROFILED_DRAM_BYTES = {(8192, 4096, 1024): 26222336, (8192, 6144, 1024): 61992960, (8192, 1024, 3072): 28405248,
                       (4096, 4096, 4096): 36336640}


def gemm_roofline(shapes, dev, steps, flush):
    """Algorithmic int8 ops per launch of the GEMM kernel / its CUDA-event duration, summed over the
    workload's GEMMs; inputs pre-quantised, L2 flushed before every launch."""
    from torch_xdna import kernels

    cases = []
    for (m, n, k) in shapes:
        xq = torch.randint(-127, 128, (m, k), dtype=torch.int8, device=dev)
        wq = torch.randint(-127, 128, (n, k), dtype=torch.int8, device=dev)
        sx = torch.rand(m, device=dev) * 0.01
        sw = torch.rand(n, device=dev) * 0.01
        y = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
        cases.append((xq, wq, k, y, sx, sw))
    stream = torch.cuda.current_stream()
    for c in cases:
        for _ in range(3):
            kernels.gemm_i8(c[0], c[1], c[2], c[3], c[4], c[5])
    total_ms, total_ops = 0.0, 0
    reps = max(5, steps)
    for (m, n, k), c in zip(shapes, cases):
        ms = []
        for _ in range(reps):
            flush.fill_(1)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            kernels.gemm_i8(c[0], c[1], c[2], c[3], c[4], c[5])
            e.record(stream)
            e.synchronize()
            ms.append(s.elapsed_time(e))
        total_ms += statistics.median(ms)
        total_ops += 2 * m * n * k
    torch.cuda.synchronize()
    peak, src = int8_peak()
    achieved = total_ops / (total_ms / 1e3) / 1e12
    traffic = None
    if all(tuple(sh) in PROFILED_DRAM_BYTES for sh in shapes):
        traffic = round(sum(PROFILED_DRAM_BYTES[tuple(sh)] for sh in shapes) / len(shapes))
    return {"bound": "tensor", "kernel": "umma_gemm_kernel (gemm_i8, dequantising epilogue, bf16 out)",
            "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TOPS",
            "frac": round(achieved / peak, 4), "peak_source": src, "traffic": traffic,
            "traffic_unit": "bytes per launch (ncu dram__bytes_read.sum + dram__bytes_write.sum)",
            "per_launch_ms": round(total_ms / len(shapes), 4)}


def e2e_measure(args, model, dev, world, work):
    """The step through torch.compile(backend="xdna"), fed from and drained to pinned host memory as a
    serving loop would: every step copies its three inputs host -> device and its six outputs device ->
    host, on their own streams (the copy engines work in both directions at once), double-buffered so
    that step i+1's inputs, step i's GEMMs and step i-1's outputs overlap; events order each step's
    copy-in, compute and copy-out. The timed region covers every step's copies."""
    import torch_xdna  # noqa: F401  (registers the backend)

    if args.workload == "square":
        return None
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
    h2d = sum(t.numel() for t in hin[0]) * 2
    d2h = sum(t.numel() for t in hout[0]) * 2
    return {"value": round(world * work * steps / sec / 1e12, 2), "unit": "TOPS", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "api": "torch.compile(backend='xdna', fallback='eager')",
            "pipeline": "copy-in / compute / copy-out streams, double-buffered pinned host and device buffers"}


# ---------------------------------------------------------------- the Qwen3 stack
V_HEAD = 151936


def stack_flops(B, L, layers, vocab):
    """Algorithmic FLOPs of one step: the projections and head per token, causal attention (QK^T and PV over
    the keys each query sees)."""
    per_token = 2 * (layers * (D * 4096 + 2048 * D + D * 6144 + INTER * D) + D * vocab)
    attn = layers * B * 2 * 2 * 16 * 128 * (L * (L + 1) // 2)
    return B * L * per_token + attn


def run_stack(args, rank, world):
    """One step = embed the token ids of this rank's sequences and run xdna_qwen3_stack (28 layers, final
    norm, head over 151936) under a causal mask; the global batch is fixed (strong scaling). The layers
    are data-parallel over sequences (independent: no collective). The head, on more than one GPU, is
    column-parallel by default: an NCCL all-gather of every rank's final hidden states
    over NVLink, then each rank computes its 151936 / N vocabulary columns for all tokens; --head dp keeps
    it with the sequences instead."""
    import torch_xdna
    from torch_xdna import kernels, parallel

    if not torch_xdna.gpu_available():
        raise SystemExit(f"no usable B200: {kernels.unavailable_reason()}")
    dev = torch.device("cuda", torch.cuda.current_device())
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
    ids = torch.randint(0, V_HEAD, (B * L,), device=dev, generator=g)
    x = torch.empty(B * L, D, device=dev)
    out = torch.empty(B_all * L if column else B * L, n_cols, dtype=torch.bfloat16, device=dev)
    ws = torch.empty(kernels.qwen3_stack_workspace(B, L), dtype=torch.uint8, device=dev)
    hidden = ws[:B * L * D * 2].view(torch.bfloat16).view(B * L, D)   # the final-normed states (workspace head)
    h_all = torch.empty(B_all * L, D, dtype=torch.bfloat16, device=dev) if column and not fused else None
    rg = parallel.RowGather(B * L, D, dev, mode="direct" if args.head == "column-direct" else "pipelined") \
        if fused else None
    launches_per_step = 1 + 7 * NL + 2

    def step(ids_dev):
        kernels.embed(ids_dev, embed, x)
        if column:
            kernels.qwen3_stack(table, final, head, None, cos, sin, 1e-6, x, B, L, kernels.MASK_CAUSAL, None, None,
                                None, ws)
            if fused:
                rg.local.copy_(hidden)
                rg.gemm(head, out)
            else:
                parallel.gather_rows(hidden, h_all)
                kernels.gemm_bf16(h_all, head, kernels.GEMM_F32ACC, out=out)
        else:
            kernels.qwen3_stack(table, final, head, None, cos, sin, 1e-6, x, B, L, kernels.MASK_CAUSAL, None, None,
                                out, ws)

    stream = torch.cuda.current_stream()
    for _ in range(max(args.warmup, 3)):
        step(ids)
    if column:   # once, untimed: this rank's vocabulary slice of 256 rows of every rank vs an f32 product
        gathered = torch.empty(B_all * L, D, dtype=torch.bfloat16, device=dev)
        parallel.gather_rows(hidden, gathered)
        for r in range(world):
            rows = slice(r * B * L, r * B * L + 256)
            ref = gathered[rows].float() @ head.float().t()
            err = float((out[rows].float() - ref).abs().max() / ref.abs().max())
            if not err < 2e-2:
                raise SystemExit(f"rank {rank}: column-parallel head rows of rank {r} disagree with the f32 "
                                 f"product (rel {err:.3g})")
        del gathered
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
    value = tokens / total_s
    flops = stack_flops(B, L, NL, V_HEAD)

    # roofline: the head GEMM (the largest single launch), timed alone per launch
    hn = torch.randn(out.shape[0], D, device=dev).to(torch.bfloat16)
    for _ in range(2):
        kernels.gemm_bf16(hn, head, kernels.GEMM_F32ACC, out=out)
    ms = []
    for _ in range(5):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        kernels.gemm_bf16(hn, head, kernels.GEMM_F32ACC, out=out)
        e.record(stream)
        e.synchronize()
        ms.append(s.elapsed_time(e))
    head_ms = statistics.median(ms)
    head_flops = 2 * out.shape[0] * n_cols * D
    peaks = json.loads((ROOT / "MEASURED_PEAKS.json").read_text()) if (ROOT / "MEASURED_PEAKS.json").exists() else {}
    peak = float(peaks.get("bf16_tflops", 1590.0))
    roof = {"bound": "tensor", "kernel": "umma_gemm_kernel bf16 (the head GEMM, EPI_F32ACC)",
            "achieved": round(head_flops / head_ms / 1e9, 1), "peak": peak, "unit": "TFLOP/s",
            "frac": round(head_flops / head_ms / 1e9 / peak, 4),
            "peak_source": "measured dense bf16 cuBLAS burst (MEASURED_PEAKS.json)" if peaks else "fallback",
            "traffic": None, "per_launch_ms": round(head_ms, 4),
            "step_tflops": round(flops * args.steps * world / total_s / 1e12, 1)}

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
    e2e = {"value": round(B_all * L * e_steps / e2e_s, 1), "unit": "tokens/s", "h2d_bytes_per_step": h_ids.numel() * 8,
           "d2h_bytes_per_step": h_out.numel() * 2, "api": "xdna_qwen3_stack C ABI (torch_xdna.kernels)"}
    if rg is not None:
        rg.close()
    cb = cpu_stack_baseline(NL, 1, 128) if (rank == 0 and world == 1) else None
    if kernels.take_device_error() != (0, 0):
        raise SystemExit("a kernel recorded a device-side timeout")
    if rank == 0:
        line = {"metric": "Qwen3-0.6B stack tokens/s (BASELINE config 5)", "value": round(value, 1),
                "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 3),
                "ms_per_step": round(total_s * 1e3 / args.steps, 3), "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (uniform token ids, N(0,0.02) weights, unit norms)",
                "config": {"workload": f"cfg5 Qwen3-0.6B stack: {NL} layers, {B_all} sequences x {L} tokens, causal "
                                       f"mask, head {V_HEAD}, bf16 with f32 accumulation", "global_batch": B_all,
                           "seq_len": L, "l2": "inputs exceed L2",
                           "parallelism": (f"dp{world} sequences; head column-parallel over {world}, " + (
                               ("peer blocks copied over NVLink once, overlapping the GEMM over this rank's rows"
                                if args.head == "column" else "the GEMM's TMA reading every rank's rows from its memory")
                               if fused else "NCCL all-gather of hidden states before the head GEMM"))
                           if column else f"dp{world} (sequences)"},
                "gpu_launches": launches_per_step * args.steps, "roofline": roof, "e2e": e2e,
                "clocks": clocks.summary()}
        if cb is not None:
            line["cpu_baseline"] = cb
        print(json.dumps(line), flush=True)


def cpu_stack_baseline(layers, seqs, seq_len):
    """The reference's parity route for the stack (the fp32 eager model) restated in torch CPU ops
    (oracle/reference_cpu.py) on a bounded sample, all host threads."""
    from oracle import reference_cpu as rc

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
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
        rc.qwen3_stack(ls, torch.ones(D), head, None, x, mask)
        t0 = time.perf_counter()
        rc.qwen3_stack(ls, torch.ones(D), head, None, x, mask)
        dt = time.perf_counter() - t0
    return {"value": round(seqs * seq_len / dt, 1), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{seqs} sequence x {seq_len} tokens through {layers} layers + head {V_HEAD}, fp32 eager "
                      f"torch CPU (the reference's parity model)"}


# ---------------------------------------------------------------- VGG16 int8 convs
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


def single_conv_roofline(dev, stream, peak, src):
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
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    ms = []
    for i in range(8):
        flush.fill_(1)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        kernels.conv3x3(xp, lay.wp, 1, 256, 256, 1536, 64, kernels.CONV_DEQUANT, shift=lay.shift, scale=lay.scale,
                        sx=sx, bias=b, relu=kernels.RELU_AFTER_BIAS, out=yo)
        e.record(stream)
        e.synchronize()
        if i >= 2:
            ms.append(s.elapsed_time(e))
    ops = 2 * 1536 * 64 * 256 * 256 * 9
    achieved = ops / statistics.median(ms) / 1e9
    return {"bound": "tensor", "kernel": "umma_gemm_kernel LOAD_CONV (conv 256->256, 1 x 1536 x 64, bias + ReLU)",
            "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TOPS", "frac": round(achieved / peak, 4),
            "peak_source": src, "per_launch_ms": round(statistics.median(ms), 4)}


def run_conv(args, rank, world):
    """One step = the 13 int8 conv3x3 layers of VGG16 (bias + ReLU, 2x2 max-pool between blocks) on this
    rank's share of a batch of 32 images 3x224x224 (batch sharded over ranks, strong scaling), as the
    backend compiles it: xdna::conv3x3_chain, the activations between convs kept as int8 codes (the next
    conv's quantise rebuilds the float values and takes the 2x2 max-pool on the codes), the last conv's
    output dequantised with bias and ReLU in its epilogue and max-pooled by torch. --conv-unchained runs
    xdna::conv3x3_fused per conv with torch's max-pool between (same values). The requantise shift of every
    layer comes from global image 0 (rank 0), broadcast to the other ranks."""
    import torch_xdna
    from torch_xdna import kernels, parallel

    if not torch_xdna.gpu_available():
        raise SystemExit(f"no usable B200: {kernels.unavailable_reason()}")
    dev = torch.device("cuda", torch.cuda.current_device())
    if world > 1:
        parallel.enable_data_parallel()
    N_all = args.images
    assert N_all % world == 0
    N = N_all // world
    layers = vgg_layers(dev)
    params = [("M" if l == "M" else (torch.nn.Parameter(l[0]), l[1])) for l in layers]
    cid = torch_xdna.ops.config_id(torch_xdna.Config(verify="first"))
    g = torch.Generator(device=dev).manual_seed(99)
    x_all = torch.randn(N_all, 3, 224, 224, device=dev, generator=g)
    x = x_all[rank * N:(rank + 1) * N].contiguous()
    del x_all

    from torch_xdna.conv import IN_CODES, IN_CODES_POOL, IN_FLOAT

    n_convs = sum(p != "M" for p in params)

    def step_unchained(inp):
        h = inp
        for p in params:
            if p == "M":
                h = torch.nn.functional.max_pool2d(h, 2)
            else:
                h = torch.ops.xdna.conv3x3_fused(h, p[0], p[1], False, cid, True)  # ReLU after the bias
        return h

    def step_chained(inp):
        h, meta, k, pool = inp, None, 0, False
        for p in params:
            if p == "M":
                if k == n_convs:   # after the last conv: a float tensor
                    h = torch.nn.functional.max_pool2d(h, 2)
                else:
                    pool = True    # taken into the next conv's quantise
                continue
            mode = IN_FLOAT if k == 0 else (IN_CODES_POOL if pool else IN_CODES)
            k += 1
            h, meta = torch.ops.xdna.conv3x3_chain(h, meta, p[0], p[1], False, cid, True, mode, k > 1, k < n_convs)
            pool = False
        return h

    step = step_unchained if args.conv_unchained else step_chained

    stream = torch.cuda.current_stream()
    with torch.no_grad():
        for _ in range(max(args.warmup, 3)):   # includes each layer's calibration and first-call verify
            step(x)
        torch.cuda.synchronize()
        # One step captured as a CUDA graph (the same kernels, launched without Python in between): with a
        # half or quarter batch per GPU the per-op host work would otherwise pace the step
        torch_xdna.stats.reset()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step(x)
        per_step = torch_xdna.stats.launches
        graph.replay()
        barrier(world)
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        with ClockSampler(dev.index) as clocks:
            barrier(world)
            for i in range(args.steps):      # 32 x 64 x 224 x 224 activations (400 MB) exceed L2
                starts[i].record(stream)
                graph.replay()
                ends[i].record(stream)
            barrier(world)
        launches = per_step * args.steps
        step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
        del graph
    total_s = max_over_ranks(sum(step_ms) / 1e3, world)
    value = 2 * vgg_macs(N_all) * args.steps / total_s / 1e12
    # roofline: the conv kernel of the largest-work layer (conv 64->64 at 224x224), timed alone
    from torch_xdna import conv as xconv

    lay = xconv._layer(params[1][0], 224, 224, False)
    xp = torch.zeros(N, 226, 226, lay.cp, dtype=torch.int8, device=dev)
    sx = torch.rand(N, device=dev)
    yo = torch.empty(N, 64, 224, 224, device=dev)
    ms = []
    for i in range(6):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        kernels.conv3x3(xp, lay.wp, N, 64, 64, 224, 224, kernels.CONV_DEQUANT, shift=lay.shift, scale=lay.scale,
                        sx=sx, bias=params[1][1], out=yo)
        e.record(stream)
        e.synchronize()
        if i:
            ms.append(s.elapsed_time(e))
    conv_ops = 2 * N * 224 * 224 * 64 * 64 * 9
    peak, src = int8_peak()
    achieved = conv_ops / statistics.median(ms) / 1e9
    roof = {"bound": "tensor", "kernel": "umma_gemm_kernel LOAD_CONV (conv 64->64 224x224, dequantise epilogue)",
            "achieved": round(achieved, 1), "peak": round(peak, 1), "unit": "TOPS", "frac": round(achieved / peak, 4),
            "peak_source": src, "traffic": None, "per_launch_ms": round(statistics.median(ms), 4)}
    # config 4's single Ci = Co = 256 conv on one 1536 x 64 image (bias, ReLU after it), timed alone
    single = single_conv_roofline(dev, stream, peak, src)
    cb = cpu_conv_baseline() if (rank == 0 and world == 1) else None
    if kernels.take_device_error() != (0, 0):
        raise SystemExit("a kernel recorded a device-side timeout")
    if rank == 0:
        line = {"metric": "int8 TOPS/GPU, conv3x3 (BASELINE config 4: VGG16 int8, batch 32)", "value": round(value, 2),
                "unit": "TOPS", "n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 3),
                "ms_per_step": round(total_s * 1e3 / args.steps, 3), "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "int8", "data": "synthetic (N(0,1) images, Kaiming weights, N(0,0.01) bias)",
                "config": {"workload": "cfg4 VGG16 conv3x3 stack int8, 32x3x224x224, bias + ReLU, 2x2 max-pool",
                           "between_convs": "fp32 tensors, torch max-pool" if args.conv_unchained
                           else "int8 codes (pool on the codes)",
                           "global_batch": N_all, "parallelism": f"dp{world} (images)", "l2": "activations exceed L2"},
                "gpu_launches": launches, "roofline": roof, "single_conv_256x1536x64": single,
                "clocks": clocks.summary()}
        if cb is not None:
            line["cpu_baseline"] = cb
        print(json.dumps(line), flush=True)


def cpu_conv_baseline(images=1):
    """The reference's CPU-integer conv route (oracle/reference_cpu.py: exact fp conv of the integers) through
    the VGG16 conv stack on a bounded sample, all host threads."""
    from oracle import reference_cpu as rc

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    layers = [("M" if l == "M" else (rc.conv_layer(l[0].cpu(), False), l[1].cpu())) for l in vgg_layers("cpu")]
    x = torch.randn(images, 3, 224, 224, generator=torch.Generator().manual_seed(3))

    def run():
        h = x
        for l in layers:
            h = torch.nn.functional.max_pool2d(h, 2) if l == "M" else torch.relu(rc.conv3x3_int8(h, l[0], l[1]))
        return h

    with torch.no_grad():
        run()
        t0 = time.perf_counter()
        run()
        dt = time.perf_counter() - t0
    return {"value": round(2 * vgg_macs(images) / dt / 1e12, 4), "unit": "TOPS", "cores": threads, "kind": "port",
            "sample": f"{images} image 3x224x224 through the 13 VGG16 convs (CPU integers: quantise, fp conv of "
                      f"the integers, requantise, dequantise)"}


def run_reference_workload(args, rank, world):
    """--impl reference for the stack and conv workloads: rank 0 times the CPU route on a bounded sample."""
    if rank != 0:
        return
    if args.workload == "stack":
        cb = cpu_stack_baseline(args.layers, 1, 128)
        metric, unit, dtype = "Qwen3-0.6B stack tokens/s (BASELINE config 5)", "tokens/s", "fp32"
        config = {"workload": f"cfg5 Qwen3-0.6B stack: {args.layers} layers, {args.seqs} sequences x {args.seq_len} "
                              f"tokens, causal, head {V_HEAD}", "global_batch": args.seqs, "seq_len": args.seq_len}
    else:
        cb = cpu_conv_baseline()
        metric, unit, dtype = "int8 TOPS/GPU, conv3x3 (BASELINE config 4: VGG16 int8, batch 32)", "TOPS", "int8"
        config = {"workload": "cfg4 VGG16 conv3x3 stack int8, 32x3x224x224", "global_batch": args.images}
    line = {"impl": "reference", "metric": metric, "value": cb["value"], "unit": unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": dtype, "data": "synthetic", "config": config, "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_kernel(args):
    """--kernel NAME --shape a,b,c: one kernel of libxdna_b200 on one shape, warm-up then 20 launches replayed
    from a CUDA graph and timed with CUDA events (the command the profiles/ summaries are captured with;
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
            if args.workload in ("stack", "conv"):
                run_reference_workload(args, rank, world)
            else:
                run_reference(args, rank, world)
        elif args.workload == "stack":
            run_stack(args, rank, world)
        elif args.workload == "conv":
            run_conv(args, rank, world)
        else:
            run_xdna(args, rank, world)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
