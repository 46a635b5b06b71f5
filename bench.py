"""Benchmark of the attention training hot path on B200.

Workload (default, --config c3): flash-attention forward + backward, bf16
inputs with fp32 accumulation, non-causal, B=8 H=16 L=4096 d=64 per GPU (the
headline shape). One step = pa_attn_fwd + pa_attn_bwd over one batch of seeded
synthetic inputs. Multi-GPU runs shard along batch x heads with no collective
on the data path: by default every rank owns its own B x H units (weak
scaling); --scaling strong splits the batches across ranks. `value` is the
FLOPs of all ranks over the slowest rank's device time. `e2e` runs the same
step through the C ABI from pinned host buffers (H2D of Q, K, V, dO and D2H of
O, LSE, dQ, dK, dV every step), pipelined over three streams; the serial figure
and the PCIe rates measured alone are kept beside it.

Other configs (side lines, same JSON contract):
  --config c4   long sequence: B=2 H=16 L=16384 d=128, bf16
  --config c1   single head:   B=1 H=1  L=128   d=32,  fp32 (split3 products)
  --config c2   the pre-LN block's attention: B=8 H=8 L=1024 d=64, fp32
  --linear      the MHA block's projection GEMMs
  --train       the data-parallel denoise training step

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c3|c4|c1|c2]
                    [--impl reference [--ref-kernels]]

Prints one JSON line (rank 0). FLOPs follow the FlashAttention convention:
fwd 4*B*H*L^2*d + bwd 10*B*H*L^2*d (the backward recomputes S), exp excluded.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from dataclasses import dataclass

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "pure-attention_b200")
sys.path.insert(0, PKG)


@dataclass(frozen=True)
class AttnConfig:
    B: int
    H: int
    L: int
    D: int
    dtype: str  # "bf16" or "f32" (tensors; the f32 path takes split3 products)

    @property
    def label(self):
        return f"B{self.B} H{self.H} N{self.L} d{self.D} {'bf16' if self.dtype == 'bf16' else 'fp32'}"

    def flops(self, B=None):
        return 14 * (self.B if B is None else B) * self.H * self.L * self.L * self.D


CONFIGS = {
    "c3": AttnConfig(8, 16, 4096, 64, "bf16"),    # headline
    "c4": AttnConfig(2, 16, 16384, 128, "bf16"),  # long sequence, head dim 128
    "c1": AttnConfig(1, 1, 128, 32, "f32"),       # single head
    "c2": AttnConfig(8, 8, 1024, 64, "f32"),      # attention of the pre-LN MHA block
}
HEADLINE = "c3"
L2_BYTES = 126 * 2 ** 20


def metric_of(cfg):
    return f"attn fwd+bwd TFLOPS/GPU ({cfg.label}) and % of dense tensor peak"


def workload_of(cfg):
    kind = ("bf16 in / fp32 accumulate" if cfg.dtype == "bf16"
            else "fp32 in/out, products as three bf16 MMAs (split3), fp32 accumulate")
    return (f"flash-attention fwd+bwd, {kind}, non-causal, B{cfg.B} H{cfg.H} L{cfg.L} d{cfg.D} "
            f"per GPU")


def config_dict(cfg, world, scaling):
    """The `config` object of the attention lines (identical in both arms)."""
    in_bytes = 4 * cfg.B * cfg.L * cfg.H * cfg.D * (2 if cfg.dtype == "bf16" else 4)
    if scaling == "strong":
        in_bytes //= world
    flush = in_bytes < L2_BYTES
    size = f"{in_bytes / 2**20:.0f} MiB" if in_bytes >= 2**20 else f"{in_bytes / 2**10:.0f} KiB"
    return {"workload": workload_of(cfg),
            "global_batch": cfg.B * world if scaling == "weak" else cfg.B,
            "seq_len": cfg.L, "heads": cfg.H, "head_dim": cfg.D,
            "parallelism": f"dp{world} (batch x head shards, no collective)",
            "l2": (f"inputs ({size}) fit in the 126 MB L2: L2 scrubbed "
                   f"(256 MiB write) before every timed step, steps timed without the scrub"
                   if flush else
                   f"inputs ({size} per GPU) exceed the 126 MB L2; no flush")}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default=HEADLINE, choices=sorted(CONFIGS))
    ap.add_argument("--scaling", default="weak", choices=["weak", "strong"],
                    help="weak: the config's B x H per GPU; strong: its B batches split across GPUs")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ref-kernels", action="store_true",
                    help="with --impl reference: time the reference's own CUDA kernels (fp32 SIMT, "
                         "built from its sources into oracle/_ref) on the GPU at C1, C2 and C3, "
                         "as context numbers")
    ap.add_argument("--linear", action="store_true",
                    help="instead of the attention step: time the fused projection calls of the "
                         "MHA block (B8 L1024 E512 fp32) against the unfused call sequence, in both "
                         "math modes, and the training step's projection shapes (bf16 math)")
    ap.add_argument("--train", action="store_true",
                    help="instead of the attention step: the data-parallel denoise training step "
                         "(6 layers, E1024 H16 FFN4096, N2048, 8 sequences per GPU, fp32 weights), "
                         "gradients averaged over the ranks with NCCL")
    ap.add_argument("--kernels", action="store_true",
                    help="instead of the attention step: each memory-bound kernel family (LayerNorm "
                         "fwd / add+fwd / bwd / bwd-accumulate, multi-tensor Adam, the attention "
                         "backward's prep and dQ-convert kernels) and the projection GEMM timed "
                         "alone with CUDA events, as achieved GB/s (or TFLOP/s) against the peak")
    ap.add_argument("--bucket-mb", type=float, default=100.0,
                    help="--train: gradient bucket size of the all-reduce")
    ap.add_argument("--tail-mb", type=float, default=0.0,
                    help="--train: the gradients backward finishes last (this many MB) go into "
                         "smaller buckets of --tail-bucket-mb")
    ap.add_argument("--tail-bucket-mb", type=float, default=4.0)
    ap.add_argument("--graph", choices=("auto", "on", "off"), default="auto",
                    help="--train: replay forward + backward as a CUDA graph (auto: on one GPU; "
                         "on: also with the gradient all-reduce captured)")
    return ap.parse_args()


def peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["bf16_tflops"], p.get("bf16_tflops_sustained"), p["hbm_gbs"], "measured"
    except Exception:
        return 1590.0, 1400.0, 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms in the background."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, dev):
        self.dev = dev
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.dev), "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ncu summaries committed under profiles/: the dominant kernel of each config
PROFILE_OF = {
    "c3": ("attn_bwd_d64_kernel_B8H16L4096d64.md", "attn_bwd_d64_kernel"),
    "c4": ("attn_bwd_kernel_d128_B2H16L16384.md", "attn_bwd_kernel<128> (bf16)"),
    "c1": (None, "attn_bwd_kernel<64, split3>"),
    "c2": ("attn_bwd_kernel_split3_B8H8L1024d64.md", "attn_bwd_kernel<64, split3>"),
}


def traffic_from_profile(cfg_name):
    """DRAM bytes per backward launch from the committed ncu summary, or None."""
    fname = PROFILE_OF[cfg_name][0]
    if not fname:
        return None
    try:
        for ln in open(os.path.join(REPO, "profiles", fname)):
            if ln.startswith("traffic_bytes_per_launch:"):
                return float(ln.split(":", 1)[1].strip())
    except OSError:
        pass
    return None


def make_host_inputs(torch, cfg, seed, b0, b1):
    """Q, K, V, dO for batches [b0, b1): seeded N(0,1)*0.5 (bf16 or fp32), on the host."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    dt = torch.bfloat16 if cfg.dtype == "bf16" else torch.float32
    ts = [(torch.randn(b1 - b0, cfg.L, cfg.H, cfg.D, generator=g) * 0.5).to(dt) for _ in range(4)]
    return [t.contiguous() for t in ts]


def _cpu_sample_shape(cfg):
    """(units, L, D) of the CPU sample: whole (batch, head) units of the config;
    for L=16384 units of L=4096 (a unit at full length takes ~a minute of CPU)."""
    L = cfg.L if cfg.L <= 4096 else 4096
    return L, cfg.D


def cpu_baseline(cfg, budget_s=12.0):
    """Time the multithreaded fp32 CPU attention (oracle/libcpuattn*.so) on a
    bounded sample of the same workload: whole (batch, head) units at the
    config's head dim, one unit per thread, repeated until ~budget_s."""
    import numpy as np
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle  # noqa: E402  (CPU baseline leg only)
    nth = oracle.cpu().cpu_hardware_threads()
    L, D = _cpu_sample_shape(cfg)
    units = min(max(1, nth), cfg.B * cfg.H)
    rng = np.random.default_rng(0)
    q, k, v, g = ((rng.standard_normal((units, L, 1, D)) * 0.5).astype(np.float32) for _ in range(4))
    outs = (np.zeros((units, L, 1, D), np.float32), np.zeros((units, L), np.float32),
            np.zeros((units, L, 1, D), np.float32), np.zeros((units, L, 1, D), np.float32),
            np.zeros((units, L, 1, D), np.float32))
    t0 = time.perf_counter()
    reps = 0
    while True:
        *_, used = oracle.cpu_attn_fwd_bwd(q, k, v, g, nthreads=nth, outs=outs)
        reps += 1
        if time.perf_counter() - t0 > budget_s / 2 or reps >= 64:
            break
    dt = time.perf_counter() - t0
    flops = 14.0 * reps * units * L * L * D
    note = "" if L == cfg.L else f" (units of L={L}: the rate per FLOP, not the full L={cfg.L})"
    return {"value": flops / dt / 1e12, "unit": "TFLOPS", "cores": int(used), "kind": "port",
            "isa": oracle.cpu_isa(),
            "sample": f"{reps} x {units} (batch, head) units of L={L} d={D} fwd+bwd, fp32, "
                      f"{dt:.1f} s wall on {used} threads{note}"}


def run_reference_arm(args):
    """--impl reference: the multithreaded CPU implementation of the same
    fwd+bwd on the host cores (the reference's own path is CUDA-only). Each
    step is a stated subset of the config's (batch, head) units."""
    import sharding
    rank, world, _ = sharding.dist_env()
    if rank != 0:
        return 0
    if args.ref_kernels:
        return run_reference_kernels(args)
    import numpy as np
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle  # noqa: E402  (reference arm)
    cfg = CONFIGS[args.config]
    nth = oracle.cpu().cpu_hardware_threads()
    L, D = _cpu_sample_shape(cfg)
    rng = np.random.default_rng(1)
    units = min(max(1, nth), cfg.B * cfg.H)
    q, k, v, g = ((rng.standard_normal((units, L, 1, D)) * 0.5).astype(np.float32) for _ in range(4))
    outs = (np.zeros((units, L, 1, D), np.float32), np.zeros((units, L), np.float32),
            np.zeros((units, L, 1, D), np.float32), np.zeros((units, L, 1, D), np.float32),
            np.zeros((units, L, 1, D), np.float32))
    for _ in range(min(args.warmup, 1)):
        oracle.cpu_attn_fwd_bwd(q, k, v, g, nthreads=nth, outs=outs)
    times = []
    used = nth
    for _ in range(args.steps):
        t0 = time.perf_counter()
        *_, used = oracle.cpu_attn_fwd_bwd(q, k, v, g, nthreads=nth, outs=outs)
        times.append(time.perf_counter() - t0)
    dt = sum(times)
    flops = 14.0 * units * L * L * D * args.steps
    val = flops / dt / 1e12
    frac = units * L * L / (cfg.B * cfg.H * cfg.L * cfg.L)
    what = ("the whole step" if frac == 1.0 else
            f"SUBSET: {units} of the {cfg.B * cfg.H} (batch, head) units (L={L} d={D}, {frac:.3g} of "
            f"the FLOPs of one {cfg.label} step); TFLOPS is the rate over that subset")
    sample = f"each step: {what}; fwd+bwd in fp32 on {used} threads ({oracle.cpu_isa()})"
    line = {"metric": metric_of(cfg), "value": val, "unit": "TFLOPS", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * dt / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": config_dict(cfg, args.gpus, "weak"),
            "reference_runs_on": "rank 0's host cores only",
            "timed_subset": {"units_per_step": units, "of_units": cfg.B * cfg.H,
                             "seq_len": L, "flop_fraction_of_step": frac},
            "cpu_baseline": {"value": val, "unit": "TFLOPS", "cores": int(used), "kind": "port",
                             "sample": sample},
            "e2e": {"value": val, "unit": "TFLOPS", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def run_reference_kernels(args):
    """The reference's own fp32 SIMT CUDA kernels (compiled unmodified from its
    sources into oracle/_ref/libpa_ref.so) timed on the GPU with CUDA events:
    its forward at C1, C2's attention shape and C3 (bf16-rounded inputs upcast
    to fp32), its shipped d=32 backward at C1, and its d=64 backward template
    relaunched with in-bounds geometry at C2 and C3 (the shipped d=64 launch
    addresses shared memory past its allocation and is not run). Context
    numbers only: the reference arm of the contract is the CPU port."""
    import numpy as np
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle  # noqa: E402  (reference arm)
    if not oracle.ref_available():
        print(json.dumps({"impl": "reference", "unavailable":
                          "oracle/_ref/libpa_ref.so not built (needs the reference sources)"}))
        return 0
    rows = []
    for name in ("c1", "c2", "c3"):
        cfg = CONFIGS[name]
        rng = np.random.default_rng(11)
        shape = (cfg.B, cfg.L, cfg.H, cfg.D)
        q, k, v, g = (rng.standard_normal(shape).astype(np.float32) * (0.5 if name == "c3" else 1.0)
                      for _ in range(4))
        reps = 20 if name == "c1" else 2
        fwd_ms, bwd_ms = oracle.ref_time_flash(q, k, v, g, reps)
        f = cfg.flops()
        rows.append({"config": name, "shape": cfg.label.replace("bf16", "fp32 (bf16-rounded inputs)"),
                     "fwd_ms": round(fwd_ms, 4), "bwd_ms": round(bwd_ms, 4),
                     "step_ms": round(fwd_ms + bwd_ms, 4),
                     "tflops": round(f / ((fwd_ms + bwd_ms) * 1e-3) / 1e12, 4),
                     "backward": "shipped launch_flash_backward (d=32)" if cfg.D == 32 else
                                 "flash_attn_backward_kernel<64,16,64> relaunched with Bc=64 geometry",
                     "reps": reps})
    print(json.dumps({"impl": "reference", "metric": "reference CUDA kernels, attn fwd+bwd TFLOPS",
                      "unit": "TFLOPS", "kind": "reference GPU kernels (fp32 SIMT)", "rows": rows,
                      "note": "the reference's dQ is a debug stub; its backward time covers dK and dV"}),
          flush=True)
    return 0


def run_attention(args):
    import torch
    import pa_capi
    import sharding
    cfg = CONFIGS[args.config]
    rank, world, local = sharding.dist_env()
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    pa_capi.load()
    peak, peak_sus, hbm, peak_src = peaks()
    stream = torch.cuda.current_stream()
    # Weak scaling: every rank owns B x H units. Strong: the B batches are split.
    b0, b1 = (0, cfg.B) if args.scaling == "weak" else sharding.shard_batches(cfg.B, world, rank)
    Bl = b1 - b0
    flops_rank = cfg.flops(Bl)
    flops_bwd = 10 * Bl * cfg.H * cfg.L * cfg.L * cfg.D
    host = make_host_inputs(torch, cfg, sharding.rank_seed(1234, rank) if args.scaling == "weak" else 1234,
                            b0, b1)
    in_bytes = sum(t.numel() * t.element_size() for t in host)
    flush_l2 = in_bytes < L2_BYTES  # small configs: flush L2 before every timed step
    scrub = torch.empty(2 * L2_BYTES, dtype=torch.uint8, device=dev) if flush_l2 else None

    def alloc():
        ins = [t.to(dev) for t in host]
        o = torch.empty_like(ins[0])
        lse = torch.empty(Bl * cfg.H, cfg.L, dtype=torch.float32, device=dev)
        grads = [torch.empty_like(ins[0]) for _ in range(3)]
        return ins, o, lse, grads

    (q, k, v, g), o, lse, (dq, dk, dv) = alloc()
    desc = pa_capi.attn_desc(q)
    ws = torch.empty(pa_capi.attn_bwd_workspace_size(desc), dtype=torch.uint8, device=dev)
    fws_n = pa_capi.attn_fwd_workspace_size(desc)
    fws = torch.empty(fws_n, dtype=torch.uint8, device=dev) if fws_n else None

    def step(ins, o, lse, grads, s=None):
        pa_capi.attn_fwd(ins[0], ins[1], ins[2], o, lse, desc, stream=s, workspace=fws)
        pa_capi.attn_bwd(ins[0], ins[1], ins[2], o, ins[3], lse, *grads, ws, desc=desc, stream=s)

    for _ in range(max(3, args.warmup)):
        step((q, k, v, g), o, lse, (dq, dk, dv))
    torch.cuda.synchronize()
    if pa_capi.device_status() != 0:
        raise SystemExit("device status reports a timed-out wait during warm-up")

    # ---------------- device-timed region: K steps, per-kernel events on the launch stream
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    clocks = ClockSampler(local)
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.25)
    t_begin = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_begin.record(stream)
    for i in range(args.steps):
        if flush_l2:
            scrub.zero_()
        ev[i][0].record(stream)
        pa_capi.attn_fwd(q, k, v, o, lse, desc, workspace=fws)
        ev[i][1].record(stream)
        pa_capi.attn_bwd(q, k, v, o, g, lse, dq, dk, dv, ws, desc=desc)
        ev[i][2].record(stream)
    t_end.record(stream)
    torch.cuda.synchronize()
    barrier()
    if flush_l2:  # the steps alone, without the L2 scrubs between them
        elapsed_ms = sharding.max_over_ranks(sum(e[0].elapsed_time(e[2]) for e in ev), dev)
    else:
        elapsed_ms = sharding.max_over_ranks(t_begin.elapsed_time(t_end), dev)
    fwd_ms = sum(e[0].elapsed_time(e[1]) for e in ev) / args.steps
    bwd_ms = sum(e[1].elapsed_time(e[2]) for e in ev) / args.steps
    status = pa_capi.device_status()

    # ---------------- end to end through the C ABI from pinned host buffers
    pinned = [t.pin_memory() for t in host]
    dt_out = host[0].dtype

    def host_outs():
        shp = (Bl, cfg.L, cfg.H, cfg.D)
        return ([torch.empty(shp, dtype=dt_out).pin_memory(),
                 torch.empty(Bl * cfg.H, cfg.L, dtype=torch.float32).pin_memory()] +
                [torch.empty(shp, dtype=dt_out).pin_memory() for _ in range(3)])

    outs_h = [host_outs(), host_outs()]
    h2d = sum(t.numel() * t.element_size() for t in pinned)
    d2h = sum(t.numel() * t.element_size() for t in outs_h[0])
    e2e_steps = max(8, args.steps // 4)  # enough that the pipeline's fill and drain are a small share

    def results(o_, lse_, grads_):
        return [o_, lse_] + list(grads_)

    # PCIe alone: the step's H2D, then its D2H, each timed by itself
    def copy_rate(pairs, n=4):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for src, dst in pairs:
            dst.copy_(src, non_blocking=True)
        e0.record(stream)
        for _ in range(n):
            for src, dst in pairs:
                dst.copy_(src, non_blocking=True)
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n

    h2d_ms = copy_rate(list(zip(pinned, (q, k, v, g))))
    d2h_ms = copy_rate(list(zip(results(o, lse, (dq, dk, dv)), outs_h[0])))

    # serial: copy in, compute, copy out, all on the compute stream
    def serial_step():
        for src, dst in zip(pinned, (q, k, v, g)):
            dst.copy_(src, non_blocking=True)
        step((q, k, v, g), o, lse, (dq, dk, dv))
        for src, dst in zip(results(o, lse, (dq, dk, dv)), outs_h[0]):
            dst.copy_(src, non_blocking=True)

    serial_step()
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        serial_step()
    e1.record(stream)
    torch.cuda.synchronize()
    serial_ms = sharding.max_over_ranks(e0.elapsed_time(e1), dev) / e2e_steps

    # pipelined: H2D of step i+1 and D2H of step i-1 overlap step i's kernels
    # (separate copy streams, two device buffer sets; PCIe copies both ways at once)
    bufs = [((q, k, v, g), o, lse, (dq, dk, dv)), alloc()]
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    h2d_done = [torch.cuda.Event() for _ in range(2)]
    comp_done = [torch.cuda.Event() for _ in range(2)]
    d2h_done = [torch.cuda.Event() for _ in range(2)]

    def pipelined(n, first_event=None, last_event=None):
        for i in range(n):
            bi = i % 2
            ins, ob, lb, grads = bufs[bi]
            with torch.cuda.stream(s_in):
                if i >= 2:
                    s_in.wait_event(comp_done[bi])
                if i == 0 and first_event is not None:
                    first_event.record(s_in)
                for src, dst in zip(pinned, ins):
                    dst.copy_(src, non_blocking=True)
                h2d_done[bi].record(s_in)
            stream.wait_event(h2d_done[bi])
            if i >= 2:
                stream.wait_event(d2h_done[bi])
            step(ins, ob, lb, grads)
            comp_done[bi].record(stream)
            with torch.cuda.stream(s_out):
                s_out.wait_event(comp_done[bi])
                for src, dst in zip(results(ob, lb, grads), outs_h[bi]):
                    dst.copy_(src, non_blocking=True)
                d2h_done[bi].record(s_out)
        if last_event is not None:
            last_event.record(s_out)

    pipelined(2)
    torch.cuda.synchronize()
    barrier()
    p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    pipelined(e2e_steps, p0, p1)
    torch.cuda.synchronize()
    e2e_ms = sharding.max_over_ranks(p0.elapsed_time(p1), dev)
    clk = clocks.stop()  # sampled across the timed regions

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(cfg)

    barrier()
    if world > 1:
        torch.distributed.destroy_process_group()
    if rank != 0:
        return 0
    ms_step = elapsed_ms / args.steps
    total_flops = world * flops_rank if args.scaling == "weak" else cfg.flops()
    value = total_flops / (ms_step * 1e-3) / 1e12
    per_gpu = value / world
    e2e_val = total_flops * e2e_steps / (e2e_ms * 1e-3) / 1e12
    bwd_tflops = flops_bwd / (bwd_ms * 1e-3) / 1e12
    e2e_step_ms = e2e_ms / e2e_steps
    comp_ms = fwd_ms + bwd_ms
    bound = max((("h2d", h2d_ms), ("d2h", d2h_ms), ("kernels", comp_ms)), key=lambda x: x[1])[0]
    line = {
        "metric": metric_of(cfg),
        "value": round(value, 2),
        "unit": "TFLOPS",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": max(3, args.warmup),
        "ms_per_step": round(ms_step, 4),
        "higher_is_better": True,
        "scaling": args.scaling,
        "vs_baseline": None,
        "dtype": cfg.dtype,
        "data": "synthetic (seeded N(0,1)*0.5)",
        "config": config_dict(cfg, world, args.scaling),
        "per_gpu_tflops": round(per_gpu, 2),
        "frac_of_dense_peak": {"measured_bf16": round(per_gpu / peak, 4),
                               "measured_bf16_sustained": (round(per_gpu / peak_sus, 4)
                                                           if peak_sus else None),
                               "datasheet_2250": round(per_gpu / 2250.0, 4)},
        "fwd_ms": round(fwd_ms, 4),
        "bwd_ms": round(bwd_ms, 4),
        "flops_no_recompute_tflops": round(value * 12 / 14, 2),
        "roofline": {"bound": "tensor", "kernel": f"{PROFILE_OF[args.config][1]} "
                                                  "(pa_attn_bwd span: prep + main + dQ convert)",
                     "achieved": round(bwd_tflops, 2), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(bwd_tflops / peak, 4), "traffic": traffic_from_profile(args.config),
                     "peak_source": f"{peak_src} burst bf16 (cuBLAS)",
                     "algorithmic_flops_per_launch": flops_bwd},
        "cpu_baseline": cpu,
        "e2e": {"value": round(e2e_val, 2), "unit": "TFLOPS", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_step_ms, 4),
                "mode": "pipelined: H2D / kernels / D2H on three streams, two buffer sets; "
                        "D2H = O, LSE, dQ, dK, dV",
                "serial_ms_per_step": round(serial_ms, 4),
                "pcie_alone": {"h2d_ms": round(h2d_ms, 4), "h2d_gbs": round(h2d / (h2d_ms * 1e-3) / 1e9, 1),
                               "d2h_ms": round(d2h_ms, 4), "d2h_gbs": round(d2h / (d2h_ms * 1e-3) / 1e9, 1),
                               "slowest_leg": bound}},
        # per step: bf16 fwd 1 + bwd 3 (prep, main, dQ convert); fp32 adds 3 + 4 operand splits
        "gpu_launches": args.steps * (4 if cfg.dtype == "bf16" else 11),
        "clocks": clk,
        "device_status": status,
    }
    print(json.dumps(line), flush=True)
    return 0


def run_linear(args):
    """Projections of the pre-LN MHA block (B8 L1024 E512, fp32), forward + backward:
    pa_linear_fwd / pa_linear_bwd against pa_matmul + pa_bias_add + pa_split_last_dim and
    pa_concat_last_dim_grad + pa_bias_grad + pa_matmul_grad_x + pa_matmul_grad_w."""
    import torch
    import pa_capi
    torch.cuda.set_device(0)
    M, E = 8 * 1024, 512
    g = torch.Generator(device="cuda").manual_seed(7)
    rnd = lambda *s: torch.randn(*s, device="cuda", generator=g)
    x, wi, bi, wo, bo = rnd(M, E), rnd(E, 3 * E) * 0.04, rnd(3 * E), rnd(E, E) * 0.04, rnd(E)
    qkv = [torch.empty(M, E, device="cuda") for _ in range(3)]
    attn, out = rnd(M, E), torch.empty(M, E, device="cuda")
    d_qkv, d_out = [rnd(M, E) for _ in range(3)], rnd(M, E)
    dx, dwi, dbi = torch.zeros(M, E, device="cuda"), torch.zeros(E, 3 * E, device="cuda"), torch.zeros(3 * E, device="cuda")
    dat, dwo, dbo = torch.zeros(M, E, device="cuda"), torch.zeros(E, E, device="cuda"), torch.zeros(E, device="cuda")
    ws = torch.empty(max(pa_capi.linear_workspace_size(M, E, 3 * E),
                         pa_capi.matmul_workspace_size(M, 3 * E, E),
                         pa_capi.matmul_workspace_size(M, E, 3 * E)), dtype=torch.uint8, device="cuda")
    proj, dproj, tmp = torch.empty(M, 3 * E, device="cuda"), torch.zeros(M, 3 * E, device="cuda"), torch.empty(M, E, device="cuda")

    def fused():
        pa_capi.linear_fwd(x, wi, bi, qkv, M, E, 3 * E, ws)
        pa_capi.linear_fwd(attn, wo, bo, [out], M, E, E, ws)
        pa_capi.linear_bwd(attn, wo, [d_out], dat, dwo, dbo, M, E, E, ws)
        pa_capi.linear_bwd(x, wi, d_qkv, dx, dwi, dbi, M, E, 3 * E, ws)

    def unfused():
        pa_capi.matmul(x, wi, proj, M, 3 * E, E, ws)
        pa_capi.bias_add(proj, bi, proj, M, 3 * E)
        pa_capi.split_last_dim(proj, qkv, M, E)
        pa_capi.matmul(attn, wo, tmp, M, E, E, ws)
        pa_capi.bias_add(tmp, bo, out, M, E)
        pa_capi.bias_grad(d_out, dbo, M, E)
        pa_capi.matmul_grad_x(d_out, wo, dat, M, E, E, ws)
        pa_capi.matmul_grad_w(attn, d_out, dwo, M, E, E, ws)
        pa_capi.concat_last_dim_grad(d_qkv, dproj, M, E)
        pa_capi.bias_grad(dproj, dbi, M, 3 * E)
        pa_capi.matmul_grad_x(dproj, wi, dx, M, E, 3 * E, ws)
        pa_capi.matmul_grad_w(x, dproj, dwi, M, E, 3 * E, ws)

    def timed(fn, n):
        for _ in range(max(3, args.warmup)):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n

    res = {}
    for mode in ("split3", "bf16"):
        pa_capi.set_f32_math(mode)
        res[mode] = {name: round(timed(fn, args.steps), 4)
                     for name, fn in (("fused_ms", fused), ("unfused_ms", unfused))}
    flops = 2 * M * E * (3 * E + E) * 3  # fwd + dX + dW of both projections
    # the training step's projection shapes (M = 8 x 2048 tokens), bf16 math, against
    # cuBLAS on bf16 operands (no conversion, bf16 output) for scale
    pa_capi.set_f32_math("bf16")
    M5 = 16384
    c5 = []
    for IN, OUT in ((1024, 3072), (1024, 1024), (1024, 4096), (4096, 1024)):
        x5, w5, b5 = rnd(M5, IN), rnd(IN, OUT) * 0.03, rnd(OUT)
        y5, dy5 = torch.empty(M5, OUT, device="cuda"), rnd(M5, OUT)
        dx5, dw5 = torch.zeros(M5, IN, device="cuda"), torch.zeros(IN, OUT, device="cuda")
        ws5 = torch.empty(pa_capi.linear_workspace_size(M5, IN, OUT), dtype=torch.uint8, device="cuda")
        f5 = 2 * M5 * IN * OUT
        tf = timed(lambda: pa_capi.linear_fwd(x5, w5, b5, [y5], M5, IN, OUT, ws5), args.steps)
        tb = timed(lambda: pa_capi.linear_bwd(x5, w5, [dy5], dx5, dw5, None, M5, IN, OUT, ws5), args.steps)
        xb, wb = x5.bfloat16(), w5.bfloat16()
        tc = timed(lambda: torch.matmul(xb, wb), args.steps)
        c5.append({"in": IN, "out": OUT, "fwd_us": round(tf * 1e3, 1),
                   "fwd_tflops": round(f5 / (tf * 1e-3) / 1e12, 1), "bwd_us": round(tb * 1e3, 1),
                   "bwd_tflops": round(2 * f5 / (tb * 1e-3) / 1e12, 1),
                   "cublas_bf16_us": round(tc * 1e3, 1)})
    pa_capi.set_f32_math("split3")
    print(json.dumps({"metric": "MHA block projections fwd+bwd (B8 L1024 E512 fp32)", "unit": "ms",
                      "split3": res["split3"], "bf16": res["bf16"],
                      "speedup_split3": round(res["split3"]["unfused_ms"] / res["split3"]["fused_ms"], 3),
                      "fused_tflops_split3": round(flops / (res["split3"]["fused_ms"] * 1e-3) / 1e12, 1),
                      "training_step_projections_bf16_math": c5,
                      "steps": args.steps, "device_status": pa_capi.device_status()}))


TRAIN = dict(layers=6, embed=1024, heads=16, ffn=4096, seq=2048, batch=8)


def train_flops_per_gpu(layers, embed, heads, ffn, seq, batch):
    """Model FLOPs of one training step on one GPU: projections and FFN
    (fwd + dX + dW) plus attention fwd+bwd in the flash convention."""
    tokens = batch * seq
    gemm = 3 * 2 * tokens * (4 * embed * embed + 2 * embed * ffn)
    attn = 14 * batch * heads * seq * seq * (embed // heads)
    return layers * (gemm + attn)


def run_train(args):
    """Denoise training step (tests/main_denoise.py model, stacked) on N GPUs,
    one process each; weak scaling (8 sequences per GPU)."""
    import datetime
    import numpy as np
    import torch
    import sharding
    rank, world, local = sharding.dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    import denoise
    peak, peak_sus, _, peak_src = peaks()
    mb = lambda x: int(x * (1 << 20))
    graph = {"auto": None, "on": True, "off": False}[args.graph]
    tr = denoise.DenoiseTrainer(lr=1e-4, math="bf16", bucket_bytes=mb(args.bucket_mb), graph=graph,
                                tail_bytes=mb(args.tail_mb),
                                tail_bucket_bytes=mb(args.tail_bucket_mb) if args.tail_mb else None,
                                **TRAIN)
    lift = denoise.embedding(TRAIN["embed"], 5)
    rng = np.random.default_rng(5 + rank)
    data = [tuple(torch.from_numpy(a).pin_memory()
                  for a in denoise.denoise_batch(rng, TRAIN["batch"], TRAIN["seq"], lift))
            for _ in range(2)]

    def barrier():
        if dist is not None:
            dist.barrier()

    warm = max(3, args.warmup)
    for i in range(warm):  # both kinds of timed step
        tr.step(*data[i % 2])
        tr.step_resident()
    tr.train([data[j % 2] for j in range(warm)])
    tr.load(*data[0])
    torch.cuda.synchronize()
    import PureAttention as pa
    if pa.device_status() != 0:
        raise SystemExit("device status reports a timed-out wait during warm-up")

    def timed(fn, calls=None):
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(args.steps if calls is None else calls):
            fn(i)
        e1.record()
        torch.cuda.synchronize()
        barrier()
        return sharding.max_over_ranks(e0.elapsed_time(e1), dev)

    clocks = ClockSampler(local)
    clocks.start()
    ms_res = timed(lambda i: tr.step_resident())
    losses = []
    # e2e: the pipelined loop (H2D of batch i+1 overlaps step i, loss read one step later)
    ms_e2e = timed(lambda i: losses.extend(tr.train([data[j % 2] for j in range(args.steps)])),
                   calls=1)
    clk = clocks.stop()
    ms_ar = None
    if tr.reducer is not None:
        ms_ar = timed(lambda i: tr.reducer())
    # the same step with fp32-level products (side figure; one untimed step
    # first, which captures its graph on one GPU)
    tr.math = "split3"
    tr.step_resident()
    ms_split3 = timed(lambda i: tr.step_resident())
    status = pa.device_status()
    tr.release_graphs()
    if dist is not None:
        dist.destroy_process_group()
    if rank != 0:
        return 0
    tokens = world * TRAIN["batch"] * TRAIN["seq"]
    step_ms = ms_res / args.steps
    flops = train_flops_per_gpu(**TRAIN)
    tflops = flops / (step_ms * 1e-3) / 1e12
    e2e_step = ms_e2e / args.steps
    h2d = 2 * TRAIN["batch"] * TRAIN["seq"] * TRAIN["embed"] * 4
    print(json.dumps({
        "metric": "denoise training tokens/s (6 layers E1024 H16 FFN4096 N2048, 8 seq/GPU)",
        "value": round(tokens / (step_ms * 1e-3), 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": warm, "ms_per_step": round(step_ms, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16 products, fp32 accumulation; fp32 master weights, activations, grads, Adam",
        "data": "synthetic denoise sequences (4 sinusoids lifted by a fixed Linear(1->1024) + noise)",
        "config": {"workload": "denoise transformer training step", **TRAIN,
                   "global_batch": TRAIN["batch"] * world, "parallelism": "dp%d" % world,
                   "params": tr.num_parameters,
                   "cuda_graph": bool(tr.graph)},
        "model_tflops_per_gpu": round(tflops, 1),
        "model_flops_per_gpu_step": flops,
        "frac_of_sustained_peak": round(tflops / (peak_sus or peak), 4),
        "peak_source": "%s sustained bf16 (cuBLAS)" % peak_src,
        "allreduce_ms": None if ms_ar is None else round(ms_ar / args.steps, 3),
        "split3_ms_per_step": round(ms_split3 / args.steps, 3),
        "allreduce_bytes": None if tr.reducer is None else tr.reducer.nbytes,
        "allreduce_buckets": None if tr.reducer is None else {
            "count": len(tr.reducer.buckets), "bucket_mb": args.bucket_mb, "tail_mb": args.tail_mb,
            "tail_bucket_mb": args.tail_bucket_mb if args.tail_mb else None,
            "in_place": tr.reducer.inplace},
        "e2e": {"value": round(tokens / (e2e_step * 1e-3), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
                "ms_per_step": round(e2e_step, 3),
                "mode": "DenoiseTrainer.train: input copies on a side stream one step ahead, "
                        "loss read one step behind"},
        "loss_first_last": [round(losses[0], 5), round(losses[-1], 5)],
        "clocks": clk, "device_status": status}), flush=True)
    return 0


def run_kernels(args):
    """Each kernel family alone at a size whose inputs exceed L2, timed with
    CUDA events over `steps` launches after `warmup`: algorithmic bytes (or
    FLOPs) per launch over the mean launch time, against the measured peak.
    Also the small-case driver of the per-kernel ncu captures."""
    import ctypes
    import torch
    import pa_capi
    torch.cuda.set_device(0)
    lib = pa_capi.load()
    peak, _, hbm, peak_src = peaks()
    g = torch.Generator(device="cuda").manual_seed(17)
    rnd = lambda *s: torch.randn(*s, device="cuda", generator=g)
    steps, warm = max(1, args.steps), args.warmup

    def timed(fn):
        for _ in range(warm):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    rows = []

    def hbm_row(kernel, shape, nbytes, ms):
        gbs = nbytes / (ms * 1e-3) / 1e9
        rows.append({"kernel": kernel, "shape": shape, "bound": "hbm", "us": round(ms * 1e3, 2),
                     "algorithmic_bytes": int(nbytes), "achieved_gbs": round(gbs, 1),
                     "frac_of_hbm": round(gbs / hbm, 4)})

    # LayerNorm, rows of 1024 fp32 (the training step's width), 128 MiB per tensor
    M, N = 32768, 1024
    x, r, dy = rnd(M, N), rnd(M, N), rnd(M, N)
    gam, bet = 1 + 0.1 * rnd(N), 0.1 * rnd(N)
    y, s, dx = torch.empty_like(x), torch.empty_like(x), torch.zeros_like(x)
    mu, rs = torch.empty(M, device="cuda"), torch.empty(M, device="cuda")
    dg, db = torch.zeros(N, device="cuda"), torch.zeros(N, device="cuda")
    ws = torch.empty(pa_capi.layer_norm_bwd_workspace_size(M, N), dtype=torch.uint8, device="cuda")
    e = 4 * M * N
    hbm_row("ln_fwd_kernel", f"M{M} N{N} fp32", 2 * e + 8 * M,
            timed(lambda: pa_capi.layer_norm_fwd(x, gam, bet, y, mu, rs)))
    hbm_row("ln_fwd_kernel (residual add fused)", f"M{M} N{N} fp32", 4 * e + 8 * M,
            timed(lambda: pa_capi.add_layer_norm_fwd(x, r, s, gam, bet, y, mu, rs)))
    hbm_row("ln_bwd_kernel + ln_param_reduce_kernel", f"M{M} N{N} fp32", 3 * e + 8 * M,
            timed(lambda: pa_capi.layer_norm_bwd(dy, x, mu, rs, gam, dx, dg, db, ws)))
    hbm_row("ln_bwd_kernel (accumulate into dX) + reduce", f"M{M} N{N} fp32", 4 * e + 8 * M,
            timed(lambda: pa_capi.layer_norm_bwd(dy, x, mu, rs, gam, dx, dg, db, ws,
                                                 accumulate=True)))
    # backward of the residual add + LayerNorm: read dY, the sum and the sum's own
    # gradient, write both addends' gradients (overwritten)
    dr = torch.empty_like(x)
    hbm_row("add_ln_bwd_kernel + ln_param_reduce_kernel", f"M{M} N{N} fp32", 5 * e + 8 * M,
            timed(lambda: pa_capi.add_layer_norm_bwd(dy, r, x, mu, rs, gam, dx, dr, dg, db, ws)))
    del x, r, dy, y, s, dx, dr

    # projection backward with the ReLU mask at the FFN's first layer (bf16 math): the
    # dY gather with the bias-gradient sums (split_colsum_kernel) and the two GEMMs;
    # the ncu capture of this call isolates the gather
    pa_capi.set_f32_math("bf16")
    Mf, INf, OUTf = 16384, 1024, 4096
    xf, wf, yf, dyf = rnd(Mf, INf), rnd(INf, OUTf) * 0.03, rnd(Mf, OUTf).relu_(), rnd(Mf, OUTf)
    dxf, dwf, dbf = torch.zeros(Mf, INf, device="cuda"), torch.zeros(INf, OUTf, device="cuda"), \
        torch.zeros(OUTf, device="cuda")
    wsf = torch.empty(pa_capi.linear_workspace_size(Mf, INf, OUTf), dtype=torch.uint8, device="cuda")
    ms_f = timed(lambda: pa_capi.linear_relu_bwd(xf, wf, yf, dyf, dxf, dwf, dbf, Mf, INf, OUTf, wsf))
    fl_f = 2 * 2 * Mf * INf * OUTf
    rows.append({"kernel": "pa_linear_relu_bwd (split_colsum_kernel + bias_grad_kernel + split_planes x2 + "
                           "gemm_pair_kernel x2)",
                 "shape": f"{Mf}x{INf} -> {OUTf}, ReLU mask, bf16 products", "bound": "tensor",
                 "us": round(ms_f * 1e3, 2), "algorithmic_flops": fl_f,
                 "achieved_tflops": round(fl_f / (ms_f * 1e-3) / 1e12, 1),
                 "gather_algorithmic_bytes": 10 * Mf * OUTf})
    pa_capi.set_f32_math("split3")
    del xf, wf, yf, dyf, dxf, dwf, dbf, wsf

    # multi-tensor Adam over the training step's 75.6 M parameters (48 tensors of its shapes)
    shapes = [(1024, 3072), (3072,), (1024, 1024), (1024,), (1024, 4096), (4096,), (4096, 1024),
              (1024,)] * 6
    ps = [rnd(*sh) for sh in shapes]
    gs = [rnd(*sh) for sh in shapes]
    ms_, vs_ = [torch.zeros_like(t) for t in ps], [torch.zeros_like(t) for t in ps]
    arr = lambda ts: (ctypes.c_void_p * len(ts))(*[t.data_ptr() for t in ts])
    P, G, Mm, V = arr(ps), arr(gs), arr(ms_), arr(vs_)
    sizes = (ctypes.c_size_t * len(ps))(*[t.numel() for t in ps])
    n_par = sum(t.numel() for t in ps)
    st = torch.cuda.current_stream().cuda_stream

    def adam():
        rc = lib.pa_adam_step_multi(P, G, Mm, V, sizes, len(ps), 1e-4, 0.9, 0.999, 1e-8, 0.1, 0.001, st)
        assert rc == 0, rc

    hbm_row("adam_multi_kernel", f"{len(ps)} tensors, {n_par / 1e6:.1f} M params", 28 * n_par,
            timed(adam))
    del ps, gs, ms_, vs_

    # projection GEMM of the training step, fp32 tensors, bf16 products (includes the
    # operand conversion to bf16 planes)
    pa_capi.set_f32_math("bf16")
    Mg, IN, OUT = 16384, 1024, 3072
    xg, wg, bg = rnd(Mg, IN), rnd(IN, OUT) * 0.03, rnd(OUT)
    yg = torch.empty(Mg, OUT, device="cuda")
    wsg = torch.empty(pa_capi.linear_workspace_size(Mg, IN, OUT), dtype=torch.uint8, device="cuda")
    ms_g = timed(lambda: pa_capi.linear_fwd(xg, wg, bg, [yg], Mg, IN, OUT, wsg))
    fl = 2 * Mg * IN * OUT
    rows.append({"kernel": "split_planes_kernel x2 + gemm_pair_kernel (pa_linear_fwd)",
                 "shape": f"{Mg}x{IN} @ {IN}x{OUT} fp32 in/out, bf16 products", "bound": "tensor",
                 "us": round(ms_g * 1e3, 2), "algorithmic_flops": fl,
                 "achieved_tflops": round(fl / (ms_g * 1e-3) / 1e12, 1),
                 "frac_of_tensor_peak": round(fl / (ms_g * 1e-3) / 1e12 / peak, 4)})
    pa_capi.set_f32_math("split3")
    del xg, wg, yg, wsg

    # pa_attn_delta runs the backward's prep kernel alone, in its Delta-only form (no
    # extension tiles, no dQ-accumulator clear); inside pa_attn_bwd the same kernel also
    # writes those, and its share of the step is in the ncu launch list
    B, L, H, D = 8, 4096, 16, 64
    o_, do_ = (rnd(B, L, H, D).bfloat16() for _ in range(2))
    delta = torch.empty(B, L, H, device="cuda")
    hbm_row("attn_bwd_prep_kernel<64, bf16> (Delta only, pa_attn_delta)", f"B{B} L{L} H{H} d{D} bf16",
            2 * B * L * H * D * 2 + 4 * B * L * H,
            timed(lambda: pa_capi.attn_delta(do_, o_, delta)))
    print(json.dumps({"metric": "per-kernel achieved bandwidth / throughput (1 x B200)",
                      "peak_hbm_gbs": hbm, "peak_bf16_tflops": peak, "peak_source": peak_src,
                      "steps": steps, "warmup": warm, "rows": rows,
                      "device_status": pa_capi.device_status()}), flush=True)
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference_arm(args)
    if args.linear:
        return run_linear(args)
    if args.train:
        return run_train(args)
    if args.kernels:
        return run_kernels(args)
    return run_attention(args)


if __name__ == "__main__":
    sys.exit(main())
