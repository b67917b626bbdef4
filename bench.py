#!/usr/bin/env python3
"""Benchmark of the fused layer-op chain (the KernRT row-op hot path) on B200.

Workload: 65536 token rows = 16 sequences x 4096 through
the SmolLM2-1.7B block's row ops — bf16 embedding gather (vocab 49152, hidden
2048) -> RMSNorm -> RoPE on 32 Q + 32 KV heads of 64 (theta 1.3e5, positions
row % 4096) -> SwiGLU over 8192 -> residual add; f32 activations ~N(0, 1),
embedding ~N(0, 0.02) in bf16, norm weight 1 + N(0, 0.1), synthetic and seeded.
Rows are sharded contiguously over the ranks with no collective on the data
path (the only collectives are the timing barrier and max-reduction).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl kernrt|reference]

One JSON line on rank 0.  `value` is device-timed with inputs resident in HBM
(10.5 GB per step at N=1, far larger than L2, so no flush is needed); `e2e`
goes through the C ABI with pinned host buffers, copies included.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from kernrt_b200 import workloads as W  # noqa: E402

WL = W.SMOLLM2_17B_65K
METRIC = "layer-op chain throughput (token rows/s)"
UNIT = "rows/s"
FALLBACK_HBM_GBS = 6650.0


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="kernrt", choices=["kernrt", "reference"])
    p.add_argument("--e2e-steps", type=int, default=3)
    p.add_argument("--cpu-seconds", type=float, default=10.0)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--rows", type=int, default=0,
                   help="profiling only: run a smaller row count than the workload's")
    return p.parse_args()


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            return float(json.load(fh)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def profile_traffic(kernel: str):
    """DRAM bytes per row that ncu measured for `kernel` on a smaller capture of
    this workload (profiles/chain_smollm2-1.7b_traffic.json); traffic grows in
    proportion to rows, so it scales to this rank's launch by rows."""
    path = os.path.join(ROOT, "profiles", "chain_smollm2-1.7b_traffic.json")
    try:
        with open(path) as fh:
            d = json.load(fh)
        return float(d["kernels"][kernel]["dram_bytes_per_row"])
    except Exception:
        return None


class ClockSampler:
    """SM clocks and throttle reasons sampled through NVML every 20 ms during
    the timed region (nvidia-smi as the fallback)."""

    REASONS = [("hw_slowdown", "nvmlClocksEventReasonHwSlowdown", 0x8),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap", 0x4)]

    def __init__(self, cuda_index: int):
        self.cuda_index = cuda_index
        self.sm, self.max_sm, self.reasons = [], [], set()
        self._stop = threading.Event()
        self._t = None
        self._nvml = None
        self._h = None
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            self._nvml = pynvml
            props = torch.cuda.get_device_properties(cuda_index)
            bus = getattr(props, "pci_bus_id", None)
            if bus is not None:
                dom = getattr(props, "pci_domain_id", 0)
                dev = getattr(props, "pci_device_id", 0)
                self._h = pynvml.nvmlDeviceGetHandleByPciBusId(f"{dom:08x}:{bus:02x}:{dev:02x}.0")
            else:
                self._h = pynvml.nvmlDeviceGetHandleByIndex(cuda_index)
        except Exception:
            self._nvml = None

    def _sample_nvml(self):
        n = self._nvml
        self.sm.append(n.nvmlDeviceGetClockInfo(self._h, n.NVML_CLOCK_SM))
        self.max_sm.append(n.nvmlDeviceGetMaxClockInfo(self._h, n.NVML_CLOCK_SM))
        get = getattr(n, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            n.nvmlDeviceGetCurrentClocksThrottleReasons
        mask = get(self._h)
        for name, const, bit in self.REASONS:
            if mask & getattr(n, const, bit):
                self.reasons.add(name)

    def _sample_smi(self):
        out = subprocess.run(["nvidia-smi", f"--id={self.cuda_index}",
                              "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
                              "clocks_event_reasons.hw_thermal_slowdown,"
                              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                              "--format=csv,noheader,nounits"], capture_output=True, text=True,
                             timeout=5).stdout.strip().split(",")
        self.sm.append(float(out[0]))
        self.max_sm.append(float(out[1]))
        for (name, _, _), v in zip(self.REASONS, out[2:]):
            if v.strip().lower().startswith("active"):
                self.reasons.add(name)

    def _run(self):
        while not self._stop.is_set():
            try:
                self._sample_nvml() if self._nvml else self._sample_smi()
            except Exception:
                pass
            self._stop.wait(0.02)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        if not self.sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no clock samples"]}
        return {"sm_mhz": statistics.median(self.sm), "sm_max_mhz": max(self.max_sm),
                "reasons": sorted(self.reasons), "samples": len(self.sm),
                "source": "nvml" if self._nvml else "nvidia-smi"}


# ---------------------------------------------------------------------------------
# reference arm: KernRT's CPU path (the oracle port of its scalar loops)
# ---------------------------------------------------------------------------------

_CPU_TABLE = None


def cpu_table():
    """The full bf16 embedding table of the workload (vocab 49152 x 2048,
    ~N(0, 0.02), RNE to bf16), made once per process on the host."""
    global _CPU_TABLE
    if _CPU_TABLE is None:
        from oracle.oracle import f32_to_bf16_bits

        rng = np.random.default_rng(1)
        out = np.empty((WL.vocab, WL.dim), np.uint16)
        step = 4096
        for lo in range(0, WL.vocab, step):
            hi = min(WL.vocab, lo + step)
            out[lo:hi] = f32_to_bf16_bits(rng.standard_normal((hi - lo, WL.dim), dtype=np.float32)
                                          * np.float32(0.02))
        _CPU_TABLE = out
    return _CPU_TABLE


def cpu_sample_inputs(rows: int, seed: int = 5):
    """`rows` rows of the workload's inputs; token ids span the whole table.
    q/k/gate are updated in place by each pass, so pristine copies are kept
    (`*0`) and restored before every pass, outside the timing."""
    rng = np.random.default_rng(seed)
    d = dict(table=cpu_table(), vocab=WL.vocab,
             tokens=rng.integers(0, WL.vocab, rows).astype(np.int32),
             positions=WL.positions(0, rows).astype(np.uint64),
             w_att=(1 + 0.1 * rng.standard_normal(WL.dim)).astype(np.float32),
             q=rng.standard_normal((rows, WL.q_dim), dtype=np.float32),
             k=rng.standard_normal((rows, WL.kv_dim), dtype=np.float32),
             gate=rng.standard_normal((rows, WL.hidden), dtype=np.float32),
             up=rng.standard_normal((rows, WL.hidden), dtype=np.float32),
             resid=rng.standard_normal((rows, WL.dim), dtype=np.float32))
    for n in ("q", "k", "gate"):
        d[n + "0"] = d[n].copy()
    return d


def cpu_restore(d) -> None:
    for n in ("q", "k", "gate"):
        np.copyto(d[n], d[n + "0"])


def cpu_chain_once(d, threads: int) -> float:
    """One timed pass of the oracle chain over the sample (in place); the
    restore of q/k/gate before it is not timed.  Returns seconds."""
    from oracle import oracle

    cpu_restore(d)
    t0 = time.perf_counter()
    oracle.chain(dim=WL.dim, q_dim=WL.q_dim, kv_dim=WL.kv_dim, hidden=WL.hidden, head=WL.head,
                 eps=WL.eps, theta=WL.theta, positions=d["positions"], w_att=d["w_att"], q=d["q"],
                 k=d["k"], gate=d["gate"], up=d["up"], resid=d["resid"], tokens=d["tokens"],
                 table=(oracle.BF16, d["table"], None, d["vocab"]), threads=threads, in_place=True)
    return time.perf_counter() - t0


def host_cpu():
    """The host CPU as lscpu names it, with its online and usable cores."""
    model = "unknown"
    try:
        with open("/proc/cpuinfo") as fh:
            for line in fh:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    try:
        usable = len(os.sched_getaffinity(0))
    except AttributeError:
        usable = os.cpu_count()
    return {"model": model, "nproc_online": os.cpu_count(), "usable_cores": usable}


def cpu_chain_rate(threads: int, seconds: float, rows: int):
    """Rows/s of the oracle chain on `threads` host threads over a bounded
    sample: passes over the same input rows (restored before each pass) until
    `seconds` of timed work accumulate."""
    d = cpu_sample_inputs(rows)
    done, el = 0, 0.0
    while el < seconds:
        el += cpu_chain_once(d, threads)
        done += rows
    return done / el, done, el


def base_config(world: int) -> dict:
    """The workload both arms run (the same dict in both JSON lines)."""
    return {"workload": WL.name, "rows": WL.rows, "hidden": WL.dim, "q_heads": WL.n_heads,
            "kv_heads": WL.n_kv_heads, "head_dim": WL.head, "intermediate": WL.hidden, "vocab": WL.vocab,
            "rope_theta": WL.theta, "positions": "row % 4096",
            "parallelism": f"row-shard x{world}, no collective",
            "l2": "inputs 10.5 GB per step > 126 MB L2; no flush needed"}


def run_reference(args, rank, world):
    if rank != 0:
        return
    from oracle import oracle

    threads = oracle.max_threads()
    per_step_rows = threads * 256
    d = cpu_sample_inputs(per_step_rows)
    times = []
    for i in range(args.warmup + args.steps):
        t = cpu_chain_once(d, threads)
        if i >= args.warmup:
            times.append(t)
    value = per_step_rows * len(times) / sum(times)
    cpu = host_cpu()
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * sum(times) / len(times),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded; bf16 embedding ~N(0,0.02), activations ~N(0,1), random init)",
        "config": base_config(world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "threads": threads, "kind": "port",
                         "cpu": cpu,
                         "sample": f"{per_step_rows} rows of the {WL.rows}-row workload per step (ids over the "
                                   f"full {WL.vocab}-row table; q/k/gate restored before each step, untimed), "
                                   f"row-parallel over {threads} host threads (KernRT is Rust and cannot be "
                                   f"built here; the C restatement of its scalar loops runs)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------
# the CUDA arm
# ---------------------------------------------------------------------------------

def run_kernrt(args, rank, world, local):
    import torch

    import kernrt_b200
    from kernrt_b200.interop import as_torch

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device(f"cuda:{local}"))

    def barrier():
        if dist is not None:
            dist.barrier()

    # Host-side check between phases (never inside the timed steps): every
    # rank must reach the phase within a bounded time, or the run stops with
    # the missing ranks named before any of the phase's launches.
    watch = None
    if dist is not None:
        from kernrt_b200.ranks import StepWatch

        watch = StepWatch(dist.distributed_c10d._get_default_store(), rank, world, timeout_s=120.0)

    def phase(name):
        if watch is not None:
            watch.enter(name)

    def sum_over_ranks(v: float) -> float:
        if dist is None:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    def gather_over_ranks(v: float) -> list:
        if dist is None:
            return [v]
        t = torch.tensor([v], dtype=torch.float64, device=f"cuda:{local}")
        out = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(out, t)
        return [float(x.item()) for x in out]

    def max_over_ranks(v: float) -> float:
        if dist is None:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    total_rows = args.rows if args.rows > 0 else WL.rows
    lo, hi = W.shard_rows(total_rows, world, rank)
    R = hi - lo
    H, Q, KV, I = WL.dim, WL.q_dim, WL.kv_dim, WL.hidden
    b = kernrt_b200.CudaBackend(local)

    # embedding table: seeded normals on the device, RNE to bf16, uploaded once
    g = torch.Generator(device=f"cuda:{local}").manual_seed(1)
    table = (torch.randn(WL.vocab, H, device=f"cuda:{local}", generator=g) * 0.02).to(torch.bfloat16)
    b.prepare_embedding(kernrt_b200.BF16, table.view(torch.int16).cpu().numpy().view(np.uint16), None,
                        WL.vocab, H)
    del table
    gr = torch.Generator(device=f"cuda:{local}").manual_seed(100 + rank)
    w_att = (1 + 0.1 * torch.randn(H, device=f"cuda:{local}", generator=gr)).cpu().numpy()
    h = {n: b.alloc(R * w) for n, w in [("x", H), ("xb", H), ("q", Q), ("k", KV), ("gate", I),
                                         ("up", I), ("resid", H)]}
    for n, w in [("q", Q), ("k", KV), ("gate", I), ("up", I), ("resid", H)]:
        as_torch(b, h[n], (R, w), device=local).copy_(
            torch.randn(R, w, device=f"cuda:{local}", generator=gr))
    tokens = torch.randint(0, WL.vocab, (R,), device=f"cuda:{local}", generator=gr,
                           dtype=torch.int32).cpu().numpy()
    positions = WL.positions(lo, hi)
    h["tokens"] = b.upload_bytes(tokens)
    h["positions"] = b.upload_bytes(positions)
    h["w_att"] = b.upload(w_att)
    # SwiGLU writes gate in place, so repeating the step on its own output
    # drifts the values (toward subnormals, or overflow where |up| > 2); every
    # step starts from this pristine copy instead, restored outside the timing.
    h["gate0"] = b.alloc(R * I)
    torch.cuda.synchronize()
    b.copy(h["gate"], 0, h["gate0"], 0, R * I)
    b.rope_prepare(WL.theta, WL.head, WL.seq_len)
    chain = dict(rows=R, dim=H, q_dim=Q, kv_dim=KV, hidden=I, head_size=WL.head, eps=WL.eps,
                 theta=WL.theta, tokens=h["tokens"], positions=h["positions"], x=h["x"], xb=h["xb"],
                 w_att=h["w_att"], q=h["q"], k=h["k"], gate=h["gate"], up=h["up"], resid=h["resid"])
    stream = torch.cuda.ExternalStream(b.stream(), device=f"cuda:{local}")

    # ---- device-resident value: CUDA events around each step's launch on the
    # backend's stream; the gate restore before each step is outside them.
    def restore_gate():
        b.copy(h["gate0"], 0, h["gate"], 0, R * I)

    phase("warmup")
    for _ in range(max(3, args.warmup)):
        restore_gate()
        b.layer_chain(**chain)
    b.synchronize()
    phase("timed")
    barrier()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    t_region = time.perf_counter()
    launches0 = kernrt_b200.kernel_launches()
    with ClockSampler(local) as clk:
        for s, e in ev:
            restore_gate()
            s.record(stream)
            b.layer_chain(**chain)
            e.record(stream)
        b.synchronize()
    torch.cuda.synchronize()
    region_s = time.perf_counter() - t_region
    launches = int(sum_over_ranks(float(kernrt_b200.kernel_launches() - launches0)))
    # Per-kernel times: further steps of the same workload with the backend's
    # stage events, which record between the two launches (an event there
    # costs the step ~2 %, so the timed steps above run without them).  The
    # headline's rows (gathered bf16 embedding rows, hidden 2048) take the
    # two-pass norm stage: k_row_scales (the row scales), then k_stream_dyn
    # (the norm rows' writes, RoPE and SwiGLU).
    stage_kernel = {"norm": "k_row_scales", "stream": "k_stream_dyn", "fused": "k_chain"}
    b.stage_timing(True)
    for _ in range(min(args.steps, 20)):
        restore_gate()
        b.layer_chain(**chain)
    stages = {stage_kernel[k]: v for k, v in b.stage_times().items()}
    b.stage_timing(False)
    per_launch = [s.elapsed_time(e) for s, e in ev]  # ms
    rank_ms = gather_over_ranks(sum(per_launch))  # each rank's timed steps, device ms
    total_ms = max(rank_ms)
    value = total_rows * args.steps / (total_ms / 1000.0)
    bpr = WL.bytes_per_row()
    peak, peak_kind = peaks()
    # The roofline is the dominant kernel's: its algorithmic bytes per launch
    # over its own mean launch time, from the backend's stage events.
    stage_bytes = {stage_kernel[k]: v for k, v in WL.stage_bytes_per_row(two_pass=True).items()}
    dominant = max((k for k in stages if stages[k][1] > 0), key=lambda k: stages[k][0])
    dom_ms, dom_n = stages[dominant]
    dom_bytes = stage_bytes.get(dominant, bpr) * R
    achieved = dom_bytes / (dom_ms / dom_n / 1000.0) / 1e9
    tpr = profile_traffic(dominant)
    step_achieved = bpr * R / (statistics.mean(per_launch) / 1000.0) / 1e9

    # ---- end to end through the C ABI with pinned host buffers
    e2e = None
    if args.e2e_steps > 0:
        host_in = {n: torch.empty(R * w, dtype=dt, pin_memory=True)
                   for n, w, dt in [("tokens", 1, torch.int32), ("positions", 1, torch.int32),
                                    ("q", Q, torch.float32), ("k", KV, torch.float32),
                                    ("gate", I, torch.float32), ("up", I, torch.float32),
                                    ("resid", H, torch.float32)]}
        host_in["tokens"].copy_(torch.from_numpy(tokens))
        host_in["positions"].copy_(torch.from_numpy(positions))
        gh = torch.Generator(device=f"cuda:{local}").manual_seed(200 + rank)
        for n, w in [("q", Q), ("k", KV), ("gate", I), ("up", I), ("resid", H)]:
            host_in[n].copy_(torch.randn(R * w, device=f"cuda:{local}", generator=gh).cpu())
        host_out = {n: torch.empty(R * w, dtype=torch.float32, pin_memory=True)
                    for n, w in [("x", H), ("xb", H), ("q", Q), ("k", KV), ("gate", I)]}
        h2d = sum(t.numel() * t.element_size() for t in host_in.values())
        d2h = sum(t.numel() * t.element_size() for t in host_out.values())

        def e2e_step():
            b.layer_chain_host(rows=R, dim=H, q_dim=Q, kv_dim=KV, hidden=I, head_size=WL.head,
                               eps=WL.eps, theta=WL.theta,
                               tokens=host_in["tokens"].data_ptr(), positions=host_in["positions"].data_ptr(),
                               q_in=host_in["q"].data_ptr(), k_in=host_in["k"].data_ptr(),
                               gate_in=host_in["gate"].data_ptr(), up=host_in["up"].data_ptr(),
                               resid=host_in["resid"].data_ptr(), x_out=host_out["x"].data_ptr(),
                               xb_out=host_out["xb"].data_ptr(), q_out=host_out["q"].data_ptr(),
                               k_out=host_out["k"].data_ptr(), gate_out=host_out["gate"].data_ptr(),
                               w_att=h["w_att"])

        phase("e2e")
        e2e_step()
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.e2e_steps):
            e2e_step()
        e2e_s = max_over_ranks(time.perf_counter() - t0)
        e2e = {"value": total_rows * args.e2e_steps / e2e_s, "unit": UNIT,
               "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world,
               "steps": args.e2e_steps,
               "path": "kernrt_cuda_layer_chain_host on page-locked host buffers (row chunks; "
                       "H2D, kernels and D2H overlapped on three streams)"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, n, el = cpu_chain_rate(1, args.cpu_seconds, 256)
        cpu = {"value": rate, "unit": UNIT, "cores": 1, "threads": 1, "kind": "port", "cpu": host_cpu(),
               "sample": f"{n} rows ({el:.1f} s timed) of the {WL.rows}-row workload in passes of 256 rows "
                         f"(ids over the full {WL.vocab}-row table; q/k/gate restored before each pass, "
                         f"untimed), single thread: the C restatement of KernRT's scalar row-op loops "
                         f"(its cpu backend runs these single-threaded)"}

    clocks = clk.summary()
    config = base_config(world)
    if total_rows != WL.rows:
        config["rows"] = total_rows
    barrier()
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": max(3, args.warmup), "ms_per_step": total_ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded; bf16 embedding ~N(0,0.02), activations ~N(0,1), random init)",
            "config": config,
            "timing": {"rows_per_gpu": R,
                       "how": "CUDA events around each step's launch(es) on the backend's stream; gate "
                              "restored from a pristine device copy before each step, outside the events; "
                              "per-kernel times (roofline) from further steps with the backend's stage events",
                       "region_wall_s_incl_restores": region_s,
                       "per_rank_ms_per_step": [m / args.steps for m in rank_ms]},
            "roofline": {"bound": "hbm", "kernel": dominant, "achieved": achieved, "peak": peak,
                         "unit": "GB/s", "frac": achieved / peak, "peak_kind": peak_kind,
                         "traffic": None if tpr is None else tpr * R,
                         "algorithmic_bytes_per_launch": dom_bytes,
                         "launch_ms_mean": dom_ms / dom_n,
                         "stages": {k: {"ms_per_launch": v[0] / v[1], "launches": v[1],
                                        "algorithmic_bytes_per_launch": stage_bytes.get(k, 0) * R,
                                        "achieved_gbs": stage_bytes.get(k, 0) * R / (v[0] / v[1] / 1000.0) / 1e9}
                                    for k, v in stages.items() if v[1] > 0},
                         "step": {"bytes_per_row": bpr, "ms_mean": statistics.mean(per_launch),
                                  "ms_min": min(per_launch), "achieved_gbs": step_achieved,
                                  "frac": step_achieved / peak}},
            "e2e": e2e,
            "cpu_baseline": cpu,
            "clocks": clocks,
            "gpu_launches": launches,
            "impl": "kernrt",
        }
        print(json.dumps(line), flush=True)
    b.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse()
    rank, world, local = dist_env()
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    run_kernrt(args, rank, world, local)


if __name__ == "__main__":
    main()
