"""Decode-GEMM benchmark on B200: the decode linears of a Qwen3-8B step.

One step = every decode linear of one Qwen3-8B decode step (36 layers x {fused QKV
4096->6144, o_proj 4096->4096, fused gate_up 4096->24576, down 12288->4096} + lm_head
4096->151936; 15.1 GB of distinct bf16 weights), run once for each decode batch M in
{1, 2, 4, 8, 16}. Weights ~ N(0, 0.02), activations ~ N(0, 1), synthetic (seeded).

Metric: decode-GEMM HBM TB/s = algorithmic bytes 2*(K*N + M*K + M*N) summed over the step's
GEMMs / device time. Every step streams 75 GB of distinct weights (5 x 15.1 GB), far more
than the 126 MB L2, so no timed GEMM finds its weight in L2.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Under torchrun (N > 1) every rank runs the same step on its own GPU (replicas only: the
single-GPU decode linears do not exchange data) and rank 0 prints the aggregate.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import torch  # noqa: E402

LAYERS = 36
HIDDEN = 4096
VOCAB = 151936
# (name, N, K) of one Qwen3-8B decoder layer's linears (32 Q + 8 KV heads x 128, MLP 12288).
LAYER_LINEARS = [("qkv", 6144, 4096), ("o_proj", 4096, 4096), ("gate_up", 24576, 4096),
                 ("down", 4096, 12288)]
LM_HEAD = ("lm_head", VOCAB, HIDDEN)
M_LIST = (1, 2, 4, 8, 16)
METRIC = "decode-GEMM HBM TB/s (Qwen3-8B decode linears, M=1..16)"
WORKLOAD = ("qwen3-8b decode linears: 36 layers x (QKV 4096x6144, o_proj 4096x4096, "
            "gate_up 4096x24576, down 12288x4096) + lm_head 4096x151936, once per M in 1,2,4,8,16")


def gemm_bytes(M, N, K):
    return 2 * (K * N + M * K + M * N)


def step_linears():
    """The (name, N, K, layer) list of one decode step's linears, in execution order."""
    out = []
    for layer in range(LAYERS):
        for name, N, K in LAYER_LINEARS:
            out.append((name, N, K, layer))
    out.append((*LM_HEAD, LAYERS))
    return out


def step_bytes(m_list):
    return sum(gemm_bytes(M, N, K) for M in m_list for (_, N, K, _) in step_linears())


# ---------------------------------------------------------------------------------------
# clocks sampled with nvidia-smi during the timed region
# ---------------------------------------------------------------------------------------
class ClockSampler:
    """SM clock and clock-event (throttle) reasons of one GPU, sampled every 10 ms by an NVML
    thread while the timed region runs (read-only queries; nothing is set). Without NVML it
    falls back to ``nvidia-smi -lms 200``."""
    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown", 0x8),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap", 0x4))
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int, period_s: float = 0.01):
        self.dev = device_index
        self.period = period_s
        self.rows = []          # (sm_mhz, reason bitmask)
        self.max_mhz = None
        self.source = None
        self._stop = None
        self._thread = None
        self._proc = None
        self._path = None

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        try:   # the CUDA device's PCI address names the same GPU under any device ordering
            pr = torch.cuda.get_device_properties(self.dev)
            bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.dev)

    def __enter__(self):
        import threading
        try:
            nv, h = self._nvml_handle()
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))
            get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons",
                                  getattr(nv, "nvmlDeviceGetCurrentClocksThrottleReasons", None))
            self._stop = threading.Event()

            def run():
                while True:
                    try:
                        self.rows.append((float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)),
                                          int(get_reasons(h))))
                    except Exception:
                        pass
                    if self._stop.wait(self.period):
                        break
            self._thread = threading.Thread(target=run, daemon=True)
            self._thread.start()
            self.source = f"nvml every {int(self.period * 1000)} ms"
        except Exception:
            fd, self._path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            try:
                self._proc = subprocess.Popen(
                    ["nvidia-smi", f"--id={self.dev}", f"--query-gpu={self.QUERY}",
                     "--format=csv,noheader,nounits", "-lms", "200"],
                    stdout=open(self._path, "w"), stderr=subprocess.DEVNULL)
                self.source = "nvidia-smi -lms 200"
            except Exception:
                self._proc = None
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=5)
        if self._proc is not None:
            self._proc.terminate()
            try:
                self._proc.wait(timeout=5)
            except Exception:
                self._proc.kill()

    def summary(self):
        names = [n for n, _, _ in self.REASONS]
        if self._path is not None:  # nvidia-smi rows
            try:
                for line in open(self._path):
                    parts = [p.strip() for p in line.split(",")]
                    if len(parts) >= 9 and parts[1].replace(".", "").isdigit():
                        mask = sum(bit for i, (_, _, bit) in enumerate(self.REASONS)
                                   if parts[5 + i] == "Active")
                        self.rows.append((float(parts[1]), mask))
                        if parts[2].replace(".", "").isdigit():
                            self.max_mhz = max(self.max_mhz or 0.0, float(parts[2]))
            except Exception:
                pass
            finally:
                try:
                    os.unlink(self._path)
                except Exception:
                    pass
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"],
                    "samples": 0, "source": self.source}
        try:
            import pynvml as nv
            bits = [getattr(nv, attr, bit) for _, attr, bit in self.REASONS]
        except Exception:
            bits = [bit for _, _, bit in self.REASONS]
        reasons = sorted({names[i] for _, m in self.rows for i in range(4) if m & bits[i]})
        return {"sm_mhz": statistics.median(r[0] for r in self.rows), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.rows), "source": self.source}


# ---------------------------------------------------------------------------------------
# CPU baseline: the reference's own code path (torch.mm on bf16 CPU tensors, the call at
# engine/kernels/decode.py:54-66 and engine/engine.py:114) on the host cores
# ---------------------------------------------------------------------------------------
def cpu_sample_linears():
    """Bounded CPU sample: layer 0's four linears plus 1/36 of the lm_head rows."""
    return [(name, N, K) for name, N, K in LAYER_LINEARS] + [("lm_head/36", VOCAB // LAYERS, HIDDEN)]


def cpu_reference(m_list, budget_s=10.0, warmup=1):
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    from neokernel_b200 import synthetic
    lin = cpu_sample_linears()
    Ws = [synthetic.weight(N, K, seed=i) for i, (_, N, K) in enumerate(lin)]
    xs = {(M, K): synthetic.activation(M, K, seed=M) for M in m_list for (_, _, K) in lin}
    ys = {(M, N): torch.empty((M, N), dtype=torch.bfloat16) for M in m_list for (_, N, _) in lin}

    def one_pass():
        for M in m_list:
            for (_, N, K), W in zip(lin, Ws):
                torch.mm(xs[(M, K)], W.t(), out=ys[(M, N)])

    for _ in range(warmup):
        one_pass()
    bytes_pass = sum(gemm_bytes(M, N, K) for M in m_list for (_, N, K) in lin)
    passes, t0 = 0, time.perf_counter()
    while True:
        one_pass()
        passes += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    tbs = bytes_pass * passes / el / 1e12
    sample = (f"layer-0 QKV/o_proj/gate_up/down + lm_head rows 0..{VOCAB // LAYERS} "
              f"(1/36 of the vocabulary) at M in {list(m_list)}; {passes} passes in {el:.1f} s; "
              f"torch.mm bf16 on CPU (ATen), {threads} threads")
    return {"value": round(tbs, 6), "unit": "TB/s", "cores": threads, "kind": "reference",
            "sample": sample, "seconds_per_pass": el / passes,
            "cpu": _cpu_model()}


def cpu_config1(runs=200, warmup=20):
    """The reference's CPU path on the single decode linear of its first benchmark case:
    torch.mm(x, W.t()) with M=1, K=1024, N=3072 (the Qwen3-0.6B gate_proj shape), W bf16
    ~N(0, 0.02), x bf16 ~N(0, 1), seed 0, fp32 accumulation, bf16 output; median of ``runs``
    timed runs after ``warmup``, all host threads."""
    from neokernel_b200 import synthetic
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    M, K, N = 1, 1024, 3072
    W = synthetic.weight(N, K, seed=0)
    x = synthetic.activation(M, K, seed=0)
    y = torch.empty((M, N), dtype=torch.bfloat16)
    for _ in range(warmup):
        torch.mm(x, W.t(), out=y)
    ts = []
    for _ in range(runs):
        t0 = time.perf_counter()
        torch.mm(x, W.t(), out=y)
        ts.append(time.perf_counter() - t0)
    us = statistics.median(ts) * 1e6
    err = float((y.float() - torch.matmul(x.float(), W.float().t())).abs().max())
    return {"shape": "M=1 K=1024 N=3072", "runs": runs, "median_us": round(us, 2),
            "GB/s": round(gemm_bytes(M, N, K) / (us * 1e-6) / 1e9, 2), "threads": threads,
            "cpu": _cpu_model(), "max_abs_err_vs_fp32": err, "tolerance": 2e-2}


def _cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return None


# ---------------------------------------------------------------------------------------
# distributed plumbing (replicas only)
# ---------------------------------------------------------------------------------------
def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v, world, local):
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device=f"cuda:{local}")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def reference_arm(args):
    world, rank, _ = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")), 0
    if rank != 0:
        return 0
    m_list = tuple(int(m) for m in args.m_list.split(","))
    budget = max(2.0, min(20.0, 1.0 * max(args.steps, 1)))
    warm = cpu_reference(m_list, budget_s=0.5, warmup=max(1, min(args.warmup, 3)))
    base = cpu_reference(m_list, budget_s=budget, warmup=0)
    line = {
        "impl": "reference", "metric": METRIC, "value": base["value"], "unit": "TB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": base["seconds_per_pass"] * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": WORKLOAD, "m": list(m_list), "reference_path": "torch.mm (CPU, ATen)",
                   "sample": base["sample"]},
        "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": base["value"], "unit": "TB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "warm_value": warm["value"],
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------------
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--m-list", default=",".join(str(m) for m in M_LIST))
    ap.add_argument("--split", type=int, default=0, help="force split-K (0 = plan's choice)")
    ap.add_argument("--kind", type=int, default=0, help="force kernel family (0 = auto)")
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-decode", action="store_true",
                    help="skip the 36-layer Qwen3-8B decode-step tok/s measurement")
    ap.add_argument("--decode-batches", default="1,16")
    ap.add_argument("--decode-arms", default="all",
                    help="comma list of decode arms to time (default all; e.g. neokernel_b200)")
    ap.add_argument("--tp-decode", choices=("on", "off"), default="on",
                    help="Qwen3-32B tensor-parallel decode tok/s at TP = N (N = 1 is the "
                         "single-GPU anchor of the curve) with token parity against one GPU")
    ap.add_argument("--tp-batches", default="1,8,32")
    ap.add_argument("--single", default=None,
                    help="N,K,M: run one decode linear --reps times and exit (profiler captures)")
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--shapes", action="store_true",
                    help="per-shape table: every Qwen3-8B (M 1..16, verify 64..256) and Qwen3-0.6B "
                         "(M 1..16) decode linear chained 20x in a graph, weights rotated beyond "
                         "L2, ours and torch.mm (cuBLAS)")
    ap.add_argument("--split-sweep", action="store_true",
                    help="Qwen3-8B decode linears at M 1 and 16 with split-K forced to 1..16")
    ap.add_argument("--no-shapes", action="store_true",
                    help="leave the per-shape table (ours vs torch.mm) out of the bench line")
    ap.add_argument("--attention", default=None,
                    help="B,KV: run --reps Qwen3-8B decode-attention launches (32 query / 8 KV "
                         "heads, synthetic cache of KV positions) on cuda:0 and exit")
    ap.add_argument("--decode-step", type=int, default=0,
                    help="B: run --reps fused Qwen3-8B decode steps at batch B, KV 1024, and exit "
                         "(profiler captures of the whole step)")
    args = ap.parse_args()
    if args.impl == "reference":
        return reference_arm(args)
    if args.single:
        return single(args)
    if args.attention:
        return attention_only(args)
    if args.shapes:
        return shapes_table(args)
    if args.split_sweep:
        return split_sweep(args)
    if args.decode_step:
        return decode_step_only(args)
    if args.warmup < 3:
        print("warning: fewer than 3 warm-up steps", file=sys.stderr)

    world, rank, local = dist_setup()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    import neokernel_b200 as nk
    from neokernel_b200 import synthetic

    m_list = tuple(int(m) for m in args.m_list.split(","))
    lin = step_linears()

    # --- resident weights: 36 layers x 4 distinct matrices + lm_head (15.1 GB) ------------
    Ws = []
    for i, (name, N, K, layer) in enumerate(lin):
        Ws.append(synthetic.weight(N, K, seed=1000 * rank + i, device=dev))
    # activations and outputs per (M, K) / (M, N); contents are re-used across layers
    Ks = sorted({K for (_, _, K, _) in lin})
    Ns = sorted({N for (_, N, _, _) in lin})
    xs = {(M, K): synthetic.activation(M, K, seed=M * 31 + K, device=dev) for M in m_list for K in Ks}
    ys = {(M, N): torch.empty((M, N), dtype=torch.bfloat16, device=dev) for M in m_list for N in Ns}
    plans = {(M, N, K): nk.plan_for(M, N, K, kind=args.kind, split_k=args.split)
             for M in m_list for (_, N, K, _) in lin}

    stream = torch.cuda.Stream(device=dev)

    def run_m(M):
        for (name, N, K, layer), W in zip(lin, Ws):
            nk.mm(xs[(M, K)], W.t(), out=ys[(M, N)], plan=plans[(M, N, K)], stream=stream)

    # eager warm-up (sizes the workspace), then one graph per M
    stream.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(stream):
        for M in m_list:
            run_m(M)
    stream.synchronize()
    graphs = {}
    for M in m_list:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            run_m(M)
        graphs[M] = g
    torch.cuda.synchronize(dev)

    def step(evs=None):
        for i, M in enumerate(m_list):
            if evs is not None:
                evs[i][0].record(stream)
            graphs[M].replay()
            if evs is not None:
                evs[i][1].record(stream)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    stream.synchronize()

    launches_per_step = len(lin) * len(m_list)
    bytes_per_step = step_bytes(m_list)
    per_m_events = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                     for _ in m_list] for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    # --- timed region -------------------------------------------------------------------
    barrier(world)
    torch.cuda.synchronize(dev)
    with ClockSampler(local) as clk:
        with torch.cuda.stream(stream):
            start.record(stream)
            for s in range(args.steps):
                step(per_m_events[s])
            end.record(stream)
        end.synchronize()
    torch.cuda.synchronize(dev)
    barrier(world)
    ms = start.elapsed_time(end)
    ms_max = max_over_ranks(ms, world, local)
    clocks = clk.summary()
    value = bytes_per_step * args.steps * world / (ms_max / 1e3) / 1e12
    per_m = {}
    for i, M in enumerate(m_list):
        t = sum(per_m_events[s][i][0].elapsed_time(per_m_events[s][i][1]) for s in range(args.steps))
        b = sum(gemm_bytes(M, N, K) for (_, N, K, _) in lin) * args.steps
        per_m[str(M)] = {"TB/s": round(b / (t / 1e3) / 1e12, 4),
                         "us_per_step": round(t * 1e3 / args.steps, 1),
                         "tok_s_linears_only": round(M * args.steps / (t / 1e3), 1)}

    # --- roofline pass: every launch bracketed by events on the launching stream ----------
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    peak_gbs = peaks.get("hbm_gbs")
    peak_src = "measured" if peak_gbs else "fallback"
    peak_gbs = peak_gbs or 6650.0
    rl_steps = max(1, min(args.steps, 3))
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(rl_steps * launches_per_step)]
    kinfo = []
    torch.cuda.synchronize(dev)
    with torch.cuda.stream(stream):
        j = 0
        for _ in range(rl_steps):
            for M in m_list:
                for (name, N, K, layer), W in zip(lin, Ws):
                    ev[j][0].record(stream)
                    nk.mm(xs[(M, K)], W.t(), out=ys[(M, N)], plan=plans[(M, N, K)], stream=stream)
                    ev[j][1].record(stream)
                    kinfo.append((plans[(M, N, K)].kind, plans[(M, N, K)].tile_m, gemm_bytes(M, N, K)))
                    j += 1
    torch.cuda.synchronize(dev)
    kt = [a.elapsed_time(b) for a, b in ev]
    # dominant kernel = the kernel instance (family, token tile) with the most device time
    fam_time, fam_bytes, fam_n = {}, {}, {}
    for (kind, tile_m, b), t in zip(kinfo, kt):
        key = (kind, tile_m)
        fam_time[key] = fam_time.get(key, 0.0) + t
        fam_bytes[key] = fam_bytes.get(key, 0) + b
        fam_n[key] = fam_n.get(key, 0) + 1
    top = max(fam_time, key=fam_time.get)
    iso_ms = fam_time[top] / fam_n[top]
    iso_bytes = fam_bytes[top] / fam_n[top]
    iso_gbs = iso_bytes / (iso_ms / 1e3) / 1e9
    # In the timed region every launch is this kernel (one plan family and token tile for
    # the whole step; the ncu launch list of the same command shows it as 100 % of kernel
    # time), so its average launch duration there is the region's device time over its
    # launches — chained as the decode step runs them, with programmatic dependent launch.
    region_kinds = {(p.kind, p.tile_m) for p in plans.values()}
    if region_kinds == {top}:
        avg_ms = ms / (args.steps * launches_per_step)
        avg_bytes = bytes_per_step / launches_per_step
        timing = ("timed region: CUDA events around the graph replays on the launching stream, "
                  "device time / launches (every launch in it is this kernel)")
    else:
        avg_ms, avg_bytes = iso_ms, iso_bytes
        timing = "each launch bracketed by CUDA events on its stream, eager"
    achieved_gbs = avg_bytes / (avg_ms / 1e3) / 1e9
    by_kind = {}
    for (M, N, K), p in plans.items():
        by_kind.setdefault(p.kind, 0)
        by_kind[p.kind] += 1
    kernel_name = {nk.KIND_TC: f"tc_kernel<{top[1]}> (tcgen05/TMEM, TMA ring, persistent)",
                   nk.KIND_GEMV: f"gemv_kernel<{top[1]},...> (CUDA cores)",
                   nk.KIND_GENERIC: "generic_kernel"}[top[0]]
    roofline = {"bound": "hbm", "achieved": round(achieved_gbs, 1), "peak": peak_gbs,
                "unit": "GB/s", "frac": round(achieved_gbs / peak_gbs, 4),
                "traffic": _traffic_per_launch(avg_bytes), "peak_source": f"{peak_src} hbm_gbs",
                "kernel": kernel_name, "share_of_kernel_time": round(fam_time[top] / sum(kt), 4),
                "avg_launch_us": round(avg_ms * 1e3, 2),
                "algorithmic_bytes_per_launch": int(avg_bytes), "timing": timing,
                "isolated": {"achieved": round(iso_gbs, 1), "frac": round(iso_gbs / peak_gbs, 4),
                             "avg_launch_us": round(iso_ms * 1e3, 2), "launches": fam_n[top],
                             "timing": "each launch bracketed by CUDA events, eager (no "
                                       "overlap with its neighbours)"}}

    # --- e2e through the public API with host buffers -------------------------------------
    e2e = None
    if not args.no_e2e:
        e2e = e2e_pass(nk, lin, Ws, m_list, plans, dev, stream, args, world, local)

    decode = None
    if not args.no_decode:
        decode = decode_bench(nk, dev, [int(b) for b in args.decode_batches.split(",")],
                              world, local, arms_filter=args.decode_arms)

    tp_decode = None
    if args.tp_decode == "on":
        tp_decode = tp_decode_bench(nk, dev, [int(b) for b in args.tp_batches.split(",")],
                                    world, rank, local)

    per_shape = None
    if world == 1 and not args.no_shapes:
        per_shape = shape_rows(dev, shape_cases())

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_reference(m_list, budget_s=args.cpu_budget)
        cpu["config1"] = cpu_config1()

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 4), "unit": "TB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_max / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations)",
            "config": {"workload": WORKLOAD, "m": list(m_list), "gemms_per_step": launches_per_step,
                       "algorithmic_bytes_per_step": bytes_per_step,
                       "l2": "inputs larger than L2: 15.1 GB of distinct weights per M pass",
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                       "timing": "CUDA graph replay per M, CUDA events on the launching stream",
                       "split_k": args.split or "plan", "kind": args.kind or "auto",
                       "plan_kinds": {str(k): v for k, v in by_kind.items()}},
            "per_m": per_m,
            "roofline": roofline,
            "cpu_baseline": ({k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample",
                                                   "config1")}
                             if cpu else None),
            "per_shape": per_shape,
            "e2e": e2e,
            "decode": decode,
            "tp_decode": tp_decode,
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    for g in graphs.values():
        del g
    graphs.clear()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


def single(args):
    """One decode linear y[M,N] = x[M,K] W[N,K]^T, launched --reps times on cuda:0 with the
    plan --kind/--split select (a small, self-contained case for ncu captures)."""
    import neokernel_b200 as nk
    from neokernel_b200 import synthetic
    N, K, M = (int(v) for v in args.single.split(","))
    dev = torch.device("cuda", 0)
    W = synthetic.weight(N, K, seed=1, device=dev)
    x = synthetic.activation(M, K, seed=2, device=dev)
    y = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    plan = nk.plan_for(M, N, K, kind=args.kind, split_k=args.split)
    for _ in range(args.reps):
        nk.mm(x, W.t(), out=y, plan=plan)
    torch.cuda.synchronize(dev)
    print(json.dumps({"single": [N, K, M], "reps": args.reps, "plan": plan.as_dict()}))
    return 0


QWEN3_0_6B_LINEARS = [("qkv", 4096, 1024), ("o_proj", 1024, 2048), ("gate_up", 6144, 1024),
                      ("down", 1024, 3072), ("lm_head", VOCAB, 1024)]


def shape_cases():
    """(model, linear, N, K, M) of every per-shape row: Qwen3-8B decode (M 1..16), Qwen3-8B
    tree verify (M 64..256), Qwen3-0.6B decode (M 1, 4, 8, 16)."""
    cases = [("qwen3-8b", name, N, K, M) for name, N, K in LAYER_LINEARS + [("lm_head", VOCAB, HIDDEN)]
             for M in (1, 2, 4, 8, 16)]
    cases += [("qwen3-8b verify", name, N, K, M) for name, N, K in LAYER_LINEARS for M in (64, 128, 256)]
    cases += [("qwen3-0.6b", name, N, K, M) for name, N, K in QWEN3_0_6B_LINEARS for M in (1, 4, 8, 16)]
    return cases


def shape_rows(dev, cases, reps=5, chain=20, cublas=True, split=0):
    """Per-shape decode-GEMM throughput as a decode step sees it: each (shape, M) launched
    ``chain`` times in one CUDA graph (programmatic dependent launch between neighbours) with
    its weight rotated over copies larger than 2 x L2, so every launch reads its weight from
    DRAM; the same for torch.mm (cuBLAS, the reference's GPU path at engine/kernels/decode.py:
    54-66) when ``cublas``. Rows carry us per launch, TB/s and the fraction of the measured HBM
    peak, and for the verify batches TFLOP/s against the measured bf16 peak."""
    import neokernel_b200 as nk
    from neokernel_b200 import synthetic
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        peaks = {}
    hbm = float(peaks.get("hbm_gbs", 6650.0)) * 1e9
    tflops = float(peaks.get("bf16_tflops", 1590.0)) * 1e12
    stream = torch.cuda.Stream(device=dev)
    weights, rows = {}, []

    def timed(call):
        with torch.cuda.stream(stream):
            for W in Ws:
                call(W)
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(chain):
                call(Ws[i % len(Ws)])
        for _ in range(2):
            g.replay()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(reps):
                g.replay()
            e1.record(stream)
        e1.synchronize()
        del g
        return e0.elapsed_time(e1) * 1e3 / (reps * chain)

    def stats(us, M, N, K, prefix=""):
        b = gemm_bytes(M, N, K)
        r = {prefix + "us": round(us, 2), prefix + "TB/s": round(b / (us * 1e-6) / 1e12, 3),
             prefix + "hbm_frac": round(b / (us * 1e-6) / hbm, 3)}
        if M >= 64:
            f = 2.0 * M * N * K
            r[prefix + "TFLOP/s"] = round(f / (us * 1e-6) / 1e12, 1)
            r[prefix + "tensor_frac"] = round(f / (us * 1e-6) / tflops, 3)
        return r

    for model, name, N, K, M in cases:
        if (N, K) not in weights:
            weights.clear()
            torch.cuda.empty_cache()
            copies = max(2, (2 * 126 * 2 ** 20) // (N * K * 2) + 2)
            weights[(N, K)] = [synthetic.weight(N, K, seed=i, device=dev) for i in range(copies)]
        Ws = weights[(N, K)]
        x = synthetic.activation(M, K, seed=M, device=dev)
        y = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
        if split < 0:
            # the balanced persistent schedule alone: the plan without its tile-aligned slices
            plan = nk.Plan(nk.m_bucket(M), N, K)
            plan.c.slices = 0
        else:
            plan = nk.plan_for(M, N, K, split_k=split)
        row = {"model": model, "linear": name, "N": N, "K": K, "M": M}
        row.update(stats(timed(lambda W: nk.mm(x, W.t(), out=y, plan=plan, stream=stream)), M, N, K))
        if cublas:
            row.update(stats(timed(lambda W: torch.mm(x, W.t(), out=y)), M, N, K, "cublas_"))
            row["speedup_vs_cublas"] = round(row["cublas_us"] / row["us"], 3)
        rows.append(row)
    weights.clear()
    torch.cuda.empty_cache()
    return {"rows": rows, "timing": f"CUDA graph of {chain} launches per shape and arm, {reps} "
            "replays, CUDA events; weights rotated over > 2 x L2",
            "peaks": {"hbm_gbs": hbm / 1e9, "bf16_tflops": tflops / 1e12}}


def shapes_table(args):
    """--shapes: the per-shape table (ours and torch.mm) as one JSON line."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    print(json.dumps({"shapes": shape_rows(dev, shape_cases())}))
    return 0


def split_sweep(args):
    """--split-sweep: the Qwen3-8B decode linears (M 1..16; gate_up and lm_head at M 1 and 16)
    and the Qwen3-0.6B layer linears (M 1, 4, 8, 16) with split-K forced to every value 1..16
    beside the plan's own schedule (split 0: tile-aligned where the plan has slices, else
    balanced) and the balanced schedule alone (split -1), us per launch as in shape_rows."""
    import neokernel_b200 as nk
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    cases = [("qwen3-8b", name, N, K, M) for name, N, K in LAYER_LINEARS
             if name in ("qkv", "o_proj", "down") for M in (1, 2, 4, 8, 16)]
    cases += [("qwen3-8b", name, N, K, M) for name, N, K in LAYER_LINEARS + [("lm_head", VOCAB, HIDDEN)]
              if name in ("gate_up", "lm_head") for M in (1, 16)]
    cases += [("qwen3-0.6b", name, N, K, M) for name, N, K in QWEN3_0_6B_LINEARS for M in (1, 4, 8, 16)]
    table, slices = {}, {}
    for _, name, N, K, M in cases:
        slices[f"{name} {N}x{K} M={M}"] = nk.plan_for(M, N, K).as_dict()["slices"]
    for split in range(-1, 17):
        for r in shape_rows(dev, cases, reps=3, cublas=False, split=split)["rows"]:
            table.setdefault(f"{r['model']} {r['linear']} M={r['M']}", {})[str(split)] = r["us"]
    print(json.dumps({"split_sweep_us": table, "plan_slices": slices,
                      "note": "split 0 = the plan's own schedule (tile-aligned with the plan's "
                      "slices, else balanced persistent); -1 = the balanced schedule alone "
                      "(slices cleared); 1..16 = one CTA per (tile, K slice)"}))
    return 0


def attention_only(args):
    """--reps launches of one Qwen3-8B layer's decode attention (32 query heads over 8 KV heads
    of 128) at batch B with KV positions cached (a small, self-contained case for ncu)."""
    from neokernel_b200 import decode_ops as ops
    from neokernel_b200 import synthetic
    B, kv = (int(v) for v in args.attention.split(","))
    dev = torch.device("cuda", 0)
    H, Hkv, D = 32, 8, 128
    cap = kv + 1
    kc = synthetic.activation(B * Hkv * cap, D, seed=3, device=dev).view(B, Hkv, cap, D)
    vc = synthetic.activation(B * Hkv * cap, D, seed=4, device=dev).view(B, Hkv, cap, D)
    q = synthetic.activation(B, H * D, seed=5, device=dev)
    out = torch.empty_like(q)
    ws = ops.attention_workspace(B, H, cap, dev)
    position = torch.tensor([kv], device=dev)
    for _ in range(args.reps):
        ops.attention_decode(q, kc, vc, position, out, ws, H, Hkv)
    torch.cuda.synchronize(dev)
    # partial + merge timed with CUDA events, L2 flushed (a 256 MB write) before each launch
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(20)]
    for e0, e1 in ev:
        flush.zero_()
        e0.record()
        ops.attention_decode(q, kc, vc, position, out, ws, H, Hkv)
        e1.record()
    torch.cuda.synchronize(dev)
    us = sorted(e0.elapsed_time(e1) * 1e3 for e0, e1 in ev)
    kv_bytes = 2 * B * Hkv * (kv + 1) * D * 2
    print(json.dumps({"attention": [B, kv], "reps": args.reps, "kv_bytes": kv_bytes,
                      "us_median_cold_l2": round(us[len(us) // 2], 2),
                      "tbs_cold_l2": round(kv_bytes / (us[len(us) // 2] * 1e-6) / 1e12, 3)}))
    return 0


REF_ENGINE_DIR = os.path.join(ROOT, "baseline", "_ref")


class _TorchWithMM:
    """The ``torch`` module as engine/kernels/decode.py resolves it, with ``mm`` bound to another
    implementation: the drop-in at the four linear call sites (decode.py:54,58,64,66) with the
    reference's source unchanged."""

    def __init__(self, mm):
        self.mm = mm

    def __getattr__(self, name):
        return getattr(torch, name)


def reference_engine():
    """The reference's own decode kernels (engine/kernels: DecodeBuffers.layer with its Triton
    norm, q/k-norm+RoPE+cache, split attention and SiLU kernels and its torch.mm linears),
    installed unmodified into baseline/_ref. Returns (modules, None) or (None, why not)."""
    if not os.path.isfile(os.path.join(REF_ENGINE_DIR, "kernels", "decode.py")):
        return None, "the reference engine is not installed in baseline/_ref"
    if REF_ENGINE_DIR not in sys.path:
        sys.path.insert(0, REF_ENGINE_DIR)
    try:
        import kernels.decode as rdecode
        import kernels.rmsnorm as rnorm
        import kernels.weights as rweights
    except Exception as e:  # report the exact import error in the bench line
        return None, f"import of the reference engine failed: {type(e).__name__}: {e}"
    return (rdecode, rweights, rnorm), None


def _module_layer(lw, d):
    """An object shaped like transformers' Qwen3DecoderLayer (the fields the reference's
    LayerWeights reads, engine/kernels/weights.py:8-29) over one of our random-init layers."""
    from types import SimpleNamespace as NS
    D = d.head_dim
    q_end, k_end = d.heads * D, d.heads * D + d.kv_heads * D
    lin = lambda w: NS(weight=w, out_features=w.shape[0])  # noqa: E731
    attn = NS(q_proj=lin(lw.qkv_weight[:q_end]), k_proj=lin(lw.qkv_weight[q_end:k_end]),
              v_proj=lin(lw.qkv_weight[k_end:]), o_proj=lin(lw.o_weight),
              q_norm=NS(weight=lw.q_norm), k_norm=NS(weight=lw.k_norm))
    I = d.intermediate
    mlp = NS(gate_proj=lin(lw.gate_up_weight[:I]), up_proj=lin(lw.gate_up_weight[I:]),
             down_proj=lin(lw.down_weight))
    return NS(self_attn=attn, mlp=mlp,
              input_layernorm=NS(weight=lw.input_norm, variance_epsilon=d.eps),
              post_attention_layernorm=NS(weight=lw.post_norm, variance_epsilon=d.eps))


class ReferenceEngineDecoder:
    """The reference engine's decode step, Engine.decode (engine/engine.py:100-117), driven on
    its own DecodeBuffers.layer (engine/kernels/decode.py:42-68) with its shipped CONFIG
    (fuse_norm_residual: carry_in/defer_out), its LayerWeights packing, cache_storage caches and
    norm_out, captured in one CUDA graph as Engine.capture_decode does (side-stream warm-up x3,
    engine/engine.py:119-129). Engine itself loads a checkpoint through transformers 4.51's
    StaticCache, so the step is driven directly, as the reference's own layer test drives
    DecodeBuffers.layer. DecodeBuffers has the Qwen3-4B widths built in (decode.py:27-37); for
    another hidden/MLP width its x/norm/branch/gate_up/product/activation buffers are
    re-allocated at that width, the only change. ``mm`` (default torch.mm, the reference as
    shipped) is what the five linear call sites resolve to."""

    def __init__(self, mods, w, batch, capacity, dev, mm=None):
        rdecode, rweights, rnorm = mods
        d = w.dims
        self.d, self.batch = d, batch
        self.mm = mm or torch.mm
        self.norm_out = rnorm.norm_out
        self.layers = [rweights.LayerWeights(_module_layer(lw, d)) for lw in w.layers]
        self.embed, self.final_norm, self.lm_head = w.embed, w.final_norm, w.lm_head
        buf = rdecode.DecodeBuffers(batch, capacity, dev)
        bf = dict(device=dev, dtype=torch.bfloat16)
        if d.hidden != buf.x.shape[1] or d.intermediate != buf.product.shape[1]:
            for name, width in (("x", d.hidden), ("norm", d.hidden), ("branch", d.hidden),
                                ("gate_up", 2 * d.intermediate), ("product", d.intermediate),
                                ("activation", d.intermediate)):
                setattr(buf, name, torch.empty(batch, width, **bf))
        self.buf = buf
        n = len(w.layers)
        self.k = [rdecode.cache_storage(batch, capacity, dev, "bhsd") for _ in range(n)]
        self.v = [rdecode.cache_storage(batch, capacity, dev, "bhsd") for _ in range(n)]
        from neokernel_b200 import qwen3
        self.cos, self.sin = qwen3.rope_tables(d, capacity, dev)
        self.position = torch.zeros((1,), device=dev, dtype=torch.int64)
        self.token_ids = torch.zeros((batch, 1), device=dev, dtype=torch.int64)
        self.flat_tokens = self.token_ids.view(batch)
        self.next_tokens = torch.zeros((batch, 1), device=dev, dtype=torch.int64)
        self.logits = torch.empty((batch, d.vocab), **bf)
        saved = rdecode.torch
        rdecode.torch = _TorchWithMM(self.mm) if mm is not None else torch
        try:
            stream = torch.cuda.Stream(device=dev)
            stream.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(stream):
                for _ in range(3):
                    self.decode()
            torch.cuda.current_stream(dev).wait_stream(stream)
            stream.synchronize()
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=stream):
                self.decode()
            torch.cuda.current_stream(dev).wait_stream(stream)
        finally:
            rdecode.torch = saved
        self.reset()

    def decode(self):
        buf = self.buf
        torch.index_select(self.embed, 0, self.flat_tokens, out=buf.x)
        for i, lw in enumerate(self.layers):
            buf.layer(lw, self.k[i], self.v[i], self.position, self.cos, self.sin,
                      carry_in=i > 0, defer_out=True)
        self.norm_out(buf.branch, self.final_norm, buf.norm, self.d.eps, buf.x, buf.x)
        self.mm(buf.norm, self.lm_head, out=self.logits)
        torch.argmax(self.logits, dim=-1, keepdim=True, out=self.next_tokens)

    def reset(self):
        for c in self.k + self.v:
            c.zero_()
        self.position.zero_()

    def step(self):
        self.graph.replay()
        self.token_ids.copy_(self.next_tokens)
        self.position.add_(1)

    def greedy(self, prompt, new_tokens):
        """Feed ``prompt`` [B, P] one token per step, then decode ``new_tokens`` greedily."""
        self.reset()
        B, P = prompt.shape
        out = torch.empty(B, new_tokens, dtype=torch.int64, device=prompt.device)
        for i in range(P):
            self.token_ids[:, 0].copy_(prompt[:, i])
            self.graph.replay()
            self.position.add_(1)
        self.token_ids.copy_(self.next_tokens)
        for j in range(new_tokens):
            out[:, j] = self.token_ids[:, 0]
            if j + 1 < new_tokens:
                self.step()
        return out


def _time_decoder(g, dev, kv, steps, warmup, world, local, vocab, B, seed):
    """ms per decode step of a graph decoder (ours or the reference engine's) at KV length kv."""
    gen = torch.Generator(device=dev).manual_seed(seed)
    caches = (g.st.k_cache + g.st.v_cache) if hasattr(g, "st") else (g.k + g.v)
    for c in caches:
        c.normal_(generator=gen)
    pos = g.st.position if hasattr(g, "st") else g.position
    tok = g.st.tokens if hasattr(g, "st") else g.flat_tokens
    pos.fill_(kv)
    tok.copy_(torch.randint(0, vocab, (B,), generator=gen, device=dev))
    for _ in range(warmup):
        g.step()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize(dev)
    a.record()
    for _ in range(steps):
        g.step()
    b.record()
    b.synchronize()
    ms = max_over_ranks(a.elapsed_time(b), world, local) / steps
    return {"ms_per_token_step": round(ms, 4), "tok_s": round(B * world / (ms / 1e3), 1)}


def decode_bench(nk, dev, batches, world, local, kv=1024, steps=20, warmup=3, arms_filter="all"):
    """Decode tokens/s of the full Qwen3-8B step (36 layers, decisive random init, CUDA graph)
    at KV length 1024. Arms:
    * neokernel_b200: the product — fused decode kernels, neokernel_b200.mm and the fused
      lm_head + argmax;
    * fused_ops_torch_mm: the same fused step with the linears on torch.mm (cuBLAS);
    * torch_ops_torch_mm: PyTorch non-linear ops and torch.mm;
    * reference_triton (N = 1): the reference engine's own decode step — its Triton kernels and
      torch.mm linears (ReferenceEngineDecoder);
    * reference_triton_nk_mm (N = 1): the same reference step with neokernel_b200.mm at its
      five linear call sites, the documented drop-in;
    and, at N = 1, greedy-token parity of the product against the reference engine, plus the
    Qwen3-4B widths the reference's DecodeBuffers has built in."""
    from neokernel_b200 import qwen3
    w = qwen3.Qwen3Weights(qwen3.QWEN3_8B, seed=7, device=dev)
    out = {"model": "qwen3-8b decisive random init, 36 layers, vocab 151936", "kv_length": kv,
           "steps": steps, "timing": "CUDA events around graph replays, max over ranks"}
    mods, why = reference_engine() if world == 1 else (None, "single-GPU comparison only")

    def ours(w, B, linear, fused, fused_head):
        return qwen3.GraphDecoder(w, B, kv + warmup + steps + 1, linear, device=dev,
                                  fused=fused, fused_head=fused_head)

    def ref_engine(w, B, mm=None):
        return ReferenceEngineDecoder(mods, w, B, kv + warmup + steps + 1, dev, mm=mm)

    arms = [("neokernel_b200", lambda w, B: ours(w, B, nk.mm, True, True)),
            ("fused_ops_torch_mm", lambda w, B: ours(w, B, torch.mm, True, False)),
            ("torch_ops_torch_mm", lambda w, B: ours(w, B, torch.mm, False, False))]
    ref_arms = [("reference_triton", lambda w, B: ref_engine(w, B)),
                ("reference_triton_nk_mm", lambda w, B: ref_engine(w, B, nk.mm))]

    def run_arms(w, arms, into):
        for name, make in arms:
            res = {}
            for B in batches:
                try:
                    g = make(w, B)
                except Exception as e:  # the reference engine's arms report why they failed
                    if not name.startswith("reference"):
                        raise
                    res = {"unavailable": f"{type(e).__name__}: {str(e)[:300]}"}
                    break
                res[str(B)] = _time_decoder(g, dev, kv, steps, warmup, world, local,
                                            w.dims.vocab, B, seed=B)
                del g
                torch.cuda.empty_cache()
            into[name] = res

    if arms_filter != "all":
        keep = set(arms_filter.split(","))
        arms = [a for a in arms if a[0] in keep]
        ref_arms = [a for a in ref_arms if a[0] in keep]
        if not ref_arms:
            mods, why = None, "not requested"
    run_arms(w, arms, out)
    if mods is None:
        for name, _ in ref_arms:
            out[name] = {"unavailable": why}
    else:
        run_arms(w, ref_arms, out)
        out["reference_engine_parity"] = _engine_parity(mods, w, nk, dev)
        del w
        torch.cuda.empty_cache()
        w4 = qwen3.Qwen3Weights(qwen3.QWEN3_4B, seed=7, device=dev)
        out4 = {"model": "qwen3-4b random init (tied embeddings), 36 layers: the widths the "
                         "reference's DecodeBuffers has built in"}
        run_arms(w4, arms[:1] + ref_arms, out4)
        out["qwen3_4b"] = out4
        del w4
    torch.cuda.empty_cache()
    return out


def _engine_parity(mods, w, nk, dev, batch=4, prompt_len=8, new=32):
    """Greedy tokens of the product step against the reference engine's own step (its Triton
    kernels and torch.mm) on the same weights and prompt."""
    from neokernel_b200 import qwen3
    cap = prompt_len + new
    gen = torch.Generator(device=dev).manual_seed(2026)
    prompt = torch.randint(0, w.dims.vocab, (batch, prompt_len), generator=gen, device=dev)
    ref = ReferenceEngineDecoder(mods, w, batch, cap, dev)
    t_ref = ref.greedy(prompt, new)
    del ref
    ours = qwen3.GraphDecoder(w, batch, cap, nk.mm, device=dev, fused=True, fused_head=True)
    t_ours = ours.greedy(prompt, new)
    del ours
    torch.cuda.synchronize(dev)
    eq = t_ours == t_ref
    first = [int((~eq[b]).nonzero()[0]) if not eq[b].all() else None for b in range(batch)]
    return {"tokens_equal": bool(eq.all()), "identical_tokens": int(eq.sum()),
            "tokens": batch * new, "batch": batch, "first_divergence": first,
            "arms": "neokernel_b200 product step vs the reference engine's DecodeBuffers.layer "
                    "step (Triton + torch.mm), same weights and prompt"}


def tp_decode_bench(nk, dev, batches, world, rank, local, kv=2048, steps=10, warmup=3):
    """Qwen3-32B-shaped tensor-parallel decode (64 layers, random init) over the N ranks of
    this run: QKV/gate_up split by column, o_proj/down by K with their fp32 partials summed
    across ranks, lm_head by vocabulary; one CUDA graph per batch; KV length 2048. The
    product ("auto") fuses each K-slice linear with the rank-order sum over NVLink peer memory
    (nk_gemm_bf16_allreduce) for batches up to 8 (NCCL's all-reduce above); at N > 1 the step
    with the unfused pair
    (mm_f32, nk_allreduce_bf16) and with NCCL's all-reduce are timed beside it. tok/s counts
    each sequence's token once (the ranks share one model)."""
    from neokernel_b200 import qwen3, tp
    d = qwen3.QWEN3_32B
    w = tp.TPWeights(d, seed=13, rank=rank, world=world, device=dev)
    arms = ("auto", "peer", "nccl") if world > 1 else ("auto",)
    # all ranks take every collective step below in the same order
    out = {}
    for collective in arms:
        res = {}
        for B in batches:
            g = qwen3.GraphDecoder(w, B, kv + warmup + steps + 1, nk.mm, device=dev,
                                   make_hooks=tp.make_hooks(w, collective=collective), fused=True)
            gen = torch.Generator(device=dev).manual_seed(100 + B)
            for c in g.st.k_cache + g.st.v_cache:
                c.normal_(generator=gen)
            g.st.position.fill_(kv)
            g.st.tokens.copy_(torch.randint(0, d.vocab, (B,), generator=torch.Generator(
                device=dev).manual_seed(B), device=dev))  # same tokens on every rank
            for _ in range(warmup):
                g.step()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            barrier(world)
            torch.cuda.synchronize(dev)
            a.record()
            for _ in range(steps):
                g.step()
            b.record()
            b.synchronize()
            ms = max_over_ranks(a.elapsed_time(b), world, local) / steps
            res[str(B)] = {"ms_per_token_step": round(ms, 3), "tok_s": round(B / (ms / 1e3), 1)}
            barrier(world)
            del g.graph  # NCCL-holding graph released before anything tears down the group
            del g
            torch.cuda.empty_cache()
        out[collective] = res
    del w
    torch.cuda.empty_cache()
    parity = _tp_parity(nk, dev, world, rank, local)
    return {"model": "qwen3-32b random-init, 64 layers, hidden 5120, MLP 25600, 64Q/8KV x 128",
            "tp": world, "kv_length": kv, "steps": steps, "batches": out["auto"],
            "tp_parity": parity,
            "batches_unfused_peer_allreduce": out.get("peer"),
            "batches_nccl_allreduce": out.get("nccl"),
            "collectives": "o_proj and down: each rank's K slice fused with the rank-order sum "
                           "over NVLink peer memory in one launch (nk_gemm_bf16_allreduce) for "
                           "batches up to 8 (mm_f32 + NCCL all-reduce above); the 'peer' arm "
                           "launches mm_f32 then "
                           "nk_allreduce_bf16, the 'nccl' arm mm_f32 then NCCL all-reduce; "
                           "lm_head: each shard's argmax in its launch (nk_gemm_bf16_argmax), "
                           "NCCL all-gather of (max, index); all captured in the CUDA graph"}


def _tp_parity(nk, dev, world, rank, local, layers=4, batch=4, prompt_len=8, new=24):
    """Greedy tokens of the tensor-parallel product step (this run's TP = N, fused kernels,
    collectives, per-shard greedy head) against the single-GPU product step of the same model
    — Qwen3-32B shapes with ``layers`` layers and the decisive init — decoded on every rank
    from the same prompt. ``tokens_equal`` holds only if it holds on every rank."""
    from neokernel_b200 import qwen3, tp
    d = qwen3.QWEN3_32B
    cap = prompt_len + new
    gen = torch.Generator(device=dev).manual_seed(4242)
    prompt = torch.randint(0, d.vocab, (batch, prompt_len), generator=gen, device=dev)
    full = qwen3.Qwen3Weights(d, seed=17, device=dev, layers=layers)
    one = qwen3.GraphDecoder(full, batch, cap, nk.mm, device=dev, fused=True, fused_head=True)
    t_one = one.greedy(prompt, new)
    del one, full
    shard = tp.TPWeights(d, seed=17, rank=rank, world=world, device=dev, layers=layers)
    g = qwen3.GraphDecoder(shard, batch, cap, nk.mm, device=dev, fused=True,
                           make_hooks=tp.make_hooks(shard))
    t_tp = g.greedy(prompt, new)
    torch.cuda.synchronize(dev)
    barrier(world)
    del g.graph  # a graph holding NCCL calls goes before anything tears the group down
    del g, shard
    torch.cuda.empty_cache()
    same = int((t_tp == t_one).sum())
    worst = -max_over_ranks(-float(same), world, local)  # min over ranks
    return {"tokens_equal": worst == batch * new, "identical_tokens_min_over_ranks": int(worst),
            "tokens": batch * new, "batch": batch, "layers": layers, "tp": world,
            "against": "the single-GPU product step of the same Qwen3-32B-shaped model "
                       "(decisive init), on every rank"}


def decode_step_only(args, kv=1024):
    """--reps graph replays of the fused Qwen3-8B decode step at batch --decode-step, KV 1024."""
    import neokernel_b200 as nk
    from neokernel_b200 import qwen3
    dev = torch.device("cuda", 0)
    B = args.decode_step
    w = qwen3.Qwen3Weights(qwen3.QWEN3_8B, seed=7, device=dev)
    g = qwen3.GraphDecoder(w, B, kv + args.reps + 1, nk.mm, device=dev, fused=True,
                           fused_head=True)
    g.st.position.fill_(kv)
    for _ in range(args.reps):
        g.step()
    torch.cuda.synchronize(dev)
    print(json.dumps({"decode_step": B, "reps": args.reps}))
    return 0


def _traffic_per_launch(avg_bytes):
    """DRAM bytes per launch from the committed ncu capture (profiles/traffic.txt), scaled to
    this run's average algorithmic bytes per launch; None when no capture is recorded."""
    path = os.path.join(ROOT, "profiles", "traffic.txt")
    try:
        for line in open(path):
            if line.startswith("dram_over_algorithmic"):
                return int(float(line.split()[1]) * avg_bytes)
    except Exception:
        pass
    return None


def e2e_pass(nk, lin, Ws, m_list, plans, dev, stream, args, world, local):
    """Same step through ``neokernel_b200.mm`` (eager), with each step's activations copied
    from pinned host memory to the device first and every result copied back after."""
    x_specs = [(M, K) for M in m_list for (_, N, K, _) in lin]
    y_specs = [(M, N) for M in m_list for (_, N, K, _) in lin]
    x_elems = sum(M * K for M, K in x_specs)
    y_elems = sum(M * N for M, N in y_specs)
    hx = torch.empty(x_elems, dtype=torch.bfloat16, pin_memory=True)
    hx.copy_(torch.randn(x_elems, dtype=torch.float32).to(torch.bfloat16))
    hy = torch.empty(y_elems, dtype=torch.bfloat16, pin_memory=True)
    dx = torch.empty(x_elems, dtype=torch.bfloat16, device=dev)
    dy = torch.empty(y_elems, dtype=torch.bfloat16, device=dev)
    xv, off = [], 0
    for M, K in x_specs:
        xv.append(dx[off:off + M * K].view(M, K))
        off += M * K
    yv, off = [], 0
    for M, N in y_specs:
        yv.append(dy[off:off + M * N].view(M, N))
        off += M * N
    calls = []
    i = 0
    for M in m_list:
        for (name, N, K, layer), W in zip(lin, Ws):
            calls.append((xv[i], W.t(), yv[i], plans[(M, N, K)]))
            i += 1

    def one():
        dx.copy_(hx, non_blocking=True)
        for x, wt, y, p in calls:
            nk.mm(x, wt, out=y, plan=p, stream=stream)
        hy.copy_(dy, non_blocking=True)

    with torch.cuda.stream(stream):
        for _ in range(max(1, min(args.warmup, 3))):
            one()
    stream.synchronize()
    steps = max(1, min(args.steps, 5))
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize(dev)
    with torch.cuda.stream(stream):
        a.record(stream)
        for _ in range(steps):
            one()
        b.record(stream)
    b.synchronize()
    ms = max_over_ranks(a.elapsed_time(b), world, local)
    return {"value": round(step_bytes(m_list) * steps * world / (ms / 1e3) / 1e12, 4),
            "unit": "TB/s", "h2d_bytes_per_step": 2 * x_elems, "d2h_bytes_per_step": 2 * y_elems,
            "steps": steps, "ms_per_step": round(ms / steps, 3),
            "path": "neokernel_b200.mm eager, pinned host buffers, cudaMemcpyAsync both ways"}


if __name__ == "__main__":
    sys.exit(main())
