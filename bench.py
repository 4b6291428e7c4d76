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
    ap.add_argument("--tp-decode", choices=("auto", "on", "off"), default="auto",
                    help="Qwen3-32B tensor-parallel decode tok/s (auto: only when N > 1)")
    ap.add_argument("--tp-batches", default="1,8,32")
    ap.add_argument("--single", default=None,
                    help="N,K,M: run one decode linear --reps times and exit (profiler captures)")
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--shapes", action="store_true",
                    help="per-shape table: every Qwen3-8B (M 1..16, verify 64..256) and Qwen3-0.6B "
                         "(M 1..16) decode linear chained 20x in a graph, weights rotated beyond L2")
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
                              world, local)

    tp_decode = None
    if args.tp_decode == "on" or (args.tp_decode == "auto" and world > 1):
        tp_decode = tp_decode_bench(nk, dev, [int(b) for b in args.tp_batches.split(",")],
                                    world, rank, local)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_reference(m_list, budget_s=args.cpu_budget)

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
            "cpu_baseline": ({k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")}
                             if cpu else None),
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


def shapes_table(args, reps=5, chain=20):
    """Per-shape decode-GEMM throughput as a decode step sees it: each (shape, M) launched
    `chain` times in one CUDA graph (programmatic dependent launch between neighbours) with
    its weight rotated over copies larger than 2 x L2, so every launch reads its weight from
    DRAM. Prints one JSON line: us per launch, TB/s and the fraction of the measured HBM peak;
    for the verify batches also TFLOP/s against the measured bf16 peak."""
    import neokernel_b200 as nk
    from neokernel_b200 import synthetic
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        peaks = {}
    hbm = float(peaks.get("hbm_gbs", 6650.0)) * 1e9
    tflops = float(peaks.get("bf16_tflops", 1590.0)) * 1e12
    cases = [("qwen3-8b", name, N, K, M) for name, N, K in LAYER_LINEARS + [("lm_head", VOCAB, HIDDEN)]
             for M in (1, 2, 4, 8, 16)]
    cases += [("qwen3-8b verify", name, N, K, M) for name, N, K in LAYER_LINEARS for M in (64, 128, 256)]
    cases += [("qwen3-0.6b", name, N, K, M) for name, N, K in QWEN3_0_6B_LINEARS for M in (1, 4, 8, 16)]
    rows = []
    stream = torch.cuda.Stream(device=dev)
    weights = {}
    for model, name, N, K, M in cases:
        if (N, K) not in weights:
            weights.clear()
            torch.cuda.empty_cache()
            copies = max(2, (2 * 126 * 2 ** 20) // (N * K * 2) + 2)
            weights[(N, K)] = [synthetic.weight(N, K, seed=i, device=dev) for i in range(copies)]
        Ws = weights[(N, K)]
        x = synthetic.activation(M, K, seed=M, device=dev)
        y = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
        plan = nk.plan_for(M, N, K)
        with torch.cuda.stream(stream):
            for W in Ws:
                nk.mm(x, W.t(), out=y, plan=plan, stream=stream)
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(chain):
                nk.mm(x, Ws[i % len(Ws)].t(), out=y, plan=plan, stream=stream)
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
        us = e0.elapsed_time(e1) * 1e3 / (reps * chain)
        b = gemm_bytes(M, N, K)
        row = {"model": model, "linear": name, "N": N, "K": K, "M": M, "us": round(us, 2),
               "TB/s": round(b / (us * 1e-6) / 1e12, 3), "hbm_frac": round(b / (us * 1e-6) / hbm, 3)}
        if M >= 64:
            f = 2.0 * M * N * K
            row["TFLOP/s"] = round(f / (us * 1e-6) / 1e12, 1)
            row["tensor_frac"] = round(f / (us * 1e-6) / tflops, 3)
        rows.append(row)
        del g
    print(json.dumps({"shapes": rows, "timing": f"CUDA graph of {chain} launches per shape, "
                      f"{reps} replays, CUDA events; weights rotated over > 2 x L2",
                      "peaks": {"hbm_gbs": hbm / 1e9, "bf16_tflops": tflops / 1e12}}))
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


def decode_bench(nk, dev, batches, world, local, kv=1024, steps=20, warmup=3):
    """Decode tokens/s of the full Qwen3-8B step (36 layers, random init, CUDA graph) at KV
    length 1024. Arms: the product (fused non-linear kernels, neokernel_b200.mm and the fused
    lm_head + argmax), the same
    fused step with the linears on torch.mm (cuBLAS, the reference's call), and the step with
    PyTorch non-linear ops and torch.mm."""
    from neokernel_b200 import qwen3
    w = qwen3.Qwen3Weights(qwen3.QWEN3_8B, seed=7, device=dev)
    out = {"model": "qwen3-8b random-init, 36 layers, vocab 151936", "kv_length": kv,
           "steps": steps, "timing": "CUDA events around graph replays, max over ranks"}
    arms = (("neokernel_b200", nk.mm, True), ("fused_ops_torch_mm", torch.mm, True),
            ("torch_ops_torch_mm", torch.mm, False))
    for name, linear, fused in arms:
        res = {}
        for B in batches:
            g = qwen3.GraphDecoder(w, B, kv + warmup + steps + 1, linear, device=dev,
                                   fused=fused, fused_head=linear is nk.mm)
            gen = torch.Generator(device=dev).manual_seed(B)
            for c in g.st.k_cache + g.st.v_cache:
                c.normal_(generator=gen)
            g.st.position.fill_(kv)
            g.st.tokens.copy_(torch.randint(0, qwen3.QWEN3_8B.vocab, (B,), generator=gen, device=dev))
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
            res[str(B)] = {"ms_per_token_step": round(ms, 4),
                           "tok_s": round(B * world / (ms / 1e3), 1)}
            del g
            torch.cuda.empty_cache()
        out[name] = res
    del w
    torch.cuda.empty_cache()
    return out


def tp_decode_bench(nk, dev, batches, world, rank, local, kv=2048, steps=10, warmup=3):
    """Qwen3-32B-shaped tensor-parallel decode (64 layers, random init) over the N ranks of
    this run: QKV/gate_up split by column, o_proj/down by K with their fp32 partials summed
    across ranks, lm_head by vocabulary; one CUDA graph per batch; KV length 2048. The
    product ("auto") sums the partials with the peer-memory all-reduce (nk_allreduce_bf16) for
    small batches and NCCL's all-reduce for large ones; at N > 1 the step with NCCL's
    all-reduce throughout is timed beside it. tok/s counts each sequence's token once (the
    ranks share one model)."""
    from neokernel_b200 import qwen3, tp
    d = qwen3.QWEN3_32B
    w = tp.TPWeights(d, seed=13, rank=rank, world=world, device=dev)
    arms = ("auto", "nccl") if world > 1 else ("auto",)
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
    return {"model": "qwen3-32b random-init, 64 layers, hidden 5120, MLP 25600, 64Q/8KV x 128",
            "tp": world, "kv_length": kv, "steps": steps, "batches": out["auto"],
            "batches_nccl_allreduce": out.get("nccl"),
            "collectives": "fp32 partials of o_proj and down summed across ranks, one bf16 "
                           "rounding: nk_allreduce_bf16 over NVLink peer memory (rank order) up "
                           "to 64K elements, NCCL all-reduce above; NCCL all-gather of (max, "
                           "index) for the vocab-split argmax; all captured in the CUDA graph"}


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
