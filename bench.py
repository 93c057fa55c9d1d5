"""Benchmark: gated-DeltaNet prefill + fused gated RMSNorm on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 1|4]
    (N > 1: python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N ...)

One "step" is one layer call of the hot path on one batch: the chunked
gated-delta-rule prefill with its gated-RMSNorm epilogue, at BASELINE config 1
(B=1, S=1141, HQK=16, HV=32, d=128, bf16 q/k/v/z, fp32 g/beta/state, random
initial state) unless --config 4 (B=32, S=4096). Inputs are seeded synthetic
tensors with the configuration's distributions (the reference publishes no
dataset for this path). With N GPUs every rank runs its own batch (sharded by
batch, no collective on the data path; weak scaling), timed on the device with
CUDA events between barriers, max over ranks.

Prints ONE JSON line (rank 0): the metric of BASELINE.json, whole-job tokens/s,
plus ``roofline`` (the prefill kernel's algorithmic bytes / its CUDA-event
duration against the measured HBM copy bandwidth; config 1 runs the
cluster-split kernel, config 4 the one-CTA-per-head kernel), ``cpu_baseline`` (the
reference's own CPU implementation on this host's cores), ``e2e`` (the same
metric through the public API with pinned host buffers and host<->device
copies inside the timed region), ``clocks`` (NVML samples taken during the
timed region), ``gpu_launches`` and ``graph`` (the same launches replayed from
a CUDA graph of ``--graph-launches`` calls, so that host launch cost is
visible separately).

``--impl reference`` times the reference's CPU implementation of the path
(transformers ``torch_chunk_gated_delta_rule`` + ``Qwen3_5RMSNormGated``, the
oracle the reference's harness imports, kernels/harness/parity_test.py:22-26)
on this host's cores for the same metric and config; under torchrun only rank
0 runs it.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "qwen-drive-edge-orin_b200"))
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "gated-DeltaNet prefill tokens/s/GPU (S=1141, 1/2/4/8 B200) and % of roofline"
CONFIGS = {
    1: dict(B=1, T=1141, HQK=16, HV=32, seed=1,
            desc="config1: B=1 S=1141 HQK=16 HV=32 d=128, bf16 q/k/v/z, fp32 g/beta/state, "
                 "random s0 ~N(0,0.02), fused gated RMSNorm, one layer"),
    4: dict(B=32, T=4096, HQK=16, HV=32, seed=4,
            desc="config4: B=32 S=4096 HQK=16 HV=32 d=128, bf16, random s0, fused gated RMSNorm"),
}
L2_BYTES = 126 * 1024 * 1024
D = 128


def alg_bytes(B, T, HQK, HV, with_s0=True):
    """Algorithmic HBM bytes of one fused call (read once / write once):
    q,k (HQK*d*2 each) + v,z,y (HV*d*2 each) + g,beta (HV*4 each) per token,
    + s0 read and sf write (HV*d*d*4 each) per sequence."""
    per_tok = 2 * HQK * D * 2 + 3 * HV * D * 2 + 2 * HV * 4
    per_seq = (2 if with_s0 else 1) * HV * D * D * 4
    return B * T * per_tok + B * per_seq


def alg_flops(B, T, HV, C=64):
    """2 * (5 C d + 3 d^2 + C^2/3) FLOP per token per v-head."""
    return B * T * HV * 2 * (5 * C * D + 3 * D * D + C * C / 3)


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", 0)), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def load_traffic(config):
    """(per-launch DRAM bytes, kernel name) of the config's prefill kernel from the committed
    ncu summary, or (None, None)."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None, None
    d = json.loads(p.read_text())
    v = d.get(f"config{config}")
    return (None, None) if v is None else (float(v["dram_bytes_per_launch"]), v.get("kernel"))


# ----------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock, power and clock-event reasons with NVML in a thread."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, index, period=0.005):
        self.ok = False
        self.samples = []
        self.period = period
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.max_mhz = None

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((mhz, rs))
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.ok:
            self._stop = threading.Event()
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        if self.ok:
            self._stop.set()
            self._t.join()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        busy = [s for s in self.samples if not (s[1] & 0x1)] or self.samples
        mhz = statistics.median(s[0] for s in busy)
        bits = 0
        for s in busy:
            bits |= s[1]
        reasons = sorted(name for b, name in self.REASONS.items() if bits & b and b != 0x1)
        return {"sm_mhz": mhz, "sm_max_mhz": self.max_mhz, "reasons": reasons, "samples": len(busy)}


# ----------------------------------------------------------------- inputs
def make_host_inputs(cfg, device_gen=False):
    from gdn_b200.synthetic import make_inputs
    return make_inputs(cfg["B"], cfg["T"], cfg["HQK"], cfg["HV"], D, seed=cfg["seed"], dist="baseline",
                       with_s0=True)


def device_inputs_from_torch(cfg, device, seed):
    """Same distributions generated on the device (large configs)."""
    g = torch.Generator(device=device).manual_seed(seed)
    B, T, HQK, HV = cfg["B"], cfg["T"], cfg["HQK"], cfg["HV"]
    n = lambda *s: torch.randn(*s, device=device, generator=g)  # noqa: E731
    q = torch.nn.functional.normalize(n(B, T, HQK, D), dim=-1, eps=1e-6).bfloat16()
    k = torch.nn.functional.normalize(n(B, T, HQK, D), dim=-1, eps=1e-6).bfloat16()
    v, z = n(B, T, HV, D).bfloat16(), n(B, T, HV, D).bfloat16()
    beta = torch.sigmoid(n(B, T, HV))
    gg = -torch.nn.functional.softplus(n(B, T, HV))
    w = (1 + 0.1 * n(D)).bfloat16()
    s0 = n(B, HV, D, D) * 0.02
    return dict(q=q, k=k, v=v, g=gg, beta=beta, z=z, w=w, s0=s0)


def to_device(inp, device):
    bf = lambda x: torch.from_numpy(x).to(device).bfloat16()  # noqa: E731
    f = lambda x: torch.from_numpy(x).to(device)  # noqa: E731
    return dict(q=bf(inp.q), k=bf(inp.k), v=bf(inp.v), g=f(inp.g), beta=f(inp.beta), z=bf(inp.z), w=bf(inp.w),
                s0=f(inp.s0))


# ----------------------------------------------------------------- CPU reference
def cpu_reference_time(cfg, inp, reps=5, warm=2, max_seconds=20.0):
    """Median seconds per call of the reference's CPU implementation (transformers torch
    fallback + Qwen3_5RMSNormGated, all host threads) on the given inputs."""
    from oracle.torch_reference import reference_gated_prefill
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    t_args = reference_inputs(inp)
    for _ in range(warm):
        reference_gated_prefill(*t_args)
    times = []
    t_start = time.perf_counter()
    for _ in range(reps):
        t0 = time.perf_counter()
        reference_gated_prefill(*t_args)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_start > max_seconds:
            break
    return statistics.median(times), threads


def reference_inputs(inp):
    bf = lambda x: torch.from_numpy(x).bfloat16()  # noqa: E731
    f = torch.from_numpy
    return (bf(inp.q), bf(inp.k), bf(inp.v), f(inp.g), f(inp.beta), bf(inp.z), bf(inp.w), f(inp.s0))


def cpu_sample_inputs(cfg):
    """Bounded CPU sample: config 1 runs whole; config 4 runs one sequence of its batch."""
    from gdn_b200.synthetic import make_inputs
    B = cfg["B"] if cfg["B"] * cfg["T"] <= 8192 else 1
    inp = make_inputs(B, cfg["T"], cfg["HQK"], cfg["HV"], D, seed=cfg["seed"], dist="baseline", with_s0=True)
    return inp, B


# ----------------------------------------------------------------- main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", type=int, default=1, choices=sorted(CONFIGS))
    ap.add_argument("--e2e-steps", type=int, default=50)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--graph-launches", type=int, default=20,
                    help="launches captured in one CUDA graph for the graph timing (0: skip)")
    args = ap.parse_args()
    cfg = CONFIGS[args.config]
    B, T, HQK, HV = cfg["B"], cfg["T"], cfg["HQK"], cfg["HV"]
    warmup = max(3, args.warmup)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        return run_reference(args, cfg, world, rank, warmup)

    import gdn_b200
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        os.environ.setdefault("NCCL_DEBUG", "WARN")  # keep rank 0's stdout to the one JSON line
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)

    # inputs: rotate through enough copies that each step's working set was evicted from L2
    step_bytes = alg_bytes(B, T, HQK, HV)
    n_sets = max(1, math.ceil(3 * L2_BYTES / step_bytes)) if step_bytes < 3 * L2_BYTES else 1
    if B * T <= 65536:
        host_inp = make_host_inputs(cfg)
        base = to_device(host_inp, device)
    else:
        host_inp = None
        base = device_inputs_from_torch(cfg, device, cfg["seed"] + 1000 * rank)
    sets = [base] + [{k: v.clone() for k, v in base.items()} for _ in range(n_sets - 1)]
    outs = [(torch.empty_like(s["v"]), torch.empty(B, HV, D, D, device=device)) for s in sets]
    lib = gdn_b200.load_library()
    stream = torch.cuda.current_stream(device)
    ws = torch.zeros(256, dtype=torch.uint8, device=device)
    import ctypes
    vp = ctypes.c_void_p

    def launch(i, st=None):
        s, (y, sf) = sets[i % n_sets], outs[i % n_sets]
        st = stream if st is None else st
        rc = lib.deltanet_chunk_prefill_gated(vp(s["q"].data_ptr()), vp(s["k"].data_ptr()), vp(s["v"].data_ptr()),
                                              vp(s["g"].data_ptr()), vp(s["beta"].data_ptr()), vp(s["z"].data_ptr()),
                                              vp(s["w"].data_ptr()), 1e-6, vp(y.data_ptr()),
                                              vp(s["s0"].data_ptr()), vp(sf.data_ptr()), B, T, HV, HQK, D, D, 64,
                                              vp(ws.data_ptr()), 256, vp(st.cuda_stream))
        if rc != 0:
            raise RuntimeError(f"deltanet_chunk_prefill_gated returned {rc}")

    for i in range(warmup):
        launch(i)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        e0.record(stream)
        for i in range(args.steps):
            launch(i)
        e1.record(stream)
        torch.cuda.synchronize()
    ms_total = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([ms_total], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total = float(t.item())
        dist.barrier()
    torch.cuda.synchronize()
    status = gdn_b200.binding.read_status() if False else _status(lib, ws, stream)
    ms_step = ms_total / args.steps
    tokens_step = B * T
    value = world * tokens_step / (ms_step / 1e3)

    # the same launches replayed from a CUDA graph: what is left is GPU-side launch cost
    graph = None
    if args.graph_launches > 0:
        gl = args.graph_launches
        cap = torch.cuda.Stream(device)
        cap.wait_stream(stream)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=cap):
            for i in range(gl):
                launch(i, cap)
        g.replay()
        torch.cuda.synchronize()
        reps = max(3, min(50, args.steps // gl))
        ge0, ge1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ge0.record(stream)
        for _ in range(reps):
            g.replay()
        ge1.record(stream)
        torch.cuda.synchronize()
        ms_graph = ge0.elapsed_time(ge1)
        if dist:
            t = torch.tensor([ms_graph], device=device, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms_graph = float(t.item())
        us_call = ms_graph * 1e3 / (reps * gl)
        graph = {"launches_per_graph": gl, "replays": reps, "us_per_call": round(us_call, 2),
                 "tokens_per_s": round(world * tokens_step / (us_call / 1e6), 1)}
        del g

    # e2e through the public API: pinned host in, pinned host out, copies inside the timed region
    e2e = run_e2e(args, cfg, device, host_inp, base, world, dist)

    hbm_gbs, tf_burst, tf_sust, peak_kind = load_peaks()
    achieved_gbs = step_bytes / (ms_step / 1e3) / 1e9
    flops = alg_flops(B, T, HV)
    traffic, traffic_kernel = load_traffic(args.config)
    override = os.environ.get("GDN_B200_KERNEL", "auto")
    if override in ("fused", "split"):  # the launcher's kernel choice was overridden
        launched = "gdn::split::gdn_prefill_split_kernel" if override == "split" else "gdn::gdn_prefill_kernel"
        if traffic_kernel != launched:  # the committed traffic figure is another kernel's
            traffic, traffic_kernel = None, launched
    roofline ={"bound": "hbm", "achieved": round(achieved_gbs, 1), "peak": hbm_gbs, "unit": "GB/s",
                "frac": round(achieved_gbs / hbm_gbs, 4), "traffic": traffic,
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else peak_kind,
                "alg_bytes_per_launch": step_bytes, "alg_flops_per_launch": flops,
                "tflops_achieved": round(flops / (ms_step / 1e3) / 1e12, 1),
                "roofline_time_us": round(max(step_bytes / (hbm_gbs * 1e9), flops / (tf_burst * 1e12)) * 1e6, 2),
                "frac_of_roofline_time": round(max(step_bytes / (hbm_gbs * 1e9), flops / (tf_burst * 1e12))
                                               / (ms_step / 1e3), 4),
                "kernel": traffic_kernel}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sample, sb = cpu_sample_inputs(cfg)
        sec, threads = cpu_reference_time(cfg, sample)
        cpu = {"value": round(sb * T / sec, 1), "unit": "tokens/s", "cores": threads, "kind": "reference",
               "sample": f"{sb}x{T} tokens, HQK={HQK} HV={HV}: transformers torch_chunk_gated_delta_rule + "
                         f"Qwen3_5RMSNormGated on {threads} host threads, median of 5 after 2 warmups "
                         f"({sec * 1e3:.1f} ms/call)"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded, BASELINE distributions)",
            "config": {"workload": cfg["desc"], "global_batch": B * world, "seq_len": T,
                       "parallelism": f"batch-sharded x{world}, no collective on the data path",
                       "l2": f"inputs rotate over {n_sets} device copies ({n_sets * step_bytes / 2**20:.0f} MiB > 126 MiB L2)"},
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
            "clocks": clk.summary(), "gpu_launches": args.steps, "status_word": status, "graph": graph,
            "impl": "ours",
        }
        print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()


def _status(lib, ws, stream):
    import ctypes
    out = ctypes.c_int(0)
    lib.deltanet_read_status(ctypes.c_void_p(ws.data_ptr()), ctypes.byref(out), 0, ctypes.c_void_p(stream.cuda_stream))
    return out.value


def run_e2e(args, cfg, device, host_inp, base, world, dist):
    """Same metric through gdn_b200.chunk_prefill_gated with pinned host buffers: every step copies
    its inputs host->device, runs, and copies y and the final state back. Copies and compute run on
    three streams with two device buffer sets, so step i+1's inputs upload while step i computes and
    step i-1's outputs download (the PCIe directions and the kernel overlap)."""
    import gdn_b200
    B, T, HQK, HV = cfg["B"], cfg["T"], cfg["HQK"], cfg["HV"]
    pinned = {k: v.detach().to("cpu").pin_memory() for k, v in base.items()}
    nbuf = 2
    dev_sets = [{k: torch.empty_like(v) for k, v in base.items()} for _ in range(nbuf)]
    y_host = [torch.empty(tuple(base["v"].shape), dtype=torch.bfloat16).pin_memory() for _ in range(nbuf)]
    sf_host = [torch.empty(B, HV, D, D, dtype=torch.float32).pin_memory() for _ in range(nbuf)]
    h2d = sum(t.numel() * t.element_size() for t in pinned.values())
    d2h = y_host[0].numel() * 2 + sf_host[0].numel() * 4
    steps = max(3, args.e2e_steps if B * T <= 65536 else 3)
    s_in, s_cmp, s_out = (torch.cuda.Stream(device) for _ in range(3))
    ev_in = [torch.cuda.Event() for _ in range(nbuf)]
    ev_done = [torch.cuda.Event() for _ in range(nbuf)]
    ev_out = [torch.cuda.Event() for _ in range(nbuf)]
    outs = [None] * nbuf

    def step(i):
        j = i % nbuf
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_done[j])  # buffer set j no longer read by step i - nbuf
            for k, v in pinned.items():
                dev_sets[j][k].copy_(v, non_blocking=True)
            ev_in[j].record(s_in)
        with torch.cuda.stream(s_cmp):
            s_cmp.wait_event(ev_in[j])
            s_cmp.wait_event(ev_out[j])  # outputs of step i - nbuf already downloaded
            d = dev_sets[j]
            outs[j] = gdn_b200.chunk_prefill_gated(d["q"], d["k"], d["v"], d["g"], d["beta"], d["z"], d["w"], d["s0"])
            ev_done[j].record(s_cmp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev_done[j])
            y_host[j].copy_(outs[j][0], non_blocking=True)
            sf_host[j].copy_(outs[j][1], non_blocking=True)
            ev_out[j].record(s_out)

    for i in range(3):
        step(i)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s_in)
    for i in range(steps):
        step(i)
    s_in.wait_stream(s_out)
    e1.record(s_in)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([ms], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / steps
    return {"value": round(world * B * T / (ms_step / 1e3), 1), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": round(ms_step, 4), "steps": steps,
            "api": "gdn_b200.chunk_prefill_gated (ctypes -> deltanet_chunk_prefill_gated)",
            "pipelining": "3 streams, 2 device buffer sets (upload i+1 | compute i | download i-1)"}


def run_reference(args, cfg, world, rank, warmup):
    """The reference's CPU implementation of the path, timed on this host's cores (rank 0 only)."""
    if rank != 0:
        return
    B, T, HQK, HV = cfg["B"], cfg["T"], cfg["HQK"], cfg["HV"]
    sample, sb = cpu_sample_inputs(cfg)
    from oracle.torch_reference import reference_gated_prefill
    threads = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads)
    t_args = reference_inputs(sample)
    for _ in range(max(1, min(warmup, 3))):
        reference_gated_prefill(*t_args)
    steps = max(1, min(args.steps, 20))
    t0 = time.perf_counter()
    for _ in range(steps):
        reference_gated_prefill(*t_args)
    sec = (time.perf_counter() - t0) / steps
    value = sb * T / sec
    desc = (f"{sb}x{T} tokens, HQK={HQK} HV={HV}: transformers torch_chunk_gated_delta_rule + "
            f"Qwen3_5RMSNormGated on {threads} host threads ({sec * 1e3:.1f} ms/call)")
    line = {"metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": steps,
            "warmup": warmup, "ms_per_step": round(sec * 1e3, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp32", "data": "synthetic (seeded, BASELINE distributions)",
            "config": {"workload": cfg["desc"], "global_batch": B, "seq_len": T, "parallelism": "host CPU"},
            "impl": "reference",
            "cpu_baseline": {"value": round(value, 1), "unit": "tokens/s", "cores": threads, "kind": "reference",
                             "sample": desc},
            "e2e": {"value": round(value, 1), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
