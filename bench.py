"""Benchmark: gated-DeltaNet prefill + fused gated RMSNorm on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 1|3|4]
    (N > 1: python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N ...)

One "step" is one layer call of the hot path on one batch: the chunked
gated-delta-rule prefill with its gated-RMSNorm epilogue. The default workload
is BASELINE config 1 (B=1, S=1141, HQK=16, HV=32, d=128, bf16 q/k/v/z, fp32
g/beta/state, random initial state); ``--config 4`` is B=32, S=4096, and
``--config 3`` the long single stream (B=1, S=65536, zero initial state). Inputs
are seeded synthetic tensors with the configuration's distributions, drawn on
the device (the reference publishes no dataset for this path).

Sharding over N GPUs (one process per GPU, no collective on the data path):
config 1 gives every rank its own batch (weak scaling); config 4 splits the
batch of 32 (strong scaling); config 3 gives rank r the v-heads
[r*32/N, (r+1)*32/N) and the qk-heads they read, h // (HV/HQK) (strong
scaling). Time is measured on the device with CUDA events between barriers,
max over ranks. After the timed region every rank's y and final state are
gathered to rank 0 with NCCL all_gather, and rank 0 recomputes each rank's
shard on its own GPU and compares (``verification``).

Prints ONE JSON line (rank 0): the metric of BASELINE.json, whole-job tokens/s,
plus ``roofline`` (the prefill kernel's algorithmic bytes / its CUDA-event
duration against the measured HBM copy bandwidth), ``windows`` (the same
K-step window repeated, median and spread), ``cpu_baseline`` (the reference's
own CPU implementation on this host's cores), ``e2e`` (the same metric through
the public API with pinned host buffers and host<->device copies inside the
timed region), ``clocks`` (NVML samples taken during the timed windows),
``gpu_launches``, ``graph`` (config 1: the launches replayed from a CUDA graph)
and, on a default one-GPU run, ``config4`` (config 4 timed the same way).

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
    1: dict(B=1, T=1141, HQK=16, HV=32, seed=1, s0=True, shard="batch-weak",
            desc="config1: B=1 S=1141 HQK=16 HV=32 d=128, bf16 q/k/v/z, fp32 g/beta/state, "
                 "random s0 ~N(0,0.02), fused gated RMSNorm, one layer"),
    3: dict(B=1, T=65536, HQK=16, HV=32, seed=3, s0=False, shard="head",
            desc="config3: B=1 S=65536 HQK=16 HV=32 d=128, bf16, zero s0, fused gated RMSNorm; "
                 "v-heads split over the GPUs"),
    4: dict(B=32, T=4096, HQK=16, HV=32, seed=4, s0=True, shard="batch",
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
    """(per-launch memory traffic in bytes, kernel name) of the config's prefill kernel from the
    committed ncu summary, or (None, None): DRAM reads plus the writes the SMs send to L2 (the
    outputs are still in L2 when a launch ends, so DRAM write counters miss them)."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None, None
    d = json.loads(p.read_text())
    v = d.get(f"config{config}")
    return (None, None) if v is None else (float(v["traffic_bytes_per_launch"]), v.get("kernel"))


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

    def read_mhz(self):
        if not self.ok:
            return None
        try:
            return self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
        except Exception:
            return None

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


# ----------------------------------------------------------------- workloads
def device_inputs(B, T, HQK, HV, seed, device, with_s0=True):
    """BASELINE distributions drawn on the device with a seeded generator: q, k ~ N(0,1)
    L2-normalised in fp32 then bf16; v, z ~ N(0,1) bf16; beta = sigmoid(N(0,1));
    g = -softplus(N(0,1)); w = 1 + 0.1 N(0,1) bf16; s0 ~ N(0, 0.02) (or none)."""
    g = torch.Generator(device=device).manual_seed(seed)
    n = lambda *s: torch.randn(*s, device=device, generator=g)  # noqa: E731
    q = torch.nn.functional.normalize(n(B, T, HQK, D), dim=-1, eps=1e-6).bfloat16()
    k = torch.nn.functional.normalize(n(B, T, HQK, D), dim=-1, eps=1e-6).bfloat16()
    v, z = n(B, T, HV, D).bfloat16(), n(B, T, HV, D).bfloat16()
    beta = torch.sigmoid(n(B, T, HV))
    gg = -torch.nn.functional.softplus(n(B, T, HV))
    w = (1 + 0.1 * n(D)).bfloat16()
    s0 = n(B, HV, D, D) * 0.02 if with_s0 else None
    return dict(q=q, k=k, v=v, g=gg, beta=beta, z=z, w=w, s0=s0)


class Workload:
    """One rank's share of a configuration: its inputs on the device, the step it runs and
    the sizes the metric needs. Rank r of N is fully determined by (config, r, N), so rank 0
    can rebuild any rank's shard to check that rank's gathered outputs."""

    def __init__(self, cid, rank, world, device):
        from gdn_b200.sharding import batch_shard, head_shard
        cfg = CONFIGS[cid]
        self.cid, self.cfg, self.rank, self.world, self.device = cid, cfg, rank, world, device
        B, T, HQK, HV = cfg["B"], cfg["T"], cfg["HQK"], cfg["HV"]
        if cfg["shard"] == "batch-weak":  # every rank its own batch of the configuration
            inp = device_inputs(B, T, HQK, HV, cfg["seed"] + 1000 * rank, device, cfg["s0"])
            self.scaling, self.job_tokens = "weak", world * B * T
            self.parallelism = f"batch: one B={B} batch per rank (x{world}), no collective on the data path"
        elif cfg["shard"] == "batch":     # the batch split over the ranks
            b0, b1 = batch_shard(B, world, rank)
            inp = device_inputs(B, T, HQK, HV, cfg["seed"], device, cfg["s0"])
            inp = {k: (None if t is None else (t if k == "w" else t[b0:b1].contiguous())) for k, t in inp.items()}
            B = b1 - b0
            self.scaling, self.job_tokens = "strong", cfg["B"] * T
            self.parallelism = f"batch: {B} of {cfg['B']} sequences per rank (x{world}), no collective on the data path"
        else:                              # v-heads split over the ranks
            sh = head_shard(HV, HQK, world, rank)
            full = device_inputs(B, T, HQK, HV, cfg["seed"], device, cfg["s0"])
            qs, vs = slice(sh.q0, sh.q1), slice(sh.v0, sh.v1)
            inp = {"q": full["q"][:, :, qs], "k": full["k"][:, :, qs], "v": full["v"][:, :, vs],
                   "g": full["g"][:, :, vs], "beta": full["beta"][:, :, vs], "z": full["z"][:, :, vs],
                   "w": full["w"], "s0": None if full["s0"] is None else full["s0"][:, vs]}
            inp = {k: (None if t is None else t.contiguous()) for k, t in inp.items()}
            del full
            HQK, HV = sh.q1 - sh.q0, sh.v1 - sh.v0
            self.scaling, self.job_tokens = "strong", B * T
            self.parallelism = (f"head: v-heads [{sh.v0},{sh.v1}) and qk-heads [{sh.q0},{sh.q1}) per rank "
                                f"(x{world}), no collective on the data path")
        self.inp, self.B, self.T, self.HQK, self.HV = inp, B, T, HQK, HV
        self.step_bytes = alg_bytes(B, T, HQK, HV, with_s0=cfg["s0"])
        self.step_flops = alg_flops(B, T, HV)
        self.segmented = cfg["shard"] == "head"
        ws_bytes = 256
        if self.segmented:  # the library's segment choice for this shape and device (256 B: one pass)
            import gdn_b200
            ws_bytes = max(256, int(gdn_b200.load_library().deltanet_segmented_workspace_size(
                B, T, HV, D, D, 64, 0)))
        self.launches_per_step = 3 if ws_bytes > 256 else 1
        self.ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=device)

    def outputs(self):
        return torch.empty_like(self.inp["v"]), torch.empty(self.B, self.HV, D, D, device=self.device)

    def step(self, s, out, stream):
        """One layer call on input set ``s`` into ``out`` = (y, sf), on ``stream``."""
        import ctypes

        import gdn_b200
        y, sf = out
        vp = ctypes.c_void_p
        lib = gdn_b200.load_library()
        s0 = s["s0"]
        if self.segmented:  # long streams: segments side by side, the library's segment choice
            rc = lib.deltanet_chunk_prefill_segmented(
                vp(s["q"].data_ptr()), vp(s["k"].data_ptr()), vp(s["v"].data_ptr()), vp(s["g"].data_ptr()),
                vp(s["beta"].data_ptr()), vp(s["z"].data_ptr()), vp(s["w"].data_ptr()), 1e-6, vp(y.data_ptr()),
                vp(0 if s0 is None else s0.data_ptr()), vp(sf.data_ptr()), self.B, self.T, self.HV, self.HQK, D, D,
                64, 0, vp(self.ws.data_ptr()), self.ws.numel(), vp(stream.cuda_stream))
            if rc != 0:
                raise RuntimeError(f"deltanet_chunk_prefill_segmented returned {rc}")
            return
        rc = lib.deltanet_chunk_prefill_gated(vp(s["q"].data_ptr()), vp(s["k"].data_ptr()), vp(s["v"].data_ptr()),
                                              vp(s["g"].data_ptr()), vp(s["beta"].data_ptr()), vp(s["z"].data_ptr()),
                                              vp(s["w"].data_ptr()), 1e-6, vp(y.data_ptr()),
                                              vp(0 if s0 is None else s0.data_ptr()), vp(sf.data_ptr()), self.B,
                                              self.T, self.HV, self.HQK, D, D, 64, vp(self.ws.data_ptr()), 256,
                                              vp(stream.cuda_stream))
        if rc != 0:
            raise RuntimeError(f"deltanet_chunk_prefill_gated returned {rc}")

    def api_call(self, d):
        """The public-API call of the e2e leg (torch's current stream)."""
        import gdn_b200
        if self.segmented:
            return gdn_b200.chunk_prefill_segmented(d["q"], d["k"], d["v"], d["g"], d["beta"], d.get("s0"),
                                                    z=d["z"], w=d["w"])
        return gdn_b200.chunk_prefill_gated(d["q"], d["k"], d["v"], d["g"], d["beta"], d["z"], d["w"], d.get("s0"))


GATE_CYCLES = 1_000_000  # ~0.5 ms of device spin ahead of a timed window (the host enqueues ~30 calls meanwhile)


def time_window(wl, sets, outs, stream, steps, start=0):
    """ms per step of one window of ``steps`` steps (inputs rotate over ``sets``). A short device
    spin is queued ahead of the first event, so that the host has enqueued the window's launches
    before the first one starts: the events then time the device's work, not the host's pace."""
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        torch.cuda._sleep(GATE_CYCLES)
    e0.record(stream)
    for i in range(start, start + steps):
        wl.step(sets[i % len(sets)], outs[i % len(sets)], stream)
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def time_windows(wl, sets, outs, stream, steps, n_windows, clk=None):
    """``n_windows`` repeats of the timed window: ms per step of each, and the SM clock read
    right after each window (the device was busy until a few microseconds before)."""
    ms, mhz = [], []
    for w in range(n_windows):
        ms.append(time_window(wl, sets, outs, stream, steps, w * steps))
        mhz.append(clk.read_mhz() if clk is not None else None)
    return ms, mhz


def max_over_ranks(x, dist, device):
    if not dist:
        return x
    t = torch.tensor(x if isinstance(x, list) else [x], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    v = t.tolist()
    return v if isinstance(x, list) else v[0]


def verify_shards(wl, dist, device, world, rank):
    """NCCL all_gather of every rank's y and final state (from its first input set) to rank 0,
    which rebuilds each rank's shard, reruns it on its own GPU and compares bit for bit. For the
    head-sharded config the assembled result is also compared with one unsharded call."""
    stream = torch.cuda.current_stream(device)
    out = wl.outputs()
    wl.step(wl.inp, out, stream)
    torch.cuda.synchronize()
    ys = [torch.empty_like(out[0]) for _ in range(world)]
    sfs = [torch.empty_like(out[1]) for _ in range(world)]
    dist.all_gather(ys, out[0])
    dist.all_gather(sfs, out[1])
    torch.cuda.synchronize()
    if rank != 0:
        return None
    dy = dsf = 0.0
    exact = True
    for r in range(world):
        other = wl if r == 0 else Workload(wl.cid, r, world, device)
        ref = other.outputs()
        other.step(other.inp, ref, stream)
        torch.cuda.synchronize()
        exact &= bool(torch.equal(ref[0], ys[r]) and torch.equal(ref[1], sfs[r]))
        dy = max(dy, float((ref[0].float() - ys[r].float()).abs().max()))
        dsf = max(dsf, float((ref[1] - sfs[r]).abs().max()))
        if r:
            del other
    res = {"collective": f"NCCL all_gather of y and final state from {world} ranks",
           "replayed_on_rank0": world, "bit_exact": exact, "max_abs_diff_y": dy, "max_abs_diff_state": dsf}
    if wl.segmented:  # the assembled heads against one unsharded one-pass call of the whole config
        full = Workload(wl.cid, 0, 1, device)
        y_all, sf_all = torch.cat(ys, dim=2), torch.cat(sfs, dim=1)
        import gdn_b200
        y1, sf1 = gdn_b200.chunk_prefill_gated(full.inp["q"], full.inp["k"], full.inp["v"], full.inp["g"],
                                               full.inp["beta"], full.inp["z"], full.inp["w"], full.inp["s0"])
        torch.cuda.synchronize()
        rel = ((y_all.float() - y1.float()).abs() / y1.float().abs().clamp_min(0.1)).max().item()
        srel = (torch.linalg.vector_norm(sf_all - sf1) / torch.linalg.vector_norm(sf1)).item()
        res["vs_unsharded_one_pass"] = {"y_max_rel_floor_0.1": rel, "state_rel_l2": srel}
        res["ok"] = exact and rel < 2e-2 and srel < 1e-4
    else:
        res["ok"] = exact
    return res


def time_config4(device, steps):
    """Config 4 on this GPU (B=32, S=4096): ms per call of deltanet_chunk_prefill_gated over
    ``steps`` calls after 3 warm-ups, CUDA events (inputs 4.5 GB, far above L2)."""
    wl = Workload(4, 0, 1, device)
    stream = torch.cuda.current_stream(device)
    out = wl.outputs()
    for _ in range(3):
        wl.step(wl.inp, out, stream)
    torch.cuda.synchronize()
    ms = time_window(wl, [wl.inp], [out], stream, steps)
    hbm_gbs = load_peaks()[0]
    gbs = wl.step_bytes / (ms / 1e3) / 1e9
    res = {"workload": CONFIGS[4]["desc"], "ms_per_step": round(ms, 4), "steps": steps,
           "tokens_per_s": round(wl.B * wl.T / (ms / 1e3), 1), "achieved_gbs": round(gbs, 1),
           "frac": round(gbs / hbm_gbs, 4), "alg_bytes_per_launch": wl.step_bytes,
           "kernel": "gdn::gdn_prefill_kernel (one CTA per (sequence, v-head); launcher's choice)"}
    del wl, out
    torch.cuda.empty_cache()
    return res


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
    return (bf(inp.q), bf(inp.k), bf(inp.v), f(inp.g), f(inp.beta), bf(inp.z), bf(inp.w),
            None if inp.s0 is None else f(inp.s0))


def cpu_sample_inputs(cfg):
    """Bounded CPU sample of a configuration: config 1 runs whole; config 4 one of its 32
    sequences; config 3 the first 4,096 tokens of its stream (all 32 heads)."""
    from gdn_b200.synthetic import make_inputs
    B = cfg["B"] if cfg["B"] * cfg["T"] <= 8192 else 1
    T = min(cfg["T"], 4096)
    inp = make_inputs(B, T, cfg["HQK"], cfg["HV"], D, seed=cfg["seed"], dist="baseline", with_s0=cfg["s0"])
    return inp, B, T


# ----------------------------------------------------------------- main
# The one JSON line goes to the process's original stdout; everything else that writes to file
# descriptor 1 (NCCL's version banner, library notices from C code) is sent to stderr, so that
# rank 0's stdout holds the JSON line alone.
_JSON_OUT = None


def emit(line):
    print(json.dumps(line), file=_JSON_OUT or sys.stdout, flush=True)


def _stdout_to_stderr():
    global _JSON_OUT
    sys.stdout.flush()
    _JSON_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)


def main():
    _stdout_to_stderr()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", type=int, default=1, choices=sorted(CONFIGS))
    ap.add_argument("--e2e-steps", type=int, default=50)
    ap.add_argument("--windows", type=int, default=10, help="repeats of the K-step window (spread)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-config4", action="store_true", help="skip the config-4 block of a default run")
    ap.add_argument("--shard-of", type=int, default=0,
                    help="diagnostic: run rank 0's shard of an N-GPU job on this one GPU (per-GPU figures)")
    ap.add_argument("--graph-launches", type=int, default=20,
                    help="launches captured in one CUDA graph for the graph timing (0: skip)")
    args = ap.parse_args()
    cfg = CONFIGS[args.config]
    warmup = max(3, args.warmup)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        return run_reference(args, cfg, world, rank, warmup)

    import gdn_b200  # noqa: F401
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)

    if args.shard_of > 1 and world == 1:  # one rank's share of an N-GPU job, alone on this GPU
        wl = Workload(args.config, 0, args.shard_of, device)
        wl.job_tokens //= (args.shard_of if wl.scaling == "weak" else 1)
        wl.parallelism = f"diagnostic: rank 0's shard of a {args.shard_of}-GPU job, alone on one GPU; " + wl.parallelism
    else:
        wl = Workload(args.config, rank, world, device)
    # inputs: rotate through enough copies that each step's working set was evicted from L2
    step_bytes = wl.step_bytes
    n_sets = max(1, math.ceil(3 * L2_BYTES / step_bytes)) if step_bytes < 3 * L2_BYTES else 1
    sets = [wl.inp] + [{k: (None if t is None else t.clone()) for k, t in wl.inp.items()} for _ in range(n_sets - 1)]
    outs = [wl.outputs() for _ in sets]
    stream = torch.cuda.current_stream(device)

    for i in range(warmup):
        wl.step(sets[i % n_sets], outs[i % n_sets], stream)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    # the timed region: exactly K steps; then the same window repeated for the spread
    n_extra = args.windows
    if n_extra and args.config != 1:  # big configurations: keep the repeats to about ten seconds
        est_ms = 1.0 if args.config == 4 else 4.0
        n_extra = max(2, min(n_extra, int(10_000 / max(1.0, args.steps * est_ms))))
    with ClockSampler(local) as clk:
        ms_total = time_window(wl, sets, outs, stream, args.steps) * args.steps
        win, win_mhz = time_windows(wl, sets, outs, stream, args.steps, n_extra, clk) if n_extra else ([], [])
    ms_total = max_over_ranks(ms_total, dist, device)
    win = max_over_ranks(win, dist, device) if win else []
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    status = _status(gdn_b200.load_library(), wl.ws, stream)
    ms_step = ms_total / args.steps
    value = wl.job_tokens / (ms_step / 1e3)
    windows = None
    if win:
        windows = {"n": len(win), "steps_each": args.steps, "ms_per_step_median": round(statistics.median(win), 5),
                   "ms_per_step_min": round(min(win), 5), "ms_per_step_max": round(max(win), 5),
                   "tokens_per_s_median": round(wl.job_tokens / (statistics.median(win) / 1e3), 1),
                   "sm_mhz_after_each": win_mhz}

    # config 1: the same launches replayed from a CUDA graph (what is left is GPU-side launch cost)
    graph = None
    if args.graph_launches > 0 and not wl.segmented:
        gl = args.graph_launches
        cap = torch.cuda.Stream(device)
        cap.wait_stream(stream)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=cap):
            for i in range(gl):
                wl.step(sets[i % n_sets], outs[i % n_sets], cap)
        g.replay()
        torch.cuda.synchronize()
        reps = max(3, min(50, args.steps // gl))
        ge0, ge1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ge0.record(stream)
        for _ in range(reps):
            g.replay()
        ge1.record(stream)
        torch.cuda.synchronize()
        ms_graph = max_over_ranks(ge0.elapsed_time(ge1), dist, device)
        us_call = ms_graph * 1e3 / (reps * gl)
        graph = {"launches_per_graph": gl, "replays": reps, "us_per_call": round(us_call, 2),
                 "tokens_per_s": round(wl.job_tokens / (us_call / 1e6), 1)}
        del g

    # e2e through the public API: pinned host in, pinned host out, copies inside the timed region
    e2e = run_e2e(args, wl, device, dist)

    verification = verify_shards(wl, dist, device, world, rank) if dist else None
    cfg4 = None
    if rank == 0 and world == 1 and args.config == 1 and not args.no_config4:
        del sets, outs
        torch.cuda.empty_cache()
        cfg4 = time_config4(device, max(3, min(args.steps, 10)))

    hbm_gbs, tf_burst, tf_sust, peak_kind = load_peaks()
    achieved_gbs = step_bytes / (ms_step / 1e3) / 1e9
    flops = wl.step_flops
    traffic, traffic_kernel = load_traffic(args.config)
    override = os.environ.get("GDN_B200_KERNEL", "auto")
    if override in ("fused", "split"):  # the launcher's kernel choice was overridden
        launched = ("gdn::split::gdn_prefill_split_kernel<false>" if override == "split"
                    else "gdn::gdn_prefill_kernel<false, false>")
        if traffic_kernel != launched:  # the committed traffic figure is another kernel's
            traffic, traffic_kernel = None, launched
    roofline = {"bound": "hbm", "achieved": round(achieved_gbs, 1), "peak": hbm_gbs, "unit": "GB/s",
                "frac": round(achieved_gbs / hbm_gbs, 4), "traffic": traffic,
                "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else peak_kind,
                "alg_bytes_per_launch": step_bytes, "alg_flops_per_launch": flops,
                "tflops_achieved": round(flops / (ms_step / 1e3) / 1e12, 1),
                "roofline_time_us": round(max(step_bytes / (hbm_gbs * 1e9), flops / (tf_burst * 1e12)) * 1e6, 2),
                "frac_of_roofline_time": round(max(step_bytes / (hbm_gbs * 1e9), flops / (tf_burst * 1e12))
                                               / (ms_step / 1e3), 4),
                "kernel": traffic_kernel}
    if wl.launches_per_step > 1:
        roofline["note"] = ("per rank, whole step (state pass, entry-state scan, output pass of the segmented "
                            "call); algorithmic bytes of one pass")

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sample, sb, st = cpu_sample_inputs(cfg)
        sec, threads = cpu_reference_time(cfg, sample)
        cpu = {"value": round(sb * st / sec, 1), "unit": "tokens/s", "cores": threads, "kind": "reference",
               "sample": f"{sb}x{st} tokens, HQK={cfg['HQK']} HV={cfg['HV']}: transformers "
                         f"torch_chunk_gated_delta_rule + Qwen3_5RMSNormGated on {threads} host threads, median "
                         f"of 5 after 2 warmups ({sec * 1e3:.1f} ms/call)"}

    if rank == 0:
        l2 = f"inputs rotate over {n_sets} device copies ({n_sets * step_bytes / 2**20:.0f} MiB > 126 MiB L2)"
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": wl.scaling,
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded on the device, BASELINE distributions)",
            "config": {"workload": cfg["desc"], "global_batch": cfg["B"] if wl.scaling == "strong" else cfg["B"] * world,
                       "seq_len": cfg["T"], "parallelism": wl.parallelism, "l2": l2},
            "roofline": roofline, "windows": windows, "cpu_baseline": cpu, "e2e": e2e,
            "clocks": clk.summary(), "gpu_launches": args.steps * wl.launches_per_step, "status_word": status,
            "graph": graph, "verification": verification, "config4": cfg4, "impl": "ours",
        }
        emit(line)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def _status(lib, ws, stream):
    import ctypes
    out = ctypes.c_int(0)
    lib.deltanet_read_status(ctypes.c_void_p(ws.data_ptr()), ctypes.byref(out), 0, ctypes.c_void_p(stream.cuda_stream))
    return out.value


def run_e2e(args, wl, device, dist):
    """Same metric through the public API (gdn_b200.chunk_prefill_gated, or chunk_prefill_segmented
    for the long stream) with pinned host buffers: every step copies its inputs host->device, runs,
    and copies y and the final state back. Copies and compute run on three streams with two device
    buffer sets, so step i+1's inputs upload while step i computes and step i-1's outputs download
    (the PCIe directions and the kernel overlap). A step's inputs sit in one pinned host buffer
    (each tensor at a 256-byte aligned offset) and go up in one copy into one device buffer whose
    views the call receives: one large transfer instead of one per tensor."""
    base = {k: t for k, t in wl.inp.items() if t is not None}
    B, HV = wl.B, wl.HV
    offs, total = {}, 0
    for k, t in base.items():
        offs[k] = total
        total += (t.numel() * t.element_size() + 255) // 256 * 256
    pinned = torch.empty(total, dtype=torch.uint8).pin_memory()
    for k, t in base.items():
        nb = t.numel() * t.element_size()
        pinned[offs[k]:offs[k] + nb].copy_(t.detach().contiguous().view(-1).view(torch.uint8).cpu())

    def views(buf):
        return {k: buf[offs[k]:offs[k] + t.numel() * t.element_size()].view(t.dtype).view(t.shape)
                for k, t in base.items()}

    nbuf = 2
    dev_bufs = [torch.empty(total, dtype=torch.uint8, device=device) for _ in range(nbuf)]
    dev_sets = [views(b) for b in dev_bufs]
    y_host = [torch.empty(tuple(base["v"].shape), dtype=torch.bfloat16).pin_memory() for _ in range(nbuf)]
    sf_host = [torch.empty(B, HV, D, D, dtype=torch.float32).pin_memory() for _ in range(nbuf)]
    h2d = total
    d2h = y_host[0].numel() * 2 + sf_host[0].numel() * 4
    steps = max(3, args.e2e_steps if wl.B * wl.T <= 65536 and not wl.segmented else 5)
    s_in, s_cmp, s_out = (torch.cuda.Stream(device) for _ in range(3))
    ev_in = [torch.cuda.Event() for _ in range(nbuf)]
    ev_done = [torch.cuda.Event() for _ in range(nbuf)]
    ev_out = [torch.cuda.Event() for _ in range(nbuf)]
    outs = [None] * nbuf

    def step(i):
        j = i % nbuf
        with torch.cuda.stream(s_in):
            s_in.wait_event(ev_done[j])  # buffer set j no longer read by step i - nbuf
            dev_bufs[j].copy_(pinned, non_blocking=True)
            ev_in[j].record(s_in)
        with torch.cuda.stream(s_cmp):
            s_cmp.wait_event(ev_in[j])
            s_cmp.wait_event(ev_out[j])  # outputs of step i - nbuf already downloaded
            outs[j] = wl.api_call(dev_sets[j])
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
    ms = max_over_ranks(e0.elapsed_time(e1), dist, device)
    ms_step = ms / steps
    api = ("gdn_b200.chunk_prefill_segmented (ctypes -> deltanet_chunk_prefill_segmented)" if wl.segmented
           else "gdn_b200.chunk_prefill_gated (ctypes -> deltanet_chunk_prefill_gated)")
    return {"value": round(wl.job_tokens / (ms_step / 1e3), 1), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": round(ms_step, 4), "steps": steps, "api": api,
            "pipelining": "3 streams, 2 device buffer sets (upload i+1 | compute i | download i-1); "
                          "inputs packed in one pinned buffer, one H2D copy per step"}


def run_reference(args, cfg, world, rank, warmup):
    """The reference's CPU implementation of the path, timed on this host's cores (rank 0 only)."""
    if rank != 0:
        return
    B, HQK, HV = cfg["B"], cfg["HQK"], cfg["HV"]
    sample, sb, T = cpu_sample_inputs(cfg)  # T: the sample's tokens per sequence
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
            "config": {"workload": cfg["desc"], "global_batch": B, "seq_len": cfg["T"], "parallelism": "host CPU"},
            "impl": "reference",
            "cpu_baseline": {"value": round(value, 1), "unit": "tokens/s", "cores": threads, "kind": "reference",
                             "sample": desc},
            "e2e": {"value": round(value, 1), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    emit(line)


if __name__ == "__main__":
    main()
