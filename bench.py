"""Benchmark of the rdv hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c5|c2|c1|c3|c4|trm]

Default workload (the configuration the metric "MLP
evals/sec at 1/2/4/8 B200" is defined across): fp16 MLP 3 -> 64 x 4 hidden
-> 4 with ReLU, fp32 accumulation, 67,108,864 rows ~U[-1,1]^3 fp32 split
evenly over the ranks, Kaiming-normal weights, zero biases, seeded synthetic
data, and a final NCCL all-gather of the fp32 outputs so every rank holds
the whole [67,108,864, 4] result. One step = one forward pass over the whole
batch plus the all-gather. Metric: MLP evals/s = rows x layers / s (5 weight
layers).

* ``value``: device time (CUDA events on the launch stream, max over ranks)
  with the input resident in HBM (805 MB > 126 MB L2, no flush). At N > 1
  the rows are cut into slabs split evenly over the ranks; the all-gather of
  slab k runs on NCCL's stream while slab k + 1 computes
  (sharding.sharded_map_overlapped).
* ``e2e``: the same metric through the public API from pinned host memory:
  each rank streams its rows in and its results out on copy streams while
  the kernels and the all-gather run (h2d/d2h bytes are whole-job figures).
* ``roofline``: tensor-pipe bound; achieved = algorithmic FLOPs of the
  rank's launches / their CUDA-event time; peak from MEASURED_PEAKS.json.
* ``cpu_baseline``: the oracle's torch-CPU restatement (float16-staged
  operands, fp32 GEMMs, all host threads) on a bounded sample, rank 0 at N=1.
* ``secondary`` (N=1): compact device-timed figures of the other BASELINE
  configs and the secondary operators from the same run.
* ``--impl reference``: the reference path's CPU restatement (the reference
  itself needs Vulkan, unavailable on this box) timed alone on the host's
  cores, rank 0 only.

``--workload c2`` runs BASELINE config 2 (4,194,304 rows per GPU, weak
scaling); c1, c3, c4 and trm run the other configs with their own metrics.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "MLP evals/sec (points x layers)"
UNIT = "evals/s"


# ----------------------------------------------------------------- workloads
def c2_spec():
    return dict(name="c2", dims=[32] + [128] * 8 + [16], rows=4_194_304, math="f16",
                x_dist="normal", w_init="kaiming_normal",
                workload="BASELINE config 2: fp16 fully-fused MLP 32->128x8->16, ReLU, fp32 accumulate")


def c1_spec():
    return dict(name="c1", dims=[3, 64, 64, 64, 4], rows=262_144, math="f32", x_dist="uniform",
                w_init="xavier_uniform", workload="BASELINE config 1: fp32 MLP 3->64->64->64->4, ReLU")


def c5_spec():
    return dict(name="c5", dims=[3, 64, 64, 64, 64, 4], rows=67_108_864, math="f16", x_dist="uniform",
                w_init="kaiming_normal",
                workload="BASELINE config 5: fp16 MLP 3->64x4->4 sharded over ranks + NCCL all-gather")


def make_weights(spec, seed_base=1000):
    dims = spec["dims"]
    layers = []
    for i in range(len(dims) - 1):
        g = torch.Generator().manual_seed(seed_base + i)
        fan_in, fan_out = dims[i], dims[i + 1]
        if spec["w_init"] == "kaiming_normal":
            W = torch.randn(fan_out, fan_in, generator=g) * math.sqrt(2.0 / fan_in)
        else:
            bound = math.sqrt(6.0 / (fan_in + fan_out))
            W = (torch.rand(fan_out, fan_in, generator=g) * 2 - 1) * bound
        layers.append({"W": W.float().contiguous(), "b": torch.zeros(fan_out), "math": spec["math"],
                       "relu": i < len(dims) - 2})
    return layers


def make_input(spec, rows, seed):
    g = torch.Generator().manual_seed(seed)
    if spec["x_dist"] == "normal":
        return torch.randn(rows, spec["dims"][0], generator=g)
    return torch.rand(rows, spec["dims"][0], generator=g) * 2 - 1


def build_map(rdv, layers, dev):
    m = None
    for l in layers:
        lin = rdv.linear(l["W"].to(dev), l["b"].to(dev), f16=(l["math"] == "f16"))
        m = lin if m is None else m >> lin
        if l["relu"]:
            m = m >> rdv.relu
    return m


def flops_per_row(dims):
    return 2 * sum(dims[i] * dims[i + 1] for i in range(len(dims) - 1))


# ------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while active."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu_index = gpu_index
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.gpu_index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        return self.summary()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ helpers
def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    except (OSError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def ncu_traffic(key):
    """Per-launch DRAM bytes recorded from an ncu capture in
    profiles/ncu_traffic.txt (lines: `<key> <bytes>`), or None."""
    path = os.path.join(ROOT, "profiles", "ncu_traffic.txt")
    try:
        with open(path) as f:
            for ln in f:
                parts = ln.split()
                if len(parts) >= 2 and parts[0] == key and not ln.startswith("#"):
                    return float(parts[1])
    except OSError:
        return None
    return None


def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        # NCCL on a high-priority stream: the overlapped all-gather's CTAs are
        # dispatched ahead of the next slab's kernel when SMs free up
        opts = dist.ProcessGroupNCCL.Options()
        opts.is_high_priority_stream = True
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local), pg_options=opts)
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v, world):
    if world == 1:
        return v
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def host_threads() -> int:
    """All of the host's cores for the CPU legs (torchrun sets
    OMP_NUM_THREADS=1 in every rank; the CPU figures are taken on rank 0 with
    the whole host)."""
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return torch.get_num_threads()


def cpu_baseline(spec, layers, seconds=8.0, chunk=65536):
    """Oracle torch-CPU restatement (float16-staged operands, fp32 GEMM,
    all host threads) on a bounded sample of the same workload."""
    from oracle import mlp as omlp

    cores = host_threads()
    lay = omlp.prestage_torch([{"W": l["W"], "b": l["b"], "math": l["math"], "relu": l["relu"]} for l in layers])
    x = make_input(spec, chunk, seed=12345)
    omlp.mlp_forward_torch_cpu(x[:1024], lay)
    done = 0
    t0 = time.perf_counter()
    while True:
        omlp.mlp_forward_torch_cpu(x, lay)
        done += chunk
        el = time.perf_counter() - t0
        if el >= seconds or done >= spec["rows"]:
            break
    n_layers = len(layers)
    return {"value": done * n_layers / el, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{done} rows in {chunk}-row chunks ({el:.1f} s), torch CPU, f16-staged operands"}


def mlp_config(spec, world):
    """The `config` object of an MLP workload line; both arms print the same
    one for the same (workload, N)."""
    sharded = spec["name"] == "c5"
    rows_per_gpu = spec["rows"] // world if sharded else spec["rows"]
    cfg = {"workload": spec["workload"], "dims": spec["dims"], "rows_per_gpu": rows_per_gpu,
           "rows_total": spec["rows"] if sharded else spec["rows"] * world,
           "l2": "inputs larger than L2, no flush",
           "parallelism": f"dp{world}" + ("+allgather" if sharded and world > 1 else "")}
    return cfg


# ---------------------------------------------------------------- reference
def run_reference(args, spec, world, rank):
    if rank != 0:
        return
    from oracle import mlp as omlp

    cores = host_threads()
    layers = make_weights(spec)
    lay = omlp.prestage_torch([{"W": l["W"], "b": l["b"], "math": l["math"], "relu": l["relu"]} for l in layers])
    sample = min(spec["rows"], 262_144)
    x = make_input(spec, sample, seed=0)
    for _ in range(args.warmup):
        omlp.mlp_forward_torch_cpu(x, lay)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        omlp.mlp_forward_torch_cpu(x, lay)
    el = time.perf_counter() - t0
    n_layers = len(layers)
    value = sample * n_layers * args.steps / el
    sample_txt = (f"{sample} of {spec['rows']} rows per step, torch CPU fp32 GEMMs on float16-staged operands, "
                  f"{cores} threads (restatement of the reference path; its Vulkan kernels are unavailable on "
                  f"this box)")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": el / args.steps * 1e3,
        "higher_is_better": True, "scaling": "strong" if spec["name"] == "c5" else "weak", "vs_baseline": None,
        "dtype": "f16" if spec["math"] == "f16" else "f32",
        "data": "synthetic (seeded torch.Generator)", "config": mlp_config(spec, args.gpus),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample_txt},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------- ours
def run_ours(args, spec, world, rank, local):
    import rdv_project_b200 as rdv
    from rdv_project_b200 import _native as N
    from rdv_project_b200.sharding import MulticastBuffer, PeerBuffer, piece_bounds, sharded_map_nvls, \
        sharded_map_overlapped, sharded_map_p2p

    dev = torch.device("cuda", torch.cuda.current_device())
    layers = make_weights(spec)
    n_layers = len(layers)
    m = build_map(rdv, layers, dev)
    sharded = spec["name"] == "c5"
    out_dim = spec["dims"][-1]
    chunks = args.chunks if args.chunks else (8 if world > 1 else 1)
    auto_reserve = 16 if world <= 2 else (32 if world <= 4 else 48)
    reserve = (args.reserve_ctas if args.reserve_ctas >= 0 else auto_reserve) if world > 1 else 0
    gather = args.gather if args.gather != "auto" else ("p2p" if world <= 4 else "nvls")
    mc_buf = None
    if sharded and world > 1 and gather == "nvls":
        try:
            mc_buf = MulticastBuffer(spec["rows"], out_dim)
        except Exception:  # no NVLink multicast (or no symmetric memory) on these GPUs
            mc_buf = None
        # every rank takes the same exchange: NCCL unless all have the buffer
        import torch.distributed as dist

        ok = torch.tensor([1.0 if mc_buf is not None else 0.0], device=torch.device("cuda", local))
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        if ok.item() < 1.0:
            if mc_buf is not None:
                mc_buf.close()
            mc_buf = None
            gather = "nccl"
    p2p = sharded and world > 1 and gather == "p2p"
    if sharded:
        n = spec["rows"]
        x_host = make_input(spec, n, seed=0)
        pieces = piece_bounds(n, world, rank, chunks)
        rows_rank = sum(e - b for b, e in pieces)
    else:
        n = spec["rows"]
        x_host = make_input(spec, n, seed=rank)
        pieces = [(0, n)]
        rows_rank = n
    x_dev = x_host.to(dev)
    peer_buf = PeerBuffer(n, out_dim) if p2p else None
    if mc_buf is not None:
        y_all = mc_buf.tensor
    else:
        y_all = peer_buf.tensor if p2p else torch.empty(n, out_dim, device=dev)
    nvls_reserve = args.reserve_ctas if args.reserve_ctas >= 0 else 16
    stream = torch.cuda.current_stream()

    def step():
        if mc_buf is not None:
            sharded_map_nvls(m, x_dev, mc_buf, chunks=chunks, reserve_ctas=nvls_reserve)
        elif p2p:
            sharded_map_p2p(m, x_dev, peer_buf, chunks=chunks)
        elif sharded:
            sharded_map_overlapped(m, x_dev, out=y_all, chunks=chunks, reserve_ctas=reserve)
        else:
            rdv.maps.evaluate_into(m, x_dev, y_all)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()

    # parity spot-check of the benchmark's own output against the oracle
    # (2048 sampled rows of the gathered result)
    parity = (None, None)
    if not args.profile_run:
        from oracle import mlp as omlp
        idx = np.sort(np.random.default_rng(7).choice(n, size=min(n, 2048), replace=False))
        got = y_all[torch.from_numpy(idx).to(dev)].cpu().numpy()
        lay_np = [{"W": l["W"].numpy(), "b": l["b"].numpy(), "math": l["math"], "relu": l["relu"]} for l in layers]
        ref = omlp.mlp_forward(x_host.numpy()[idx], lay_np)
        parity = omlp.rel_errors(got, ref)

    # ---- device-timed region ----
    sampler = ClockSampler(local) if rank == 0 else None
    # the sampler starts (and warms up) before the barrier, so every rank
    # enters the timed loop together
    if sampler:
        sampler.start()
        time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    launches0 = N.launch_count()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    launches = N.launch_count() - launches0
    clocks = sampler.stop() if sampler else None
    barrier(world)
    t_dev = max_over_ranks(ev0.elapsed_time(ev1) / 1e3, world)

    # kernel-only time of this rank's launches (no collective), for the roofline
    def kernels_only():
        for b, e in pieces:
            rdv.maps.evaluate_into(m, x_dev[b:e], y_all[b:e])

    torch.cuda.synchronize()
    ev0.record(stream)
    for _ in range(args.steps):
        kernels_only()
    ev1.record(stream)
    torch.cuda.synchronize()
    t_kern = ev0.elapsed_time(ev1) / 1e3
    barrier(world)

    # ---- end-to-end through the public API with pinned host buffers ----
    e2e_steps = 0 if args.profile_run else max(1, min(args.steps, 5))
    t_e2e = None
    if e2e_steps:
        x_pin = x_host.pin_memory()
        y_pin = torch.empty(n, out_dim).pin_memory()
        e2e_chunks = args.e2e_chunks

        def e2e_step():
            if sharded:
                sharded_map_overlapped(m, x_host=x_pin, y_host=y_pin, out=y_all, chunks=max(e2e_chunks, chunks),
                                       reserve_ctas=reserve)
            else:
                sharded_map_overlapped(m, x_host=x_pin, y_host=y_pin, out=y_all, chunks=e2e_chunks, shard=False)

        e2e_step()
        barrier(world)
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(e2e_steps):
            e2e_step()
        ev1.record(stream)
        torch.cuda.synchronize()
        t_e2e = max_over_ranks(ev0.elapsed_time(ev1) / 1e3, world)

    if peer_buf is not None:
        peer_buf.close()  # collective: every rank, before rank 0 reports
    if mc_buf is not None:
        mc_buf.close()
    if rank != 0:
        return
    units_per_step = (n if sharded else n * world) * n_layers
    value = units_per_step * args.steps / t_dev
    ms = t_dev / args.steps * 1e3
    peaks, peak_kind = measured_peaks()
    flops_launch = flops_per_row(spec["dims"]) * rows_rank
    achieved = flops_launch / (t_kern / args.steps) / 1e12
    key = "bf16_tflops"
    peak = float(peaks.get(key, 1590.0))
    traffic = ncu_traffic(f"mlp_tc_{spec['name']}")
    rows_io = n if sharded else n * world
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong" if sharded else "weak", "vs_baseline": None,
        "dtype": "f16" if spec["math"] == "f16" else "f32", "data": "synthetic (seeded torch.Generator)",
        "config": mlp_config(spec, world),
        "e2e": {"value": units_per_step * e2e_steps / t_e2e if e2e_steps else None, "unit": UNIT,
                "h2d_bytes_per_step": int(rows_io * spec["dims"][0] * 4),
                "d2h_bytes_per_step": int(rows_io * out_dim * 4)},
        "gpu_launches": int(launches),
        "roofline": {"bound": "tensor" if spec["math"] != "f32" else "fp32-cuda-core", "achieved": achieved,
                     "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak, "traffic": traffic,
                     "peak_source": f"{peak_kind} {key}", "flops_per_launch": flops_launch,
                     "kernel_ms": t_kern / args.steps * 1e3},
        "parity": {"rows": 2048, "normwise": parity[0], "elementwise": parity[1]},
        "clocks": clocks,
    }
    if mc_buf is not None:
        line["overlap"] = {"gather": "nvls: multimem.st copy kernel into a multicast symmetric buffer, slab by slab",
                           "chunks": chunks, "reserve_ctas": nvls_reserve}
    elif p2p:
        line["overlap"] = {"gather": "p2p: copy engines into peer-mapped buffers, slab by slab", "chunks": chunks}
    elif sharded and world > 1:
        line["overlap"] = {"gather": "nccl", "chunks": chunks, "reserve_ctas": reserve}
    if world == 1 and not args.profile_run:
        line["cpu_baseline"] = cpu_baseline(spec, layers)
        if not args.no_secondary:
            line["secondary"] = secondary_summaries(args, local, spec["name"])
    print(json.dumps(line), flush=True)


def _r(v, nd=4):
    """Rounded number for the compact secondary section."""
    if v is None:
        return None
    return float(f"{v:.{nd}g}")


def secondary_summaries(args, local, headline):
    """Compact device-timed figures of the other configs and operators on
    this GPU (one object per workload: value, unit, ms, roofline fraction,
    parity against the oracle). Prose descriptions are in DESIGN.md."""
    out = {}
    for name, spec_fn in (("c2", c2_spec), ("c5", c5_spec), ("c1", c1_spec)):
        if name != headline:
            out[name] = mlp_summary(spec_fn())
    out["c3"] = run_c3(args, 1, 0, local, summary=True)
    out["c4"] = run_c4(args, 1, 0, local, summary=True)
    out["trm"] = run_trm(args, 1, 0, local, summary=True)
    out["rt"] = ratiotracking_summary()
    out["pbvr"] = pbvr_summary()
    out["chain"] = chain_summary()
    out["conv_tc"] = conv_family_summary()
    out["samplers"] = sampler_summary()
    return out


# ------------------------------------------------- config 3: Winograd conv
C3_SHAPE = (8, 256, 256, 64)  # NHWC float16 input, 64 output channels


def c3_data():
    x = torch.randn(C3_SHAPE, generator=torch.Generator().manual_seed(0)).half()
    w = torch.randn((64, 64, 3, 3), generator=torch.Generator().manual_seed(1000)) * math.sqrt(2.0 / 576)
    return x, w.permute(2, 3, 1, 0).contiguous(), torch.zeros(64)  # weight -> [3, 3, CIN, COUT]


def c3_bytes(n_img, out_bytes=4):
    _, h, w, c = C3_SHAPE
    return n_img * h * w * c * (2 + out_bytes) + 16 * 64 * 64 * 2


def time_steps(fn, steps, flush=None, stream=None):
    """Sum of per-step CUDA-event times (s) on `stream`, L2 flushed between
    steps (outside the timed intervals) when `flush` is given."""
    stream = stream or torch.cuda.current_stream()
    total = 0.0
    for i in range(steps):
        if flush is not None:
            flush.fill_(i & 0xFF)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        fn()
        e1.record(stream)
        e1.synchronize()
        total += e0.elapsed_time(e1) / 1e3
    return total


def run_c3(args, world, rank, local, summary=False):
    import rdv_project_b200 as rdv
    from rdv_project_b200 import _native as N
    from rdv_project_b200.sharding import all_gather_rows, shard_range

    dev = torch.device("cuda", torch.cuda.current_device())
    x_all, w33io, b = c3_data()
    ib, ie = shard_range(C3_SHAPE[0], world, rank)
    n_img = ie - ib
    x_host = x_all[ib:ie].contiguous()
    x = x_host.to(dev)
    conv = rdv.Conv3x3Winograd(w33io, b)
    y = torch.empty(x.shape[:3] + (64,), dtype=torch.float32, device=dev)
    y_all = torch.empty(C3_SHAPE[:3] + (64,), dtype=torch.float32, device=dev) if world > 1 else None
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # > 126 MB L2

    def step():
        conv(x, out=y)
        if world > 1:
            all_gather_rows(y, C3_SHAPE[0], out=y_all)

    steps = 5 if summary else args.steps
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    parity = (None, None)
    if not args.profile_run:
        parity = c3_oracle_parity(y[0].cpu().numpy(), x_host[0], w33io, b)
    sampler = ClockSampler(local) if (rank == 0 and not summary) else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    l0 = N.launch_count()
    t_kernel = time_steps(lambda: conv(x, out=y), steps, flush)
    barrier(world)  # ranks enter the collective loop together
    t_step = time_steps(step, steps, flush)
    launches = N.launch_count() - l0
    clocks = sampler.stop() if sampler else None
    t_kernel = max_over_ranks(t_kernel, world)
    t_step = max_over_ranks(t_step, world)
    peaks, peak_kind = measured_peaks()
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    achieved = c3_bytes(n_img) / (t_kernel / steps) / 1e9
    value = c3_bytes(C3_SHAPE[0]) * steps / t_step / 1e9
    if summary:
        # the F(4x4,3x3) extension (CUDA cores, fp32 operands) on the same input
        conv43 = rdv.Conv3x3Winograd(w33io, b, variant="F4x4")
        for _ in range(3):
            conv43(x, out=y)
        torch.cuda.synchronize()
        t43 = time_steps(lambda: conv43(x, out=y), steps, flush) / steps
        p43 = c3_oracle_parity(y[0].cpu().numpy(), x_host[0], w33io, b)
        return {"value": _r(value), "unit": "GB/s", "ms": _r(t_step / steps * 1e3), "frac": _r(achieved / hbm, 3),
                "parity": _r(parity[1], 2), "f4x4_ms": _r(t43 * 1e3), "f4x4_parity": _r(p43[1], 2)}
    # end to end through the public API with host buffers
    x_pin = x_host.pin_memory()
    y_pin = torch.empty(y.shape, dtype=torch.float32).pin_memory()
    e2e_steps = 0 if args.profile_run else max(1, min(args.steps, 5))

    def e2e_step():
        yy = conv(x_pin.to(dev, non_blocking=True))
        y_pin.copy_(yy, non_blocking=True)

    t_e2e = max_over_ranks(time_steps(e2e_step, e2e_steps, flush), world) if e2e_steps else None
    if rank != 0:
        return None
    line = {
        "metric": "Winograd GB/s", "value": value, "unit": "GB/s", "n_gpus": world, "steps": steps,
        "warmup": max(args.warmup, 3), "ms_per_step": t_step / steps * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic (seeded torch.Generator)",
        "config": {"workload": "BASELINE config 3: Winograd F(2x2,3x3) conv, stride 1, pad 1, NHWC fp16 "
                               "8x256x256x64 -> 64 (fp32 out), Kaiming-normal weights",
                   "images_per_gpu": n_img, "algorithmic_bytes_per_step": c3_bytes(C3_SHAPE[0]),
                   "l2": "flushed between steps (256 MB write, outside the timed intervals)",
                   "parallelism": f"images split over {world} rank(s), NCCL all-gather of the outputs"},
        "e2e": {"value": c3_bytes(C3_SHAPE[0]) * e2e_steps / t_e2e / 1e9 if e2e_steps else None, "unit": "GB/s",
                "h2d_bytes_per_step": int(x_pin.numel() * 2), "d2h_bytes_per_step": int(y_pin.numel() * 4)},
        "gpu_launches": int(launches),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                     "traffic": ncu_traffic("winograd_f23_c3"), "peak_source": f"{peak_kind} hbm_gbs",
                     "bytes_per_launch": c3_bytes(n_img)},
        "parity": {"against": "oracle float64 direct conv, image 0 rows 0-31", "normwise": parity[0],
                   "elementwise": parity[1]},
        "clocks": clocks,
    }
    if world == 1 and not args.profile_run:
        line["cpu_baseline"] = c3_cpu_baseline(x_all, w33io, b)
    print(json.dumps(line), flush=True)
    return line


def c3_oracle_parity(y0, x0, w33io, b, rows=32):
    """(normwise, elementwise) error of output rows [0, rows) of one image
    against the oracle's float64 direct convolution (the reference's
    Conv2DTensorOp arithmetic, conv2d_tensor_op.h:21-87) of the same
    float16-rounded input; input rows [0, rows] feed those outputs."""
    from oracle import mlp as omlp
    from oracle import winograd as owg

    xs = x0[:rows + 1].float().numpy()[None]
    ref = owg.conv3x3_direct(xs, w33io.numpy(), b.numpy())[0, :rows]
    return omlp.rel_errors(np.asarray(y0[:rows], dtype=np.float64), ref)


def c3_cpu_baseline(x_all, w33io, b, seconds=6.0):
    """torch CPU fp32 conv2d (the direct convolution the reference's op
    approximates) on float16-rounded images, all host threads."""
    import torch.nn.functional as F

    cores = host_threads()
    wt = w33io.permute(3, 2, 0, 1).contiguous()  # -> [COUT, CIN, 3, 3]
    done, t0 = 0, time.perf_counter()
    while True:
        xi = x_all[done % x_all.shape[0]:done % x_all.shape[0] + 1].float().permute(0, 3, 1, 2)
        F.conv2d(xi, wt, b, padding=1)
        done += 1
        el = time.perf_counter() - t0
        if el >= seconds or done >= x_all.shape[0]:
            break
    return {"value": c3_bytes(done) / el / 1e9, "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"{done} of {x_all.shape[0]} images ({el:.1f} s), torch CPU fp32 conv2d on float16-rounded "
                      f"input, algorithmic bytes of those images per second"}


# ------------------------------------------------------- config 4: ray-march
C4 = dict(width=1920, height=1080, dims=[3, 64, 64, 4], samples=128)


def c4_layers():
    spec = dict(dims=C4["dims"], math="f16", w_init="kaiming_normal")
    return make_weights(spec)


def run_c4(args, world, rank, local, summary=False):
    import rdv_project_b200 as rdv
    from rdv_project_b200 import _native as N
    from rdv_project_b200.sharding import all_gather_rows, shard_range
    from oracle import raymarch as orm

    dev = torch.device("cuda", torch.cuda.current_device())
    layers = c4_layers()
    ren = rdv.VolumeRenderer(build_map(rdv, layers, dev))
    W, H = C4["width"], C4["height"]
    pose = torch.from_numpy(orm.orbit_pose(0))
    rb, re_ = shard_range(H, world, rank)
    band = torch.empty((re_ - rb, W, 4), device=dev)
    img = torch.empty((H, W, 4), device=dev) if world > 1 else None

    def render():
        ren.render(pose, W, H, row_begin=rb, row_end=re_, out=band)

    def step():
        render()
        if world > 1:
            all_gather_rows(band, H, out=img)

    steps = 5 if summary else args.steps
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    hits = int(ren._ws[dev.index][:4].view(torch.int32).item())
    parity = (None, None)
    if not args.profile_run and rb <= 537 < re_ - 2:
        got = band[537 - rb:540 - rb].cpu().numpy()
        lay_np = [{"W": l["W"].numpy(), "b": l["b"].numpy(), "math": "f16", "relu": l["relu"]} for l in layers]
        ref = orm.render_emission_absorption(pose.numpy(), W, H, 128, lay_np, row_begin=537, row_end=540)
        from oracle import mlp as omlp
        parity = omlp.rel_errors(got, ref)
    sampler = ClockSampler(local) if (rank == 0 and not summary) else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    l0 = N.launch_count()
    t_kernel = time_steps(render, steps)
    barrier(world)  # ranks enter the collective loop together
    t_step = time_steps(step, steps)
    launches = N.launch_count() - l0
    clocks = sampler.stop() if sampler else None
    t_kernel = max_over_ranks(t_kernel, world)
    t_step = max_over_ranks(t_step, world)
    peaks, peak_kind = measured_peaks()
    peak = float(peaks.get("bf16_tflops", 1590.0))
    flops_sample = flops_per_row(C4["dims"])
    achieved = hits * 128 * flops_sample / (t_kernel / steps) / 1e12
    fps = steps / t_step
    if summary:
        return {"value": _r(fps), "unit": "frames/s", "ms": _r(t_step / steps * 1e3), "frac": _r(achieved / peak, 3),
                "parity": _r(parity[1], 2)}
    if rank != 0:
        return None
    line = {
        "metric": "ray-march frames/s", "value": fps, "unit": "frames/s", "n_gpus": world, "steps": steps,
        "warmup": max(args.warmup, 3), "ms_per_step": t_step / steps * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic (seeded weights, orbit pose 0)",
        "config": {"workload": "BASELINE config 4: volume ray-march 1920x1080, one pinhole ray per pixel, 128 "
                               "uniform samples per ray, MLP 3-64-64-4 fp16 (softplus density, sigmoid RGB), "
                               "front-to-back compositing",
                   "rays_hit_box_rank0": hits, "samples_per_frame_evaluated_rank0": hits * 128,
                   "l2": "weights only are reused; the RGBA output is written once",
                   "parallelism": f"row bands over {world} rank(s), NCCL all-gather of the image"},
        "e2e": {"value": fps, "unit": "frames/s", "h2d_bytes_per_step": 36,
                "d2h_bytes_per_step": int(H * W * 16)},
        "gpu_launches": int(launches),
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                     "traffic": None, "peak_source": f"{peak_kind} bf16_tflops",
                     "flops_per_launch": hits * 128 * flops_sample},
        "parity": {"against": "oracle render of rows 537-539", "normwise": parity[0], "elementwise": parity[1]},
        "clocks": clocks,
    }
    if not args.profile_run:
        # end to end: host pose in, RGBA image back to pinned host memory
        out_pin = torch.empty((re_ - rb, W, 4)).pin_memory()

        def e2e_step():
            render()
            out_pin.copy_(band, non_blocking=True)

        t_e2e = time_steps(e2e_step, max(1, min(args.steps, 5)))
        line["e2e"] = {"value": max(1, min(args.steps, 5)) / t_e2e, "unit": "frames/s", "h2d_bytes_per_step": 36,
                       "d2h_bytes_per_step": int(out_pin.numel() * 4)}
        if world == 1:
            line["cpu_baseline"] = c4_cpu_baseline(layers)
    print(json.dumps(line), flush=True)
    return line


def c4_cpu_baseline(layers, rows=4):
    """Oracle restatement (numpy, float16-staged MLP) on a band of full-width
    rows through the middle of the image, extrapolated to frames/s."""
    from oracle import raymarch as orm

    cores = host_threads()
    lay_np = [{"W": l["W"].numpy(), "b": l["b"].numpy(), "math": "f16", "relu": l["relu"]} for l in layers]
    t0 = time.perf_counter()
    orm.render_emission_absorption(orm.orbit_pose(0), C4["width"], C4["height"], 128, lay_np, row_begin=538,
                                   row_end=538 + rows)
    el = time.perf_counter() - t0
    return {"value": rows / el / C4["height"], "unit": "frames/s", "cores": cores, "kind": "port",
            "sample": f"{rows} full-width rows through the cube ({el:.1f} s, numpy/BLAS), extrapolated to 1080 rows "
                      f"(the middle rows hit the box more than the frame average, so this favours the CPU)"}


def run_reference_c34(args):
    """Reference arm for configs 3 and 4: the CPU restatement of the
    reference path on the host cores (rank 0 only)."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    if args.workload == "c3":
        x_all, w33io, b = c3_data()
        cb = c3_cpu_baseline(x_all, w33io, b, seconds=max(5.0, float(args.steps)))
        metric, unit = "Winograd GB/s", "GB/s"
    elif args.workload == "trm":
        cb = trm_cpu_baseline(trm_layers())
        metric, unit = "extinction evaluations/s", "evaluations/s"
    else:
        cb = c4_cpu_baseline(c4_layers())
        metric, unit = "ray-march frames/s", "frames/s"
    line = {"impl": "reference", "metric": metric, "value": cb["value"], "unit": unit, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": None, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32" if args.workload == "c3" else "f16",
            "data": "synthetic (seeded)",
            "config": {"workload": "RaymarchingTransmittance" if args.workload == "trm"
                       else f"BASELINE config {args.workload[1]}"},
            "cpu_baseline": cb, "e2e": {"value": cb["value"], "unit": unit, "h2d_bytes_per_step": 0,
                                        "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------- RaymarchingTransmittance (the reference's absorption sensor)
TRM = dict(width=1920, height=1080, dims=[3, 64, 64, 1], step=0.01, scale=1.0)


def trm_layers():
    spec = dict(dims=TRM["dims"], math="f16", w_init="kaiming_normal")
    layers = make_weights(spec)
    for l in layers:
        l["relu"] = True  # ReLU after every layer: extinction >= 0
    return layers


def trm_flop():
    d = TRM["dims"]
    return 2 * sum(d[i] * d[i + 1] for i in range(len(d) - 1))


def trm_rays():
    from oracle import raymarch as orm

    o, w = orm.camera_rays(orm.orbit_pose(0), TRM["width"], TRM["height"])
    return torch.from_numpy(np.concatenate([o, w], axis=1).astype(np.float32))


def run_trm(args, world, rank, local, summary=False):
    """RaymarchingTransmittance (the reference's absorption sensor) over the
    config-4 camera's rays, extinction ReLU(MLP 3->64->64->1) with LinearFast
    layers (Kaiming-normal, seeded), step 0.01, density scale 1. Rays are
    split in contiguous ranges over the ranks, one all-gather of T."""
    import rdv_project_b200 as rdv
    from rdv_project_b200 import _native as N
    from rdv_project_b200.sharding import all_gather_rows, shard_range
    from oracle import mlp as omlp
    from oracle import raymarch as orm

    dev = torch.device("cuda", torch.cuda.current_device())
    layers = trm_layers()
    node = rdv.RaymarchingTransmittance(build_map(rdv, layers, dev), step_size=TRM["step"],
                                        density_scale=TRM["scale"])
    rays_all = trm_rays()
    n_all = rays_all.shape[0]
    rb, re_ = shard_range(n_all, world, rank)
    rays_host = rays_all[rb:re_].contiguous()
    rays = rays_host.to(dev)
    T_all = torch.empty((n_all, 1), device=dev) if world > 1 else None
    state = {}

    def march():
        state["T"] = node(rays).as_tensor("torch")

    def step():
        march()
        if world > 1:
            all_gather_rows(state["T"], n_all, out=T_all)

    steps = 3 if summary else args.steps
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    evals_rank = node.last_evaluations()
    parity = (None, None)
    if not args.profile_run:
        mid = (TRM["height"] // 2) * TRM["width"]
        if rb <= mid and mid + 2048 <= re_:
            got = state["T"][mid - rb:mid - rb + 2048, 0].cpu().numpy()
            lay_np = [{"W": l["W"].numpy(), "b": l["b"].numpy(), "math": "f16", "relu": l["relu"]} for l in layers]
            sample = rays_all[mid:mid + 2048].numpy()
            ref = orm.raymarching_transmittance(sample[:, :3], sample[:, 3:], TRM["step"], TRM["scale"],
                                                orm.mlp_extinction(lay_np))
            parity = omlp.rel_errors(got, ref)
    sampler = ClockSampler(local) if (rank == 0 and not summary) else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    barrier(world)
    torch.cuda.synchronize()
    l0 = N.launch_count()
    t_kernel = time_steps(march, steps)
    barrier(world)
    t_step = time_steps(step, steps)
    launches = N.launch_count() - l0
    clocks = sampler.stop() if sampler else None
    evals_total = evals_rank
    if world > 1:
        import torch.distributed as dist
        tv = torch.tensor([evals_rank], dtype=torch.float64, device=dev)
        dist.all_reduce(tv)
        evals_total = int(tv.item())
    t_kernel = max_over_ranks(t_kernel, world)
    t_step = max_over_ranks(t_step, world)
    peaks, peak_kind = measured_peaks()
    peak = float(peaks.get("bf16_tflops", 1590.0))
    achieved = evals_rank * trm_flop() / (t_kernel / steps) / 1e12  # rank 0's launches
    value = evals_total * steps / t_step
    roof = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
            "peak_source": f"{peak_kind} bf16_tflops",
            "note": "MLP flops of the evaluated steps over the call's three launches (setup, fused MLP, combine)"}
    e2e = None
    if not args.profile_run and not summary:
        # end to end on every rank: its rays from pinned host memory, its T
        # back to pinned host memory; max over ranks
        rays_pin = rays_host.pin_memory()
        T_pin = torch.empty((re_ - rb, 1)).pin_memory()

        def e2e_step():
            rays.copy_(rays_pin, non_blocking=True)
            march()
            T_pin.copy_(state["T"], non_blocking=True)

        k = max(1, min(args.steps, 5))
        barrier(world)
        t_e2e = max_over_ranks(time_steps(e2e_step, k), world)
        e2e = {"value": evals_total * k / t_e2e, "unit": "evaluations/s",
               "h2d_bytes_per_step": int(rays_pin.numel() * 4) * world,
               "d2h_bytes_per_step": int(T_pin.numel() * 4) * world}
    if summary:
        return {"value": _r(value), "unit": "evaluations/s", "ms": _r(t_step / steps * 1e3),
                "frac": _r(achieved / peak, 3), "parity": _r(parity[1], 2)}
    if rank != 0:
        return None
    roof["traffic"] = ncu_traffic("mlp_tc_march_trm")
    roof["flops_per_launch"] = evals_rank * trm_flop()
    line = {
        "metric": "extinction evaluations/s", "value": value, "unit": "evaluations/s", "n_gpus": world,
        "steps": steps, "warmup": max(args.warmup, 3), "ms_per_step": t_step / steps * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded weights, orbit pose 0 camera rays)",
        "config": {"workload": "RaymarchingTransmittance (rdv/domain/volumes.py:124-141) over 1920x1080 pinhole "
                               "rays, extinction ReLU(MLP 3->64->64->1) LinearFast, step 0.01, density scale 1",
                   "rays": n_all, "evaluations_per_step": evals_total,
                   "l2": "rays (12 MB) stay in L2 between steps; the work is the MLP per step",
                   "parallelism": f"ray ranges over {world} rank(s), NCCL all-gather of T"},
        "e2e": None,
        "gpu_launches": int(launches),
        "roofline": roof,
        "parity": {"against": "oracle march of 2048 rays through the image middle", "normwise": parity[0],
                   "elementwise": parity[1]},
        "clocks": clocks,
    }
    if e2e is not None:
        line["e2e"] = e2e
    if not args.profile_run and world == 1:
        line["cpu_baseline"] = trm_cpu_baseline(layers)
    print(json.dumps(line), flush=True)
    return line


def trm_cpu_baseline(layers, n=65536):
    """Oracle restatement (numpy, the reference's per-step loop with early
    exit, float16-staged MLP) on n rays through the image middle."""
    from oracle import raymarch as orm

    cores = host_threads()
    lay_np = [{"W": l["W"].numpy(), "b": l["b"].numpy(), "math": "f16", "relu": l["relu"]} for l in layers]
    rays = trm_rays()
    mid = (TRM["height"] // 2) * TRM["width"]
    sample = rays[mid:mid + n].numpy()
    t0 = time.perf_counter()
    _, evals = orm.raymarching_transmittance(sample[:, :3], sample[:, 3:], TRM["step"], TRM["scale"],
                                             orm.mlp_extinction(lay_np), return_evaluations=True)
    el = time.perf_counter() - t0
    return {"value": evals / el, "unit": "evaluations/s", "cores": cores, "kind": "port",
            "sample": f"{n} rays through the image middle ({evals} evaluations, {el:.1f} s, numpy/BLAS)"}


def trm_majorant(layers, cells=16, sub=4, margin=1.3):
    """Voxel majorant [cells^3, 1] of the extinction chain: the largest value
    on a sub^3 lattice of every cell (faces included), times margin, + 0.05."""
    from oracle import mlp as omlp

    lay_np = [{"W": l["W"].numpy(), "b": l["b"].numpy(), "math": "f16", "relu": l["relu"]} for l in layers]
    k = cells * (sub - 1) + 1
    ax = np.linspace(-1, 1, k, dtype=np.float32)
    Z, Y, X = np.meshgrid(ax, ax, ax, indexing="ij")
    v = omlp.mlp_forward_f64(np.stack([X, Y, Z], -1).reshape(-1, 3), lay_np)[:, 0].reshape(k, k, k)
    g = np.zeros((cells, cells, cells), dtype=np.float32)
    s = sub - 1
    for a in range(cells):
        for b in range(cells):
            blk = v[a * s:a * s + sub, b * s:b * s + sub, :]
            for c in range(cells):
                g[a, b, c] = max(float(blk[:, :, c * s:c * s + sub].max()), 0.0) * margin + 0.05
    return torch.from_numpy(g[..., None]), lay_np


def ratiotracking_summary(steps=3):
    """RatiotrackingTransmittance over the config-4 camera's rays (1920x1080,
    orbit pose 0), extinction ReLU(MLP 3->64->64->1) LinearFast (the
    transmittance workload's chain), a 16^3 voxel majorant of it, density
    scale 1, fixed seeds; CUDA-core kernel, one thread per ray. The oracle
    restatement on 65,536 middle rays is the CPU figure."""
    import rdv_project_b200 as rdv
    from oracle import raymarch as orm

    dev = torch.device("cuda", torch.cuda.current_device())
    layers = trm_layers()
    grid, lay_np = trm_majorant(layers)
    ext = build_map(rdv, layers, dev)
    node = rdv.RatiotrackingTransmittance(ext, grid.to(dev), density_scale=TRM["scale"])
    rays = trm_rays().to(dev)
    seeds = (1234567, 7654321, 1357911, 2468024)
    for _ in range(2):
        node(rays, seeds=seeds)
    torch.cuda.synchronize()
    t = time_steps(lambda: node(rays, seeds=seeds), steps) / steps
    evals = node.last_evaluations()
    flop = trm_flop() * evals
    nominal = 148 * 128 * 2 * 1.965e9 / 1e12
    n_cpu = 65536
    mid = (TRM["height"] // 2) * TRM["width"]
    sample = trm_rays()[mid:mid + n_cpu].numpy()
    t0 = time.perf_counter()
    _, ev_cpu = orm.ratiotracking_transmittance(sample[:, :3], sample[:, 3:], TRM["scale"],
                                                orm.mlp_extinction(lay_np), grid.numpy(), seeds,
                                                index=np.arange(mid, mid + n_cpu), return_evaluations=True)
    el = time.perf_counter() - t0
    return {"value": _r(evals / t), "unit": "evaluations/s", "ms": _r(t * 1e3), "rays_per_s": _r(rays.shape[0] / t),
            "frac_fp32_nominal": _r(flop / t / 1e12 / nominal, 3), "cpu": _r(ev_cpu / el)}


def sphere_from_voxel(g):
    """A SphereMajorantField grid [D, H, W, 2] from a voxel majorant grid
    [D, H, W]: radius 1.5 voxels, the majorant the largest voxel majorant of
    the 3x3x3 neighbourhood (edge-clamped)."""
    p = np.pad(g, 1, mode="edge")
    D, H, W = g.shape
    m = np.full_like(g, -np.inf)
    for a in range(3):
        for b in range(3):
            for c in range(3):
                m = np.maximum(m, p[a:a + D, b:b + H, c:c + W])
    return np.stack([m, np.full_like(m, 1.5)], -1).astype(np.float32)


def pbvr_summary(steps=3):
    """PBVR over the config-4 camera's rays (1920x1080, orbit pose 0): the
    transmittance workload's extinction chain, its 16^3 voxel majorant (and
    a sphere field built from it, radius 1.5 voxels), a constant
    environment, albedo 0.8, g = 0.3, at most 8 bounces, fixed seeds;
    CUDA-core kernel, one thread per path; and PBVRT (next-event estimation
    toward a directional light) on the voxel field. The oracle restatement
    on 8,192 middle rays is the CPU figure."""
    import rdv_project_b200 as rdv
    from oracle import raymarch as orm

    dev = torch.device("cuda", torch.cuda.current_device())
    layers = trm_layers()
    grid, lay_np = trm_majorant(layers)
    ext = build_map(rdv, layers, dev)
    env = rdv.Constant([0.8, 0.9, 1.0])
    kw = dict(albedo=(0.8, 0.8, 0.8), g=0.3, max_bounces=8)
    node = rdv.PBVR(ext, env, grid.to(dev), **kw)
    sph = sphere_from_voxel(grid.numpy()[..., 0])
    node_s = rdv.PBVR(ext, env, rdv.SphereMajorantField(torch.from_numpy(sph).to(dev)), **kw)
    node_t = rdv.PBVRT(ext, grid.to(dev), env, rdv.Constant([0.8, 0.8, 0.8]), light_direction=(0.3, 1.0, -0.2),
                       light_intensity=(2.0, 2.0, 2.0), g=0.3, max_bounces=8)
    rays = trm_rays().to(dev)
    seeds = (1234567, 7654321, 1357911, 2468024)
    res = {}
    for name, nd in (("voxel", node), ("sphere", node_s), ("pbvrt", node_t)):
        for _ in range(2):
            nd(rays, seeds=seeds)
        torch.cuda.synchronize()
        res[name] = (time_steps(lambda: nd(rays, seeds=seeds), steps) / steps, nd.last_evaluations())
    t, evals = res["voxel"]
    flop = trm_flop() * evals
    nominal = 148 * 128 * 2 * 1.965e9 / 1e12
    n_cpu = 8192
    mid = (TRM["height"] // 2) * TRM["width"]
    sample = trm_rays()[mid:mid + n_cpu].numpy()
    t0 = time.perf_counter()
    _, ev_cpu = orm.pbvr(sample[:, :3], sample[:, 3:], orm.mlp_extinction(lay_np),
                         orm.constant_environment([0.8, 0.9, 1.0]),
                         lambda x, w: orm.voxel_majorant(grid.numpy()[..., 0], x, w), seeds,
                         index=np.arange(mid, mid + n_cpu), return_evaluations=True, **kw)
    el = time.perf_counter() - t0
    return {"value": _r(evals / t), "unit": "evaluations/s", "ms": _r(t * 1e3), "rays_per_s": _r(rays.shape[0] / t),
            "frac_fp32_nominal": _r(flop / t / 1e12 / nominal, 3), "sphere_ms": _r(res["sphere"][0] * 1e3),
            "sphere_evals": int(res["sphere"][1]), "pbvrt_ms": _r(res["pbvrt"][0] * 1e3),
            "pbvrt_evals": int(res["pbvrt"][1]), "cpu": _r(ev_cpu / el)}


def chain_summary(rows=1 << 20, steps=3):
    """TensorOperation pipeline of the config-2 architecture
    (LinearTensorOpSmall / ReLUTensorOp, 17 ops) on `rows` rows: one dispatch
    per op (each op reads and writes its fp32 result in HBM) against
    evaluate_chain(), which runs the pipeline as one fused launch."""
    import rdv_project_b200 as rdv

    dev = torch.device("cuda", torch.cuda.current_device())
    spec = c2_spec()
    layers = make_weights(spec)
    cur = make_input(spec, rows, seed=0).to(dev)
    ops = []
    for l in layers:
        cur = rdv.LinearTensorOpSmall(cur, l["W"].to(dev), l["b"].to(dev))
        ops.append(cur)
        if l["relu"]:
            cur = rdv.ReLUTensorOp(cur)
            ops.append(cur)
    final = ops[-1]

    def per_op():
        for op in ops:
            op.evaluate()

    for _ in range(2):
        per_op()
    torch.cuda.synchronize()
    t_ops = time_steps(per_op, steps)
    ref = final.as_type("torch").clone()
    for _ in range(2):
        final.evaluate_chain()
    torch.cuda.synchronize()
    t_fused = time_steps(final.evaluate_chain, steps)
    same = bool(torch.equal(final.as_type("torch"), ref))
    from oracle import mlp as omlp
    idx = np.sort(np.random.default_rng(3).choice(rows, size=2048, replace=False))
    x_np = make_input(spec, rows, seed=0).numpy()[idx]
    lay_np = [{"W": l["W"].numpy(), "b": l["b"].numpy(), "math": "f16", "relu": l["relu"]} for l in layers]
    got = final.as_type("torch")[torch.from_numpy(idx).to(dev)].cpu().numpy()
    parity = omlp.rel_errors(got, omlp.mlp_forward(x_np, lay_np))
    return {"ms": _r(t_fused / steps * 1e3), "per_op_ms": _r(t_ops / steps * 1e3), "speedup": _r(t_ops / t_fused, 3),
            "exact_vs_per_op": same, "parity": _r(parity[1], 2)}


def sampler_summary(points=1 << 24, steps=5):
    """TensorSampler and GridSampler, trilinear with clamp, on a 64^3 x 8
    fp32 grid (8 MiB, L2-resident) at 2^24 uniform points: points/s and the
    HBM rate of the per-point stream (12 B of coordinates in, 32 B of
    features out); the corner gathers hit L2."""
    import rdv_project_b200 as rdv

    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device="cpu").manual_seed(7)
    t = torch.randn(64, 64, 64, 8, generator=g).to(dev)
    x = (torch.rand(points, 3, generator=g) * 2 - 1).to(dev)
    out = {}
    for name, smp in (("tensor", rdv.TensorSampler(t)), ("grid", rdv.GridSampler(t))):
        for _ in range(2):
            smp(x)
        torch.cuda.synchronize()
        ms = time_steps(lambda: smp(x), steps) / steps * 1e3
        out[name + "_ms"] = _r(ms)
        out[name + "_gbs"] = _r(points * (12 + 32) / (ms * 1e-3) / 1e9)
    out["points_per_s"] = _r(points / (out["grid_ms"] * 1e-3))
    return out


def conv_family_summary(steps=5):
    """The reference's tensor-core direct convolution (Conv2DTensorOpSimple3x3
    arithmetic: float16 operands, fp32 accumulation) at config 3's shape
    (8x256x256x64 -> 64, 3x3), on the tcgen05 implicit-GEMM kernel and on the
    CUDA-core kernel with the same staged operands, L2 flushed between steps."""
    from rdv_project_b200 import _native as N

    dev = torch.device("cuda", torch.cuda.current_device())
    x_h, w33io, b = c3_data()
    n, h, w, c = C3_SHAPE
    x = x_h.reshape(n * h * w, c).to(dev)
    wt, bd = w33io.to(dev), b.to(dev)
    lib = N.lib()
    wp = torch.empty(int(lib.rdvb_conv_tc_packed_bytes(3, 3, c, c)), dtype=torch.uint8, device=dev)
    N.check(lib.rdvb_conv_tc_pack(wt.data_ptr(), 3, 3, c, c, N.RDVB_F16, wp.data_ptr(), None), "rdvb_conv_tc_pack")
    y = torch.empty(n * h * w, c, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def tc():
        N.check(lib.rdvb_conv2d_tc(x.data_ptr(), N.RDVB_F16, n, h, w, c, c, 3, 3, wp.data_ptr(), N.RDVB_F16,
                                   bd.data_ptr(), y.data_ptr(), None), "rdvb_conv2d_tc")

    def cuda_cores():
        N.check(lib.rdvb_conv2d_direct_staged(x.data_ptr(), N.RDVB_F16, n, h, w, c, c, 3, 3, wt.data_ptr(),
                                              bd.data_ptr(), N.RDVB_MATH_F16, 1, y.data_ptr(), None),
                "rdvb_conv2d_direct_staged")

    out = {}
    flops = 2 * n * h * w * c * c * 9
    for name, fn, k in (("tc", tc, steps), ("cuda_cores", cuda_cores, 1)):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        out[name] = time_steps(fn, k, flush=flush) / k
    peaks, peak_kind = measured_peaks()
    peak = float(peaks.get("bf16_tflops", 1590.0))
    tf = flops / out["tc"] / 1e12
    return {"ms": _r(out["tc"] * 1e3), "tflops": _r(tf), "frac": _r(tf / peak, 3),
            "cuda_core_ms": _r(out["cuda_cores"] * 1e3)}


def mlp_summary(spec, steps=5):
    """Device-timed MLP evals/s of another MLP config on this GPU (inputs
    resident in HBM), for the secondary section of the headline line."""
    import rdv_project_b200 as rdv

    dev = torch.device("cuda", torch.cuda.current_device())
    layers = make_weights(spec)
    m = build_map(rdv, layers, dev)
    x = rdv.wrap(make_input(spec, spec["rows"], seed=0).to(dev))
    for _ in range(3):
        m(x)
    torch.cuda.synchronize()
    t = time_steps(lambda: m(x), steps)
    peaks, peak_kind = measured_peaks()
    achieved = flops_per_row(spec["dims"]) * spec["rows"] / (t / steps) / 1e12
    out = {"value": _r(spec["rows"] * len(layers) * steps / t), "unit": UNIT, "ms": _r(t / steps * 1e3)}
    if spec["math"] != "f32":
        out["frac"] = _r(achieved / float(peaks.get("bf16_tflops", 1590.0)), 3)
    else:
        out["tflops_fp32"] = _r(achieved)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["c5", "c2", "c1", "c3", "c4", "trm"], default="c5")
    ap.add_argument("--gather", choices=["auto", "p2p", "nvls", "nccl"], default="auto",
                    help="config 5 at N > 1: p2p = slabs whose rows are copied into every rank's mapped buffer by "
                         "the copy engines over NVLink while the next slab computes; nccl = slabs with overlapped "
                         "NCCL all-gathers; nvls = slabs whose rows a 16-SM copy kernel writes once to the NVLink "
                         "multicast address of a symmetric buffer (multimem.st); auto (default) = p2p on 2 and 4 "
                         "GPUs, nvls on 8 (nccl where the GPUs offer no multicast). Measured ms per step: 2 B200s "
                         "p2p 2.94, nvls 3.21, nccl 3.20; 4: p2p 2.10, nccl 2.14; 8: p2p 2.62, nvls 1.64, nccl 1.85")
    ap.add_argument("--chunks", type=int, default=0,
                    help="slabs of the sharded config-5 step (default 8 at N > 1, 1 at N = 1)")
    ap.add_argument("--reserve-ctas", type=int, default=-1,
                    help="SMs left free of the persistent MLP kernel for the overlapped NCCL all-gather (N > 1); "
                         "default 16 on 2 GPUs, 32 on 4, 48 on 8 (measured ms per step, 8 slabs: 2 B200s 3.19 "
                         "with 16, 3.58 with 32; 4: 2.33 / 2.25 / 2.14 / 2.19 with 16 / 24 / 32 / 48; 8: 2.13 / "
                         "1.98 / 1.85 / 1.98 with 16 / 32 / 48 / 64)")
    ap.add_argument("--e2e-chunks", type=int, default=16,
                    help="pieces of the end-to-end leg's host-streaming pipeline")
    ap.add_argument("--rows", type=int, default=None,
                    help="rows per GPU instead of the config's (small cases for ncu captures)")
    ap.add_argument("--no-secondary", action="store_true",
                    help="headline line only (skip the other configs' device-timed summaries)")
    ap.add_argument("--profile-run", action="store_true",
                    help="timed loop only: no parity check, end-to-end leg or CPU baseline")
    args = ap.parse_args()
    if args.workload in ("c3", "c4", "trm"):
        if args.impl == "reference":
            run_reference_c34(args)
            return
        world, rank, local = dist_setup(args.gpus)
        try:
            {"c3": run_c3, "c4": run_c4, "trm": run_trm}[args.workload](args, world, rank, local)
        finally:
            if world > 1:
                import torch.distributed as dist
                dist.barrier()
                dist.destroy_process_group()
        return
    spec = {"c2": c2_spec, "c1": c1_spec, "c5": c5_spec}[args.workload]()
    if args.rows:
        spec["rows"] = args.rows
        spec["workload"] += f" (reduced to {args.rows} rows)"
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, spec, world, rank)
        return
    world, rank, local = dist_setup(args.gpus)
    try:
        run_ours(args, spec, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
