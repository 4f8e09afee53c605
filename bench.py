#!/usr/bin/env python
"""Benchmark of the chunkwise gated fast-weight scan, fwd+bwd (one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME] [--impl ours|reference]

A step is one forward + backward of the mixer core (phases 1-3 of
train_ablation.py:142-187, i.e. the B200 op ``chunk_fast_weight``) over one
batch of the workload, default config 1 of the baseline: B8 H16 T4096 dh128,
chunk 64, delta rule, bf16 activations with fp32 state.  Inputs are seeded
synthetic tensors with the distributions the baseline names (no dataset).

  value     whole-job tokens/s (B*T per rank per step, summed over ranks) with
            the inputs resident in HBM, timed by CUDA events, max over ranks.
  e2e       the same metric through the public API from pinned host buffers,
            host->device copy of the inputs and device->host copy of o and all
            gradients inside the timed region.
  roofline  the dominant kernel: algorithmic work per launch / its average
            launch time (CUDA events on its own stream, over the timed region).
  cpu_baseline  the CPU oracle (a port of the reference's eager path) on a
            bounded sample of the same workload, rank 0, N=1 only.

Multi-GPU (torchrun, one process per GPU): the default ``--scaling strong``
splits the one global B8*H16 batch the metric names into contiguous (b, h)
shards, one per rank (16 sequences per GPU at N=8), and counts the global B*T
tokens per step; ``--scaling weak`` runs a full config-1 batch per rank.  At
N > 1 the other mode is timed briefly as well (``other_scaling``), and every
rank's step and kernel times are gathered (``per_rank``).  The scan has no
data-path collective: the timing barrier, the max-over-ranks reduction and the
per-rank gather are the only NCCL traffic.

``--impl reference`` times the reference algorithm on the host cores instead
(the oracle port; the reference itself is Python and is not present on the
GPU box), rank 0 only, on a bounded sample scaled to the same metric.
"""

from __future__ import annotations

import argparse
import importlib
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import torch  # noqa: E402

PKG_NAME = "gmdn-gated-muon-deltanet_b200"
METRIC = "scan tokens/s fwd+bwd B8·H16·T4096·d128 bf16 at 1/2/4/8 GPU; % roofline"

CONFIGS = {
    "config1_delta": dict(B=8, H=16, T=4096, dh=128, chunk=64, rule=0, ns=5),
    "config2_muon": dict(B=8, H=16, T=4096, dh=128, chunk=64, rule=1, ns=5),
    "config3_adam": dict(B=8, H=16, T=4096, dh=128, chunk=64, rule=2, ns=5),
    "config3_adam_long": dict(B=1, H=16, T=65536, dh=128, chunk=64, rule=2, ns=5),
}
RULE_NAMES = {0: "delta", 1: "muon", 2: "adam"}


# ---------------------------------------------------------------------------
# algorithmic work per kernel launch (units: flops or bytes for one launch)
# ---------------------------------------------------------------------------

def kernel_work(name: str, cfg: dict) -> tuple[str, float, float]:
    """(bound, bf16 work, fp32-state work) per launch of a library kernel: flops
    for tensor-bound kernels (the second figure counts the fp32-state products,
    whose roofline rate is TF32, half the bf16 rate), bytes for HBM-bound ones.

    Per chunk-head (C tokens, head dim d; config 1: C=64, d=128; mm = 2 d^3):
      chunk_fwd_tc        the forward's products 2C^2d + 4Cd^2 + 4C^2d + 2Cd^2 (phases
                          1 and 3) + mm (state product) = 13.63 MFLOP (delta, adam)
      chunk_fwd_muon_tc   the same + 3 ns mm of Newton-Schulz (fp32 state)
      chunk_bwd1_tc       the reverse chain's products: P = q k^T (2C^2d),
                          dE^T = dO^T A + Gb (wk)^T (2C^2d + 2Cd^2), dO^T q and dE^T k
                          (2 x 2Cd^2) = 8.39 MFLOP (delta, adam)
      chunk_bwd1_muon_tc  the same + 8 ns mm: the msign VJP, 3 recomputed and 5
                          cotangent products per step (fp32 state)
      chunk_bwd2_tc       bytes, the backward's algorithmic HBM traffic of the
                          survey's definition: q, k, v, dO in (4 C d 2), dq, dk, dv out
                          (3 C d 2), every gate of the rule in and its cotangent out
                          (2 n_g C 4; n_g = 2 delta, 3 muon, 4 adam) = 115,712 B for delta.
                          The S_j and Gb_j histories it also reads by design (2 d^2 2, muon
                          + Gb_j lo d^2 2) are reported apart as design bytes.  Where the
                          delta backward is fused (cfg["n_fused"] > 0 tiles done beside the
                          chains), this launch does the other tiles only.
      chunk_bwd_fused_tc  bytes: the chains' inputs (q, k, dO 3 C d 2 and the gates n_g C 4
                          per chunk-head) and the token bytes of its n_fused tiles.
    Newton-Schulz counts the algorithmic products once (the kernels spend three
    split-bf16 MMAs on each).  The exact-fp32 kernels count their products.
    """
    B, H, T, d, C = cfg["B"], cfg["H"], cfg["T"], cfg["dh"], cfg["chunk"]
    N = T // C
    units = B * H * N
    ns = cfg["ns"] if cfg["rule"] == 1 else 0
    mm = 2.0 * d ** 3
    fwd = 2 * C * C * d + 4 * C * d * d + 4 * C * C * d + 2 * C * d * d + mm
    bwd1 = 2 * C * C * d + (2 * C * C * d + 2 * C * d * d) + 2 * (2 * C * d * d)
    flops = {
        "chunk_fwd_tc": (fwd, 0.0),
        "chunk_fwd_muon_tc": (fwd, 3 * ns * mm),
        "chunk_bwd1_tc": (bwd1, 0.0),
        "chunk_bwd1_muon_tc": (bwd1, 8 * ns * mm),
        "chunk_prep": (4.0 * C * d * d, 0.0),
        "chunk_out": (6.0 * C * C * d + 2.0 * C * d * d, 0.0),
        "chunk_state_grad": (4.0 * C * C * d + 2.0 * C * d * d, 0.0),
        "chunk_token_grad": (14.0 * C * C * d + 10.0 * C * d * d, 0.0),
        "scan_fwd_ieee": (0.0, mm * (1 + 3 * ns)),
        "scan_bwd_ieee": (0.0, mm * (3 + 8 * ns)),
    }
    n_g = {0: 2, 1: 3, 2: 4}[cfg["rule"]]
    bw2 = 7 * C * d * 2 + 2 * n_g * C * 4
    nf = int(cfg.get("n_fused", 0) or 0)
    if name == "chunk_bwd2_tc":
        return "hbm", float(bw2 * (units - nf)), 0.0
    if name == "chunk_bwd_fused_tc":
        return "hbm", float(bw2 * nf + (3 * C * d * 2 + n_g * C * 4) * units), 0.0
    if name in flops:
        f16, f32 = flops[name]
        return "tensor", float(f16 * units), float(f32 * units)
    return "tensor", float("nan"), 0.0


def design_bytes(name: str, cfg: dict) -> float | None:
    """Bytes a launch moves by design beyond the algorithmic ones: the state
    histories the token-gradient kernel reads (S_j and Gb_j bf16, muon also the
    bf16 remainder of Gb_j), per launch."""
    if name != "chunk_bwd2_tc":
        return None
    B, H, T, d, C = cfg["B"], cfg["H"], cfg["T"], cfg["dh"], cfg["chunk"]
    per = 2 * d * d * 2 + (d * d * 2 if cfg["rule"] == 1 else 0)
    nf = int(cfg.get("n_fused", 0) or 0)
    return float(kernel_work(name, cfg)[1] + per * (B * H * (T // C) - nf))


def step_work(cfg: dict) -> tuple[float, float, float]:
    """(bf16 flops, fp32-state flops, HBM bytes) of one mixer-core fwd+bwd, the
    survey's algorithmic definition: phases 1 and 3 forward 2C^2d + 4Cd^2 +
    4C^2d + 2Cd^2 per chunk-head and twice that backward; the state products
    4 mm(d^3) (muon + 11 ns mm); q, k, v, o, dO, dq, dk, dv (bf16) and three
    passes over the rule's gates (fp32)."""
    B, H, T, d, C = cfg["B"], cfg["H"], cfg["T"], cfg["dh"], cfg["chunk"]
    units = B * H * (T // C)
    fwd = 2 * C * C * d + 4 * C * d * d + 4 * C * C * d + 2 * C * d * d
    mm = 2.0 * d ** 3
    ns = cfg["ns"] if cfg["rule"] == 1 else 0
    n_g = {0: 2, 1: 3, 2: 4}[cfg["rule"]]
    nbytes = 11 * B * H * T * d * 2 + 3 * n_g * B * H * T * 4
    return 3.0 * fwd * units, (4 + 11 * ns) * mm * units, float(nbytes)


def step_roofline(cfg: dict, ms_per_step: float, peaks: dict, kind: str) -> dict:
    """The whole step against the survey's roofline: the slower of the tensor
    time (bf16 products at the bf16 peak, fp32-state products at TF32 = half
    of it) and the HBM time, at the nominal peaks (2.25 PFLOP/s, 8 TB/s) and at
    the measured ones."""
    f16, f32, nbytes = step_work(cfg)
    spec = max(f16 / 2.25e15 + f32 / 1.125e15, nbytes / 8e12)
    bf = peaks["bf16_tflops"] * 1e12
    meas = max(f16 / bf + f32 / (bf / 2), nbytes / (peaks["hbm_gbs"] * 1e9))
    t = ms_per_step / 1e3
    return {"spec_us": spec * 1e6, "measured_us": meas * 1e6, "step_us": t * 1e6,
            "frac_spec": spec / t, "frac_measured": meas / t,
            "bf16_gflop": f16 / 1e9, "fp32_state_gflop": f32 / 1e9, "hbm_gb": nbytes / 1e9,
            "peaks": ("nominal 2.25 PFLOP/s bf16, 1.125 TF32, 8 TB/s; measured "
                      + ("MEASURED_PEAKS.json" if kind == "measured" else "fallback")
                      + " bf16 burst and HBM copy, TF32 = bf16 / 2 (assumed)")}


def load_peaks() -> tuple[dict, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def load_traffic() -> dict:
    """DRAM bytes per launch by workload and kernel, from the committed ncu
    summary (profiles/ncu_traffic.txt: `workload kernel bytes source`)."""
    out: dict = {}
    p = os.path.join(ROOT, "profiles", "ncu_traffic.txt")
    if os.path.exists(p):
        for line in open(p):
            parts = line.split()
            if len(parts) >= 3 and not line.startswith("#"):
                out.setdefault(parts[0], {})[parts[1]] = int(parts[2])
    return out


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------

class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 10 ms.  Started
    before the warm-up (the tool takes ~0.2 s to come up); mark() brackets the
    timed region and summary() keeps the samples inside it (the nearest one
    when the region is shorter than the sampling period)."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: torch.device):
        import threading
        self.rows: list = []
        self.window = None
        self.proc = None
        try:
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            target = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
            cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                   "-lms", "10", "-i", target]
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                         text=True, bufsize=1)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            t0 = time.time()
            while not self.rows and time.time() - t0 < 3.0 and self.proc.poll() is None:
                time.sleep(0.01)
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append((time.time(), line))

    def mark(self, start: bool):
        now = time.time()
        if start:
            self.window = [now, None]
        elif self.window:
            self.window[1] = now

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict | None:
        parsed = []
        for ts, line in self.rows:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                parsed.append(dict(ts=ts, sm=float(parts[0]), max=float(parts[1]),
                                   reasons={k: parts[3 + i].lower() == "active" for i, k in
                                            enumerate(("hw_slowdown", "hw_thermal_slowdown",
                                                       "sw_thermal_slowdown", "sw_power_cap"))}))
            except ValueError:
                continue
        if not parsed or not self.window or self.window[1] is None:
            return None
        lo, hi = self.window
        inside = [r for r in parsed if lo <= r["ts"] <= hi + 0.02]
        if not inside:
            after = [r for r in parsed if r["ts"] >= lo]
            inside = after[:1] or parsed[-1:]
        reasons = sorted({k for r in inside for k, v in r["reasons"].items() if v})
        return {"sm_mhz": statistics.median(r["sm"] for r in inside),
                "sm_max_mhz": max(r["max"] for r in inside), "samples": len(inside),
                "window_ms": round(1e3 * (hi - lo), 2), "reasons": reasons}


# ---------------------------------------------------------------------------
# CPU legs (oracle port of the reference's eager path)
# ---------------------------------------------------------------------------

def cpu_sample_cfg(cfg: dict) -> dict:
    s = dict(cfg)
    s["B"] = 1
    s["H"] = min(cfg["H"], 4 if cfg["rule"] != 0 else 16)
    return s


def cpu_oracle_step(pkg, oracle_mod, scfg: dict, inp) -> float:
    t0 = time.perf_counter()
    names = ["q", "k", "v", "alpha", "beta", "mu", "nu"]
    ins = [None if getattr(inp, n) is None else getattr(inp, n).clone().requires_grad_(True)
           for n in names]
    o = oracle_mod.mixer_core_forward(*ins, scfg["rule"], scfg["ns"], scfg["chunk"])
    o.backward(inp.dO)
    return time.perf_counter() - t0


def cpu_tokens(cfg: dict, scfg: dict) -> float:
    """Config-equivalent tokens of one sample step: B_s*T scaled by the share of
    heads the sample covers (heads are independent)."""
    return scfg["B"] * scfg["T"] * scfg["H"] / cfg["H"]


def cpu_baseline(pkg, cfg: dict, reps: int = 3) -> dict:
    import oracle as oracle_mod
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    scfg = cpu_sample_cfg(cfg)
    inp = pkg.workloads.mixer_inputs(scfg["B"], scfg["H"], scfg["T"], scfg["dh"], scfg["rule"],
                                     scfg["chunk"], seed=0)
    cpu_oracle_step(pkg, oracle_mod, scfg, inp)  # warm-up
    times = [cpu_oracle_step(pkg, oracle_mod, scfg, inp) for _ in range(reps)]
    t = statistics.median(times)
    return {"value": cpu_tokens(cfg, scfg) / t, "unit": "tokens/s", "cores": threads,
            "kind": "port",
            "sample": (f"oracle mixer core fwd+bwd fp32 on B{scfg['B']} H{scfg['H']} "
                       f"T{scfg['T']} dh{scfg['dh']} ({RULE_NAMES[cfg['rule']]}), "
                       f"median of {reps} after 1 warm-up, {t:.2f} s/step; tokens scaled by "
                       f"heads covered ({scfg['H']}/{cfg['H']})")}


def load_workloads():
    """The seeded input generator, loaded by file path: importing it as a
    submodule would import the package, which maps libgmdn_b200.so, and the
    reference arm must run without the product's native code."""
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "gmdn_b200_workloads", os.path.join(ROOT, PKG_NAME, "workloads.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def job_config(args, cfg: dict, world: int) -> dict:
    """The `config` object of the JSON line, identical for both arms at the
    same N (cfg is the workload as named, before any per-rank sharding)."""
    B, H, T, dh, C = (cfg[k] for k in ("B", "H", "T", "dh", "chunk"))
    strong = args.scaling == "strong"
    per_rank = B * H // world if strong else B * H
    return {"workload": args.config, "model": "mixer core fwd+bwd",
            "global_batch": B * (1 if strong else world), "seq_len": T, "heads": H,
            "head_dim": dh, "chunk": C, "rule": RULE_NAMES[cfg["rule"]], "ns": cfg["ns"],
            "precision": args.precision,
            "parallelism": f"dp{world} (B*H shards, {per_rank} sequences per rank)",
            "l2": f"inputs larger than L2 (q,k,v,dO bf16 = "
                  f"{4 * per_rank * T * dh * 2 / 1e6:.0f} MB per rank)"}


def reference_sample_cfg(cfg: dict) -> dict:
    """What one reference-arm step computes: the whole workload when one CPU
    step of it takes seconds (delta: ~5-6 s at config 1 on 16 cores), else the
    bounded CPU sample (adam / muon steps take minutes at full size)."""
    return dict(cfg) if cfg["rule"] == 0 else cpu_sample_cfg(cfg)


def run_reference_arm(args, cfg: dict) -> None:
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    wl = load_workloads()
    import oracle as oracle_mod

    class _P:
        workloads = wl
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    scfg = reference_sample_cfg(cfg)
    inp = wl.mixer_inputs(scfg["B"], scfg["H"], scfg["T"], scfg["dh"], scfg["rule"],
                          scfg["chunk"], seed=0)
    # activations as the GPU arm's kernels see them (bf16), computed in fp32
    for n in ("q", "k", "v", "dO"):
        setattr(inp, n, getattr(inp, n).to(torch.bfloat16).float())
    for _ in range(args.warmup):
        cpu_oracle_step(_P, oracle_mod, scfg, inp)
    times = [cpu_oracle_step(_P, oracle_mod, scfg, inp) for _ in range(args.steps)]
    total = sum(times)
    value = cpu_tokens(cfg, scfg) * args.steps / total
    full = scfg == cfg
    sample = (f"oracle port of the reference eager path (fast_scan.py:72-95 + "
              f"train_ablation.py:142-187), fp32 autograd on {threads} threads, "
              f"B{scfg['B']} H{scfg['H']} T{scfg['T']} dh{scfg['dh']} per step" +
              ("" if full else "; tokens scaled by heads covered"))
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * total / args.steps, "higher_is_better": True,
        "scaling": args.scaling, "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": job_config(args, cfg, world),
        "workload_per_step": "full" if full else "sample",
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

def timed_steps(step, L, steps: int, stream, device, no_graph: bool):
    """Total ms of `steps` steps on `stream` (CUDA events; CUDA-graph replays
    of the step unless no_graph, see graph_of), and the library's per-kernel
    times from as many plain steps (at most five) right after."""
    run, _, gerr = (step, None, "disabled") if no_graph else graph_of(step, device)
    for _ in range(2):
        run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        run()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    L.prof_report()
    L.prof_enable(True)
    for _ in range(min(steps, 5)):
        step()
    torch.cuda.synchronize()
    L.prof_enable(False)
    return ms, L.prof_report(), "cuda_graph" if gerr is None else f"plain steps ({gerr})"


def run_epilogue(args) -> None:
    """The mixer epilogue alone (train_ablation.py:188-189 up to the output
    projection): per-head RMSNorm of o (B8 H16 T4096 d128, bf16) into the
    (B, T, D) layout, forward + backward per step, inputs resident in HBM (larger
    than L2).  One JSON line; the roofline is HBM bytes per launch of the
    dominant kernel: forward reads o and writes y, backward reads o and dy and
    writes do (dweight is 512 B)."""
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    pkg = importlib.import_module(PKG_NAME)
    L = importlib.import_module(PKG_NAME + "._lib")
    B, H, T, dh = 8, 16, 4096, 128
    g = torch.Generator().manual_seed(0)
    o = torch.randn(B, H, T, dh, generator=g).to(device, torch.bfloat16).requires_grad_(True)
    w = (1.0 + 0.5 * torch.randn(dh, generator=g)).to(device).requires_grad_(True)
    dy = torch.randn(B, T, H * dh, generator=g).to(device, torch.bfloat16)

    def step():
        y = pkg.head_rmsnorm(o, w)
        return torch.autograd.grad(y, (o, w), dy)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ms, kt, launch = timed_steps(step, L, args.steps, stream, device, args.no_graph)
    row_bytes = B * H * T * dh * 2
    work = {"head_rmsnorm_fwd": 2 * row_bytes, "head_rmsnorm_bwd": 3 * row_bytes}
    peaks, kind = load_peaks()
    kernel_times, roof = {}, None
    for name, (tms, n) in kt.items():
        kernel_times[name] = {"total_ms": tms, "launches": n, "avg_ms": tms / max(n, 1)}
    if kt:
        top = max(kt, key=lambda k: kt[k][0])
        achieved = work.get(top, 0) / (kt[top][0] / kt[top][1] / 1e3) / 1e9
        roof = {"kernel": top, "bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"], "traffic": None,
                "peak_source": ("measured (MEASURED_PEAKS.json hbm_gbs, copy)" if kind == "measured"
                                else "fallback (6.65 TB/s)")}
    print(json.dumps({
        "metric": "epilogue tokens/s fwd+bwd (per-head RMSNorm into (B, T, D)), B8·H16·T4096·d128 bf16",
        "value": B * T * args.steps / (ms / 1e3), "unit": "tokens/s", "n_gpus": 1,
        "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms / args.steps,
        "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "epilogue_config1", "l2": "inputs larger than L2 (o 134 MB)"},
        "roofline": roof, "kernel_times": kernel_times, "launch": launch}), flush=True)


def run_prologue(args) -> None:
    """The mixer prologue alone (train_ablation.py:124-140 after the two
    projections, which are plain GEMMs and not timed): conv + SiLU + q/k norm +
    head layout and the gate sigmoids at config-1 size (B8 T4096 D2048, H16,
    bf16), forward + backward per step, inputs resident in HBM.  Roofline: HBM
    bytes per launch of the dominant kernel (forward reads u and writes q, k,
    v; backward reads u, dq, dk, dv and writes du; gates are 2 % of it)."""
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    pkg = importlib.import_module(PKG_NAME)
    L = importlib.import_module(PKG_NAME + "._lib")
    B, T, H, dh, nG = 8, 4096, 16, 128, 3
    D3 = 3 * H * dh
    g = torch.Generator().manual_seed(0)
    u = torch.randn(B, T, D3, generator=g).to(device, torch.bfloat16).requires_grad_(True)
    w = (torch.randn(D3, 1, 4, generator=g) * 0.5).to(device).requires_grad_(True)
    bb = (torch.randn(D3, generator=g) * 0.1).to(device).requires_grad_(True)
    gl = torch.randn(B, T, nG * H, generator=g).to(device, torch.bfloat16).requires_grad_(True)
    cot = [torch.randn(B, H, T, dh, generator=g).to(device, torch.bfloat16) for _ in range(3)]
    cot.append(torch.randn(nG, B, H, T, generator=g).to(device, torch.bfloat16))

    def step():
        outs = pkg.mixer_prologue(u, w, bb, gl, H)
        return torch.autograd.grad(outs, (u, w, bb, gl), cot)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ms, kt, launch = timed_steps(step, L, args.steps, stream, device, args.no_graph)
    ub = B * T * D3 * 2
    work = {"mixer_prologue_fwd": 2 * ub, "mixer_prologue_bwd": 3 * ub}
    peaks, kind = load_peaks()
    kernel_times, roof = {}, None
    for name, (tms, n) in kt.items():
        kernel_times[name] = {"total_ms": tms, "launches": n, "avg_ms": tms / max(n, 1)}
    if kt:
        top = max(kt, key=lambda k: kt[k][0])
        achieved = work.get(top, 0) / (kt[top][0] / kt[top][1] / 1e3) / 1e9
        roof = {"kernel": top, "bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"], "traffic": None,
                "peak_source": ("measured (MEASURED_PEAKS.json hbm_gbs, copy)" if kind == "measured"
                                else "fallback (6.65 TB/s)")}
    print(json.dumps({
        "metric": "prologue tokens/s fwd+bwd (conv + SiLU + q/k norm + gates), B8·T4096·D2048·H16 bf16",
        "value": B * T * args.steps / (ms / 1e3), "unit": "tokens/s", "n_gpus": 1,
        "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms / args.steps,
        "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "prologue_config1", "l2": "inputs larger than L2 (u 403 MB)"},
        "roofline": roof, "kernel_times": kernel_times, "launch": launch}), flush=True)


def run_scan(args) -> None:
    """The scan-only drop-in (fast_state_scan / _TritonScan, fast_scan.py:334-414)
    at config-1 shapes: fp32 U, K (B8 H16 N64 128x128), delta rule, forward +
    backward per step through ``state_scan`` at the reference's default
    precision (tf32 -> GMDN_PREC_FAST: the tensor-core scan), inputs resident in
    HBM.  Roofline: the algorithmic HBM bytes of each launch (forward reads U,
    K and writes S, 1.61 GB; the backward's chain reads K, gS and writes dU, its
    dK kernel reads S, dU and writes dK, 1.61 GB each; the exact backward reads
    U, K, S, gS and writes dU, dK, 3.22 GB).  ``--precision ieee`` times the
    exact kernels."""
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    pkg = importlib.import_module(PKG_NAME)
    L = importlib.import_module(PKG_NAME + "._lib")
    B, H, N, dh = args.batch or 8, 16, 64, 128
    g = torch.Generator().manual_seed(0)
    mk = lambda *sh, sc=1.0: (torch.randn(*sh, generator=g) * sc).to(device)
    U = mk(B, H, N, dh, dh, sc=0.1).requires_grad_(True)
    K = mk(B, H, N, dh, dh, sc=0.01).requires_grad_(True)
    gate = lambda: torch.full((B, H, N), 0.9, device=device).requires_grad_(True)
    a, b, m, n = gate(), gate(), gate(), gate()
    gS = mk(B, H, N, dh, dh)

    prec = pkg.GMDN_PREC_FAST if args.precision == "fast" else pkg.GMDN_PREC_IEEE

    def step():
        S = pkg.state_scan(U, K, a, b, m, n, 0, 5, prec)
        return torch.autograd.grad(S, (U, K, a, b, m, n), gS)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ms, kt, launch = timed_steps(step, L, args.steps, stream, device, args.no_graph)
    mat = B * H * N * dh * dh * 4
    # algorithmic HBM bytes per launch: forward U, K in and S out; exact
    # backward U, K, S, gS in and dU, dK out; tensor-core backward: the chain
    # reads K, gS and writes dU, then dK reads S, dU and writes dK
    work = {"scan_fwd_ieee": 3 * mat, "scan_bwd_ieee": 6 * mat, "scan_fwd_tc": 3 * mat,
            "scan_bwd_chain_tc": 3 * mat, "scan_bwd_dk_tc": 3 * mat}
    peaks, kind = load_peaks()
    kernel_times, roof = {}, None
    for name, (tms, cnt) in kt.items():
        kernel_times[name] = {"total_ms": tms, "launches": cnt, "avg_ms": tms / max(cnt, 1)}
    if kt:
        top = max(kt, key=lambda k: kt[k][0])
        achieved = work.get(top, 0) / (kt[top][0] / kt[top][1] / 1e3) / 1e9
        roof = {"kernel": top, "bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"],
                "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"], "traffic": None,
                "peak_source": ("measured (MEASURED_PEAKS.json hbm_gbs, copy)" if kind == "measured"
                                else "fallback (6.65 TB/s)")}
    print(json.dumps({
        "metric": "scan-only tokens/s fwd+bwd (fast_state_scan, fp32 U/K), B8·H16·N64·d128 delta",
        "value": B * N * 64 * args.steps / (ms / 1e3), "unit": "tokens/s", "n_gpus": 1,
        "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms / args.steps,
        "higher_is_better": True, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "scan_config1", "precision": args.precision,
                   "l2": "inputs larger than L2 (U, K 537 MB each)"},
        "roofline": roof, "kernel_times": kernel_times, "launch": launch}), flush=True)


def run_train(args) -> None:
    """Config 4 of the baseline: one optimisation step of the ablation language
    model (train_ablation.py:197-314, 453-474; 12 layers, d_model 768, 12 heads
    of 64, 4x GELU MLP, vocab 32000, tied head) on the B200 mixer ops, bf16
    autocast, outer Muon on the hidden matrices and AdamW on the rest, seq 2048
    and a micro-batch of 8 sequences per GPU (global batch 64 at N = 8), tokens
    uniform in [0, 32000) from the seed.  At N > 1 the model is wrapped in DDP
    on the NCCL backend, so the step includes the bucketed gradient all-reduce
    over NVLink; the step's other work per GPU is fixed (weak scaling)."""
    import datetime
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=device)
    pkg = importlib.import_module(PKG_NAME)
    tr = importlib.import_module(PKG_NAME + ".training")
    L = importlib.import_module(PKG_NAME + "._lib")
    torch.backends.cuda.matmul.allow_tf32 = True   # as the reference's trainer (its msign is fp32)
    vocab, d, layers, heads, T, mb = 32000, 768, 12, 12, 2048, args.batch or 8
    inner = {0: "delta", 1: "muon", 2: "adam"}[CONFIGS[args.config]["rule"]]
    torch.manual_seed(0)
    model = tr.LanguageModel(vocab, d, layers, heads, inner, chunk=64, ns_steps=3,
                             mlp=args.mlp).to(device)
    net = model
    if dist is not None:
        net = torch.nn.parallel.DistributedDataParallel(model, device_ids=[local],
                                                        gradient_as_bucket_view=True)
    opts = tr.build_optimizers(net)
    sched = tr.LrSchedule(opts)   # the trainer's defaults: warm-up 500 of 9600 steps
    g = torch.Generator().manual_seed(1234 + rank)
    n_batches = max(args.warmup, 3) + args.steps
    data = torch.randint(0, vocab, (n_batches, mb, T + 1), generator=g).to(device)

    def step(i):
        sched.set_step(i)
        return tr.train_step(net, opts, data[i, :, :-1], data[i, :, 1:])

    for i in range(max(args.warmup, 3)):
        step(i)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    stream = torch.cuda.current_stream(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    L.prof_report()
    L.prof_enable(True)
    e0.record(stream)
    losses = [step(max(args.warmup, 3) + i) for i in range(args.steps)]
    e1.record(stream)
    torch.cuda.synchronize()
    L.prof_enable(False)
    kt = L.prof_report()
    ms = e0.elapsed_time(e1)
    if dist is not None:
        dist.barrier()
    ms = pkg.sharding.max_over_ranks(ms, device)
    tokens = world * mb * T * args.steps
    line = {
        "metric": "config-4 training tokens/s (12-layer GMDN LM, d768, H12, vocab 32000, seq 2048)",
        "value": tokens / (ms / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "config4_train", "inner": inner, "mlp": args.mlp,
                   "micro_batch_per_gpu": mb,
                   "global_batch": world * mb, "seq_len": T, "layers": layers, "d_model": d,
                   "heads": heads, "vocab": vocab,
                   "parallelism": f"dp{world}" + (" (DDP, NCCL all-reduce)" if world > 1 else ""),
                   "params_M": sum(p.numel() for p in model.parameters()) / 1e6},
        "loss_first_last": [float(losses[0]), float(losses[-1])],
        "lr_schedule": "train_ablation.py's: linear warm-up over 500 steps, these are steps "
                       f"0-{max(args.warmup, 3) + args.steps - 1}",
        "kernel_times": {k: {"avg_ms": v[0] / max(v[1], 1), "launches": v[1]} for k, v in kt.items()},
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def graph_of(step, device):
    """The step captured into a CUDA graph (warm-up on a side stream, then one
    capture), so that the timed loop replays the same launches without the
    host's per-launch work (the ctypes calls, tensor-map encoding and autograd
    bookkeeping of the custom ops): the replay runs the step's every kernel,
    and at strong-scaling sizes the host was otherwise slower than the GPU.
    Returns (replay, outputs of the captured step, None) or (step, None,
    reason) when capture is not possible."""
    try:
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):
            for _ in range(2):
                step()
        torch.cuda.current_stream(device).wait_stream(side)
        torch.cuda.synchronize(device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            out = step()
        torch.cuda.synchronize(device)
        return g.replay, out, None
    except Exception as e:   # capture not available: time the plain step
        torch.cuda.synchronize(device)
        return step, None, f"{type(e).__name__}: {str(e)[:120]}"


def graph_matches(replay, out, step) -> bool:
    """One replay's gradients equal a plain step's: dq, dk, dv bit for bit (the
    kernels are deterministic; a difference means the capture missed work),
    the gate gradients to 1e-5 (their per-chunk partials are summed with float
    atomics across CTAs, in no fixed order)."""
    replay()
    ref = step()
    torch.cuda.synchronize()
    for i, (a, b) in enumerate(zip(out, ref)):
        if i < 3:
            if not torch.equal(a, b):
                return False
        elif (a.float() - b.float()).abs().max().item() > 1e-5 * (b.float().abs().max().item() + 1e-30):
            return False
    return True


def time_config(pkg, L, name: str, prec: int, steps: int, warmup: int, peaks: dict,
                peak_kind: str) -> dict:
    """One GPU, another configuration of the baseline on the same box and
    clocks: mixer-core fwd+bwd per step, inputs resident in HBM, CUDA events,
    kernel times from the library's own per-launch events, and the step
    against the survey's roofline."""
    cfg = dict(CONFIGS[name])
    B, H, T, dh, C, rule, ns = (cfg[k] for k in ("B", "H", "T", "dh", "chunk", "rule", "ns"))
    cfg["n_fused"] = L.chunk_bwd_fused_tiles(B, H, T, dh, C, rule, prec)
    dev = pkg.workloads.mixer_inputs(B, H, T, dh, rule, C, seed=0).to("cuda", torch.bfloat16)
    leaves = [dev.q, dev.k, dev.v, dev.alpha, dev.beta, dev.mu] + ([dev.nu] if rule == 2 else [])
    for t in leaves:
        t.requires_grad_(True)

    def step():
        o = pkg.chunk_fast_weight(dev.q, dev.k, dev.v, dev.alpha, dev.beta, dev.mu,
                                  dev.nu if rule == 2 else None, rule, ns, C, prec)
        return torch.autograd.grad(o, leaves, dev.dO)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    run, gout, gerr = graph_of(step, torch.device("cuda"))
    stream = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(2):
        run()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(steps):
        run()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    # per-kernel times from the library's per-launch events, on plain steps
    L.prof_report()
    L.prof_enable(True)
    for _ in range(min(steps, 5)):
        step()
    torch.cuda.synchronize()
    L.prof_enable(False)
    kt = L.prof_report()
    return {"config": name, "rule": RULE_NAMES[rule], "B": B, "H": H, "T": T, "ns": ns,
            "ms_per_step": ms, "value": B * T / (ms / 1e3), "unit": "tokens/s", "steps": steps,
            "launch": "cuda_graph" if gerr is None else f"plain ({gerr})",
            "step_roofline": step_roofline(cfg, ms, peaks, peak_kind),
            "kernel_times": {k: {"avg_ms": v[0] / max(v[1], 1), "launches": v[1]}
                             for k, v in kt.items()}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="config1_delta", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--precision", default="fast", choices=["fast", "ieee"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-others", action="store_true",
                    help="skip the one-GPU lines of configs 2, 3 and 3-long in the default run")
    ap.add_argument("--batch", type=int, default=None,
                    help="override B of the workload (small ncu captures)")
    ap.add_argument("--workload", default="mixer",
                    choices=["mixer", "epilogue", "prologue", "scan", "train"],
                    help="epilogue / prologue: that part of the mixer alone; scan: the "
                         "scan-only drop-in (fast_state_scan) on fp32 U, K; one GPU each")
    ap.add_argument("--no-graph", action="store_true",
                    help="time plain steps instead of CUDA-graph replays of the step")
    ap.add_argument("--mlp", default="gelu", choices=["gelu", "swiglu"],
                    help="train workload: the reference trainer's GELU MLP, or the SwiGLU MLP "
                         "that the config-4 benchmark description names")
    ap.add_argument("--scaling", default="strong", choices=["weak", "strong"],
                    help="strong (default): the one global batch the metric names split into "
                         "(b, h) shards over the ranks; weak: a full batch per rank.  At N > 1 "
                         "the other mode is also timed briefly and reported as an extra key")
    args = ap.parse_args()
    cfg = dict(CONFIGS[args.config])
    if args.batch:
        cfg["B"] = args.batch

    if args.impl == "reference":
        run_reference_arm(args, cfg)
        return
    if args.workload == "epilogue":
        run_epilogue(args)
        return
    if args.workload == "prologue":
        run_prologue(args)
        return
    if args.workload == "scan":
        run_scan(args)
        return
    if args.workload == "train":
        run_train(args)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    pkg = importlib.import_module(PKG_NAME)
    L = importlib.import_module(PKG_NAME + "._lib")
    prec = pkg.GMDN_PREC_FAST if args.precision == "fast" else pkg.GMDN_PREC_IEEE

    B, H, T, dh, C, rule, ns = (cfg[k] for k in ("B", "H", "T", "dh", "chunk", "rule", "ns"))
    B_global, H_global = B, H
    job_cfg = dict(cfg)   # the workload as named (the CPU sample scales against it)
    if args.scaling == "strong":
        # this rank's contiguous share of the global (b, h) sequences, as one batch
        start, end = pkg.sharding.shard_bh(B * H, rank, world)
        B, H = 1, end - start
        cfg["B"], cfg["H"] = B, H
    # delta with fewer sequences than SMs: tiles the fused backward does beside its chains
    cfg["n_fused"] = L.chunk_bwd_fused_tiles(B, H, T, dh, C, rule, prec)
    host = pkg.workloads.mixer_inputs(B, H, T, dh, rule, C, seed=rank)
    dev = host.to(device, torch.bfloat16)
    leaves = [dev.q, dev.k, dev.v, dev.alpha, dev.beta, dev.mu] + ([dev.nu] if rule == 2 else [])
    for t in leaves:
        t.requires_grad_(True)
    nu = dev.nu if rule == 2 else None

    def step():
        o = pkg.chunk_fast_weight(dev.q, dev.k, dev.v, dev.alpha, dev.beta, dev.mu, nu, rule,
                                  ns, C, prec)
        return torch.autograd.grad(o, leaves, dev.dO)

    def barrier():
        if dist is not None:
            dist.barrier()

    clocks = ClockSampler(device)
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    # the timed loop replays the step as one CUDA graph (graph_of); the graph
    # is checked against a plain step first
    run, gout, gerr = (step, None, "disabled") if args.no_graph else graph_of(step, device)
    graph_ok = None if gerr is not None else graph_matches(run, gout, step)
    if graph_ok is False:
        run, gerr = step, "replay differed from a plain step"
    for _ in range(max(args.warmup, 3)):
        run()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()

    stream = torch.cuda.current_stream(device)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = L.kernel_launches()
    step()   # one plain step: the library's launch counter per step
    torch.cuda.synchronize()
    launches_per_step = L.kernel_launches() - launches0
    barrier()
    torch.cuda.synchronize()
    clocks.mark(True)
    ev0.record(stream)
    for _ in range(args.steps):
        run()
    ev1.record(stream)
    torch.cuda.synchronize()
    clocks.mark(False)
    launches = launches_per_step * args.steps
    elapsed = ev0.elapsed_time(ev1)  # ms
    # per-kernel times from the library's per-launch CUDA events, on plain
    # steps right after the timed loop (events cannot sit inside the graph)
    L.prof_report()  # drop anything recorded so far
    L.prof_enable(True)
    for _ in range(min(args.steps, 5)):
        step()
    torch.cuda.synchronize()
    L.prof_enable(False)
    kt = L.prof_report()
    own_ms = elapsed
    barrier()
    elapsed = pkg.sharding.max_over_ranks(elapsed, device)
    tokens_per_step = B_global * T * (world if args.scaling == "weak" else 1)
    value = tokens_per_step * args.steps / (elapsed / 1e3)

    # ---- per-rank step times and kernel times (names the limiting rank) ----
    per_rank = None
    mine = {"rank": rank, "ms_per_step": own_ms / args.steps,
            "sequences": B * H,
            "kernels_ms": {k: round(v[0] / max(v[1], 1), 5) for k, v in kt.items()}}
    if dist is not None:
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        per_rank = gathered
    else:
        per_rank = [mine]

    # ---- the other scaling mode, briefly (N > 1): weak = a full batch per rank ----
    other = None
    if world > 1:
        mode = "weak" if args.scaling == "strong" else "strong"
        if mode == "weak":
            oB, oH = B_global, H_global
        else:
            s0, s1 = pkg.sharding.shard_bh(B_global * H_global, rank, world)
            oB, oH = 1, s1 - s0
        oh = pkg.workloads.mixer_inputs(oB, oH, T, dh, rule, C, seed=100 + rank).to(
            device, torch.bfloat16)
        oleaves = [oh.q, oh.k, oh.v, oh.alpha, oh.beta, oh.mu] + ([oh.nu] if rule == 2 else [])
        for t in oleaves:
            t.requires_grad_(True)

        def ostep():
            o = pkg.chunk_fast_weight(oh.q, oh.k, oh.v, oh.alpha, oh.beta, oh.mu,
                                      oh.nu if rule == 2 else None, rule, ns, C, prec)
            return torch.autograd.grad(o, oleaves, oh.dO)

        for _ in range(3):
            ostep()
        torch.cuda.synchronize()
        orun = ostep if args.no_graph else graph_of(ostep, device)[0]
        for _ in range(2):
            orun()
        osteps = max(3, min(args.steps, 10))
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(osteps):
            orun()
        e1.record(stream)
        torch.cuda.synchronize()
        oms = pkg.sharding.max_over_ranks(e0.elapsed_time(e1), device)
        otok = B_global * T * (world if mode == "weak" else 1)
        other = {"scaling": mode, "value": otok * osteps / (oms / 1e3), "unit": "tokens/s",
                 "ms_per_step": oms / osteps, "steps": osteps, "tokens_per_step": otok,
                 "sequences_per_rank": oB * oH}
        del oh, oleaves

    # ---- end to end through the public API from pinned host memory ----
    # Every step copies its inputs host->device and o plus every gradient
    # device->host; copies run on their own streams so that step i+1's inputs
    # and step i's results move while step i or i+1 computes (two device
    # input buffers).
    e2e = None
    if not args.no_e2e:
        act = ("q", "k", "v", "dO")
        gate_names = ("alpha", "beta", "mu") + (("nu",) if rule == 2 else ())
        pin = {n: getattr(host, n).to(torch.bfloat16 if n in act else torch.float32).pin_memory()
               for n in act + gate_names}
        outs = {"o": torch.empty(B, H, T, dh, dtype=torch.bfloat16).pin_memory()}
        for n in ("q", "k", "v"):
            outs["d" + n] = torch.empty(B, H, T, dh, dtype=torch.bfloat16).pin_memory()
        for n in gate_names:
            outs["d" + n] = torch.empty(B, H, T, dtype=torch.float32).pin_memory()
        h2d = sum(t.numel() * t.element_size() for t in pin.values())
        d2h = sum(t.numel() * t.element_size() for t in outs.values())
        dbuf = [{n: torch.empty(t.shape, dtype=t.dtype, device=device) for n, t in pin.items()}
                for _ in range(2)]
        s_h2d, s_d2h = torch.cuda.Stream(device), torch.cuda.Stream(device)
        ev_in = [torch.cuda.Event() for _ in range(2)]
        ev_used = [torch.cuda.Event() for _ in range(2)]
        gnames = ["dq", "dk", "dv"] + ["d" + n for n in gate_names]

        def e2e_run(nsteps):
            for i in range(nsteps):
                b = i & 1
                d = dbuf[b]
                with torch.cuda.stream(s_h2d):
                    if i >= 2:
                        s_h2d.wait_event(ev_used[b])
                    for n, t in pin.items():
                        d[n].copy_(t, non_blocking=True)
                    ev_in[b].record(s_h2d)
                stream.wait_event(ev_in[b])
                ins = [d[n].requires_grad_(True) for n in ("q", "k", "v") + gate_names]
                o = pkg.chunk_fast_weight(d["q"], d["k"], d["v"], d["alpha"], d["beta"], d["mu"],
                                          d.get("nu") if rule == 2 else None, rule, ns, C, prec)
                grads = torch.autograd.grad(o, ins, d["dO"])
                for t in ins:
                    t.requires_grad_(False)
                ev_used[b].record(stream)
                with torch.cuda.stream(s_d2h):
                    s_d2h.wait_event(ev_used[b])
                    outs["o"].copy_(o.detach(), non_blocking=True)
                    o.record_stream(s_d2h)
                    for n, g in zip(gnames, grads):
                        outs[n].copy_(g, non_blocking=True)
                        g.record_stream(s_d2h)

        e2e_run(2)
        torch.cuda.synchronize()
        barrier()
        # the copies of one step fill the pipeline before the first and drain it
        # after the last: time twice the device-timed steps (8..30) to amortise that
        e2e_steps = max(8, min(2 * args.steps, 30))
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(s_h2d)
        stream.wait_event(e0)
        s_d2h.wait_event(e0)
        e2e_run(e2e_steps)
        s_d2h.wait_stream(stream)
        s_d2h.wait_stream(s_h2d)
        e1.record(s_d2h)
        torch.cuda.synchronize()
        e_ms = pkg.sharding.max_over_ranks(e0.elapsed_time(e1), device)
        e2e = {"value": tokens_per_step * e2e_steps / (e_ms / 1e3), "unit": "tokens/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": e2e_steps,
               "ms_per_step": e_ms / e2e_steps,
               "pipelining": "inputs of step i+1 and results of step i copied on side streams"}

    # ---- roofline of the dominant kernel ----
    peaks, peak_kind = load_peaks()
    traffic = load_traffic()
    roofline = None
    kernel_times = {}
    if kt:
        for name, (ms, n) in kt.items():
            kernel_times[name] = {"total_ms": ms, "launches": n, "avg_ms": ms / max(n, 1),
                                  "share": ms / max(sum(v[0] for v in kt.values()), 1e-9)}
        top = max(kt, key=lambda k: kt[k][0])
        bound, work, work32 = kernel_work(top, cfg)
        avg_s = kt[top][0] / kt[top][1] / 1e3
        if bound == "tensor":
            source = ("measured (MEASURED_PEAKS.json bf16_tflops, burst)" if peak_kind == "measured"
                      else "fallback (1.59 PFLOP/s)")
            # bf16 products at the bf16 peak, fp32-state products at TF32 = bf16 / 2
            bf16 = peaks["bf16_tflops"]
            roof_s = work / (bf16 * 1e12) + work32 / (bf16 / 2 * 1e12)
            achieved = (work + work32) / avg_s / 1e12
            peak = (work + work32) / roof_s / 1e12 if roof_s > 0 else bf16
            unit = "TFLOP/s"
            if work32 > 0:
                source += "; fp32-state products at TF32 = bf16 / 2 (assumed, not measured)"
        else:
            source = ("measured (MEASURED_PEAKS.json hbm_gbs, copy)" if peak_kind == "measured"
                      else "fallback (6.65 TB/s)")
            achieved = work / avg_s / 1e9
            peak = peaks["hbm_gbs"]
            unit = "GB/s"
        tr = traffic.get(args.config, {}).get(top)
        if tr is not None and args.batch:
            tr = None   # the committed figure is for the named workload, not a resized one
        roofline = {"kernel": top, "bound": bound, "achieved": achieved, "peak": peak,
                    "unit": unit, "frac": achieved / peak, "traffic": tr,
                    "peak_source": source}
        if bound == "hbm":
            roofline["algorithmic_bytes"] = work
            dbytes = design_bytes(top, cfg)
            if dbytes is not None:
                roofline["design_bytes"] = dbytes
                roofline["design_frac"] = dbytes / avg_s / 1e9 / peak
                if tr is not None:
                    roofline["traffic_over_design"] = tr / dbytes
            if tr is not None:
                roofline["traffic_over_algorithmic"] = tr / work

    # ---- the other baseline configurations on the same box and clocks (one GPU) ----
    other_configs = None
    if world == 1 and args.config == "config1_delta" and not args.batch and not args.no_others:
        other_configs = [time_config(pkg, L, name, prec, 5, 3, peaks, peak_kind)
                         for name in ("config2_muon", "config3_adam", "config3_adam_long")]

    clocks.stop()
    clock_info = clocks.summary()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(pkg, job_cfg)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3),
            "ms_per_step": elapsed / args.steps, "higher_is_better": True,
            "scaling": args.scaling,
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": job_config(args, job_cfg, world),
            "roofline": roofline,
            "step_roofline": step_roofline(cfg, elapsed / args.steps, peaks, peak_kind),
            "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": launches, "clocks": clock_info,
            "launch": ("cuda_graph (each timed step replays the captured fwd+bwd; checked "
                       "against a plain step)") if gerr is None else f"plain steps ({gerr})",
            "kernel_times": kernel_times, "per_rank": per_rank, "other_scaling": other,
            "other_configs": other_configs,
            # rank 0's backward: token-gradient tiles done beside the chains in the fused
            # launch (chunk_bwd_fused_tc), of all its chunk-heads
            "backward_split": {"fused_tiles": cfg["n_fused"], "tiles": B * H * (T // C)},
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
