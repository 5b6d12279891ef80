#!/usr/bin/env python
"""ALPHABET forward benchmark: tokens/s and HBM roofline on B200, next to the CPU path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--config 4|1|2|3|5]

Default workload (the north-star case): synthetic uint8
224x224x3 images ~U(0,255), normalised with the ImageNet mean/std and
patchified 4x4 into x [B=256, T=3136, C=48] bf16; ALPHABET with D=96,
M=48 complex modes (real poles, log-uniform decay in [1e-3, 1]), K5/D4
depthwise convs, 1000 classes; random-init weights rounded to bf16.

* ``value``: device time of K forward passes through the C ABI with inputs
  resident in HBM (L2 flushed between steps, outside the per-step CUDA-event
  pair), whole-job tokens/s.  The batch is the configured global B=256 split
  into contiguous row shards over the N ranks (strong scaling, as BASELINE
  config 4 specifies; no collective on the data path); time = max over ranks.
* ``prepared``: the same with the operands prepared once, eager and replayed
  from a captured CUDA graph; ``weak_scaling``: every rank its own B=256 batch.
* ``multi_gpu_check`` (N > 1): the gathered sharded logits against a
  single-GPU forward of the same rows, and the config-5 time split against the
  unsplit forward, as max relative errors.
* ``e2e``: the same metric through the public module API with each rank's
  input rows copied from pinned host memory and the logits copied back every
  step.
* ``roofline``: the dominant kernel's algorithmic bytes per launch / its
  average CUDA-event duration measured during the timed region.
* ``cpu_baseline``: the CPU oracle (numpy restatement of the reference path) on
  the whole batch, rows split over one single-threaded worker per host core,
  rank 0 at N = 1 only.

``--impl reference`` times that CPU path alone (rank 0; other ranks exit).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import re
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "lnet-h200-imagenet1k-pg-ab_b200"))
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402

METRIC = "ALPHABET fwd tokens/sec"
UNIT = "tokens/s"

CONFIGS = {
    "4": dict(workload="alphabet_cfg4_imagenet224_patch4_b256_t3136_c48_d96_m48_k1000_bf16",
              B=256, T=3136, C=48, D=96, M=48, K=1000, dtype="bf16", images=True),
    "2": dict(workload="alphabet_cfg2_b128_t1024_c128_d128_m64_k10_fp32",
              B=128, T=1024, C=128, D=128, M=64, K=10, dtype="fp32", images=False),
    "5": dict(workload="alphabet_cfg5_b16_t65536_c256_d256_m64_k10_bf16",
              B=16, T=65536, C=256, D=256, M=64, K=10, dtype="bf16", images=False),
    # timed through the module API only (run_module): metadata / the Laplace layer
    "3": dict(workload="alphabet_cfg3_b64_t2048_c64_d64_m32_k10_fp32_dt_obs_valid",
              B=64, T=2048, C=64, D=64, M=32, K=10, dtype="fp32", images=False, meta=True),
    "1": dict(workload="laplace_cfg1_b64_t512_c16_per_channel8_fp32", B=64, T=512, C=16,
              per_channel=8, dtype="fp32", laplace=True),
}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# ---------------------------------------------------------------- model / inputs
def make_params(cfg, seed=0):
    """Seeded random-init ALPHABET parameters of the configured shape (state_dict names,
    materialised frames).  Real poles: raw_frequency = 0 and decay rates
    lambda ~ LogUniform[1.1e-3, 1]; depthwise conv weights ~ N(0, 1/5)."""
    import torch

    g = torch.Generator().manual_seed(seed)
    D, M, C, K = cfg["D"], cfg["M"], cfg["C"], cfg["K"]

    def rn(*shape, scale=1.0):
        return torch.randn(*shape, generator=g) * scale

    p = {}
    q, _ = torch.linalg.qr(rn(D, C))
    p["stem.projection.weight"] = q if D >= C else torch.linalg.qr(rn(C, D))[0].T
    p["stem.local.weight"] = rn(D, 1, 5, scale=1 / math.sqrt(5))
    p["stem.local.bias"] = rn(D, scale=0.1)
    for blk in ("forward_block", "backward_block"):
        lam = torch.exp(torch.empty(M).uniform_(math.log(1.1e-3), 0.0, generator=g))
        p[f"{blk}.raw_decay"] = torch.logit((lam - 1e-3) / (2.0 - 1e-3))
        p[f"{blk}.raw_frequency"] = torch.zeros(M)
        p[f"{blk}.norm.weight"] = 1.0 + rn(D, scale=0.1)
        p[f"{blk}.frame.weight"] = torch.linalg.qr(rn(D, 2 * M))[0]
    p["forward_block.direct_scale"] = rn(D, scale=0.3)
    p["forward_block.layer_scale"] = rn(D, scale=0.3)
    p["second_local.weight"] = rn(D, 1, 5, scale=1 / math.sqrt(5))
    p["second_local.bias"] = rn(D, scale=0.1)
    p["head.classifier.weight"] = rn(K, 14 * M, scale=1 / math.sqrt(14 * M))
    p["head.classifier.bias"] = rn(K, scale=0.1)
    if cfg["dtype"] == "bf16":
        p = {k: v.to(torch.bfloat16).float() for k, v in p.items()}
    return p


def make_images(cfg, device, seed=1):
    """Synthetic uint8 images [B, 224, 224, 3] ~U(0, 255) (image configs)."""
    import torch

    g = torch.Generator(device=device).manual_seed(seed)
    return torch.randint(0, 256, (cfg["B"], 224, 224, 3), generator=g, device=device,
                         dtype=torch.uint8)


def make_inputs(cfg, device, seed=1):
    """x [B, T, C] on `device` (bf16 for bf16 configs)."""
    import torch

    g = torch.Generator(device=device).manual_seed(seed)
    B, T, C = cfg["B"], cfg["T"], cfg["C"]
    if cfg["images"]:
        img = make_images(cfg, device, seed)
        mean = torch.tensor([0.485, 0.456, 0.406], device=device)
        std = torch.tensor([0.229, 0.224, 0.225], device=device)
        v = (img.float() / 255.0 - mean) / std  # [B, 224, 224, 3]
        v = v.reshape(B, 56, 4, 56, 4, 3).permute(0, 1, 3, 2, 4, 5).reshape(B, 56 * 56, 48)
        x = v
    else:
        x = torch.randn(B, T, C, generator=g, device=device)
    return x.to(torch.bfloat16 if cfg["dtype"] == "bf16" else torch.float32).contiguous()


def build_model(cfg, device):
    from lnet_b200 import AlphabetConfig, B200Alphabet

    m = B200Alphabet(AlphabetConfig(cfg["C"], cfg["D"], cfg["M"], cfg["K"]), cfg["K"]).eval()
    m.load_effective_parameters(make_params(cfg))
    return m.to(device)


# ---------------------------------------------------------------- clocks
REASON_BITS = {
    0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
    0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
    0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
    0x100: "display_clock_setting",
}


class ClockSampler:
    """Samples SM clock and clock-event (throttle) reasons every ~5 ms during the timed
    region through NVML (read-only queries); falls back to nvidia-smi at 200 ms."""

    def __init__(self, index: int):
        self.index = index
        self.samples: list[tuple[float, float, int]] = []
        self._stop = threading.Event()
        self.thread = None

    def _run_nvml(self, pynvml):
        h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
        mx = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
        while not self._stop.is_set():
            sm = float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
            try:
                bits = int(pynvml.nvmlDeviceGetCurrentClocksEventReasons(h))
            except AttributeError:
                bits = int(pynvml.nvmlDeviceGetCurrentClocksThrottleReasons(h))
            self.samples.append((sm, mx, bits))
            self._stop.wait(0.005)

    def _run_smi(self):
        proc = subprocess.Popen(
            ["nvidia-smi", f"--id={self.index}",
             "--query-gpu=clocks.sm,clocks.max.sm,clocks_event_reasons.active",
             "--format=csv,noheader,nounits", "-lms", "200"],
            stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        try:
            for line in proc.stdout:
                parts = [p.strip() for p in line.split(",")]
                try:
                    self.samples.append((float(parts[0]), float(parts[1]), int(parts[2], 16)))
                except (ValueError, IndexError):
                    pass
                if self._stop.is_set():
                    break
        finally:
            proc.terminate()

    def __enter__(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            target = lambda: self._run_nvml(pynvml)  # noqa: E731
        except Exception:  # noqa: BLE001
            target = self._run_smi
        self.thread = threading.Thread(target=target, daemon=True)
        self.thread.start()
        time.sleep(0.02)
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self.thread:
            self.thread.join(timeout=5)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        reasons = set()
        for _, _, bits in self.samples:
            for bit, name in REASON_BITS.items():
                if bits & bit and name != "gpu_idle":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(s[0] for s in self.samples),
                "sm_max_mhz": max(s[1] for s in self.samples), "reasons": sorted(reasons),
                "samples": len(self.samples)}


# ---------------------------------------------------------------- roofline helpers
def measured_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            d = json.loads(path.read_text())
            return float(d["hbm_gbs"]), "measured"
        except (ValueError, KeyError):
            pass
    return 6650.0, "fallback"


def algorithmic_bytes(kernel: str, cfg) -> float | None:
    """Minimum HBM bytes one launch of `kernel` must move for the workload."""
    B, T, C, D, M = cfg["B"], cfg["T"], cfg["C"], cfg["D"], cfg["M"]
    sx = 2 if cfg["dtype"] == "bf16" else 4
    sa = 2 if cfg["dtype"] == "bf16" else 4
    bt = B * T
    table = {
        # fused route: x (+8-step halo re-read is not algorithmic) in, stream v out
        "fused_writer_kernel": bt * (C * sx + D * sa),
        # fused route: stream v in (moments out are negligible)
        "fused_reader_kernel": bt * D * sa,
        # general route
        "gemm(stem)": bt * (C * sx + D * 4),
        "gemm(drive)": bt * (D * 4 + 2 * M * 4),
        "gemm(synthesis)": bt * (2 * M * 4 + D * 4),
        "scan_local_kernel": bt * 2 * M * 4,
        "scan_apply_kernel": bt * 2 * M * 8,
        "moments_partial_kernel": bt * 2 * M * 4,
        "rmsnorm_kernel": bt * D * 8,
        "drive_kernel": bt * 2 * M * 8,
        "depthwise_conv(stem)": bt * D * 8,
        "depthwise_conv(reader)": bt * D * 8,
        "residual_kernel": bt * D * 16,
    }
    v = table.get(kernel)
    return None if v is None else float(v)


def committed_traffic(kernel: str, cfg) -> float | None:
    """DRAM bytes per launch from the committed ncu summary of this kernel, scaled to the
    bench workload by tokens (line 'dram_bytes_per_token: N' in profiles/<kernel>*.md)."""
    for path in sorted((ROOT / "profiles").glob(f"{kernel.split('(')[0]}*.md")):
        m = re.search(r"dram_bytes_per_token:\s*([0-9.eE+]+)", path.read_text())
        w = re.search(r"workload:\s*(\S+)", path.read_text())
        if m and w and w.group(1) == cfg["workload"]:
            return float(m.group(1)) * cfg["B"] * cfg["T"]
    return None


# ---------------------------------------------------------------- CPU path
def _cpu_rows_worker(job):
    """One worker process: the numpy oracle (fp32) on its rows; returns seconds.
    Its BLAS pool is limited to one thread, so one worker = one core."""
    cfg, rows, seed, params_np = job
    try:
        from threadpoolctl import threadpool_limits

        threadpool_limits(1)
    except ImportError:
        pass
    from oracle import alphabet_oracle as A

    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, cfg["T"], cfg["C"])).astype(np.float32)
    t0 = time.perf_counter()
    A.alphabet_forward(x, params_np, dtype=np.float32)
    return time.perf_counter() - t0


class CpuBaseline:
    """The CPU path of the reference restated by the numpy oracle, run on every host
    core: `rows` rows split over one single-threaded worker process per core (the
    oracle's loop over T is serial Python, so cores are used by splitting rows;
    rows are independent).  A step = all `rows` rows; its time is the wall time of
    the pool (the slowest worker bounds it)."""

    def __init__(self, cfg, rows: int, cores: int | None = None):
        import multiprocessing as mp

        self.cfg = {k: cfg[k] for k in ("T", "C", "D", "M", "K", "dtype")}
        self.rows = rows
        self.cores = max(1, min(cores or os.cpu_count() or 1, rows))
        self.params = params_numpy(cfg)
        base, extra = divmod(rows, self.cores)
        self.split = [base + (1 if i < extra else 0) for i in range(self.cores)]
        self.pool = mp.get_context("spawn").Pool(self.cores)

    def step(self) -> float:
        jobs = [(self.cfg, r, 3 + i, self.params) for i, r in enumerate(self.split) if r]
        t0 = time.perf_counter()
        self.pool.map(_cpu_rows_worker, jobs, chunksize=1)
        return time.perf_counter() - t0

    def close(self):
        self.pool.close()
        self.pool.join()

    def describe(self, secs: float, steps: int) -> str:
        return (f"{self.rows} rows x T={self.cfg['T']} per step ({steps} step(s), {secs:.2f} s), "
                f"numpy oracle restating the reference eager path in fp32, rows split over "
                f"{self.cores} single-threaded worker processes (one per core; the oracle's loop "
                f"over T is serial, rows are independent, so time scales linearly in rows)")


def params_numpy(cfg):
    return {k: v.numpy().astype(np.float32) for k, v in make_params(cfg).items()}


# ---------------------------------------------------------------- arms
def run_reference(args, cfg):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    rows = args.ref_rows or cfg["B"]
    cpu = CpuBaseline(cfg, rows)
    try:
        for _ in range(args.warmup):
            cpu.step()
        times = [cpu.step() for _ in range(args.steps)]
    finally:
        cpu.close()
    total = sum(times)
    value = rows * cfg["T"] * args.steps / total
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "impl": "reference",
        "config": {"workload": cfg["workload"], "global_batch": cfg["B"],
                   "rows_per_step": rows, "same_config": rows == cfg["B"]},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cpu.cores, "kind": "port",
                         "sample": cpu.describe(total, args.steps)},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


TRAIN_METRIC = "ALPHABET train step tokens/sec"


def run_train(args, cfg):
    """Training step (``--mode train``, one GPU): forward + backward of
    ``sum(logits * dlogits)`` + an SGD update through the module API
    (``B200Alphabet.train()``: lnet_b200_alphabet_train_forward /
    lnet_b200_alphabet_backward), inputs resident in HBM, L2 flushed between
    steps.  The reference arm times the numpy backward oracle (forward with
    the saved activations + VJP, float32) on ``--ref-rows`` rows per step."""
    import torch

    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        if rank != 0:
            return 0
        from oracle import alphabet_grad_oracle as G

        rows = args.ref_rows or 8
        p = params_numpy(cfg)
        try:
            from threadpoolctl import threadpool_limits

            threadpool_limits(1)  # the line reports one core
        except ImportError:
            pass
        rng = np.random.default_rng(3)
        x = rng.standard_normal((rows, cfg["T"], cfg["C"])).astype(np.float32)
        dl = rng.standard_normal((rows, cfg["K"])).astype(np.float32)
        times = []
        for i in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            G.alphabet_backward(x, p, dl, dtype=np.float32)
            if i >= args.warmup:
                times.append(time.perf_counter() - t0)
        total = sum(times)
        value = rows * cfg["T"] * args.steps / total
        print(json.dumps({
            "metric": TRAIN_METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": cfg["workload"], "sample_rows_per_step": rows},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": 1, "kind": "port",
                             "sample": f"{rows} of {cfg['B']} rows x T={cfg['T']} per step, numpy "
                                       "backward oracle (forward + VJP) in fp32"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}), flush=True)
        return 0
    from lnet_b200 import _lib

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    model = build_model(cfg, dev).train()
    x = make_inputs(cfg, dev)
    B, T = cfg["B"], cfg["T"]
    dl = torch.randn(B, cfg["K"], generator=torch.Generator(device=dev).manual_seed(9), device=dev)
    opt = torch.optim.SGD(model.parameters(), lr=1e-4, foreach=True)
    meta = synthetic_metadata(cfg, dev) if cfg.get("meta") else {}
    model.validate_metadata = False  # validated once, as in the forward bench

    def step():
        opt.zero_grad(set_to_none=True)
        (model(x, **meta) * dl).sum().backward()
        opt.step()

    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    stops = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    _lib.profile_enable(True)
    launches = 0
    with ClockSampler(0) as clocks:
        for i in range(args.steps):
            flush.zero_()
            starts[i].record()
            step()
            launches += _lib.last_launch_count()
            stops[i].record()
        torch.cuda.synchronize()
    prof = _lib.profile_read()
    _lib.profile_enable(False)
    total_ms = sum(a.elapsed_time(b) for a, b in zip(starts, stops))
    captured = captured_train_step(args, model, x, meta, flush)
    print(json.dumps({
        "metric": TRAIN_METRIC, "value": B * T * args.steps / (total_ms / 1e3), "unit": UNIT,
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": total_ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32 (TF32 GEMMs for bf16 inputs)" if cfg["dtype"] == "bf16"
        else "f32", "data": "synthetic",
        "config": {"workload": cfg["workload"], "path": "module API, training step (SGD)",
                   "l2": "256 MiB flush between steps, outside the per-step event pair"},
        "clocks": clocks.summary(), "gpu_launches_backward": launches,
        "captured": captured, "kernels": _lib_kernels(prof)}), flush=True)
    return 0


def captured_train_step(args, model, x, meta, flush):
    """The same model trained with a cross-entropy loss and SGD, eagerly and
    through ``lnet_b200.prepare_exact_split_training`` (one CUDA-graph launch per
    step), each timed by CUDA events over ``args.steps`` steps."""
    import torch
    from torch.nn import functional as F

    from lnet_b200 import prepare_exact_split_training

    dev = x.device
    labels = torch.randint(0, model.head.classifier.out_features, (x.shape[0],),
                           generator=torch.Generator(device=dev).manual_seed(2), device=dev)
    opt = torch.optim.SGD(model.parameters(), lr=1e-4)

    def eager():
        opt.zero_grad(set_to_none=False)
        F.cross_entropy(model(x, **meta), labels).backward()
        opt.step()

    rt = prepare_exact_split_training(
        model, opt, x, labels, example_time_delta=meta.get("time_delta"),
        example_observation_mask=meta.get("observation_mask"),
        example_valid_mask=meta.get("valid_mask"))

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)]
        for a, b in ev:
            flush.zero_()
            a.record()
            fn()
            b.record()
        torch.cuda.synchronize()
        return sum(a.elapsed_time(b) for a, b in ev) / args.steps

    eager_ms = timed(eager)
    graph_ms = timed(rt.step_static)
    rt.close()
    return {"eager_ms_per_step": eager_ms, "graph_ms_per_step": graph_ms,
            "note": "cross-entropy loss + SGD: module API eagerly, and one replay of the "
                    "step captured by lnet_b200.prepare_exact_split_training"}


def synthetic_metadata(cfg, dev, seed=5):
    """Config 3's request metadata: Delta t ~ Exp(1) clipped to [0.05, 4],
    channel observation mask ~ Bernoulli(0.8), right-padded valid lengths
    ~ U(T/2, T)."""
    import torch

    g = torch.Generator().manual_seed(seed)
    B, T = cfg["B"], cfg["T"]
    dt = (-torch.log(torch.rand(B, T, generator=g).clamp_min(1e-12))).clamp(0.05, 4.0)
    obs = (torch.rand(B, T, cfg["C"], generator=g) < 0.8).float()
    lengths = torch.randint(T // 2, T + 1, (B,), generator=g)
    valid = (torch.arange(T).view(1, -1) < lengths.view(-1, 1)).float()
    return {"time_delta": dt.to(dev), "observation_mask": obs.to(dev),
            "valid_mask": valid.to(dev)}


def run_module(args, cfg):
    """Configs 1 and 3 (one GPU): K forwards through the module API with the
    inputs resident in HBM, L2 flushed between steps, CUDA events per step.
    Config 3 carries all metadata (Delta t ~ Exp(1) clipped to [0.05, 4],
    channel observation mask ~ Bernoulli(0.8), right-padded valid lengths
    ~ U(T/2, T)); config 1 is the pole-residue Laplace layer with 8 real poles
    per channel (p = -e^u, u ~ U(ln 0.01, 0)), block-diagonal residues."""
    import math

    import torch

    from lnet_b200 import _lib

    if args.impl == "reference":
        print(json.dumps({"impl": "reference", "unavailable":
                          "configs 1 and 3 are timed on the GPU path only; the reference arm "
                          "times config 4 (and 2, 5)"}), flush=True)
        return 0
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator().manual_seed(5)
    B, T = cfg["B"], cfg["T"]
    if cfg.get("laplace"):
        from lnet_b200 import B200PoleResidueTemporalMixing

        c, per = cfg["C"], cfg["per_channel"]
        u = torch.empty(c, per, dtype=torch.float64).uniform_(math.log(0.01), 0.0, generator=g)
        poles = -torch.exp(u).reshape(-1)
        r = torch.randn(c, per, generator=g, dtype=torch.float64) / math.sqrt(per)
        residues = torch.zeros(c, c * per, c, dtype=torch.float64)
        for ch in range(c):
            residues[ch, ch * per:(ch + 1) * per, ch] = r[ch]
        layer = B200PoleResidueTemporalMixing(c, c * per)
        layer.load_transfer_parameters(poles=poles, residues=residues,
                                       direct_term=torch.diag(torch.randn(c, generator=g,
                                                                          dtype=torch.float64)),
                                       bias=torch.zeros(c, dtype=torch.float64))
        layer = layer.to(dev)
        x = torch.randn(B, T, c, generator=g).to(dev)
        fwd = lambda: layer(x)  # noqa: E731
    else:
        model = build_model(cfg, dev)
        x = make_inputs(cfg, dev)
        meta = synthetic_metadata(cfg, dev)
        # serving setup of the reference's compiled inference wrapper
        # (alphabet_backbone.py:1225-1243): metadata validated once, not per call
        model.validate_metadata = False
        fwd = lambda: model(x, **meta)  # noqa: E731
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    with torch.no_grad():
        for _ in range(args.warmup):
            fwd()
        torch.cuda.synchronize()
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        stops = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        _lib.profile_enable(True)
        with ClockSampler(0) as clocks:
            for i in range(args.steps):
                flush.zero_()
                starts[i].record()
                fwd()
                stops[i].record()
            torch.cuda.synchronize()
        prof = _lib.profile_read()
        _lib.profile_enable(False)
    total_ms = sum(s_.elapsed_time(e_) for s_, e_ in zip(starts, stops))
    print(json.dumps({
        "metric": METRIC if not cfg.get("laplace") else "Laplace layer fwd tokens/sec",
        "value": B * T * args.steps / (total_ms / 1e3), "unit": UNIT, "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
        "higher_is_better": True, "dtype": cfg["dtype"], "data": "synthetic",
        "config": {"workload": cfg["workload"], "path": "module API (general route)",
                   "metadata_validation": False if cfg.get("meta") else None,
                   "l2": "256 MiB flush between steps, outside the per-step event pair"},
        "clocks": clocks.summary(), "kernels": _lib_kernels(prof)}), flush=True)
    return 0


def _time_steps(fn, steps, stream, flush, world, dist, dev):
    """K steps of `fn`, each bracketed by CUDA events on `stream` (L2 flushed before
    each, outside the pair); barrier + synchronize on both sides; returns the total
    device time in ms, max over ranks."""
    import torch

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    stops = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    for i in range(steps):
        flush.zero_()
        starts[i].record(stream)
        fn()
        stops[i].record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t = torch.tensor([sum(a.elapsed_time(b) for a, b in zip(starts, stops))], device=dev,
                     dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def multi_gpu_check(model, x_full, world, rank, dev, dist):
    """Correctness of the multi-GPU paths inside the scaling run (rank 0 reports):
    * batch sharding: sharded_forward's gathered logits of the 256 rows against
      rank 0's single-GPU forward of the same rows;
    * time split (BASELINE config 5's variant): timesplit_forward of one config-5
      row over all ranks against the unsplit forward of that row.
    Both are max relative errors (normwise); None at N=1."""
    import torch

    from lnet_b200.sharding import sharded_forward
    from lnet_b200.timesplit import timesplit_forward

    if world == 1:
        return {"note": "single GPU: nothing to compare"}
    with torch.no_grad():
        gathered = sharded_forward(model, x_full)
        out = {}
        if rank == 0:
            single = model(x_full)
            out["batch_shard_rel_err"] = float((gathered - single).abs().max() /
                                               single.abs().max())
        c5 = CONFIGS["5"]
        m5 = build_model(dict(c5), dev)
        g = torch.Generator(device=dev).manual_seed(11)
        x5 = torch.randn(1, c5["T"], c5["C"], generator=g, device=dev).to(torch.bfloat16)
        split = timesplit_forward(m5, x5)
        if rank == 0:
            whole = m5(x5)
            out["time_split_rel_err"] = float((split - whole).abs().max() / whole.abs().max())
            out["time_split_case"] = f"config 5, 1 row x T={c5['T']}, {world} ranks"
    return out if rank == 0 else None


def run_b200(args, cfg):
    import ctypes

    import torch
    import torch.distributed as dist

    from lnet_b200 import _lib
    from lnet_b200.alphabet import _workspace_bytes
    from lnet_b200.graph import CudaGraphForward
    from lnet_b200.sharding import shard_bounds

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        log(f"warning: WORLD_SIZE={world} but --gpus={args.gpus}; using WORLD_SIZE")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    lib = _lib.load()
    model = build_model(cfg, dev)
    x_full = make_inputs(cfg, dev)  # the same seeded batch on every rank
    B, T = cfg["B"], cfg["T"]
    lo, hi = shard_bounds(B, world, rank)  # strong scaling: this rank's rows of the batch
    x = x_full[lo:hi].contiguous()
    b_loc = hi - lo
    act = _lib.LNET_BF16 if cfg["dtype"] == "bf16" else _lib.LNET_F32
    params, _keep = model._effective(dev)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def c_abi_forward(xt, prepared=False):
        req = model._request(xt, None, None, None, act)
        nbytes = _workspace_bytes(params, req)
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        logits = torch.empty(xt.shape[0], cfg["K"], device=dev, dtype=torch.float32)
        if prepared:
            _lib.check(lib.lnet_b200_alphabet_prepare(ctypes.byref(params), ctypes.byref(req),
                                                      ws.data_ptr(), nbytes, stream.cuda_stream),
                       "lnet_b200_alphabet_prepare")
        fn_c = lib.lnet_b200_alphabet_forward_prepared if prepared else \
            lib.lnet_b200_alphabet_forward

        def fwd():
            _lib.check(fn_c(ctypes.byref(params), ctypes.byref(req), ws.data_ptr(), nbytes,
                            logits.data_ptr(), None, None, stream.cuda_stream),
                       "lnet_b200_alphabet_forward")
            return _lib.last_launch_count()
        return fwd

    # ---- value: the configured workload (global B split over the ranks), C ABI, inputs in
    # HBM, operands rebuilt in every step
    fwd = c_abi_forward(x)
    for _ in range(max(args.warmup, 3)):
        fwd()
    launches = [0]

    def counted():
        launches[0] += fwd()

    _lib.profile_enable(True)
    with ClockSampler(local) as clocks:
        total_ms = _time_steps(counted, args.steps, stream, flush, world, dist, dev)
    prof = _lib.profile_read()
    _lib.profile_enable(False)
    tokens_all = B * T * args.steps
    value = tokens_all / (total_ms / 1e3)

    # ---- prepared operands (lnet_b200_alphabet_prepare once), eager launches, and the
    # same prepared forward replayed from a captured CUDA graph
    fwd_p = c_abi_forward(x, prepared=True)
    for _ in range(max(args.warmup, 3)):
        fwd_p()
    prepared_ms = _time_steps(fwd_p, args.steps, stream, flush, world, dist, dev)
    with torch.no_grad():
        runner = CudaGraphForward(model, x)
        for _ in range(max(args.warmup, 3)):
            runner(x)
        graph_ms = _time_steps(lambda: runner(x), args.steps, stream, flush, world, dist, dev)
    prepared = {"value": tokens_all / (prepared_ms / 1e3), "unit": UNIT,
                "ms_per_step": prepared_ms / args.steps,
                "graph_value": tokens_all / (graph_ms / 1e3),
                "graph_ms_per_step": graph_ms / args.steps,
                "note": "operands built once (lnet_b200_alphabet_prepare); `graph_*`: the "
                        "prepared module forward replayed from a captured CUDA graph "
                        "(lnet_b200.graph.CudaGraphForward, includes its input copy); `value` "
                        "rebuilds the operands in every step"}

    # ---- image configuration: the forward from uint8 images already in HBM, with the
    # normalise + patchify inside the fused writer (lnet_b200_alphabet_forward_images)
    # and, beside it, the two-kernel form (lnet_b200_patchify_images, then the forward
    # on the bf16 tokens)
    images_res = None
    if cfg["images"] and b_loc > 0:
        from lnet_b200.images import IMAGENET_MEAN, IMAGENET_STD

        img_dev = make_images(cfg, dev)[lo:hi].contiguous()
        hh, ww = int(img_dev.shape[1]), int(img_dev.shape[2])
        mean_c = (ctypes.c_float * 3)(*IMAGENET_MEAN)
        std_c = (ctypes.c_float * 3)(*IMAGENET_STD)
        n_i = ctypes.c_size_t(0)
        _lib.check(lib.lnet_b200_alphabet_images_workspace_size(
            ctypes.byref(params), b_loc, hh, ww, ctypes.byref(n_i)),
            "lnet_b200_alphabet_images_workspace_size")
        ws_i = torch.zeros(max(int(n_i.value), 1), dtype=torch.uint8, device=dev)
        logits_i = torch.empty(b_loc, cfg["K"], device=dev, dtype=torch.float32)

        def fwd_images():
            _lib.check(lib.lnet_b200_alphabet_forward_images(
                ctypes.byref(params), img_dev.data_ptr(), b_loc, hh, ww, mean_c, std_c, 0,
                ws_i.data_ptr(), int(n_i.value), logits_i.data_ptr(), None, None,
                stream.cuda_stream), "lnet_b200_alphabet_forward_images")

        tok = torch.empty(b_loc, T, cfg["C"], dtype=torch.bfloat16, device=dev)
        fwd_tok = c_abi_forward(tok)

        def fwd_two():
            _lib.check(lib.lnet_b200_patchify_images(img_dev.data_ptr(), b_loc, hh, ww, 4,
                                                     mean_c, std_c, tok.data_ptr(),
                                                     _lib.LNET_BF16, stream.cuda_stream),
                       "lnet_b200_patchify_images")
            fwd_tok()

        for fn_w in (fwd_images, fwd_two):
            for _ in range(max(args.warmup, 3)):
                fn_w()
        img_ms = _time_steps(fwd_images, args.steps, stream, flush, world, dist, dev)
        two_ms = _time_steps(fwd_two, args.steps, stream, flush, world, dist, dev)
        images_res = {"value": tokens_all / (img_ms / 1e3), "unit": UNIT,
                      "ms_per_step": img_ms / args.steps,
                      "patchify_then_forward_ms_per_step": two_ms / args.steps,
                      "note": "uint8 images resident in HBM; `value`: patchify inside the "
                              "fused writer (lnet_b200_alphabet_forward_images); beside it "
                              "the patchify kernel then the forward on bf16 tokens"}
        del img_dev, ws_i, tok

    # ---- weak scaling: every rank its own full B-row batch (reported beside `value`)
    weak = None
    if world > 1 or args.weak:
        fwd_w = c_abi_forward(x_full)
        for _ in range(max(args.warmup, 3)):
            fwd_w()
        weak_ms = _time_steps(fwd_w, args.steps, stream, flush, world, dist, dev)
        weak = {"value": B * T * world * args.steps / (weak_ms / 1e3), "unit": UNIT,
                "ms_per_step": weak_ms / args.steps, "batch_per_gpu": B,
                "global_batch": B * world}

    trace = None
    if args.trace:
        _lib.trace_enable(True)
        fwd()
        torch.cuda.synchronize()
        raw = _lib.trace_read()
        _lib.trace_enable(False)
        trace = {k: {ph: round(c / max(v["items"], 1)) for ph, c in v.items() if ph != "items"}
                 | {"items": v["items"]} for k, v in raw.items()}
    check = multi_gpu_check(model, x_full, world, rank, dev, dist) if not args.skip_e2e else None
    if args.skip_e2e:
        if rank == 0:
            print(json.dumps({"value": value, "ms_per_step": total_ms / args.steps,
                              "prepared": prepared, "images": images_res,
                              "weak_scaling": weak,
                              "kernels": _lib_kernels(prof), "trace_cycles_per_item": trace}),
                  flush=True)
        if world > 1:
            dist.destroy_process_group()
        return 0

    # ---- end to end through the public module API: this rank's rows copied from pinned host
    # memory (uint8 images for the image config, GPU normalise + patchify) and the logits
    # copied back, every step; the copy of step k+1 overlaps the forward of step k
    from lnet_b200.pipeline import run_pipelined

    model.prepare_for_inference_(sequence_length=T, batch_size=b_loc)  # serving setup
    if cfg["images"]:
        src_host = make_images(cfg, "cpu")[lo:hi].contiguous().pin_memory()
        fn = model.forward_images
    else:
        src_host = x.cpu().pin_memory()
        fn = model
    h2d_bytes = src_host.numel() * src_host.element_size()
    with torch.no_grad():
        warm = max(args.warmup, 3)
        run_pipelined(fn, [src_host] * warm,
                      [torch.empty(b_loc, cfg["K"]).pin_memory() for _ in range(warm)], dev)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        outs = [torch.empty(b_loc, cfg["K"], dtype=torch.float32).pin_memory()
                for _ in range(args.steps)]
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        run_pipelined(fn, [src_host] * args.steps, outs, dev, start_event=e0)
        e1.record(stream)
        torch.cuda.synchronize()
    e2e_local_ms = e0.elapsed_time(e1)
    e2e_ms = torch.tensor([e2e_local_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_value = tokens_all / (float(e2e_ms.item()) / 1e3)
    h2d_gbs = torch.tensor([h2d_bytes * args.steps / (e2e_local_ms / 1e3) / 1e9], device=dev,
                           dtype=torch.float64)
    if world > 1:
        dist.all_reduce(h2d_gbs, op=dist.ReduceOp.MIN)

    if rank == 0:
        # dominant kernel during the timed region
        dom = max(prof.items(), key=lambda kv: kv[1][0]) if prof else ("", (0.0, 1))
        name, (k_ms, k_n) = dom
        avg_s = k_ms / max(k_n, 1) / 1e3
        kcfg = dict(cfg, B=b_loc)
        alg = algorithmic_bytes(name, kcfg)
        peak, peak_kind = measured_peaks()
        achieved = alg / avg_s / 1e9 if alg and avg_s > 0 else None
        roofline = {
            "bound": "hbm", "kernel": name,
            "achieved": achieved, "peak": peak, "unit": "GB/s",
            "frac": achieved / peak if achieved else None,
            "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
            "traffic": committed_traffic(name, kcfg),
            "algorithmic_bytes_per_launch": alg,
            "avg_launch_ms": avg_s * 1e3,
            "share_of_step": k_ms / sum(v[0] for v in prof.values()) if prof else None,
        }
        kernels = {k: {"ms_total": round(v[0], 4), "launches": v[1]} for k, v in prof.items()}
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            base = CpuBaseline(cfg, args.cpu_rows or B)
            try:
                base.step()  # worker start-up and imports, untimed
                secs = base.step()
            finally:
                base.close()
            cpu = {"value": base.rows * T / secs, "unit": UNIT, "cores": base.cores,
                   "kind": "port", "sample": base.describe(secs, 1)}
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": cfg["dtype"], "data": "synthetic (uint8 images / N(0,1), random-init weights)",
            "config": {"workload": cfg["workload"], "global_batch": B,
                       "batch_per_gpu": [shard_bounds(B, world, r)[1] - shard_bounds(B, world, r)[0]
                                         for r in range(world)],
                       "seq_len": T, "raw_channels": cfg["C"], "model_dim": cfg["D"],
                       "modes": cfg["M"], "classes": cfg["K"], "parallelism": f"batch{world}",
                       "l2": "256 MiB flush between steps, outside the per-step event pair"},
            "e2e": {"value": e2e_value, "unit": UNIT,
                    "input": "uint8 images [B,224,224,3] (normalise + patchify inside the "
                             "fused writer)"
                             if cfg["images"] else "tokens",
                    "overlap": "copy of step k+1 overlaps the forward of step k",
                    "module": "B200Alphabet after prepare_for_inference_",
                    "h2d_bytes_per_step": h2d_bytes * world if B % world == 0 else None,
                    "h2d_bytes_per_step_rank0": h2d_bytes,
                    "h2d_gbs_per_rank_min": float(h2d_gbs.item()),
                    "d2h_bytes_per_step": B * cfg["K"] * 4},
            "prepared": prepared,
            "images": images_res,
            "weak_scaling": weak,
            "multi_gpu_check": check,
            "gpu_launches": launches[0],
            "roofline": roofline,
            "clocks": clocks.summary(),
            "kernels": kernels,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


def run_split(args, cfg):
    """``--split time|channel`` (config 5's multi-GPU variants): every rank holds the
    whole request and runs its share of the split forward through the module-level
    API (lnet_b200.timesplit / lnet_b200.channelsplit), collectives included in the
    timed region; time = max over ranks of the summed per-step CUDA-event times.
    Rank 0 also compares the split logits with its unsplit forward of the same rows."""
    import torch
    import torch.distributed as dist

    from lnet_b200.channelsplit import channelsplit_forward
    from lnet_b200.timesplit import timesplit_forward

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    model = build_model(cfg, dev)
    x = make_inputs(cfg, dev)
    fn = timesplit_forward if args.split == "time" else channelsplit_forward
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    with torch.no_grad():
        for _ in range(max(args.warmup, 3)):
            fn(model, x)
        with ClockSampler(local) as clocks:
            total_ms = _time_steps(lambda: fn(model, x), args.steps, stream, flush, world, dist,
                                   dev)
        out = fn(model, x)
        err = None
        if rank == 0:
            ref = model(x)
            err = float((out - ref).abs().max() / ref.abs().max())
    if rank == 0:
        B, T = cfg["B"], cfg["T"]
        print(json.dumps({
            "metric": METRIC, "value": B * T * args.steps / (total_ms / 1e3), "unit": UNIT,
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": total_ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": cfg["dtype"],
            "data": "synthetic", "config": {"workload": cfg["workload"],
                                            "parallelism": f"{args.split}-split x{world}",
                                            "path": f"lnet_b200.{args.split}split",
                                            "l2": "256 MiB flush between steps"},
            "split_vs_unsplit_rel_err": err, "clocks": clocks.summary()}), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


def _lib_kernels(prof):
    return {k: {"ms_total": round(v[0], 4), "launches": v[1]} for k, v in prof.items()}


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="4")
    ap.add_argument("--cpu-rows", type=int, default=0,
                    help="rows of the CPU baseline step (default: the whole batch)")
    ap.add_argument("--ref-rows", type=int, default=0,
                    help="rows per reference-arm step (default: the whole batch)")
    ap.add_argument("--split", choices=["batch", "time", "channel"], default="batch",
                    help="time / channel: config 5's split variants across the ranks")
    ap.add_argument("--weak", action="store_true",
                    help="also time the weak-scaling workload at N=1 (always at N>1)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=None,
                    help="global batch override (small cases for profiling only)")
    ap.add_argument("--skip-e2e", action="store_true", help="profiling runs only")
    ap.add_argument("--mode", choices=["forward", "train"], default="forward",
                    help="train: forward + backward + SGD step (one GPU, ALPHABET configs)")
    ap.add_argument("--trace", action="store_true",
                    help="after the timed region, one traced forward: per-phase cycles per item")
    args = ap.parse_args()
    if args.warmup < 3:
        log("warmup raised to 3 (minimum)")
        args.warmup = 3
    cfg = dict(CONFIGS[args.config])
    if args.batch:
        cfg["B"] = args.batch
        cfg["workload"] = cfg["workload"].replace(f"_b{CONFIGS[args.config]['B']}_",
                                                  f"_b{args.batch}_")
    if args.mode == "train":
        if cfg.get("laplace"):
            log("--mode train covers the ALPHABET configs (2, 3, 4, 5)")
            return 2
        return run_train(args, cfg)
    if args.split != "batch":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable":
                              "the split variants are timed on the GPU path only"}), flush=True)
            return 0
        return run_split(args, cfg)
    if args.impl == "reference" and not (cfg.get("meta") or cfg.get("laplace")):
        return run_reference(args, cfg)
    if cfg.get("meta") or cfg.get("laplace"):
        return run_module(args, cfg)
    return run_b200(args, cfg)


if __name__ == "__main__":
    sys.exit(main())
