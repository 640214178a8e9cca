"""Benchmark: fwd+bwd pixel-triangle evaluations/s at B=32, T=128, 256x256.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one forward + per-image MSE + analytic backward over a batch of 32
seeded synthetic scenes (benchmark config 2's headline cell, sigma 0.0015),
through the C ABI (dr_loss_backward, the fused_loss_backward semantics). The
metric counts dense pairs B*T*H*W per step, as the reference's own
"fwd+bwd pixel*triangle evals/s" would.

Timing: W untimed warm-up steps; then K steps, each preceded by an untimed L2
flush (a 256 MiB write; the working set is smaller than the 126 MB L2), each
timed with CUDA events on the launching stream; barrier + synchronize around
the timed region; the MAX over ranks. Multi-GPU (torchrun): the 32-scene batch
is split over the ranks, 32/N scenes each (strong scaling, as benchmark config 2
is stated; no data-path collective); `--scaling weak` gives every rank its own
32. Under torchrun the line also carries config 4 row-sharded over the ranks
(`config4_sharded`: the in-place NCCL all-reduce of the gradient inside the
step).

At N=1 the line carries secondary measurements: the config 1 fit (`secondary`),
every other benchmark config timed on this GPU with its oracle CPU rate on a
bounded sample (`configs`: the config 2 grid at sigma 0.0015 and 0.01, the
config 3 torch op with its e2e, config 4, config 5 at three sigmas), the box's
CPU model and core count (`host`), and the oracle's single-thread calibration
against the reference's published i9 times (`cpu_baseline.calibration`).

`e2e` is the same metric through the public torch API with host (pinned)
buffers: diffrast.torch_layer.fused_loss on CPU tensors, so every step copies
params + targets host->device and losses + grads device->host.

`--impl reference` times the reference's CPU algorithm (the C++ oracle port,
oracle/: the Rust crate cannot be built here) with every host thread, on the
same config and metric; under torchrun only rank 0 runs it.
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

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "differentiable-rasterizer_b200")
for _p in (REPO, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402

B, T, H, W, SIGMA = 32, 128, 256, 256, 0.0015
CELL = 5  # config 2 grid cell index for (T=128, 256^2)
METRIC = "fwd+bwd pixel*triangle evals/s (B=32,T=128,256^2)"
UNIT = "pair-evals/s"
FLOP_PER_PAIR = 170  # fwd 62 + bwd 108 FP32 FLOP per bounding-box pair
TRAFFIC_BYTES = 26_370_560  # DRAM bytes per raster launch (ncu, see roofline below)
REF_BUDGET_S = 120.0  # --impl reference: wall time all its steps share


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-fit", action="store_true", help="skip the secondary fit metric")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the per-config secondary lines (configs 2-5)")
    ap.add_argument("--scaling", default="strong", choices=["strong", "weak"],
                    help="N>1: split the 32-scene batch over the ranks (strong, config 2 as "
                         "BASELINE.json states it) or give every rank its own 32 (weak)")
    return ap.parse_args()


def dense_pairs(batch: int) -> int:
    return batch * T * H * W


def bbox_pairs(params: np.ndarray) -> int:
    """Bounding-box pairs (raster.rs:144-168 boxes of live triangles)."""
    from diffrast.scenes import bbox_pairs as count

    return count(params, W, H, SIGMA)


def inputs(rank: int):
    from diffrast.scenes import uniform_scenes

    params = uniform_scenes(B, T, 2000 + CELL + 1000 * rank)
    target_scenes = uniform_scenes(B, T, 3000 + CELL + 1000 * rank)
    return params, target_scenes


def echo_nccl_init(path: str, rank: int, world: int, local: int) -> None:
    """This rank's NCCL communicator set-up lines (from NCCL_DEBUG_FILE) on
    stderr, so a log shows the ranks and devices that took part."""
    import torch

    lines = []
    try:
        with open(path) as f:
            lines = [ln.rstrip() for ln in f if "Init COMPLETE" in ln or "nRanks" in ln]
    except OSError:
        pass
    ver = ".".join(str(v) for v in torch.cuda.nccl.version())
    print(f"[bench] rank {rank}/{world} on cuda:{local}, NCCL {ver}", file=sys.stderr, flush=True)
    for ln in lines[:4]:
        print(f"[bench] {ln}", file=sys.stderr, flush=True)


def rank_slice(rank: int, world: int) -> tuple[int, int]:
    """Scenes [lo, hi) of the 32-scene batch that rank `rank` of `world` owns
    under strong scaling: contiguous, as even as possible."""
    lo = rank * B // world
    return lo, (rank + 1) * B // world


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []
        self.first = 0
        self.window = "timed region"

    def start(self):
        """Starts sampling every 50 ms and returns once the first sample is in
        (at most 5 s), so that nvidia-smi's own start-up stays outside the
        timed region; samples before the next mark() are not counted."""
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
            return
        t0 = time.time()
        while not self.lines and time.time() - t0 < 5.0 and self.proc.poll() is None:
            time.sleep(0.01)

    def mark(self):
        """The timed region starts: count samples from here on."""
        self.first = len(self.lines)

    def samples(self) -> int:
        return len(self.lines) - self.first

    def extend(self, step, want: int = 2, limit_s: float = 2.0):
        """A timed region shorter than the sampling interval may hold no sample:
        keep running the same step, untimed, until `want` samples arrive (at
        most limit_s), and say so in the line."""
        if self.proc is None or self.samples() >= want:
            return
        self.window = "timed steps, continued untimed until two samples arrived"
        t0 = time.time()
        while (self.samples() < want and time.time() - t0 < limit_s
               and self.proc.poll() is None):
            step()

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
        rows = []
        for ln in self.lines[self.first:]:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, v in enumerate(r)
                          if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": rows[0][1],
                "reasons": reasons, "samples": len(rows), "window": self.window}


def peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return json.load(f)
    except OSError:
        return {}


def cpu_reference_rate(params, target, threads: int = 0, max_scenes: int = B,
                       min_seconds: float = 10.0, max_steps: int = 50):
    """The oracle's fwd+loss+bwd on the host, whole steps repeated until
    min_seconds have passed (at most max_steps): (dense pairs/s, seconds,
    scenes per step, steps)."""
    import oracle

    oracle.build()
    p, t = params[:max_scenes], target[:max_scenes]
    steps = 0
    per = []
    t0 = time.perf_counter()
    while steps < max_steps:
        ts = time.perf_counter()
        oracle.backward_batch(p, t, SIGMA, threads=threads)
        per.append(time.perf_counter() - ts)
        steps += 1
        if time.perf_counter() - t0 >= min_seconds:
            break
    dt = time.perf_counter() - t0
    cpu_reference_rate.step_ms = [1e3 * min(per), 1e3 * statistics.median(per), 1e3 * max(per)]
    return steps * dense_pairs(p.shape[0]) / dt, dt, p.shape[0], steps


def fit_metric(dev, with_cpu: bool):
    """Secondary benchmark metric: Adam fit iterations/s on config 1 (150
    triangles fitted to a 176x176 target for 800 iterations, FitConfig
    defaults), the whole loop on the device (dr_fit, one CUDA graph)."""
    import torch

    from diffrast import _native
    from diffrast.fit import mean_color, seed_colors
    from diffrast.scenes import config1_target_scene, seed_scene_geometry

    # The target is rendered by this library; the initial scene follows
    # fit.rs:356-385 (seed_colors / mean_color).
    t_dev = _native.render(torch.from_numpy(config1_target_scene(150, 0)).to(dev), 176, 176,
                           0.0015)[0].contiguous()
    target = t_dev.cpu().numpy()
    p = seed_scene_geometry(150, 1)
    seed_colors(target, p)
    bg = mean_color(target)
    p_dev = torch.from_numpy(p).to(dev)
    kw = dict(iters=800, patience=None)
    _native.fit(t_dev, p_dev, [float(v) for v in bg], **kw)  # capture + warm-up
    torch.cuda.synchronize(dev)
    reps = 3
    stream = torch.cuda.current_stream(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        rep = _native.fit(t_dev, p_dev, [float(v) for v in bg], **kw)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    dt = e0.elapsed_time(e1) / 1e3 / reps
    out = {"metric": "Adam fit iters/s (config 1: T=150, 176x176, 800 iters)",
           "value": len(rep["losses"]) / dt, "unit": "iters/s",
           "timing": "CUDA events around dr_fit (one graph launch per 800-iteration fit)",
           "final_best_loss": rep["best_loss"]}
    if with_cpu:
        import oracle

        oracle.build()
        t0 = time.perf_counter()
        r = oracle.fit(target, p, bg, oracle.FitConfig(iters=200, patience=None))
        cdt = time.perf_counter() - t0
        out["cpu_baseline"] = {"value": len(r.losses) / cdt, "unit": "iters/s", "cores": 1,
                               "kind": "port", "sample": "first 200 of the 800 iterations, "
                                                         "single thread (Fitter is sequential)"}
    return out


def forward_metric(dev, P, sm_mhz: float, sms: int) -> dict:
    """The headline cell's forward alone: `dr_render` into a (B, 3, H, W) image,
    what `torch_layer.rasterize` runs (62 FP32 FLOP and 3 SFU operations per
    bounding-box pair; the image written is 12 bytes per pixel)."""
    import torch

    from diffrast import _native
    from diffrast import scenes as S

    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    ms = time_device(lambda: _native.render(P, H, W, SIGMA, layout=_native.LAYOUT_BCHW), 50, 5,
                     flush, stream)
    n_bbox = S.bbox_pairs(P.cpu().numpy(), H, W, SIGMA)
    fp32, sfu = peaks_at(sm_mhz, sms)
    img_bytes = P.shape[0] * 3 * H * W * 4
    s = ms / 1e3
    return {"metric": "forward-only render (dr_render, BCHW, the rasterize forward)",
            "ms_per_step": ms, "dense_pair_evals_per_s": P.shape[0] * P.shape[1] * H * W / s,
            "bbox_pair_evals_per_s": n_bbox / s, "fp32_frac": n_bbox * 62 / s / fp32,
            "sfu_frac": n_bbox * 3 / s / sfu, "image_bytes": img_bytes,
            "image_write_gb_s": img_bytes / s / 1e9,
            "timing": "CUDA events, median of 50 calls, L2 flushed before each; set-up and "
                      "raster kernels"}


def host_identity() -> dict:
    """CPU model and logical core count of the box the CPU baselines run on."""
    model = None
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"cpu_model": model, "nproc": os.cpu_count()}


SFU_PER_PAIR = 7  # fwd 3 + bwd 4 MUFU operations per bounding-box pair


def peaks_at(sm_mhz: float, sms: int):
    """Nominal FP32 FLOP/s and SFU op/s at a clock: 148 SMs x 128 FP32 lanes x 2
    and 148 SMs x 16 SFU lanes on a B200."""
    return sms * 128 * 2 * sm_mhz * 1e6, sms * 16 * sm_mhz * 1e6


def time_device(fn, steps: int, warmup: int, flush, stream) -> float:
    """Median CUDA-event time of fn() in ms, L2 flushed before every call."""
    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ev = []
    for _ in range(steps):
        flush.fill_(1)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        fn()
        e1.record(stream)
        ev.append((e0, e1))
    torch.cuda.synchronize()
    return statistics.median(a.elapsed_time(b) for a, b in ev)


def cpu_sample_rate(params, target, sigma, threads: int, budget_s: float):
    """The oracle's fwd+loss+bwd on a bounded sample: the first n scenes, n
    chosen from one timed scene so that the sample takes about budget_s.
    Returns (dense pairs/s, seconds, scenes)."""
    import oracle

    B, T = params.shape[:2]
    H, W = target.shape[1], target.shape[2]
    t0 = time.perf_counter()
    oracle.backward_batch(params[:1], target[:1], sigma, threads=1)
    one = max(time.perf_counter() - t0, 1e-6)
    n = int(max(1, min(B, budget_s * min(threads, B) / one)))
    t0 = time.perf_counter()
    oracle.backward_batch(params[:n], target[:n], sigma, threads=threads)
    dt = time.perf_counter() - t0
    return n * T * H * W / dt, dt, n


def config_line(name, workload, ms, dense, bbox, sm_mhz, sms, cpu=None, **extra):
    fp32, sfu = peaks_at(sm_mhz, sms)
    s = ms / 1e3
    line = {"config": name, "workload": workload, "ms_per_step": ms,
            "dense_pair_evals_per_s": dense / s, "bbox_pair_evals_per_s": bbox / s,
            "bbox_pairs": bbox,
            "fp32_frac": bbox * FLOP_PER_PAIR / s / fp32,
            "sfu_frac": bbox * SFU_PER_PAIR / s / sfu}
    if cpu is not None:
        line["cpu_baseline"] = cpu
    line.update(extra)
    return line


def run_configs(dev, sm_mhz: float, with_cpu: bool, budget_s: float = 1.5):
    """Secondary timed lines for every benchmark configuration (BASELINE.json
    configs 2-5) on this GPU, each with its oracle CPU rate on a bounded sample
    when with_cpu. Device-resident inputs, L2 flushed before every step."""
    import numpy as np
    import torch
    import torch.nn.functional as F

    import oracle
    from diffrast import _native, torch_layer
    from diffrast import scenes as S

    if with_cpu:
        oracle.build()
    thr = oracle.num_threads() if with_cpu else 0
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    out = []

    def cpu_dict(rate, dt, n, total, threads):
        return {"value": rate, "unit": UNIT, "cores": threads, "kind": "port",
                "sample": f"{n} of {total} scenes, {dt:.2f} s"}

    # Config 2: the 9-cell grid at sigma 0.0015 and 0.01 (B=32).
    for sigma in (0.0015, 0.01):
        for ti, tris in enumerate((32, 128, 512)):
            for si, size in enumerate((64, 128, 256)):
                p, tp = S.config2_params(32, tris, ti * 3 + si)
                P = torch.from_numpy(p).to(dev)
                tgt = _native.render(torch.from_numpy(tp).to(dev), size, size, sigma)
                ms = time_device(lambda: _native.loss_backward(P, tgt, sigma), 20, 3, flush,
                                 stream)
                cpu = None
                if with_cpu:
                    rate, dt, n = cpu_sample_rate(p, tgt.cpu().numpy(), sigma, thr, budget_s / 3)
                    cpu = cpu_dict(rate, dt, n, 32, thr)
                out.append(config_line(
                    "config2", f"B=32 T={tris} {size}x{size} sigma={sigma} fwd+mse+bwd", ms,
                    32 * tris * size * size, S.bbox_pairs(p, size, size, sigma), sm_mhz, sms, cpu,
                    path=_native.query_path(32, tris, size, size)))

    # Config 3: the torch op, rasterize -> F.mse_loss -> backward at B=256.
    g = torch.Generator().manual_seed(2)
    raw = torch.randn(256, 64, 10, generator=g)
    params = torch_layer.activate(raw)
    tparams = torch_layer.random_params(256, 64, generator=torch.Generator().manual_seed(3))
    targets = torch_layer.rasterize(tparams.to(dev), 128, 128, 0.0015).detach()
    p_dev = params.to(dev)

    def op_step(p_src):
        q = p_src.detach().to(dev).requires_grad_(True)
        loss = F.mse_loss(torch_layer.rasterize(q, 128, 128, 0.0015), targets)
        loss.backward()
        return loss, q.grad

    ms = time_device(lambda: op_step(p_dev), 10, 3, flush, stream)
    p_pin = params.clone().pin_memory()
    t_pin = targets.cpu().pin_memory()

    def op_step_e2e():
        q = p_pin.to(dev, non_blocking=True).requires_grad_(True)
        tg = t_pin.to(dev, non_blocking=True)
        loss = F.mse_loss(torch_layer.rasterize(q, 128, 128, 0.0015), tg)
        loss.backward()
        return loss.item(), q.grad.cpu()

    for _ in range(3):
        op_step_e2e()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(10):
        op_step_e2e()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / 10
    p_np = params.numpy()
    cpu = None
    if with_cpu:
        rate, dt, n = cpu_sample_rate(p_np, targets.permute(0, 2, 3, 1).cpu().numpy(), 0.0015,
                                      thr, budget_s)
        cpu = cpu_dict(rate, dt, n, 256, thr)
    dense = 256 * 64 * 128 * 128
    out.append(config_line(
        "config3", "B=256 T=64 128x128 sigma=0.0015 rasterize -> F.mse_loss -> backward "
                   "(torch op, device tensors)", ms, dense,
        S.bbox_pairs(p_np, 128, 128, 0.0015), sm_mhz, sms, cpu,
        e2e={"value": dense / (e2e_ms / 1e3), "unit": UNIT, "ms_per_step": e2e_ms,
             "h2d_bytes_per_step": p_pin.numel() * 4 + t_pin.numel() * 4,
             "d2h_bytes_per_step": p_pin.numel() * 4 + 4,
             "api": "pinned host params and targets copied in, loss and params.grad read "
                    "back, every step"}))

    # Config 4: one 1024^2 scene, T=4096: fwd+bwd+Adam (one GPU).
    p4 = S.config4_params(4096, 4000)
    t4 = _native.render(torch.from_numpy(S.config4_params(4096, 4001)).to(dev), 1024, 1024,
                        0.0015)
    P4 = torch.from_numpy(p4).to(dev)
    m4, v4 = torch.zeros_like(P4), torch.zeros_like(P4)
    it = [0]

    def step4():
        losses, grads = _native.loss_backward(P4, t4, 0.0015)
        it[0] += 1
        _native.adam_step(P4, m4, v4, grads, it[0])

    ms = time_device(step4, 10, 3, flush, stream)
    cpu = None
    if with_cpu:
        t0 = time.perf_counter()
        oracle.backward_batch(p4, t4.cpu().numpy(), 0.0015, threads=1)
        dt = time.perf_counter() - t0
        cpu = {"value": 4096 * 1024 * 1024 / dt, "unit": UNIT, "cores": 1, "kind": "port",
               "sample": f"one full step, single thread (a single scene is sequential in the "
                         f"reference), {dt:.2f} s"}
    out.append(config_line("config4", "B=1 T=4096 1024x1024 sigma=0.0015 fwd+mse+bwd+Adam",
                           ms, 4096 * 1024 * 1024, S.bbox_pairs(p4, 1024, 1024, 0.0015), sm_mhz,
                           sms, cpu, path=_native.query_path(1, 4096, 1024, 1024)))

    # Config 5: B=16, T=2048, 512^2 stress at the three sigmas.
    p5 = S.config5_params(16, 2048, 5000)
    P5 = torch.from_numpy(p5).to(dev)
    for sigma in (0.00015, 0.0015, 0.015):
        t5 = _native.render(torch.from_numpy(S.config5_params(16, 2048, 5100)).to(dev), 512,
                            512, sigma)
        ms = time_device(lambda: _native.loss_backward(P5, t5, sigma), 10, 3, flush, stream)
        cpu = None
        if with_cpu:
            rate, dt, n = cpu_sample_rate(p5, t5.cpu().numpy(), sigma, thr, budget_s)
            cpu = cpu_dict(rate, dt, n, 16, thr)
        out.append(config_line("config5", f"B=16 T=2048 512x512 sigma={sigma} fwd+mse+bwd", ms,
                               16 * 2048 * 512 * 512, S.bbox_pairs(p5, 512, 512, sigma), sm_mhz,
                               sms, cpu, path=_native.query_path(16, 2048, 512, 512)))
    return out


def calibration(threads: int = 1):
    """The oracle's single-thread fwd+bwd on the reference's own bench shapes
    (Scene::random(n, bg, 0.15) small triangles, sigma 0.01) beside the
    published i9-13900 single-thread times (docs/gpu-report.txt:143,146)."""
    import numpy as np

    import oracle

    rows = []
    for size, tris, ref_ms in ((128, 64, 3.02), (256, 256, 48.25)):
        rng = np.random.default_rng(42)
        c = rng.uniform(0, 1, size=(1, tris, 1, 2))
        v = c + rng.uniform(-0.15, 0.15, size=(1, tris, 3, 2))
        p = np.concatenate([v.reshape(1, tris, 6), rng.uniform(0, 1, (1, tris, 3)),
                            rng.uniform(0.3, 0.8, (1, tris, 1))], -1).astype(np.float32)
        tgt = np.full((1, size, size, 3), 0.5, np.float32)
        oracle.backward_batch(p, tgt, 0.01, threads=threads)
        reps, t0 = 0, time.perf_counter()
        while reps < 3 or time.perf_counter() - t0 < 1.0:
            oracle.backward_batch(p, tgt, 0.01, threads=threads)
            reps += 1
        ms = 1e3 * (time.perf_counter() - t0) / reps
        rows.append({"shape": f"{size}x{size}, {tris} triangles, sigma 0.01", "oracle_ms": ms,
                     "reference_i9_ms": ref_ms, "ratio": ms / ref_ms})
    return rows


def run_reference(args, rank: int, world: int):
    """--impl reference: the reference CPU algorithm, all host threads."""
    if rank != 0:
        return
    import oracle

    oracle.build()
    params, tscenes = inputs(0)
    target = oracle.render_batch(tscenes, H, W, SIGMA)
    threads = oracle.num_threads()
    # Each step is a bounded sample: the first n scenes of the batch, n chosen
    # from a timed full step so that all steps take about REF_BUDGET_S.
    t0 = time.perf_counter()
    oracle.backward_batch(params, target, SIGMA, threads=threads)
    full = time.perf_counter() - t0
    per_step = REF_BUDGET_S / max(args.steps + args.warmup, 1)
    n = max(1, min(B, int(B * per_step / max(full, 1e-9))))
    p_s, t_s = params[:n], target[:n]
    for _ in range(max(args.warmup, 0)):
        oracle.backward_batch(p_s, t_s, SIGMA, threads=threads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        oracle.backward_batch(p_s, t_s, SIGMA, threads=threads)
        times.append(time.perf_counter() - t0)
    ms = 1e3 * statistics.mean(times)
    spread = [1e3 * min(times), 1e3 * statistics.median(times), 1e3 * max(times)]
    value = dense_pairs(n) / (ms / 1e3)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded PCG64 scenes, config 2 distribution)",
        "config": {"workload": "config2 B=32 T=128 256x256 sigma=0.0015 fwd+mse+bwd",
                   "entry": "oracle (C++ restatement of the Rust CPU path)",
                   "global_batch": B, "seq_len": None, "parallelism": "cpu threads"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{n} of the {B} scenes per step (a full step takes "
                                   f"{full:.2f} s), {args.steps} steps",
                         "step_ms_min_median_max": spread, "host": host_identity()},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference Rust crate cannot be built in this image (no cargo); timed the C++ "
                "restatement of its CPU path (oracle/diffrast_oracle.cpp)",
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    import torch

    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        if args.impl == "ours":
            # NCCL's communicator set-up lines (ranks, devices, channels) on
            # stderr, so a log shows how many ranks took part; stdout keeps the
            # one JSON line.
            import tempfile

            nccl_log = os.path.join(tempfile.gettempdir(), f"dr_bench_nccl.{os.getpid()}.log")
            os.environ["NCCL_DEBUG"] = "INFO"
            os.environ["NCCL_DEBUG_SUBSYS"] = "INIT"
            os.environ["NCCL_DEBUG_FILE"] = nccl_log
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local))
            dist.barrier()
            echo_nccl_init(nccl_log, rank, world, local)
        else:
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))

    if args.impl == "reference":
        run_reference(args, rank, world)
        if dist is not None:
            dist.destroy_process_group()
        return

    from diffrast import _native
    from diffrast import torch_layer

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    strong = world > 1 and args.scaling == "strong"
    if strong:
        lo, hi = rank_slice(rank, world)
        params_np, tscenes_np = (a[lo:hi] for a in inputs(0))
    else:
        params_np, tscenes_np = inputs(rank)
    n_local = params_np.shape[0]
    P = torch.from_numpy(params_np).to(dev)
    TS = torch.from_numpy(tscenes_np).to(dev)
    target = _native.render(TS, H, W, SIGMA)  # targets = independent scenes rendered
    grads_dummy = None
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        return _native.loss_backward(P, target, SIGMA)

    for _ in range(max(args.warmup, 3)):
        grads_dummy = step()
    torch.cuda.synchronize(dev)

    clocks = ClockSampler(local)
    clocks.start()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    clocks.mark()
    times = []
    for _ in range(args.steps):
        flush.fill_(1)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        grads_dummy = step()
        e1.record(stream)
        times.append((e0, e1))
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)

    def untimed():
        flush.fill_(1)
        step()
        torch.cuda.synchronize(dev)

    clocks.extend(untimed)
    clock_info = clocks.stop()
    total_ms = sum(a.elapsed_time(b) for a, b in times)
    t_ms = torch.tensor([total_ms], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(t_ms, op=dist.ReduceOp.MAX)
    total_ms = float(t_ms.item())
    ms_per_step = total_ms / args.steps
    global_scenes = B if strong else world * B
    value = dense_pairs(global_scenes) / (ms_per_step / 1e3)
    del grads_dummy

    # Config 4 row-sharded over the ranks: fwd+bwd, the in-place all-reduce of
    # the 4096 x 10 gradient and the loss sums, and Adam, every step.
    sharded4 = None
    if world > 1:
        from diffrast.scenes import config4_params
        from diffrast.sharded import ShardedSceneStep

        st4 = ShardedSceneStep(torch.from_numpy(config4_params(4096, 4000)).to(dev))
        t4 = _native.render(torch.from_numpy(config4_params(4096, 4001)).to(dev), 1024, 1024,
                            SIGMA)
        for _ in range(3):
            st4.step(t4, SIGMA)
        torch.cuda.synchronize(dev)
        dist.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(10):
            st4.step(t4, SIGMA)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        ms4 = torch.tensor([e0.elapsed_time(e1) / 10], dtype=torch.float64, device=dev)
        dist.all_reduce(ms4, op=dist.ReduceOp.MAX)
        sharded4 = {"config": "config4", "workload": f"B=1 T=4096 1024x1024 sigma={SIGMA} "
                    f"fwd+mse+bwd+all-reduce+Adam, tile rows sharded over {world} GPUs",
                    "ms_per_step": float(ms4.item()),
                    "dense_pair_evals_per_s": 4096 * 1024 * 1024 / (float(ms4.item()) / 1e3),
                    "collective": "NCCL all_reduce of the 4096x10 f32 gradient and the f64 "
                                  "loss sum, in place"}
        del st4, t4

    # e2e: public API with pinned host buffers (H2D of inputs, D2H of results).
    p_host = torch.from_numpy(params_np).pin_memory()
    t_host = target.cpu().pin_memory()
    # Warm-up creates the pipeline's streams, device buffers and pinned results.
    for _ in range(5):
        torch_layer.fused_loss(p_host, t_host, SIGMA)
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    e2e_steps = max(3, min(args.steps, 50))
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        losses_h, grads_h = torch_layer.fused_loss(p_host, t_host, SIGMA)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = torch.tensor([e0.elapsed_time(e1) / e2e_steps], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_ms = float(e2e_ms.item())
    h2d = p_host.numel() * 4 + t_host.numel() * 4
    d2h = losses_h.numel() * 4 + grads_h.numel() * 4
    # The box's plain pinned upload rate for the same bytes: e2e's copy bound.
    dst = torch.empty(h2d // 4, dtype=torch.float32, device=dev)
    src = torch.empty(h2d // 4, dtype=torch.float32).pin_memory()
    for _ in range(3):
        dst.copy_(src, non_blocking=True)
    torch.cuda.synchronize(dev)
    e0.record(stream)
    for _ in range(10):
        dst.copy_(src, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    h2d_gbs = h2d / (e0.elapsed_time(e1) / 10 / 1e3) / 1e9
    del dst, src

    if rank == 0:
        pk = peaks()
        n_bbox = bbox_pairs(params_np)  # this GPU's share of the batch
        sm_mhz = (clock_info or {}).get("sm_mhz") or pk.get("sm_max_mhz", 1965.0)
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        fp32_peak, sfu_peak = peaks_at(sm_mhz, sms)
        achieved = n_bbox * FLOP_PER_PAIR / (ms_per_step / 1e3)
        sfu_achieved = n_bbox * SFU_PER_PAIR / (ms_per_step / 1e3)
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "strong" if strong or world == 1 else "weak",
            "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded PCG64 scenes, config 2 distribution)",
            "config": {"workload": "config2 B=32 T=128 256x256 sigma=0.0015 fwd+mse+bwd",
                       "entry": "dr_loss_backward",
                       "global_batch": global_scenes, "seq_len": None,
                       "parallelism": (f"batch-sharded x{world}: {n_local} scenes per GPU, "
                                       "no collective"),
                       "l2": "flushed (256 MiB write) before every timed step"},
            "e2e": {"value": dense_pairs(global_scenes) / (e2e_ms / 1e3), "unit": UNIT,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "pinned_h2d_gbs": h2d_gbs,
                    "copy_bound_ms": h2d / (h2d_gbs * 1e9) * 1e3,
                    "api": "diffrast.torch_layer.fused_loss on pinned CPU tensors "
                           "(dr_loss_backward_host: chunked upload, kernels and download "
                           "in one call)"},
            "gpu_launches": 2 * args.steps,
            "roofline": {"bound": "fp32", "achieved": achieved / 1e12,
                         "peak": fp32_peak / 1e12, "unit": "TFLOP/s",
                         "frac": achieved / fp32_peak,
                         "sfu_achieved": sfu_achieved / 1e12, "sfu_peak": sfu_peak / 1e12,
                         "sfu_unit": "Tops/s", "sfu_frac": sfu_achieved / sfu_peak,
                         # dram read + write of one raster launch, ncu capture in
                         # profiles/raster_kernel_config2_b32_t128_256.md
                         "traffic": TRAFFIC_BYTES,
                         "pairs_per_step": n_bbox, "flop_per_pair": FLOP_PER_PAIR,
                         "sfu_per_pair": SFU_PER_PAIR,
                         "peak_source": f"nominal FP32 ({sms} SMs x 128 lanes x 2) and SFU "
                                        f"({sms} SMs x 16) at the sampled SM clock "
                                        f"{sm_mhz:.0f} MHz; MEASURED_PEAKS.json has no FP32 "
                                        "or SFU figure",
                         "timed": "whole step (set-up + raster kernels) per CUDA events"},
            "clocks": clock_info,
            "host": host_identity(),
        }
        if sharded4 is not None:
            line["config4_sharded"] = sharded4
        if not args.no_fit and world == 1:
            line["secondary"] = fit_metric(dev, not args.no_cpu_baseline)
        if not args.no_configs and world == 1:
            line["forward"] = forward_metric(dev, P, sm_mhz, sms)
        if not args.no_configs and world == 1:
            line["configs"] = run_configs(dev, sm_mhz, not args.no_cpu_baseline)
        if not args.no_cpu_baseline and world == 1:
            import oracle

            tgt_np = target.cpu().numpy()
            thr = oracle.num_threads()
            rate, dt, ns, nsteps = cpu_reference_rate(params_np, tgt_np, threads=thr,
                                                      max_scenes=B)
            line["cpu_baseline"] = {"value": rate, "unit": UNIT, "cores": thr, "kind": "port",
                                    "sample": f"{nsteps} full steps of {ns} scenes ({dt:.1f} s "
                                              f"wall on {thr} threads), C++ restatement of the "
                                              "Rust CPU path",
                                    "step_ms_min_median_max": cpu_reference_rate.step_ms,
                                    "calibration": calibration()}
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
