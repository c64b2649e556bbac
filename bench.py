"""Benchmark: plans/sec and p50 plan latency of the LeWM iCEM planning hot path.

Workload (one "step" = one full iCEM plan for one env on each GPU):
  LeWM predictor (width 192, 6 layers, 16 heads x 64, MLP 4x, AdaLN-zero action
  conditioning, action dim 2 x frameskip 5 = 10), horizon 5, history 1, bucketed
  iCEM 300 -> 60 samples over 30 iterations (2820 model-cost evaluations), 30
  elites, brown colored noise (beta 2) over raw time, elite retention 3 (10% of
  30), bf16 rollout with fp32 costs / ranking, in-kernel Philox noise.
  Synthetic random-init weights and N(0,1) latents (no checkpoint / dataset).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Multi-GPU: one process per GPU (torchrun); each rank plans its own env (weak
scaling, no collective on the plan path); time is the max over ranks.
"""

from __future__ import annotations

import argparse
import json
import os
import platform
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "plans/sec and p50 plan latency (ms), 300-sample iCEM H=5"
WORKLOAD = "icem_bucketed_300_1env_bf16"
# Canonical algorithmic FLOPs per candidate (width 192, 6 layers, H=1, T=5): new window
# tokens 1+1+1+3+3 = 9 through the 6 blocks, AdaLN for 5 action tokens x 6 layers,
# Embedder for 5 action tokens.
D, L, INNER, MLP, A, T = 192, 6, 1024, 768, 10, 5
F_BLOCK_TOKEN = 2 * (D * 3 * INNER + INNER * D + 2 * D * MLP)  # per token per layer
F_CANON = 9 * L * F_BLOCK_TOKEN + T * L * 2 * D * 6 * D + T * 2 * (A * A + A * 4 * D + 4 * D * D)


# DRAM bytes (read + write) of one launch of the dominant kernel classes, from the ncu
# captures summarised in profiles/k_qkv_attn_s60_w3_6tiles.md, profiles/k_ffn_s60_w3_6tiles.md
# and profiles/k_partial_gemm_outproj_fc2_s300_w3_8tiles.md (ncu flushes L2 between passes,
# so these are cold-cache first-touch bytes; the timed run keeps weights in L2).
NCU_TRAFFIC = {
    "qkv_attn": {"bytes": 2121728, "launch": "QKV + attention, 180 rows (60 candidates x window 3), 6 tiles x 16 heads"},
    "ffn": {"bytes": 1268480, "launch": "fused FFN, 180 rows (60 candidates x window 3), 6 tiles x 4 hidden quarters"},
    "out_proj": {"bytes": 2382592, "launch": "out-proj K halves, 900 rows (300 candidates x window 3), 8 tiles"},
    "fc2": {"bytes": 1792768, "launch": "FC2 hidden quarters, 900 rows (300 candidates x window 3), 8 tiles"},
}


def percentile(values, q):
    """Interpolated percentile (reference tools/benchmarks/metrics.py:64-76)."""
    xs = sorted(values)
    if not xs:
        return None
    pos = (len(xs) - 1) * q / 100.0
    lo, hi = int(np.floor(pos)), int(np.ceil(pos))
    return xs[lo] + (xs[hi] - xs[lo]) * (pos - lo)


def plan_options():
    from lewm_flash_b200.runtime import PlanOptions

    return PlanOptions(num_samples=300, topk=30, n_steps=30, sample_decay=1.25, sample_count_bucket_size=60,
                       elite_retention=3, beta=2.0, time_axis="raw", action_block=5, seed=0)


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled while the timed region runs.

    NVML is polled every 10 ms (read-only queries on the device matched by UUID, so the
    index is right under CUDA_VISIBLE_DEVICES); without NVML, nvidia-smi every 200 ms.
    """

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpu_index: int, uuid: str | None = None):
        self.gpu = gpu_index
        self.uuid = uuid
        self.rows = []  # (sm_mhz, max_mhz, {reason: active})
        self.source = "nvidia-smi"
        self._stop = threading.Event()
        self._nvml = None
        try:
            import pynvml
            pynvml.nvmlInit()
            h = (pynvml.nvmlDeviceGetHandleByUUID(self.uuid) if self.uuid
                 else pynvml.nvmlDeviceGetHandleByIndex(self.gpu))
            self._nvml = (pynvml, h)
            self.source = "nvml"
        except Exception:
            self._nvml = None
        self._t = threading.Thread(target=self._run, daemon=True)

    def _sample_nvml(self):
        nv, h = self._nvml
        sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
        mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
        masks = (nv.nvmlClocksEventReasonHwSlowdown, nv.nvmlClocksEventReasonHwThermalSlowdown,
                 nv.nvmlClocksEventReasonSwThermalSlowdown, nv.nvmlClocksEventReasonSwPowerCap)
        self.rows.append((float(sm), float(mx), {n: bool(bits & m) for n, m in zip(self.REASONS, masks)}))

    def _sample_smi(self):
        out = subprocess.run(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                              "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5)
        for line in out.stdout.strip().splitlines():
            r = [x.strip() for x in line.split(",")]
            self.rows.append((float(r[1]), float(r[2]),
                              {n: v.lower() in ("active", "1", "yes") for n, v in zip(self.REASONS, r[5:9])}))

    def _run(self):
        period = 0.01 if self._nvml else 0.2
        while not self._stop.is_set():
            try:
                self._sample_nvml() if self._nvml else self._sample_smi()
            except Exception:
                pass
            self._stop.wait(period)

    def __enter__(self):
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        sms = [r[0] for r in self.rows]
        mx = self.rows[-1][1] if self.rows else None
        reasons = sorted({n for r in self.rows for n, on in r[2].items() if on})
        return {"sm_mhz": percentile(sms, 50) if sms else None, "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(sms), "source": self.source}


def measured_peak_tflops() -> float:
    """Dense bf16 TFLOP/s measured on this pool's B200s (burst), else the earlier fallback."""
    try:
        return float(json.loads((REPO / "MEASURED_PEAKS.json").read_text())["bf16_tflops"])
    except Exception:
        return 1590.0


def l2_flush(buf):
    buf.add_(1.0)  # write 256 MiB (> 126 MB L2) between timed plans


def cpu_info():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return platform.processor()


def run_cpu_plan(n_plans: int):
    """The oracle port (numpy) of the reference iCEM chain, on the host cores."""
    from lewm_flash_b200.model import ModelDesc, synthetic_state_dict
    from oracle import icem_oracle as io
    from oracle import lewm_oracle as lo

    desc = ModelDesc()
    sd = synthetic_state_dict(desc, 0)
    rng = np.random.default_rng(0)
    emb = rng.standard_normal((1, 1, desc.dim)).astype(np.float32)
    goal = rng.standard_normal((1, 1, desc.dim)).astype(np.float32)
    counts = io.sample_counts(30, 300, 30, 1.25, 60)
    times = []
    for _ in range(n_plans):
        white = [rng.standard_normal((1, c, 2, 25)) for c in counts]
        noise = [io.color_white_noise(w, 5, 10, 2.0, 5, "raw") for w in white]
        mean = np.zeros((1, 5, 10), np.float32)
        var = np.ones_like(mean)
        t0 = time.perf_counter()
        io.run_static_icem_chain(lambda e, g, c: lo.get_cost_from_embeddings(e, g, c, sd, desc), emb, goal, mean,
                                 var, noise, topk=30, elite_retention=3)
        times.append(time.perf_counter() - t0)
    return times


def reference_gpu_arm(args):
    """--impl reference-gpu: the reference's own PyTorch path for the same plan on this GPU.

    ICEMSolver.solve (lewm/solvers/icem.py) from the installed reference package in
    baseline/_ref, with the same solver settings, bf16 model-cost autocast and
    float32 matmul precision "high", timed end to end per plan (CUDA events around
    solve, batch of one env, p50 over at least 50 plans) eager and with get_cost_from_embeddings under
    torch.compile(mode="reduce-overhead"), prewarmed on the bucket sizes
    300/240/180/120/60 as the reference's benchmark does
    (tools/benchmarks/lewm_plan_benchmark.py:596-700). A comparator for the
    single-env latency target; the driver's reference arm is the CPU path
    (--impl reference). Same synthetic weights and latents as the main arm."""
    ref = REPO / "baseline" / "_ref"
    if not (ref / "lewm" / "jepa.py").is_file():
        print(json.dumps({"impl": "reference_gpu", "unavailable": "reference not installed in baseline/_ref"}))
        return 0
    sys.path.insert(0, str(ref))
    from types import SimpleNamespace

    import torch
    from lewm.jepa import JEPA
    from lewm.module import ARPredictor, Embedder
    from lewm.solvers.icem import ICEMSolver

    from lewm_flash_b200.model import ModelDesc, synthetic_state_dict

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    desc = ModelDesc()
    pred = ARPredictor(num_frames=desc.num_frames, depth=desc.depth, heads=desc.heads, mlp_dim=desc.mlp_dim,
                       input_dim=desc.dim, hidden_dim=desc.dim, dim_head=desc.dim_head)
    enc = Embedder(input_dim=desc.action_dim, smoothed_dim=desc.smoothed_dim, emb_dim=desc.dim,
                   mlp_scale=desc.embed_hidden // desc.dim)
    model = JEPA(encoder=torch.nn.Identity(), predictor=pred, action_encoder=enc, pred_proj=None)
    model.load_state_dict({k: torch.from_numpy(v) for k, v in synthetic_state_dict(desc, 0).items()}, strict=True)
    model = model.to(dev).eval()
    torch.set_float32_matmul_precision("high")
    model.set_model_cost_autocast("bf16")
    # cached latents: get_cost goes straight to get_cost_from_embeddings
    model.set_embedding_cache(True).set_compile_cost(True)

    class Box:
        def __init__(self, shape):
            self.shape = shape
            self.low = -np.inf * np.ones(shape, dtype=np.float32)
            self.high = np.inf * np.ones(shape, dtype=np.float32)

    solver = ICEMSolver(model=model, batch_size=1, num_samples=300, n_steps=30, topk=30, device=dev, seed=0,
                        elite_retention=3, colored_noise="brown", colored_noise_time="raw", sample_decay=1.25,
                        sample_count_bucket_size=60)
    solver.configure(action_space=Box((1, desc.action_dim // 5)), n_envs=1,
                     config=SimpleNamespace(horizon=5, action_block=5))
    rng = np.random.default_rng(100)
    emb = torch.as_tensor(rng.standard_normal((1, 1, desc.dim)), dtype=torch.float32, device=dev)
    goal = torch.as_tensor(rng.standard_normal((1, 1, desc.dim)), dtype=torch.float32, device=dev)

    def plans(n):
        ms = []
        for _ in range(n):
            info = {"emb": emb, "goal_emb": goal, "pixels": torch.zeros(1, 1, device=dev),
                    "goal": torch.zeros(1, 1, device=dev)}
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            with torch.inference_mode():
                solver.solve(info)
            b.record()
            torch.cuda.synchronize(dev)
            ms.append(a.elapsed_time(b))
        return ms

    steps = max(args.steps, 50)  # p50 over at least 50 plans
    plans(max(args.warmup, 2))
    eager = plans(steps)
    out = {"impl": "reference_gpu", "metric": "p50 plan latency (ms), 300-sample iCEM H=5, 1 env",
           "unit": "ms", "higher_is_better": False, "steps": steps, "warmup": max(args.warmup, 2),
           "eager_ms": eager, "eager_p50_ms": percentile(eager, 50),
           "settings": "ICEMSolver.solve, bf16 model-cost autocast, matmul precision high, cached latents"}
    try:
        model.get_cost_from_embeddings = torch.compile(model.get_cost_from_embeddings, mode="reduce-overhead",
                                                       fullgraph=False)
        for n in (300, 240, 180, 120, 60):
            with torch.inference_mode():
                model.get_cost_from_embeddings(torch.zeros(1, 1, desc.dim, device=dev),
                                               torch.zeros(1, 1, desc.dim, device=dev),
                                               torch.zeros(1, n, 5, desc.action_dim, device=dev))
        torch.cuda.synchronize(dev)
        plans(max(args.warmup, 2))
        comp = plans(steps)
        out.update({"compiled_ms": comp, "compiled_p50_ms": percentile(comp, 50)})
    except Exception as exc:  # torch.compile unavailable or failing on the box: say so
        out["compiled"] = f"failed: {type(exc).__name__}: {str(exc)[:200]}"
    print(json.dumps(out))
    return 0


def reference_arm(args, rank, world):
    """--impl reference: the reference algorithm's CPU implementation (numpy oracle port) on host cores."""
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    run_cpu_plan(1) if args.warmup > 0 else None
    times = run_cpu_plan(max(args.steps, 1))
    per = float(np.mean(times))
    value = 1.0 / per
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "plans/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per * 1e3,
        "p50_plan_ms": percentile([t * 1e3 for t in times], 50), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "envs_per_gpu": 1, "candidates_per_plan": 2820},
        "cpu_baseline": {"value": value, "unit": "plans/s", "cores": threads, "kind": "port",
                         "sample": f"{len(times)} full plans (2820 candidates each) on {cpu_info()}"},
        "e2e": {"value": value, "unit": "plans/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def model_cost_case(S, repeat, envs=1):
    """R predictor rollouts of S candidates per env: 1 env with history 1 (5 calls x 6 layers,
    windows 1, 2, 3, 3, 3), or B envs with history 3 (3 calls x 6 layers, windows 3, 3, 3).
    A fixed launch sequence for ncu captures of one kernel at a known geometry."""
    import torch

    from lewm_flash_b200.model import ModelDesc, synthetic_state_dict
    from lewm_flash_b200.runtime import Runtime

    dev = torch.device("cuda", 0)
    desc = ModelDesc()
    rt = Runtime(desc, synthetic_state_dict(desc, 0), dev)
    rng = np.random.default_rng(7)
    hist = 1 if envs == 1 else 3
    emb = torch.as_tensor(rng.standard_normal((envs, hist, desc.dim)), dtype=torch.float32, device=dev)
    goal = torch.as_tensor(rng.standard_normal((envs, 1, desc.dim)), dtype=torch.float32, device=dev)
    cand = torch.as_tensor(rng.standard_normal((envs, S, 5, desc.action_dim)), dtype=torch.float32, device=dev)
    ms = []
    for _ in range(repeat):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        costs = rt.model_cost(emb, goal, cand)
        b.record()
        torch.cuda.synchronize(dev)
        ms.append(a.elapsed_time(b))
    rt.sync()
    print(json.dumps({"case": "model_cost", "envs": envs, "samples": S, "ms": ms, "cost0": float(costs[0, 0])}))
    return 0


def encoder_case(n_img: int, repeat: int) -> int:
    """``--encoder N``: N images through the observation encoder, `repeat` times (for ncu)."""
    import torch

    from lewm_flash_b200.encoder import B200Encoder, EncoderDesc, flat_weights, synthetic_weights

    dev = torch.device("cuda", 0)
    desc = EncoderDesc()
    vit, proj = synthetic_weights(desc, 0)
    enc = B200Encoder(desc, flat_weights(vit, proj, desc), dev)
    pix = torch.as_tensor(np.random.default_rng(17).standard_normal((n_img, 3, 224, 224), dtype=np.float32),
                          device=dev)
    ms = []
    for _ in range(repeat):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        out = enc.encode_pixels(pix)
        b.record()
        enc.sync()
        ms.append(a.elapsed_time(b))
    frames = torch.as_tensor(np.random.default_rng(18).integers(0, 256, size=(n_img, 224, 224, 3), dtype=np.uint8),
                             device=dev)
    host_f32 = pix.cpu().pin_memory()
    host_u8 = frames.cpu().pin_memory()

    def ev_ms(fn):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        enc.sync()
        return a.elapsed_time(b)

    phases = {}
    for name, fn in (("encode_frames_u8", lambda: enc.encode_frames(frames)),
                     ("h2d_f32", lambda: host_f32.to(dev, non_blocking=True)),
                     ("h2d_u8", lambda: host_u8.to(dev, non_blocking=True))):
        ev_ms(fn)
        phases[name] = [ev_ms(fn) for _ in range(repeat)]
    print(json.dumps({"case": "encoder", "images": n_img, "ms": ms, "emb0": float(out[0, 0]), "phases_ms": phases}))
    return 0


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference", "reference-gpu"])
    ap.add_argument("--cpu-baseline-plans", type=int, default=2)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--model-cost", type=int, default=0, metavar="S",
                    help="profiling case: time R model-cost calls of S candidates per env (horizon 5; 1 env "
                         "with history 1, or --envs B with history 3) and exit; no bench line")
    ap.add_argument("--encoder", type=int, default=0, metavar="N",
                    help="profiling case: run the observation encoder R times on N 224 px images and exit; "
                         "no bench line")
    ap.add_argument("--envs", type=int, default=1)
    ap.add_argument("--repeat", type=int, default=3)
    args = ap.parse_args()
    if args.model_cost:
        return model_cost_case(args.model_cost, args.repeat, args.envs)
    if args.encoder:
        return encoder_case(args.encoder, args.repeat)

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        return reference_arm(args, rank, world)
    if args.impl == "reference-gpu":
        return reference_gpu_arm(args)
    if args.warmup < 3:
        print("warmup must be >= 3", file=sys.stderr)
        return 2

    import torch

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    from lewm_flash_b200 import _lib
    from lewm_flash_b200.model import ModelDesc, synthetic_state_dict
    from lewm_flash_b200.runtime import Runtime
    from lewm_flash_b200.solver import B200ICEMSolver

    desc = ModelDesc()
    rt = Runtime(desc, synthetic_state_dict(desc, 0), dev)
    opts = plan_options()
    rng = np.random.default_rng(100 + rank)
    emb = torch.as_tensor(rng.standard_normal((1, 1, desc.dim)), dtype=torch.float32, device=dev)
    goal = torch.as_tensor(rng.standard_normal((1, 1, desc.dim)), dtype=torch.float32, device=dev)
    mean = torch.zeros(1, 5, 10, device=dev)
    std = torch.ones(1, 5, 10, device=dev)
    flush = torch.zeros(64 * 1024 * 1024, device=dev)  # 256 MiB
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if dist is not None:
            dist.barrier()

    # ---------------------------------------------------------------- device-resident plans
    for i in range(args.warmup):
        rt.plan(opts, emb, goal, mean, std, plan_index=i)
    rt.sync()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(local, "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)) as clocks:
        t_all0 = torch.cuda.Event(enable_timing=True)
        t_all1 = torch.cuda.Event(enable_timing=True)
        t_all0.record(stream)
        for i in range(args.steps):
            l2_flush(flush)
            ev[i][0].record(stream)
            rt.plan(opts, emb, goal, mean, std, plan_index=1000 + i)
            ev[i][1].record(stream)
        t_all1.record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    rt.sync()
    plan_ms = [a.elapsed_time(b) for a, b in ev]
    busy_ms = float(sum(plan_ms))
    worst = torch.tensor([busy_ms], device=dev)
    if dist is not None:
        dist.all_reduce(worst, op=dist.ReduceOp.MAX)
    worst_ms = float(worst.item())
    value = world * args.steps / (worst_ms / 1e3)
    p50 = percentile(plan_ms, 50)

    # ---------------------------------------------------------------- end to end through the solver API
    solver = B200ICEMSolver(rt, num_samples=300, n_steps=30, topk=30, elite_retention=3, colored_noise="brown",
                            colored_noise_time="raw", sample_decay=1.25, sample_count_bucket_size=60, seed=0,
                            device=dev)

    class Box:
        shape = (1, 2)
        low = -np.ones((1, 2), np.float32)
        high = np.ones((1, 2), np.float32)

    class Cfg:
        horizon, action_block = 5, 5

    solver.configure(action_space=Box(), n_envs=1, config=Cfg())
    host_emb = emb.cpu().pin_memory()
    host_goal = goal.cpu().pin_memory()
    info = {"emb": host_emb, "goal_emb": host_goal}
    for _ in range(args.warmup):
        solver.solve(info)
    barrier()
    e2e_ms = []
    for i in range(args.steps):
        l2_flush(flush)
        torch.cuda.synchronize(dev)
        t0 = time.perf_counter()
        out = solver.solve(info)  # H2D of emb/goal/mean/var, plan, D2H of actions/var/costs
        e2e_ms.append((time.perf_counter() - t0) * 1e3)
    worst_e2e = torch.tensor([sum(e2e_ms)], device=dev)
    if dist is not None:
        dist.all_reduce(worst_e2e, op=dist.ReduceOp.MAX)
    e2e_value = world * args.steps / (float(worst_e2e.item()) / 1e3)
    h2d = host_emb.numel() * 4 + host_goal.numel() * 4 + 2 * 5 * 10 * 4
    d2h = out["actions"].numel() * 4 + out["var"][0].numel() * 4 + len(out["costs"]) * 4

    # ---------------------------------------------------------------- batched planning (64 envs, history 3)
    batched = batched_pass(rt, dev, args.steps, args.warmup, flush)

    # ---------------------------------------------------------------- observation encoder (64 images, 224 px)
    encoder = encoder_pass(dev, args.steps, args.warmup, flush)

    # ---------------------------------------------------------------- per-kernel-class timing pass (diagnostic, last)
    kinfo = kernel_class_pass(rt, opts, emb, goal, mean, std, dev)
    per_plan_launches = kinfo["launches_per_plan"]
    flops_plan = F_CANON * 2820
    line = {
        "metric": METRIC, "value": value, "unit": "plans/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": worst_ms / args.steps, "p50_plan_ms": p50,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init weights, N(0,1) latents)",
        "config": {"workload": WORKLOAD, "envs_per_gpu": 1, "candidates_per_plan": 2820, "horizon": 5,
                   "history": 1, "topk": 30, "iterations": 30, "colored_noise": "brown/raw", "elite_retention": 3,
                   "width": 192, "layers": 6, "parallelism": f"env-sharded x{world}, no collective",
                   "l2": "256 MiB write between timed plans"},
        "e2e": {"value": e2e_value, "unit": "plans/s", "p50_ms": percentile(e2e_ms, 50),
                "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                "api": "B200ICEMSolver.solve with pinned host emb/goal"},
        "gpu_launches": int(per_plan_launches * args.steps),
        "plan_roofline": {"bound": "tensor", "achieved": flops_plan / (p50 / 1e3) / 1e12,
                          "peak": kinfo["peak"], "unit": "TFLOP/s",
                          "frac": flops_plan / (p50 / 1e3) / 1e12 / kinfo["peak"],
                          "flops_per_plan": flops_plan},
        "roofline": kinfo["roofline"],
        "kernel_classes": kinfo["classes"],
        "batched": batched,
        "encoder": encoder,
        "clocks": clocks.summary(),
    }
    if rank == 0 and not args.no_cpu_baseline:
        times = run_cpu_plan(max(args.cpu_baseline_plans, 1))
        line["cpu_baseline"] = {"value": 1.0 / float(np.mean(times)), "unit": "plans/s",
                                "cores": os.cpu_count() or 1, "kind": "port",
                                "sample": f"{len(times)} full plans (2820 candidates) of the numpy oracle port "
                                          f"on {cpu_info()}"}
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    rt.close()
    return 0


def batched_pass(rt, dev, steps, warmup, flush, n_envs=64, history=3):
    """Batched planning (64 independent envs with their own N(0,1) latents, history 3): one
    plan call solves every env; device-resident inputs, L2 flushed between calls."""
    import torch

    opts = plan_options()
    rng = np.random.default_rng(7)
    emb = torch.as_tensor(rng.standard_normal((n_envs, history, 192)), dtype=torch.float32, device=dev)
    goal = torch.as_tensor(rng.standard_normal((n_envs, 1, 192)), dtype=torch.float32, device=dev)
    mean = torch.zeros(n_envs, 5, 10, device=dev)
    std = torch.ones(n_envs, 5, 10, device=dev)
    for i in range(max(warmup, 1)):
        rt.plan(opts, emb, goal, mean, std, plan_index=5000 + i)
    n = max(1, min(steps, 5))
    stream = torch.cuda.current_stream(dev)
    ms = []
    for i in range(n):
        l2_flush(flush)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        rt.plan(opts, emb, goal, mean, std, plan_index=6000 + i)
        b.record(stream)
        torch.cuda.synchronize(dev)
        ms.append(a.elapsed_time(b))
    rt.sync()
    p50 = percentile(ms, 50)
    return {"workload": f"icem_bucketed_300_{n_envs}env_h{history}_bf16", "envs": n_envs, "history": history,
            "plans_per_s": n_envs / (p50 / 1e3), "p50_call_ms": p50, "calls": n,
            "note": "one plan call solves all envs; per-GPU throughput, device-resident inputs"}


def encoder_pass(dev, steps, warmup, flush, n_img=64):
    """Observation encoder (ViT-tiny 224 px / patch 14, 12 layers, 2048-wide BatchNorm projector)
    on one observation per env of the 64-env batch: device-timed with resident pixels, end to
    end from pinned host pixels, and the same modules in eager PyTorch (transformers ViTModel)
    on the same GPU for comparison."""
    import torch

    from lewm_flash_b200.encoder import (B200Encoder, EncoderDesc, encoder_flops, encoder_launches, flat_weights,
                                         synthetic_weights)

    desc = EncoderDesc()
    vit, proj = synthetic_weights(desc, 0)
    enc = B200Encoder(desc, flat_weights(vit, proj, desc), dev)
    rng = np.random.default_rng(17)
    host = torch.as_tensor(rng.standard_normal((n_img, 3, 224, 224), dtype=np.float32)).pin_memory()
    pix = host.to(dev)
    out_host = torch.empty(n_img, desc.proj_out).pin_memory()
    stream = torch.cuda.current_stream(dev)
    for _ in range(max(warmup, 1)):
        enc.encode_pixels(pix)
    enc.sync()
    n = max(5, min(steps, 20))

    def timed(fn):
        ms = []
        for _ in range(n):
            l2_flush(flush)
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(stream)
            fn()
            b.record(stream)
            torch.cuda.synchronize(dev)
            ms.append(a.elapsed_time(b))
        return percentile(ms, 50)

    out = torch.empty(n_img, desc.proj_out, device=dev)
    dev_ms = timed(lambda: enc.encode_pixels(pix, out))

    def e2e():
        p = host.to(dev, non_blocking=True)
        enc.encode_pixels(p, out)
        out_host.copy_(out, non_blocking=True)

    e2e_ms = timed(e2e)
    frames_host = torch.as_tensor(rng.integers(0, 256, size=(n_img, 224, 224, 3), dtype=np.uint8)).pin_memory()

    def e2e_u8():  # raw frames: the policy's image transform runs inside the encoder's first kernel
        f = frames_host.to(dev, non_blocking=True)
        enc.encode_frames(f, out=out)
        out_host.copy_(out, non_blocking=True)

    for _ in range(max(warmup, 1)):
        e2e_u8()
    e2e_u8_ms = timed(e2e_u8)
    enc.sync()
    flops = encoder_flops(desc) * n_img
    peak = measured_peak_tflops()
    res = {"workload": f"vit_tiny_224_p14_12l_proj2048bn_{n_img}img", "images": n_img,
           "images_per_s": n_img / (dev_ms / 1e3), "ms_per_batch": dev_ms,
           "e2e": {"images_per_s": n_img / (e2e_ms / 1e3), "ms_per_batch": e2e_ms,
                   "h2d_bytes_per_step": int(host.numel() * 4), "d2h_bytes_per_step": int(out_host.numel() * 4)},
           "e2e_uint8_frames": {"images_per_s": n_img / (e2e_u8_ms / 1e3), "ms_per_batch": e2e_u8_ms,
                                "h2d_bytes_per_step": int(frames_host.numel()),
                                "d2h_bytes_per_step": int(out_host.numel() * 4),
                                "api": "B200Encoder.encode_frames (uint8 HWC frames, ImageNet normalization fused)"},
           "roofline": {"bound": "tensor", "achieved": flops / (dev_ms / 1e3) / 1e12, "peak": peak,
                        "unit": "TFLOP/s", "frac": flops / (dev_ms / 1e3) / 1e12 / peak,
                        "flops_per_image": encoder_flops(desc)},
           "gpu_launches_per_batch": encoder_launches(desc), "l2": "256 MiB write between timed batches"}
    try:  # the same modules in eager PyTorch: transformers ViTModel + Linear/BatchNorm/GELU/Linear
        import transformers

        cfg = transformers.ViTConfig(hidden_size=192, num_hidden_layers=12, num_attention_heads=3,
                                     intermediate_size=768, image_size=224, patch_size=14, layer_norm_eps=1e-12)
        vm = transformers.ViTModel(cfg, add_pooling_layer=False).eval()
        vm.load_state_dict({k: torch.from_numpy(v) for k, v in vit.items()}, strict=True)
        pj = torch.nn.Sequential(torch.nn.Linear(192, 2048), torch.nn.BatchNorm1d(2048), torch.nn.GELU(),
                                 torch.nn.Linear(2048, 192)).eval()
        pj.load_state_dict({k.replace("net.", ""): torch.from_numpy(v) for k, v in proj.items()}, strict=False)
        vm, pj = vm.to(dev), pj.to(dev)

        def torch_fwd(autocast):
            with torch.inference_mode(), torch.autocast("cuda", dtype=torch.bfloat16, enabled=autocast):
                pj(vm(pix, interpolate_pos_encoding=True).last_hidden_state[:, 0])

        for ac in (False, True):
            for _ in range(max(warmup, 1)):
                torch_fwd(ac)
        res["torch_eager_fp32_ms"] = timed(lambda: torch_fwd(False))
        res["torch_eager_bf16_autocast_ms"] = timed(lambda: torch_fwd(True))
        del vm, pj
    except Exception as exc:  # pragma: no cover - transformers is in the image
        res["torch_eager"] = f"unavailable: {exc}"
    del enc
    return res


def kernel_class_pass(rt, opts, emb, goal, mean, std, dev):
    """Untimed pass: per-kernel-class device time of one plan via the library's event profiler."""
    import ctypes as C

    import torch

    from lewm_flash_b200 import _lib

    peaks = {}
    try:
        peaks = json.loads((REPO / "MEASURED_PEAKS.json").read_text())
    except Exception:
        pass
    peak = float(peaks.get("bf16_tflops", 1590.0))
    peak_kind = "measured" if "bf16_tflops" in peaks else "fallback"
    res = rt.profile_plan(opts, emb, goal, mean, std)
    classes = res["classes"]
    top = max(classes, key=lambda k: classes[k]["ms"])
    c = classes[top]
    achieved = c["flops"] / (c["ms"] / 1e3) / 1e12 if c["ms"] > 0 else 0.0
    ncu = NCU_TRAFFIC.get(top)
    roof = {"kernel": top, "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
            "frac": achieved / peak, "traffic": ncu["bytes"] if ncu else None,
            "traffic_launch": ncu["launch"] if ncu else None, "peak_source": peak_kind,
            "method": "CUDA events around every launch of this class in an untimed plan; "
                      "algorithmic FLOPs = valid rows x GEMM shape"}
    return {"roofline": roof, "classes": classes, "launches_per_plan": res["launches"], "peak": peak}


if __name__ == "__main__":
    raise SystemExit(main())
