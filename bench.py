"""Benchmark: plans/sec and p50 plan latency of the LeWM iCEM planning hot path.

Workload (one "step" = one full iCEM plan for one env on each GPU):
  LeWM predictor (width 192, 6 layers, 16 heads x 64, MLP 4x, AdaLN-zero action
  conditioning), action dim 2 x frameskip 5 = 10, horizon 5, history 1, bucketed
  iCEM 300 -> 60 samples over 30 iterations (2820 model-cost evaluations), 30
  elites, brown colored noise (beta 2) over raw time, elite retention 3 (10% of
  30), bf16 rollout with fp32 costs / ranking, in-kernel Philox noise.
  Synthetic random-init weights and N(0,1) latents (no checkpoint / dataset).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Further legs of the same line: ``batched`` (64 envs with history 3 in one plan
call), ``sharded`` (1024 envs split over the ranks, each rank one batched plan
call: strong scaling, no collective), ``stress`` (width 384 / 12 layers /
horizon 10 / 3000 -> 600 samples, 32 envs per rank: 256 envs on 8 GPUs),
``encoder``, ``reference_gpu`` (the reference's own PyTorch solver on this GPU,
eager and compiled; 1 GPU only) and ``cpu_baseline`` (the reference's own solver on
the host cores).

Multi-GPU: one process per GPU (torchrun); each rank plans its own env (weak
scaling, no collective on the plan path); time is the max over ranks.

--impl reference: the reference's own ICEMSolver.solve (unmodified, from the
package installed in baseline/_ref) for the same plan on the host cores, fp32,
all host threads; rank 0 only.
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


# DRAM bytes (read + write) of one launch of the dominant kernel classes, from ncu
# captures (dram__bytes_read.sum + dram__bytes_write.sum) of one launch at the geometry
# named beside each figure (ncu flushes L2 between passes, so these are cold-cache
# first-touch bytes; the timed run keeps weights in L2).
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


REF_DIR = REPO / "baseline" / "_ref"
# Solver settings of the bench plan, as ICEMSolver keyword arguments.
ICEM_KW = dict(num_samples=300, n_steps=30, topk=30, elite_retention=3, colored_noise="brown",
               colored_noise_time="raw", sample_decay=1.25, sample_count_bucket_size=60, seed=0)


def bench_config(world):
    """The `config` of the headline line; the reference arm prints the same keys."""
    return {"workload": WORKLOAD, "envs_per_gpu": 1, "candidates_per_plan": 2820, "horizon": 5,
            "history": 1, "topk": 30, "iterations": 30, "colored_noise": "brown/raw", "elite_retention": 3,
            "width": 192, "layers": 6, "parallelism": f"env-sharded x{world}, no collective",
            "l2": "256 MiB write between timed plans"}


def bench_latents(rank, dim=192):
    rng = np.random.default_rng(100 + rank)
    return (rng.standard_normal((1, 1, dim)).astype(np.float32), rng.standard_normal((1, 1, dim)).astype(np.float32))


def reference_package():
    """The unmodified reference (lewm/...) installed in baseline/_ref, or None if absent."""
    if not (REF_DIR / "lewm" / "jepa.py").is_file():
        return None
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    from lewm import jepa, module
    from lewm.solvers import icem
    return {"jepa": jepa, "module": module, "icem": icem}


def reference_solver(ref, device, n_envs=1):
    """The reference JEPA (synthetic weights, seed 0) and its ICEMSolver at the bench settings."""
    from types import SimpleNamespace

    import torch

    from lewm_flash_b200.model import ModelDesc, synthetic_state_dict

    desc = ModelDesc()
    pred = ref["module"].ARPredictor(num_frames=desc.num_frames, depth=desc.depth, heads=desc.heads,
                                     mlp_dim=desc.mlp_dim, input_dim=desc.dim, hidden_dim=desc.dim,
                                     dim_head=desc.dim_head)
    enc = ref["module"].Embedder(input_dim=desc.action_dim, smoothed_dim=desc.smoothed_dim, emb_dim=desc.dim,
                                 mlp_scale=desc.embed_hidden // desc.dim)
    model = ref["jepa"].JEPA(encoder=torch.nn.Identity(), predictor=pred, action_encoder=enc, pred_proj=None)
    model.load_state_dict({k: torch.from_numpy(v) for k, v in synthetic_state_dict(desc, 0).items()}, strict=True)
    model = model.to(device).eval()
    # cached latents: get_cost goes straight to get_cost_from_embeddings
    model.set_embedding_cache(True).set_compile_cost(True)

    class Box:
        def __init__(self, shape):
            self.shape = shape
            self.low = -np.inf * np.ones(shape, dtype=np.float32)
            self.high = np.inf * np.ones(shape, dtype=np.float32)

    solver = ref["icem"].ICEMSolver(model=model, batch_size=n_envs, device=device, **ICEM_KW)
    solver.configure(action_space=Box((n_envs, desc.action_dim // 5)), n_envs=n_envs,
                     config=SimpleNamespace(horizon=5, action_block=5))
    return model, solver


def quiet(fn, *a, **kw):
    """Run a reference call with its progress prints sent to stderr (stdout carries the JSON line)."""
    import contextlib

    with contextlib.redirect_stdout(sys.stderr):
        return fn(*a, **kw)


def reference_cpu_plans(n_plans: int, warmup: int, rank: int = 0):
    """The reference's own ICEMSolver.solve on the host cores (fp32, every host thread), the
    bench plan with the bench's weights and latents. Falls back to the numpy oracle port of
    the same chain only when the reference package is absent. Returns (seconds per plan, info)."""
    import torch

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    ref = reference_package()
    emb_np, goal_np = bench_latents(rank)
    if ref is not None:
        _, solver = reference_solver(ref, "cpu")
        info = {"emb": torch.from_numpy(emb_np), "goal_emb": torch.from_numpy(goal_np),
                "pixels": torch.zeros(1, 1), "goal": torch.zeros(1, 1)}
        for _ in range(warmup):
            quiet(solver.solve, dict(info))
        times = []
        for _ in range(n_plans):
            t0 = time.perf_counter()
            quiet(solver.solve, dict(info))
            times.append(time.perf_counter() - t0)
        return times, {"kind": "reference", "cores": threads,
                       "sample": f"{len(times)} full plans (2820 candidates each) of the reference ICEMSolver.solve "
                                 f"(fp32, torch {torch.__version__}, {threads} threads) on {cpu_info()}"}
    # reference package absent: the numpy restatement of the same chain (one thread of numpy)
    from lewm_flash_b200.model import ModelDesc, synthetic_state_dict
    from oracle import icem_oracle as io
    from oracle import lewm_oracle as lo

    desc = ModelDesc()
    sd = synthetic_state_dict(desc, 0)
    rng = np.random.default_rng(0)
    counts = io.sample_counts(30, 300, 30, 1.25, 60)
    times = []
    for i in range(warmup + n_plans):
        noise = [io.color_white_noise(rng.standard_normal((1, c, 2, 25)), 5, 10, 2.0, 5, "raw") for c in counts]
        mean = np.zeros((1, 5, 10), np.float32)
        t0 = time.perf_counter()
        io.run_static_icem_chain(lambda e, g, c: lo.get_cost_from_embeddings(e, g, c, sd, desc), emb_np, goal_np,
                                 mean, np.ones_like(mean), noise, topk=30, elite_retention=3)
        if i >= warmup:
            times.append(time.perf_counter() - t0)
    return times, {"kind": "port", "cores": 1,
                   "sample": f"{len(times)} full plans of the numpy oracle port (reference package absent) "
                             f"on {cpu_info()}"}


def reference_gpu_pass(dev, eager_plans=20, compiled_plans=50, warmup=2):
    """The reference's own PyTorch path for the same plan on this GPU: ICEMSolver.solve from
    baseline/_ref with the same solver settings, weights and latents, bf16 model-cost autocast
    and float32 matmul precision "high", one env, CUDA events around each solve; eager, and
    with get_cost_from_embeddings under torch.compile(mode="reduce-overhead") prewarmed on the
    bucket sizes 300/240/180/120/60 as the reference's benchmark does
    (tools/benchmarks/lewm_plan_benchmark.py:596-700). The comparator of the single-env
    latency target."""
    import torch

    ref = reference_package()
    if ref is None:
        return {"unavailable": "reference not installed in baseline/_ref"}
    torch.set_float32_matmul_precision("high")
    model, solver = reference_solver(ref, dev)
    model.set_model_cost_autocast("bf16")
    emb_np, goal_np = bench_latents(0)
    emb = torch.as_tensor(emb_np, device=dev)
    goal = torch.as_tensor(goal_np, device=dev)

    def plans(n):
        ms = []
        for _ in range(n):
            info = {"emb": emb, "goal_emb": goal, "pixels": torch.zeros(1, 1, device=dev),
                    "goal": torch.zeros(1, 1, device=dev)}
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize(dev)
            a.record()
            with torch.inference_mode():
                quiet(solver.solve, info)
            b.record()
            torch.cuda.synchronize(dev)
            ms.append(a.elapsed_time(b))
        return ms

    plans(warmup)
    eager = plans(eager_plans)
    out = {"api": "reference ICEMSolver.solve (baseline/_ref), bf16 model-cost autocast, matmul precision high, "
                  "cached latents, 1 env", "eager_plans": eager_plans, "eager_p50_ms": percentile(eager, 50)}
    t0 = time.perf_counter()
    try:
        model.get_cost_from_embeddings = torch.compile(model.get_cost_from_embeddings, mode="reduce-overhead",
                                                       fullgraph=False)
        for n in (300, 240, 180, 120, 60):
            with torch.inference_mode():
                model.get_cost_from_embeddings(torch.zeros(1, 1, 192, device=dev), torch.zeros(1, 1, 192, device=dev),
                                               torch.zeros(1, n, 5, 10, device=dev))
        torch.cuda.synchronize(dev)
        plans(warmup)
        out["compile_s"] = time.perf_counter() - t0
        comp = plans(compiled_plans)
        out.update({"compiled_plans": compiled_plans, "compiled_p50_ms": percentile(comp, 50)})
    except Exception as exc:  # torch.compile unavailable or failing on the box: say so
        out["compiled"] = f"failed: {type(exc).__name__}: {str(exc)[:200]}"
    del model, solver
    torch.cuda.empty_cache()
    return out


def reference_gpu_arm(args):
    """--impl reference-gpu: only the reference_gpu leg, as its own JSON line."""
    import torch

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    out = reference_gpu_pass(dev, eager_plans=max(args.steps, 20), compiled_plans=max(args.steps, 50),
                             warmup=max(args.warmup, 2))
    out["impl"] = "reference_gpu"
    print(json.dumps(out))
    return 0


def reference_arm(args, rank, world):
    """--impl reference: the reference's own ICEMSolver.solve on the host cores (rank 0 only)."""
    if rank != 0:
        return 0
    times, info = reference_cpu_plans(max(args.steps, 1), args.warmup, rank)
    per = float(np.mean(times))
    value = 1.0 / per
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "plans/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per * 1e3,
        "p50_plan_ms": percentile([t * 1e3 for t in times], 50), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (random-init weights, N(0,1) latents)",
        "config": bench_config(world),
        "cpu_baseline": dict(info, value=value, unit="plans/s"),
        "e2e": {"value": value, "unit": "plans/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def model_cost_case(S, repeat, envs=1, mode="bf16"):
    """R predictor rollouts of S candidates per env: 1 env with history 1 (5 calls x 6 layers,
    windows 1, 2, 3, 3, 3), or B envs with history 3 (3 calls x 6 layers, windows 3, 3, 3).
    A fixed launch sequence for ncu captures of one kernel at a known geometry. mode "bf16"
    (tensor cores), "fp32" (model_cost_autocast "none") or "grad" (the float32 forward and
    reverse pass, lewm_model_cost_grad)."""
    import torch

    from lewm_flash_b200.model import ModelDesc, synthetic_state_dict
    from lewm_flash_b200.runtime import Runtime

    dev = torch.device("cuda", 0)
    desc = ModelDesc()
    rt = Runtime(desc, synthetic_state_dict(desc, 0), dev, model_cost_autocast="none" if mode == "fp32" else "bf16")
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
        costs = rt.model_cost_grad(emb, goal, cand)[0] if mode == "grad" else rt.model_cost(emb, goal, cand)
        b.record()
        torch.cuda.synchronize(dev)
        ms.append(a.elapsed_time(b))
    rt.sync()
    print(json.dumps({"case": "model_cost", "mode": mode, "envs": envs, "samples": S, "ms": ms,
                      "cost0": float(costs[0, 0])}))
    return 0


def plan_case(envs: int, repeat: int, history: int = 3) -> int:
    """``--plan N``: `repeat` bucketed iCEM plans (the bench's settings) of N envs with history 3,
    in-kernel noise: a fixed launch sequence for ncu captures of the sampling and top-k / refit
    kernels at a known geometry."""
    import torch

    from lewm_flash_b200.model import ModelDesc, synthetic_state_dict
    from lewm_flash_b200.runtime import Runtime

    dev = torch.device("cuda", 0)
    rt = Runtime(ModelDesc(), synthetic_state_dict(ModelDesc(), 0), dev)
    rng = np.random.default_rng(7)
    emb = torch.as_tensor(rng.standard_normal((envs, history, 192)), dtype=torch.float32, device=dev)
    goal = torch.as_tensor(rng.standard_normal((envs, 1, 192)), dtype=torch.float32, device=dev)
    mean = torch.zeros(envs, 5, 10, device=dev)
    std = torch.ones(envs, 5, 10, device=dev)
    ms = []
    for i in range(repeat):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        rt.plan(plan_options(), emb, goal, mean, std, plan_index=9000 + i)
        b.record()
        torch.cuda.synchronize(dev)
        ms.append(a.elapsed_time(b))
    rt.sync()
    print(json.dumps({"case": "plan", "envs": envs, "history": history, "ms": ms}))
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
    ap.add_argument("--no-reference-gpu", action="store_true", help="skip the reference PyTorch GPU comparator")
    ap.add_argument("--no-sharded", action="store_true", help="skip the 1024-env sharded leg")
    ap.add_argument("--no-stress", action="store_true", help="skip the width-384 stress leg")
    ap.add_argument("--no-fp32", action="store_true", help="skip the float32 CEM and CEM-GD gradient legs")
    ap.add_argument("--no-policy", action="store_true", help="skip the 100-env get_action leg")
    ap.add_argument("--model-cost", type=int, default=0, metavar="S",
                    help="profiling case: time R model-cost calls of S candidates per env (horizon 5; 1 env "
                         "with history 1, or --envs B with history 3) and exit; no bench line")
    ap.add_argument("--encoder", type=int, default=0, metavar="N",
                    help="profiling case: run the observation encoder R times on N 224 px images and exit; "
                         "no bench line")
    ap.add_argument("--plan", type=int, default=0, metavar="N",
                    help="profiling case: --repeat plans of N envs (history 3) and exit")
    ap.add_argument("--envs", type=int, default=1)
    ap.add_argument("--mode", default="bf16", choices=["bf16", "fp32", "grad"],
                    help="--model-cost arithmetic: bf16, fp32 or the float32 gradient")
    ap.add_argument("--repeat", type=int, default=3)
    args = ap.parse_args()
    if args.model_cost:
        return model_cost_case(args.model_cost, args.repeat, args.envs, args.mode)
    if args.encoder:
        return encoder_case(args.encoder, args.repeat)
    if args.plan:
        return plan_case(args.plan, args.repeat)

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
    emb_np, goal_np = bench_latents(rank, desc.dim)
    emb = torch.as_tensor(emb_np, device=dev)
    goal = torch.as_tensor(goal_np, device=dev)
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
    fp32_cem = fp32_cem_pass(dev, args.steps, args.warmup, flush) if not args.no_fp32 else None
    cem_gd = cem_gd_pass(rt, dev) if world == 1 and not args.no_fp32 else None

    # ---------------------------------------------------------------- 1024 envs split over the ranks
    sharded = sharded_pass(rt, dev, rank, world, barrier, dist, flush) if not args.no_sharded else None
    # the same 1024 envs with history 1 (5 predictor calls per iteration, windows 1, 2, 3, 3, 3)
    sharded_h1 = (sharded_pass(rt, dev, rank, world, barrier, dist, flush, history=1, n_calls=2, own_runtime=True)
                  if not args.no_sharded else None)

    # ---------------------------------------------------------------- width 384 / 12 layers, 32 envs per rank
    stress = stress_pass(dev, rank, world, barrier, dist, flush) if not args.no_stress else None

    # ---------------------------------------------------------------- observation encoder (64 images, 224 px)
    encoder = encoder_pass(dev, args.steps, args.warmup, flush)

    # ---------------------------------------------------------------- policy get_action, 100 envs
    policy = policy_pass(rt, dev) if not args.no_policy else None

    # ---------------------------------------------------------------- per-kernel-class timing pass (diagnostic, last)
    kinfo = kernel_class_pass(rt, opts, emb, goal, mean, std, dev)
    per_plan_launches = kinfo["launches_per_plan"]
    flops_plan = F_CANON * 2820
    line = {
        "metric": METRIC, "value": value, "unit": "plans/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": worst_ms / args.steps, "p50_plan_ms": p50,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init weights, N(0,1) latents)",
        "config": bench_config(world),
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
        "fp32_cem": fp32_cem,
        "cem_gd": cem_gd,
        "sharded": sharded,
        "sharded_h1": sharded_h1,
        "stress": stress,
        "encoder": encoder,
        "policy": policy,
        "clocks": clocks.summary(),
    }
    if rank == 0 and world == 1 and not args.no_reference_gpu:
        ref_gpu = reference_gpu_pass(dev)
        if "eager_p50_ms" in ref_gpu:
            ref_gpu["speedup_vs_eager"] = ref_gpu["eager_p50_ms"] / p50
        if "compiled_p50_ms" in ref_gpu:
            ref_gpu["speedup_vs_compiled"] = ref_gpu["compiled_p50_ms"] / p50
        line["reference_gpu"] = ref_gpu
    # The host-core baseline runs at N = 1 only: under torchrun the other ranks would wait at the
    # closing barrier (and spin on their CPU cores) for the whole CPU run.
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        times, info = reference_cpu_plans(max(args.cpu_baseline_plans, 1), 1, rank)
        line["cpu_baseline"] = dict(info, value=1.0 / float(np.mean(times)), unit="plans/s")
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    rt.close()
    return 0


def timed_shard_calls(dev, barrier, dist, flush, plan_call, n_calls):
    """Time `n_calls` plan calls of this rank (CUDA events, host barrier first, L2 flushed before
    each) and return the max over ranks of the summed call time in ms."""
    import torch

    stream = torch.cuda.current_stream(dev)
    total = 0.0
    for _ in range(n_calls):
        l2_flush(flush)
        barrier()
        torch.cuda.synchronize(dev)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        plan_call()
        b.record(stream)
        torch.cuda.synchronize(dev)
        total += a.elapsed_time(b)
    worst = torch.tensor([total], device=dev)
    if dist is not None:
        dist.all_reduce(worst, op=dist.ReduceOp.MAX)
    return float(worst.item())


def sharded_pass(rt, dev, rank, world, barrier, dist, flush, n_envs=1024, history=3, n_calls=3, own_runtime=False):
    """1024 independent envs (own N(0,1) latents, history 3) split contiguously over the ranks
    (lewm_flash_b200.shard.env_range); each rank plans its envs as one batched plan call, with
    no collective in the timed region. plans/s = 1024 / (max over ranks of the call time):
    total work fixed, so strong scaling over the GPU count. The plans are gathered to rank 0
    on the host afterwards (gather_plans, gloo), outside the timed region. own_runtime:
    plan on a context of its own, released afterwards (its workspace for 1024 envs does not
    stay allocated beside the later legs)."""
    import torch

    from lewm_flash_b200.shard import env_range, gather_plans, plan_shard

    if own_runtime:
        from lewm_flash_b200.model import ModelDesc, synthetic_state_dict
        from lewm_flash_b200.runtime import Runtime

        rt = Runtime(ModelDesc(), synthetic_state_dict(ModelDesc(), 0), dev)

    opts = plan_options()
    rng = np.random.default_rng(3)
    emb = torch.as_tensor(rng.standard_normal((n_envs, history, 192)), dtype=torch.float32)
    goal = torch.as_tensor(rng.standard_normal((n_envs, 1, 192)), dtype=torch.float32)
    s, e = env_range(n_envs, rank, world)
    inputs = {"emb": emb.to(dev), "goal_emb": goal.to(dev), "mean": torch.zeros(n_envs, 5, 10, device=dev),
              "std": torch.ones(n_envs, 5, 10, device=dev)}
    box = {}

    def call(idx=[7000]):
        idx[0] += 1
        box["out"] = plan_shard(lambda **t: rt.plan(opts, t["emb"], t["goal_emb"], t["mean"], t["std"],
                                                    plan_index=idx[0])[:3], inputs, rank, world)

    call()  # warm-up: workspace growth and graph capture for this shape
    rt.sync()
    worst_ms = timed_shard_calls(dev, barrier, dist, flush, call, n_calls)
    rt.sync()
    per_call = worst_ms / n_calls
    gathered = None
    if dist is not None:
        group = dist.new_group(backend="gloo")
        res = gather_plans(box["out"], n_envs, [(5, 10), (5, 10), ()], group=group)
        gathered = None if res is None else int(res[0].shape[0])
        dist.destroy_process_group(group)
    else:
        gathered = int(box["out"][0].shape[0])
    box.clear()
    if own_runtime:
        rt.close()
    return {"workload": f"icem_bucketed_300_{n_envs}env_h{history}_bf16", "envs": n_envs, "envs_this_rank": e - s,
            "history": history, "plans_per_s": n_envs / (per_call / 1e3), "ms_per_call": per_call, "calls": n_calls,
            "gathered_envs": gathered, "scaling": "strong",
            "note": "each rank plans its contiguous env range as one batched plan call; time = max over ranks; "
                    "device-resident inputs, L2 flushed between calls"}


def stress_pass(dev, rank, world, barrier, dist, flush, envs_per_rank=32, n_calls=1):
    """Scaled stress configuration: predictor width 384, 12 layers, 16 heads, MLP 1536, action
    dim 10, horizon 10, history 3, iCEM 3000 samples / 300 elites / 30 iterations with the
    bucketed schedule (decay 1.25, bucket 600: 28,200 candidates per env), brown noise, bf16
    rollout; 32 envs per rank (256 envs on 8 GPUs), one batched plan call per rank."""
    import torch

    from lewm_flash_b200.model import STRESS_DESC, synthetic_state_dict
    from lewm_flash_b200.runtime import PlanOptions, Runtime

    rt = Runtime(STRESS_DESC, synthetic_state_dict(STRESS_DESC, 5), dev)
    opts = PlanOptions(num_samples=3000, topk=300, n_steps=30, sample_decay=1.25, sample_count_bucket_size=600,
                       elite_retention=30, beta=2.0, time_axis="raw", action_block=5, seed=0)
    rng = np.random.default_rng(500 + rank)
    emb = torch.as_tensor(rng.standard_normal((envs_per_rank, 3, 384)), dtype=torch.float32, device=dev)
    goal = torch.as_tensor(rng.standard_normal((envs_per_rank, 1, 384)), dtype=torch.float32, device=dev)
    mean = torch.zeros(envs_per_rank, 10, 10, device=dev)
    std = torch.ones(envs_per_rank, 10, 10, device=dev)
    idx = [9000]

    def call():
        idx[0] += 1
        rt.plan(opts, emb, goal, mean, std, plan_index=idx[0])

    call()
    rt.sync()
    worst_ms = timed_shard_calls(dev, barrier, dist, flush, call, n_calls)
    rt.sync()
    rt.close()
    torch.cuda.empty_cache()
    per_call = worst_ms / n_calls
    flops = 1809.9e6 * 28200 * envs_per_rank
    return {"workload": "icem_bucketed_3000_w384_l12_t10_h3_bf16", "envs_per_rank": envs_per_rank,
            "envs": envs_per_rank * world, "candidates_per_plan": 28200,
            "plans_per_s": envs_per_rank * world / (per_call / 1e3), "ms_per_call": per_call, "calls": n_calls,
            "tflops_per_gpu": flops / (per_call / 1e3) / 1e12, "scaling": "weak",
            "note": "one batched plan call per rank; time = max over ranks; elite retention 30 (10% of 300)"}


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


def fp32_cem_pass(dev, steps, warmup, flush, n_envs=1):
    """The float32 configuration: plain CEM 300 samples / 30 elites / 30 iterations, 1 env,
    history 1, with the model cost in float32 throughout (model_cost_autocast "none", the
    reference's default arithmetic). Device-resident inputs, L2 flushed between plans."""
    import torch

    from lewm_flash_b200.model import ModelDesc, synthetic_state_dict
    from lewm_flash_b200.runtime import PlanOptions, Runtime

    rt = Runtime(ModelDesc(), synthetic_state_dict(ModelDesc(), 0), dev, model_cost_autocast="none")
    opts = PlanOptions(num_samples=300, topk=30, n_steps=30, sample_decay=1.0, sample_count_bucket_size=0,
                       elite_retention=0, beta=0.0, action_block=5, seed=0)
    emb, goal = (torch.as_tensor(x, device=dev) for x in bench_latents(0))
    mean = torch.zeros(n_envs, 5, 10, device=dev)
    std = torch.ones(n_envs, 5, 10, device=dev)
    for i in range(max(warmup, 1)):
        rt.plan(opts, emb, goal, mean, std, plan_index=7000 + i)
    stream = torch.cuda.current_stream(dev)
    ms = []
    for i in range(max(1, min(steps, 10))):
        l2_flush(flush)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        rt.plan(opts, emb, goal, mean, std, plan_index=8000 + i)
        b.record(stream)
        torch.cuda.synchronize(dev)
        ms.append(a.elapsed_time(b))
    rt.sync()
    rt.close()
    p50 = percentile(ms, 50)
    flops = F_CANON * 300 * 30 * n_envs
    out = {"workload": "cem_300_30_30_1env_h1_fp32", "envs": n_envs, "plans_per_s": n_envs / (p50 / 1e3),
           "p50_plan_ms": p50, "plans": len(ms), "tflops_fp32": flops / (p50 / 1e3) / 1e12,
           "flops_per_plan": flops,
           "note": "float32 CUDA-core model cost (no tensor cores); canonical FLOPs (window rows the "
                   "bf16 path computes), the fp32 path recomputes full windows (~1.3x)"}
    if n_envs == 1:
        out["reference_gpu"] = reference_fp32_cem(dev)
        if "eager_p50_ms" in out["reference_gpu"]:
            out["reference_gpu"]["speedup"] = out["reference_gpu"]["eager_p50_ms"] / p50
    return out


def reference_fp32_cem(dev, plans=5, warmup=2):
    """The reference's own CEMExactSolver.solve (baseline/_ref) for the same float32 plan on this
    GPU: same weights and latents, model cost in float32 (the JEPA default "none"), float32
    matmul precision "highest" (no TF32), one env, eager, CUDA events around each solve."""
    from types import SimpleNamespace

    import torch

    ref = reference_package()
    if ref is None:
        return {"unavailable": "reference not installed in baseline/_ref"}
    from lewm.solvers.cem_exact import CEMExactSolver

    prec = torch.get_float32_matmul_precision()
    torch.set_float32_matmul_precision("highest")
    try:
        model, _ = reference_solver(ref, dev)
        model.set_model_cost_autocast("none")
        solver = CEMExactSolver(model=model, batch_size=1, num_samples=300, n_steps=30, topk=30, device=dev, seed=0)

        class Box:
            shape = (1, 2)
            low = -np.inf * np.ones((1, 2), dtype=np.float32)
            high = np.inf * np.ones((1, 2), dtype=np.float32)

        solver.configure(action_space=Box(), n_envs=1, config=SimpleNamespace(horizon=5, action_block=5))
        emb_np, goal_np = bench_latents(0)
        emb = torch.as_tensor(emb_np, device=dev)
        goal = torch.as_tensor(goal_np, device=dev)
        ms = []
        for i in range(warmup + plans):
            info = {"emb": emb, "goal_emb": goal, "pixels": torch.zeros(1, 1, device=dev),
                    "goal": torch.zeros(1, 1, device=dev)}
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize(dev)
            a.record()
            with torch.inference_mode():
                quiet(solver.solve, info)
            b.record()
            torch.cuda.synchronize(dev)
            if i >= warmup:
                ms.append(a.elapsed_time(b))
        del model, solver
        torch.cuda.empty_cache()
        return {"api": "reference CEMExactSolver.solve (baseline/_ref), float32 model cost, matmul precision "
                       "highest, cached latents, 1 env, eager", "plans": plans, "eager_p50_ms": percentile(ms, 50)}
    finally:
        torch.set_float32_matmul_precision(prec)


def cem_gd_pass(rt, dev, n_seeds=30, repeat=20):
    """The gradient CEM-GD's refinement steps on (reference lewm/solvers/cem_gd.py:459-606): costs
    and d cost / d actions of 30 seed candidates (1 env, history 1, horizon 5) in float32. The
    device's forward + reverse pass (lewm_model_cost_grad) against the reference model's own
    torch autograd of get_cost_from_embeddings (baseline/_ref, float32, matmul precision
    "highest") on the same GPU and inputs; CUDA events, p50."""
    import torch

    g = np.random.default_rng(11)
    emb = torch.as_tensor(g.standard_normal((1, 1, 192)), dtype=torch.float32, device=dev)
    goal = torch.as_tensor(g.standard_normal((1, 1, 192)), dtype=torch.float32, device=dev)
    cand = torch.as_tensor(g.standard_normal((1, n_seeds, 5, 10)), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def timed(fn, n):
        ms = []
        for _ in range(n):
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(stream)
            fn()
            b.record(stream)
            torch.cuda.synchronize(dev)
            ms.append(a.elapsed_time(b))
        return ms

    timed(lambda: rt.model_cost_grad(emb, goal, cand), 3)
    dev_ms = percentile(timed(lambda: rt.model_cost_grad(emb, goal, cand), repeat), 50)
    _, grad = rt.model_cost_grad(emb, goal, cand)
    rt.sync()
    out = {"workload": f"cost_grad_1env_{n_seeds}seeds_h1_fp32", "device_p50_ms": dev_ms, "repeat": repeat}
    ref = reference_package()
    if ref is None:
        out["reference"] = "unavailable: reference not installed in baseline/_ref"
        return out
    prev = torch.get_float32_matmul_precision()
    torch.set_float32_matmul_precision("highest")
    try:
        model, _ = reference_solver(ref, dev)
        model.requires_grad_(False)
        box = {}

        def ref_step():
            c = cand.clone().requires_grad_(True)
            model.get_cost_from_embeddings(emb, goal, c).sum().backward()
            box["grad"] = c.grad

        timed(ref_step, 3)
        ref_ms = percentile(timed(ref_step, repeat), 50)
        err = float((grad - box["grad"]).abs().max() / box["grad"].abs().max())
        out.update({"reference_autograd_p50_ms": ref_ms, "speedup_vs_reference_autograd": ref_ms / dev_ms,
                    "max_grad_diff_of_max": err,
                    "reference": "JEPA.get_cost_from_embeddings + backward, eager torch, float32 (baseline/_ref)"})
        del model
    finally:
        torch.set_float32_matmul_precision(prev)
    return out


def policy_pass(rt, dev, n_envs=100, replans=3):
    """``get_action`` through ``B200PlanningPolicy`` for ``n_envs`` envs with the eval plan_config
    (horizon 5, receding_horizon 5, action_block 5: one plan every 25 calls, history 1): uint8
    224 px observation and goal frames from pinned host memory, the ViT-tiny encoder with the
    image transform fused, one bucketed iCEM 300 plan of all envs, one device->host read of the
    actions per plan. get_action returns host actions, so each call is timed on the host clock;
    p50 / p90 over all calls (the definition of the reference README's get_action figures) and
    the mean of the planning calls alone."""
    import time

    import torch

    from lewm_flash_b200.encoder import B200Encoder, EncoderDesc, flat_weights, synthetic_weights
    from lewm_flash_b200.policy import B200PlanningPolicy
    from lewm_flash_b200.solver import B200ICEMSolver

    desc = EncoderDesc()
    vit, proj = synthetic_weights(desc, 0)
    enc = B200Encoder(desc, flat_weights(vit, proj, desc), dev)
    solver = B200ICEMSolver(rt, num_samples=300, n_steps=30, topk=30, elite_retention=3, colored_noise="brown",
                            colored_noise_time="raw", sample_decay=1.25, sample_count_bucket_size=60, seed=0,
                            history_size=1, device=dev)

    class Box:
        shape = (n_envs, 2)
        low = -np.ones((n_envs, 2), np.float32)
        high = np.ones((n_envs, 2), np.float32)

    cfg = {"horizon": 5, "receding_horizon": 5, "action_block": 5}
    policy = B200PlanningPolicy(solver, cfg, encoder=enc)
    policy.set_env(type("Env", (), {"num_envs": n_envs, "action_space": Box()})())
    rng = np.random.default_rng(23)
    frames = [{k: torch.as_tensor(rng.integers(0, 256, (n_envs, 1, 224, 224, 3), dtype=np.uint8)).pin_memory()
               for k in ("pixels", "goal")} for _ in range(2)]
    per_plan = 25
    for i in range(per_plan):  # warm-up cycle: graph capture, encoder and plan workspaces
        policy.get_action(frames[i % 2])
    ms, plan_ms, serve_ms = [], [], []
    for i in range(replans * per_plan):
        plans = policy.solves
        t0 = time.perf_counter()
        policy.get_action(frames[i % 2])
        dt = (time.perf_counter() - t0) * 1e3
        ms.append(dt)
        (plan_ms if policy.solves > plans else serve_ms).append(dt)
    del enc
    return {"workload": f"get_action_{n_envs}env_icem_bucketed_300_h1_vit_tiny_224_u8", "envs": n_envs,
            "calls": len(ms), "plans": len(plan_ms), "p50_ms": percentile(ms, 50), "p90_ms": percentile(ms, 90),
            "plan_call_ms": float(np.mean(plan_ms)), "serve_call_p50_ms": percentile(serve_ms, 50),
            "h2d_bytes_per_plan": int(2 * n_envs * 224 * 224 * 3),
            "note": "host-clock time per get_action; planning calls encode obs + goal frames and plan all envs"}


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
