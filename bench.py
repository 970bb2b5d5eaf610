"""Headline benchmark: MaskGIT transformer steps/s (config 1: 24 layers, M=257, Q8_0, batch 1).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--quant gq8|gq4] [--impl cuda|reference]

One process per GPU (torchrun for N>1); each rank runs its own replica of the config-1 step
(the path shards by independent images, so there is no collective), timing is on the device
with CUDA events, max over ranks, and `value` is the whole-job steps/s.  Rank 0 prints ONE
JSON line.  `--impl reference` times the reference's own CPU implementation instead.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

MODEL_DIR = Path(os.environ.get("MGC_BENCH_DIR", "/tmp/mgc_bench"))


def peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int, period_ms: int = 50):
        self.index, self.period_ms, self.rows, self._p = index, period_ms, [], None
        self._t = threading.Thread(target=self._read, daemon=True)

    def _read(self):
        for line in self._p.stdout:
            cols = [c.strip() for c in line.split(",")]
            if len(cols) >= 9:
                self.rows.append(cols)

    def __enter__(self):
        # one nvidia-smi in loop mode for the whole timed region (no per-sample process start)
        try:
            self._p = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                        "--format=csv,noheader,nounits", f"-lms={self.period_ms}"],
                                       stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t.start()
            time.sleep(0.3)   # first sample lands before the timed work starts
        except OSError:
            self._p = None
        return self

    def __exit__(self, *a):
        if self._p is not None:
            self._p.terminate()
            try:
                self._p.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._p.kill()
            self._t.join(timeout=5)

    def summary(self) -> dict:
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in self.rows for n, v in zip(names, r[5:9]) if v.strip().lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


# ----------------------------------------------------------------------------- models
def ensure_model(quant: str, n_layer: int = 24, twin: bool = False) -> tuple[Path, Path | None]:
    from edge_maskgit_b200 import synth
    MODEL_DIR.mkdir(parents=True, exist_ok=True)
    path = MODEL_DIR / f"c1_{quant}_L{n_layer}.gguf"
    tpath = MODEL_DIR / f"c1_{quant}_L{n_layer}_f32.gguf" if twin else None
    if not path.exists() or (twin and not tpath.exists()):
        tmp = path.with_suffix(f".tmp{os.getpid()}")
        ttmp = tpath.with_suffix(f".tmp{os.getpid()}") if twin else None
        synth.make_model(tmp, synth.ModelSpec(n_layer=n_layer, quant=quant), dequant_twin=ttmp)
        os.replace(tmp, path)
        if twin:
            os.replace(ttmp, tpath)
    return path, tpath


# ----------------------------------------------------------------------------- CPU baselines
def reference_cpu_step_s(quant: str, reps: int = 1) -> tuple[float, str, str]:
    """Seconds per config-1 forward of the reference's own CPU executor (mg-cpu, scalar F32,
    single-threaded by construction) on the dequantised twin.  A bounded sample: 1- and
    2-layer models are timed and the per-layer cost is extrapolated to 24 layers."""
    from edge_maskgit_b200 import synth
    from oracle import oracle as O
    tok = synth.config1_tokens()
    if O.ref_available():
        _, f1 = ensure_model(quant, 1, twin=True)
        _, f2 = ensure_model(quant, 2, twin=True)
        t = {}
        for L, f in ((1, f1), (2, f2)):
            best = 1e30
            for _ in range(reps):
                t0 = time.perf_counter()
                O.ref_forward(f, tok, 768, L, 2025)
                best = min(best, time.perf_counter() - t0)
            t[L] = best
        per_layer = t[2] - t[1]
        step = t[1] + 23 * per_layer
        return step, "reference", (f"mg-cpu F32 executor on the dequantised twin, M=257: 1-layer {t[1]:.2f}s, "
                                   f"2-layer {t[2]:.2f}s, extrapolated to 24 layers")
    # reference tree not built on this host: the oracle port, full model
    p, _ = ensure_model(quant, 24)
    m = O.OracleModel(p)
    t0 = time.perf_counter()
    m.forward(tok)
    return time.perf_counter() - t0, "port", "oracle int8-dot restatement, full 24-layer M=257 forward"


def run_reference_arm(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from edge_maskgit_b200 import synth
    from oracle import oracle as O
    # calibrate once (1- vs 2-layer), then each step times the 1-layer sample and adds the
    # 23 remaining layers at the calibrated per-layer cost
    cal, kind, sample = reference_cpu_step_s(args.quant)
    tok = synth.config1_tokens()
    step_s = 0.0
    if kind == "reference":
        _, f1 = ensure_model(args.quant, 1, twin=True)
        _, f2 = ensure_model(args.quant, 2, twin=True)
        t0 = time.perf_counter(); O.ref_forward(f1, tok, 768, 1, 2025); t1 = time.perf_counter() - t0
        per_layer = (cal - t1) / 23.0
        for i in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            O.ref_forward(f1, tok, 768, 1, 2025)
            s = time.perf_counter() - t0 + 23 * per_layer
            if i >= args.warmup:
                step_s += s
    else:
        for i in range(args.warmup + args.steps):
            s, kind, sample = reference_cpu_step_s(args.quant)
            if i >= args.warmup:
                step_s += s
    step_s /= args.steps
    v = 1.0 / step_s
    print(json.dumps({
        "impl": "reference", "metric": "transformer steps/s", "value": v, "unit": "steps/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_s * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"config1 step-1 forward, 24 layers, M=257, {args.quant}, batch 1"},
        "cpu_baseline": {"value": v, "unit": "steps/s", "cores": 1, "kind": kind, "sample": sample},
        "e2e": {"value": v, "unit": "steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ----------------------------------------------------------------------------- CUDA arm
def qgemm_algorithmic_bytes(quant: str, M: int = 257) -> tuple[float, int]:
    """Sum over one forward's quantized GEMM launches of the algorithmic bytes
    W_packed + 4*M*K (X f32) + 4*M*N (Y f32) + 4*N (bias) [+ 4*M*N residual]."""
    E, F = 768, 3072
    wb = (lambda N, K: N * K * 34 / 32) if quant == "gq8" else (lambda N, K: N * K * 144 / 256)
    shapes = [(3 * E, E, False), (E, E, True), (F, E, False), (E, F, True)] * 24 + [(E, E, False)]
    total = 0.0
    for N, K, res in shapes:
        total += wb(N, K) + 4 * M * K + 4 * M * N + 4 * N + (4 * M * N if res else 0)
    return total, len(shapes)


def run_cuda_arm(args) -> None:
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    from edge_maskgit_b200 import runtime as rt, synth

    if rank == 0 or world == 1:
        path, _ = ensure_model(args.quant)
    if world > 1:
        dist.barrier()
        path, _ = ensure_model(args.quant)
    S, V = 257, 2025
    r = rt.CudaRuntime(path, max_rows=S, device=local)
    stream = torch.cuda.ExternalStream(r.stream_handle, device=torch.device("cuda", local))
    tok_host = synth.config1_tokens()
    logits_host = np.empty((S, V), np.float32)   # reused every step, like the reference decode loop
    tok_dev = torch.from_numpy(tok_host).cuda()
    logits_dev = torch.empty((S, V), dtype=torch.float32, device="cuda")

    # ---- per-kernel profile (eager, CUDA events around each launch): roofline of the qGEMM
    r.profile_enable(True)
    for _ in range(3):
        r.forward(tok_host)
    r.profile_reset()
    for _ in range(5):
        r.forward(tok_host)
    prof = {p.op: p for p in r.profile_report()}
    r.profile_enable(False)

    # ---- device-resident timing: CUDA-graph replay, inputs in HBM
    for _ in range(args.warmup):
        r.forward_dev(tok_dev, logits_dev, 1, S)
        r.forward(tok_host, out=logits_host)   # the host path's own graph is captured here
    r.sync()
    launches_per_fwd = r.kernel_count()   # kernels in the captured step graph
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk, torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(args.steps):
            r.forward_dev(tok_dev, logits_dev, 1, S)
        e1.record(stream)
        torch.cuda.synchronize()
        dev_ms = e0.elapsed_time(e1)
        # ---- end to end through the public API: host tokens in, host logits out
        t_e2e0 = torch.cuda.Event(enable_timing=True); t_e2e1 = torch.cuda.Event(enable_timing=True)
        t_e2e0.record(stream)
        for _ in range(args.steps):
            r.forward(tok_host, out=logits_host)
        t_e2e1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = t_e2e0.elapsed_time(t_e2e1)
    if world > 1:
        dist.barrier()
    r.sync()
    ms = torch.tensor([dev_ms, e2e_ms], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    dev_ms, e2e_ms = ms.tolist()

    if rank == 0:
        hbm, src = peaks()
        alg, n_q = qgemm_algorithmic_bytes(args.quant)
        q = prof.get("MulMat(q)")
        q_ms = q.ms / q.count if q else float("nan")
        achieved = (alg / n_q) / (q_ms * 1e-3) / 1e9 if q else None
        traffic = None
        tf = ROOT / "profiles" / f"qgemm_{args.quant}_traffic.txt"
        if tf.exists():
            for line in tf.read_text().splitlines():
                if line.startswith("bytes_per_launch:"):
                    traffic = float(line.split(":")[1])
        out = {
            "metric": "transformer steps/s", "value": world * args.steps / (dev_ms * 1e-3), "unit": "steps/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": dev_ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8-dot/f32",
            "data": "synthetic",
            "config": {"workload": f"config1 step-1 forward, 24 layers, M=257, {args.quant}, batch 1 per GPU",
                       "parallelism": f"replicas x{world} (independent images, no collective)",
                       "l2": "inputs larger than L2 (190 MB of weights streamed per step)"},
            "e2e": {"value": world * args.steps / (e2e_ms * 1e-3), "unit": "steps/s",
                    "h2d_bytes_per_step": int(tok_host.nbytes), "d2h_bytes_per_step": S * V * 4},
            "gpu_launches": launches_per_fwd * args.steps,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": (achieved / hbm) if achieved else None, "traffic": traffic,
                         "kernel": "qgemm (MulMat(q)), mean over the 97 launches of one step",
                         "peak_source": src},
            "kernel_ms_per_step": {k: p.ms / 5 for k, p in prof.items()},
            "clocks": clk.summary(),
        }
        if world == 1 and not args.no_cpu_baseline:
            s, kind, sample = reference_cpu_step_s(args.quant)
            out["cpu_baseline"] = {"value": 1.0 / s, "unit": "steps/s", "cores": 1 if kind == "reference" else os.cpu_count(),
                                   "kind": kind, "sample": sample}
        print(json.dumps(out), flush=True)
    r.close()
    if world > 1:
        dist.destroy_process_group()


def run_tp_workload(args) -> None:
    """Config 5: step-1 forward at M=4097 (64x64 tokens + class), batch 4, Q4_K, column-split
    over the ranks with NCCL all-gathers.  Total work is fixed, so scaling is strong."""
    import torch
    import torch.distributed as dist
    from edge_maskgit_b200 import synth
    from edge_maskgit_b200.tp import TPForward

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    MODEL_DIR.mkdir(parents=True, exist_ok=True)
    path = MODEL_DIR / "c5_gq4_n4096.gguf"
    spec = synth.ModelSpec(n_tokens=4096, quant="gq4")
    if rank == 0 and not path.exists():
        tmp = path.with_suffix(f".tmp{os.getpid()}")
        synth.make_model(tmp, spec)
        os.replace(tmp, path)
    if world > 1:
        dist.barrier()
    tp = TPForward(path, rank, world)
    tokens = np.tile(synth.config1_tokens(spec), (4, 1))
    tokens[:, 0] = 1024 + np.array([207, 1, 500, 999])
    for _ in range(args.warmup):
        tp.forward(tokens)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        logits = tp.forward(tokens)
    e1.record()
    torch.cuda.synchronize()
    ms = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms.item())
    if rank == 0:
        print(json.dumps({
            "metric": "transformer steps/s", "value": args.steps / (ms * 1e-3), "unit": "steps/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8-dot/f32",
            "data": "synthetic",
            "config": {"workload": "config5 step-1 forward, 24 layers, M=4097, batch 4, gq4",
                       "parallelism": f"column-split tensor parallel x{world}, NCCL all-gather"},
        }), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_decode_workload(args) -> None:
    """Config 4: batched decode of 64 images (classes from default_rng(7), seed 7+i), Q8_0, 8 steps,
    sharded by image over the ranks (each rank batches its images into one forward per step);
    one all-gather of the token grids at the end.  Total work is fixed: strong scaling.  Each
    timed step is one full 8-step decode of the 64 images; timing is CUDA events on the runtime's
    stream (the loop is host-driven, so host gaps count), max over ranks."""
    import torch
    import torch.distributed as dist
    from edge_maskgit_b200 import runtime as rt, shard

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    if rank == 0:
        path, _ = ensure_model("gq8")
    if world > 1:
        dist.barrier()
    path, _ = ensure_model("gq8")
    n_img, S = 64, 257
    classes, seeds = shard.batch_classes(n_img), shard.batch_seeds(n_img)
    lo, hi = shard.shard_range(n_img, rank, world)
    r = rt.CudaRuntime(path, max_rows=S * max(1, hi - lo), device=local)
    stream = torch.cuda.ExternalStream(r.stream_handle, device=torch.device("cuda", local))
    gen = lambda c, sd, steps, t: r.generate(c, sd, steps, t)
    for _ in range(args.warmup):
        shard.decode_shard(gen, classes, seeds, rank, world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(args.steps):
        local_tok = shard.decode_shard(gen, classes, seeds, rank, world)
    e1.record(stream)
    torch.cuda.synchronize()
    ms = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        grids = shard.gather_tokens(local_tok, n_img, S)
    else:
        grids = local_tok
    ms = float(ms.item())
    if rank == 0:
        print(json.dumps({
            "metric": "images/s", "value": n_img * args.steps / (ms * 1e-3), "unit": "images/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8-dot/f32",
            "data": "synthetic",
            "config": {"workload": "config4 batched decode, 64 images x 8 steps, gq8, seq 257",
                       "parallelism": f"images sharded over {world} rank(s), one all-gather of the token grids",
                       "tokens_checksum": int(np.asarray(grids, dtype=np.int64).sum())},
        }), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default: 300 for c1, 10 for c5, 20 for the reference arm)")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--quant", default="gq8", choices=["gq8", "gq4"])
    ap.add_argument("--impl", default="cuda", choices=["cuda", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="c1", choices=["c1", "c4", "c5"],
                    help="c1: the headline config-1 step (default); c4: 64-image batched decode; "
                         "c5: M=4097 tensor-parallel step")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = 20 if args.impl == "reference" else 10 if args.workload == "c5" else 3 if args.workload == "c4" else 300
    if args.workload == "c5" and args.impl == "cuda":
        run_tp_workload(args)
        return
    if args.workload == "c4" and args.impl == "cuda":
        run_decode_workload(args)
        return
    if args.impl == "reference":
        run_reference_arm(args)
    else:
        run_cuda_arm(args)


if __name__ == "__main__":
    main()
