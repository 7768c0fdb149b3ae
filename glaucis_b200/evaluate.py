"""CUDA evaluator backend for kernel templates, with the request / result
contract of the Glaucis pod evaluator (KE/docker/evaluate.py).

    python -m glaucis_b200.evaluate --eval-payload <base64 json>
    python -m glaucis_b200.evaluate --eval-payload-file payload.b64

Request (base64 JSON): {variant_id, kernel_code, reference_code, shapes,
rtol, atol} or, batch mode, {batch: true, variants: [{variant_id,
kernel_code}], reference_code, shapes, rtol, atol}.  Output: one line per
variant, ``EVAL_RESULT:{json}`` with status COMPILE_ERROR / INCORRECT /
SUCCESS, fitness (= speedup), latency_ms, speedup, flops and metadata
(benchmark statistics of the kernel and the reference).

Stages (KE/docker/evaluate.py:98-424, 928-1072), plus an optional deep
profile (request key "deep_profile": true, KE/docker/evaluate.py:478-889):
  1. compile      exec() the template text (stage_compile :98-104)
  2. correctness  each shape: kernel fn vs reference fn; scalar results must
                  satisfy max|diff| <= atol (:107-127); array results are
                  checked element-wise with |diff| <= atol + rtol*|ref|
  3. benchmark    3 warm-up calls, then N calls each bracketed by CUDA events
                  on the current stream (replaces jax.jit + xprof clustering)
  4. reference    the same benchmark on the reference code -> speedup
  5. deep profile ncu counters of one call (child process) -> compute_ratio,
                  memory_transfer_ratio, metadata.hw_utilization
The TPU-specific stages (libtpu dumps, XPlane parsing, HLO/LLO analysis,
GCS upload) have no counterpart here.
"""
from __future__ import annotations

import argparse
import base64
import json
import os
import subprocess
import sys
import time
import traceback
from typing import Any, Callable, Optional

import numpy as np


def decode_request(b64_payload: str) -> dict:
    return json.loads(base64.b64decode(b64_payload).decode())


def encode_request(payload: dict) -> str:
    return base64.b64encode(json.dumps(payload).encode()).decode()


def _resolve_compute_fn(exec_globals: dict, *, allow_reference: bool = False):
    names = ["optimized_compute", "kernel_fn"]
    if allow_reference:
        names += ["simple_compute", "reference_fn"]
    for name in names:
        fn = exec_globals.get(name)
        if fn is not None:
            return fn
    return None


def _has_cuda() -> bool:
    try:
        import torch
        if not torch.cuda.is_available():
            return False
        major, _ = torch.cuda.get_device_capability()
        return major == 10
    except Exception:
        return False


def _to_numpy(x) -> np.ndarray:
    try:
        import torch
        if isinstance(x, torch.Tensor):
            return x.detach().float().cpu().numpy()
    except ImportError:
        pass
    return np.asarray(x, dtype=np.float64)


# ---------------------------------------------------------------------------
# Stages
# ---------------------------------------------------------------------------
def stage_compile(kernel_code: str) -> dict:
    try:
        g: dict = {}
        exec(kernel_code, g)
        return {"ok": True, "globals": g}
    except Exception:
        return {"ok": False, "error": f"Compilation error: {traceback.format_exc()}"}


def stage_correctness(kernel_code: str, reference_code: str, shapes, rtol: float, atol: float,
                      exec_globals: dict) -> dict:
    try:
        ref_globals: dict = {}
        exec(reference_code, ref_globals)
        kernel_fn = _resolve_compute_fn(exec_globals)
        ref_fn = _resolve_compute_fn(ref_globals, allow_reference=True)
        if kernel_fn is None or ref_fn is None:
            return {"ok": False, "error": "Could not find kernel_fn/reference_fn", "max_diff": 0.0}
        worst = 0.0
        for shape in shapes:
            got = _to_numpy(kernel_fn(**shape))
            ref = _to_numpy(ref_fn(**shape))
            if got.shape != ref.shape:
                return {"ok": False, "max_diff": float("inf"),
                        "error": f"Shape mismatch for {shape}: {got.shape} vs {ref.shape}"}
            if not np.isfinite(got).all():
                return {"ok": False, "max_diff": float("inf"),
                        "error": f"Non-finite kernel output for shape {shape}"}
            diff = np.abs(got - ref)
            max_diff = float(diff.max()) if diff.size else 0.0
            worst = max(worst, max_diff)
            if got.ndim == 0:
                bad = max_diff > atol
            else:
                bad = bool((diff > atol + rtol * np.abs(ref)).any())
            if bad:
                return {"ok": False, "max_diff": max_diff,
                        "error": f"Correctness failed for shape {shape}: max_diff={max_diff}"}
        return {"ok": True, "max_diff": worst}
    except Exception:
        return {"ok": False, "error": f"Correctness error: {traceback.format_exc()}",
                "max_diff": 0.0}


def benchmark_stats(times_ms, compile_time_ms: float, peak_memory_mb, source: str) -> dict:
    t = np.asarray(times_ms, dtype=np.float64)
    med = float(np.median(t))
    return {"lower_time_ms": 0.0, "compile_time_ms": compile_time_ms,
            "evaluation_times_ms": [float(x) for x in t], "peak_memory_mb": peak_memory_mb,
            "median_ms": med, "min_ms": float(t.min()), "max_ms": float(t.max()),
            "stddev_ms": float(t.std()), "cv": float(t.std() / med) if med > 0 else 0.0,
            "timing_source": source}


def _cuda_timer() -> Callable[[Callable[[], Any]], float]:
    import torch

    def run(fn):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1)
    return run


def stage_benchmark(exec_globals: dict, shapes, warmup: int = 3, n_iters: int = 5,
                    timer: Optional[Callable] = None) -> dict:
    """Times the compute function on the first shape: the first call
    (module load, allocation) is reported as compile time, then `warmup`
    untimed calls and `n_iters` timed calls."""
    try:
        fn = _resolve_compute_fn(exec_globals, allow_reference=True)
        if fn is None:
            return {"ok": False, "error": "No compute function found"}
        shape = shapes[0]
        source = "cuda_events"
        peak = None
        if timer is None:
            import torch
            timer = _cuda_timer()
            torch.cuda.reset_peak_memory_stats()
        else:
            source = "injected"
        compile_ms = timer(lambda: fn(**shape))
        for _ in range(warmup):
            fn(**shape)
        times = [timer(lambda: fn(**shape)) for _ in range(n_iters)]
        if source == "cuda_events":
            import torch
            peak = torch.cuda.max_memory_allocated() / (1024 * 1024)
        bench = benchmark_stats(times, compile_ms, peak, source)
        return {"ok": True, "latency_ms": bench["median_ms"], "benchmark": bench}
    except Exception:
        return {"ok": False, "error": f"Benchmark error: {traceback.format_exc()}"}


def forward_flops(shape: dict) -> float:
    """Algorithmic forward FLOPs of the two scored kernels for a shape dict."""
    if {"M", "K", "N"} <= set(shape):
        return 2.0 * shape["M"] * shape["K"] * shape["N"]
    if {"B", "T", "H", "K", "V"} <= set(shape):
        C = shape.get("chunk_size", 64)
        K, V = shape["K"], shape["V"]
        return float(shape["B"]) * shape["T"] * shape["H"] * (2 * C * K + 2 * C * V + 4 * K * V)
    return 0.0


# ---------------------------------------------------------------------------
# Deep profile (replaces the TPU evaluator's xprof counters / LLO analysis,
# KE/docker/evaluate.py:286-377, 427-475, 478-889): the kernel function runs
# once more in a child process under ncu, restricted to a cudaProfilerStart /
# Stop window around one call, and the per-launch counters are averaged
# (weighted by launch time) into the result's compute_ratio /
# memory_transfer_ratio and metadata["hw_utilization"].
# ---------------------------------------------------------------------------
NCU_METRICS = {
    "gpu__time_duration.sum": "duration_ns",
    "sm__throughput.avg.pct_of_peak_sustained_elapsed": "sm_throughput_pct",
    "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed": "dram_util_pct",
    "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_elapsed": "tensor_util_pct",
    "sm__pipe_fma_cycles_active.avg.pct_of_peak_sustained_elapsed": "fma_util_pct",
    "sm__pipe_alu_cycles_active.avg.pct_of_peak_sustained_elapsed": "alu_util_pct",
    "sm__pipe_shared_cycles_active.avg.pct_of_peak_sustained_elapsed": "shared_pipe_util_pct",
    "smsp__issue_active.avg.pct_of_peak_sustained_active": "issue_active_pct",
    "l1tex__throughput.avg.pct_of_peak_sustained_elapsed": "l1_util_pct",
    "lts__throughput.avg.pct_of_peak_sustained_elapsed": "l2_util_pct",
    "dram__bytes_read.sum": "dram_read_bytes",
    "dram__bytes_write.sum": "dram_write_bytes",
}
_UNIT_SCALE = {"byte": 1.0, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9, "Tbyte": 1e12,
               "nsecond": 1.0, "usecond": 1e3, "msecond": 1e6, "second": 1e9,
               "ns": 1.0, "us": 1e3, "ms": 1e6, "s": 1e9, "%": 1.0, "": 1.0}


def parse_ncu_csv(text: str) -> list:
    """ncu `--csv` output (one row per launch and metric) -> one dict per
    launch: {"kernel": name, <NCU_METRICS keys>: value in bytes / ns / %}."""
    import csv
    import io
    lines = [ln for ln in text.splitlines() if ln.startswith('"')]
    if not lines:
        return []
    rows = list(csv.reader(io.StringIO("\n".join(lines))))
    hdr = rows[0]
    need = ("ID", "Kernel Name", "Metric Name", "Metric Unit", "Metric Value")
    if not all(h in hdr for h in need):
        return []
    ix = {h: hdr.index(h) for h in need}
    launches = {}
    for r in rows[1:]:
        if len(r) < len(hdr):
            continue
        name = r[ix["Metric Name"]]
        if name not in NCU_METRICS:
            continue
        try:
            val = float(r[ix["Metric Value"]].replace(",", ""))
        except ValueError:
            continue
        val *= _UNIT_SCALE.get(r[ix["Metric Unit"]], 1.0)
        d = launches.setdefault(r[ix["ID"]], {"kernel": r[ix["Kernel Name"]]})
        d[NCU_METRICS[name]] = val
    return list(launches.values())


def summarize_launches(launches: list) -> dict:
    """Time-weighted averages of the per-launch counters.  compute_ratio is
    the SM share and memory_transfer_ratio the DRAM share of
    (SM throughput % + DRAM throughput %), so the two add up to 1 as the TPU
    evaluator's compute / memory-transfer split does."""
    tot = sum(l.get("duration_ns", 0.0) for l in launches)
    if not launches or tot <= 0:
        return {"ok": False, "error": "no profiled launches"}
    util = {}
    for key in NCU_METRICS.values():
        if key in ("duration_ns", "dram_read_bytes", "dram_write_bytes"):
            continue
        vals = [(l[key], l.get("duration_ns", 0.0)) for l in launches if key in l]
        if vals:
            util[key] = sum(v * w for v, w in vals) / max(sum(w for _, w in vals), 1e-30)
    util["dram_bytes"] = sum(l.get("dram_read_bytes", 0.0) + l.get("dram_write_bytes", 0.0)
                             for l in launches)
    util["kernel_time_ms"] = tot / 1e6
    util["launches"] = len(launches)
    sm, dram = util.get("sm_throughput_pct", 0.0), util.get("dram_util_pct", 0.0)
    share = sm / (sm + dram) if sm + dram > 0 else None
    return {"ok": True, "compute_ratio": share,
            "memory_transfer_ratio": None if share is None else 1.0 - share,
            "hw_utilization": util,
            "kernels": sorted({l["kernel"] for l in launches})}


def profile_command(payload_b64: str, ncu: str = "ncu") -> list:
    """ncu command that profiles the launches of one kernel call (the child
    brackets the call with cudaProfilerStart / Stop)."""
    return [ncu, "--profile-from-start", "off", "--clock-control", "none", "--csv",
            "--print-units", "base", "--metrics", ",".join(NCU_METRICS), sys.executable, "-m", "glaucis_b200.evaluate",
            "--profile-child", payload_b64]


def _profile_child(request: dict) -> int:
    """Child side of the deep profile: compile, one warm-up call, then one
    call inside the profiler window."""
    import torch
    comp = stage_compile(request["kernel_code"])
    if not comp["ok"]:
        print(comp["error"], file=sys.stderr)
        return 1
    fn = _resolve_compute_fn(comp["globals"], allow_reference=True)
    shape = request["shapes"][0]
    fn(**shape)
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    fn(**shape)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    return 0


def stage_profile_deep(request: dict, runner: Optional[Callable] = None, timeout: int = 600) -> dict:
    """Runs the child once without ncu (it must exit 0 first) and once under
    ncu, then summarises the counters.  `runner(argv) -> (returncode, stdout,
    stderr)` replaces subprocess for tests."""
    import shutil
    if runner is None:
        ncu = shutil.which("ncu") or "/usr/local/cuda/bin/ncu"
        if not os.path.exists(ncu):
            return {"ok": False, "error": "ncu not found"}

        def runner(argv):
            p = subprocess.run(argv, capture_output=True, text=True, timeout=timeout)
            return p.returncode, p.stdout, p.stderr
    else:
        ncu = "ncu"
    payload = encode_request({"kernel_code": request["kernel_code"], "shapes": request["shapes"]})
    plain = [sys.executable, "-m", "glaucis_b200.evaluate", "--profile-child", payload]
    rc, _, err = runner(plain)
    if rc != 0:
        return {"ok": False, "error": f"profile child failed without ncu: {err[-500:]}"}
    rc, out, err = runner(profile_command(payload, ncu))
    if rc != 0:
        return {"ok": False, "error": f"ncu failed: {err[-500:]}"}
    return summarize_launches(parse_ncu_csv(out))


def evaluate(request: dict, timer: Optional[Callable] = None) -> dict:
    """Runs the stages for one variant and returns the result dict."""
    job = request.get("variant_id", "unknown")
    comp = stage_compile(request["kernel_code"])
    if not comp["ok"]:
        return {"status": "COMPILE_ERROR", "variant_id": job, "error": comp["error"]}
    corr = stage_correctness(request["kernel_code"], request["reference_code"], request["shapes"],
                             request.get("rtol", 1e-2), request.get("atol", 1e-2), comp["globals"])
    if not corr["ok"]:
        return {"status": "INCORRECT", "variant_id": job, "error": corr["error"],
                "max_diff": corr["max_diff"]}
    bench = stage_benchmark(comp["globals"], request["shapes"], timer=timer)
    if not bench["ok"]:
        return {"status": "COMPILE_ERROR", "variant_id": job, "error": bench["error"]}
    ref_comp = stage_compile(request["reference_code"])
    ref_bench = (stage_benchmark(ref_comp["globals"], request["shapes"], timer=timer)
                 if ref_comp["ok"] else {"ok": False})
    ref_latency = ref_bench.get("latency_ms", bench["latency_ms"])
    speedup = ref_latency / bench["latency_ms"] if bench["latency_ms"] > 0 else 0.0
    deep = stage_profile_deep(request) if request.get("deep_profile") else None
    deep_ok = bool(deep and deep.get("ok"))
    return {
        "status": "SUCCESS", "variant_id": job, "fitness": speedup,
        "latency_ms": bench["latency_ms"], "speedup": speedup,
        "flops": forward_flops(request["shapes"][0]),
        "compute_ratio": deep["compute_ratio"] if deep_ok else None,
        "memory_transfer_ratio": deep["memory_transfer_ratio"] if deep_ok else None,
        "max_diff": corr["max_diff"],
        "metadata": {"reference_latency_ms": ref_latency,
                     "reference_perf_ok": ref_bench.get("ok", False),
                     "benchmark": bench.get("benchmark"),
                     "reference_benchmark": ref_bench.get("benchmark"),
                     "hw_utilization": deep.get("hw_utilization") if deep_ok else None,
                     "profile": None if deep is None else
                     {k: v for k, v in deep.items() if k not in ("hw_utilization",)}},
    }


def batch_dispatch(payload: dict, per_variant_timeout: int = 1500,
                   argv_prefix: Optional[list] = None) -> list:
    """One subprocess per variant (GPU isolation); a crash or timeout becomes
    a COMPILE_ERROR line (KE/src/kernel_evolve/docker_evaluate_helpers.py:15-77)."""
    prefix = argv_prefix or [sys.executable, "-m", "glaucis_b200.evaluate"]
    lines = []
    for variant in payload["variants"]:
        vid = variant["variant_id"]
        single = {"variant_id": vid, "kernel_code": variant["kernel_code"],
                  "reference_code": payload["reference_code"], "shapes": payload["shapes"],
                  "rtol": payload.get("rtol", 1e-2), "atol": payload.get("atol", 1e-2)}
        env = dict(os.environ, VARIANT_ID=vid)
        try:
            proc = subprocess.run(prefix + ["--eval-payload", encode_request(single)],
                                  capture_output=True, text=True, timeout=per_variant_timeout,
                                  env=env)
            found = None
            for line in proc.stdout.splitlines():
                if "EVAL_RESULT:" in line:
                    found = json.loads(line.split("EVAL_RESULT:", 1)[1].strip())
                    found.setdefault("variant_id", vid)
                    break
            if found is None:
                err = proc.stderr[-500:] if proc.stderr else "No EVAL_RESULT in output"
                found = {"variant_id": vid, "status": "COMPILE_ERROR", "error": err}
        except subprocess.TimeoutExpired:
            found = {"variant_id": vid, "status": "COMPILE_ERROR",
                     "error": f"Subprocess timeout after {per_variant_timeout}s"}
        lines.append(f"EVAL_RESULT:{json.dumps(found)}")
    return lines


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="CUDA evaluator backend (EVAL_RESULT contract)")
    ap.add_argument("--eval-payload")
    ap.add_argument("--eval-payload-file")
    ap.add_argument("--profile-child", help=argparse.SUPPRESS)
    args = ap.parse_args(argv)
    if args.profile_child:
        return _profile_child(decode_request(args.profile_child))
    if args.eval_payload_file:
        with open(args.eval_payload_file) as f:
            b64 = f.read().strip()
    elif args.eval_payload:
        b64 = args.eval_payload
    else:
        ap.error("--eval-payload or --eval-payload-file is required")
    request = decode_request(b64)
    if request.get("batch"):
        for line in batch_dispatch(request):
            print(line)
        return 0
    if not _has_cuda():
        print("ERROR: no sm_100 CUDA device. This evaluator requires a B200.", file=sys.stderr)
        return 1
    print(f"EVAL_RESULT:{json.dumps(evaluate(request))}", flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
