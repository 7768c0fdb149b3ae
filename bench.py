"""Benchmark of the B200 grouped FP8 matmul forward (headline) and the fused
chunked-GLA forward, one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Headline workload: gmm_moe_up — G=128 experts, M=32768 routed rows (4096
tokens x top-8, Zipf(1.2) routing, some experts empty), K=7168, N=2048, e4m3
operands with 1x128 / 128x128 fp32 block scales, bf16 output.  One step = one
grouped-matmul launch over the resident, pre-quantised operands (inputs are
larger than L2: 2.1 GB of e4m3 operands, so no flush is needed).
`value` = whole-job TFLOP/s (algorithmic 2*M*K*N per step, summed over ranks,
divided by the slowest rank's time).

Multi-GPU (torchrun, one process per GPU): weak scaling — every rank runs
its own instance of the workload (its own seeded routing), no data-path
collective; timing is the max over ranks.

`e2e` times the public op gmm_fp8_blockwise(lhs, rhs, group_sizes) from
pinned host activations: H2D of lhs + group_sizes, activation and weight
quantisation, the grouped matmul, D2H of the bf16 output.  The bf16 weights
stay resident on the device (model parameters).

`--impl reference` times the CPU restatement of the same path (the reference
itself is JAX + tokamax on TPU and cannot run here) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "FP8 GMM TFLOP/s & chunk_gla fwd tokens/s at 1/2/4/8 B200, % of roofline"
HEADLINE = "gmm_moe_up"
GLA_WORKLOAD = "gla_b8_t4096"
GLA_LONG_WORKLOAD = "gla_b1_t32768"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return dict(PEAKS_FALLBACK), "fallback"


def ncu_traffic(kernel: str, workload: str):
    """DRAM bytes (read + write) per launch of `kernel` on `workload` as
    recorded from an ncu capture in profiles/ncu_traffic.json, else None."""
    p = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        d = json.load(f)
    e = d.get(f"{kernel}@{workload}")
    return None if e is None else e.get("dram_bytes_per_launch")


# ---------------------------------------------------------------------------
# Clock sampling (NVML, polled from a thread during the timed region)
# ---------------------------------------------------------------------------
_REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
            0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
            0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
            0x100: "display_clock_setting"}


class ClockSampler:
    def __init__(self, device_index: int):
        self.samples = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            uuid = None
            try:
                import torch
                uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            except Exception:
                pass
            h = None
            if uuid:
                for i in range(pynvml.nvmlDeviceGetCount()):
                    hh = pynvml.nvmlDeviceGetHandleByIndex(i)
                    u = pynvml.nvmlDeviceGetUUID(hh)
                    u = u.decode() if isinstance(u, bytes) else u
                    if u.replace("GPU-", "") == uuid.replace("GPU-", ""):
                        h = hh
            self._h = h if h is not None else pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self._nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._ok = True
        except Exception:
            self._ok = False

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                self.reasons |= int(nv.nvmlDeviceGetCurrentClocksEventReasons(self._h))
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self._ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._ok:
            self._t.join()

    def summary(self):
        if not self._ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"],
                    "samples": 0}
        names = [n for bit, n in _REASONS.items() if self.reasons & bit and n != "gpu_idle"]
        return {"sm_mhz": float(statistics.median(self.samples)), "sm_max_mhz": self.max_mhz,
                "reasons": names, "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# Distributed plumbing
# ---------------------------------------------------------------------------
def dist_setup(n_gpus: int):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}; launch with torchrun")
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    """Slowest rank's value (NCCL on the device, gloo on the host)."""
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def whole_job_rate(units_per_rank: float, world: int, ms_slowest: float) -> float:
    """Weak scaling: every rank processes `units_per_rank`; the job's rate is
    the units of all ranks over the slowest rank's time (units per second)."""
    return world * units_per_rank / (ms_slowest * 1e-3)


def timed(fn, steps: int, warmup: int, world: int, sampler=None):
    """Device time per step (ms) with CUDA events on the launching stream,
    bracketed by barrier + synchronize; max over ranks."""
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier(world)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    ctx = sampler if sampler is not None else _Null()
    with ctx:
        torch.cuda.synchronize()
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
    barrier(world)
    return max_over_ranks(e0.elapsed_time(e1) / steps, world)


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


# ---------------------------------------------------------------------------
# CPU baselines (the oracle restatement, timed on the host cores)
# ---------------------------------------------------------------------------
def cpu_gmm_step(sample_rows: int, seed: int = 0):
    """Builds a bounded sample of the headline workload (its first non-empty
    experts, about `sample_rows` rows, full K and N) for the BLAS-backed CPU
    restatement.  Returns (step_fn, flops_per_step, description)."""
    import torch
    from glaucis_b200 import configs
    from oracle import cpu_fast
    cfg = configs.GMM_CONFIGS[HEADLINE]
    sizes = configs.group_sizes(cfg.routing, cfg.G, cfg.M, seed=seed, topk=cfg.topk, zipf=cfg.zipf)
    sel = []
    rows = 0
    for g in range(cfg.G):
        if sizes[g] > 0:
            sel.append(int(sizes[g]))
            rows += int(sizes[g])
            if rows >= sample_rows:
                break
    gen = torch.Generator().manual_seed(seed)
    lhs = torch.randn((rows, cfg.K), generator=gen).to(torch.bfloat16)
    rhs = (torch.randn((len(sel), cfg.K, cfg.N), generator=gen) * cfg.rhs_std).to(torch.bfloat16)

    def step():
        cpu_fast.gmm_fp8_blockwise(lhs, rhs, sel)

    flops = 2.0 * rows * cfg.K * cfg.N
    desc = (f"{len(sel)} of {cfg.G} experts of {HEADLINE} ({rows} of {cfg.M} rows, K={cfg.K}, "
            f"N={cfg.N}): quantise lhs+rhs, dequantised fp32 GEMM per expert (torch CPU, BLAS)")
    return step, flops, desc


def cpu_gla_step(tokens: int, seed: int = 0):
    import torch
    from glaucis_b200 import configs
    from oracle import cpu_fast
    cfg = configs.GLA_CONFIGS[GLA_WORKLOAD]
    inp = configs.make_gla_inputs(configs.GLAConfig("cpu", B=1, T=tokens, H=cfg.H), device="cpu",
                                  seed=seed)

    def step():
        cpu_fast.chunk_gla_fwd(inp["q"], inp["k"], inp["v"], g=inp["g"], scale=128 ** -0.5)

    desc = (f"B=1, T={tokens}, H={cfg.H} of {GLA_WORKLOAD} (K=V=128, C=64, per-key gate): "
            f"fp32 chunked restatement (torch CPU, BLAS)")
    return step, tokens, desc


def cpu_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def time_cpu(step, reps: int):
    step()  # warm
    ts = []
    for _ in range(reps):
        t = time.perf_counter()
        step()
        ts.append(time.perf_counter() - t)
    return statistics.median(ts)


# ---------------------------------------------------------------------------
# Reference arm
# ---------------------------------------------------------------------------
def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    cores = cpu_cores()
    try:
        import torch
        torch.set_num_threads(cores)
    except Exception:
        pass
    # keep the whole arm to a couple of minutes whatever --steps/--warmup are
    rows = max(256, int(args.cpu_rows * min(1.0, 13.0 / (args.steps + args.warmup))))
    step, flops, desc = cpu_gmm_step(sample_rows=rows)
    for _ in range(args.warmup):
        step()
    t = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t) / args.steps
    value = flops / dt / 1e12
    gstep, gtok, gdesc = cpu_gla_step(tokens=args.cpu_gla_tokens)
    gdt = time_cpu(gstep, 3)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "e4m3 x e4m3 -> fp32 (dequantised fp32 GEMM on the host)",
        "data": "synthetic",
        "config": {"workload": HEADLINE, "G": 128, "M": 32768, "K": 7168, "N": 2048,
                   "routing": "zipf(1.2) top-8", "sample": desc},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": cores, "kind": "port",
                         "sample": desc},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "gla": {"workload": GLA_WORKLOAD, "tokens_per_s": gtok / gdt, "sample": gdesc},
        "note": ("the reference path (JAX + qwix + tokamax Pallas on TPU) cannot run on this "
                 "box; this arm times the CPU restatement of the same forward in oracle/"),
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# B200 arm
# ---------------------------------------------------------------------------
def run_b200(args):
    import torch
    from glaucis_b200 import configs, ops
    rank, world, local = dist_setup(args.gpus)
    peaks, peak_kind = load_peaks()
    traffic = ncu_traffic("gmm_fp8_fwd_kernel", args.workload)
    fp8_peak = 2.0 * peaks["bf16_tflops"]

    # ---------------------------------------------------------------- GMM
    cfg = configs.GMM_CONFIGS[args.workload]
    lhs, rhs, gs = configs.make_gmm_inputs(cfg, device="cuda", seed=args.seed + rank)
    a_q, a_s = ops.quant_act_1x128(lhs)
    b_q, b_s = ops.quant_w_128x128(rhs)
    out = torch.empty((cfg.M, cfg.N), dtype=torch.bfloat16, device="cuda")
    sizes = gs.cpu().numpy()
    g_nz = int((sizes > 0).sum())
    flops = 2.0 * float(sizes.sum()) * cfg.K * cfg.N
    alg_bytes = (cfg.M * cfg.K + 4 * cfg.M * cfg.K / 128 + g_nz * cfg.K * cfg.N
                 + 4 * g_nz * (cfg.K / 128) * (cfg.N / 128) + 4 * cfg.G + 2 * cfg.M * cfg.N)

    def gmm_step():
        ops.gmm_fp8_fwd(a_q, a_s, b_q, b_s, gs, out=out)

    sampler = ClockSampler(local) if rank == 0 else None
    ms = timed(gmm_step, args.steps, args.warmup, world, sampler)
    status = ops.device_status()
    if status != 0:
        raise SystemExit(f"device error word {status} after the timed region")
    value = whole_job_rate(flops, world, ms) / 1e12
    ai = flops / alg_bytes
    ridge = fp8_peak * 1e12 / (peaks["hbm_gbs"] * 1e9)
    bound = "hbm" if ai < ridge else "tensor"
    if bound == "hbm":
        achieved = alg_bytes / (ms * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / peaks["hbm_gbs"], "traffic": traffic,
                "peak_source": f"{peak_kind} hbm_gbs"}
    else:
        achieved = flops / (ms * 1e-3) / 1e12
        roof = {"bound": "tensor", "achieved": achieved, "peak": fp8_peak, "unit": "TFLOP/s",
                "frac": achieved / fp8_peak, "traffic": traffic,
                "peak_source": f"2 x {peak_kind} bf16_tflops (dense e4m3 rate)"}
    roof["kernel"] = "gmm_fp8_fwd_kernel"
    roof["fp8_tensor_frac"] = flops / (ms * 1e-3) / 1e12 / fp8_peak
    roof["algorithmic_bytes_per_launch"] = alg_bytes
    roof["algorithmic_flops_per_launch"] = flops

    # quantiser rows (separately timed kernels of the same forward)
    # outputs preallocated: the timed region holds the quantiser kernels only
    qa_o, sa_o = torch.empty_like(a_q), torch.empty_like(a_s)
    qw_o, sw_o = torch.empty_like(b_q), torch.empty_like(b_s)
    qs_act = ClockSampler(local) if rank == 0 else None
    q_act_ms = timed(lambda: ops.quant_act_1x128(lhs, qa_o, sa_o), max(5, args.steps // 2), 3, world,
                     qs_act)
    qs_w = ClockSampler(local) if rank == 0 else None
    q_w_ms = timed(lambda: ops.quant_w_128x128(rhs, qw_o, sw_o), max(5, args.steps // 10), 3, world,
                   qs_w)
    del qa_o, sa_o, qw_o, sw_o
    # algorithmic bytes: bf16 in, e4m3 out, fp32 scales out
    q_act_bytes = lhs.numel() * 3 + lhs.numel() // 128 * 4
    q_w_bytes = rhs.numel() * 3 + rhs.numel() // (128 * 128) * 4
    quantisers = {
        name: {"ms": ms_, "achieved_gbs": by / (ms_ * 1e-3) / 1e9,
               "frac": by / (ms_ * 1e-3) / 1e9 / peaks["hbm_gbs"], "algorithmic_bytes": by,
               "sm_mhz": cs.summary()["sm_mhz"] if cs else None}
        for name, ms_, by, cs in (("quant_act_1x128", q_act_ms, q_act_bytes, qs_act),
                                  ("quant_w_128x128", q_w_ms, q_w_bytes, qs_w))}

    # ---------------------------------------------------------------- e2e
    # ------------------------------------------------- GMM backward rows
    # dlhs (grouped kernel, weight transposed) and drhs (tgmm) on the same
    # workload with a synthetic output gradient, quantised inputs resident.
    gen = torch.Generator(device="cuda").manual_seed(args.seed + 7 + rank)
    grad = torch.randn((cfg.M, cfg.N), device="cuda", generator=gen).to(torch.bfloat16)
    dq1, ds1 = ops.quant_act_1x128(grad)
    dq2, ds2 = ops.quant_col_128x1(grad)
    lq, ls = ops.quant_col_128x1(lhs)
    dlhs = torch.zeros((cfg.M, cfg.K), dtype=torch.bfloat16, device="cuda")
    drhs = torch.empty((cfg.G, cfg.K, cfg.N), dtype=torch.bfloat16, device="cuda")
    dl_ms = timed(lambda: ops.gmm_fp8_dlhs(dq1, ds1, b_q, b_s, gs, out=dlhs), max(5, args.steps // 2), 3, world)
    tg_ms = timed(lambda: ops.tgmm_fp8(lq, ls, dq2, ds2, gs, out=drhs), max(5, args.steps // 2), 3, world)
    qc_ms = timed(lambda: ops.quant_col_128x1(grad, dq2, ds2), max(5, args.steps // 2), 3, world)
    if ops.device_status() != 0:
        raise SystemExit("device error word set after the backward rows")
    dl_bytes = (cfg.M * cfg.N + 4 * cfg.M * cfg.N / 128 + g_nz * cfg.K * cfg.N
                + 4 * g_nz * (cfg.K / 128) * (cfg.N / 128) + 2 * cfg.M * cfg.K)
    tg_bytes = (cfg.M * cfg.K + 4 * cfg.M * cfg.K / 128 + cfg.M * cfg.N + 4 * cfg.M * cfg.N / 128
                + 2 * cfg.G * cfg.K * cfg.N)
    qc_bytes = grad.numel() * 3 + grad.numel() // 128 * 4

    def row(ms_, by, fl):
        gbs = by / (ms_ * 1e-3) / 1e9
        r = {"ms": ms_, "achieved_gbs": gbs, "hbm_frac": gbs / peaks["hbm_gbs"],
             "algorithmic_bytes": by}
        if fl:
            r["tflops"] = world * fl / (ms_ * 1e-3) / 1e12
            r["fp8_tensor_frac"] = fl / (ms_ * 1e-3) / 1e12 / fp8_peak
        return r

    gmm_bwd = {"workload": args.workload,
               "dlhs": row(dl_ms, dl_bytes, flops), "tgmm": row(tg_ms, tg_bytes, flops),
               "quant_col_128x1": row(qc_ms, qc_bytes, 0.0),
               "note": "dlhs = gl_gmm_fp8_dlhs (grouped kernel, K-major weight); tgmm writes "
                       "drhs [G, K, N] bf16 for every group (empty ones as zeros)"}
    del grad, dq1, ds1, dq2, ds2, lq, ls, dlhs, drhs
    torch.cuda.empty_cache()

    e2e = None
    if not args.skip_e2e:
        lhs_h = lhs.cpu().pin_memory()
        gs_h = gs.cpu().pin_memory()
        out_h = torch.empty((cfg.M, cfg.N), dtype=torch.bfloat16).pin_memory()
        n_chunks = len(ops._plan_chunks(gs_h.numpy(), 16)[0])

        def e2e_step():
            # public host-input op: pinned activations and group sizes in,
            # pinned bf16 output back; copies overlap the kernels
            ops.gmm_fp8_blockwise_host(lhs_h, rhs, gs_h, out=out_h, out_dtype=torch.bfloat16)

        e_steps = max(1, min(args.steps, args.e2e_steps))
        e_ms = timed(e2e_step, e_steps, min(args.warmup, 2), world)
        # the host link at the time of the run: plain pinned copies of the
        # same activations and output (best of three, CUDA events), so the
        # e2e figure can be read against the PCIe bound of this box
        def copy_ms(dst, src):
            best = float("inf")
            for _ in range(3):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                dst.copy_(src, non_blocking=True)
                e1.record()
                e1.synchronize()
                best = min(best, e0.elapsed_time(e1))
            return best
        h2d_ms = copy_ms(lhs, lhs_h)
        out_d = torch.empty((cfg.M, cfg.N), dtype=torch.bfloat16, device="cuda")
        d2h_ms = copy_ms(out_h, out_d)
        del out_d
        e2e = {"value": world * flops / (e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
               "h2d_bytes_per_step": lhs_h.numel() * 2 + n_chunks * cfg.G * 4,
               "d2h_bytes_per_step": out_h.numel() * 2, "ms_per_step": e_ms,
               "link": {"h2d_gbs": lhs_h.numel() * 2 / (h2d_ms * 1e-3) / 1e9,
                        "d2h_gbs": out_h.numel() * 2 / (d2h_ms * 1e-3) / 1e9,
                        "h2d_ms": h2d_ms, "d2h_ms": d2h_ms,
                        "note": "one plain pinned copy each way of the step's activations / output"},
               "path": "gmm_fp8_blockwise_host(lhs, rhs, group_sizes): H2D lhs in 16 row chunks "
                       "overlapping quantise lhs (per chunk) + rhs and the grouped matmul, D2H bf16 out "
                       "per chunk"}
        del lhs_h, out_h

    del lhs, rhs, a_q, b_q, out
    torch.cuda.empty_cache()

    # ---------------------------------------------------------------- GLA
    def gla_block(workload):
        gcfg = configs.GLA_CONFIGS[workload]
        inp = configs.make_gla_inputs(gcfg, device="cuda", seed=args.seed + rank)
        go = torch.empty_like(inp["v"])
        ght = torch.empty((gcfg.B, gcfg.H, 128, 128), device="cuda")

        def gla_step():
            ops.chunk_gla_fwd(inp["q"], inp["k"], inp["v"], inp["g_gamma"], 128 ** -0.5, 64,
                              g=inp["g"], h0=inp["h0"], output_final_state=True, o=go, ht=ght)

        gla_ms = timed(gla_step, args.steps, args.warmup, world)
        if ops.device_status() != 0:
            raise SystemExit("device error word set after the GLA timed region")
        gla_bytes = configs.gla_bytes(gcfg.B, gcfg.T, gcfg.H, has_h0=gcfg.h0_std > 0)
        gla_flops = configs.gla_flops(gcfg.B, gcfg.T, gcfg.H)
        gla_gbs = gla_bytes / (gla_ms * 1e-3) / 1e9
        blk = {"workload": workload, "B": gcfg.B, "T": gcfg.T, "H": gcfg.H,
               "tokens_per_s": world * gcfg.B * gcfg.T / (gla_ms * 1e-3), "ms_per_step": gla_ms,
               "tflops": world * gla_flops / (gla_ms * 1e-3) / 1e12,
               "roofline": {"bound": "hbm", "achieved": gla_gbs, "peak": peaks["hbm_gbs"],
                            "unit": "GB/s", "frac": gla_gbs / peaks["hbm_gbs"],
                            "bf16_tensor_frac": gla_flops / (gla_ms * 1e-3) / 1e12 / peaks["bf16_tflops"],
                            "kernel": "chunk_gla_fwd_kernel", "peak_source": f"{peak_kind} hbm_gbs",
                            "algorithmic_bytes_per_step": gla_bytes,
                            "traffic": ncu_traffic("chunk_gla_fwd_kernel", workload)}}
        # backward: the training forward (o, ht and the per-chunk states h)
        # and the backward (reverse state-gradient scan + chunk-parallel
        # dq/dk/dv kernel) on a synthetic output gradient, buffers resident
        gh = torch.empty((gcfg.B, gcfg.T // 64, gcfg.H, 128, 128), dtype=torch.bfloat16,
                         device="cuda")

        def fwd_states_step():
            ops.chunk_gla_fwd(inp["q"], inp["k"], inp["v"], inp["g_gamma"], 128 ** -0.5, 64,
                              g=inp["g"], h0=inp["h0"], output_final_state=True, output_states=True,
                              o=go, ht=ght, h=gh)

        fs_ms = timed(fwd_states_step, max(5, args.steps // 2), 3, world)
        gen = torch.Generator(device="cuda").manual_seed(args.seed + 11 + rank)
        gdo = torch.randn(inp["v"].shape, generator=gen, device="cuda").to(torch.bfloat16)
        dq, dk, dv = (torch.empty_like(inp[n]) for n in ("q", "k", "v"))
        gws = torch.empty(ops.chunk_gla_bwd_workspace_bytes(gcfg.B, gcfg.T, gcfg.H),
                          dtype=torch.uint8, device="cuda")

        def bwd_step():
            ops.chunk_gla_bwd(inp["q"], inp["k"], inp["v"], gdo, gh, inp["g_gamma"], 128 ** -0.5, 64,
                              g=inp["g"], dq=dq, dk=dk, dv=dv, workspace=gws)

        bw_ms = timed(bwd_step, max(5, args.steps // 2), 3, world)
        if ops.device_status() != 0:
            raise SystemExit("device error word set after the GLA backward rows")
        pk = inp["g"] is not None
        bw_bytes = configs.gla_bwd_bytes(gcfg.B, gcfg.T, gcfg.H, per_key_gate=pk)
        bw_min = configs.gla_bwd_bytes(gcfg.B, gcfg.T, gcfg.H, per_key_gate=pk, fused_minimum=True)
        bw_flops = configs.gla_bwd_flops(gcfg.B, gcfg.T, gcfg.H)
        bw_gbs = bw_bytes / (bw_ms * 1e-3) / 1e9
        blk["bwd"] = {
            "ms_per_step": bw_ms, "tokens_per_s": world * gcfg.B * gcfg.T / (bw_ms * 1e-3),
            "tflops": world * bw_flops / (bw_ms * 1e-3) / 1e12,
            "achieved_gbs": bw_gbs, "hbm_frac": bw_gbs / peaks["hbm_gbs"],
            "algorithmic_bytes_per_step": bw_bytes,
            "fused_minimum_bytes": bw_min,
            "fused_minimum_frac": bw_min / (bw_ms * 1e-3) / 1e9 / peaks["hbm_gbs"],
            "fwd_with_states_ms": fs_ms,
            "kernels": "chunk_gla_fwd_kernel in reverse-scan mode (+ its state-only pre-pass and "
                       "fold when the sequence is split), then chunk_gla_bwd_kernel",
        }
        del inp, go, ght, gh, gdo, dq, dk, dv, gws
        torch.cuda.empty_cache()
        return blk

    gla = gla_block(GLA_WORKLOAD)
    gla_long = gla_block(GLA_LONG_WORKLOAD)

    # ------------------------------------------ one instance across ranks
    sharded = None
    if world > 1 and not args.skip_sharded:
        sharded = run_sharded(args, rank, world, max(3, args.steps // 2), 3)

    # ------------------------------------------------------- CPU baseline
    cpu = None
    if rank == 0 and world == 1 and not args.skip_cpu:
        cores = cpu_cores()
        torch.set_num_threads(cores)
        step, cflops, desc = cpu_gmm_step(sample_rows=args.cpu_rows)
        ct = time_cpu(step, 3)
        cpu = {"value": cflops / ct / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "port",
               "sample": desc}
        gstep, gtok, gdesc = cpu_gla_step(tokens=args.cpu_gla_tokens)
        gct = time_cpu(gstep, 3)
        gla["cpu_baseline"] = {"value": gtok / gct, "unit": "tokens/s", "cores": cores,
                               "kind": "port", "sample": gdesc}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "e4m3 x e4m3 -> fp32 acc, bf16 out", "data": "synthetic",
            "config": {"workload": args.workload, "G": cfg.G, "M": cfg.M, "K": cfg.K,
                       "N": cfg.N, "routing": cfg.routing, "empty_groups": cfg.G - g_nz,
                       "parallelism": f"weak: one workload instance per GPU x{world}",
                       "l2": "operands (2.1 GB e4m3) exceed L2; no flush"},
            "roofline": roof,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": args.steps,
            "clocks": sampler.summary() if sampler else None,
            "quantisers": quantisers,
            "gmm_bwd": gmm_bwd,
            "gla": gla,
            "gla_long": gla_long,
            "sharded": sharded,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


def run_sharded(args, rank, world, steps, warmup):
    """Strong scaling of one workload instance across the ranks (N > 1 only):
    gmm_dense_expert split by expert group (row ranges at 128-row cuts) with
    an all-gather of the output rows, gla_b1_t32768 split by head with an
    all-gather of the head blocks.  Compute-only and gather-inclusive device
    times (max over ranks); rank 0 checks the gathered result against the
    single-GPU one (GMM: bit for bit; GLA: to rounding, its sequence split
    differs)."""
    import torch
    from glaucis_b200 import configs, ops, shard
    res = {}
    # ------------------------------------------------ GMM by expert group
    cfg = configs.GMM_CONFIGS["gmm_dense_expert"]
    lhs, rhs, gs = configs.make_gmm_inputs(cfg, device="cuda", seed=args.seed)
    sizes = gs.cpu().numpy()
    parts = shard.gmm_partition(sizes, world)
    me = parts[rank]
    counts = [p.rows for p in parts]
    a_q, a_s = ops.quant_act_1x128(lhs[me.r0:me.r1].contiguous())
    b_q, b_s = ops.quant_w_128x128(rhs[me.g0:me.g1].contiguous())
    gs_l = torch.from_numpy(me.sizes).to("cuda")
    out_l = torch.empty((me.rows, cfg.N), dtype=torch.bfloat16, device="cuda")
    out_full = torch.empty((sum(counts), cfg.N), dtype=torch.bfloat16, device="cuda")

    def gmm_local():
        if me.rows:
            ops.gmm_fp8_fwd(a_q, a_s, b_q, b_s, gs_l, out=out_l)

    def gmm_gathered():
        gmm_local()
        shard.all_gather_rows(out_l, counts, out_full)

    c_ms = timed(gmm_local, steps, warmup, world)
    g_ms = timed(gmm_gathered, steps, warmup, world)
    flops = 2.0 * float(sizes.sum()) * cfg.K * cfg.N
    same = None
    if rank == 0:
        fa, fs = ops.quant_act_1x128(lhs)
        fb, fbs = ops.quant_w_128x128(rhs)
        single = ops.gmm_fp8_fwd(fa, fs, fb, fbs, gs, out_dtype=torch.bfloat16)
        same = bool(torch.equal(single[: sum(counts)], out_full))
        single_cmp = single[: sum(counts)].clone()
        del fa, fs, fb, fbs, single
    if ops.device_status() != 0:
        raise SystemExit("device error word set after the sharded GMM")
    # Overlapped gather without a collective: the rank's rows are multiplied
    # in row chunks straight into its own IPC-shared output buffer, and each
    # finished chunk (a contiguous block of rows) goes to every peer's buffer
    # with one copy-engine transfer per peer over NVLink while the next chunk
    # is computed; a stream-ordered all-reduce of one int orders the readers.
    fused = None
    try:
        import torch.distributed as dist
        peers = shard.PeerBuffers(sum(counts), cfg.N)
        peer_views = [shard.tensor_at(ptr, (sum(counts), cfg.N)) for ptr in peers.ptrs]
        flag = torch.zeros(1, dtype=torch.int32, device="cuda")
        plan, _ = ops._plan_chunks(me.sizes, 4, 1024)
        chunks = [(r0, r1, torch.tensor(sub, dtype=torch.int32, device="cuda"), g_a, len(sub))
                  for r0, r1, g_a, sub in plan]
        # one copy stream per peer, so the transfers to different peers run
        # on different copy engines at the same time
        s_mm = torch.cuda.Stream()
        others = [(rank + i) % world for i in range(1, world)]
        s_cp = {r: torch.cuda.Stream() for r in others}

        def gmm_overlapped():
            cur = torch.cuda.current_stream()
            s_mm.wait_stream(cur)
            for s in s_cp.values():
                s.wait_stream(cur)
            for r0, r1, gsub, g_a, ng in chunks:
                rows = slice(me.r0 + r0, me.r0 + r1)
                with torch.cuda.stream(s_mm):
                    ops.gmm_fp8_fwd(a_q[r0:r1], a_s[r0:r1], b_q[g_a:g_a + ng], b_s[g_a:g_a + ng], gsub,
                                    out=peers.local[rows])
                    done = s_mm.record_event()
                for r in others:
                    with torch.cuda.stream(s_cp[r]):
                        s_cp[r].wait_event(done)
                        peer_views[r][rows].copy_(peers.local[rows], non_blocking=True)
            cur.wait_stream(s_mm)
            for s in s_cp.values():
                cur.wait_stream(s)
            dist.all_reduce(flag)

        f_ms = timed(gmm_overlapped, steps, warmup, world)
        fsame = bool(torch.equal(single_cmp, peers.local)) if rank == 0 else None
        fused = {"with_gather_ms": f_ms, "tflops_with_gather": flops / (f_ms * 1e-3) / 1e12,
                 "matches_single_gpu": fsame, "chunks": len(chunks),
                 "how": "row-chunked matmul into IPC-shared outputs, one copy-engine transfer per "
                        "peer per chunk (one stream per peer) overlapping the next chunk, all-reduce "
                        "barrier"}
        # One kernel: the matmul's epilogue stages every finished 32-row
        # slice in shared memory and TMA-stores it into every rank's buffer
        # (its own and the peers', over NVLink) while the next tile runs.
        peers.local.zero_()
        torch.cuda.synchronize()
        dist.barrier()

        def gmm_scatter():
            shard.gmm_fp8_fwd_gathered(a_q, a_s, b_q, b_s, me, peers, group_sizes=gs_l)

        x_ms = timed(gmm_scatter, steps, warmup, world)
        xsame = bool(torch.equal(single_cmp, peers.local)) if rank == 0 else None
        fused["epilogue_scatter"] = {
            "with_gather_ms": x_ms, "tflops_with_gather": flops / (x_ms * 1e-3) / 1e12,
            "matches_single_gpu": xsame,
            "how": "shard.gmm_fp8_fwd_gathered (gl_gmm_fp8_fwd_scatter): one kernel; each 32x128 "
                   "output slice is staged in shared memory and TMA-stored to every rank's "
                   "IPC-shared buffer"}
        del peer_views
        peers.close()
    except Exception as e:  # peer mappings unavailable: report, keep the NCCL rows
        fused = {"unavailable": f"{type(e).__name__}: {str(e)[:160]}"}
    if ops.device_status() != 0:
        raise SystemExit("device error word set after the fused sharded GMM")
    res["gmm"] = {"workload": "gmm_dense_expert", "split": "expert groups, 128-row cuts",
                  "rows_per_rank": counts, "groups_per_rank": [p.g1 - p.g0 for p in parts],
                  "compute_ms": c_ms, "with_gather_ms": g_ms,
                  "tflops_compute": flops / (c_ms * 1e-3) / 1e12,
                  "tflops_with_gather": flops / (g_ms * 1e-3) / 1e12,
                  "gather_bytes_per_rank": 2 * cfg.N * (cfg.M - me.rows),
                  "matches_single_gpu": same, "fused_gather": fused, "scaling": "strong"}
    del lhs, rhs, a_q, a_s, b_q, b_s, out_l, out_full
    if rank == 0:
        del single_cmp
    torch.cuda.empty_cache()
    # ------------------------------------------------------- GLA by head
    gcfg = configs.GLA_CONFIGS["gla_b1_t32768"]
    inp = configs.make_gla_inputs(gcfg, device="cuda", seed=args.seed)
    hr = shard.gla_head_partition(gcfg.H, world)[rank]
    heads = [len(r) for r in shard.gla_head_partition(gcfg.H, world)]
    sl = lambda t: t[:, :, hr.start:hr.stop].contiguous()
    q, k, v, g = sl(inp["q"]), sl(inp["k"]), sl(inp["v"]), sl(inp["g"])
    h0 = inp["h0"][:, hr.start:hr.stop].contiguous()
    o_l = torch.empty_like(v)
    ht_l = torch.empty_like(h0)
    blk = gcfg.B * gcfg.T * gcfg.V  # elements of one head's output

    def gla_local():
        ops.chunk_gla_fwd(q, k, v, None, 128 ** -0.5, 64, g=g, h0=h0, output_final_state=True,
                          o=o_l, ht=ht_l)

    # head-block-major staging: rank r's [B, T, H_r, V] block is row r
    width = max(heads) * blk
    stage = torch.empty((world, width), dtype=torch.bfloat16, device="cuda")

    def gla_gathered():
        gla_local()
        row = o_l.reshape(1, -1)
        if row.shape[1] < width:  # unequal head counts: pad this rank's block
            row = torch.nn.functional.pad(row, (0, width - row.shape[1]))
        shard.all_gather_rows(row, [1] * world, stage)

    c2 = timed(gla_local, steps, warmup, world)
    g2 = timed(gla_gathered, steps, warmup, world)
    err = None
    if rank == 0:
        full = ops.chunk_gla_fwd(inp["q"], inp["k"], inp["v"], None, 128 ** -0.5, 64, g=inp["g"],
                                 h0=inp["h0"], output_final_state=True).o
        worst = 0.0
        for r, hrange in enumerate(shard.gla_head_partition(gcfg.H, world)):
            got = stage[r, : gcfg.B * gcfg.T * len(hrange) * gcfg.V].view(
                gcfg.B, gcfg.T, len(hrange), gcfg.V).float()
            want = full[:, :, hrange.start:hrange.stop].float()
            worst = max(worst, float((got - want).norm() / want.norm()))
        err = worst
        del full
    if ops.device_status() != 0:
        raise SystemExit("device error word set after the sharded GLA")
    res["gla"] = {"workload": "gla_b1_t32768", "split": "heads", "heads_per_rank": heads,
                  "compute_ms": c2, "with_gather_ms": g2,
                  "tokens_per_s_compute": gcfg.B * gcfg.T / (c2 * 1e-3),
                  "tokens_per_s_with_gather": gcfg.B * gcfg.T / (g2 * 1e-3),
                  "gathered_layout": "[world, B, T, H/world, V] head blocks",
                  "rel_err_vs_single_gpu": err, "scaling": "strong"}
    del inp, q, k, v, g, h0, o_l, ht_l, stage
    torch.cuda.empty_cache()
    return res


def run_profile(args):
    """Small-footprint run of one kernel for ncu captures: the GMM on the
    headline workload with the bf16 weights freed after quantisation (about
    2.3 GB resident), the two quantisers on a slice of its operands, or the
    GLA forward on its workload."""
    import torch
    from glaucis_b200 import configs, ops
    torch.cuda.set_device(0)
    if args.profile == "gmm":
        cfg = configs.GMM_CONFIGS[args.workload]
        lhs, rhs, gs = configs.make_gmm_inputs(cfg, device="cuda", seed=args.seed)
        a_q, a_s = ops.quant_act_1x128(lhs)
        b_q, b_s = ops.quant_w_128x128(rhs)
        del lhs, rhs
        torch.cuda.empty_cache()
        out = torch.empty((cfg.M, cfg.N), dtype=torch.bfloat16, device="cuda")
        fn = lambda: ops.gmm_fp8_fwd(a_q, a_s, b_q, b_s, gs, out=out)
    elif args.profile == "quant":
        # both quantisers on a slice of the headline operands: activations
        # [16384, 7168] (235 MB bf16) and 16 experts [16, 7168, 2048] (470 MB)
        gen = torch.Generator(device="cuda").manual_seed(args.seed)
        x = torch.randn((16384, 7168), device="cuda", generator=gen).to(torch.bfloat16)
        w = (torch.randn((16, 7168, 2048), device="cuda", generator=gen) * 0.02).to(torch.bfloat16)

        def fn():
            ops.quant_act_1x128(x)
            ops.quant_w_128x128(w)
    elif args.profile == "gmm_bwd":
        # dlhs and tgmm on a 16-expert slice of the headline workload (the
        # same routing, K and N; M = 4096 rows): about 0.9 GB resident
        cfg = configs.GMMConfig("gmm_moe_up_g16", G=16, M=4096, K=7168, N=2048, routing="zipf_topk")
        lhs, rhs, gs = configs.make_gmm_inputs(cfg, device="cuda", seed=args.seed)
        b_q, b_s = ops.quant_w_128x128(rhs)
        lq, ls = ops.quant_col_128x1(lhs)
        del lhs, rhs
        gen = torch.Generator(device="cuda").manual_seed(args.seed + 7)
        grad = torch.randn((cfg.M, cfg.N), device="cuda", generator=gen).to(torch.bfloat16)
        dq1, ds1 = ops.quant_act_1x128(grad)
        dq2, ds2 = ops.quant_col_128x1(grad)
        del grad
        torch.cuda.empty_cache()
        dlhs = torch.zeros((cfg.M, cfg.K), dtype=torch.bfloat16, device="cuda")
        drhs = torch.empty((cfg.G, cfg.K, cfg.N), dtype=torch.bfloat16, device="cuda")

        def fn():
            ops.gmm_fp8_dlhs(dq1, ds1, b_q, b_s, gs, out=dlhs)
            ops.tgmm_fp8(lq, ls, dq2, ds2, gs, out=drhs)
    elif args.profile == "gla_bwd":
        # the GLA backward (reverse scan + gradient kernel) on the GLA
        # workload: inputs, the states h, E and the gradients resident
        gcfg = configs.GLA_CONFIGS[args.gla_workload]
        inp = configs.make_gla_inputs(gcfg, device="cuda", seed=args.seed)
        h = ops.chunk_gla_fwd(inp["q"], inp["k"], inp["v"], inp["g_gamma"], 128 ** -0.5, 64,
                              g=inp["g"], h0=inp["h0"], output_states=True).h
        gen = torch.Generator(device="cuda").manual_seed(args.seed + 11)
        do = torch.randn(inp["v"].shape, generator=gen, device="cuda").to(torch.bfloat16)
        dq, dk, dv = (torch.empty_like(inp[n]) for n in ("q", "k", "v"))
        ws = torch.empty(ops.chunk_gla_bwd_workspace_bytes(gcfg.B, gcfg.T, gcfg.H),
                         dtype=torch.uint8, device="cuda")
        fn = lambda: ops.chunk_gla_bwd(inp["q"], inp["k"], inp["v"], do, h, inp["g_gamma"],
                                       128 ** -0.5, 64, g=inp["g"], dq=dq, dk=dk, dv=dv, workspace=ws)
    else:
        gcfg = configs.GLA_CONFIGS[args.gla_workload]
        inp = configs.make_gla_inputs(gcfg, device="cuda", seed=args.seed)
        fn = lambda: ops.chunk_gla_fwd(inp["q"], inp["k"], inp["v"], inp["g_gamma"], 128 ** -0.5,
                                       64, g=inp["g"], h0=inp["h0"], output_final_state=True)
    ms = timed(fn, args.steps, args.warmup, 1)
    status = ops.device_status()
    print(json.dumps({"profile": args.profile, "ms_per_step": ms, "status": status}), flush=True)
    return 0 if status == 0 else 1


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--workload", default=HEADLINE)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--skip-e2e", action="store_true")
    ap.add_argument("--skip-sharded", action="store_true",
                    help="N > 1: skip the strong-scaling rows (one workload split across ranks)")
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--cpu-rows", type=int, default=8192,
                    help="rows of the headline workload in one CPU-baseline step")
    ap.add_argument("--cpu-gla-tokens", type=int, default=4096)
    ap.add_argument("--profile", choices=["gmm", "gmm_bwd", "gla", "gla_bwd", "quant"], default=None,
                    help="run one kernel only, small footprint (for ncu captures)")
    ap.add_argument("--gla-workload", default=GLA_WORKLOAD)
    args = ap.parse_args(argv)
    if args.profile:
        return run_profile(args)
    if args.warmup < 3 and args.impl == "b200":
        print("note: fewer than 3 warm-up steps", file=sys.stderr)
    if args.impl == "reference":
        return run_reference(args)
    return run_b200(args)


if __name__ == "__main__":
    sys.exit(main())
