"""Benchmark of the B200 grouped FP8 matmul forward (headline) and the fused
chunked-GLA forward, one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Headline workload: gmm_dense_expert — G=8 experts, M=65536 rows (seeded
uniform-random group sizes, one expert empty), K=4096, N=14336, e4m3 operands
with 1x128 / 128x128 fp32 block scales, bf16 output (7.70 TFLOP per step, the
tensor-bound configuration).  Strong scaling: one instance of the workload is
split across the N ranks by expert group (contiguous 128-row cuts balanced by
rows; a cut may fall inside an expert) and one step = each rank's
grouped-matmul launch whose epilogue stores every finished output slice into
every rank's output buffer over NVLink (the output all-gather inside the
kernel), bracketed by two stream-ordered all-reduces of one int.  At N=1 the
step is the plain launch.  `value` = the instance's 2*M*K*N / the slowest
rank's step time.  Operands (0.74 GB e4m3) and the 1.9 GB output exceed L2,
so no flush.  The same instance with an NCCL all-gather after the matmul,
and plain copy-engine peer copies of each rank's output slab (the measured
link peak the gather is compared with), are timed beside it.

Secondary rows, one instance per rank (weak scaling): gmm_moe_up (G=128,
M=32768, K=7168, N=2048; HBM-bound) with its quantisers and the backward
kernels, gmm_small (G=8, M=2048, K=N=1024), and the GLA forward / backward
on gla_b8_t4096 and gla_b1_t32768; for N > 1 also gla_b1_t32768 split by
head (strong).

`e2e` times the public host-input op gmm_fp8_blockwise_host(lhs, rhs,
group_sizes) on the headline workload (each rank its shard of rows and
experts): H2D of the pinned activations, activation and weight quantisation,
the grouped matmul, D2H of the bf16 output rows, copies overlapping the
kernels.  The bf16 weights stay resident on the device (model parameters).

`--impl reference` times the CPU restatement of the same path (the reference
itself is JAX + tokamax on TPU, and JAX is not installed on this box) on the
host cores.
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
HEADLINE = "gmm_dense_expert"
MOE_WORKLOAD = "gmm_moe_up"
SMALL_WORKLOAD = "gmm_small"
GLA_WORKLOAD = "gla_b8_t4096"
GLA_LONG_WORKLOAD = "gla_b1_t32768"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# Back-to-back tcgen05.mma.kind::f8f6f4 128x256x32 from shared memory, one CTA
# per SM, no loads and no promotion (a microbenchmark, 69.4 ns per MMA at the
# burst clock): the rate the tensor pipe sustains for this instruction shape.
MMA_STREAM_TFLOPS = 4470.0


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
def cpu_gmm_step(sample_rows: int, seed: int = 0, workload: str = HEADLINE):
    """Builds a bounded sample of a grouped-matmul workload (its first
    `sample_rows` rows in group order, with the experts they belong to, full
    K and N) for the BLAS-backed CPU restatement.  Returns (step_fn,
    flops_per_step, description)."""
    import torch
    from glaucis_b200 import configs
    from oracle import cpu_fast
    cfg = configs.GMM_CONFIGS[workload]
    sizes = configs.group_sizes(cfg.routing, cfg.G, cfg.M, seed=seed, topk=cfg.topk, zipf=cfg.zipf)
    sel = []
    rows = 0
    for g in range(cfg.G):
        if sizes[g] > 0 and rows < sample_rows:
            take = min(int(sizes[g]), sample_rows - rows)
            sel.append(take)
            rows += take
    gen = torch.Generator().manual_seed(seed)
    lhs = torch.randn((rows, cfg.K), generator=gen).to(torch.bfloat16)
    rhs = (torch.randn((len(sel), cfg.K, cfg.N), generator=gen) * cfg.rhs_std).to(torch.bfloat16)

    def step():
        cpu_fast.gmm_fp8_blockwise(lhs, rhs, sel)

    flops = 2.0 * rows * cfg.K * cfg.N
    desc = (f"first {rows} of {cfg.M} rows of {workload} ({len(sel)} of {cfg.G} experts, "
            f"K={cfg.K}, N={cfg.N}): quantise lhs+rhs, dequantised fp32 GEMM per expert "
            f"(torch CPU, BLAS)")
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
    from glaucis_b200 import configs
    cfg = configs.GMM_CONFIGS[HEADLINE]
    # keep the whole arm to a couple of minutes whatever --steps/--warmup are
    rows = max(128, int(args.cpu_rows * min(1.0, 13.0 / (args.steps + args.warmup))))
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
        "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "e4m3 x e4m3 -> fp32 (dequantised fp32 GEMM on the host)",
        "data": "synthetic",
        "config": {"workload": HEADLINE, "G": cfg.G, "M": cfg.M, "K": cfg.K, "N": cfg.N,
                   "routing": configs.routing_desc(cfg), "sample": desc},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": cores, "kind": "port",
                         "sample": desc},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "gla": {"workload": GLA_WORKLOAD, "tokens_per_s": gtok / gdt, "sample": gdesc},
        "note": ("the reference path (JAX + qwix + tokamax Pallas on TPU) cannot run on this "
                 "box (JAX is not installed here or on the B200 box); this arm times the CPU "
                 "restatement of the same forward in oracle/"),
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# B200 arm
# ---------------------------------------------------------------------------
def gmm_bytes(cfg, g_nz: int, rows: int = None) -> float:
    """Algorithmic HBM bytes of one grouped-matmul launch on pre-quantised
    operands: e4m3 activations + their 1x128 scales, the e4m3 weights and
    128x128 scales of the non-empty experts, the group sizes, the bf16 output."""
    m = cfg.M if rows is None else rows
    return (m * cfg.K + 4 * m * cfg.K / 128 + g_nz * cfg.K * cfg.N
            + 4 * g_nz * (cfg.K / 128) * (cfg.N / 128) + 4 * cfg.G + 2 * m * cfg.N)


def headline_gmm(args, rank, world, local, peaks, peak_kind):
    """gmm_dense_expert split across the ranks by expert group, the output
    gathered on every rank by the matmul's own epilogue (strong scaling)."""
    import torch
    from glaucis_b200 import configs, ops, shard
    cfg = configs.GMM_CONFIGS[HEADLINE]
    fp8_peak = 2.0 * peaks["bf16_tflops"]
    lhs, rhs, gs = configs.make_gmm_inputs(cfg, device="cuda", seed=args.seed)  # same on every rank
    sizes = gs.cpu().numpy()
    parts = shard.gmm_partition(sizes, world)
    me = parts[rank]
    counts = [p.rows for p in parts]
    rows_total = sum(counts)
    flops_total = 2.0 * rows_total * cfg.K * cfg.N
    flops_me = 2.0 * me.rows * cfg.K * cfg.N
    g_nz_me = int((me.sizes > 0).sum())
    a_q, a_s = ops.quant_act_1x128(lhs[me.r0:me.r1].contiguous())
    b_q, b_s = ops.quant_w_128x128(rhs[me.g0:me.g1].contiguous())
    gs_l = torch.from_numpy(np.ascontiguousarray(me.sizes, np.int32)).to("cuda")
    sampler = ClockSampler(local) if rank == 0 else None
    res = {"rows_per_rank": counts, "groups_per_rank": [p.g1 - p.g0 for p in parts]}
    peers = None
    if world == 1:
        out = torch.empty((cfg.M, cfg.N), dtype=torch.bfloat16, device="cuda")

        def step():
            ops.gmm_fp8_fwd(a_q, a_s, b_q, b_s, gs_l, out=out)

        ms = timed(step, args.steps, args.warmup, world, sampler)
        compute_ms = ms
    else:
        out_l = torch.empty((me.rows, cfg.N), dtype=torch.bfloat16, device="cuda")
        compute_ms = timed(lambda: ops.gmm_fp8_fwd(a_q, a_s, b_q, b_s, gs_l, out=out_l),
                           max(5, args.steps // 2), args.warmup, world)
        peers = shard.PeerBuffers(rows_total, cfg.N)

        def step():
            shard.gmm_fp8_fwd_gathered(a_q, a_s, b_q, b_s, me, peers, group_sizes=gs_l)

        ms = timed(step, args.steps, args.warmup, world, sampler)
    if ops.device_status() != 0:
        raise SystemExit("device error word set after the headline timed region")
    res.update(ms=ms, compute_ms=compute_ms, flops_total=flops_total, flops_per_rank=flops_me,
               sampler=sampler)
    achieved = flops_me / (ms * 1e-3) / 1e12
    res["roofline"] = {
        "bound": "tensor", "achieved": achieved, "peak": fp8_peak, "unit": "TFLOP/s",
        "frac": achieved / fp8_peak, "traffic": ncu_traffic("gmm_fp8_fwd_kernel", HEADLINE),
        "peak_source": f"2 x {peak_kind} bf16_tflops (dense e4m3 rate)",
        "kernel": "gmm_fp8_fwd_kernel" if world == 1 else "gmm_fp8_fwd_kernel (scatter epilogue)",
        "per": "one GPU: its rows' 2*m*K*N over the step time" if world > 1 else "the launch",
        "mma_stream_frac": achieved / MMA_STREAM_TFLOPS,
        "mma_stream_tflops": MMA_STREAM_TFLOPS,
        "compute_only_frac": flops_me / (compute_ms * 1e-3) / 1e12 / fp8_peak,
        "algorithmic_flops_per_launch": flops_me,
        "algorithmic_bytes_per_launch": gmm_bytes(cfg, g_nz_me, me.rows),
    }
    if world > 1:
        # -------------------------------------------------- the gather's links
        row_bytes = 2 * cfg.N
        slab = me.rows * row_bytes
        pushed = slab * (world - 1)
        received = (rows_total - me.rows) * row_bytes
        same = None
        if rank == 0:
            fa, fs = ops.quant_act_1x128(lhs)
            fb, fbs = ops.quant_w_128x128(rhs)
            single = ops.gmm_fp8_fwd(fa, fs, fb, fbs, gs, out_dtype=torch.bfloat16)
            same = bool(torch.equal(single[:rows_total], peers.local))
            del fa, fs, fb, fbs, single
        views = [shard.tensor_at(ptr, (rows_total, cfg.N)) for ptr in peers.ptrs]
        own = peers.local[me.r0:me.r1]
        nxt = (rank + 1) % world
        others = [(rank + i) % world for i in range(1, world)]
        streams = {r: torch.cuda.Stream() for r in others}

        def copy_one():
            views[nxt][me.r0:me.r1].copy_(own, non_blocking=True)

        def copy_all():
            cur = torch.cuda.current_stream()
            for r in others:
                streams[r].wait_stream(cur)
                with torch.cuda.stream(streams[r]):
                    views[r][me.r0:me.r1].copy_(own, non_blocking=True)
            for r in others:
                cur.wait_stream(streams[r])

        one_ms = timed(copy_one, 5, 2, world)
        all_ms = timed(copy_all, 5, 2, world)
        out_full = torch.empty((rows_total, cfg.N), dtype=torch.bfloat16, device="cuda")

        def nccl_step():
            ops.gmm_fp8_fwd(a_q, a_s, b_q, b_s, gs_l, out=out_l)
            shard.all_gather_rows(out_l, counts, out_full)

        nccl_ms = timed(nccl_step, max(5, args.steps // 2), 3, world)
        if ops.device_status() != 0:
            raise SystemExit("device error word set after the gather rows")
        peer_all_gbs = pushed / (all_ms * 1e-3) / 1e9
        res["gather"] = {
            "in_kernel": "each rank's matmul epilogue TMA-stores every finished 32x128 output "
                         "slice into every rank's IPC-shared buffer (own + peers over NVLink)",
            "matches_single_gpu": same,
            "bytes_pushed_per_rank": pushed, "bytes_received_per_rank": received,
            "nvlink_gbs_per_rank": pushed / (ms * 1e-3) / 1e9,
            "peer_copy_one_gbs": slab / (one_ms * 1e-3) / 1e9,
            "peer_copy_all_gbs": peer_all_gbs,
            "frac_of_peer_copy_all": (pushed / (ms * 1e-3) / 1e9) / peer_all_gbs,
            "link_bound_ms": max(compute_ms, all_ms),
            "peer_copy": "copy engines, cudaMemcpyAsync of this rank's output slab into the next "
                         "rank's buffer (one) and into every peer's buffer at once, one stream "
                         "per peer (all); max over ranks",
            "nccl_allgather_after_matmul_ms": nccl_ms,
            "nccl_tflops": flops_total / (nccl_ms * 1e-3) / 1e12,
        }
        del views, own, out_full, out_l
        peers.close()
    # ------------------------------------------------------------------ e2e
    if not args.skip_e2e:
        lhs_h = lhs[me.r0:me.r1].cpu().pin_memory()
        rhs_l = rhs[me.g0:me.g1].contiguous()
        gs_h = torch.from_numpy(np.ascontiguousarray(me.sizes, np.int32)).pin_memory()
        out_h = torch.empty((me.rows, cfg.N), dtype=torch.bfloat16).pin_memory()
        n_chunks = len(ops._plan_chunks(me.sizes, 16)[0])

        def e2e_step():
            # public host-input op: pinned activations and group sizes in,
            # pinned bf16 output back; copies overlap the kernels
            ops.gmm_fp8_blockwise_host(lhs_h, rhs_l, gs_h, out=out_h, out_dtype=torch.bfloat16)

        e_steps = max(1, min(args.steps, args.e2e_steps))
        e_ms = timed(e2e_step, e_steps, min(args.warmup, 2), world)

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

        lhs_d = torch.empty(lhs_h.shape, dtype=lhs_h.dtype, device="cuda")
        h2d_ms = copy_ms(lhs_d, lhs_h)
        out_d = torch.empty(out_h.shape, dtype=torch.bfloat16, device="cuda")
        d2h_ms = copy_ms(out_h, out_d)
        res["e2e"] = {
            "value": flops_total / (e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
            "h2d_bytes_per_step": lhs_h.numel() * 2 + n_chunks * (me.g1 - me.g0) * 4,
            "d2h_bytes_per_step": out_h.numel() * 2, "ms_per_step": e_ms,
            "link": {"h2d_gbs": lhs_h.numel() * 2 / (h2d_ms * 1e-3) / 1e9,
                     "d2h_gbs": out_h.numel() * 2 / (d2h_ms * 1e-3) / 1e9,
                     "h2d_ms": h2d_ms, "d2h_ms": d2h_ms,
                     "note": "one plain pinned copy each way of this rank's activations / output"},
            "path": "gmm_fp8_blockwise_host(lhs, rhs, group_sizes) on each rank's shard: H2D lhs "
                    "rows in up to 16 chunks overlapping quantise lhs (per chunk) + rhs and the "
                    "grouped matmul, D2H of the bf16 output rows per chunk; the ranks' outputs "
                    "together are the whole [M, N] in host memory",
            "bytes_note": "per rank (each rank copies its own shard)"}
        del lhs_h, rhs_l, out_h, lhs_d, out_d
    del lhs, rhs, a_q, a_s, b_q, b_s
    torch.cuda.empty_cache()
    return res


def rw_rates(nbytes: int = 2 << 30, reps: int = 10):
    """Write-only and read-only HBM rates of this GPU (GB/s), measured with
    torch's fill and fp32 sum over a 2 GiB bf16 buffer (larger than L2),
    median of `reps` CUDA-event timings.  Writes alone run well below reads
    alone on B200 (about 3.9 vs 6.1 TB/s), which bounds the write-heavy
    backward kernels."""
    import statistics
    import torch
    buf = torch.empty(nbytes // 2, dtype=torch.bfloat16, device="cuda")

    def med(fn):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(reps):
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            b.synchronize()
            ts.append(a.elapsed_time(b))
        return statistics.median(ts)

    w = nbytes / (med(lambda: buf.fill_(1.0)) * 1e-3) / 1e9
    r = nbytes / (med(lambda: torch.sum(buf, dtype=torch.float32)) * 1e-3) / 1e9
    del buf
    return {"write_only_gbs": w, "read_only_gbs": r,
            "how": "torch fill_ / fp32 sum over a 2 GiB bf16 buffer, median of 10 CUDA-event timings"}


def secondary_gmm(args, workload, rank, world, peaks, peak_kind, with_extras: bool):
    """One instance of a grouped-matmul workload per rank (weak scaling), with
    its HBM / tensor roofline; with_extras adds the quantiser and backward rows."""
    import torch
    from glaucis_b200 import configs, ops
    fp8_peak = 2.0 * peaks["bf16_tflops"]
    cfg = configs.GMM_CONFIGS[workload]
    lhs, rhs, gs = configs.make_gmm_inputs(cfg, device="cuda", seed=args.seed + rank)
    a_q, a_s = ops.quant_act_1x128(lhs)
    b_q, b_s = ops.quant_w_128x128(rhs)
    out = torch.empty((cfg.M, cfg.N), dtype=torch.bfloat16, device="cuda")
    sizes = gs.cpu().numpy()
    g_nz = int((sizes > 0).sum())
    flops = 2.0 * float(sizes.sum()) * cfg.K * cfg.N
    alg_bytes = gmm_bytes(cfg, g_nz)
    ms = timed(lambda: ops.gmm_fp8_fwd(a_q, a_s, b_q, b_s, gs, out=out), args.steps, args.warmup,
               world)
    if ops.device_status() != 0:
        raise SystemExit(f"device error word set after the {workload} timed region")
    ai = flops / alg_bytes
    ridge = fp8_peak * 1e12 / (peaks["hbm_gbs"] * 1e9)
    gbs = alg_bytes / (ms * 1e-3) / 1e9
    tfl = flops / (ms * 1e-3) / 1e12
    blk = {"workload": workload, "G": cfg.G, "M": cfg.M, "K": cfg.K, "N": cfg.N,
           "routing": configs.routing_desc(cfg), "empty_groups": cfg.G - g_nz,
           "ms_per_step": ms, "tflops": world * tfl,
           "roofline": {"bound": "hbm" if ai < ridge else "tensor",
                        "achieved": gbs if ai < ridge else tfl,
                        "unit": "GB/s" if ai < ridge else "TFLOP/s",
                        "peak": peaks["hbm_gbs"] if ai < ridge else fp8_peak,
                        "frac": gbs / peaks["hbm_gbs"] if ai < ridge else tfl / fp8_peak,
                        "fp8_tensor_frac": tfl / fp8_peak, "mma_stream_frac": tfl / MMA_STREAM_TFLOPS,
                        "traffic": ncu_traffic("gmm_fp8_fwd_kernel", workload),
                        "algorithmic_bytes_per_launch": alg_bytes,
                        "algorithmic_flops_per_launch": flops, "kernel": "gmm_fp8_fwd_kernel",
                        "peak_source": f"{peak_kind} hbm_gbs / 2 x {peak_kind} bf16_tflops"}}
    if workload == SMALL_WORKLOAD:
        # A problem this small is bound by the launch path of the eager call
        # (Python, tensor-map encoding, launch), so the same call is also
        # captured once in a CUDA graph and replayed: the row's device rate.
        fn = lambda: ops.gmm_fp8_fwd(a_q, a_s, b_q, b_s, gs, out=out)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                fn()
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        g_ms = timed(graph.replay, args.steps, args.warmup, world)
        blk["graph"] = {"ms_per_step": g_ms, "tflops": world * flops / (g_ms * 1e-3) / 1e12,
                        "how": "the same gmm_fp8_fwd call captured in a torch.cuda.CUDAGraph and "
                               "replayed; the eager ms_per_step includes the launch path"}
        del graph
    if not with_extras:
        del lhs, rhs, a_q, a_s, b_q, b_s, out
        torch.cuda.empty_cache()
        return blk
    # quantiser rows (separately timed kernels of the same forward); outputs
    # preallocated: the timed region holds the quantiser kernels only
    qa_o, sa_o = torch.empty_like(a_q), torch.empty_like(a_s)
    qw_o, sw_o = torch.empty_like(b_q), torch.empty_like(b_s)
    q_act_ms = timed(lambda: ops.quant_act_1x128(lhs, qa_o, sa_o), max(5, args.steps // 2), 3, world)
    q_w_ms = timed(lambda: ops.quant_w_128x128(rhs, qw_o, sw_o), max(5, args.steps // 10), 3, world)
    del qa_o, sa_o, qw_o, sw_o
    q_act_bytes = lhs.numel() * 3 + lhs.numel() // 128 * 4
    q_w_bytes = rhs.numel() * 3 + rhs.numel() // (128 * 128) * 4
    blk["quantisers"] = {
        name: {"ms": ms_, "achieved_gbs": by / (ms_ * 1e-3) / 1e9,
               "frac": by / (ms_ * 1e-3) / 1e9 / peaks["hbm_gbs"], "algorithmic_bytes": by}
        for name, ms_, by in (("quant_act_1x128", q_act_ms, q_act_bytes),
                              ("quant_w_128x128", q_w_ms, q_w_bytes))}
    # backward: dlhs (grouped kernel, weight transposed) and drhs (tgmm) with a
    # synthetic output gradient, quantised inputs resident
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

    # bytes written by each kernel (the rest of its algorithmic bytes are reads)
    dl_w = 2 * cfg.M * cfg.K
    tg_w = 2 * cfg.G * cfg.K * cfg.N
    qc_w = grad.numel() + grad.numel() // 128 * 4
    rw = rw_rates()

    def row(ms_, by, fl, wr):
        g = by / (ms_ * 1e-3) / 1e9
        r = {"ms": ms_, "achieved_gbs": g, "hbm_frac": g / peaks["hbm_gbs"], "algorithmic_bytes": by,
             "written_bytes": wr}
        # floor of a kernel that reads R and writes W bytes: the slowest of the
        # read-only, write-only and copy rates measured on this GPU
        floor_ms = max((by - wr) / rw["read_only_gbs"], wr / rw["write_only_gbs"],
                       by / peaks["hbm_gbs"]) / 1e6
        r["rw_floor_ms"] = floor_ms
        r["frac_of_rw_floor"] = floor_ms / ms_
        if fl:
            r["tflops"] = world * fl / (ms_ * 1e-3) / 1e12
            r["fp8_tensor_frac"] = fl / (ms_ * 1e-3) / 1e12 / fp8_peak
        return r

    blk["bwd"] = {"dlhs": row(dl_ms, dl_bytes, flops, dl_w), "tgmm": row(tg_ms, tg_bytes, flops, tg_w),
                  "quant_col_128x1": row(qc_ms, qc_bytes, 0.0, qc_w),
                  "rw_rates": rw,
                  "note": "dlhs = gl_gmm_fp8_dlhs (grouped kernel, K-major weight); tgmm writes "
                          "drhs [G, K, N] bf16 for every group (empty ones as zeros), so it is "
                          "bound by the write-only rate"}
    del grad, dq1, ds1, dq2, ds2, lq, ls, dlhs, drhs, lhs, rhs, a_q, a_s, b_q, b_s, out
    torch.cuda.empty_cache()
    return blk


def gla_block(args, workload, rank, world, peaks, peak_kind, local=0):
    import torch
    from glaucis_b200 import configs, ops
    gcfg = configs.GLA_CONFIGS[workload]
    inp = configs.make_gla_inputs(gcfg, device="cuda", seed=args.seed + rank)
    go = torch.empty_like(inp["v"])
    ght = torch.empty((gcfg.B, gcfg.H, 128, 128), device="cuda")

    def gla_step():
        ops.chunk_gla_fwd(inp["q"], inp["k"], inp["v"], inp["g_gamma"], 128 ** -0.5, 64,
                          g=inp["g"], h0=inp["h0"], output_final_state=True, o=go, ht=ght)

    def gla_bf16_step():
        ops.chunk_gla_fwd(inp["q"], inp["k"], inp["v"], inp["g_gamma"], 128 ** -0.5, 64,
                          g=inp["g"], h0=inp["h0"], output_final_state=True, o=go, ht=ght,
                          exact_intra=False)

    # The GLA kernels are latency-bound, so their time follows the SM clock:
    # a longer warm-up lets the clock settle after the power-capped matmul
    # rows, and the clock is recorded beside each timing.
    gwarm = max(args.warmup, 100)
    cs_ex = ClockSampler(local) if rank == 0 else None
    gla_ms = timed(gla_step, args.steps, gwarm, world, cs_ex)
    cs_bf = ClockSampler(local) if rank == 0 else None
    bf_ms = timed(gla_bf16_step, args.steps, gwarm, world, cs_bf)
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
                        "traffic": ncu_traffic("chunk_gla_fwd_kernel", workload)},
           "precision": "tril(A) enters the intra-chunk product as a bf16 hi + lo pair (~2^-17 "
                        "relative): the fp32 A of the template's output kernel",
           "clocks": cs_ex.summary() if cs_ex else None,
           "bf16_intra": {"ms_per_step": bf_ms,
                          "clocks": cs_bf.summary() if cs_bf else None,
                          "tokens_per_s": world * gcfg.B * gcfg.T / (bf_ms * 1e-3),
                          "hbm_frac": gla_bytes / (bf_ms * 1e-3) / 1e9 / peaks["hbm_gbs"],
                          "precision": "tril(A) rounded to bf16 once (the jnp oracle's einsum at "
                                       "TPU default precision), exact_intra=False"}}
    # backward: the training forward (o, ht and the per-chunk states h) and the
    # backward (reverse state-gradient scan + chunk-parallel dq/dk/dv kernel)
    # on a synthetic output gradient, buffers resident
    gh = torch.empty((gcfg.B, gcfg.T // 64, gcfg.H, 128, 128), dtype=torch.bfloat16, device="cuda")

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
        "algorithmic_bytes_per_step": bw_bytes, "fused_minimum_bytes": bw_min,
        "fused_minimum_frac": bw_min / (bw_ms * 1e-3) / 1e9 / peaks["hbm_gbs"],
        "fwd_with_states_ms": fs_ms,
        "kernels": "chunk_gla_fwd_kernel in reverse-scan mode (+ its state-only pre-pass and "
                   "fold when the sequence is split), then chunk_gla_bwd_kernel",
    }
    del inp, go, ght, gh, gdo, dq, dk, dv, gws
    torch.cuda.empty_cache()
    return blk


def run_b200(args):
    import torch
    from glaucis_b200 import configs
    rank, world, local = dist_setup(args.gpus)
    peaks, peak_kind = load_peaks()
    cfg = configs.GMM_CONFIGS[HEADLINE]

    head = headline_gmm(args, rank, world, local, peaks, peak_kind)
    ms = head["ms"]
    value = head["flops_total"] / (ms * 1e-3) / 1e12
    moe = secondary_gmm(args, MOE_WORKLOAD, rank, world, peaks, peak_kind, with_extras=True)
    small = secondary_gmm(args, SMALL_WORKLOAD, rank, world, peaks, peak_kind, with_extras=False)
    gla = gla_block(args, GLA_WORKLOAD, rank, world, peaks, peak_kind, local)
    gla_long = gla_block(args, GLA_LONG_WORKLOAD, rank, world, peaks, peak_kind, local)

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
        sampler = head.pop("sampler")
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "e4m3 x e4m3 -> fp32 acc, bf16 out", "data": "synthetic",
            "config": {"workload": HEADLINE, "G": cfg.G, "M": cfg.M, "K": cfg.K, "N": cfg.N,
                       "routing": configs.routing_desc(cfg),
                       "parallelism": ("one GPU" if world == 1 else
                                       f"expert-group shards x{world}, output all-gathered on "
                                       "every rank inside the matmul epilogue"),
                       "rows_per_rank": head["rows_per_rank"],
                       "l2": "operands (0.74 GB e4m3) and output (1.9 GB) exceed L2; no flush"},
            "roofline": head["roofline"],
            "compute_only_ms": head["compute_ms"],
            "gather": head.get("gather"),
            "cpu_baseline": cpu,
            "e2e": head.get("e2e"),
            "gpu_launches": args.steps,
            "clocks": sampler.summary() if sampler else None,
            "moe_up": moe,
            "small": small,
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
    """Strong scaling of gla_b1_t32768 across the ranks (N > 1 only), split by
    head with an all-gather of the head blocks.  Compute-only and
    gather-inclusive device times (max over ranks); rank 0 checks the
    gathered result against the single-GPU one (to rounding: the sequence
    split differs with the head count).  The grouped matmul's strong scaling
    is the headline itself."""
    import torch
    from glaucis_b200 import configs, ops, shard
    res = {}
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
    # the same gather inside the forward: every chunk's O is TMA-stored into
    # block `rank` of every rank's IPC-shared buffer (shard.gla_fwd_gathered)
    peers = shard.PeerBuffers(world, width)

    def gla_scattered():
        shard.gla_fwd_gathered(q, k, v, g, h0, 128 ** -0.5, peers, width, ht=ht_l)

    k2 = timed(gla_scattered, steps, warmup, world)
    err = err_k = None
    if rank == 0:
        full = ops.chunk_gla_fwd(inp["q"], inp["k"], inp["v"], None, 128 ** -0.5, 64, g=inp["g"],
                                 h0=inp["h0"], output_final_state=True).o
        worst = worst_k = 0.0
        for r, hrange in enumerate(shard.gla_head_partition(gcfg.H, world)):
            n_r = gcfg.B * gcfg.T * len(hrange) * gcfg.V
            want = full[:, :, hrange.start:hrange.stop].float()
            got = stage[r, :n_r].view(gcfg.B, gcfg.T, len(hrange), gcfg.V).float()
            worst = max(worst, float((got - want).norm() / want.norm()))
            got = peers.local[r, :n_r].view(gcfg.B, gcfg.T, len(hrange), gcfg.V).float()
            worst_k = max(worst_k, float((got - want).norm() / want.norm()))
        err, err_k = worst, worst_k
        del full
    peers.close()
    if ops.device_status() != 0:
        raise SystemExit("device error word set after the sharded GLA")
    res["gla"] = {"workload": "gla_b1_t32768", "split": "heads", "heads_per_rank": heads,
                  "compute_ms": c2, "with_gather_ms": g2,
                  "tokens_per_s_compute": gcfg.B * gcfg.T / (c2 * 1e-3),
                  "tokens_per_s_with_gather": gcfg.B * gcfg.T / (g2 * 1e-3),
                  "gathered_layout": "[world, B, T, H/world, V] head blocks",
                  "rel_err_vs_single_gpu": err,
                  "with_gather_in_kernel_ms": k2,
                  "tokens_per_s_with_gather_in_kernel": gcfg.B * gcfg.T / (k2 * 1e-3),
                  "in_kernel_rel_err_vs_single_gpu": err_k,
                  "gather": "with_gather: NCCL all-gather after the forward; in_kernel: the forward "
                            "TMA-stores every chunk's O into every rank's IPC-shared buffer",
                  "scaling": "strong"}
    del inp, q, k, v, g, h0, o_l, ht_l, stage
    torch.cuda.empty_cache()
    return res


def run_profile(args):
    """Small-footprint run of one kernel for ncu captures: the GMM on the
    --workload grouped-matmul workload (default the headline) with the bf16
    operands freed after quantisation, the two quantisers on a slice of
    gmm_moe_up's operands, the grouped-matmul backward on a 16-expert slice
    of gmm_moe_up, or the GLA forward / backward on its workload."""
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
        # both quantisers on a slice of gmm_moe_up's operands: activations
        # [16384, 7168] (235 MB bf16) and 16 experts [16, 7168, 2048] (470 MB)
        gen = torch.Generator(device="cuda").manual_seed(args.seed)
        x = torch.randn((16384, 7168), device="cuda", generator=gen).to(torch.bfloat16)
        w = (torch.randn((16, 7168, 2048), device="cuda", generator=gen) * 0.02).to(torch.bfloat16)

        def fn():
            ops.quant_act_1x128(x)
            ops.quant_w_128x128(w)
    elif args.profile == "gmm_bwd":
        # dlhs and tgmm on a 16-expert slice of gmm_moe_up (the
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
        if args.gla_heads:
            # heads 0 .. gla_heads-1 only: one rank's share of the head split
            # (gla_b1_t32768 at N=8: 4 heads, a 38-segment sequence split)
            hh = args.gla_heads
            inp = {n: (None if t is None else
                       t[:, :hh].contiguous() if n == "h0" else
                       t[:hh].contiguous() if n == "g_gamma" else
                       t[:, :, :hh].contiguous())
                   for n, t in inp.items()}
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
    ap.add_argument("--cpu-rows", type=int, default=4096,
                    help="rows of the headline workload in one CPU-baseline step")
    ap.add_argument("--cpu-gla-tokens", type=int, default=4096)
    ap.add_argument("--profile", choices=["gmm", "gmm_bwd", "gla", "gla_bwd", "quant"], default=None,
                    help="run one kernel only, small footprint (for ncu captures)")
    ap.add_argument("--gla-workload", default=GLA_WORKLOAD)
    ap.add_argument("--gla-heads", type=int, default=0,
                    help="--profile gla: run only the first H heads of the GLA workload")
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
