"""Benchmark of the llm_kernels inference op set on B200 (one JSON line on stdout).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--quick]

Headline workload (the metric's first clause):
flash-attention forward, causal, bf16, B=4 H=32 N=4096 D=128, TFLOP/s with causal FLOPs
counted as half of dense (4*B*H*N^2*D / 2).  One step = one flash_attn_forward call over
one batch.  Inputs are 384 MiB per step (larger than the 126 MB L2), so no L2 flush is
needed between steps.  The other two clauses of the metric (int8 GEMM+dequant TOPS at
4096^3 and RMSNorm+Linear ms at 512x4096->4096) and the rest of the op set are measured in
the same run and reported under "ops".

Multi-GPU (launched by torchrun, one process per GPU): the batch is sharded — every rank
runs its own B=4 slice of a global batch of 4*N (weak scaling), no collective on the data
path; the timed region is bracketed by barriers and the max over ranks is reported.

--impl reference times the reference's CPU path on the host cores: torch SDPA in fp32 on
the CPU (the reference's FA test oracle; its FA itself is GPU-only Triton), on a bounded
sample of the same workload per step; rank 0 only.
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "flash-attn-from-scratch_b200"))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "FA fwd TFLOP/s (causal bf16 N=4096 D=128); int8 GEMM+dequant TOPS; RMSNorm+Lin ms"
B, H, N, D = 4, 32, 4096, 128
FLOPS_CAUSAL = 4.0 * B * H * N * N * D / 2  # causal counted as half of dense


CONFIG = {
    "workload": "flash-attention forward causal bf16, B=4 H=32 N=4096 D=128 per GPU "
                "(global batch 4*n_gpus, batch-sharded)",
    "B_per_gpu": B, "H": H, "N": N, "D": D, "causal": True,
    "flops_per_step_per_gpu": FLOPS_CAUSAL,
    "l2": "inputs larger than L2 (384 MiB per step), no flush",
}


def fa_flops(b, h, n, d, causal):
    return 4.0 * b * h * n * n * d * (0.5 if causal else 1.0)


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def profile_traffic():
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary."""
    try:
        with open(os.path.join(ROOT, "profiles", "roofline_traffic.json")) as f:
            return json.load(f)
    except Exception:
        return {}


# ---------------------------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def wait_first(self, timeout_s: float = 10.0):
        """Blocks until nvidia-smi has printed its first sample (its start-up can take seconds
        on a fresh machine) or `timeout_s` has passed, so the timed window that follows is
        sampled from its start."""
        t0 = time.time()
        while self.proc is not None and not self.lines and time.time() - t0 < timeout_s:
            if self.proc.poll() is not None:
                break
            time.sleep(0.01)

    def stop(self, window=None):
        """Summary of the samples received inside `window` = (t_start, t_end) host seconds."""
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.1)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, smax, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ts, ln in self.lines:
            if window is not None and not (window[0] <= ts <= window[1] + 0.05):
                continue
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(nm)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(smax) if smax else None,
            "power_w_max": max(power) if power else None,
            "samples": len(sm),
            "reasons": sorted(reasons),
        }


# ---------------------------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------------------------
def dist_setup(gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------------------------
# device timing helpers
# ---------------------------------------------------------------------------------------------
def time_loop(fn, steps: int, warmup: int, world: int) -> float:
    """Total device ms of `steps` back-to-back calls (events on the current stream), max over ranks."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record(s)
    for _ in range(steps):
        fn()
    b.record(s)
    torch.cuda.synchronize()
    barrier(world)
    return max_over_ranks(a.elapsed_time(b), world)


def time_each_flushed(fn, reps: int, warmup: int, flush: torch.Tensor) -> float:
    """Median device ms of one call, with L2 flushed (a 256 MiB write) before every call."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    ts = []
    for _ in range(reps):
        flush.zero_()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(s)
        fn()
        b.record(s)
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    return statistics.median(ts)


# ---------------------------------------------------------------------------------------------
# CPU baselines (the oracle port of the reference's CPU path)
# ---------------------------------------------------------------------------------------------
def cpu_fa_sample(heads: int, reps: int):
    import oracle

    g = torch.Generator().manual_seed(1)
    q = torch.randn(1, heads, N, D, generator=g)
    k = torch.randn(1, heads, N, D, generator=g)
    v = torch.randn(1, heads, N, D, generator=g)
    oracle.attention_fp32(q[:, :1, :512], k[:, :1, :512], v[:, :1, :512], True)  # warm
    t0 = time.perf_counter()
    for _ in range(reps):
        torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True)
    dt = (time.perf_counter() - t0) / reps
    return fa_flops(1, heads, N, D, True) / dt / 1e12, dt


def cpu_baselines():
    """The reference's CPU path timed on this host: returns dict of op -> baseline."""
    import oracle

    threads = torch.get_num_threads()
    out = {}
    tf, dt = cpu_fa_sample(heads=32, reps=2)
    out["flash_attn_causal"] = {"value": tf, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                                "sample": f"torch SDPA fp32 causal, B=1 H=32 N=4096 D=128 (1/4 of the batch), "
                                          f"{dt * 1e3:.0f} ms/call"}
    g = torch.Generator().manual_seed(0)
    x = torch.randn(512, 4096, generator=g)
    wn = 1 + 0.1 * torch.randn(4096, generator=g)
    wl = torch.randn(4096, 4096, generator=g) / 64
    oracle.rmsnorm_linear_ref(x, wn, wl)
    t0 = time.perf_counter()
    for _ in range(5):
        oracle.rmsnorm_linear_ref(x, wn, wl)
    dt = (time.perf_counter() - t0) / 5
    out["rmsnorm_linear"] = {"value": dt * 1e3, "unit": "ms", "cores": threads, "kind": "port",
                             "sample": "fp32 RMSNorm+Linear 512x4096->4096 (the full config-1 problem), 5 calls"}
    a = torch.randint(-127, 128, (512, 4096), dtype=torch.int8).numpy()
    bm = torch.randint(-127, 128, (4096, 4096), dtype=torch.int8).numpy()
    t0 = time.perf_counter()
    acc = oracle.int8_gemm_i32(a, bm, "nk", threads=threads)
    oracle.dequant_f16(acc, torch.full((512,), 1e-3).numpy(), torch.full((4096,), 1e-3).numpy())
    dt = time.perf_counter() - t0
    out["int8_gemm_dequant"] = {"value": 2 * 512 * 4096 * 4096 / dt / 1e12, "unit": "TOPS", "cores": threads,
                                "kind": "port",
                                "sample": "int32 GEMM + dequant, M=512 rows of the 4096^3 problem (1/8), C restatement"}
    return out


# ---------------------------------------------------------------------------------------------
# the reference arm
# ---------------------------------------------------------------------------------------------
def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = torch.get_num_threads()
    heads = 2 if args.quick else 8  # per step: B=1, `heads` heads of the B4 H32 N4096 D128 problem
    import oracle

    g = torch.Generator().manual_seed(1)
    q = torch.randn(1, heads, N, D, generator=g)
    k = torch.randn(1, heads, N, D, generator=g)
    v = torch.randn(1, heads, N, D, generator=g)
    fn = lambda: torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True)  # noqa: E731
    for _ in range(args.warmup):
        fn()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        fn()
    dt = time.perf_counter() - t0
    flops = fa_flops(1, heads, N, D, True) * args.steps
    val = flops / dt / 1e12
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": val,
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": dt * 1e3 / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded N(0,1) q/k/v)",
        "config": CONFIG,
        "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": f"B=1 H={heads} of the workload per step, torch SDPA fp32 causal"},
        "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------------------
def run_ours(args):
    import llm_kernels

    world, rank, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    peaks, peaks_kind = measured_peaks()

    # ---- headline: causal FA config 2 on every rank (its own batch shard) ----
    g = torch.Generator().manual_seed(1 + rank)
    q = torch.randn(B, H, N, D, generator=g).to(torch.bfloat16).to(dev)
    k = torch.randn(B, H, N, D, generator=g).to(torch.bfloat16).to(dev)
    v = torch.randn(B, H, N, D, generator=g).to(torch.bfloat16).to(dev)
    step = lambda: llm_kernels.flash_attn_forward(q, k, v, causal=True)  # noqa: E731

    clocks = ClockSampler(local)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    clocks.start()
    clocks.wait_first()  # only samples inside the timed window count
    time.sleep(0.05)
    t_start = time.time()
    total_ms = time_loop(step, args.steps, 0, world)
    clk = clocks.stop(window=(t_start, time.time()))
    ms = total_ms / args.steps
    value = FLOPS_CAUSAL * world / (ms * 1e-3) / 1e12  # whole job: all ranks' work / max time
    launches = args.steps  # one fa_fwd_kernel launch per step

    # ---- end to end through the public API, host buffers (rank-local) ----
    # Every step uploads its q, k, v from pinned host memory, runs flash_attn_forward and reads
    # its output back into pinned host memory, all inside the timed region.  Steps alternate
    # between two device buffer sets and the copies run on their own streams, so step i's
    # upload overlaps step i-1's kernel and step i-2's download (PCIe moves both directions at
    # once): how a serving loop would drive the op.
    qh = q.cpu().pin_memory()
    kh = k.cpu().pin_memory()
    vh = v.cpu().pin_memory()
    cur = torch.cuda.current_stream()
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
    sets = [(torch.empty_like(q), torch.empty_like(k), torch.empty_like(v), torch.empty_like(q)) for _ in range(2)]
    ohs = [torch.empty_like(qh).pin_memory() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]  # set s may be refilled: its output has been read back
    for ev in free:
        ev.record(cur)
    step_no = [0]

    def e2e_step():
        s_ = step_no[0] % 2
        step_no[0] += 1
        qd, kd, vd, od = sets[s_]
        h2d.wait_event(free[s_])
        with torch.cuda.stream(h2d):
            qd.copy_(qh, non_blocking=True)
            kd.copy_(kh, non_blocking=True)
            vd.copy_(vh, non_blocking=True)
        up = torch.cuda.Event()
        up.record(h2d)
        cur.wait_event(up)
        llm_kernels.flash_attn_forward(qd, kd, vd, causal=True, out=od)
        done = torch.cuda.Event()
        done.record(cur)
        d2h.wait_event(done)
        with torch.cuda.stream(d2h):
            ohs[s_].copy_(od, non_blocking=True)
        free[s_].record(d2h)

    def e2e_time(steps_, warmup_):
        for _ in range(warmup_):
            e2e_step()
        torch.cuda.synchronize()
        barrier(world)
        torch.cuda.synchronize()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(cur)
        h2d.wait_stream(cur)  # the first timed upload starts after the start event
        for _ in range(steps_):
            e2e_step()
        cur.wait_stream(d2h)  # the end event follows the last download
        b.record(cur)
        torch.cuda.synchronize()
        barrier(world)
        return max_over_ranks(a.elapsed_time(b), world)

    e2e_steps = max(3, args.steps // 4)
    e2e_ms = e2e_time(e2e_steps, 2) / e2e_steps
    e2e_val = FLOPS_CAUSAL * world / (e2e_ms * 1e-3) / 1e12
    nbytes = q.numel() * q.element_size()

    torch.cuda.synchronize()
    del qh, kh, vh, sets, ohs
    decoder = decoder_layer_measure(args, llm_kernels, world, rank, dev)
    sharded = sharded_gather_measure(args, llm_kernels, world, rank, dev) if world > 1 else None

    ops = {}
    cpu = None
    if rank == 0:
        # The metric's other clauses (single-GPU ops) are measured in the 1-GPU run only: at
        # N > 1 the other ranks would idle at a barrier meanwhile.
        if world == 1:
            ops = secondary_ops(args, llm_kernels, peaks)
            cpu = cpu_baselines()
        ops["decoder_layer_config5"] = decoder
        if sharded is not None:
            ops["column_sharded_int8_linear"] = sharded

    traffic = profile_traffic().get("flash_attn_causal_bf16_B4_H32_N4096_D128")
    # Denominator: the measured cuBLAS bf16 burst peak.  The timed region is a loop of this
    # one kernel, i.e. a kernel timed alone, whatever its length; the fraction of the
    # sustained (power-capped) figure is reported beside it for long regions.
    achieved = FLOPS_CAUSAL / (ms * 1e-3) / 1e12
    burst = float(peaks["bf16_tflops"])
    sustained = float(peaks.get("bf16_tflops_sustained", burst))
    peak = burst
    line = {
        "metric": METRIC,
        "value": value,
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) q/k/v; no dataset)",
        "config": CONFIG,
        "roofline": {
            "bound": "tensor",
            "achieved": achieved,
            "peak": peak,
            "unit": "TFLOP/s",
            "frac": achieved / peak,
            "peak_kind": f"{peaks_kind} bf16 burst (cuBLAS); timed region {total_ms:.0f} ms of back-to-back launches",
            "frac_of_sustained": achieved / sustained,
            "kernel": "lk::fa::fa_fwd_kernel<128, bf16>",
            "traffic": traffic.get("dram_bytes_per_launch") if traffic else None,
            "algorithmic_bytes": 4 * nbytes,
        },
        "e2e": {"value": e2e_val, "unit": "TFLOP/s", "h2d_bytes_per_step": 3 * nbytes,
                "d2h_bytes_per_step": nbytes, "steps": e2e_steps,
                "overlap": "two device buffer sets; uploads and downloads on their own streams overlap the "
                           "neighbouring steps' kernels"},
        "gpu_launches": launches,
        "clocks": clk,
        "ops": ops,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu["flash_attn_causal"]
        line["cpu_baselines"] = cpu
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


def sharded_gather_measure(args, llm_kernels, world, rank, dev):
    """N > 1 only: the column-sharded int8 linear (weight split by output columns, N / g per
    rank, replicated [M, N] output wanted), with the gather fused into the GEMM epilogue (peer
    stores over NVLink) against the local GEMM + NCCL all_gather_into_tensor; both include the
    quantise of x.  Device ms per call, max over ranks; every result is checked equal to the
    NCCL path's."""
    from llm_kernels.sharding import (MulticastBuffers, PeerBuffers, column_sharded_int8_linear,
                                      column_sharded_int8_linear_fused, column_sharded_int8_linear_multicast,
                                      shard_columns)

    out = {}
    for M, K, N in ((4096, 4096, 11008), (8192, 4096, 4096)):
        if N % (8 * world):
            continue
        g = torch.Generator().manual_seed(M + N)
        x = torch.randn(M, K, generator=g).to(torch.float16).to(dev)
        w = torch.randn(N, K, generator=g).to(torch.float16).to(dev)
        layer = llm_kernels.Int8Linear(K, N).to(dev)
        layer.quantize_weights(w)
        wq = shard_columns(layer.w_q, rank, world).contiguous()
        sw = shard_columns(layer.scale_w[:, None], rank, world)[:, 0].contiguous()
        buf = PeerBuffers((M, N))
        reps = 10
        ms_f = time_loop(lambda: column_sharded_int8_linear_fused(x, wq, sw, buf), reps, 2, world) / reps
        ms_n = time_loop(lambda: column_sharded_int8_linear(x, wq, sw, N), reps, 2, world) / reps
        ref = column_sharded_int8_linear(x, wq, sw, N)
        same = bool(torch.equal(column_sharded_int8_linear_fused(x, wq, sw, buf), ref))
        buf.close()
        entry = {"fused_gather_ms": ms_f, "gemm_then_nccl_all_gather_ms": ms_n, "speedup": ms_n / ms_f,
                 "bit_identical": same}
        try:
            mbuf = MulticastBuffers((M, N))
        except Exception as e:  # noqa: BLE001
            mbuf = None
            entry["multicast"] = {"unavailable": str(e)[:100]}
        if mbuf is not None:
            ms_m = time_loop(lambda: column_sharded_int8_linear_multicast(x, wq, sw, mbuf), reps, 2, world) / reps
            y = column_sharded_int8_linear_multicast(x, wq, sw, mbuf)
            torch.cuda.synchronize()
            entry["multicast_gather_ms"] = ms_m
            entry["multicast_speedup_vs_nccl"] = ms_n / ms_m
            entry["multicast_bit_identical"] = bool(torch.equal(y, ref))
            mbuf.close()
        out[f"M{M}_K{K}_N{N}"] = entry
        del x, w, layer, wq, sw, buf
    torch.cuda.empty_cache()
    return out


def decoder_layer_measure(args, llm_kernels, world, rank, dev):
    """Config 5: the Llama-7B-shaped decoder-layer op mix (RMSNorm+QKV, causal attention,
    int8 O-proj, int8 MLP-up) on a global batch of 64 x 2048 tokens split over the ranks
    (strong scaling: 64 / n_gpus sequences per GPU), weights N(0, 0.02), x N(0, 1) bf16."""
    T, GB = 2048, 64
    from llm_kernels.sharding import shard_range

    s, e = shard_range(GB, rank, world)
    g = torch.Generator().manual_seed(4)
    layer = llm_kernels.DecoderLayerOps().to(dev)
    layer.init_weights(g)
    gx = torch.Generator().manual_seed(40 + rank)
    x = torch.randn(e - s, T, 4096, generator=gx).to(torch.bfloat16).to(dev)
    step = lambda: layer(x)  # noqa: E731
    reps = 2 if args.quick else 4
    ms = time_loop(step, reps, 2, world) / reps
    fl = layer.flops(GB, T)
    total = sum(fl.values())
    del x, layer
    torch.cuda.empty_cache()
    return {"value": GB * T / (ms * 1e-3), "unit": "tokens/s", "ms_per_layer": ms,
            "ops_per_s": total / (ms * 1e-3), "tera_ops_per_layer": {k: v / 1e12 for k, v in fl.items()},
            "sequences_per_gpu": e - s, "scaling": "strong (global batch 64 x 2048 fixed)"}


def roofline_entry(bound, achieved, peak, unit, peak_kind):
    return {"bound": bound, "achieved": achieved, "peak": peak, "unit": unit, "frac": achieved / peak,
            "peak_kind": peak_kind}


def secondary_ops(args, llm_kernels, peaks):
    """The metric's other clauses and the rest of the op set (rank 0, L2 flushed per call)."""
    dev = torch.device("cuda", torch.cuda.current_device())
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    reps = 5 if args.quick else 20
    ops = {}
    hbm = float(peaks["hbm_gbs"])
    # int8 GEMM + dequant, M=N=K=4096, per-row quantised operands (config 3)
    g = torch.Generator().manual_seed(2)
    A_fp = torch.randn(4096, 4096, generator=g).to(torch.float16).to(dev)
    B_fp = torch.randn(4096, 4096, generator=g).to(torch.float16).to(dev)
    A_q, sa = llm_kernels.quantize_symmetric(A_fp)
    B_q, sb = llm_kernels.quantize_symmetric(B_fp)
    B_kn = B_q.t().contiguous()
    ms = time_each_flushed(lambda: llm_kernels.int8_gemm_dequant_fwd(A_q, B_kn, sa, sb), reps, 3, flush)
    tops = 2 * 4096 ** 3 / (ms * 1e-3) / 1e12
    ops["int8_gemm_dequant_4096"] = {"value": tops, "unit": "TOPS", "ms": ms,
                                     "frac_of_4500_dense_int8_spec": tops / 4500,
                                     "layout": "B [K,N] (reference API)",
                                     "roofline": roofline_entry("tensor", tops, 4500.0, "TOPS",
                                                                "dense int8 spec (no measured int8 peak)")}
    ms = time_each_flushed(lambda: llm_kernels.int8_gemm_dequant_nk(A_q, B_q, sa, sb), reps, 3, flush)
    ops["int8_gemm_dequant_4096_nk"] = {"value": 2 * 4096 ** 3 / (ms * 1e-3) / 1e12, "unit": "TOPS", "ms": ms,
                                        "layout": "B [N,K] (Int8Linear weight)"}
    # The same GEMM with the raw int32 accumulator as output (like-for-like with the vendor line).
    ms = time_each_flushed(lambda: llm_kernels.int8_gemm_i32(A_q, B_q, "nk"), reps, 3, flush)
    ops["int8_gemm_i32_4096"] = {"value": 2 * 4096 ** 3 / (ms * 1e-3) / 1e12, "unit": "TOPS", "ms": ms,
                                 "layout": "B [N,K], int32 output"}
    # For comparison only (not part of the product): the vendor int8 GEMM (cuBLASLt through
    # torch._int_mm, int32 output, no dequant) on the same operands, timed the same way.
    try:
        B_cm = B_q.t()  # [K, N] view of the [N, K] codes: column-major, as _int_mm wants
        ms = time_each_flushed(lambda: torch._int_mm(A_q, B_cm), reps, 3, flush)
        ops["vendor_int8_gemm_i32_4096"] = {"value": 2 * 4096 ** 3 / (ms * 1e-3) / 1e12, "unit": "TOPS", "ms": ms,
                                            "what": "cuBLASLt int8 x int8 -> int32 via torch._int_mm (comparison)"}
    except Exception as e:  # noqa: BLE001
        ops["vendor_int8_gemm_i32_4096"] = {"unavailable": str(e)[:120]}
    # The O projection of the decoder layer with its output re-quantised for the MLP-up
    # projection: one kernel (int8_gemm_dequant_requant) against GEMM + quantize_symmetric.
    M5 = 131072
    a5 = torch.randint(-127, 128, (M5, 4096), dtype=torch.int8, device=dev)
    s5 = torch.rand(M5, device=dev) * 1e-3
    ms_f = time_each_flushed(lambda: llm_kernels.int8_gemm_dequant_requant(a5, B_q, s5, sb, "nk"), max(3, reps // 4), 2,
                             flush)
    ms_2 = time_each_flushed(lambda: llm_kernels.quantize_symmetric(llm_kernels.int8_gemm_dequant_nk(a5, B_q, s5, sb)),
                             max(3, reps // 4), 2, flush)
    tops = 2 * M5 * 4096 * 4096 / (ms_f * 1e-3) / 1e12
    ops["int8_gemm_requant_131072x4096x4096"] = {
        "value": tops, "unit": "TOPS", "ms": ms_f, "gemm_then_quantize_ms": ms_2,
        "roofline": roofline_entry("tensor", tops, 4500.0, "TOPS", "dense int8 spec (no measured int8 peak)")}
    del a5, s5
    # quantize_symmetric 4096x4096 fp16 (config 3b)
    ms = time_each_flushed(lambda: llm_kernels.quantize_symmetric(A_fp), reps, 3, flush)
    qbytes = 4096 * 4096 * 2 + 4096 * 4096 + 4096 * 4
    ops["quantize_4096_f16"] = {"value": qbytes / (ms * 1e-3) / 1e9, "unit": "GB/s", "ms": ms,
                                "frac_of_hbm": qbytes / (ms * 1e-3) / 1e9 / hbm,
                                "roofline": roofline_entry("hbm", qbytes / (ms * 1e-3) / 1e9, hbm, "GB/s",
                                                           "measured HBM copy")}
    # The same quantiser on a config-5 activation (131072 tokens x 4096, bf16, 1 GiB): the size
    # it runs at inside the decoder layer, where launch and tail costs no longer dominate.
    xa = torch.randn(131072, 4096, dtype=torch.bfloat16, device=dev)
    ms = time_each_flushed(lambda: llm_kernels.quantize_symmetric(xa), max(3, reps // 4), 2, flush)
    qb = 131072 * 4096 * 3 + 131072 * 4
    ops["quantize_131072x4096_bf16"] = {"value": qb / (ms * 1e-3) / 1e9, "unit": "GB/s", "ms": ms,
                                        "roofline": roofline_entry("hbm", qb / (ms * 1e-3) / 1e9, hbm, "GB/s",
                                                                   "measured HBM copy")}
    del xa
    # fused RMSNorm + Linear, config 1 shape (bf16 and fp16)
    g = torch.Generator().manual_seed(0)
    x = torch.randn(512, 4096, generator=g)
    wn = (1 + 0.1 * torch.randn(4096, generator=g))
    wl = torch.randn(4096, 4096, generator=g) / 64
    for dt, tag in ((torch.bfloat16, "bf16"), (torch.float16, "f16")):
        xd, wnd, wld = x.to(dt).to(dev), wn.to(dt).to(dev), wl.to(dt).to(dev)
        llm_kernels.fused_rmsnorm_linear(xd, wnd, wld)  # folds the weight once (cached per weight version)
        ms = time_each_flushed(lambda: llm_kernels.fused_rmsnorm_linear(xd, wnd, wld), reps, 3, flush)
        tf = 2 * 512 * 4096 * 4096 / (ms * 1e-3) / 1e12
        ops[f"rmsnorm_linear_512x4096x4096_{tag}"] = {
            "value": ms, "unit": "ms", "tflops": tf,
            "roofline": roofline_entry("tensor", tf, float(peaks["bf16_tflops"]), "TFLOP/s", "measured bf16 burst"),
            "hbm_frac": 4.195e7 / (ms * 1e-3) / 1e9 / hbm}
    # non-causal FA config 2
    g = torch.Generator().manual_seed(1)
    q = torch.randn(B, H, N, D, generator=g).to(torch.bfloat16).to(dev)
    k = torch.randn(B, H, N, D, generator=g).to(torch.bfloat16).to(dev)
    v = torch.randn(B, H, N, D, generator=g).to(torch.bfloat16).to(dev)
    ms = time_loop(lambda: llm_kernels.flash_attn_forward(q, k, v, causal=False), reps, 2, 1) / reps
    tf = fa_flops(B, H, N, D, False) / (ms * 1e-3) / 1e12
    ops["flash_attn_noncausal_bf16_B4H32N4096D128"] = {
        "value": tf, "unit": "TFLOP/s", "ms": ms,
        "roofline": roofline_entry("tensor", tf, float(peaks["bf16_tflops"]), "TFLOP/s", "measured bf16 burst")}
    # grouped-query attention: 8 K/V heads shared by 32 query heads, read in place
    kg, vg = k[:, :8].contiguous(), v[:, :8].contiguous()
    ms = time_loop(lambda: llm_kernels.flash_attn_forward(q, kg, vg, causal=True), reps, 2, 1) / reps
    tf = fa_flops(B, H, N, D, True) / (ms * 1e-3) / 1e12
    ops["flash_attn_gqa_causal_bf16_B4H32KV8N4096D128"] = {
        "value": tf, "unit": "TFLOP/s", "ms": ms,
        "roofline": roofline_entry("tensor", tf, float(peaks["bf16_tflops"]), "TFLOP/s", "measured bf16 burst")}
    # training path at the config-2 shape: forward with LSE + backward (dQ, dK, dV), causal
    # bf16.  FLOPs counted as the 5 matmuls of the backward (S, dP, dV, dK, dQ: 2.5x the forward),
    # the usual algorithmic count; this implementation runs 7 (its dQ pass recomputes S and dP).
    from llm_kernels.flash_attn_bwd import _backward, _forward_lse
    do = torch.randn(B, H, N, D, generator=g).to(torch.bfloat16).to(dev)
    scale = D ** -0.5
    out, lse = _forward_lse(q, k, v, True, scale)
    ms = time_loop(lambda: _backward(q, k, v, out, do, lse, True, scale), reps, 2, 1) / reps
    ops["flash_attn_bwd_causal_bf16_B4H32N4096D128"] = {
        "value": 2.5 * FLOPS_CAUSAL / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms": ms,
        "flops": "2.5x the forward (S, dP, dV, dK, dQ); the kernels execute 3.5x (S and dP recomputed for dQ)",
        "frac_of_burst": 2.5 * FLOPS_CAUSAL / (ms * 1e-3) / 1e12 / float(peaks["bf16_tflops"]),
        "roofline": roofline_entry("tensor", 2.5 * FLOPS_CAUSAL / (ms * 1e-3) / 1e12, float(peaks["bf16_tflops"]),
                                   "TFLOP/s", "measured bf16 burst")}
    del q, k, v, kg, vg, do, out, lse
    # config 4 sweep: fp16, B8 H16 D64
    sweep = {}
    for n in ([512, 4096] if args.quick else [512, 1024, 2048, 4096, 8192, 16384]):
        g = torch.Generator().manual_seed(3)
        q = torch.randn(8, 16, n, 64, generator=g).to(torch.float16).to(dev)
        k = torch.randn(8, 16, n, 64, generator=g).to(torch.float16).to(dev)
        v = torch.randn(8, 16, n, 64, generator=g).to(torch.float16).to(dev)
        r = max(3, min(reps, int(2e4 / n)))
        for causal in (True, False):
            ms = time_loop(lambda: llm_kernels.flash_attn_forward(q, k, v, causal=causal), r, 2, 1) / r
            sweep[f"N{n}_{'causal' if causal else 'dense'}"] = round(fa_flops(8, 16, n, 64, causal) / (ms * 1e-3) / 1e12, 1)
        del q, k, v
    ops["flash_attn_sweep_f16_B8H16D64_tflops"] = sweep
    ops["reference_gpu_same_box"] = reference_gpu_ops(args, llm_kernels, dev, flush, reps)
    del flush
    return ops


def reference_gpu_ops(args, llm_kernels, dev, flush, reps):
    """The reference's own GPU implementations timed on this B200 beside this library's kernels
    on the same inputs (comparison context only; this benchmark's reference arm is the
    reference's CPU path).  Its kernels take fp16 only, so the attention line is fp16 here."""
    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_dir, "kernels")):
        return {"unavailable": "the reference is not installed in baseline/_ref"}
    try:
        if ref_dir not in sys.path:
            sys.path.append(ref_dir)
        import kernels as ref
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"import failed: {str(e)[:100]}"}
    out = {}
    g = torch.Generator().manual_seed(1)
    q, k, v = (torch.randn(B, H, N, D, generator=g).to(torch.float16).to(dev) for _ in range(3))
    r = max(3, reps // 2)
    theirs = time_loop(lambda: ref.flash_attn_forward(q, k, v, causal=True), r, 2, 1) / r
    ours = time_loop(lambda: llm_kernels.flash_attn_forward(q, k, v, causal=True), r, 2, 1) / r
    out["flash_attn_causal_f16_B4H32N4096D128"] = {
        "reference_triton_tflops": FLOPS_CAUSAL / (theirs * 1e-3) / 1e12,
        "ours_tflops": FLOPS_CAUSAL / (ours * 1e-3) / 1e12, "speedup": theirs / ours}
    del q, k, v
    A_q = torch.randint(-127, 128, (4096, 4096), dtype=torch.int8, device=dev)
    B_kn = torch.randint(-127, 128, (4096, 4096), dtype=torch.int8, device=dev)
    sa = torch.rand(4096, device=dev) * 1e-3
    sb = torch.rand(4096, device=dev) * 1e-3
    theirs = time_each_flushed(lambda: ref.int8_gemm_dequant_fwd(A_q, B_kn, sa, sb), reps, 3, flush)
    ours = time_each_flushed(lambda: llm_kernels.int8_gemm_dequant_fwd(A_q, B_kn, sa, sb), reps, 3, flush)
    out["int8_gemm_dequant_4096"] = {"reference_triton_tops": 2 * 4096 ** 3 / (theirs * 1e-3) / 1e12,
                                     "ours_tops": 2 * 4096 ** 3 / (ours * 1e-3) / 1e12, "speedup": theirs / ours}
    x = torch.randn(512, 4096, generator=g).to(torch.float16).to(dev)
    wn = (1 + 0.1 * torch.randn(4096, generator=g)).to(torch.float16).to(dev)
    wl = (torch.randn(4096, 4096, generator=g) / 64).to(torch.float16).to(dev)
    llm_kernels.fused_rmsnorm_linear(x, wn, wl)
    theirs = time_each_flushed(lambda: ref.fused_rmsnorm_linear(x, wn, wl), reps, 3, flush)
    ours = time_each_flushed(lambda: llm_kernels.fused_rmsnorm_linear(x, wn, wl), reps, 3, flush)
    from kernels.fused_rmsnorm_linear import fused_ops as ref_ops
    # The reference's CUDA extension builds but does not import (csrc/bindings.cpp:12 declares
    # launch_fused_rmsnorm_linear with at::Half pointers, csrc/fused_rmsnorm_linear.cu:105 defines
    # it with half pointers: an undefined symbol), so its dispatcher runs the PyTorch path.
    out["rmsnorm_linear_512x4096x4096_f16"] = {
        "reference_ms": theirs, "ours_ms": ours, "speedup": theirs / ours,
        "reference_path": "CUDA extension" if ref_ops._HAS_CUDA_EXT else
        "PyTorch fallback (its CUDA extension fails to import: undefined launch_fused_rmsnorm_linear symbol)"}
    xq = torch.randn(4096, 4096, generator=g).to(torch.float16).to(dev)
    theirs = time_each_flushed(lambda: ref.quantize_symmetric(xq), reps, 3, flush)
    ours = time_each_flushed(lambda: llm_kernels.quantize_symmetric(xq), reps, 3, flush)
    out["quantize_4096_f16"] = {"reference_torch_ms": theirs, "ours_ms": ours, "speedup": theirs / ours}
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--quick", action="store_true", help="fewer repetitions of the secondary ops")
    ap.add_argument("--only", choices=["fa", "fa_dense", "fa_bwd", "int8", "quantize", "quantize_c5", "requant",
                                       "rmsnorm"], default=None,
                    help="run just one op's device loop (warmup + steps) and print nothing else: "
                         "the command the ncu profiles under profiles/ are taken on")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.only:
        run_only(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


def run_only(args):
    """One op's kernels alone (for ncu); no timing, no output besides a done line."""
    import llm_kernels

    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(1)
    if args.only in ("fa", "fa_dense", "fa_bwd"):
        q = torch.randn(B, H, N, D, generator=g).to(torch.bfloat16).to(dev)
        k = torch.randn(B, H, N, D, generator=g).to(torch.bfloat16).to(dev)
        v = torch.randn(B, H, N, D, generator=g).to(torch.bfloat16).to(dev)
        fn = lambda: llm_kernels.flash_attn_forward(q, k, v, causal=args.only == "fa")  # noqa: E731
        if args.only == "fa_bwd":
            from llm_kernels.flash_attn_bwd import _backward, _forward_lse
            do = torch.randn(B, H, N, D, generator=g).to(torch.bfloat16).to(dev)
            out, lse = _forward_lse(q, k, v, True, D ** -0.5)
            fn = lambda: _backward(q, k, v, out, do, lse, True, D ** -0.5)  # noqa: E731
    elif args.only in ("int8", "quantize"):
        A_fp = torch.randn(4096, 4096, generator=g).to(torch.float16).to(dev)
        B_fp = torch.randn(4096, 4096, generator=g).to(torch.float16).to(dev)
        A_q, sa = llm_kernels.quantize_symmetric(A_fp)
        B_q, sb = llm_kernels.quantize_symmetric(B_fp)
        B_kn = B_q.t().contiguous()
        if args.only == "int8":
            fn = lambda: llm_kernels.int8_gemm_dequant_fwd(A_q, B_kn, sa, sb)  # noqa: E731
        else:
            fn = lambda: llm_kernels.quantize_symmetric(A_fp)  # noqa: E731
    elif args.only == "quantize_c5":
        xa = torch.randn(131072, 4096, dtype=torch.bfloat16, device=dev)
        fn = lambda: llm_kernels.quantize_symmetric(xa)  # noqa: E731
    elif args.only == "requant":
        # 16384 rows of the O projection (64 row blocks x 16 tiles): a profiling-size case
        a5 = torch.randint(-127, 128, (16384, 4096), dtype=torch.int8, device=dev)
        w5 = torch.randint(-127, 128, (4096, 4096), dtype=torch.int8, device=dev)
        s5 = torch.rand(16384, device=dev) * 1e-3
        t5 = torch.rand(4096, device=dev) * 1e-3
        fn = lambda: llm_kernels.int8_gemm_dequant_requant(a5, w5, s5, t5, "nk")  # noqa: E731
    else:
        x = torch.randn(512, 4096, generator=g).to(torch.bfloat16).to(dev)
        wn = (1 + 0.1 * torch.randn(4096, generator=g)).to(torch.bfloat16).to(dev)
        wl = (torch.randn(4096, 4096, generator=g) / 64).to(torch.bfloat16).to(dev)
        fn = lambda: llm_kernels.fused_rmsnorm_linear(x, wn, wl)  # noqa: E731
    for _ in range(args.warmup + args.steps):
        fn()
    torch.cuda.synchronize()
    print(f"only={args.only} done", flush=True)


if __name__ == "__main__":
    main()
