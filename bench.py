"""Benchmark of the KV-compression hot path on B200.

    python bench.py [--gpus N --steps K --warmup W] [--impl engine|reference]

Workload (per GPU, weak scaling): the 2-bit-mode configuration -- K and V
tensors fp16 [B=1, H=16, S=40000, D=256] (N(0,1) with 2% Student-t(3)
channels, seeded), compressed to code bits + residual sign bits + two norms
per row.  One step = one fused launch over both tensors (1.28M rows).  Inputs
(655 MB per step) exceed the 126 MB L2, so no flush is needed between steps.
Also reported: decode attention over a 2-bit compressed cache (q bf16
[32, 16, 128], S = 40000) in us per step and us per token.

``--impl reference`` times the reference algorithm's CPU implementation (the
oracle port of KudaHitamCUDA.cu:13-195, OpenMP over every host thread) on a
bounded sample of the same workload; for context its line also carries the
reference's own CUDA kernel v8 timed on this GPU on the same rows, when that
kernel has been built from the reference source (oracle/build_ref.py).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import pathlib
import statistics
import subprocess
import sys
import threading
import time

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "kudahitam-quant_b200"))
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = ("KV rows compressed/sec and HBM GB/s (% of peak); "
          "decode-attn µs/token at 40k ctx")
B, H, S, D = 1, 16, 40000, 256
ROWS_PER_TENSOR = B * H * S
ALG_BYTES_PER_ROW = D * 2 + 2 * D // 8 + 8   # read fp16 row; write 2 planes + 2 norms
DEC_B, DEC_H, DEC_S, DEC_D = 32, 16, 40000, 128
DEC_BYTES_PER_ROW = 2 * (2 * DEC_D // 8 + 8)  # K and V: 2 planes + 2 norms each
FALLBACK_HBM_GBS = 6650.0

# dram__bytes_read.sum + dram__bytes_write.sum per compressed row, from an ncu
# capture of compress_tc_kernel<__half,256> on 524,288 rows of the same row
# format: 268.48 MB read + 8.79 MB written.  Reads equal the algorithmic
# bytes; most of the packed output is still in L2 when the kernel ends, so
# the DRAM write count is below the 72 B/row written.  Traffic grows in
# proportion to the rows, so it is scaled to a full launch.
NCU_TRAFFIC_BYTES_PER_ROW = (268.480256e6 + 8.786688e6) / 524288
# Same for the decode step (an ncu capture of decode_v3_kernel<128> on the
# bench's decode workload itself): bytes per cached row of K and V.
NCU_DECODE_TRAFFIC_BYTES_PER_ROW = (1.639534e9 + 3.693824e6) / (512 * 40000)


def peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def synth_kv(seed: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    g = torch.Generator(device=device).manual_seed(seed)
    out = []
    for t in range(2):
        x = torch.randn(B, H, S, D, device=device, generator=g)
        n = round(0.02 * D)
        ch = torch.randperm(D, device=device, generator=g)[: n]
        # Student-t(3) = N / sqrt(chi2_3 / 3)
        z = torch.randn(B, H, S, n, device=device, generator=g)
        chi = (torch.randn(B, H, S, n, 3, device=device, generator=g) ** 2).sum(-1)
        x[..., ch] = z / torch.sqrt(chi / 3.0)
        out.append(x.half())
    return out[0], out[1]


class ClockSampler:
    """SM clock and clock-event (throttle) reasons, sampled through NVML
    (read-only queries) every 0.5 ms from a host thread.  Samples carry host
    timestamps so that the ones taken inside the timed region can be told
    apart from those of the adjacent loaded loops (warm-up and per-launch
    timing of the same kernel)."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
               "hw_thermal_slowdown": 0x40, "sw_power_cap": 0x4}

    def __init__(self, index: int, period_s: float = 0.0005):
        self.index = index
        self.period = period_s
        self.samples: list[tuple[float, float, int]] = []  # (t, MHz, reasons mask)
        self.max_mhz = None
        self.err = None
        self.region = None
        self._stop = threading.Event()

    def __enter__(self):
        try:
            import pynvml as N
            N.nvmlInit()
            self._N = N
            self._h = N.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = float(N.nvmlDeviceGetMaxClockInfo(self._h, N.NVML_CLOCK_SM))
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        except Exception as e:  # NVML missing: report, do not fail the bench
            self.err = repr(e)
            self._N = None
        return self

    def _run(self):
        N = self._N
        while not self._stop.is_set():
            try:
                mhz = float(N.nvmlDeviceGetClockInfo(self._h, N.NVML_CLOCK_SM))
                mask = int(N.nvmlDeviceGetCurrentClocksEventReasons(self._h))
                self.samples.append((time.perf_counter(), mhz, mask))
            except Exception as e:
                self.err = repr(e)
                return
            self._stop.wait(self.period)

    def mark_region(self, t0: float, t1: float) -> None:
        self.region = (t0, t1)

    def __exit__(self, *exc):
        self._stop.set()
        if self._N is not None:
            self._t.join(timeout=2)

    def summary(self) -> dict:
        inside = [s for s in self.samples
                  if self.region and self.region[0] <= s[0] <= self.region[1]]
        use = inside if len(inside) >= 3 else self.samples
        mask = 0
        for s in self.samples:
            mask |= s[2]
        out = {"sm_mhz": statistics.median(s[1] for s in use) if use else None,
               "sm_max_mhz": self.max_mhz,
               "reasons": sorted(k for k, b in self.REASONS.items() if mask & b),
               "samples": len(use), "samples_in_timed_region": len(inside),
               "window": ("timed region" if use is inside else
                          "timed region + adjacent warm-up and per-launch loops of "
                          "the same kernel (timed region shorter than 3 samples)")}
        if self.err:
            out["error"] = self.err
        return out


def dist_setup(args):
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


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    from kudahitam.dist import max_over_ranks as m
    return m(v, device=torch.device("cuda", torch.cuda.current_device()))


def host_cores() -> int:
    """Host threads this process may run on (torch.distributed.run sets
    OMP_NUM_THREADS=1 in every rank; the CPU baseline passes this count to
    the oracle explicitly instead of inheriting that)."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):  # pragma: no cover
        return os.cpu_count() or 1


class CpuSample:
    """A bounded sample of the workload's fp16 rows for the CPU baseline,
    generated once (the same distribution: N(0,1) with 2 % Student-t(3)
    channels) and compressed by the oracle port (KudaHitamCUDA.cu:13-195
    restated) on every host core."""

    def __init__(self, target_s: float, max_rows: int = 1 << 22):
        from oracle import oracle as O
        from kudahitam.codebook import lloyd_max, rademacher
        self.O = O
        self.cores = host_cores()
        self.d = rademacher(D, 1).numpy()
        self.c = lloyd_max(1, D).numpy()
        self.rng = np.random.default_rng(2)
        probe = self._rows(16384)
        self.run(probe)  # first touch / thread pool start
        dt = self.run(probe)
        n = int(min(max_rows, max(16384, 16384 * target_s / max(dt, 1e-6))))
        self.x = self._rows(n)

    def _rows(self, n: int) -> np.ndarray:
        x = self.rng.standard_normal((n, D)).astype(np.float32)
        k = round(0.02 * D)
        ch = self.rng.choice(D, k, replace=False)
        x[:, ch] = self.rng.standard_t(3, size=(n, k))
        return x.astype(np.float16)

    def run(self, x=None) -> float:
        """Seconds to compress the sample (or x) on every host core."""
        x = self.x if x is None else x
        t0 = time.perf_counter()
        self.O.compress_v8(x, self.d, self.c, want=("norms", "rnorms", "signs", "idx"),
                           n_threads=self.cores)
        return time.perf_counter() - t0

    def describe(self, value: float, dt: float) -> dict:
        return {"value": value, "unit": "rows/s", "cores": self.cores, "kind": "port",
                "sample": f"{self.x.shape[0]} fp16 rows of the D=256 2-bit-mode workload "
                          f"(same distribution), {dt:.2f} s per pass"}


def all_ranks(v: float, world: int) -> list[float]:
    """A per-rank scalar from every rank (rank order), for the record."""
    if world == 1:
        return [float(v)]
    import torch.distributed as dist
    t = torch.tensor([float(v)], dtype=torch.float64, device=torch.cuda.current_device())
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [float(x.item()) for x in out]


def cpu_baseline_run(target_s: float = 10.0, max_rows: int = 1 << 22) -> dict:
    """The oracle port on a bounded sample of the workload, all host threads."""
    smp = CpuSample(target_s, max_rows)
    dt = smp.run()
    return smp.describe(smp.x.shape[0] / dt, dt)


def run_reference(args, world, rank):
    """The reference arm: the CPU restatement of the reference kernel on every
    host core, rank 0 only (other ranks exit without work).  Each step
    compresses the same bounded sample of the workload (about 2 s)."""
    if rank != 0:
        return
    cfg = workload_config(world)  # the engine arm's config at this N
    smp = CpuSample(target_s=2.0)
    small = smp.x[:16384]
    for _ in range(args.warmup):
        smp.run(small)
    times = [smp.run() for _ in range(args.steps)]
    t_med = statistics.median(times)
    v = smp.x.shape[0] / t_med
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "rows/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": t_med * 1e3, "sample_rows_per_step": smp.x.shape[0],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic", "config": cfg,
            "cpu_baseline": smp.describe(v, t_med),
            "e2e": {"value": v, "unit": "rows/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    gk = reference_kernel_on_gpu(args)
    if gk is not None:
        line["reference_kernel_v8_on_this_gpu"] = gk
    print(json.dumps(line), flush=True)


def reference_kernel_on_gpu(args):
    """For context: the reference's own CUDA kernel v8 (KudaHitamCUDA.cu:13-231,
    built from the reference source into oracle/_ref) on this GPU, on the same
    K and V rows, through its own launcher (which allocates the 6D+8 bytes per
    row of reference-layout outputs each call), beside this engine's compat
    operator on the same rows.  None without a GPU or that build."""
    if not torch.cuda.is_available():
        return None
    from oracle import oracle as O
    ref = O.reference_kernels()
    if ref is None:
        return None
    from kudahitam.codebook import lloyd_max, rademacher
    dev = torch.device("cuda", 0)
    k, v = synth_kv(2, dev)
    rows = [t.reshape(-1, D).contiguous() for t in (k, v)]
    assert (rows[0].shape[0] * D) % 2048 == 0  # the kernel is only safe on whole blocks
    d, c = rademacher(D, 1).to(dev), lloyd_max(1, D).to(dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        for r in rows:
            ref.ultra_fused_full_fusion(r, d, c)

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    ms = statistics.median(time_loop(step, max(5, min(args.steps, 20)), stream))
    n = 2 * rows[0].shape[0]
    peak, _ = peaks()
    moved = n * (D * 2 + 6 * D + 8)
    out = {"rows_per_s": n / (ms / 1e3), "ms_per_step": ms,
           "bytes_per_row": D * 2 + 6 * D + 8, "gbs": moved / (ms / 1e3) / 1e9,
           "frac_of_measured_hbm": moved / (ms / 1e3) / 1e9 / peak,
           "note": "reference kernel v8 with its own launcher, same K and V fp16 rows"}
    del rows
    eng = engine_compat_timing(args, k, v)
    eng["speedup_vs_reference_kernel"] = ms / eng["ms_per_step"]
    out["engine_compat_op_same_outputs"] = eng
    del k, v
    torch.cuda.empty_cache()
    return out


def engine_compat_timing(args, k=None, v=None) -> dict:
    """This engine's compat operator with the reference kernel's five
    outputs (ops.ultra_fused_full_fusion: compress + materialize) on the
    bench's K and V fp16 rows, outputs allocated per call like the
    reference launcher."""
    from kudahitam import ops
    from kudahitam.codebook import lloyd_max, rademacher
    dev = torch.device("cuda", torch.cuda.current_device())
    if k is None:
        k, v = synth_kv(2, dev)
    rows = [t.reshape(-1, D).contiguous() for t in (k, v)]
    dh, ch = rademacher(D, 1), lloyd_max(1, D)
    stream = torch.cuda.current_stream(dev)

    def step():
        for r in rows:
            ops.ultra_fused_full_fusion(r, dh, ch)

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    ms = statistics.median(time_loop(step, max(5, min(args.steps, 20)), stream))
    n = 2 * rows[0].shape[0]
    peak, _ = peaks()
    moved = n * (D * 2 + 6 * D + 8)
    return {"rows_per_s": n / (ms / 1e3), "ms_per_step": ms, "bytes_per_row": D * 2 + 6 * D + 8,
            "gbs": moved / (ms / 1e3) / 1e9, "frac_of_measured_hbm": moved / (ms / 1e3) / 1e9 / peak,
            "note": "ops.ultra_fused_full_fusion: the reference's five outputs (idx u8, norms, "
                    "k_mse f32, r_norms, signs i8) from compress + materialize, outputs "
                    "allocated per call like the reference launcher"}


def workload_config(world: int) -> dict:
    return {"workload": "kv-compress 2-bit mode (code bits + QJL residual signs + 2 norms), "
                        "K and V fp16 [1,16,40000,256] per GPU",
            "head_dim": D, "input_dtype": "fp16", "rows_per_step": 2 * ROWS_PER_TENSOR * world,
            "global_batch": 2 * ROWS_PER_TENSOR * world, "seq_len": S,
            "parallelism": f"shard b*h x{world}, no comm",
            "l2": "inputs 655 MB per GPU per step > 126 MB L2: no flush"}


def time_loop(fn, steps: int, stream) -> list[float]:
    """Per-step CUDA-event times (ms) on `stream`."""
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(steps)]
    for a, b in evs:
        a.record(stream)
        fn()
        b.record(stream)
    torch.cuda.synchronize()
    return [a.elapsed_time(b) for a, b in evs]


def run_engine(args, world, rank, local):
    from kudahitam import KudahitamCompressorV2, ops
    from kudahitam.codebook import lloyd_max, rademacher
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    peak, peak_kind = peaks()

    if args.only == "decode":
        dec = decode_bench(dev, args, world, rank)
        if rank == 0:
            print(json.dumps({"decode": dec}), flush=True)
        return
    if args.only == "score":
        if rank == 0:
            print(json.dumps({"score": score_bench(dev, args)}), flush=True)
        return
    if args.only == "fp32":
        if rank == 0:
            print(json.dumps({"fp32_1bit": fp32_1bit_bench(dev, args)}), flush=True)
        return
    if args.only == "compat":
        if rank == 0:
            print(json.dumps({"compat": engine_compat_timing(args)}), flush=True)
        return
    if args.only == "cfg5":
        c5 = cfg5_bench(dev, args, world, rank)
        if rank == 0:
            print(json.dumps({"sharded_8gpu_workload": c5}), flush=True)
        return
    if args.only == "layers":
        lay = layers_bench(dev, args)
        if rank == 0:
            print(json.dumps({"layers_28": lay}), flush=True)
        return
    k, v = synth_kv(2 + 1000 * rank, dev)
    d = rademacher(D, 1)
    c = lloyd_max(1, D)
    outs = [ops.empty_packed(k.shape, 1, True, dev), ops.empty_packed(v.shape, 1, True, dev)]
    stream = torch.cuda.current_stream(dev)

    def step():
        ops.compress_many([k, v], d, c, residual=True, outs=outs)

    with ClockSampler(local) as clk:
        for _ in range(max(args.warmup, 3)):
            step()
        torch.cuda.synchronize()
        barrier(world)
        torch.cuda.synchronize()
        h0 = time.perf_counter()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(args.steps):
            step()  # one kernel launch per step
        t1.record(stream)
        torch.cuda.synchronize()
        clk.mark_region(h0, time.perf_counter())
        barrier(world)
        torch.cuda.synchronize()
        ms_local = t0.elapsed_time(t1)
        ms = max_over_ranks(ms_local, world)
        per_rank_ms = all_ranks(ms_local, world)
        rows_all = 2 * ROWS_PER_TENSOR * world * args.steps
        value = rows_all / (ms / 1e3)
    # average launch duration over the timed region (one launch per step,
    # back to back on this stream; inter-launch gaps count against it)
    launch_ms = ms_local / args.steps
    rows_launch = 2 * ROWS_PER_TENSOR
    achieved = rows_launch * ALG_BYTES_PER_ROW / (launch_ms / 1e3) / 1e9
    roof = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
            "frac": achieved / peak, "peak_kind": peak_kind,
            "traffic": (NCU_TRAFFIC_BYTES_PER_ROW * rows_launch
                        if NCU_TRAFFIC_BYTES_PER_ROW else None),
            "algorithmic_bytes": rows_launch * ALG_BYTES_PER_ROW,
            "launch_ms_mean": launch_ms, "launches_timed": args.steps,
            "launch_ms_mean_per_rank": [t / args.steps for t in per_rank_ms],
            "timing": "CUDA events around the timed region / launches in it",
            "kernel": ("compress_simt_kernel<__half,256,Sym2,RES>"
                       if os.environ.get("KUDAHITAM_COMPRESS_PATH") == "simt"
                       else "compress_tc_kernel<__half,256,Sym2,RES>")}

    # e2e through the public API with host buffers: K and V in pinned host
    # memory, packed caches back to pinned host memory, every step.  The API
    # streams 64 MB chunks with uploads, kernels and downloads overlapped.
    comp = KudahitamCompressorV2(D, 1, seed=1)
    hk = k.cpu().pin_memory()
    hv = v.cpu().pin_memory()
    host_outs = [ops.empty_packed_pinned(t.shape, 1, True) for t in (hk, hv)]

    def e2e_step():
        return comp.compress_to_host([hk, hv], device=dev, outs=host_outs)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e2e_steps = max(2, min(args.steps, 10))
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world)
    h2d = hk.numel() * 2 + hv.numel() * 2
    d2h = sum(p.nbytes() for p in host_outs)
    e2e = {"value": 2 * ROWS_PER_TENSOR * world * e2e_steps / (e2e_ms / 1e3), "unit": "rows/s",
           "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
           "ms_per_step": e2e_ms / e2e_steps,
           "h2d_gbs": h2d / (e2e_ms / e2e_steps / 1e3) / 1e9,
           "api": "KudahitamCompressorV2.compress_to_host (pinned host in and out)"}
    del hk, hv, host_outs

    dec = decode_bench(dev, args, world, rank) if args.only == "all" else None
    lay = (layers_bench(dev, args)
           if args.only == "all" and not args.no_layers and world == 1 else None)
    f32 = fp32_1bit_bench(dev, args) if args.only == "all" and world == 1 else None
    sco = score_bench(dev, args) if args.only == "all" and world == 1 else None
    torch.cuda.empty_cache()
    c5 = cfg5_bench(dev, args, world, rank) if args.only == "all" and not args.no_cfg5 else None

    line = {"metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic", "config": workload_config(world),
            "hbm_gbs": achieved, "hbm_frac_of_measured": achieved / peak,
            "hbm_frac_of_spec_8000": achieved / 8000.0,
            "roofline": roof, "e2e": e2e, "decode": dec, "layers_28": lay,
            "fp32_1bit": f32, "score": sco, "sharded_8gpu_workload": c5,
            "gpu_launches": args.steps, "clocks": clk.summary()}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_run()
    if rank == 0:
        print(json.dumps(line), flush=True)


def score_bench(dev, args) -> dict:
    """Asymmetric scores (the reference's asymmetric_attention_scores) of q
    [32, 16, 128] against a packed K cache [32, 16, 40000, 128] with the
    residual plane: the bits=1 codebook (40 B read and 4 B written per cached
    row) and the bits=2 codebook (2-bit code plane: 56 B read, 4 written)."""
    from kudahitam import ops
    from kudahitam.codebook import lloyd_max, rademacher
    G, S_, Dq = DEC_B * DEC_H, DEC_S, DEC_D
    q = torch.randn(G, 1, Dq, generator=torch.Generator().manual_seed(4)).to(dev)
    out = torch.empty(G, 1, S_, device=dev)
    stream = torch.cuda.current_stream(dev)
    K = ops.ext()
    peak, _ = peaks()
    res = {"config": "q [32,16,1,128] vs packed K [32,16,40000,128] (code + residual planes)"}
    for bits in (1, 2):
        d, c = rademacher(Dq, 10), lloyd_max(bits, Dq)
        g = torch.Generator(device=dev).manual_seed(5)
        pk = ops.empty_packed((G, S_, Dq), bits, True, dev)
        for i in range(0, G, 64):
            x = torch.randn(64, S_, Dq, device=dev, generator=g).to(torch.bfloat16)
            ops.compress(x, d, c, out=pk.rows(i * S_, (i + 64) * S_))
        dh, ch = ops._host_f32(d), ops._host_f32(c)

        def step():
            # the operator's own launch, writing into a preallocated output
            K.score_out(q, pk.code, pk.res, pk.norms, pk.rnorms, S_, dh, ch, out)

        for _ in range(3):
            step()
        torch.cuda.synchronize()
        ms = statistics.median(time_loop(step, 20, stream))
        bpr = (Dq // 32 if bits == 1 else Dq // 16) * 4 + Dq // 8 + 8 + 4
        bytes_step = G * S_ * bpr
        entry = {"us_per_step": ms * 1e3, "bytes_per_row": bpr,
                 "gbs": bytes_step / (ms / 1e3) / 1e9,
                 "frac_of_measured_hbm": bytes_step / (ms / 1e3) / 1e9 / peak,
                 "kernel": ("score_tab_kernel<128, residual>" if bits == 1
                            else "score_tab2b_kernel<residual>")}
        if bits == 1:
            res.update(entry)  # the bits=1 figures at the top level, as before
        else:
            res["bits2"] = entry
        del pk
    return res


def fp32_1bit_bench(dev, args) -> dict:
    """The CPU-runnable configuration in 1-bit mode on the GPU: K and V fp32
    [1, 16, 10000, 128], N(0,1) with 3 channels per head scaled by 10
    (seeded), code + norm per row (532 B/row), both tensors in one launch;
    plus the same at S = 40000 (655 MB of input, above L2)."""
    from kudahitam import ops
    from kudahitam.codebook import lloyd_max, rademacher
    d, c = rademacher(128, 1), lloyd_max(1, 128)
    peak, _ = peaks()
    stream = torch.cuda.current_stream(dev)
    out = {"config": "K, V fp32 [1,16,S,128], 3 outlier channels x10 per head, 1-bit mode"}
    for S_ in (10000, 40000):
        g = torch.Generator(device=dev).manual_seed(0)
        xs = []
        for _ in range(2):
            x = torch.randn(1, 16, S_, 128, device=dev, generator=g)
            for h in range(16):
                ch = torch.randperm(128, device=dev, generator=g)[:3]
                x[0, h][:, ch] *= 10.0
            xs.append(x)
        outs = [ops.empty_packed(x.shape, 1, False, dev) for x in xs]

        def step():
            ops.compress_many(xs, d, c, residual=False, outs=outs)

        for _ in range(3):
            step()
        torch.cuda.synchronize()
        # host cost of one API call (the GPU is idle between short launches),
        # through ops.compress_many and through the bare operator
        h0 = time.perf_counter()
        for _ in range(20):
            step()
        host_us = (time.perf_counter() - h0) / 20 * 1e6
        torch.cuda.synchronize()
        K = ops.ext()
        dh, ch = ops._host_f32(d), ops._host_f32(c)
        codes, norms = [o.code for o in outs], [o.norms for o in outs]
        h0 = time.perf_counter()
        for _ in range(20):
            K.compress_many_out(xs, dh, ch, False, codes, [], norms, [])
        op_host_us = (time.perf_counter() - h0) / 20 * 1e6
        torch.cuda.synchronize()
        per = time_loop(step, 20, stream)
        # the same launch replayed from a CUDA graph: kernel time without the
        # host's per-call work
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            step()
            with torch.cuda.graph(graph, stream=side):
                step()
        stream.wait_stream(side)
        torch.cuda.synchronize()
        gper = time_loop(graph.replay, 20, stream)
        del graph
        ms, gms = statistics.median(per), statistics.median(gper)
        rows = 2 * 16 * S_
        bpr = 128 * 4 + 128 // 8 + 4
        out[f"S{S_}"] = {"rows": rows, "us_per_step": ms * 1e3, "rows_per_s": rows / (ms / 1e3),
                         "gbs": rows * bpr / (ms / 1e3) / 1e9,
                         "frac_of_measured_hbm": rows * bpr / (ms / 1e3) / 1e9 / peak,
                         "graph_us_per_step": gms * 1e3,
                         "graph_frac_of_measured_hbm": rows * bpr / (gms / 1e3) / 1e9 / peak,
                         "host_us_per_call": host_us,
                         "op_host_us_per_call": op_host_us,
                         "l2": "fits in L2" if rows * 512 < 126e6 else "above L2"}
        del xs, outs
    return out


def layers_bench(dev, args) -> dict:
    """28-layer batched compression: per layer K and V bf16 [32, 16, 8192, 128]
    (N(0, 0.5^2) times a per-layer scale drawn from U[0.5, 2]), 56 tensors of
    4.19 M rows (60.1 GB resident) compressed in one batched launch per step,
    in 1-bit mode (code + norm, 20 B/row) and 2-bit mode (40 B/row)."""
    from kudahitam import ops
    from kudahitam.codebook import lloyd_max, rademacher
    L, Bc, Hc, Sc, Dc = 28, 32, 16, 8192, 128
    if args.seq:  # profiling: shrink S
        Sc = min(Sc, args.seq)
    scales = torch.empty(L).uniform_(0.5, 2.0, generator=torch.Generator().manual_seed(3))
    xs = []
    for l in range(L):
        g = torch.Generator(device=dev).manual_seed(3 + l)
        for _ in range(2):
            x = torch.empty(Bc, Hc, Sc, Dc, device=dev, dtype=torch.bfloat16)
            for b in range(Bc):  # fp32 temporaries one batch entry at a time
                x[b] = (torch.randn(Hc, Sc, Dc, device=dev, generator=g)
                        * (0.5 * float(scales[l]))).to(torch.bfloat16)
            xs.append(x)
    d, c = rademacher(Dc, 1), lloyd_max(1, Dc)
    rows = len(xs) * Bc * Hc * Sc
    stream = torch.cuda.current_stream(dev)
    peak, _ = peaks()
    out = {"config": f"28 layers x (K, V) bf16 [32,16,{Sc},128], one batched launch per step",
           "rows_per_step": rows, "input_gb": rows * Dc * 2 / 1e9}
    for mode, residual in (("1bit", False), ("2bit", True)):
        outs = [ops.empty_packed(x.shape, 1, residual, dev) for x in xs]

        def step():
            ops.compress_many(xs, d, c, residual=residual, outs=outs)

        for _ in range(2):
            step()
        torch.cuda.synchronize()
        per = time_loop(step, 5, stream)
        ms = statistics.median(per)
        bpr = Dc * 2 + (2 * Dc // 8 + 8 if residual else Dc // 8 + 4)
        gbs = rows * bpr / (ms / 1e3) / 1e9
        out[mode] = {"ms_per_step": ms, "rows_per_s": rows / (ms / 1e3), "gbs": gbs,
                     "frac_of_measured_hbm": gbs / peak, "bytes_per_row": bpr}
        del outs
    del xs
    torch.cuda.empty_cache()
    return out


def decode_bench(dev, args, world: int = 1, rank: int = 0) -> dict:
    """Decode step over the 40k-token compressed cache.  With N ranks the
    sequence is sharded (S/N rows per group on each rank) and the split-K
    records are merged per rank and exchanged with one NCCL all-gather; the
    time is the max over ranks (strong scaling: the total S is fixed)."""
    from kudahitam import dist as khdist
    from kudahitam import ops
    from kudahitam.codebook import lloyd_max, rademacher
    G = DEC_B * DEC_H
    a, b = khdist.shard_range(DEC_S, world, rank)
    S_loc = b - a
    g = torch.Generator(device=dev).manual_seed(5 + 7919 * rank)
    dk, dv = rademacher(DEC_D, 10), rademacher(DEC_D, 11)
    c = lloyd_max(1, DEC_D)
    pk = ops.empty_packed((G, S_loc, DEC_D), 1, True, dev)
    pv = ops.empty_packed((G, S_loc, DEC_D), 1, True, dev)
    for p, dd in ((pk, dk), (pv, dv)):
        for i in range(0, G, 64):
            x = torch.randn(64, S_loc, DEC_D, device=dev, generator=g).to(torch.bfloat16)
            ops.compress(x, dd, c, out=p.rows(i * S_loc, (i + 64) * S_loc))
    q = torch.randn(G, DEC_D, generator=torch.Generator().manual_seed(4)).to(torch.bfloat16).to(dev)
    dec = decode_timing(dev, args, world, q.float(), pk, pv, dk, dv, c, S_loc, DEC_S)
    dec["roofline"]["traffic"] = NCU_DECODE_TRAFFIC_BYTES_PER_ROW * G * DEC_S / world
    dec["roofline"]["kernel"] = "decode_v3_kernel<128> + decode_combine_kernel<128>"
    if world == 1:
        # the same decode over caches of the 4-level (bits=2) codebook: 2-bit
        # code plane, 56 B per cached row and tensor
        del pk, pv
        c2 = lloyd_max(2, DEC_D)
        g2 = torch.Generator(device=dev).manual_seed(5)
        pk = ops.empty_packed((G, S_loc, DEC_D), 2, True, dev)
        pv = ops.empty_packed((G, S_loc, DEC_D), 2, True, dev)
        for p, dd in ((pk, dk), (pv, dv)):
            for i in range(0, G, 64):
                x = torch.randn(64, S_loc, DEC_D, device=dev, generator=g2).to(torch.bfloat16)
                ops.compress(x, dd, c2, out=p.rows(i * S_loc, (i + 64) * S_loc))
        d2 = decode_timing(dev, args, world, q.float(), pk, pv, dk, dv, c2, S_loc, DEC_S,
                           bytes_per_row=2 * (DEC_D // 16 * 4 + DEC_D // 8 + 8))
        d2["roofline"]["kernel"] = "decode_b2_kernel + decode_combine_kernel<128>"
        dec["bits2_codebook"] = {k: d2[k] for k in ("us_per_step", "n_splits",
                                                    "phase_us_max_over_ranks", "roofline",
                                                    "sustained")}
        del pk, pv
    return {"config": "q bf16 [32,16,128]; K and V 2-bit-mode packed, S=40000"
                      + (f", sequence-sharded over {world} GPUs + one NCCL all-gather"
                         if world > 1 else ""),
            **dec, "us_per_token": dec["us_per_step"] / DEC_B}


CFG5_B, CFG5_H, CFG5_S, CFG5_D = 64, 16, 131072, 128
CFG5_BLOCK = 16384  # sequence rows per generated block (S / 8: every N in 1, 2, 4, 8 aligns)


def cfg5_outlier_channels() -> torch.Tensor:
    """3 outlier channels per head (scaled x10), the same for K and V and
    for every batch entry: [16, 3] from a CPU generator seeded 4."""
    g = torch.Generator().manual_seed(4)
    return torch.stack([torch.randperm(CFG5_D, generator=g)[:3] for _ in range(CFG5_H)])


def cfg5_block(dev, tensor: int, group: int, block: int, ch: torch.Tensor) -> torch.Tensor:
    """Rows [block * 16384, (block + 1) * 16384) of (batch, head) group
    `group` of K (tensor 0) or V (tensor 1) of the 8-GPU workload: bf16
    N(0, 1) with the head's 3 outlier channels x10, from a CUDA generator
    seeded by (tensor, group, block), so that every rank count generates the
    same rows."""
    seed = 4_000_000 + (tensor * CFG5_B * CFG5_H + group) * (CFG5_S // CFG5_BLOCK) + block
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(CFG5_BLOCK, CFG5_D, device=dev, generator=g)
    x[:, ch[group % CFG5_H].to(dev)] *= 10.0
    return x.to(torch.bfloat16)


def cfg5_bench(dev, args, world: int, rank: int) -> dict:
    """The 8-GPU workload: K and V bf16 [64, 16, 131072, 128] (N(0,1), 3
    outlier channels x10 per head, seeded).
    * compression sharded by batch x head (1024 groups / N per rank, no
      communication), 2-bit mode, one batched launch over the rank's K and V
      per step; weak in nothing: the total work is fixed (strong scaling);
    * decode attention over the sequence-sharded compressed cache (S / N rows
      of every group per rank, B = 64: 1024 query rows), records merged per
      rank and exchanged with one NCCL all-gather; max over ranks."""
    from kudahitam import dist as khdist
    from kudahitam import ops
    from kudahitam.codebook import lloyd_max, rademacher
    G = CFG5_B * CFG5_H
    nblk = CFG5_S // CFG5_BLOCK
    ch = cfg5_outlier_channels()
    d, c = rademacher(CFG5_D, 1), lloyd_max(1, CFG5_D)
    peak, _ = peaks()
    stream = torch.cuda.current_stream(dev)
    out = {"config": "K, V bf16 [64,16,131072,128], 3 outlier channels x10 per head; "
                     "compression sharded by batch x head, decode sequence-sharded "
                     "(strong scaling: total work fixed)"}

    # ---- compression: this rank's (batch, head) groups, whole sequences
    g0, g1 = khdist.shard_range(G, world, rank)
    xs = []
    for t in range(2):
        x = torch.empty(g1 - g0, CFG5_S, CFG5_D, device=dev, dtype=torch.bfloat16)
        for gi in range(g0, g1):
            for j in range(nblk):
                x[gi - g0, j * CFG5_BLOCK:(j + 1) * CFG5_BLOCK] = cfg5_block(dev, t, gi, j, ch)
        xs.append(x)
    outs = [ops.empty_packed(x.shape, 1, True, dev) for x in xs]

    def step():
        ops.compress_many(xs, d, c, residual=True, outs=outs)

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    barrier(world)
    n_steps = max(3, min(args.steps, 10))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(n_steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    ms_local = e0.elapsed_time(e1) / n_steps
    ms = max_over_ranks(ms_local, world)
    rows_rank = 2 * (g1 - g0) * CFG5_S
    bpr = CFG5_D * 2 + 2 * CFG5_D // 8 + 8
    out["compress"] = {
        "rows_per_step": 2 * G * CFG5_S, "rows_per_rank": rows_rank, "ms_per_step": ms,
        "rows_per_s": 2 * G * CFG5_S / (ms / 1e3),
        "frac_of_measured_hbm_per_gpu": rows_rank * bpr / (ms / 1e3) / 1e9 / peak,
        "per_rank_ms": all_ranks(ms_local, world), "steps": n_steps,
        "bytes_per_row": bpr}
    if world > 1:
        del outs
    # ---- decode: this rank's sequence shard of every group
    b0, b1 = khdist.shard_range(nblk, world, rank)
    S_loc = (b1 - b0) * CFG5_BLOCK
    if world == 1:
        pk, pv = outs
    else:
        del xs
        torch.cuda.empty_cache()
        pk = ops.empty_packed((G, S_loc, CFG5_D), 1, True, dev)
        pv = ops.empty_packed((G, S_loc, CFG5_D), 1, True, dev)
        for t, p in ((0, pk), (1, pv)):
            for gi in range(G):
                x = torch.cat([cfg5_block(dev, t, gi, j, ch) for j in range(b0, b1)])
                ops.compress(x, d, c, out=p.rows(gi * S_loc, (gi + 1) * S_loc))
    q = torch.randn(G, CFG5_D, generator=torch.Generator().manual_seed(44)).to(
        torch.bfloat16).float().to(dev)
    dec = decode_timing(dev, args, world, q, pk, pv, d, d, c, S_loc, CFG5_S)
    out["decode"] = {"config": f"q [64,16,128] vs K, V 2-bit-mode packed, S=131072"
                               f"{f', {S_loc} rows per group on each of {world} GPUs' if world > 1 else ''}",
                     **dec, "us_per_token": dec["us_per_step"] / CFG5_B}
    out["gpus_active"] = world
    del pk, pv
    if world == 1:
        del xs, outs
    torch.cuda.empty_cache()
    return out


def decode_timing(dev, args, world, q, pk, pv, dk, dv, c, S_loc, S_total,
                  bytes_per_row: int = None) -> dict:
    """Times decode attention (q [R, D] against R groups of S_loc cached rows
    on this rank; S_total over all ranks): whole steps, each phase on its
    own (partial kernel, local merge, NCCL all-gather, combine), the
    peer-memory exchanges (N > 1), and whole steps again after half a second
    of back-to-back steps (`sustained`, with the SM clock of that window);
    every time the max over ranks of the median of CUDA-event timings."""
    from kudahitam import dist as khdist
    from kudahitam import ops
    R, D = q.shape
    n_splits = ops.default_splits(R, S_loc, dev)
    stream = torch.cuda.current_stream(dev)
    sm = 1 / math.sqrt(D)
    rec = D + 2
    buf = torch.empty(khdist.seq_sharded_workspace_numel(R, n_splits, world, D), device=dev)
    outp = torch.empty(R, D, device=dev)
    local = buf[: R * n_splits * rec].view(R, n_splits, rec)
    off = R * n_splits * rec
    if world > 1:
        merged = buf[off: off + R * rec].view(R, rec)
        gathered = buf[off + R * rec: off + R * rec * (1 + world)].view(world, R, rec)

    def step():
        return khdist.decode_attention_seq_sharded(q, pk, pv, dk, dv, c, sm, n_splits,
                                                   partials=buf)

    phases = {
        "partial": lambda: ops.decode_partial(q, pk, pv, dk, dv, c, sm, n_splits, local,
                                              n_splits, 0, S_loc),
    }
    if world > 1:
        phases["merge"] = lambda: ops.decode_merge(local, merged)
        phases["all_gather"] = lambda: khdist.gather_records(merged, out=gathered)
        phases["combine"] = lambda: ops.decode_combine_records(gathered.transpose(0, 1), dv, outp)
    else:
        phases["combine"] = lambda: ops.decode_combine(local, n_splits, dv, outp)
    # One idle second first: right after the 8-GPU workload's compression
    # (at the power cap) the first decode steps ran up to 40 % slower than
    # the same steps a second later.  Then two figures:
    # * us_per_step: ten warm-up steps, then n timed steps (a few ms of load),
    #   followed by each phase alone and the peer-memory variants, all in the
    #   same few-ms state;
    # * sustained, last: after at least half a second of back-to-back steps, when
    #   the power limit has lowered the SM clock (sw_power_cap), with the SM
    #   clock sampled in that window.  The warm-up step count comes from three
    #   timed steps and is the max over ranks, so every rank runs the same
    #   number of collectives.
    torch.cuda.synchronize()
    time.sleep(1.0)
    barrier(world)
    for _ in range(max(10, args.warmup)):
        step()
    torch.cuda.synchronize()
    barrier(world)
    n = max(5, min(args.steps, 20))
    ms = max_over_ranks(statistics.median(time_loop(step, n, stream)), world)
    phase_us = {}
    for name, fn in phases.items():
        barrier(world)
        phase_us[name] = max_over_ranks(statistics.median(time_loop(fn, n, stream)), world) * 1e3
    peer = None
    if world > 1:
        # the same step with the records exchanged inside the merge kernel
        # over peer (symmetric) memory instead of the NCCL all-gather
        ex = khdist.PeerRecordExchange(R, D, device=dev)

        def step_peer():
            return khdist.decode_attention_seq_sharded(q, pk, pv, dk, dv, c, sm, n_splits,
                                                       partials=buf, exchange=ex)

        for _ in range(3):
            step_peer()
        torch.cuda.synchronize()
        khdist.check_peer_timeout(dev)
        barrier(world)
        pms = max_over_ranks(statistics.median(time_loop(step_peer, n, stream)), world)
        torch.cuda.synchronize()
        khdist.check_peer_timeout(dev)
        barrier(world)
        del ex
        # the exchange fused into the partial kernel: its CTAs store their
        # split records into every rank's buffer and merge the rows once all
        # flags arrived (one kernel per step when the launch fits at once)
        exf = khdist.PeerRecordExchange(R, D, device=dev, n_parts=n_splits)

        def step_fused():
            return khdist.decode_attention_seq_sharded(q, pk, pv, dk, dv, c, sm, n_splits,
                                                       partials=buf, exchange=exf)

        for _ in range(3):
            step_fused()
        torch.cuda.synchronize()
        khdist.check_peer_timeout(dev)
        barrier(world)
        fms = max_over_ranks(statistics.median(time_loop(step_fused, n, stream)), world)
        torch.cuda.synchronize()
        khdist.check_peer_timeout(dev)
        barrier(world)
        del exf
        peer = {"us_per_step": pms * 1e3,
                "note": "kh_decode_merge_to_peers + kh_decode_combine_from_peers (plain "
                        "stores to every rank's symmetric buffer, epoch flags) in place of "
                        "merge + NCCL all-gather + combine",
                "fused_in_partial_us_per_step": fms * 1e3,
                "fused_note": "kh_decode_partial_to_peers with out: the partial kernel stores "
                              "its split records to every rank and merges the rows itself"}
    t3 = statistics.median(time_loop(step, 3, stream))
    n_warm = int(max_over_ranks(float(math.ceil(500.0 / max(t3, 1e-3))), world))
    with ClockSampler(torch.cuda.current_device(), period_s=0.002) as clk:
        for i in range(n_warm):
            step()
            if i % 50 == 49:
                torch.cuda.synchronize()
        torch.cuda.synchronize()
        barrier(world)
        t0 = time.perf_counter()
        ms_sus = max_over_ranks(statistics.median(time_loop(step, n, stream)), world)
        clk.mark_region(t0, time.perf_counter())
    sustained = {"us_per_step": ms_sus * 1e3, "warmup_steps": n_warm,
                 "clocks": clk.summary()}
    if bytes_per_row is None:
        bytes_per_row = 2 * (2 * D // 8 + 8)  # K and V: 2 one-bit planes + 2 norms each
    bytes_step = R * S_total * bytes_per_row  # whole job
    peak, _ = peaks()
    per_gpu = bytes_step / world / (ms / 1e3) / 1e9
    return {"us_per_step": ms * 1e3, "n_splits": n_splits, "rows_per_group_per_gpu": S_loc,
            "scaling": "strong" if world > 1 else None,
            "phase_us_max_over_ranks": phase_us, "peer_exchange": peer,
            "gbs": bytes_step / (ms / 1e3) / 1e9,
            "frac_of_measured_hbm_per_gpu": per_gpu / peak,
            "roofline": {"bound": "hbm", "achieved": per_gpu, "peak": peak, "unit": "GB/s",
                         "frac": per_gpu / peak, "algorithmic_bytes": bytes_step / world},
            "sustained": {**sustained,
                          "frac_of_measured_hbm_per_gpu":
                              bytes_step / world / (ms_sus / 1e3) / 1e9 / peak}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["engine", "reference"], default="engine")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-layers", action="store_true",
                    help="skip the 28-layer batched compression line (60 GB resident)")
    ap.add_argument("--no-cfg5", action="store_true",
                    help="skip the 8-GPU workload line (K, V bf16 [64,16,131072,128])")
    ap.add_argument("--only", choices=["all", "compress", "decode", "layers", "fp32", "score",
                                       "cfg5", "compat"], default="all",
                    help="run one part (small cases for profiler captures)")
    ap.add_argument("--seq", type=int, default=None,
                    help="override S of the compression workload (profiling only)")
    args = ap.parse_args()
    if args.seq:
        global S, ROWS_PER_TENSOR
        S = args.seq
        ROWS_PER_TENSOR = B * H * S
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, world, rank)
        return
    world, rank, local = dist_setup(args)
    try:
        run_engine(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
