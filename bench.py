"""Benchmark of the quantized GEMV path on B200.

Workload (the large low-bit configuration): y = x . W^T for one
W[28672 x 8192] in each of Q2_K, Q3_K and Q5_K (weights ~ N(0, 0.02^2) plus
0.1% outliers ~ N(0, 0.5^2), packed by this library), x[1 x 8192] ~ N(0,1).
One decode pass = the three GEMVs; one step = --passes decode passes (256 by
default, so the timed region lasts about half a second on one GPU).  With N
GPUs the same matrices are row-sharded (strong scaling): rank r holds rows
[r*28672/N, (r+1)*28672/N) of each and its GEMV epilogue stores its output
rows straight into every rank's copy of the full output over NVLink
(symmetric buffers, no separate collective).  The three packed matrices
(340 MB) exceed the 126 MB L2, so consecutive passes read them from HBM.

Metric: packed-weight GB/s of the whole job (higher is better).  On one GPU
the line also carries the batched GEMM (M = 128 tokens, TFLOP/s) and the
pack sweep (2^30 elements, GB/s read), each with its roofline and the
reference's CPU figure.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--passes P] [--impl reference]

Under torchrun (N > 1) every rank runs; rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

ROWS, K_DIM, M_TOK = 28672, 8192, 1
FORMATS = ("Q2_K", "Q3_K", "Q5_K")
PASSES = 320
GEMM_TOKENS = 128
METRIC = "Quant matmul weight GB/s (GEMV), TOPS (GEMM) at 1/2/4/8 B200 vs AVX2 host"
WORKLOAD = ("low-bit large GEMV: y = x.W^T, W[28672x8192] in Q2_K, Q3_K, Q5_K, x[1x8192], rows sharded "
            "across the GPUs")


def packed_bytes(fmt: str, rows: int = ROWS, cols: int = K_DIM) -> int:
    be = 32 if fmt in ("Q8_0", "Q4_0") else 256
    bb = {"Q8_0": 34, "Q4_0": 18, "Q2_K": 84, "Q3_K": 110, "Q4_K": 144, "Q5_K": 176, "Q6_K": 210}[fmt]
    return rows * ((cols + be - 1) // be) * bb


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d.get("hbm_gbs", 6650.0)), "measured"
    return 6650.0, "fallback"


def load_traffic(fmt: str):
    """dram bytes (read + write) per launch of the format's GEMV kernel from
    the committed ncu summary (profiles/traffic.json), or None."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        try:
            with open(p) as f:
                return json.load(f).get(f"gemv_{fmt}")
        except Exception:
            return None
    return None


class ClockSampler:
    """nvidia-smi clock/throttle samples taken during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for n, v in zip(names, r[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(rows)}


# ------------------------------------------------------------------ CPU arms

def cpu_pack_reference(fmt, W, threads):
    import oracle
    ref = oracle.ref()
    out = np.empty(packed_bytes(fmt, W.shape[0], W.shape[1]), dtype=np.uint8)
    if ref is not None:
        rc = ref.lib.ref_quantize_threads(oracle.FORMATS[fmt], W.ctypes.data, W.shape[0], W.shape[1],
                                          out.ctypes.data, threads)
        if rc != 0:
            raise RuntimeError("reference quantize failed")
        return out
    return oracle.orc().quantize(fmt, W)


def make_weights_np(fmt_index, rows, cols, seed):
    rng = np.random.default_rng(seed + fmt_index)
    W = (rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02))
    m = rng.random((rows, cols), dtype=np.float32) < 0.001
    W[m] = rng.standard_normal(int(m.sum()), dtype=np.float32) * np.float32(0.5)
    return W


class CpuArm:
    """The reference's CPU matmul on the host cores: its own kernels compiled
    from its sources (oracle/_ref, kind "reference"), or the C restatement
    (kind "port") where that library is absent.  Rows are split across all
    host threads (the reference kernels are single-threaded)."""

    def __init__(self, packed, x, threads):
        import oracle
        self.threads = threads
        self.ref = oracle.ref()
        self.kind = "reference" if self.ref is not None else "port"
        self.jobs = []
        self.bytes = 0
        for fmt, q, rows in packed:
            self.bytes += q.size
            if self.ref is not None:
                self.jobs.append(oracle.MatmulJob(self.ref, fmt, q, x, rows, K_DIM, threads))
            else:
                self.jobs.append((fmt, q, rows))
        self.x = x

    def step(self):
        import concurrent.futures as cf
        import oracle
        if self.ref is not None:
            for j in self.jobs:
                j.run()
            return
        orc = oracle.orc()
        for fmt, q, rows in self.jobs:
            out = np.empty((rows, self.x.shape[1]), dtype=np.float32)
            with cf.ThreadPoolExecutor(self.threads) as ex:
                chunks = [(rows * t // self.threads, rows * (t + 1) // self.threads) for t in range(self.threads)]
                list(ex.map(lambda c: orc.matmul_rows(fmt, q, self.x, out, rows, K_DIM, c[0], c[1]), chunks))

    def close(self):
        if self.ref is not None:
            for j in self.jobs:
                j.close()


def bench_config(world: int) -> dict:
    """The workload's config, identical in both arms."""
    return {"workload": WORKLOAD, "rows": ROWS, "K": K_DIM, "M": M_TOK, "formats": list(FORMATS),
            "parallelism": (f"row-shard x{world} ({ROWS // world} rows per GPU), outputs stored into every "
                            "rank's copy by the GEMV epilogue over NVLink") if world > 1 else "single GPU",
            "l2": "inputs larger than L2 (340 MB of packed weights per pass)"}


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    rows = ROWS
    x = np.random.default_rng(2).standard_normal((K_DIM, M_TOK), dtype=np.float32)
    packed = []
    for i, fmt in enumerate(FORMATS):
        W = make_weights_np(i, rows, K_DIM, 9)
        packed.append((fmt, cpu_pack_reference(fmt, W, threads), rows))
        del W
    arm = CpuArm(packed, x, threads)
    for _ in range(args.warmup):
        arm.step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        arm.step()
    dt = (time.perf_counter() - t0) / args.steps
    arm.close()
    gbs = arm.bytes / dt / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 4), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": bench_config(world),
        "step": {"passes": 1, "what": "one decode pass (the three GEMVs over all 28672 rows) per step on the host"},
        "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": threads, "kind": arm.kind,
                         "sample": f"one pass per step: {len(FORMATS)} GEMVs over all {rows} rows"},
        "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ GPU arm

def _graph(fn, reps):
    """fn() captured `reps` times in one CUDA graph, or None if capture fails."""
    import torch
    try:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, capture_error_mode="thread_local"):
            for _ in range(reps):
                fn()
        return graph
    except Exception as exc:
        print(f"graph capture failed, timing eagerly: {exc}", file=sys.stderr)
        torch.cuda.synchronize()
        return None


def run_gpu(args):
    import torch
    import torch.distributed as dist
    import axon_b200 as ax

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    if ROWS % world:
        raise SystemExit(f"{ROWS} rows do not split over {world} GPUs")
    rows_l = ROWS // world
    r0 = rank * rows_l
    passes = args.passes

    # The one matrix per format (same seed on every rank, so the shards are
    # the rows of one weight), this rank's rows packed by our quantize kernel.
    g = torch.Generator(device=dev).manual_seed(9)
    qs = {}
    for fmt in FORMATS:
        W = torch.randn(ROWS, K_DIM, device=dev, generator=g) * 0.02
        m = torch.rand(ROWS, K_DIM, device=dev, generator=g) < 0.001
        W[m] = torch.randn(int(m.sum().item()), device=dev, generator=g) * 0.5
        del m
        qt = ax.QTensor.empty(rows_l, K_DIM, ax.QuantFormat[fmt], device=dev)
        ax.quantize(qt, W[r0:r0 + rows_l].contiguous(), ax.QuantFormat[fmt])
        del W
        qs[fmt] = qt
    torch.cuda.synchronize()
    xg = torch.Generator(device=dev).manual_seed(2)
    x = torch.randn(M_TOK, K_DIM, device=dev, generator=xg)
    comm = ax.Communicator.from_process_group() if world > 1 else None
    # one GPU: the three outputs in one buffer (one read-back); several: one
    # symmetric buffer per format holding the full output on every rank
    y_all = torch.empty(len(FORMATS), M_TOK, ROWS, device=dev)
    ys = {f: y_all[i] for i, f in enumerate(FORMATS)}
    symm = {f: ax.SymmetricBuffer(comm, 4 * ROWS * M_TOK) for f in FORMATS} if world > 1 else None
    ws = ax.Workspace()
    stream = torch.cuda.current_stream()

    def run_fmt(fmt, q=None, xin=None):
        q = qs[fmt] if q is None else q
        xin = x if xin is None else xin
        if world > 1:
            ax.matmul_sharded_p2p(symm[fmt], q, xin, ROWS, b_tokmajor=True, workspace=ws, wait=False)
        else:
            ax.linear_q(xin, q, out=ys[fmt], workspace=ws)

    def wait_fmt(fmt):
        if world > 1:
            symm[fmt].wait()

    def wait_all():
        if world > 1:
            ax.wait_all([symm[f] for f in FORMATS])

    def one_pass():
        # the three matmuls back to back, then their completion waits (one kernel)
        for fmt in FORMATS:
            run_fmt(fmt)
        wait_all()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    # a step is `passes` decode passes: graphs of `chunk` passes, replayed
    chunk = 16 if passes % 16 == 0 else 1
    for _ in range(3):
        one_pass()
    barrier()
    g_chunk = _graph(one_pass, chunk)
    replay = (lambda: g_chunk.replay()) if g_chunk is not None else one_pass
    n_replay = passes // chunk if g_chunk is not None else passes

    def step():
        for _ in range(n_replay):
            replay()

    for _ in range(max(args.warmup, 3)):
        step()
    barrier()

    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    barrier()
    t0.record(stream)
    for _ in range(args.steps):
        step()
    t1.record(stream)
    barrier()
    ms = t0.elapsed_time(t1) / args.steps
    clocks = sampler.stop() if sampler else None

    # Each format's matmul alone (prep + GEMV, plus the peer wait on several
    # GPUs), 16 calls per graph over enough weight copies (> 2x L2) that no
    # call finds its weights in L2: the per-launch duration of the roofline.
    fmt_ms = {}
    for f in FORMATS:
        nb = packed_bytes(f, rows_l)
        ncopy = max(2, -(-(300 << 20) // nb) + 1)
        copies = [qs[f]] + [ax.QTensor(qs[f].data.clone(), qs[f].shape, qs[f].fmt) for _ in range(ncopy - 1)]
        it = [0]

        def one(f=f, copies=copies, it=it):
            run_fmt(f, q=copies[it[0] % len(copies)])
            wait_fmt(f)
            it[0] += 1

        for _ in range(3):
            one()
        barrier()
        gf = _graph(one, 16)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        reps = max(4, min(64, int(200.0 / max(ms / passes, 1e-3) / 16)))
        barrier()
        e0.record(stream)
        for _ in range(reps):
            if gf is not None:
                gf.replay()
            else:
                for _ in range(16):
                    one()
        e1.record(stream)
        barrier()
        fmt_ms[f] = e0.elapsed_time(e1) / (16 * reps)
        del gf, copies
    torch.cuda.empty_cache()

    # End to end through the public API with host buffers: every pass copies
    # x from pinned host memory, runs the three matmuls and their waits, and
    # copies the three full outputs back to pinned host memory; `chunk`
    # passes are captured in one CUDA graph (the copies are graph nodes).
    xh = torch.randn(M_TOK, K_DIM).pin_memory()
    yh = torch.empty(len(FORMATS) * M_TOK * ROWS).pin_memory()
    xd = torch.empty_like(x)

    def e2e_pass():
        xd.copy_(xh, non_blocking=True)
        for fmt in FORMATS:
            run_fmt(fmt, xin=xd)
        wait_all()
        if world > 1:
            for i, f in enumerate(FORMATS):
                yh[i * ROWS * M_TOK:(i + 1) * ROWS * M_TOK].copy_(symm[f].tensor((ROWS * M_TOK,)), non_blocking=True)
        else:
            yh.copy_(y_all.view(-1), non_blocking=True)

    for _ in range(3):
        e2e_pass()
    barrier()
    g_e2e = _graph(e2e_pass, chunk)
    e2e_replay = (lambda: g_e2e.replay()) if g_e2e is not None else e2e_pass
    e2e_n = passes // chunk if g_e2e is not None else passes
    for _ in range(2):
        for _ in range(e2e_n):
            e2e_replay()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        for _ in range(e2e_n):
            e2e_replay()
    e1.record(stream)
    barrier()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    del g_chunk, g_e2e  # graphs go before the communicator
    if world > 1:
        t = torch.tensor([ms, e2e_ms] + [fmt_ms[f] for f in FORMATS], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms = float(t[0]), float(t[1])
        fmt_ms = {f: float(t[2 + i]) for i, f in enumerate(FORMATS)}

    total_w = sum(packed_bytes(f) for f in FORMATS) * passes
    value = total_w / (ms / 1e3) / 1e9
    e2e_val = total_w / (e2e_ms / 1e3) / 1e9
    peak, peak_kind = load_peaks()
    # Roofline of each format's matmul on one GPU's rows: algorithmic bytes
    # (packed weights + fp32 activations read + fp32 outputs written) / its
    # event-timed duration; the reported kernel has the largest share.
    by_fmt = {}
    for f in FORMATS:
        alg = packed_bytes(f, rows_l) + 4 * K_DIM * M_TOK + 4 * rows_l * M_TOK
        ach = alg / (fmt_ms[f] / 1e3) / 1e9
        by_fmt[f] = {"achieved": round(ach, 1), "frac": round(ach / peak, 4), "ms_per_launch": round(fmt_ms[f], 5),
                     "algorithmic_bytes": alg, "traffic": load_traffic(f) if world == 1 else None}
    dom = max(FORMATS, key=lambda f: fmt_ms[f])
    line = None
    if rank == 0:
        extra = {}
        if world == 1 and not args.no_extras:
            extra["gemm"] = gemm_record(qs, ws, peak)
            extra["pack"] = pack_record(peak)
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline(qs, x)
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "int8-dp4a/f32-acc", "data": "synthetic",
            "config": bench_config(world),
            "step": {"passes": passes, "what": "decode passes (the three GEMVs) per step; graphs of "
                                               f"{chunk} passes replayed"},
            "roofline": {"bound": "hbm", "achieved": by_fmt[dom]["achieved"], "peak": peak, "unit": "GB/s",
                         "frac": by_fmt[dom]["frac"], "peak_source": peak_kind,
                         "kernel": f"matmul {dom} (act prep + gemv), largest share of the step",
                         "ms_per_launch": by_fmt[dom]["ms_per_launch"], "traffic": by_fmt[dom]["traffic"],
                         "by_format": by_fmt},
            "e2e": {"value": round(e2e_val, 2), "unit": "GB/s", "h2d_bytes_per_step": 4 * K_DIM * M_TOK * passes,
                    "d2h_bytes_per_step": 4 * M_TOK * ROWS * len(FORMATS) * passes,
                    "how": "public API per pass (linear_q / matmul_sharded_p2p) with the pinned-host copies, "
                           f"{chunk} passes per CUDA graph"},
            # per matmul: activation prep + GEMV; with several ranks one wait per pass
            "gpu_launches": (2 * len(FORMATS) + (1 if world > 1 else 0)) * passes * args.steps,
            "clocks": clocks,
        }
        line.update(extra)
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()
        for b in symm.values():
            b.destroy()
        comm.destroy()
        dist.barrier()
        dist.destroy_process_group()
    return 0


def gemm_record(qs, ws, peak_hbm):
    """Batched GEMM on the same matrices: X[128 x 8192] . W^T for each format
    (tensor-core path), 16 calls per CUDA graph over rotating weight copies;
    TFLOP/s = 2*M*N*K / time against the measured dense bf16 peak (the MMA
    is kind::f16 with fp16 operands, whose dense rate equals bf16's); beside
    it the reference's CPU matmul at 128 tokens on a row sample."""
    import torch
    import axon_b200 as ax
    dev = qs[FORMATS[0]].data.device
    n = GEMM_TOKENS
    mp = os.path.join(ROOT, "MEASURED_PEAKS.json")
    tpk = json.load(open(mp)).get("bf16_tflops") if os.path.exists(mp) else None
    tkind = "measured (cuBLAS bf16, burst)" if tpk else "fallback"
    tpk = float(tpk or 1590.0)
    X = torch.randn(n, K_DIM, device=dev, generator=torch.Generator(device=dev).manual_seed(12))
    Y = torch.empty(n, ROWS, device=dev)
    by = {}
    for f in FORMATS:
        nb = packed_bytes(f)
        copies = [qs[f]] + [ax.QTensor(qs[f].data.clone(), qs[f].shape, qs[f].fmt)
                            for _ in range(max(1, -(-(300 << 20) // nb)))]
        it = [0]

        def one(copies=copies, it=it):
            ax.linear_q(X, copies[it[0] % len(copies)], out=Y, workspace=ws)
            it[0] += 1

        for _ in range(3):
            one()
        torch.cuda.synchronize()
        gr = _graph(one, 16)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(8):
            gr.replay() if gr is not None else [one() for _ in range(16)]
        e1.record()
        torch.cuda.synchronize()
        t = e0.elapsed_time(e1) / (8 * 16)
        by[f] = {"ms": round(t, 5), "tflops": round(2.0 * n * ROWS * K_DIM / (t / 1e3) / 1e12, 1)}
        del gr, copies
    torch.cuda.empty_cache()
    dom = max(FORMATS, key=lambda f: by[f]["ms"])
    ach = by[dom]["tflops"]
    rec = {"workload": f"batched GEMM: Y = X.W^T, W[28672x8192] in Q2_K, Q3_K, Q5_K, X[{n}x8192]",
           "unit": "TFLOP/s", "value": round(sum(2.0 * n * ROWS * K_DIM for _ in FORMATS) /
                                          (sum(by[f]["ms"] for f in FORMATS) / 1e3) / 1e12, 1),
           "by_format": by,
           "roofline": {"bound": "tensor", "achieved": ach, "peak": tpk, "unit": "TFLOP/s",
                        "frac": round(ach / tpk, 4), "peak_source": tkind,
                        "kernel": f"matmul {dom} (fp16 activation tiles + tcgen05 GEMM kind::f16)",
                        "traffic": None}}
    # the reference's CPU matmul (its kernels re-decode each weight row for
    # every token column) on 1/64 of the rows, all host threads
    try:
        import oracle
        ref = oracle.ref()
        threads = os.cpu_count() or 1
        rows = ROWS // 64
        xn = X.t().contiguous().cpu().numpy()
        flops, secs = 0.0, 0.0
        for f in FORMATS:
            qn = qs[f].data[: rows * packed_bytes(f, 1)].cpu().numpy()
            if ref is not None:
                job = oracle.MatmulJob(ref, f, qn, xn, rows, K_DIM, threads)
                t0 = time.perf_counter()
                job.run()
                secs += time.perf_counter() - t0
                job.close()
            else:
                t0 = time.perf_counter()
                oracle.orc().matmul(f, qn, xn, rows, K_DIM)
                secs += time.perf_counter() - t0
            flops += 2.0 * n * rows * K_DIM
        rec["cpu_baseline"] = {"value": round(flops / secs / 1e12, 6), "unit": "TFLOP/s",
                               "cores": threads if ref is not None else 1,
                               "kind": "reference" if ref is not None else "port",
                               "sample": f"{rows} of {ROWS} rows x {n} tokens, each format once"}
    except Exception as exc:  # the baseline is reported, never required
        rec["cpu_baseline"] = {"unavailable": str(exc)[:200]}
    return rec


def pack_record(peak_hbm):
    """Pack sweep at 2^30 fp32 elements ([262144 x 4096], N(0,1) with 1%
    U(-50, 50)) into all seven formats: GB/s of fp32 read per format; the
    roofline is the slowest format's (fp32 read + packed bytes written) /
    time against measured HBM; beside it the reference's cpu::quantize on
    2^24 elements per format over all host threads."""
    import torch
    import axon_b200 as ax
    dev = torch.device("cuda", torch.cuda.current_device())
    rows, cols = 1 << 18, 4096
    n = rows * cols
    g = torch.Generator(device=dev).manual_seed(11)
    src = torch.randn(rows, cols, device=dev, generator=g)
    m = torch.rand(rows, cols, device=dev, generator=g) < 0.01
    src[m] = torch.rand(int(m.sum().item()), device=dev, generator=g) * 100 - 50
    del m
    fmts = ("Q8_0", "Q4_0", "Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K")
    by = {}
    for f in fmts:
        F = ax.QuantFormat[f]
        dst = torch.empty(ax.quantized_size_2d(rows, cols, F), dtype=torch.uint8, device=dev)
        for _ in range(2):
            ax.quantize(dst, src, F)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(5):
            ax.quantize(dst, src, F)
        e1.record()
        torch.cuda.synchronize()
        t = e0.elapsed_time(e1) / 5
        by[f] = {"ms": round(t, 4), "read_GBps": round(4.0 * n / (t / 1e3) / 1e9, 1),
                 "hbm_frac": round((4.0 * n + dst.numel()) / (t / 1e3) / 1e9 / peak_hbm, 4),
                 "bytes": int(4 * n + dst.numel())}
        del dst
    sample = src[: (1 << 24) // cols].cpu().numpy()
    del src
    torch.cuda.empty_cache()
    dom = max(fmts, key=lambda f: by[f]["ms"])
    ach = by[dom]["bytes"] / (by[dom]["ms"] / 1e3) / 1e9
    peak, kind = load_peaks()
    rec = {"workload": "pack sweep: 2^30 fp32 elements (rows of 4096) into all seven formats", "unit": "GB/s",
           "value": round(4.0 * n * len(fmts) / (sum(by[f]["ms"] for f in fmts) / 1e3) / 1e9, 1),
           "value_is": "fp32 GB/s read over the sweep", "by_format": by,
           "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
                        "frac": round(ach / peak, 4), "peak_source": kind, "kernel": f"pack_kernel {dom}",
                        "traffic": None}}
    try:
        threads = os.cpu_count() or 1
        secs = 0.0
        for f in fmts:
            t0 = time.perf_counter()
            cpu_pack_reference(f, sample, threads)
            secs += time.perf_counter() - t0
        import oracle
        rec["cpu_baseline"] = {"value": round(4.0 * sample.size * len(fmts) / secs / 1e9, 3), "unit": "GB/s",
                               "cores": threads, "kind": "reference" if oracle.ref() is not None else "port",
                               "sample": "2^24 elements of the same tensor, each format once"}
    except Exception as exc:
        rec["cpu_baseline"] = {"unavailable": str(exc)[:200]}
    return rec


def cpu_baseline(qs, x):
    """Reference CPU path (rank 0, N=1) on a bounded sample: the pass's
    three GEMVs over 1/4 of the rows, with all host threads, ~10 s."""
    rows = ROWS // 4
    threads = os.cpu_count() or 1
    xn = x.t().contiguous().cpu().numpy()  # reference B layout [K x N]
    packed = []
    for fmt in FORMATS:
        rb = packed_bytes(fmt, 1)
        packed.append((fmt, qs[fmt].data[: rows * rb].cpu().numpy(), rows))
    arm = CpuArm(packed, xn, threads)
    arm.step()
    n, t0 = 0, time.perf_counter()
    while True:
        arm.step()
        n += 1
        dt = time.perf_counter() - t0
        if dt > 10.0 or n >= 50:
            break
    arm.close()
    return {"value": round(arm.bytes * n / dt / 1e9, 4), "unit": "GB/s", "cores": threads, "kind": arm.kind,
            "sample": f"{n} passes of {len(FORMATS)} GEMVs over {rows} of {ROWS} rows"}


# ------------------------------------------------------------------ suite

def run_suite(args):
    """Every configuration of the quantized path on one GPU, one JSON line
    each (not the driver's headline line).  Weights ~ N(0, 0.02^2) (C4 with
    0.1% outliers ~ N(0, 0.5^2)), activations ~ N(0,1); enough weight copies
    are rotated that each timed pass streams > 2x the 126 MB L2."""
    import torch
    import axon_b200 as ax

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(5)
    ws = ax.Workspace()
    peak, _ = load_peaks()
    mp = os.path.join(ROOT, "MEASURED_PEAKS.json")
    bf16_peak = json.load(open(mp)).get("bf16_tflops", 1663.3) if os.path.exists(mp) else 1590.0

    def weights(rows, cols, fmt, outliers=False):
        F = ax.QuantFormat[fmt]
        W = torch.randn(rows, cols, device=dev, generator=g) * 0.02
        if outliers:
            m = torch.rand(rows, cols, device=dev, generator=g) < 0.001
            W[m] = torch.randn(int(m.sum().item()), device=dev, generator=g) * 0.5
        q = ax.QTensor.empty(rows, cols, F, device=dev)
        ax.quantize(q, W, F)
        return q

    def copies(rows, cols, fmt, outliers=False):
        nbytes = ax.quantized_size_2d(rows, cols, ax.QuantFormat[fmt])
        n = max(1, -(-(300 << 20) // nbytes))
        base = weights(rows, cols, fmt, outliers)
        out = [base]
        for _ in range(n - 1):
            out.append(ax.QTensor(base.data.clone(), base.shape, base.fmt))
        return out

    def time_calls(fn, n_iter):
        for i in range(3):
            fn(i)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(n_iter):
            fn(i)
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n_iter

    def time_graph(fn, n_iter, replays=5):
        """Per-call time with the n_iter calls captured once in a CUDA graph
        and replayed (no host launch cost); None if capture fails."""
        for i in range(3):
            fn(i)
        torch.cuda.synchronize()
        try:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, capture_error_mode="thread_local"):
                for i in range(n_iter):
                    fn(i)
            graph.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(replays):
                graph.replay()
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / (replays * n_iter)
            del graph
            return ms
        except Exception as exc:  # capture unsupported: report eager timing only
            print(f"graph capture failed: {exc}", file=sys.stderr)
            torch.cuda.synchronize()
            return None

    def emit(d):
        print(json.dumps(d), flush=True)

    # C1, C2, C4: matmuls
    cases = [("C1", "Q8_0", 4096, 4096, [1], False), ("C2", "Q4_0", 4096, 4096, [1, 16, 64, 256, 512], False)]
    for fmt in ("Q2_K", "Q3_K", "Q5_K"):
        cases.append(("C4", fmt, 28672, 8192, [1, 8, 128], True))
    for cfg, fmt, rows, K, Ms, outl in cases:
        qs = copies(rows, K, fmt, outl)
        for M in Ms:
            x = torch.randn(M, K, device=dev, generator=g)
            y = torch.empty(M, rows, device=dev)
            call = (lambda i, x=x, y=y, qs=qs: ax.linear_q(x, qs[i % len(qs)], out=y, workspace=ws))
            ms_eager = time_calls(call, 20)
            ms_graph = time_graph(call, 20)
            ms = ms_graph if ms_graph is not None else ms_eager
            wbytes = ax.quantized_size_2d(rows, K, ax.QuantFormat[fmt])
            gbs = (wbytes + 4 * K * M + 4 * rows * M) / (ms / 1e3) / 1e9
            tops = 2.0 * rows * K * M / (ms / 1e3) / 1e12
            emit({"config": cfg, "format": fmt, "rows": rows, "K": K, "M": M, "ms": round(ms, 5),
                  "timing": "cuda-graph replay" if ms_graph is not None else "eager",
                  "eager_ms": round(ms_eager, 5),
                  "weight_GBps": round(wbytes / (ms / 1e3) / 1e9, 1), "algo_GBps": round(gbs, 1),
                  "hbm_frac": round(gbs / peak, 3), "TOPS": round(tops, 2),
                  "bf16_peak_frac": round(tops / bf16_peak, 3)})
        del qs

    # C3: MLP block y = W_down . (SiLU(X W_gate^T) * (X W_up^T))
    up = copies(11008, 4096, "Q4_K")
    gate = copies(11008, 4096, "Q4_K")
    down = copies(4096, 11008, "Q6_K")
    for M in (1, 32):
        x = torch.randn(M, 4096, device=dev, generator=g)
        yo = torch.empty(M, 4096, device=dev)

        def mlp(i, x=x, yo=yo):
            # fused gate/up pass (silu * product in the epilogue), then W_down
            ax.mlp_q(x, gate[i % len(gate)], up[i % len(up)], down[i % len(down)], out=yo, workspace=ws)

        ms_eager = time_calls(mlp, 20)
        ms_graph = time_graph(mlp, 20)
        ms = ms_graph if ms_graph is not None else ms_eager
        wbytes = 2 * ax.quantized_size_2d(11008, 4096, ax.QuantFormat.Q4_K) + \
            ax.quantized_size_2d(4096, 11008, ax.QuantFormat.Q6_K)
        emit({"config": "C3", "format": "Q4_K+Q6_K MLP", "M": M, "ms": round(ms, 5),
              "timing": "cuda-graph replay" if ms_graph is not None else "eager", "eager_ms": round(ms_eager, 5),
              "weight_GBps": round(wbytes / (ms / 1e3) / 1e9, 1),
              "TOPS": round(3 * 2.0 * 11008 * 4096 * M / (ms / 1e3) / 1e12, 2)})

    # C5: pack sweep (fp32 read GB/s)
    for p in (20, 24, 27, 30):
        n = 1 << p
        src = torch.randn(n // 4096, 4096, device=dev, generator=g)
        m = torch.rand(n // 4096, 4096, device=dev, generator=g) < 0.01
        src[m] = torch.rand(int(m.sum().item()), device=dev, generator=g) * 100 - 50
        del m
        for fmt in ("Q8_0", "Q4_0", "Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K"):
            F = ax.QuantFormat[fmt]
            dst = torch.empty(ax.quantized_size_2d(n // 4096, 4096, F), dtype=torch.uint8, device=dev)
            ms = time_calls(lambda i: ax.quantize(dst, src, F), 5 if p >= 27 else 20)
            emit({"config": "C5", "format": fmt, "elements": n, "ms": round(ms, 4),
                  "read_GBps": round(4 * n / (ms / 1e3) / 1e9, 1),
                  "hbm_frac": round((4 * n + dst.numel()) / (ms / 1e3) / 1e9 / peak, 3)})
            del dst
        del src
    return 0


def run_case(args):
    """One matmul configuration, e.g. --case Q5_K:28672:8192:128 (format,
    rows, K, tokens): --warmup untimed calls then --steps timed calls on
    rotating weight copies; prints one JSON line.  Small enough to run under
    a profiler."""
    import torch
    import axon_b200 as ax

    parts = args.case.split(":")
    if parts[0] == "PACK":
        return run_case_pack(args, parts[1], int(parts[2]), int(parts[3]))
    fmt, rows, K, M = parts
    rows, K, M = int(rows), int(K), int(M)
    dev = torch.device("cuda", 0)
    if fmt == "F32":
        return run_case_f32(args, rows, K, M)
    F = ax.QuantFormat[fmt]
    g = torch.Generator(device=dev).manual_seed(3)
    W = torch.randn(rows, K, device=dev, generator=g) * 0.02
    base = ax.QTensor.empty(rows, K, F, device=dev)
    ax.quantize(base, W, F)
    del W
    nbytes = ax.quantized_size_2d(rows, K, F)
    qs = [base] + [ax.QTensor(base.data.clone(), base.shape, base.fmt) for _ in range(max(0, -(-(300 << 20) // nbytes) - 1))]
    x = torch.randn(M, K, device=dev, generator=g)
    y = torch.empty(M, rows, device=dev)
    ws = ax.Workspace()
    for i in range(args.warmup):
        ax.linear_q(x, qs[i % len(qs)], out=y, workspace=ws)
    torch.cuda.synchronize()
    graph = None
    if args.case_graph:
        # the timed calls as one CUDA graph, so small shards are not timed
        # at the host's launch rate
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(args.steps):
                ax.linear_q(x, qs[i % len(qs)], out=y, workspace=ws)
        graph.replay()
        torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    if graph is not None:
        graph.replay()
    else:
        for i in range(args.steps):
            ax.linear_q(x, qs[i % len(qs)], out=y, workspace=ws)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / max(1, args.steps)
    print(json.dumps({"case": args.case, "graph": bool(graph), "ms": round(ms, 5),
                      "TOPS": round(2.0 * rows * K * M / (ms / 1e3) / 1e12, 2),
                      "weight_GBps": round(nbytes / (ms / 1e3) / 1e9, 1)}), flush=True)
    return 0


def run_case_pack(args, fmt, rows, cols):
    """Pack timing (--case PACK:FMT:ROWS:COLS): an fp32 [ROWS x COLS] tensor,
    N(0,1) with 1% U(-50, 50), packed --warmup untimed then --steps timed
    times; prints fp32 GB/s read and the HBM fraction of read + written
    bytes.  Small enough to run under a profiler."""
    import torch
    import axon_b200 as ax
    dev = torch.device("cuda", 0)
    F = ax.QuantFormat[fmt]
    g = torch.Generator(device=dev).manual_seed(11)
    src = torch.randn(rows, cols, device=dev, generator=g)
    m = torch.rand(rows, cols, device=dev, generator=g) < 0.01
    src[m] = torch.rand(int(m.sum().item()), device=dev, generator=g) * 100 - 50
    del m
    dst = torch.empty(ax.quantized_size_2d(rows, cols, F), dtype=torch.uint8, device=dev)
    for _ in range(args.warmup):
        ax.quantize(dst, src, F)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        ax.quantize(dst, src, F)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / max(1, args.steps)
    peak, _ = load_peaks()
    n = rows * cols
    print(json.dumps({"case": args.case, "ms": round(ms, 5), "read_GBps": round(4.0 * n / (ms / 1e3) / 1e9, 1),
                      "hbm_frac": round((4.0 * n + dst.numel()) / (ms / 1e3) / 1e9 / peak, 4),
                      "bytes_per_launch": int(4 * n + dst.numel())}), flush=True)
    return 0


def run_case_f32(args, rows, K, M):
    """fp32 matmul for unquantized A (--case F32:M:K:N): out[M x N] = a . b
    through axon_b200.matmul (the library's fp32 kernel), CUDA events over
    --steps calls; beside it the reference's cpu::matmul (oracle/_ref) on
    all host threads' worth of one call, timed once."""
    import torch
    import axon_b200 as ax
    import oracle

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(4)
    a = torch.randn(rows, K, device=dev, generator=g)
    b = torch.randn(K, M, device=dev, generator=g)
    out = torch.empty(rows, M, device=dev)
    for _ in range(max(3, args.warmup)):
        ax.matmul(out, a, b)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        ax.matmul(out, a, b)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / max(1, args.steps)
    flops = 2.0 * rows * K * M
    line = {"case": args.case, "ms": round(ms, 5), "TFLOPs": round(flops / (ms / 1e3) / 1e12, 2),
            "math": "fp32 multiply-adds (no TF32)"}
    ref = oracle.ref()
    if ref is not None:
        # the reference's single-threaded loop on a bounded row sample
        # (about 2 GFLOP), so large shapes stay quick
        rs = max(1, min(rows, int(2e9 / max(1.0, 2.0 * K * M))))
        an, bn = a[:rs].cpu().numpy(), b.cpu().numpy()
        t0 = time.perf_counter()
        ref.matmul_f32(an, bn)
        line["reference_cpu_GFLOPs"] = round(2.0 * rs * K * M / (time.perf_counter() - t0) / 1e9, 2)
        line["reference_sample_rows"] = rs
    print(json.dumps(line), flush=True)
    return 0


def run_axon(args):
    """Loading weights from an .axon file (the reference's format) into
    device memory: the headline workload's three packed matrices (340 MB,
    Q2_K / Q3_K / Q5_K [28672 x 8192]) saved with save_axon, then loaded with
    load_axon (file -> pinned staging -> device).  The file is read back from
    the page cache (it was just written), so this measures the loader, not a
    disk.  Beside it: the reference's own load_tensor (serialize.cpp:98-123,
    oracle/_ref) on an fp32 file of the same size into host memory (it cannot
    load packed tensors at all).  One JSON line."""
    import torch
    import axon_b200 as ax
    import oracle

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(11)
    ws = {}
    for fmt in FORMATS:
        q = ax.QTensor.empty(ROWS, K_DIM, ax.QuantFormat[fmt], device=dev)
        ax.quantize(q, torch.randn(ROWS, K_DIM, device=dev, generator=g) * 0.02, ax.QuantFormat[fmt])
        ws[fmt] = q
    total = sum(packed_bytes(f) for f in FORMATS)
    tmp = tempfile.mkdtemp(prefix="axq_axon_")
    path = os.path.join(tmp, "c4.axon")
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ax.save_axon(path, ws)
    save_s = time.perf_counter() - t0
    loads = []
    for _ in range(max(3, min(args.steps, 5))):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        back = ax.load_axon(path)
        torch.cuda.synchronize()
        loads.append(time.perf_counter() - t0)
        del back
    for fmt in FORMATS:  # loaded bytes equal the saved ones
        b = ax.load_axon(path)[fmt]
        if not torch.equal(b.data[:packed_bytes(fmt)], ws[fmt].data[:packed_bytes(fmt)]):
            raise RuntimeError(f"{fmt}: loaded bytes differ")
        del b
    line = {"config": "C6 .axon weights -> device", "bytes": total, "load_GBps": round(total / min(loads) / 1e9, 2),
            "load_ms": round(min(loads) * 1e3, 2), "save_GBps": round(total / save_s / 1e9, 2),
            "source": "page cache (file just written)"}
    ref = oracle.ref()
    if ref is not None:
        fpath = os.path.join(tmp, "f32.axon")
        n = total // 4
        ref.save_tensor(fpath, [n], 0, 0, np.zeros(n, dtype=np.float32))
        ref.load_tensor(fpath, cap=16)  # warm the page cache
        t0 = time.perf_counter()
        _, err = ref.load_tensor(fpath, cap=16)
        dt = time.perf_counter() - t0
        line["reference_load_tensor_fp32_host_GBps"] = round(total / dt / 1e9, 2) if err is None else err
        os.remove(fpath)
    os.remove(path)
    os.rmdir(tmp)
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="axon_b200", choices=["axon_b200", "reference"])
    ap.add_argument("--passes", type=int, default=PASSES, help="decode passes per step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip the GEMM and pack records")
    ap.add_argument("--suite", action="store_true", help="time every configuration (one JSON line each)")
    ap.add_argument("--case", default=None, help="time one matmul, FMT:ROWS:K:TOKENS (or PACK:FMT:ROWS:COLS)")
    ap.add_argument("--case-graph", action="store_true", help="--case: time the calls as one replayed CUDA graph")
    ap.add_argument("--axon", action="store_true", help="time loading the packed weights from an .axon file")
    args = ap.parse_args()
    if args.axon:
        return run_axon(args)
    if args.suite:
        return run_suite(args)
    if args.case:
        return run_case(args)
    if args.impl == "reference":
        return run_reference_arm(args)
    return run_gpu(args)


if __name__ == "__main__":
    sys.exit(main())
