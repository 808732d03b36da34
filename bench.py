"""bench.py — Q4_0 prefill GEMM throughput on B200 (benchmark config 2), driver contract.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Benchmark configs (seeded synthetic data: Q4_0 weights d = f16(|N(0,1)|*0.02), nibbles U{0..15};
activations N(0,1)):
  1  decode matvec, 8960 x 1536 Q4_0 x Q8_0, batch 1;
  2  prefill GEMM, 512 tokens x K 1536 -> 8960 features and 512 x K 8960 -> 1536, f16 in/out;
  3  Qwen2.5-1.5B-architecture prefill of 2048 tokens + 256 greedy decode tokens;
  4  Llama-3.2-3B-architecture decode at context 4096, batch 1 / 8 / 32;
  5  row-sharded lm_head 128256 x 3072 and FFN 8192 x 3072 over the GPUs, M in 1..8192.

The headline is config 2: a step is both projections, f16 activations, fp32 accumulation, f16
outputs, 2 * 14,092,861,440 FLOP per step.  value: whole-job TFLOP/s with inputs resident in HBM,
the median of several timed replays of a K-step CUDA graph (CUDA events on the launch stream, max
over ranks, spread in `timing_spread`); a pool of input sets larger than L2 is rotated between
steps.  e2e: the same metric through the C ABI with host buffers (pinned host -> device copies of
the step's activations, device -> host copies of its outputs, inside the timed region).
--gpus N > 1: one process per GPU, each rank prefilling its own ubatches (independent prompts,
no collective: weak scaling).  The same line carries `secondary` (config 1 and the decode
attention kernel, GB/s), `sharded` (config 5 at this run's GPU count, with the exchange step,
a g = 1 reference and a bit-identity parity flag) and, at N = 1, `decode` (config 4) and
`generate` (config 3), each with its CPU baseline (--no-extras: headline only).
--impl reference: the reference's own CPU implementation of the path (the C restatement of
sulimo-cpu's AVX2 prefill: per token quantize_f32_to_q8_0 + matvec_q4_0_q8_0_avx2), all host threads.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

T, K_UP, F_UP = 512, 1536, 8960          # up/gate projection
K_DN, F_DN = 8960, 1536                   # down projection
FLOP_PER_GEMM = 2 * T * K_UP * F_UP       # == 2 * T * K_DN * F_DN
FLOP_PER_STEP = 2 * FLOP_PER_GEMM
METRIC = "Q4_0 prefill GEMM TFLOP/s"
L2_BYTES = 126 * 1024 * 1024
REPEATS = 9                               # timed replays of the headline's K-step graph


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained"), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def ncu_traffic(kernel):
    p = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    if os.path.exists(p):
        return json.load(open(p)).get(kernel)
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled while the timed region runs."""
    FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def stop(self, t0, t1):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(2)
        except Exception:
            self.proc.kill()
        rows = []
        for ts, line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 7:
                continue
            rows.append((ts, parts))
        inside = [r for ts, r in rows if t0 - 0.15 <= ts <= t1 + 0.15] or [r for _, r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        mhz, maxmhz = [], []
        for r in inside:
            try:
                mhz.append(float(r[0]))
                maxmhz.append(float(r[1]))
            except ValueError:
                pass
            for i, n in enumerate(names):
                if r[3 + i].lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(mhz) if mhz else None,
                "sm_max_mhz": max(maxmhz) if maxmhz else None,
                "reasons": sorted(reasons), "samples": len(inside)}


def dist_setup(n_gpus):
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def make_inputs(seed):
    import numpy as np
    import torch
    rng = np.random.default_rng(seed)

    def q4(rows, cols):
        nb = rows * cols // 32
        d = (np.abs(rng.standard_normal(nb, dtype=np.float32)) * np.float32(0.02)).astype(np.float16)
        q = rng.integers(0, 256, nb * 16, dtype=np.uint8)
        return (torch.from_numpy(d.view(np.int16).copy()).cuda(), torch.from_numpy(q).cuda())

    up = q4(F_UP, K_UP)
    dn = q4(F_DN, K_DN)
    x_up = torch.randn(T * K_UP, device="cuda", dtype=torch.float16, generator=None)
    x_dn = torch.randn(T * K_DN, device="cuda", dtype=torch.float16)
    y_up = torch.empty(T * F_UP, device="cuda", dtype=torch.float16)
    y_dn = torch.empty(T * F_DN, device="cuda", dtype=torch.float16)
    return dict(up=up, dn=dn, x_up=x_up, x_dn=x_dn, y_up=y_up, y_dn=y_dn)


def set_bytes(s):
    b = 0
    for k in ("x_up", "x_dn", "y_up", "y_dn"):
        b += s[k].numel() * s[k].element_size()
    for k in ("up", "dn"):
        b += sum(t.numel() * t.element_size() for t in s[k])
    return b


def run_ours(args, rank, world, local):
    import torch
    import sulimo_b200 as sb

    torch.manual_seed(1234 + rank)
    ctx = sb.CudaContext(local, stream=torch.cuda.current_stream())
    sets = [make_inputs(seed=rank * 100 + i) for i in range(1)]
    per_set = set_bytes(sets[0])
    n_sets = max(2, -(-int(1.5 * L2_BYTES) // per_set))
    sets += [make_inputs(seed=rank * 100 + i) for i in range(1, n_sets)]

    def step(s):
        sb.gemm_q4_0_f16(ctx, s["up"][0], s["up"][1], s["x_up"], s["y_up"], F_UP, K_UP, T)
        sb.gemm_q4_0_f16(ctx, s["dn"][0], s["dn"][1], s["x_dn"], s["y_dn"], F_DN, K_DN, T)

    # eager warm-up steps (first calls set kernel attributes, outside any capture)
    for i in range(args.warmup):
        step(sets[i % n_sets])
    ctx.finish()

    # The timed steps are one CUDA graph (the launches are ~10 us of device work each, so a
    # host-side launch loop would time Python, not the GPU).
    launches0 = ctx.launch_count
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        ctx.set_stream(torch.cuda.current_stream())
        for j in range(args.steps):
            step(sets[j % n_sets])
    ctx.set_stream(torch.cuda.current_stream())
    launches = ctx.launch_count - launches0

    sampler = ClockSampler(local)
    sampler.start()
    t_w = time.time()
    n_w = 0
    while time.time() - t_w < 1.0:   # keep the GPU under the same load until the timed region
        graph.replay()
        torch.cuda.synchronize()
        n_w += 1
    # timed replays of the K-step graph (about half a second of them, at least REPEATS), each
    # bracketed by events on the launch stream; the value is the median replay (max over ranks),
    # the spread is reported beside it
    per_replay_s = (time.time() - t_w) / max(n_w, 1)
    reps_n = int(min(2000, max(REPEATS, 0.5 / max(per_replay_s, 1e-6))))
    reps_n = int(max_over_ranks(float(reps_n), world))  # every rank replays the same count
    barrier(world)
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(reps_n)]
    t0 = time.time()
    for e0, e1 in evs:
        e0.record()
        graph.replay()
        e1.record()
    torch.cuda.synchronize()
    t1 = time.time()
    barrier(world)
    reps = [e0.elapsed_time(e1) for e0, e1 in evs]
    if world > 1:  # one collective for all replays: the max over ranks of each
        import torch.distributed as dist
        t = torch.tensor(reps, dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        reps = t.tolist()
    clocks = sampler.stop(t_w, t1)
    clocks["window"] = (f"1 s of identical graph replays before the timed replays + the "
                        f"{reps_n} timed replays ({t1 - t0:.2f} s)")
    ctx.finish()
    del graph
    ms_max = statistics.median(reps)
    ms = ms_max
    value = FLOP_PER_STEP * args.steps * world / (ms_max / 1e3) / 1e12
    spread = {"replays": reps_n, "steps_per_replay": args.steps,
              "median_ms": round(ms_max, 5), "min_ms": round(min(reps), 5),
              "max_ms": round(max(reps), 5),
              "tflops_min_max": [round(FLOP_PER_STEP * args.steps * world / (t / 1e3) / 1e12, 1)
                                 for t in (max(reps), min(reps))]}

    # ---- e2e through the C ABI with host buffers ----
    e2e = run_e2e(args, ctx, sets[0], world)

    # ---- roofline of the dominant kernel (the tcgen05 GEMM: both launches of a step) ----
    hbm, tf_burst, tf_sust, src = peaks()
    per_launch_ms = ms / (2 * args.steps)
    achieved = FLOP_PER_GEMM / (per_launch_ms / 1e3) / 1e12
    roof = {"bound": "tensor", "achieved": round(achieved, 2), "peak": tf_burst,
            "unit": "TFLOP/s", "frac": round(achieved / tf_burst, 4),
            "traffic": ncu_traffic("gemm_q4_0_pair_kernel"),
            "peak_source": f"{src} bf16 dense burst (MEASURED_PEAKS.json)"
            if src == "measured" else "fallback 1.59 PFLOP/s"}

    secondary = None
    if rank == 0 and not args.no_secondary:
        secondary = run_secondary(ctx, hbm)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(time_budget_s=args.cpu_seconds)

    return dict(value=value, ms=ms_max, launches=launches, clocks=clocks, e2e=e2e, roof=roof,
                secondary=secondary, cpu=cpu, n_sets=n_sets, set_bytes=per_set, spread=spread)


def run_e2e(args, ctx, s, world):
    """Host buffers in, host buffers out, through the C-ABI buffer + GEMM entry points."""
    import ctypes as C
    import torch
    from sulimo_b200 import capi
    import sulimo_b200 as sb

    hx_up = torch.randn(T * K_UP, dtype=torch.float16).pin_memory()
    hx_dn = torch.randn(T * K_DN, dtype=torch.float16).pin_memory()
    hy_up = torch.empty(T * F_UP, dtype=torch.float16).pin_memory()
    hy_dn = torch.empty(T * F_DN, dtype=torch.float16).pin_memory()
    bufs = {}
    for name, n in (("x_up", hx_up.numel() * 2), ("x_dn", hx_dn.numel() * 2),
                    ("y_up", hy_up.numel() * 2), ("y_dn", hy_dn.numel() * 2)):
        h = C.c_void_p()
        capi.call("sulimo_cuda_buffer_alloc", ctx.handle, n, C.byref(h))
        bufs[name] = h
    L = capi.load()
    ptr = {k: L.sulimo_cuda_buffer_device_ptr(v) for k, v in bufs.items()}

    def step():
        capi.call("sulimo_cuda_buffer_write", bufs["x_up"], 0, hx_up.data_ptr(), hx_up.numel() * 2)
        capi.call("sulimo_cuda_buffer_write", bufs["x_dn"], 0, hx_dn.data_ptr(), hx_dn.numel() * 2)
        sb.gemm_q4_0_f16(ctx, s["up"][0], s["up"][1], ptr["x_up"], ptr["y_up"], F_UP, K_UP, T)
        sb.gemm_q4_0_f16(ctx, s["dn"][0], s["dn"][1], ptr["x_dn"], ptr["y_dn"], F_DN, K_DN, T)
        capi.call("sulimo_cuda_buffer_read", bufs["y_up"], 0, hy_up.data_ptr(), hy_up.numel() * 2)
        capi.call("sulimo_cuda_buffer_read", bufs["y_dn"], 0, hy_dn.data_ptr(), hy_dn.numel() * 2)

    for _ in range(max(3, args.warmup // 10)):
        step()
    ctx.finish()
    n = max(10, args.steps // 10)
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(n):
        step()
    ctx.finish()
    dt = time.perf_counter() - t0
    dt = max_over_ranks(dt, world)
    for h in bufs.values():
        capi.call("sulimo_cuda_buffer_free", h)
    return {"value": round(FLOP_PER_STEP * n * world / dt / 1e12, 3), "unit": "TFLOP/s",
            "h2d_bytes_per_step": (hx_up.numel() + hx_dn.numel()) * 2,
            "d2h_bytes_per_step": (hy_up.numel() + hy_dn.numel()) * 2, "steps": n,
            "how": "C-ABI sulimo_cuda_buffer_write -> 2x sulimo_cuda_gemm_q4_0_f16 -> "
                   "sulimo_cuda_buffer_read, pinned host memory, wall clock, max over ranks"}


def graph_time_us(ctx, launch, iters):
    """Average device time of launch(i) over `iters` calls replayed as one CUDA graph."""
    import torch
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        ctx.set_stream(torch.cuda.current_stream())
        for i in range(iters):
            launch(i)
    ctx.set_stream(torch.cuda.current_stream())
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    del g
    return e0.elapsed_time(e1) * 1e3 / iters


def run_secondary(ctx, hbm):
    """Decode-side kernels (configs 1/4 shapes), HBM GB/s against the measured copy peak; each
    timed as a CUDA graph of back-to-back launches over rotated inputs larger than L2."""
    import numpy as np
    import torch
    import sulimo_b200 as sb

    out = {}
    rng = np.random.default_rng(7)

    def gemv_case(rows, cols, batch, name, static=False, fast=False):
        nbytes_w = rows * cols // 32 * 18
        copies = max(2, -(-int(1.5 * L2_BYTES) // nbytes_w))
        ws = [torch.randint(0, 1 << 14, (rows * cols // 32,), dtype=torch.int16, device="cuda")
              .bitwise_and_(0x3fff) for _ in range(copies)]
        wq = [torch.randint(0, 256, (rows * cols // 32 * 16,), dtype=torch.uint8, device="cuda")
              for _ in range(copies)]
        xq = torch.randint(-100, 100, (batch * cols // 32 * 34,), dtype=torch.int8,
                           device="cuda").view(torch.uint8)
        xq.view(-1, 34)[:, :2] = 0x2C  # sane f16 scales
        y = torch.empty(batch * rows, dtype=torch.float32, device="cuda")
        fn = sb.matvec_q4_0_q8_0_fast if fast else sb.dispatch_matvec_q4_0_q8_0
        for i in range(5):
            fn(ctx, ws[i % copies], wq[i % copies], xq, rows, cols, y, batch, static)
        iters = max(20, copies * 4)
        us = graph_time_us(ctx, lambda i: fn(
            ctx, ws[i % copies], wq[i % copies], xq, rows, cols, y, batch, static), iters)
        alg = nbytes_w + batch * cols // 32 * 34 + batch * rows * 4
        out[name] = {"us_per_launch": round(us, 2), "GBps": round(alg / us / 1e3, 1),
                     "frac_of_measured_hbm": round(alg / us / 1e3 / hbm, 3),
                     "alg_bytes": alg, "l2": f"{copies} rotated weight copies",
                     "mode": ("fast, tensor-core form (exact block sums, fp32 block-order "
                              "accumulation)" if batch > 1 else
                              "fast (exact block sums, fp32 lane tree)") if fast
                             else "bit-exact AVX2 order"}

    gemv_case(8960, 1536, 1, "gemv_config1_8960x1536_b1")
    # the decode engine's form: model weights are static, so back-to-back matvecs overlap their
    # weight streams (sulimo_cuda_gemv_q4_0_q8_0_static)
    gemv_case(8960, 1536, 1, "gemv_config1_8960x1536_b1_static_weights", static=True)
    gemv_case(151936, 1536, 1, "gemv_lm_head_151936x1536_b1")
    gemv_case(8192, 3072, 8, "gemv_ffn_8192x3072_b8")
    # fast mode (sulimo_cuda_gemv_q4_0_q8_0_fast): the form the decode step streams weights with
    gemv_case(8960, 1536, 1, "gemv_config1_8960x1536_b1_fast", static=True, fast=True)
    gemv_case(151936, 1536, 1, "gemv_lm_head_151936x1536_b1_fast", static=True, fast=True)
    gemv_case(8192, 3072, 8, "gemv_ffn_8192x3072_b8_fast", static=True, fast=True)
    gemv_case(8192, 3072, 32, "gemv_ffn_8192x3072_b32_fast", static=True, fast=True)

    # decode attention, Llama-3.2-3B geometry at ctx 4096, batch 1
    H, Hkv, hd, cap = 24, 8, 128, 4096
    ring_bytes = cap * Hkv * hd // 32 * 34
    copies = max(2, -(-int(1.5 * L2_BYTES) // (2 * ring_bytes)))
    ks = [torch.randint(-127, 127, (ring_bytes,), dtype=torch.int8, device="cuda").view(torch.uint8)
          for _ in range(copies)]
    vs = [torch.randint(-127, 127, (ring_bytes,), dtype=torch.int8, device="cuda").view(torch.uint8)
          for _ in range(copies)]
    for r in ks + vs:
        r.view(-1, 34)[:, 0] = 0x00
        r.view(-1, 34)[:, 1] = 0x20
    q = torch.randn(H * hd, device="cuda")
    o = torch.empty(H * hd, device="cuda")
    for i in range(5):
        sb.causal_gqa_decode(ctx, q, ks[i % copies], vs[i % copies], cap, cap, H, Hkv, hd, o)
    iters = max(20, copies * 4)
    us = graph_time_us(ctx, lambda i: sb.causal_gqa_decode(
        ctx, q, ks[i % copies], vs[i % copies], cap, cap, H, Hkv, hd, o), iters)
    alg = 2 * ring_bytes + 2 * H * hd * 4
    out["attn_decode_llama3b_ctx4096_b1"] = {"us_per_call": round(us, 2),
                                             "GBps": round(alg / us / 1e3, 1),
                                             "frac_of_measured_hbm": round(alg / us / 1e3 / hbm, 3),
                                             "alg_bytes": alg}
    return out


def cpu_baseline(time_budget_s=10.0, steps=None):
    """The reference's CPU prefill of the two projections (C restatement), all host threads,
    on a bounded token sample; returns TFLOP/s scaled to the full-step FLOP count."""
    import numpy as np
    import oracle.ffi as O

    threads = os.cpu_count() or 1
    rng = np.random.default_rng(0)

    def q4(rows, cols):
        nb = rows * cols // 32
        d = (np.abs(rng.standard_normal(nb, dtype=np.float32)) * np.float32(0.02)).astype(np.float16)
        return d.view(np.uint16).copy(), rng.integers(0, 256, nb * 16, dtype=np.uint8)

    ws_u, wq_u = q4(F_UP, K_UP)
    ws_d, wq_d = q4(F_DN, K_DN)

    def run(tokens):
        x_u = rng.standard_normal((tokens, K_UP)).astype(np.float32)
        x_d = rng.standard_normal((tokens, K_DN)).astype(np.float32)
        t0 = time.perf_counter()
        O.cpu_prefill_projection(ws_u, wq_u, x_u, F_UP, K_UP, tokens, threads)
        O.cpu_prefill_projection(ws_d, wq_d, x_d, F_DN, K_DN, tokens, threads)
        return time.perf_counter() - t0

    t1 = run(threads)  # calibration: one token per thread
    per_tok = t1 / threads
    tokens = int(max(threads, min(T, time_budget_s / max(per_tok, 1e-9))))
    tokens = max(threads, (tokens // threads) * threads)
    dt = run(tokens)
    tf = 2 * 2 * tokens * K_UP * F_UP / dt / 1e12
    return {"value": round(tf, 5), "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{tokens} of the {T} tokens of both projections (per token: "
                      f"quantize_f32_to_q8_0 + matvec_q4_0_q8_0_avx2, {threads} threads), "
                      f"{dt:.1f} s"}


def run_reference(args, rank, world):
    """--impl reference: the reference's own CPU implementation of the path, all host threads."""
    if rank != 0:
        return None
    import numpy as np
    import oracle.ffi as O

    threads = os.cpu_count() or 1
    rng = np.random.default_rng(0)

    def q4(rows, cols):
        nb = rows * cols // 32
        d = (np.abs(rng.standard_normal(nb, dtype=np.float32)) * np.float32(0.02)).astype(np.float16)
        return d.view(np.uint16).copy(), rng.integers(0, 256, nb * 16, dtype=np.uint8)

    ws_u, wq_u = q4(F_UP, K_UP)
    ws_d, wq_d = q4(F_DN, K_DN)
    x_u = rng.standard_normal((T, K_UP)).astype(np.float32)
    x_d = rng.standard_normal((T, K_DN)).astype(np.float32)

    def step(tokens, off):
        O.cpu_prefill_projection(ws_u, wq_u, x_u[off:off + tokens], F_UP, K_UP, tokens, threads)
        O.cpu_prefill_projection(ws_d, wq_d, x_d[off:off + tokens], F_DN, K_DN, tokens, threads)

    t0 = time.perf_counter()
    step(threads, 0)
    per_tok = (time.perf_counter() - t0) / threads
    budget = 90.0 / max(1, args.steps + args.warmup)   # whole run ~1.5 min
    tokens = int(max(1, min(T, budget / max(per_tok, 1e-9))))
    for i in range(args.warmup):
        step(tokens, 0)
    t0 = time.perf_counter()
    for i in range(args.steps):
        step(tokens, (i * tokens) % max(1, T - tokens + 1))
    dt = time.perf_counter() - t0
    value = 2 * 2 * tokens * K_UP * F_UP * args.steps / dt / 1e12
    return {"metric": METRIC, "value": round(value, 6), "unit": "TFLOP/s", "impl": "reference",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16 in / int8+fp32 CPU math",
            "data": "synthetic",
            "config": {"workload": "config2 prefill GEMM pair, bounded token sample per step",
                       "tokens_per_step": tokens, "of_tokens": T,
                       "shapes": "512x1536->8960 and 512x8960->1536"},
            "cpu_baseline": {"value": round(value, 6), "unit": "TFLOP/s", "cores": threads,
                             "kind": "port",
                             "sample": f"{tokens} tokens of both projections per step"},
            "e2e": {"value": round(value, 6), "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def run_sharded(args, rank, world, local, parity_m=128):
    """Row-sharded Q4_0 projections (config 5): W_lm 128256x3072 and W_ffn 8192x3072 split by
    rows over the ranks, X [M, 3072] f16 replicated, M in {1, 16, 128, 1024, 8192}.  Per
    (weight, M), each timed with CUDA events over `steps` iterations after `warmup`, max over
    ranks: the unsharded single-GPU GEMM of the whole weight on every rank at once (the g = 1
    reference), this rank's shard GEMM, the NCCL all-gather, the NCCL end-to-end forward (GEMM +
    all-gather + row-major unshard) and the fused forward (all-gather in the GEMM epilogue).
    Parity at M = parity_m for the lm_head: every rank's fused and NCCL results bit-identical to
    the unsharded GEMM's (same per-output arithmetic: neither splits K at that size; the FFN's
    unsharded GEMM does, so its results differ in summation order).  One dict per (weight, M)."""
    import torch
    import torch.distributed as dist
    import sulimo_b200 as sb
    from sulimo_b200.sharded import FusedShardedQ4Projection, ShardedQ4Projection, shard_weight
    ctx = sb.CudaContext(local, stream=torch.cuda.current_stream())
    K = 3072
    lines = []
    for wname, F in (("lm_head 128256x3072", 128256), ("ffn 8192x3072", 8192)):
        gen = torch.Generator(device="cuda")
        gen.manual_seed(F)
        nb = F * K // 32
        d = (torch.randn(nb, device="cuda", generator=gen).abs() * 0.02).half().view(torch.int16)
        qn = torch.randint(0, 256, (nb * 16,), device="cuda", dtype=torch.uint8, generator=gen)
        s_r, q_r, fs = shard_weight(d, qn, F, K, rank, world)
        proj = ShardedQ4Projection(ctx, s_r, q_r, F, K, fs)
        fused = FusedShardedQ4Projection(ctx, s_r, q_r, F, K, fs, m_max=8192)
        for M in (1, 16, 128, 1024, 8192):
            x = torch.randn(M * K, device="cuda", dtype=torch.float16, generator=gen)
            g, y = proj.buffers(M, sb.OUT_F16)
            y1 = torch.empty(M * F, dtype=torch.float16, device="cuda")

            def timed(fn):
                for _ in range(args.warmup):
                    fn()
                barrier(world)
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(args.steps):
                    fn()
                e1.record()
                torch.cuda.synchronize()
                return max_over_ranks(e0.elapsed_time(e1) / args.steps, world)

            t_single = timed(lambda: sb.gemm_q4_0_f16(ctx, d, qn, x, y1, F, K, M, sb.OUT_F16))
            t_gemm = timed(lambda: proj.local_gemm(x, M, g, sb.OUT_F16))
            t_ag = timed(lambda: proj.all_gather(M, g)) if world > 1 else 0.0
            t_e2e = timed(lambda: proj.forward(x, M, g, y, sb.OUT_F16))
            t_fused = timed(lambda: fused.forward_fused(x, M))
            flop = 2.0 * M * K * F
            ag_bytes = M * F * 2 * (world - 1) / world
            wbytes = nb * 18
            ent = {
                "weight": wname, "m_tokens": M, "rows_per_gpu": fs,
                "single_gpu_ms": round(t_single, 4), "gemm_ms": round(t_gemm, 4),
                "allgather_ms": round(t_ag, 4), "nccl_e2e_ms": round(t_e2e, 4),
                "fused_ms": round(t_fused, 4),
                "fused_tflops": round(flop / (t_fused * 1e-3) / 1e12, 2),
                "nccl_e2e_tflops": round(flop / (t_e2e * 1e-3) / 1e12, 2),
                "gemm_tflops_per_gpu": round(flop / world / (t_gemm * 1e-3) / 1e12, 2),
                "gemm_weight_GBps_per_gpu": round(wbytes / world / (t_gemm * 1e-3) / 1e9, 1),
                "allgather_GBps_per_gpu": round(ag_bytes / (t_ag * 1e-3) / 1e9, 1)
                if t_ag > 0 else None,
                "efficiency_fused_vs_g1": round(t_single / (world * t_fused), 3),
                "efficiency_nccl_vs_g1": round(t_single / (world * t_e2e), 3)}
            if M == parity_m and F > 100000:
                fused.forward_fused(x, M)
                yf = torch.empty(M * F, dtype=torch.float16, device="cuda")
                from sulimo_b200 import capi
                # a stream-ordered copy of this rank's fused Y (a library buffer) into yf
                capi.call("sulimo_cuda_unshard_rows", ctx.handle,
                          ctx.device_ptr(fused.y_buf), yf.data_ptr(), 1, M, F, F, 2)
                proj.forward(x, M, g, y, sb.OUT_F16)
                sb.gemm_q4_0_f16(ctx, d, qn, x, y1, F, K, M, sb.OUT_F16)
                ctx.finish()
                ok = torch.tensor([int(torch.equal(yf.view(torch.int16), y1.view(torch.int16)) and
                                       torch.equal(y.view(torch.int16), y1.view(torch.int16)))],
                                  device="cuda")
                if world > 1:
                    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
                ent["parity_bit_identical_to_single_gpu"] = bool(ok.item())
                del yf
            lines.append(ent)
            del x, g, y, y1
        barrier(world)  # no rank unmaps its peers' buffers while a store may be in flight
        fused.close()
        del proj, fused, s_r, q_r, d, qn
        torch.cuda.empty_cache()
    ctx.close()
    return lines


def cpu_forward_token_baseline(w, rings, cfg, pos, token, budget_s):
    """The reference's CPU decode (forward_token, crates/sulimo-engine/src/forward_pass.rs:
    190-417, restated in the oracle: AVX2 matvecs, 1 thread) on a host copy of the same model
    and K/V rings, timed at the same position: seconds per token over a bounded sample."""
    import numpy as np
    import oracle.ffi as O

    def h(t):
        if t is None:
            return None
        a = t.detach().cpu().numpy()
        return a.view(np.uint16) if a.dtype == np.int16 else a

    wh = dict(cfg=cfg, tok=(h(w["tok"][0]), h(w["tok"][1])), out_norm=h(w["out_norm"]),
              layers=[{k: ((h(v[0]), h(v[1])) if isinstance(v, tuple) else h(v))
                       for k, v in L.items()} for L in w["layers"]])
    wh["out"] = wh["tok"]
    om = O.OracleModel(wh)
    slot = cfg["head_count_kv"] * cfg["head_dim"] // 32 * 34
    for (kr, vr), (ok, ov) in zip(rings, om.rings):
        ok[:] = kr.detach().cpu().numpy()[:cfg["kv_capacity"] * slot]
        ov[:] = vr.detach().cpu().numpy()[:cfg["kv_capacity"] * slot]
    t0 = time.time()
    n = 0
    while n == 0 or time.time() - t0 < budget_s:
        om.forward_token(token, pos)
        n += 1
    return (time.time() - t0) / n, n


def run_decode(args, rank, world, local):
    """Config 4: Llama-3.2-3B-architecture decode at context 4096 (each sequence's ring
    pre-filled with 4096 positions of random Q8_0 K/V), batch 1 / 8 / 32 independent sequences.
    A step is one sulimo_cuda_forward_token (28 layers + vocab projection) plus the greedy
    argmax, captured once as a CUDA graph and replayed `steps` times.  Decode is replicated,
    not sharded: with N ranks each runs its own sequences and the tok/s add up."""
    import torch
    import sulimo_b200 as sb
    from sulimo_b200.model import DecodeModel
    from sulimo_b200.synthetic import LLAMA_3B, make_model_torch, weight_bytes
    ctx = sb.CudaContext(local, stream=torch.cuda.current_stream())
    cfg = dict(LLAMA_3B)
    cap = 4096
    w = make_model_torch(cfg, seed=rank, kv_capacity=cap)
    wbytes = weight_bytes(cfg)
    slot = cfg["head_count_kv"] * cfg["head_dim"] // 32 * 34
    scale = torch.tensor([0.02], dtype=torch.float16).view(torch.uint8).cuda()
    lines = []
    for b in args.decode_batches:
        dm = DecodeModel(ctx, w, batch=b)
        gen = torch.Generator(device="cuda")
        gen.manual_seed(100 + b)
        for kr, vr in dm.rings:
            for r in (kr, vr):
                r.copy_(torch.randint(0, 256, r.shape, dtype=torch.uint8, device="cuda",
                                      generator=gen))
                r.view(-1, 34)[:, 0:2] = scale
        tokens = torch.randint(0, cfg["vocab"], (b,), dtype=torch.int32, device="cuda",
                               generator=gen)
        pos = cap - 1
        for _ in range(args.warmup):
            dm.forward_token(tokens, pos)
            dm.greedy()
        ctx.finish()
        launches0 = ctx.launch_count
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            ctx.set_stream(torch.cuda.current_stream())
            dm.forward_token(tokens, pos)
            dm.greedy()
        ctx.set_stream(torch.cuda.current_stream())
        launches = ctx.launch_count - launches0
        for _ in range(3):
            graph.replay()
        barrier(world)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)
        step_bytes = wbytes + b * cfg["n_layers"] * 2 * cap * slot
        hbm, _, _, src = peaks()
        lines.append({
            "mode": "decode", "workload": "config 4: Llama-3.2-3B-arch decode, ctx 4096",
            "batch_per_gpu": b, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 4), "tok_per_s": round(b * world / (ms * 1e-3), 1),
            "bytes_per_step": step_bytes, "GBps": round(step_bytes / (ms * 1e-3) / 1e9, 1),
            "frac_of_measured_hbm": round(step_bytes / (ms * 1e-3) / 1e9 / hbm, 3),
            "gpu_launches_per_step": launches, "dtype": "q4_0 weights x q8_0 activations",
            "data": "synthetic (seeded Q4_0 weights, random Q8_0 K/V rings)"})
        if b == 1 and rank == 0 and world == 1 and not args.no_cpu:
            sec, n = cpu_forward_token_baseline(w, dm.rings, w["cfg"], pos,
                                                int(tokens[0].item()), args.cpu_seconds)
            lines[-1]["cpu_baseline"] = {
                "value": round(1.0 / sec, 3), "unit": "tok/s", "cores": 1, "kind": "port",
                "sample": f"{n} forward_token call(s) at position {pos} (context {cap}) of the "
                          "same model and rings, oracle restatement, 1 thread"}
        del graph, dm
        torch.cuda.empty_cache()
    ctx.close()
    return lines


def run_generate(args, rank, world, local):
    """Config 3: Qwen2.5-1.5B-architecture generation -- prefill of 2048 random token ids as
    4 ubatches of 512 (execute_prefill_ubatch), then 256 greedy decode tokens into the
    4096-slot Q8_0 ring (forward_token + on-device argmax; the next token never leaves the
    GPU).  Prefill and decode are timed separately with CUDA events; decode steps are launched
    eagerly (the context grows every step).  Replicated per rank."""
    import torch
    import sulimo_b200 as sb
    from sulimo_b200.model import DecodeModel
    from sulimo_b200.synthetic import QWEN_1_5B, make_model_torch, weight_bytes
    ctx = sb.CudaContext(local, stream=torch.cuda.current_stream())
    cfg = dict(QWEN_1_5B)
    w = make_model_torch(cfg, seed=rank, kv_capacity=4096)
    dm = DecodeModel(ctx, w, batch=1)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(7 + rank)
    n_prompt, ub, n_gen = 2048, 512, args.gen_tokens
    prompt = torch.randint(0, cfg["vocab"], (n_prompt,), dtype=torch.int32, device="cuda",
                           generator=gen)

    def prefill():
        lg = None
        for s0 in range(0, n_prompt, ub):
            lg = dm.prefill(prompt[s0:s0 + ub], s0)
        return lg

    def decode(lg):
        dm.greedy(lg)
        for i in range(n_gen):
            dm.forward_token(dm.next_tokens, n_prompt + i)
            dm.greedy()

    for _ in range(max(1, args.warmup // 3)):
        decode(prefill())
    ctx.finish()
    barrier(world)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    ev[0].record()
    lg = prefill()
    ev[1].record()
    decode(lg)
    ev[2].record()
    torch.cuda.synchronize()
    t_pre = max_over_ranks(ev[0].elapsed_time(ev[1]), world)
    t_dec = max_over_ranks(ev[1].elapsed_time(ev[2]), world)
    L, E, F = cfg["n_layers"], cfg["embd"], cfg["ffn"]
    qd, kvd = cfg["head_count"] * cfg["head_dim"], cfg["head_count_kv"] * cfg["head_dim"]
    layer_params = E * (qd + 2 * kvd) + qd * E + 3 * E * F
    pre_flop = 2.0 * n_prompt * L * layer_params + 2.0 * cfg["vocab"] * E * (n_prompt // ub)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        # the reference's CPU prefill is forward_token per prompt token (engine.rs:287-318)
        sec, n = cpu_forward_token_baseline(w, dm.rings, w["cfg"], n_prompt - 1,
                                            int(prompt[-1].item()), args.cpu_seconds)
        cpu = {"prefill_tok_per_s": round(1.0 / sec, 3), "decode_tok_per_s": round(1.0 / sec, 3),
               "unit": "tok/s", "cores": 1, "kind": "port",
               "sample": f"{n} forward_token call(s) at position {n_prompt - 1} of the same model "
                         "and rings (the CPU prefill runs forward_token per prompt token), oracle "
                         "restatement, 1 thread"}
    ctx.close()
    out = {
        "mode": "generate", "workload": "config 3: Qwen2.5-1.5B-arch, prefill 2048 (4 x 512) + "
                                        f"{n_gen} greedy decode tokens, 4096-slot Q8_0 ring",
        "n_gpus": world, "prefill_ms": round(t_pre, 3),
        "prefill_tok_per_s": round(n_prompt * world / (t_pre * 1e-3), 1),
        "prefill_tflops_projections": round(pre_flop / (t_pre * 1e-3) / 1e12, 1),
        "decode_ms": round(t_dec, 3), "decode_ms_per_token": round(t_dec / n_gen, 4),
        "decode_tok_per_s": round(n_gen * world / (t_dec * 1e-3), 1),
        "decode_weight_GBps": round(weight_bytes(cfg) * n_gen / (t_dec * 1e-3) / 1e9, 1),
        "dtype": "q4_0 weights; f16 prefill activations, q8_0 decode activations",
        "data": "synthetic (seeded Q4_0 weights, random token ids)"}
    if cpu is not None:
        out["cpu_baseline"] = cpu
    return [out]


def run_probe(args, local):
    """One kernel on a fixed case, for profiler captures (`ncu ... python bench.py --mode probe
    --kernel K`): `warmup` + `steps` eager launches on rotated inputs, then one JSON line with
    the mean time per launch from CUDA events.  Kernels:
      gemm_up / gemm_down   benchmark config 2's two projections (512 tokens), f16 out;
      gemv_fast / gemv_exact  config 1 (8960 x 1536 Q4_0 x Q8_0, batch 1), fast / AVX2-order;
      gemv_batched          config 4's gate projection (8192 x 3072) in fast mode for
                            --probe-batch sequences (the tensor-core form from 2);
      attn                  decode attention, Llama-3.2-3B geometry (24 / 8 heads, hd 128),
                            context 4096, batch 1, random Q8_0 rings;
      attn_prefill          prefill attention, Qwen2.5-1.5B geometry (12 / 2 heads, hd 128),
                            a 512-token ubatch at positions 1536..2047 (--probe-start to move
                            it), random Q8_0 rings of 4096 slots;
      decode_step           one config-4 forward_token at context 4096 for --probe-batch
                            sequences."""
    import numpy as np
    import torch
    import sulimo_b200 as sb
    ctx = sb.CudaContext(local, stream=torch.cuda.current_stream())
    g = torch.Generator(device="cuda")
    g.manual_seed(5)

    def q4(rows, cols):
        nb = rows * cols // 32
        d = (torch.randn(nb, device="cuda", generator=g).abs() * 0.02).half().view(torch.int16)
        return d, torch.randint(0, 256, (nb * 16,), device="cuda", dtype=torch.uint8, generator=g)

    kern = args.kernel
    sets = []
    if kern in ("gemm_up", "gemm_down"):
        f, k = (F_UP, K_UP) if kern == "gemm_up" else (F_DN, K_DN)
        for _ in range(4):
            sets.append((q4(f, k), torch.randn(T * k, device="cuda", generator=g).half(),
                         torch.empty(T * f, device="cuda", dtype=torch.float16)))

        def launch(s):
            sb.gemm_q4_0_f16(ctx, s[0][0], s[0][1], s[1], s[2], f, k, T)
    elif kern in ("gemv_fast", "gemv_exact"):
        rows, cols = 8960, 1536
        for _ in range(20):
            xq = torch.empty(cols // 32 * 34, device="cuda", dtype=torch.uint8)
            sb.quantize_f32_to_q8_0(ctx, torch.randn(cols, device="cuda", generator=g), xq)
            sets.append((q4(rows, cols), xq, torch.empty(rows, device="cuda")))

        def launch(s):
            if kern == "gemv_fast":
                sb.matvec_q4_0_q8_0_fast(ctx, s[0][0], s[0][1], s[1], rows, cols, s[2],
                                         static_weights=True)
            else:
                sb.dispatch_matvec_q4_0_q8_0(ctx, s[0][0], s[0][1], s[1], rows, cols, s[2])
    elif kern == "gemv_batched":
        rows, cols, nb = 8192, 3072, args.probe_batch if args.probe_batch > 1 else 8
        for _ in range(8):
            xq = torch.empty(nb * cols // 32 * 34, device="cuda", dtype=torch.uint8)
            sb.quantize_f32_to_q8_0(ctx, torch.randn(nb * cols, device="cuda", generator=g), xq)
            sets.append((q4(rows, cols), xq, torch.empty(nb * rows, device="cuda")))

        def launch(s):
            sb.matvec_q4_0_q8_0_fast(ctx, s[0][0], s[0][1], s[1], rows, cols, s[2], nb,
                                     static_weights=True)
    elif kern == "attn":
        H, Hkv, hd, cap = 24, 8, 128, 4096
        for _ in range(20):
            ring = lambda: torch.randint(0, 256, (cap * Hkv * hd // 32 * 34,), device="cuda",  # noqa: E731
                                         dtype=torch.uint8, generator=g)
            kr, vr = ring(), ring()
            for r in (kr, vr):
                r.view(-1, 34)[:, 0:2] = torch.tensor([0.02], dtype=torch.float16).view(
                    torch.uint8).cuda()
            sets.append((torch.randn(H * hd, device="cuda", generator=g), kr, vr,
                         torch.empty(H * hd, device="cuda")))

        def launch(s):
            sb.causal_gqa_decode(ctx, s[0], s[1], s[2], cap, cap, H, Hkv, hd, s[3])
    elif kern == "attn_prefill":
        H, Hkv, hd, cap, n = 12, 2, 128, 4096, 512
        start = args.probe_start
        for _ in range(4):
            ring = lambda: torch.randint(-127, 128, (cap * Hkv * hd // 32, 34), device="cuda",  # noqa: E731
                                         dtype=torch.int32, generator=g).to(torch.int8)
            kr, vr = ring(), ring()
            for r in (kr, vr):
                r[:, 0:2] = torch.tensor([0.02], dtype=torch.float16).view(torch.int8).cuda()
            sets.append((torch.randn(n * H * hd, device="cuda", generator=g), kr, vr,
                         torch.empty(n * H * hd, device="cuda", dtype=torch.float16)))

        def launch(s):
            sb.causal_gqa_attention_prefill(ctx, s[0], s[1], s[2], start, cap, n, H, Hkv, hd,
                                            s[3])
    elif kern == "decode_step":
        from sulimo_b200.model import DecodeModel
        from sulimo_b200.synthetic import LLAMA_3B, make_model_torch
        w = make_model_torch(dict(LLAMA_3B), seed=0, kv_capacity=4096)
        dm = DecodeModel(ctx, w, batch=args.probe_batch)
        tok = torch.zeros(args.probe_batch, dtype=torch.int32, device="cuda")
        sets.append(None)

        def launch(s):
            dm.forward_token(tok, 4095)
    else:
        raise SystemExit(f"unknown --kernel {kern}")
    for i in range(args.warmup):
        launch(sets[i % len(sets)])
    ctx.finish()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        launch(sets[i % len(sets)])
    e1.record()
    torch.cuda.synchronize()
    ctx.close()
    return {"mode": "probe", "kernel": kern, "launches": args.steps,
            "us_per_launch_eager": round(e0.elapsed_time(e1) * 1e3 / args.steps, 3)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=500)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-secondary", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="headline only: skip the config 3/4 (N = 1) and config 5 keys")
    ap.add_argument("--extra-steps", type=int, default=30,
                    help="timed steps of each extra key's cases (capped by --steps)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--decode-batches", type=int, nargs="+", default=[1, 8, 32],
                    help="--mode decode: sequences per GPU to measure")
    ap.add_argument("--gen-tokens", type=int, default=256,
                    help="--mode generate: greedy decode tokens after the 2048-token prefill")
    ap.add_argument("--probe-batch", type=int, default=1,
                    help="sequences per launch for --mode probe (gemv_batched: 8 if 1)")
    ap.add_argument("--kernel", default="attn",
                    help="--mode probe: gemm_up, gemm_down, gemv_fast, gemv_exact, "
                         "gemv_batched, attn, attn_prefill, decode_step")
    ap.add_argument("--probe-start", type=int, default=1536,
                    help="--mode probe --kernel attn_prefill: the ubatch's first position")
    ap.add_argument("--mode", default="headline",
                    choices=["headline", "sharded", "decode", "generate", "probe", "secondary"],
                    help="headline: the contract line (config 2); sharded: the row-sharded "
                         "lm_head/FFN sweep with an NCCL all-gather; decode: config 4 "
                         "(Llama-3B decode steps); generate: config 3 (Qwen-1.5B prefill + "
                         "greedy decode); one JSON line per case; secondary: the decode-side "
                         "kernel table of the headline line alone")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        line = run_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return

    rank, world, local = dist_setup(args.gpus)
    if args.mode == "probe":
        print(json.dumps(run_probe(args, local)), flush=True)
        return
    if args.mode == "secondary":
        import torch
        import sulimo_b200 as sb
        ctx = sb.CudaContext(local, stream=torch.cuda.current_stream())
        print(json.dumps({"mode": "secondary", "cases": run_secondary(ctx, peaks()[0])}),
              flush=True)
        ctx.close()
        return
    if args.mode in ("sharded", "decode", "generate"):
        run = {"sharded": run_sharded, "decode": run_decode, "generate": run_generate}[args.mode]
        for line in run(args, rank, world, local):
            if rank == 0:
                print(json.dumps(line), flush=True)
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()
        return
    r = run_ours(args, rank, world, local)
    extras = {}
    if not args.no_extras:
        import torch
        torch.cuda.empty_cache()
        xa = argparse.Namespace(**vars(args))
        xa.steps = max(3, min(args.steps, args.extra_steps))
        xa.warmup = max(3, min(args.warmup, 10))
        # config 5 on every rank (the row-sharded lm_head / FFN with its exchange step)
        extras["sharded"] = {
            "workload": "config 5: row-sharded Q4_0 lm_head 128256x3072 and FFN 8192x3072, "
                        f"x [M][3072] f16, over the {world} GPU(s) of this run",
            "steps": xa.steps, "warmup": xa.warmup,
            "cases": run_sharded(xa, rank, world, local)}
        torch.cuda.empty_cache()
        if world == 1:
            # configs 4 and 3 (decode is replicated, not sharded: measured on one GPU)
            extras["decode"] = run_decode(xa, rank, world, local)
            torch.cuda.empty_cache()
            extras["generate"] = run_generate(xa, rank, world, local)[0]
            torch.cuda.empty_cache()
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(r["value"], 3), "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(r["ms"] / args.steps, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (seeded Q4_0 weights d=f16(|N|*0.02), nibbles U{0..15}; x f16 N(0,1))",
            "config": {"workload": "benchmark config 2: Q4_0 prefill GEMM, 512 tokens x K1536 -> "
                                   "N8960 and 512 x K8960 -> N1536 per step",
                       "global_batch": T * world, "seq_len": T,
                       "parallelism": f"dp{world} (independent ubatches per rank)",
                       "l2": f"inputs rotated over {r['n_sets']} sets of "
                             f"{r['set_bytes'] / 2**20:.0f} MiB (> 126 MB L2)"},
            "e2e": r["e2e"], "gpu_launches": r["launches"], "roofline": r["roof"],
            "clocks": r["clocks"],
        }
        if r["cpu"] is not None:
            line["cpu_baseline"] = r["cpu"]
        if r["secondary"] is not None:
            line["secondary"] = r["secondary"]
        line["timing_spread"] = r["spread"]
        line.update(extras)
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
