"""Benchmark: Llama-3-8B-shaped Q4_K_M batch-1 greedy decode on B200.

Metric: decode tok/s, Llama-3-8B shape, Q4_K_M random-init
weights (synthetic), 1 session, greedy, after a 2048-token prompt; plus the
Q4_K GEMV's achieved HBM GB/s as the roofline of the dominant kernel.

A "step" is one decode token (one pass of the quantized projection path over
all 32 layers and the LM head).  `value` is device-timed (CUDA events on the
session's stream, inputs resident in HBM, argmax fed back on the device);
`e2e` is the same metric through the reference-facing session call with host
buffers (token in, argmax out, host<->device copies inside the timed region).

Arms:
  python bench.py [--gpus N --steps K --warmup W]         this implementation
  python bench.py --impl reference [...]                  the reference CPU path
      (the C restatement in oracle/, all host threads; the reference is C#/.NET
      with no runtime in this image)
Multi-GPU (torchrun, N > 1): the model is split tensor-parallel over the N
GPUs (heads, FFN rows and vocabulary; exact, see ovf_model_create_tp); value
= the sequence's tokens / the max-over-ranks device time (strong scaling).
The other BASELINE configs (single GEMV, prefill GEMM sweep, Qwen2-0.5B,
16 concurrent sessions) and the CPU baseline are reported at N = 1.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PROMPT = 2048
METRIC = "decode tok/s (Llama-3-8B-shape Q4_K_M, batch 1)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--prompt", type=int, default=PROMPT)
    ap.add_argument("--layers", type=int, default=None, help="debug only: fewer layers (invalid as a bench number)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--kv", default="f16", choices=["f16", "f32"],
                    help="KV cache of the timed session: f16 (the benchmark config) or f32 (the reference's default, "
                         "bit-exact attention)")
    ap.add_argument("--no-extra", action="store_true",
                    help="only the headline decode line (skip the other BASELINE configs and the exact-cache lines)")
    ap.add_argument("--profile-target", default=None, choices=sorted(PROFILE_TARGETS),
                    help="run only a few launches of one kernel on a small case (for ncu captures) and exit")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


class ClockSampler:
    """Samples nvidia-smi clocks/throttle reasons during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------ CPU baseline
def _oracle_llama8b(max_ctx: int):
    """The C restatement of the reference's CPU path (oracle/) holding a
    Llama-3-8B Q4_K_M model in host memory: one layer's weights quantized by
    the restated encoders and copied into 32 distinct layer buffers (every
    token streams 32 x 148 MB of layer weights plus the 431 MB LM head from
    DRAM, as the full model does; nothing can stay cache-resident)."""
    from oracle import oracle as orc
    from overfit_b200.engine import LLAMA3_8B as cfg

    D, H, KVH, hd, FF, V = (cfg[k] for k in ("d_model", "n_heads", "n_kv_heads", "head_dim", "d_ff", "vocab"))

    def qmat(rows, cols, enc, seed):
        out = []
        step = 8192
        for r0 in range(0, rows, step):
            r = min(step, rows - r0)
            w = orc.fill_normal(r * cols, seed * 1000 + r0, 0.0, 0.02).reshape(r, cols)
            out.append(enc(w))
        return np.concatenate(out)

    t0 = time.time()
    base = dict(wq=(orc.Q4_K, qmat(H * hd, D, orc.quantize_q4k, 1), None, H * hd, D),
                wk=(orc.Q4_K, qmat(KVH * hd, D, orc.quantize_q4k, 2), None, KVH * hd, D),
                wv=(orc.Q6_K, qmat(KVH * hd, D, orc.quantize_q6k, 3), None, KVH * hd, D),
                gate=(orc.Q4_K, qmat(FF, D, orc.quantize_q4k, 5), None, FF, D),
                up=(orc.Q4_K, qmat(FF, D, orc.quantize_q4k, 6), None, FF, D),
                down=(orc.Q6_K, qmat(D, FF, orc.quantize_q6k, 7), None, D, FF))
    q, sc = orc.requant_q8_0(orc.Q4_K, qmat(D, H * hd, orc.quantize_q4k, 4), D, H * hd)
    base["wo"] = (orc.Q8_0, q, sc, D, H * hd)
    layers = []
    for _ in range(cfg["n_layers"]):
        L = dict(attn_norm=np.ones(D, np.float32), ffn_norm=np.ones(D, np.float32))
        for k, (t, data, scales, r, c) in base.items():
            L[k] = (t, data.copy(), None if scales is None else scales.copy(), r, c)
        layers.append(L)
    weights = dict(layers=layers, embed=(orc.Q4_K, qmat(V, D, orc.quantize_q4k, 8), None, V, D),
                   final_norm=np.ones(D, np.float32), lm_head=(orc.Q6_K, qmat(V, D, orc.quantize_q6k, 9), None, V, D))
    gen_s = time.time() - t0
    return orc, cfg, orc.OracleSession(cfg, weights, max_ctx), gen_s


def cpu_decode_sample(context: int, samples: int, threads: int | None = None) -> dict:
    """Times the reference CPU path (the C restatement, OpenMP over the host
    threads, the reference's output-row bands) on the benchmark's own decode:
    Llama-3-8B Q4_K_M, distinct per-layer weights, at the GPU arm's context
    (the F32 cache filled with `context` synthetic rows).  The value is the
    median over `samples` single-token decodes."""
    from oracle import oracle as orc0

    if threads:
        orc0.set_threads(threads)
    orc, cfg, sess, gen_s = _oracle_llama8b(context + samples + 4)
    sess.fill_context(context)
    tok = 1
    sess.decode(tok)  # warm-up token
    times = []
    for _ in range(samples):
        t0 = time.perf_counter()
        lg = sess.decode(tok)
        times.append(time.perf_counter() - t0)
        tok = int(np.argmax(lg))
    med = float(np.median(times))
    return {"tok_s": 1.0 / med, "s_per_token": med, "cores": orc.num_threads(), "gen_s": gen_s,
            "samples_s": times,
            "sample": f"median of {samples} single-token greedy decodes of the full 32-layer + LM-head Llama-3-8B "
                      f"Q4_K_M step (distinct per-layer weights) at context {context + 1}..{context + samples + 1}"}


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    samples = max(5, min(args.steps, 8))
    r = cpu_decode_sample(args.prompt, samples)
    line = {"impl": "reference", "metric": METRIC, "value": r["tok_s"], "unit": "tok/s", "n_gpus": 0,
            "steps": samples, "warmup": 1, "ms_per_step": r["s_per_token"] * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8 dot / fp32", "data": "synthetic",
            "config": {"workload": "llama3-8b-q4_k_m greedy decode batch 1 at context %d (C restatement of the "
                                   "reference CPU path)" % args.prompt,
                       "model": "Llama-3-8B shape", "global_batch": 1, "seq_len": args.prompt},
            "cpu_baseline": {"value": r["tok_s"], "unit": "tok/s", "cores": r["cores"], "kind": "port",
                             "sample": r["sample"]},
            "e2e": {"value": r["tok_s"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------- GPU arm
def _timed(torch, fn, reps: int) -> float:
    """Mean seconds per call of fn over `reps` calls, CUDA events on the
    launching stream, after 3 warm-up calls.  The calls are captured into a
    CUDA graph and replayed, so the figure is device time per call, not the
    Python/ctypes launch rate (a small GEMV finishes faster than the host can
    issue the next call); if capture is refused the calls run eagerly."""
    for _ in range(3):
        fn(0)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    try:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, capture_error_mode="thread_local"):
            for i in range(reps):
                fn(i)
        g.replay()
        torch.cuda.synchronize()
        st = torch.cuda.current_stream()
        e0.record(st)
        g.replay()
        e1.record(st)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / 1e3 / reps
    except Exception:  # capture not possible: eager loop
        torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    e0.record(st)
    for i in range(reps):
        fn(i)
    e1.record(st)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / 1e3 / reps


def gemv_roofline(torch, eng_cfg, model_file, device, peaks) -> dict:
    """Times the dominant kernel alone with CUDA events: the fused Q4_K
    gate/up GEMV of Llama-3-8B (2 x [14336 x 4096] Q4_K), rotating across
    the 32 layers' weights so no launch is served from L2."""
    from overfit_b200.kernels import Q4KDotKernel, Q4KWeight

    FF, D = eng_cfg["d_ff"], eng_cfg["d_model"]
    layers = model_file["layers"]
    gates = [Q4KWeight(torch.from_numpy(L["gate"][1]).to(device), D, FF) for L in layers]
    ups = [Q4KWeight(torch.from_numpy(L["up"][1]).to(device), D, FF) for L in layers]
    x = torch.randn(D, device=device)
    g, u = torch.empty(FF, device=device), torch.empty(FF, device=device)
    q = torch.empty(D, dtype=torch.int8, device=device)
    s = torch.empty(D // 256, device=device)
    b = torch.empty(D // 16, dtype=torch.int16, device=device)
    n = len(gates)
    dt = _timed(torch, lambda i: Q4KDotKernel.project_gate_up_parallel(x, gates[i % n], ups[i % n], g, u, q, s, b),
                4 * n)
    alg = 2 * FF * D // 256 * 144 + 4 * D + 2 * 4 * FF  # weights + x + outputs
    achieved = alg / dt / 1e9
    peak = peaks.get("hbm_gbs", 6650.0)
    del gates, ups
    return {"bound": "hbm", "kernel": "gemv_kernel (Q4_K gate+up pair, 2x14336x4096)", "achieved": achieved,
            "peak": peak, "unit": "GB/s", "frac": achieved / peak, "traffic": None,
            "traffic_note": "one ncu capture of `bench.py --profile-target gemv_gateup`: 66.78 MB DRAM read+write per launch (1.009x algorithmic)",
            "launch_us": dt * 1e6, "algorithmic_bytes": alg,
            "peak_source": "MEASURED_PEAKS.json hbm_gbs (measured)" if "hbm_gbs" in peaks else "fallback 6650"}


def gemv_config1(torch, device, peaks) -> dict:
    """the single Q4_K projection y = W x (ProjectParallel:
    the Q8_K quantization of x and the GEMV), W [N x 4096] ~ N(0, 0.02) from
    seed 0 quantized by the reference's Q4_K scheme, x ~ N(0, 1), N = 4096 and
    14336.  Copies of W rotate so the weights in flight exceed 4x L2."""
    from overfit_b200.kernels import GgmlQuant, Q4KDotKernel, Q4KWeight

    K = 4096
    peak = peaks.get("hbm_gbs", 6650.0)
    out = {}
    for N in (4096, 14336):
        g = torch.Generator(device=device).manual_seed(0)
        w = GgmlQuant.quantize_q4_k(torch.randn(N, K, device=device, generator=g) * 0.02, K, N)
        copies = max(2, -(-4 * 126 * 2 ** 20 // w.numel()))
        ws = [Q4KWeight(w.clone(), K, N) for _ in range(copies)]
        x = torch.randn(K, device=device, generator=g)
        y = torch.empty(N, device=device)
        q = torch.empty(K, dtype=torch.int8, device=device)
        s = torch.empty(K // 256, device=device)
        b = torch.empty(K // 16, dtype=torch.int16, device=device)
        dt = _timed(torch, lambda i: Q4KDotKernel.project_parallel(x, ws[i % copies], None, y, q, s, b), 8 * copies)
        alg = N * K // 256 * 144 + 4 * K + 4 * N
        out[str(N)] = {"us": dt * 1e6, "achieved_gbs": alg / dt / 1e9, "frac": alg / dt / 1e9 / peak,
                       "algorithmic_bytes": alg, "rotating_copies": copies}
        del ws, w
    return {"kernel": "gemv_kernel via ovf_kq_project (Q4_K, K=4096)", "peak_gbs": peak, "unit": "GB/s",
            "rows": out}


def prefill_gemm(torch, device) -> dict:
    """the prefill projection (ProjectBatched /
    ProjectBatchedWeightStationary) on a [14336 x 4096] weight, Q4_K and
    Q8_0, M in {1, 16, 128, 512, 2048} activation rows ~ N(0, 1), CUDA-event
    timed over 4 rotating weight copies (quantization of the rows included).
    2*M*N*K integer operations per launch."""
    from overfit_b200.kernels import GgmlQuant, Q4KDotKernel, Q4KWeight, Q8DotKernel, Q8Weight, tc_scratch_bytes

    N, K = 14336, 4096
    g = torch.Generator(device=device).manual_seed(0)
    w32 = torch.randn(N, K, device=device, generator=g) * 0.02
    q4 = [Q4KWeight(GgmlQuant.quantize_q4_k(w32, K, N).clone(), K, N) for _ in range(4)]
    q8g = GgmlQuant.quantize_q8_0(w32)
    q8 = [Q8Weight.from_gguf(q8g, K, N) for _ in range(4)]
    del w32
    out = {}
    for M in (1, 16, 128, 512, 2048):
        x = torch.randn(M * K, device=device, generator=g)
        y = torch.empty(M * N, device=device)
        aq = torch.empty(M * K, dtype=torch.int8, device=device)
        a4 = torch.empty(M * K // 256, device=device)
        ab = torch.empty(M * K // 16, dtype=torch.int16, device=device)
        a8 = torch.empty(M * K // 32, device=device)
        reps = 8 if M >= 512 else 32
        d4 = _timed(torch, lambda i: Q4KDotKernel.project_batched(x, M, q4[i % 4], None, y, aq, a4, ab), reps)
        d8 = _timed(torch, lambda i: Q8DotKernel.project_batched(x, M, q8[i % 4], None, y, aq, a8), reps)
        sc = torch.empty(tc_scratch_bytes(M, K), dtype=torch.uint8, device=device)
        dt = _timed(torch, lambda i: Q4KDotKernel.project_batched_tensor_cores(x, M, q4[i % 4], None, y, aq, a4, ab,
                                                                               sc), reps)
        d8t = _timed(torch, lambda i: Q8DotKernel.project_batched_tensor_cores(x, M, q8[i % 4], None, y, aq, a8, sc),
                     reps)
        out[str(M)] = {"q4_k_us": d4 * 1e6, "q4_k_int_tops": 2 * M * N * K / d4 / 1e12,
                       "q4_k_tc_us": dt * 1e6, "q4_k_tc_tops": 2 * M * N * K / dt / 1e12,
                       "q8_0_us": d8 * 1e6, "q8_0_int_tops": 2 * M * N * K / d8 / 1e12,
                       "q8_0_tc_us": d8t * 1e6, "q8_0_tc_tops": 2 * M * N * K / d8t / 1e12}
        del sc
    return {"kernel": "batched_project_kernel (weight-stationary, dp4a); tc_q4k_project_kernel (tcgen05 kind::f16, "
                      "exact-integer operands); tc_q80_project_kernel (tcgen05 kind::i8)", "n": N, "k": K, "rows": out}


def qwen_config3(torch, device) -> dict:
    """Qwen2-0.5B-shaped Q8_0 model (seed 1), 128-token
    uniform-random prompt, 256 greedy decode steps, batch 1, on the F32 KV
    cache (the reference's default; exact attention order)."""
    from overfit_b200 import engine

    cfg = dict(engine.QWEN2_05B)
    mf = engine.synthetic_model(cfg, seed=1, device=device)
    eng = engine.CudaLlamaInferenceEngine(cfg, mf, device=device)
    out = {}
    for kv in ("f32", "f16"):
        s = eng.create_session(128 + 256 + 16, kv)
        prompt = np.random.default_rng(3).integers(0, cfg["vocab"], 128)
        t0 = time.perf_counter()
        s.prefill(prompt)
        pf = time.perf_counter() - t0
        s.generate_greedy(3)
        st = torch.cuda.ExternalStream(s.stream_handle, device=device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(device)
        e0.record(st)
        s.generate_greedy(253)
        e1.record(st)
        torch.cuda.synchronize(device)
        dt = e0.elapsed_time(e1) / 1e3
        out[kv] = {"tok_s": 253 / dt, "ms_per_token": dt / 253 * 1e3, "prefill_s": pf}
        s.close()
    eng.close()
    return {"model": "Qwen2-0.5B shape, Q8_0, tied embeddings, q/k/v bias", "prompt": 128, "steps": 256,
            "kv_caches": out, "weight_bytes_per_step": None}


def sessions16(torch, eng, cfg, prompt, steps, device) -> dict:
    """BASELINE config 4 at 16 concurrent sessions: the 2048-token prompt is
    prefilled once and restored into 16 sessions (RestorePrefix), each then
    takes a different token; `steps` rounds of one decode in every session
    as one batch (ovf_session_decode_batch, weights read once per round).
    Aggregate tokens / s by the host clock (each round returns to the host)."""
    n = 16
    base = eng.create_session(len(prompt) + steps + 8, "f16")
    base.prefill(prompt)
    snap = base.save_prefix()
    base.close()
    ss = [eng.create_session(len(prompt) + steps + 8, "f16") for _ in range(n)]
    toks = []
    for i, s in enumerate(ss):
        s.restore_prefix(snap)
        toks.append(s.prefill([1000 + 17 * i]))
    for _ in range(2):
        toks = list(eng.decode_batch(ss, toks, want_logits=False))
    torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    for _ in range(steps):
        toks = list(eng.decode_batch(ss, toks, want_logits=False))
    dt = time.perf_counter() - t0
    for s in ss:
        s.close()
    return {"sessions": n, "rounds": steps, "tok_s": n * steps / dt, "ms_per_round": dt / steps * 1e3,
            "context": len(prompt), "kv_cache": "f16"}


def max_over_ranks(value: float, device=None) -> float:
    """The job's time: the max of every rank's device-timed interval
    (all-reduce MAX over the process group; NCCL on GPUs, gloo on CPU)."""
    import torch
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64,
                     device=f"cuda:{device}" if device is not None else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def replica_value(steps_per_rank: int, world: int, seconds: float) -> float:
    """Whole-job throughput when every rank decodes its own stream of
    steps_per_rank tokens and the job ends with the slowest rank."""
    return world * steps_per_rank / seconds


def run_ours(args):
    import torch

    rank, world, local = dist_env()
    group = None
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
        group = dist.group.WORLD
    device = local
    torch.cuda.set_device(device)
    from overfit_b200 import build, engine

    build.build()
    cfg = dict(engine.LLAMA3_8B)
    if args.layers:
        cfg["n_layers"] = args.layers
    peaks = {}
    pp = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(pp):
        peaks = json.load(open(pp))
    extra = world == 1 and not args.no_extra and not args.layers

    # every rank draws the same weights (seeded device generator) and keeps
    # its tensor-parallel shard of them
    t0 = time.time()
    mf = engine.synthetic_model(cfg, seed=1, device=device)
    eng = engine.CudaLlamaInferenceEngine(cfg, mf, device=device, tp_group=group)
    gen_s = time.time() - t0
    e2e_steps = min(args.steps, 64)
    max_ctx = args.prompt + args.warmup + args.steps + e2e_steps + 64
    prompt = np.random.default_rng(1234).integers(0, cfg["vocab"], args.prompt).astype(np.int32)

    # the reference's own cache types (F32, its default, and Q8), attended in
    # the reference's exact order, timed on shorter runs beside the
    # benchmark config's fp16 cache
    exact = {}
    if extra and args.kv == "f16":
        for kvx in ("f32", "q8"):
            sx = eng.create_session(max_ctx, kvx)
            sx.prefill(prompt)
            sx.generate_greedy(args.warmup)
            stx = torch.cuda.ExternalStream(sx.stream_handle, device=device)
            ex0, ex1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            nx = min(args.steps, 64)
            torch.cuda.synchronize(device)
            ex0.record(stx)
            sx.generate_greedy(nx)
            ex1.record(stx)
            torch.cuda.synchronize(device)
            dtx = ex0.elapsed_time(ex1) / 1e3
            exact[kvx] = {"kv_cache": kvx, "value": nx / dtx, "unit": "tok/s", "steps": nx,
                          "ms_per_step": dtx / nx * 1e3}
            sx.close()

    sess = eng.create_session(max_ctx, args.kv)
    t0 = time.time()
    sess.prefill(prompt)
    prefill_s = time.time() - t0
    sess.generate_greedy(args.warmup)

    stream = torch.cuda.ExternalStream(sess.stream_handle, device=device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(device)
    clocks = ClockSampler(device)
    clocks.start()
    time.sleep(0.3)
    e0.record(stream)
    toks = sess.generate_greedy(args.steps)
    e1.record(stream)
    torch.cuda.synchronize(device)
    clk = clocks.stop()
    dt = max_over_ranks(e0.elapsed_time(e1) / 1e3, device)
    value = args.steps / dt  # one sequence's tokens: the whole job's output

    # e2e: the session call with host buffers (token in, argmax out), host clock
    tok = int(toks[-1])
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(device)
    h0 = time.perf_counter()
    for _ in range(e2e_steps):
        tok = sess.decode(tok, want_logits=False)
    e2e_dt = max_over_ranks(time.perf_counter() - h0, device)
    e2e = e2e_steps / e2e_dt

    weight_bytes = eng.weight_bytes
    # K and V of every layer read once per step, at the run's mean context
    kv_elem = 2 if args.kv == "f16" else 4
    kv_bytes = 2 * cfg["n_layers"] * cfg["n_kv_heads"] * cfg["head_dim"] * kv_elem * (args.prompt + args.warmup +
                                                                                      args.steps // 2)
    roof = gemv_roofline(torch, cfg, mf, device, peaks) if rank == 0 and world == 1 and not args.layers else None
    cfg1 = gemv_config1(torch, device, peaks) if extra else None
    pgemm = prefill_gemm(torch, device) if extra else None
    multi = sessions16(torch, eng, cfg, prompt, min(args.steps, 32), device) if extra else None
    sess.close()
    eng.close()
    del mf
    qwen = qwen_config3(torch, device) if extra else None
    launches_per_step = (2 + 5 * cfg["n_layers"]) if world == 1 else (3 + 7 * cfg["n_layers"])
    cpu = None
    if rank == 0 and extra and not args.no_cpu_baseline:
        try:
            r = cpu_decode_sample(args.prompt, 5)
            cpu = {"value": r["tok_s"], "unit": "tok/s", "cores": r["cores"], "kind": "port", "sample": r["sample"]}
        except Exception as ex:  # report, never fail the GPU line
            cpu = {"value": None, "unit": "tok/s", "cores": None, "kind": "port", "sample": f"failed: {ex}"}
    if rank == 0:
        # bytes every rank streams per step: its shard (world == 1: all)
        step_bytes = weight_bytes + kv_bytes // world
        hbm = peaks.get("hbm_gbs", 6650.0)
        line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "int8 dot (Q4_K/Q6_K/Q8_0 x Q8_K/Q8_0), fp32 accum",
                "data": "synthetic (random-init N(0,0.02), quantized on device)",
                "config": {"workload": "llama3-8b-q4_k_m greedy decode batch 1, prompt %d, %s KV cache"
                                       % (args.prompt, args.kv),
                           "kv_cache": args.kv,
                           "model": "Llama-3-8B shape" + ("" if not args.layers else f" ({args.layers} layers)"),
                           "global_batch": 1, "seq_len": args.prompt,
                           "parallelism": "tp%d" % world if world > 1 else "single GPU",
                           "l2": "inputs larger than L2 (%.2f GB of weights per step per GPU)" % (weight_bytes / 1e9)},
                "bytes_per_step_per_gpu": step_bytes,
                "step_roofline": {"bound": "hbm", "tok_s_bound": hbm * 1e9 / step_bytes,
                                  "frac": value / (hbm * 1e9 / step_bytes)},
                "roofline": roof, "cpu_baseline": cpu, "clocks": clk,
                "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4,
                        "clock": "host perf_counter around ovf_session_decode calls"},
                "gpu_launches": launches_per_step * args.steps,
                "f32_kv_exact": exact.get("f32"),
                "q8_kv_exact": exact.get("q8"),
                "gemv_config1": cfg1,
                "prefill_gemm_config2": pgemm,
                "qwen2_05b_config3": qwen,
                "sessions16_config4": multi,
                "setup_s": {"model_gen_upload": gen_s, "prefill": prefill_s}}
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


# ------------------------------------------------------- profile targets
def _prof_attn(kv: str):
    """3 warm-up + 3 timed launches of the exact decode attention at the
    Llama-3-8B layout (32 query / 8 KV heads, hd 128) over 2048 cached
    positions."""
    import torch

    from overfit_b200 import build
    from overfit_b200.kernels import CachedAttentionKernel as A

    build.build()
    H, KVH, hd, seq = 32, 8, 128, 2048
    dt = torch.float16 if kv == "f16" else torch.float32
    g = torch.Generator(device="cuda").manual_seed(0)
    kc = torch.randn(KVH, seq, hd, device="cuda", generator=g).to(dt)
    vc = torch.randn(KVH, seq, hd, device="cuda", generator=g).to(dt)
    q = torch.randn(H * hd, device="cuda", generator=g)
    out = torch.empty(H * hd, device="cuda")
    fn = A.compute_single_head_f16_all if kv == "f16" else A.compute_single_head_all
    for _ in range(6):
        fn(q, kc, vc, out, H, KVH, hd, seq, 1.0 / hd ** 0.5)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(20):
        fn(q, kc, vc, out, H, KVH, hd, seq, 1.0 / hd ** 0.5)
    e1.record()
    torch.cuda.synchronize()
    print(json.dumps({"profile_target": f"attn_exact_{kv}", "launches": 26, "us_per_launch": e0.elapsed_time(e1) * 50}))


def _prof_gemv_gateup():
    """3 warm-up + 3 launches of the fused Q4_K gate/up GEMV (2 x 14336 x
    4096), rotating over 8 weight pairs (264 MB, larger than L2)."""
    import torch

    from overfit_b200 import build
    from overfit_b200.kernels import GgmlQuant, Q4KDotKernel, Q4KWeight

    build.build()
    FF, D = 14336, 4096
    g = torch.Generator(device="cuda").manual_seed(0)
    ws = []
    for _ in range(8):
        a = GgmlQuant.quantize_q4_k(torch.randn(FF, D, device="cuda", generator=g) * 0.02, D, FF)
        b = GgmlQuant.quantize_q4_k(torch.randn(FF, D, device="cuda", generator=g) * 0.02, D, FF)
        ws.append((Q4KWeight(a, D, FF), Q4KWeight(b, D, FF)))
    x = torch.randn(D, device="cuda", generator=g)
    gy, uy = torch.empty(FF, device="cuda"), torch.empty(FF, device="cuda")
    q = torch.empty(D, dtype=torch.int8, device="cuda")
    s = torch.empty(D // 256, device="cuda")
    bs = torch.empty(D // 16, dtype=torch.int16, device="cuda")
    for i in range(6):
        Q4KDotKernel.project_gate_up_parallel(x, ws[i % 8][0], ws[i % 8][1], gy, uy, q, s, bs)
    torch.cuda.synchronize()
    print(json.dumps({"profile_target": "gemv_gateup", "launches": 6}))


def _prof_gemv_config1(N: int):
    """3 warm-up + 3 launches of the config-1 Q4_K projection (ProjectParallel,
    K = 4096) over 8 rotating weight copies."""
    import torch

    from overfit_b200 import build
    from overfit_b200.kernels import GgmlQuant, Q4KDotKernel, Q4KWeight

    build.build()
    K = 4096
    g = torch.Generator(device="cuda").manual_seed(0)
    w = GgmlQuant.quantize_q4_k(torch.randn(N, K, device="cuda", generator=g) * 0.02, K, N)
    ws = [Q4KWeight(w.clone(), K, N) for _ in range(8)]
    x = torch.randn(K, device="cuda", generator=g)
    y = torch.empty(N, device="cuda")
    q = torch.empty(K, dtype=torch.int8, device="cuda")
    s = torch.empty(K // 256, device="cuda")
    b = torch.empty(K // 16, dtype=torch.int16, device="cuda")
    for i in range(6):
        Q4KDotKernel.project_parallel(x, ws[i % 8], None, y, q, s, b)
    torch.cuda.synchronize()
    print(json.dumps({"profile_target": f"gemv_config1_{N}", "launches": 6}))


def _prof_prefill_tc(M: int):
    """2 warm-up + 2 launches of the tensor-core Q4_K prefill projection,
    M activation rows x [14336 x 4096], over 2 weight copies (0.7 GB)."""
    import torch

    from overfit_b200 import build
    from overfit_b200.kernels import GgmlQuant, Q4KDotKernel, Q4KWeight, tc_scratch_bytes

    build.build()
    N, K = 14336, 4096
    g = torch.Generator(device="cuda").manual_seed(0)
    w = GgmlQuant.quantize_q4_k(torch.randn(N, K, device="cuda", generator=g) * 0.02, K, N)
    ws = [Q4KWeight(w.clone(), K, N) for _ in range(2)]
    x = torch.randn(M * K, device="cuda", generator=g)
    y = torch.empty(M * N, device="cuda")
    q = torch.empty(M * K, dtype=torch.int8, device="cuda")
    s = torch.empty(M * K // 256, device="cuda")
    b = torch.empty(M * K // 16, dtype=torch.int16, device="cuda")
    sc = torch.empty(tc_scratch_bytes(M, K), dtype=torch.uint8, device="cuda")
    for i in range(4):
        Q4KDotKernel.project_batched_tensor_cores(x, M, ws[i % 2], None, y, q, s, b, sc)
    torch.cuda.synchronize()
    print(json.dumps({"profile_target": f"prefill_tc_{M}", "launches": 4}))


def _prof_prefill_layers():
    """A 2048-token prefill (8 chunks of 256 rows) through 2 layers of the
    Llama-3-8B shape (Q4_K_M, fp16 KV cache): every per-layer launch of the
    batched prefill, for a launch list."""
    import time

    import torch

    from overfit_b200 import build, engine

    build.build()
    cfg = dict(engine.LLAMA3_8B, n_layers=2)
    mf = engine.synthetic_model(cfg, seed=1, device=0)
    eng = engine.CudaLlamaInferenceEngine(cfg, mf, device=0)
    s = eng.create_session(2048 + 8, "f16")
    prompt = np.random.default_rng(5).integers(0, cfg["vocab"], 2048)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    s.prefill(prompt)
    dt = time.perf_counter() - t0
    s.close()
    eng.close()
    print(json.dumps({"profile_target": "prefill_2layers", "prefill_s": dt}))


PROFILE_TARGETS = {
    "prefill_2layers": _prof_prefill_layers,
    "prefill_tc_512": lambda: _prof_prefill_tc(512),
    "gemv_config1_4096": lambda: _prof_gemv_config1(4096),
    "gemv_config1_14336": lambda: _prof_gemv_config1(14336),
    "attn_exact_f16": lambda: _prof_attn("f16"),
    "attn_exact_f32": lambda: _prof_attn("f32"),
    "gemv_gateup": _prof_gemv_gateup,
}


def main():
    args = parse()
    if args.profile_target:
        PROFILE_TARGETS[args.profile_target]()
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
