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
Multi-GPU (torchrun, N > 1): independent replicas, one per GPU ("replicas
only" until tensor parallelism lands); value = sum over ranks with the
max-over-ranks time.
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
    ap.add_argument("--no-f32-line", action="store_true", help="skip the extra F32-KV (exact) measurement")
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
def cpu_decode_sample(n_tokens: int, threads: int | None = None) -> dict:
    """Times the reference CPU path (the C restatement, OpenMP over all host
    threads) on the same Llama-3-8B Q4_K_M decode: 32 layers that share one
    layer's weights (each token still streams 32 x 148 MB of layer weights
    plus the 431 MB LM head from DRAM, as the full model would; the
    working set is far above the host caches) at a short context."""
    from oracle import oracle as orc
    from overfit_b200.engine import LLAMA3_8B as cfg

    if threads:
        orc.set_threads(threads)
    cores = orc.num_threads()
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
    L = dict(attn_norm=np.ones(D, np.float32), ffn_norm=np.ones(D, np.float32))
    L["wq"] = (orc.Q4_K, qmat(H * hd, D, orc.quantize_q4k, 1), None, H * hd, D)
    L["wk"] = (orc.Q4_K, qmat(KVH * hd, D, orc.quantize_q4k, 2), None, KVH * hd, D)
    L["wv"] = (orc.Q6_K, qmat(KVH * hd, D, orc.quantize_q6k, 3), None, KVH * hd, D)
    wo = qmat(D, H * hd, orc.quantize_q4k, 4)
    q, s = orc.requant_q8_0(orc.Q4_K, wo, D, H * hd)
    L["wo"] = (orc.Q8_0, q, s, D, H * hd)
    L["gate"] = (orc.Q4_K, qmat(FF, D, orc.quantize_q4k, 5), None, FF, D)
    L["up"] = (orc.Q4_K, qmat(FF, D, orc.quantize_q4k, 6), None, FF, D)
    L["down"] = (orc.Q6_K, qmat(D, FF, orc.quantize_q6k, 7), None, D, FF)
    weights = dict(layers=[L] * cfg["n_layers"], embed=(orc.Q4_K, qmat(V, D, orc.quantize_q4k, 8), None, V, D),
                   final_norm=np.ones(D, np.float32), lm_head=(orc.Q6_K, qmat(V, D, orc.quantize_q6k, 9), None, V, D))
    gen_s = time.time() - t0
    sess = orc.OracleSession(cfg, weights, max_ctx=n_tokens + 8)
    sess.decode(1)  # warm-up token
    t0 = time.perf_counter()
    tok = 1
    for _ in range(n_tokens):
        lg = sess.decode(tok)
        tok = int(np.argmax(lg))
    dt = time.perf_counter() - t0
    return {"tok_s": n_tokens / dt, "s_per_token": dt / n_tokens, "cores": cores, "gen_s": gen_s,
            "sample": f"{n_tokens} greedy decode tokens of the full 32-layer + LM-head Llama-3-8B Q4_K_M step "
                      f"(layers share one layer's weights), context <= {n_tokens + 1}"}


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    steps = max(1, min(args.steps, 16))
    r = cpu_decode_sample(steps)
    line = {"impl": "reference", "metric": METRIC, "value": r["tok_s"], "unit": "tok/s", "n_gpus": 0,
            "steps": steps, "warmup": 1, "ms_per_step": r["s_per_token"] * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8 dot / fp32", "data": "synthetic",
            "config": {"workload": "llama3-8b-q4_k_m greedy decode, batch 1 (CPU restatement of the reference)",
                       "model": "Llama-3-8B shape", "global_batch": 1},
            "cpu_baseline": {"value": r["tok_s"], "unit": "tok/s", "cores": r["cores"], "kind": "port",
                             "sample": r["sample"]},
            "e2e": {"value": r["tok_s"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------- GPU arm
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
    for i in range(3):
        Q4KDotKernel.project_gate_up_parallel(x, gates[i % n], ups[i % n], g, u, q, s, b)
    torch.cuda.synchronize()
    reps = 4 * n
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for i in range(reps):
        Q4KDotKernel.project_gate_up_parallel(x, gates[i % n], ups[i % n], g, u, q, s, b)
    e1.record(st)
    torch.cuda.synchronize()
    dt = e0.elapsed_time(e1) / 1e3 / reps
    alg = 2 * FF * D // 256 * 144 + 4 * D + 2 * 4 * FF  # weights + x + outputs
    achieved = alg / dt / 1e9
    peak = peaks.get("hbm_gbs", 6650.0)
    del gates, ups
    return {"bound": "hbm", "kernel": "gemv_kernel (Q4_K gate+up pair, 2x14336x4096)", "achieved": achieved,
            "peak": peak, "unit": "GB/s", "frac": achieved / peak, "traffic": profiled_traffic(),
            "launch_us": dt * 1e6, "algorithmic_bytes": alg,
            "peak_source": "MEASURED_PEAKS.json hbm_gbs (measured)" if "hbm_gbs" in peaks else "fallback 6650"}


def prefill_gemm(torch, eng_cfg, model_file, device) -> dict:
    """Config-2 prefill projection: the weight-stationary batched Q4_K
    kernel (ProjectBatchedWeightStationary) on the gate matrices
    [14336 x 4096] for M activation rows, CUDA-event timed, rotating over the
    layers' weights.  2*M*N*K integer multiply-adds per launch."""
    from overfit_b200.kernels import Q4KDotKernel, Q4KWeight

    FF, D = eng_cfg["d_ff"], eng_cfg["d_model"]
    layers = model_file["layers"][:8]
    gates = [Q4KWeight(torch.from_numpy(L["gate"][1]).to(device), D, FF) for L in layers]
    out = {}
    for M in (16, 128, 512):
        x = torch.randn(M * D, device=device)
        y = torch.empty(M * FF, device=device)
        q = torch.empty(M * D, dtype=torch.int8, device=device)
        s = torch.empty(M * D // 256, device=device)
        b = torch.empty(M * D // 16, dtype=torch.int16, device=device)
        for i in range(3):
            Q4KDotKernel.project_batched(x, M, gates[i % len(gates)], None, y, q, s, b)
        torch.cuda.synchronize()
        reps = 2 * len(gates)
        st = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for i in range(reps):
            Q4KDotKernel.project_batched(x, M, gates[i % len(gates)], None, y, q, s, b)
        e1.record(st)
        torch.cuda.synchronize()
        dt = e0.elapsed_time(e1) / 1e3 / reps
        out[str(M)] = {"us": dt * 1e6, "int_tops": 2 * M * FF * D / dt / 1e12}
    del gates
    return {"kernel": "batched_project_kernel (Q4_K, 14336 x 4096, quantize included)", "rows": out}


def profiled_traffic():
    """DRAM bytes per launch of the gate/up GEMV from the committed ncu
    summary (profiles/gemv_q4k_gateup.md, line `traffic_bytes_per_launch:`),
    or None when no capture has been summarised."""
    p = os.path.join(ROOT, "profiles", "gemv_q4k_gateup.md")
    try:
        for ln in open(p):
            if ln.strip().startswith("traffic_bytes_per_launch:"):
                return float(ln.split(":", 1)[1].strip().split()[0])
    except OSError:
        pass
    return None


def max_over_ranks(value: float, device=None) -> float:
    """The job's time for a weak-scaling replica run: the max of every
    rank's device-timed interval (all-reduce MAX over the process group; the
    NCCL group on GPUs, gloo on CPU)."""
    import torch
    import torch.distributed as dist

    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64,
                     device=f"cuda:{device}" if device is not None else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def replica_value(steps_per_rank: int, world: int, seconds: float) -> float:
    """Whole-job throughput: every rank decodes steps_per_rank tokens of its
    own session; the job is done when the slowest rank is."""
    return world * steps_per_rank / seconds


def run_ours(args):
    import torch

    rank, world, local = dist_env()
    if world > 1:
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
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

    t0 = time.time()
    mf = engine.synthetic_model(cfg, seed=1, device=device)
    eng = engine.CudaLlamaInferenceEngine(cfg, mf, device=device)
    gen_s = time.time() - t0
    max_ctx = args.prompt + args.warmup + args.steps + 64
    prompt = np.random.default_rng(1234 + rank).integers(0, cfg["vocab"], args.prompt).astype(np.int32)

    # The reference's default F32 KV cache (exact attention order), timed on
    # a shorter run and reported beside the benchmark config's fp16 cache.
    # The reference's own cache types (F32, its default, and Q8), attended in
    # the reference's exact order, timed on shorter runs beside the
    # benchmark config's fp16 cache.
    exact = {}
    if args.kv == "f16" and not args.no_f32_line:
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
            dtx = max_over_ranks(ex0.elapsed_time(ex1) / 1e3, device)
            exact[kvx] = {"kv_cache": kvx, "value": replica_value(nx, world, dtx), "unit": "tok/s", "steps": nx,
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
    value = replica_value(args.steps, world, dt)

    # e2e: the session call with host buffers (token in, argmax out).
    e2e_steps = min(args.steps, 64)
    tok = int(toks[-1])
    torch.cuda.synchronize(device)
    e0.record(stream)
    for _ in range(e2e_steps):
        tok = sess.decode(tok, want_logits=False)
    e1.record(stream)
    torch.cuda.synchronize(device)
    e2e_dt = max_over_ranks(e0.elapsed_time(e1) / 1e3, device)
    e2e = replica_value(e2e_steps, world, e2e_dt)

    weight_bytes = eng.weight_bytes
    # K and V of every layer read once per step, at the run's mean context
    kv_elem = 2 if args.kv == "f16" else 4
    kv_bytes = 2 * cfg["n_layers"] * cfg["n_kv_heads"] * cfg["head_dim"] * kv_elem * (args.prompt + args.warmup +
                                                                                      args.steps // 2)
    roof = gemv_roofline(torch, cfg, mf, device, peaks) if rank == 0 else None
    pgemm = prefill_gemm(torch, cfg, mf, device) if rank == 0 and not args.layers else None
    sess.close()
    eng.close()
    del mf
    launches_per_step = 1 + 5 * cfg["n_layers"] + 1
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            r = cpu_decode_sample(6)
            cpu = {"value": r["tok_s"], "unit": "tok/s", "cores": r["cores"], "kind": "port", "sample": r["sample"]}
        except Exception as ex:  # report, never fail the GPU line
            cpu = {"value": None, "unit": "tok/s", "cores": None, "kind": "port", "sample": f"failed: {ex}"}
    if rank == 0:
        step_bytes = weight_bytes + kv_bytes
        hbm = peaks.get("hbm_gbs", 6650.0)
        line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "int8 dot (Q4_K/Q6_K/Q8_0 x Q8_K/Q8_0), fp32 accum",
                "data": "synthetic (random-init N(0,0.02), quantized on device)",
                "config": {"workload": "llama3-8b-q4_k_m greedy decode batch 1, prompt %d, %s KV cache"
                                       % (args.prompt, args.kv),
                           "kv_cache": args.kv,
                           "model": "Llama-3-8B shape" + ("" if not args.layers else f" ({args.layers} layers)"),
                           "global_batch": world, "seq_len": args.prompt, "parallelism": f"replicas x{world}",
                           "l2": "inputs larger than L2 (%.2f GB of weights per step)" % (weight_bytes / 1e9)},
                "bytes_per_step": step_bytes,
                "step_roofline": {"bound": "hbm", "tok_s_bound": hbm * 1e9 / step_bytes,
                                  "frac": value / world / (hbm * 1e9 / step_bytes)},
                "roofline": roof, "cpu_baseline": cpu, "clocks": clk,
                "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4},
                "gpu_launches": launches_per_step * args.steps,
                "f32_kv_exact": exact.get("f32"),
                "q8_kv_exact": exact.get("q8"),
                "prefill_gemm": pgemm,
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


PROFILE_TARGETS = {
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
