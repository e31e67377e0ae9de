"""Benchmark: Qwen3-4B Q4_K_M batch-1 decode on B200, one JSON line.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload decode|gemv]

decode (default): synthetic random-init Q4_K_M weights
of the Qwen3-4B shapes, fp16 KV cache pre-filled with N(0,1) to 4095
positions; each step decodes one token at position 4095 (context 4096) with
the greedy token fed back on the device. N > 1 (torchrun, one process per
GPU) shards the model tensor-parallel over NCCL; value is tok/s of the
whole job (strong scaling: the same model and token stream at every N).

gemv (BASELINE configs[0]/[1]): the Q4_K 9728x2560 matrix-vector product,
value in GB/s of algorithmic bytes, 20 distinct weight copies in rotation.
swiglu / attention: the decode step's fused gate/up product and its decode
attention alone (profiling targets).

--impl reference: the reference's hot path on this host's CPU cores (the
C restatement in oracle/, OpenMP over output rows; the reference has no CPU
implementation of its own, its test oracle MatmulReference.hpp:42-64 is the
only host dequant+dot), same metric and config; rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "qwen3-4b-q4_k_m-inference-engine_b200", "python"))

SEED = 0x5EED
CTX = 4096
POS = CTX - 1
TOKEN0 = 4242
MODEL = "Qwen3-4B-Q4_K_M (synthetic random-init weights, BASELINE configs[2])"
METRIC_DECODE = "Qwen3-4B decode tok/s (batch 1, context 4096, fp16 KV)"
METRIC_GEMV = "Q4_K GEMV 9728x2560 HBM GB/s"


def load_peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p.get("bf16_tflops", 1590.0)), "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.t0 = self.t1 = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200", "-i",
                 str(self.device)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def mark(self, begin: bool):
        if begin:
            self.t0 = time.time()
        else:
            self.t1 = time.time()

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = []
        for line in out.splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[4:]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        loaded = [r for r in rows if r[0] > 0.5 * r[1]] or rows
        names = ["active", "hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in loaded for i in range(1, 5) if r[2][i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(loaded)}


def dist_init():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# --------------------------------------------------------------- CPU leg
def cpu_decode_model(threads: int = 0):
    """Host copies of the same synthetic weights and KV cache for the oracle."""
    from concurrent.futures import ThreadPoolExecutor

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as o
    import q4kb200 as q

    cfg = q.qwen3_4b_config(CTX)
    specs = q.model_tensors(cfg)
    with ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        datas = list(ex.map(lambda s: q.synth_tensor_host(SEED, s[0], s[1], s[2], s[3]), specs))
    tensors = {s[0]: (s[1], d) for s, d in zip(specs, datas)}
    c = cfg.as_dict()
    model = o.Model(c, tensors)
    L, KVH, D = c["layers"], c["kv_heads"], c["head_dim"]
    kc = np.zeros((L, CTX, KVH * D), np.float32)
    vc = np.zeros_like(kc)

    def fill(job):
        layer, kv = job
        arr = kc if kv == "k" else vc
        for h in range(KVH):
            vals = q.synth_f16_host(SEED, f"kv.{layer}.{kv}", h * (1 << 20) * D, POS * D)
            arr[layer, :POS, h * D:(h + 1) * D] = vals.view(np.float16).astype(np.float32).reshape(POS, D)

    with ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        list(ex.map(fill, [(layer, kv) for layer in range(L) for kv in ("k", "v")]))
    return model, kc.ravel(), vc.ravel()


def cpu_decode_steps(model, kc, vc, steps: int, threads: int = 0) -> float:
    t0 = time.perf_counter()
    tok = TOKEN0
    for _ in range(steps):
        tok, _, _ = model.forward(kc, vc, CTX, [tok], POS, kv_round_f16=True, want_logits=False, want_hidden=False,
                                  threads=threads)
    return time.perf_counter() - t0


def cpu_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ------------------------------------------------------------ GPU legs
def time_gemv(q, torch, qtype: int, K: int, N: int, copies: int, reps: int, swiglu: bool = False):
    """Average device time (s) of one product launch over `copies` distinct
    weight copies in rotation (together larger than L2), CUDA events on the
    launching stream."""
    import ctypes as C

    rows_b = q.device_bytes(qtype, K, N)
    nmat = 2 if swiglu else 1
    weights = torch.empty((copies * nmat, rows_b), dtype=torch.uint8, device="cuda")
    for i in range(copies * nmat):
        q.check(q.lib().q4k_synth_tensor_device(SEED + i, b"bench.w", qtype, K, N, weights[i].data_ptr(), None))
    x = torch.empty(K, device="cuda")
    q.check(q.lib().q4k_synth_f32_device(SEED, b"bench.x", K, x.data_ptr(), None))
    gamma = torch.ones(K, device="cuda")
    y = torch.empty(N, device="cuda")
    torch.cuda.synchronize()
    stream = torch.cuda.Stream()  # a capturable (non-default) stream
    sp = stream.cuda_stream
    L = q.lib()

    def launch(i):
        if swiglu:
            w = (C.c_void_p * 2)(weights[2 * i].data_ptr(), weights[2 * i + 1].data_ptr())
            rc = L.q4k_matmul_ex(x.data_ptr(), gamma.data_ptr(), 1e-6, 2, w, (C.c_int * 2)(qtype, qtype),
                                 (C.c_int64 * 2)(N, N), (C.c_void_p * 2)(y.data_ptr(), y.data_ptr()), K, 1,
                                 q.EPI_SWIGLU, None, None, sp)
        else:
            rc = L.q4k_matmul(x.data_ptr(), weights[i].data_ptr(), qtype, K, N, y.data_ptr(), 1, sp)
        q.check(rc)

    for i in range(3 * copies):
        launch(i % copies)
    torch.cuda.synchronize()
    # The launches are captured in a CUDA graph so that host-side call
    # overhead (ctypes, planning) does not starve the device between launches.
    per_graph = max(copies, min(reps, 4 * copies))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        sp = stream.cuda_stream
        for i in range(per_graph):
            launch(i % copies)
    replays = max(1, reps // per_graph)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):  # replay() launches on the current stream
        graph.replay()
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(replays):
            graph.replay()
        ev1.record(stream)
    torch.cuda.synchronize()
    secs = ev0.elapsed_time(ev1) / 1e3 / (replays * per_graph)
    del graph
    del weights
    torch.cuda.empty_cache()
    return secs


def time_attention(q, torch, kv_heads: int = 8, ctx: int = CTX, layers: int = 8, reps: int = 200):
    """Average device time (s) of one decode-attention launch at position
    ctx-1 over `layers` distinct fp16 KV caches in rotation (graph-timed)."""
    import ctypes as C

    H, D = 4 * kv_heads, 128
    k = torch.empty((layers, kv_heads * ctx * D), dtype=torch.int16, device="cuda").random_(0, 15000)
    v = torch.empty_like(k).random_(0, 15000)
    qkv = torch.randn((H + 2 * kv_heads) * D, device="cuda")
    g = torch.ones(D, device="cuda")
    pos = torch.tensor([ctx - 1], dtype=torch.int32, device="cuda")
    out = torch.empty(H * D, device="cuda")
    scratch = torch.zeros(q.lib().q4k_attention_decode_scratch_bytes(H, kv_heads), dtype=torch.uint8, device="cuda")
    stream = torch.cuda.Stream()
    L = q.lib()

    def launch(i):
        q.check(L.q4k_attention_decode_f16(qkv.data_ptr(), g.data_ptr(), g.data_ptr(), k[i].data_ptr(), v[i].data_ptr(),
                                           ctx, pos.data_ptr(), H, kv_heads, D, 1e-6, 1e6, out.data_ptr(),
                                           scratch.data_ptr(), stream.cuda_stream))

    torch.cuda.synchronize()
    for i in range(layers):
        launch(i)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(layers):
            launch(i)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    replays = max(1, reps // layers)
    with torch.cuda.stream(stream):
        graph.replay()
        torch.cuda.synchronize()
        ev0.record(stream)
        for _ in range(replays):
            graph.replay()
        ev1.record(stream)
    torch.cuda.synchronize()
    secs = ev0.elapsed_time(ev1) / 1e3 / (replays * layers)
    del graph, k, v
    torch.cuda.empty_cache()
    return secs, 2 * kv_heads * ctx * D * 2


def gemv_bytes(q, qtype, K, N, nmat=1, norm=False):
    return nmat * N * q.gguf_row_bytes(qtype, K) + K * 4 * (2 if norm else 1) + N * 4


def read_traffic(name: str):
    path = os.path.join(ROOT, "profiles", name)
    if not os.path.exists(path):
        return None
    with open(path) as f:
        for line in f:
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1])
    return None


def run_decode(args, world, rank, local):
    import torch

    import q4kb200 as q

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=__import__("datetime").timedelta(seconds=300))
    cfg = q.qwen3_4b_config(CTX)
    cfg.tp_rank, cfg.tp_world, cfg.device = rank, world, local
    nccl_id = None
    if world > 1:
        idt = torch.zeros(128, dtype=torch.uint8, device="cuda")
        if rank == 0:
            idt.copy_(torch.frombuffer(bytearray(q.nccl_unique_id()), dtype=torch.uint8))
        dist.broadcast(idt, 0)
        nccl_id = bytes(idt.cpu().numpy().tobytes())
    eng = q.Engine(cfg, nccl_id)
    eng.load_synthetic(SEED)
    eng.fill_kv_synthetic(SEED, POS)

    stream = torch.cuda.ExternalStream(eng.stream)
    clocks = ClockSampler(local)
    clocks.start()
    eng.generate(TOKEN0, POS, max(args.warmup, 3), advance=False, want_tokens=False)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks.mark(True)
    ev0.record(stream)
    eng.generate(TOKEN0, POS, args.steps, advance=False, want_tokens=False)
    ev1.record(stream)
    torch.cuda.synchronize()
    clocks.mark(False)
    if dist:
        dist.barrier()
    secs = ev0.elapsed_time(ev1) / 1e3
    if dist:
        t = torch.tensor([secs], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        secs = float(t.item())
    clk = clocks.stop()

    # e2e: the public API call per token, host buffers, H2D token+position,
    # D2H next token, synchronous (host wall clock, max over ranks)
    e2e_steps = max(min(args.steps, 200), 3)
    eng.decode(TOKEN0, POS)
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    tok = TOKEN0
    for _ in range(e2e_steps):
        tok, _, _ = eng.decode(tok, POS)
    e2e_secs = time.perf_counter() - t0
    if dist:
        t = torch.tensor([e2e_secs], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_secs = float(t.item())
    eng.close()

    result = None
    if rank == 0:
        peaks = load_peaks()
        # dominant kernel: the fused RMSNorm + gate/up + SiLU product (28 MB of
        # Q4_K weights per layer, ~40% of the step's bytes), timed alone
        torch.cuda.empty_cache()
        K, N = 2560, 9728 // world // 256 * 256 if world > 1 else 9728
        t_sw = time_gemv(q, torch, q.Q4_K, 2560, N, copies=8, reps=200, swiglu=True)
        sw_bytes = gemv_bytes(q, q.Q4_K, 2560, N, nmat=2, norm=True)
        achieved = sw_bytes / t_sw / 1e9
        gemv = {}
        for tag, qt, kk, nn in (("q4k_9728x2560", q.Q4_K, 2560, 9728), ("q6k_2560x9728", q.Q6_K, 9728, 2560),
                                ("q6k_151936x2560", q.Q6_K, 2560, 151936)):
            copies = 20 if nn * q.gguf_row_bytes(qt, kk) < 64e6 else 2
            t = time_gemv(q, torch, qt, kk, nn, copies=copies, reps=100 if copies > 2 else 20)
            gemv[tag] = {"us": round(t * 1e6, 3), "gbs": round(gemv_bytes(q, qt, kk, nn) / t / 1e9, 1),
                         "frac": round(gemv_bytes(q, qt, kk, nn) / t / 1e9 / peaks["hbm_gbs"], 4)}
        t_att, att_bytes = time_attention(q, torch, kv_heads=8 // world)
        gemv["attention_decode_ctx4096"] = {"us": round(t_att * 1e6, 3), "gbs": round(att_bytes / t_att / 1e9, 1),
                                            "frac": round(att_bytes / t_att / 1e9 / peaks["hbm_gbs"], 4)}
        step_bytes = (2503489024 + 36 * 2 * CTX * 8 * 128 * 2) / world
        value = args.steps / secs
        kernels_per_step = 1 + 36 * 5 + 2 + (72 if world > 1 else 0)
        result = {
            "metric": METRIC_DECODE,
            "value": round(value * 1.0, 2),
            "unit": "tok/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": max(args.warmup, 3),
            "ms_per_step": round(secs / args.steps * 1e3, 4),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "q4k/q6k weights, int8 activations (dp4a), fp32 accumulate, fp16 KV",
            "data": "synthetic (seeded random-init Q4_K_M weights and N(0,1) fp16 KV; no checkpoint)",
            "config": {"workload": "decode batch 1 at context 4096 (BASELINE configs[2])", "model": MODEL,
                       "global_batch": 1, "seq_len": CTX, "parallelism": f"tp{world}",
                       "l2": "inputs larger than L2: 3.1 GB of weights + KV streamed per step"},
            "step_roofline": {"bytes_per_step_per_gpu": step_bytes,
                              "achieved_gbs": round(step_bytes * value / 1e9, 1),
                              "frac": round(step_bytes * value / 1e9 / peaks["hbm_gbs"], 4),
                              "peak": peaks["hbm_gbs"], "peak_src": peaks["src"]},
            "roofline": {"kernel": "gemv_kernel<1,2> (RMSNorm + ffn_gate/ffn_up Q4_K 2560x9728 + SiLU)",
                         "bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(achieved / peaks["hbm_gbs"], 4),
                         "traffic": read_traffic("gemv_swiglu_q4k_2560x9728.md"),
                         "algorithmic_bytes": sw_bytes, "launch_us": round(t_sw * 1e6, 3),
                         "peak_src": peaks["src"] + " (burst copy bandwidth, kernel timed alone)"},
            "gemv": gemv,
            "e2e": {"value": round(e2e_steps / e2e_secs, 2), "unit": "tok/s", "h2d_bytes_per_step": 12,
                    "d2h_bytes_per_step": 8, "steps": e2e_steps,
                    "how": "q4k_engine_decode per token (pinned H2D of token/position/advance, graph launch, "
                           "D2H of the token and the error word, stream sync), host wall clock"},
            "gpu_launches": kernels_per_step * args.steps,
            "clocks": clk,
        }
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return result


def run_gemv(args, world, rank, local):
    import torch

    import q4kb200 as q

    torch.cuda.set_device(local)
    peaks = load_peaks()
    clocks = ClockSampler(local)
    clocks.start()
    clocks.mark(True)
    t = time_gemv(q, torch, q.Q4_K, 2560, 9728, copies=20, reps=args.steps)
    clocks.mark(False)
    clk = clocks.stop()
    b = gemv_bytes(q, q.Q4_K, 2560, 9728)
    gbs = b / t / 1e9
    return {"metric": METRIC_GEMV, "value": round(gbs, 1), "unit": "GB/s", "n_gpus": 1, "steps": args.steps,
            "warmup": 60, "ms_per_step": round(t * 1e3, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "q4k weights, int8 activations (dp4a), fp32 accumulate",
            "data": "synthetic (seeded)",
            "config": {"workload": "Q4_K GEMV 9728x2560 batch 1 (BASELINE configs[0])", "model": MODEL,
                       "global_batch": 1, "seq_len": 1, "parallelism": "replica",
                       "l2": "20 distinct weight copies (280 MB) in rotation"},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(gbs / peaks["hbm_gbs"], 4), "traffic": read_traffic("gemv_q4k_9728x2560.md"),
                         "algorithmic_bytes": b},
            "gpu_launches": args.steps, "clocks": clk}


def run_swiglu(args, world, rank, local):
    """The decode step's dominant kernel alone: RMSNorm + ffn_gate/ffn_up
    Q4_K 2560x9728 + SiLU*up in one launch, 8 distinct weight pairs
    (224 MB) in rotation: the profiling target behind the decode line's
    roofline object."""
    import torch

    import q4kb200 as q

    torch.cuda.set_device(local)
    peaks = load_peaks()
    t = time_gemv(q, torch, q.Q4_K, 2560, 9728, copies=8, reps=args.steps, swiglu=True)
    b = gemv_bytes(q, q.Q4_K, 2560, 9728, nmat=2, norm=True)
    gbs = b / t / 1e9
    return {"metric": "fused RMSNorm+gate/up+SiLU Q4_K 2x9728x2560 HBM GB/s", "value": round(gbs, 1),
            "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": 24, "ms_per_step": round(t * 1e3, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "q4k weights, int8 activations (dp4a), fp32 accumulate", "data": "synthetic (seeded)",
            "config": {"workload": "gate/up SwiGLU product, batch 1", "model": MODEL, "global_batch": 1,
                       "seq_len": 1, "parallelism": "replica", "l2": "8 distinct weight pairs (224 MB) in rotation"},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(gbs / peaks["hbm_gbs"], 4),
                         "traffic": read_traffic("gemv_swiglu_q4k_2560x9728.md"), "algorithmic_bytes": b},
            "gpu_launches": args.steps}


def run_attention(args, world, rank, local):
    """Decode attention alone (one layer's 8 KV heads at context 4096,
    8 caches in rotation): the profiling target for the attention kernel."""
    import torch

    import q4kb200 as q

    torch.cuda.set_device(local)
    peaks = load_peaks()
    t, b = time_attention(q, torch, kv_heads=8, reps=args.steps)
    gbs = b / t / 1e9
    return {"metric": "decode attention HBM GB/s (ctx 4096, 8 KV heads, fp16 KV)", "value": round(gbs, 1),
            "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": 8, "ms_per_step": round(t * 1e3, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp16 KV, fp32 softmax",
            "data": "synthetic", "config": {"workload": "attention decode, one layer", "model": MODEL,
                                            "global_batch": 1, "seq_len": CTX, "parallelism": "replica",
                                            "l2": "8 distinct caches (134 MB) in rotation"},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(gbs / peaks["hbm_gbs"], 4), "traffic": None, "algorithmic_bytes": b},
            "gpu_launches": args.steps}


def run_prefill(args, world, rank, local):
    """Prompt prefill (q4k_engine_prefill, the reference's Engine::inference
    over a whole prompt): a 512-token prompt on the synthetic Qwen3-4B, plus
    the reference benchmark's first-token latency shape (a 23-token prompt,
    then one decode step; benchmark.cpp:86-91). The roofline object is the
    tensor-core product behind it (ffn_gate/ffn_up SwiGLU at 512 rows)."""
    import ctypes as C

    import numpy as np
    import torch

    import q4kb200 as q

    torch.cuda.set_device(local)
    peaks = load_peaks()
    n = 512
    cfg = q.qwen3_4b_config(CTX)
    eng = q.Engine(cfg)
    eng.load_synthetic(SEED)
    rng = np.random.default_rng(SEED)
    toks = rng.integers(0, cfg.vocab, n).astype(np.uint32)
    for _ in range(max(3, args.warmup)):
        eng.prefill(toks, 0)
    steps = max(1, min(args.steps, 20))
    stream = torch.cuda.ExternalStream(eng.stream)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    ev0.record(stream)
    for _ in range(steps):
        eng.prefill(toks, 0)
    ev1.record(stream)
    torch.cuda.synchronize()
    wall = (time.perf_counter() - t0) / steps
    dev = ev0.elapsed_time(ev1) / 1e3 / steps
    # first-token latency: 23-token prompt + one decode step, host wall clock
    short = rng.integers(0, cfg.vocab, 23).astype(np.uint32)
    firsts = []
    for _ in range(5):
        a = time.perf_counter()
        nxt, _ = eng.prefill(short, 0)
        eng.decode(nxt, 23)
        firsts.append(time.perf_counter() - a)
    eng.close()
    # the dominant product alone, events around each launch pair (quantise + GEMM)
    K, N = 2560, 9728
    ws = []
    for nm in ("gate", "up"):
        raw = q.synth_tensor_host(SEED, f"bench.pf.{nm}", q.Q4_K, K, N)
        buf = torch.empty(q.device_bytes(q.Q4_K, K, N), dtype=torch.uint8, device="cuda")
        q.check(q.lib().q4k_weight_upload(q.Q4_K, K, N, q.hptr(raw), buf.data_ptr(), None))
        ws.append(buf)
    x = torch.from_numpy(q.synth_f32_host(SEED, "bench.pf.x", n * K)).cuda()
    y = torch.empty(n * N, device="cuda")
    call = lambda: q.check(q.lib().q4k_matmul_batch(
        x.data_ptr(), None, 0.0, 2, (C.c_void_p * 2)(ws[0].data_ptr(), ws[1].data_ptr()), (C.c_int * 2)(q.Q4_K, q.Q4_K),
        (C.c_int64 * 2)(N, N), (C.c_void_p * 2)(y.data_ptr(), y.data_ptr()), N, K, n, q.EPI_SWIGLU, None))
    for _ in range(3):
        call()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(20):
        call()
    e1.record()
    torch.cuda.synchronize()
    launch = e0.elapsed_time(e1) / 1e3 / 20
    flops = 2.0 * n * 2 * N * K
    tf = flops / launch / 1e12
    return {"metric": "Qwen3-4B prompt prefill tok/s (512-token prompt)", "value": round(n / dev, 1),
            "unit": "tok/s", "n_gpus": 1, "steps": steps, "warmup": max(3, args.warmup),
            "ms_per_step": round(dev * 1e3, 3), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "fp16 tensor-core products of Q8-dequantised activations and dequantised weights, fp32 accumulate",
            "data": "synthetic (seeded random-init Q4_K_M weights, random token ids)",
            "config": {"workload": "prefill of a 512-token prompt from an empty cache", "model": MODEL,
                       "global_batch": 1, "seq_len": n, "parallelism": "tp1",
                       "l2": "2.5 GB of weights streamed per prompt (larger than L2)"},
            "first_token_ms": round(min(firsts) * 1e3, 3),
            "first_token_note": "23-token prompt prefill + 1 decode step, host wall clock (reference benchmark.cpp "
                                "'first token' shape; BASELINE.md quotes 186.5 ms on an RTX 4060 Laptop GPU)",
            "roofline": {"kernel": "prefill_quantise + prefill_gemm_kernel (ffn_gate/ffn_up SwiGLU, 512 x 2560 x "
                                   "2x9728, Q4_K)", "bound": "tensor", "achieved": round(tf, 2),
                         "peak": peaks["bf16_tflops"], "unit": "TFLOP/s", "frac": round(tf / peaks["bf16_tflops"], 4),
                         "traffic": None, "algorithmic_flops": flops, "launch_us": round(launch * 1e6, 2)},
            "e2e": {"value": round(n / wall, 1), "unit": "tok/s", "h2d_bytes_per_step": 4 * n, "d2h_bytes_per_step": 8,
                    "how": "q4k_engine_prefill per prompt from host token ids, host wall clock"},
            # per 512-row prompt: embed; per layer 4 x (quantise + GEMM), 2 split-K
            # reduces (O, down), QK-norm/RoPE, attention; head GEMV; finish
            "gpu_launches": steps * (1 + 36 * 12 + 2)}


def run_batch(args, world, rank, local):
    """Batched decode (q4k_engine_decode_batch): 64 sequences, each at context
    4096 over the same synthetic cache rows, one new token per sequence per
    step; every step reads each weight once for all 64 (the tensor-core
    products) and each sequence's own 16.8 MB of fp16 K/V per layer."""
    import numpy as np
    import torch

    import q4kb200 as q

    torch.cuda.set_device(local)
    peaks = load_peaks()
    B = 64
    cfg = q.qwen3_4b_config(CTX)
    cfg.sequences = B
    eng = q.Engine(cfg)
    eng.load_synthetic(SEED)
    eng.fill_kv_synthetic(SEED, CTX - 1)
    rng = np.random.default_rng(SEED)
    seqs = np.arange(B, dtype=np.int32)
    pos = np.full(B, CTX - 1, np.int32)  # fixed context: each step re-decodes the last position
    toks = rng.integers(0, cfg.vocab, B).astype(np.uint32)
    for _ in range(max(3, args.warmup)):
        toks, _ = eng.decode_batch(seqs, toks, pos)
    steps = max(1, min(args.steps, 20))
    stream = torch.cuda.ExternalStream(eng.stream)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    ev0.record(stream)
    for _ in range(steps):
        toks, _ = eng.decode_batch(seqs, toks, pos)
    ev1.record(stream)
    torch.cuda.synchronize()
    wall = (time.perf_counter() - t0) / steps
    dev = ev0.elapsed_time(ev1) / 1e3 / steps
    eng.close()
    # bytes a step must stream: the weights once, each sequence's K/V
    kv_bytes = B * cfg.layers * cfg.kv_heads * CTX * cfg.head_dim * 2 * 2
    w_bytes = sum(q.device_bytes(t, a, b) for _, t, a, b in q.model_tensors(cfg) if t != q.F32)
    step_bytes = w_bytes + kv_bytes
    gbs = step_bytes / dev / 1e9
    return {"metric": "Qwen3-4B batched decode tok/s (64 sequences, context 4096, fp16 KV)",
            "value": round(B / dev, 1), "unit": "tok/s", "n_gpus": 1, "steps": steps,
            "warmup": max(3, args.warmup), "ms_per_step": round(dev * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "fp16 tensor-core products, fp16 KV, fp32 softmax and accumulation",
            "data": "synthetic (seeded random-init Q4_K_M weights and N(0,1) fp16 KV)",
            "config": {"workload": "64 sequences x 1 token per step at context 4096", "model": MODEL,
                       "global_batch": B, "seq_len": CTX, "parallelism": "tp1",
                       "l2": f"{step_bytes / 1e9:.1f} GB streamed per step (weights + 64 caches)"},
            "roofline": {"kernel": "whole step", "bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": round(gbs / peaks["hbm_gbs"], 4), "traffic": None,
                         "algorithmic_bytes": step_bytes},
            "e2e": {"value": round(B / wall, 1), "unit": "tok/s", "h2d_bytes_per_step": 12 * B,
                    "d2h_bytes_per_step": 4 * B + 4, "how": "q4k_engine_decode_batch per step, host wall clock"},
            "gpu_launches": steps * (1 + 36 * 11 + 3)}


def run_reference(args, world, rank):
    if rank != 0:
        return None
    steps = max(1, min(args.steps, 5))
    warm = 1
    model, kc, vc = cpu_decode_model()
    cpu_decode_steps(model, kc, vc, warm)
    secs = cpu_decode_steps(model, kc, vc, steps)
    value = steps / secs
    cores = cpu_cores()
    return {"impl": "reference", "metric": METRIC_DECODE, "value": round(value, 4), "unit": "tok/s", "n_gpus": world,
            "steps": steps, "warmup": warm, "ms_per_step": round(secs / steps * 1e3, 2), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "fp32 activations (Q8-quantised), double accumulate",
            "data": "synthetic (same seeded weights and KV as the GPU arm)",
            "config": {"workload": "decode batch 1 at context 4096 (BASELINE configs[2])", "model": MODEL,
                       "global_batch": 1, "seq_len": CTX, "parallelism": "cpu"},
            "cpu_baseline": {"value": round(value, 4), "unit": "tok/s", "cores": cores, "kind": "port",
                             "sample": f"{steps} full decode steps (36 layers + head, context 4096) on {cores} "
                                       "host threads; oracle/q4k_oracle.c restating MatmulReference.hpp:42-64 "
                                       "and Engine.cpp:37-114"},
            "e2e": {"value": round(value, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=("decode", "gemv", "swiglu", "attention", "prefill", "batch"),
                    default="decode")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    world, rank, local = dist_init()

    if args.impl == "reference":
        out = run_reference(args, world, rank)
        if out is not None:
            print(json.dumps(out), flush=True)
        return

    if args.workload == "decode":
        out = run_decode(args, world, rank, local)
    elif args.workload == "attention":
        out = run_attention(args, world, rank, local)
    elif args.workload == "swiglu":
        out = run_swiglu(args, world, rank, local)
    elif args.workload == "prefill":
        out = run_prefill(args, world, rank, local)
    elif args.workload == "batch":
        out = run_batch(args, world, rank, local)
    else:
        out = run_gemv(args, world, rank, local)
    if rank == 0 and out is not None:
        if world == 1 and args.workload == "decode" and not args.no_cpu_baseline:
            model, kc, vc = cpu_decode_model()
            cpu_decode_steps(model, kc, vc, 1)
            secs = cpu_decode_steps(model, kc, vc, 1)
            cores = cpu_cores()
            out["cpu_baseline"] = {"value": round(1 / secs, 4), "unit": "tok/s", "cores": cores, "kind": "port",
                                   "sample": f"1 full decode step (36 layers + head, context 4096) on {cores} host "
                                             "threads, oracle/q4k_oracle.c (MatmulReference.hpp:42-64 restated, "
                                             "OpenMP over output rows)"}
        elif args.workload == "gemv" and not args.no_cpu_baseline:
            sys.path.insert(0, os.path.join(ROOT, "oracle"))
            import oracle as o
            import q4kb200 as q

            raw = q.synth_tensor_host(SEED, "bench.cpu", q.Q4_K, 2560, 9728)
            x = q.synth_f32_host(SEED, "bench.x", 2560)
            o.matmul(x, raw, q.Q4_K, 2560, 9728)
            reps = 20
            t0 = time.perf_counter()
            for _ in range(reps):
                o.matmul(x, raw, q.Q4_K, 2560, 9728)
            t = (time.perf_counter() - t0) / reps
            cores = cpu_cores()
            out["cpu_baseline"] = {"value": round(gemv_bytes(q, q.Q4_K, 2560, 9728) / t / 1e9, 3), "unit": "GB/s",
                                   "cores": cores, "kind": "port",
                                   "sample": f"{reps} Q4_K 9728x2560 products on {cores} host threads"}
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
