"""Benchmark: Qwen3-4B Q4_K_M batch-1 decode on B200, one JSON line.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload decode|gemv|...]

decode (default): synthetic random-init Q4_K_M weights
of the Qwen3-4B shapes, fp16 KV cache pre-filled with N(0,1) to 4095
positions; each step decodes one token at position 4095 (context 4096) with
the greedy token fed back on the device. N > 1 (torchrun, one process per
GPU) shards the model tensor-parallel over NCCL; value is tok/s of the
whole job (strong scaling: the same model and token stream at every N).
The same line carries two sub-objects measured on the same engine, each
with its own clock record, roofline and CPU baseline: "prefill" (a
512-token prompt) and "batch" (64 sequences with
contexts uniform in [512, 4096], one token each per step, configs[4]).

gemv (BASELINE configs[0]/[1]): the Q4_K 9728x2560 matrix-vector product,
value in GB/s of algorithmic bytes, 20 distinct weight copies in rotation.
swiglu / attention / prefill / batch: parts of the default line alone
(profiling targets).

--impl reference: the reference's hot path on this host's CPU cores (the
C restatement in oracle/, OpenMP over output rows with one thread per host
core; the reference has no CPU implementation of its own, its test oracle
MatmulReference.hpp:42-64 is the only host dequant+dot), same metric and
config, its synthetic model built by oracle/ alone; rank 0 only.
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
    """nvidia-smi clocks and throttle reasons of every GPU of the job, one
    sample per GPU every 200 ms, from ONE nvidia-smi process on rank 0 that
    starts before the model is built: its start-up (about a second on an
    8-GPU host, during which eight concurrent per-rank samplers were seen to
    stall a tensor-parallel step) stays outside every timed region. Each timed
    region registers a record with begin()/end(); stop() fills the records
    from the samples stamped inside their regions."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, devices=()):
        self.devices = list(devices)
        self.proc = None
        self.records = []

    @staticmethod
    def gpu_ids(devices) -> list:
        """nvidia-smi ids of CUDA devices: their UUIDs (CUDA_VISIBLE_DEVICES
        renumbers devices, nvidia-smi does not), else the indices."""
        try:
            import torch

            ids = []
            for d in devices:
                u = str(torch.cuda.get_device_properties(d).uuid)
                ids.append(u if u.startswith("GPU-") else "GPU-" + u)
            return ids
        except Exception:
            return [str(d) for d in devices]

    def start(self):
        if not self.devices:
            return
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200", "-i",
                 ",".join(self.gpu_ids(self.devices))], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def begin(self) -> dict:
        rec = {"_t0": time.time()}
        self.records.append(rec)
        return rec

    @staticmethod
    def end(rec: dict):
        rec["_t1"] = time.time()

    @staticmethod
    def _stamp(s: str) -> float:
        import datetime

        return datetime.datetime.strptime(s.strip(), "%Y/%m/%d %H:%M:%S.%f").timestamp()

    def stop(self):
        rows = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            for line in out.splitlines():
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 10:
                    continue
                try:
                    rows.append((self._stamp(parts[0]), float(parts[2]), float(parts[3]),
                                 [p.lower().startswith("active") for p in parts[6:10]]))
                except ValueError:
                    continue
        for rec in self.records:
            t0, t1 = rec.pop("_t0"), rec.pop("_t1", time.time())
            rec.update(self.summary(rows, t0, t1))

    def summary(self, rows, t0, t1) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        inside = [r for r in rows if t0 - 0.05 <= r[0] <= t1 + 0.05]
        where = "inside the timed region"
        if not inside:
            # a region shorter than the sampling period: the samples within
            # half a second of it (warm-up before, the e2e loop after)
            inside = [r for r in rows if t0 - 0.5 <= r[0] <= t1 + 0.5]
            where = "within 0.5 s of the timed region (shorter than the 200 ms period)"
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"], "samples": 0}
        loaded = [r for r in inside if r[1] > 0.5 * r[2]] or inside
        return {"sm_mhz": statistics.median(r[1] for r in loaded), "sm_max_mhz": max(r[2] for r in inside),
                "reasons": sorted({self.REASONS[i] for r in loaded for i in range(4) if r[3][i]}),
                "samples": len(loaded), "gpus": len(self.devices), "window": where}


CLOCKS = ClockSampler()


def dist_init():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# --------------------------------------------------------------- CPU leg
# The CPU legs (cpu_baseline and --impl reference) build the synthetic model
# with oracle/ alone: the process never loads the product library.
def _oracle():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as o

    return o


def cpu_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_threads() -> int:
    """Threads the oracle's OpenMP regions get when asked for one per host
    core (explicitly, so that torchrun's OMP_NUM_THREADS=1 does not apply)."""
    return _oracle().omp_threads(cpu_cores())


def cpu_model(layers: int | None = None, ctx_rows: int = POS):
    """The seeded synthetic model (oracle/q4k_synth.c) and fp32 KV caches
    holding the fp16 N(0,1) fill for positions [0, ctx_rows); `layers`
    limits the model to its first layers (bounded CPU samples)."""
    from concurrent.futures import ThreadPoolExecutor

    o = _oracle()
    c = o.qwen3_4b_config(CTX)
    if layers is not None:
        c = dict(c, layers=layers)
    specs = [t for t in o.model_tensors(c)]
    with ThreadPoolExecutor(max_workers=4) as ex:
        datas = list(ex.map(lambda t: o.synth_tensor(SEED, t[0], t[1], t[2], t[3]), specs))
    model = o.Model(c, {t[0]: (t[1], d) for t, d in zip(specs, datas)})
    L, KVH, D = c["layers"], c["kv_heads"], c["head_dim"]
    kc = np.zeros((L, CTX, KVH * D), np.float32)
    vc = np.zeros_like(kc)

    def fill(job):
        layer, kv = job
        arr = kc if kv == "k" else vc
        for h in range(KVH):
            vals = o.synth_f16(SEED, f"kv.{layer}.{kv}", h * (1 << 20) * D, ctx_rows * D)
            arr[layer, :ctx_rows, h * D:(h + 1) * D] = vals.view(np.float16).astype(np.float32).reshape(ctx_rows, D)

    if ctx_rows:
        with ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
            list(ex.map(fill, [(layer, kv) for layer in range(L) for kv in ("k", "v")]))
    return model, kc.ravel(), vc.ravel()


def cpu_decode_steps(model, kc, vc, steps: int, threads: int, pos: int = POS) -> float:
    t0 = time.perf_counter()
    tok = TOKEN0
    for _ in range(steps):
        tok, _, _ = model.forward(kc, vc, CTX, [tok], pos, kv_round_f16=True, want_logits=False, want_hidden=False,
                                  threads=threads)
    return time.perf_counter() - t0


def cpu_prefill_sample(threads: int, n: int = 512) -> dict:
    """A 512-token prompt pass timed through one and through two layers of
    the model (embedding and head included in both); the whole pass is
    estimated as t1 + 35 x (t2 - t1)."""
    rng = np.random.default_rng(SEED)
    toks = rng.integers(0, 151936, n).astype(np.uint32)
    times = {}
    for layers in (1, 2):
        model, kc, vc = cpu_model(layers=layers, ctx_rows=0)
        t0 = time.perf_counter()
        model.forward(kc, vc, CTX, toks, 0, kv_round_f16=True, want_logits=False, want_hidden=False, threads=threads)
        times[layers] = time.perf_counter() - t0
        del model, kc, vc
    per_layer = max(times[2] - times[1], 1e-9)
    total = times[1] + 35 * per_layer
    return {"value": round(n / total, 3), "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"a {n}-token prompt through 1 and 2 of the 36 layers (+ embedding and head) on {threads} host "
                      f"threads, whole pass estimated as t1 + 35 x (t2 - t1) = {total:.2f} s; oracle/q4k_oracle.c "
                      "restating Engine.cpp:37-114 with tokens = 512"}


def cpu_batch_sample(threads: int, positions, seqs: int = 2) -> dict:
    """The reference serves each sequence as its own session: `seqs` of the
    batch's sequences decoded one after the other at their own contexts."""
    model, kc, vc = cpu_model()
    t = 0.0
    for p in positions[:seqs]:
        t += cpu_decode_steps(model, kc, vc, 1, threads, pos=int(p))
    return {"value": round(seqs / t, 4), "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"{seqs} of the 64 sequences (contexts {', '.join(str(int(p) + 1) for p in positions[:seqs])}), "
                      f"one decode step each, one after the other as separate sessions, on {threads} host threads"}


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


def make_engine(q, torch, world, rank, local, dist, sequences: int = 1):
    """The synthetic Qwen3-4B on this rank (its tensor-parallel shard when
    world > 1), KV positions [0, 4095) of every sequence filled."""
    cfg = q.qwen3_4b_config(CTX)
    cfg.tp_rank, cfg.tp_world, cfg.device = rank, world, local
    cfg.sequences = sequences
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
    return eng, cfg


def max_over_ranks(torch, dist, secs: float) -> float:
    if dist is None:
        return secs
    t = torch.tensor([secs], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


PREFILL_N = 512
BATCH = 64


def batch_rows():
    """64 sequences with contexts uniform in [512, 4096]
    (seeded): positions of their new tokens, their sequence slots (not in
    index order) and their tokens."""
    rng = np.random.default_rng(SEED + BATCH)
    ctx = rng.integers(512, CTX + 1, BATCH)
    return ((ctx - 1).astype(np.int32), rng.permutation(BATCH).astype(np.int32),
            rng.integers(0, 151936, BATCH).astype(np.uint32))


def time_prefill(q, torch, eng, args, dist, local, peaks, world):
    """A 512-token prompt into sequence 1, from an
    empty cache, timed on the device; e2e with host token ids per call."""
    rng = np.random.default_rng(SEED)
    toks = rng.integers(0, eng.cfg.vocab, PREFILL_N).astype(np.uint32)
    warm = max(3, args.warmup)
    for _ in range(warm):
        eng.prefill_seq(1, toks, 0)
    stream = torch.cuda.ExternalStream(eng.stream)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk = CLOCKS.begin()
    t0 = time.perf_counter()
    ev0.record(stream)
    for _ in range(args.steps):
        eng.prefill_seq(1, toks, 0)
    ev1.record(stream)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    CLOCKS.end(clk)
    dev = max_over_ranks(torch, dist, ev0.elapsed_time(ev1) / 1e3) / args.steps
    wall = max_over_ranks(torch, dist, wall) / args.steps
    return {"metric": "Qwen3-4B prompt prefill tok/s (512-token prompt, BASELINE configs[3])",
            "value": round(PREFILL_N / dev, 1), "unit": "tok/s", "steps": args.steps, "warmup": warm,
            "ms_per_step": round(dev * 1e3, 3), "higher_is_better": True,
            "dtype": "fp16 tensor-core products of Q8-dequantised activations and dequantised weights, fp32 "
                     "accumulate; fp16 KV",
            "config": {"workload": "prefill of a 512-token prompt into an empty sequence", "seq_len": PREFILL_N,
                       "parallelism": f"tp{world}", "l2": "2.5 GB of weights streamed per prompt (larger than L2)"},
            "e2e": {"value": round(PREFILL_N / wall, 1), "unit": "tok/s", "h2d_bytes_per_step": 4 * PREFILL_N + 12,
                    "d2h_bytes_per_step": 8, "how": "q4k_engine_prefill_seq per prompt from host token ids, "
                                                   "synchronous, host wall clock (max over ranks)"},
            # embed; per layer 4 x (quantise + GEMM), split-K reduces, QK-norm/RoPE, attention
            # (+2 all-reduce and residual-add launches with tp); head GEMV; finish
            "gpu_launches": args.steps * (1 + 36 * (12 + (2 if world > 1 else 0)) + 2),
            "clocks": clk}


def prefill_roofline(q, torch, peaks):
    """The prefill's dominant product alone: ffn_gate/ffn_up SwiGLU over 512
    rows (quantise + tcgen05 GEMM, each launch pair timed with CUDA events)."""
    import ctypes as C

    n, K, N = PREFILL_N, 2560, 9728
    ws = []
    for nm in ("gate", "up"):
        buf = torch.empty(q.device_bytes(q.Q4_K, K, N), dtype=torch.uint8, device="cuda")
        q.check(q.lib().q4k_synth_tensor_device(SEED, f"bench.pf.{nm}".encode(), q.Q4_K, K, N, buf.data_ptr(), None))
        ws.append(buf)
    x = torch.empty(n * K, device="cuda")
    q.check(q.lib().q4k_synth_f32_device(SEED, b"bench.pf.x", n * K, x.data_ptr(), None))
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
    del ws, x, y
    return {"kernel": "prefill_quantise + prefill_gemm_kernel (ffn_gate/ffn_up SwiGLU, 512 x 2560 x 2x9728, Q4_K)",
            "bound": "tensor", "achieved": round(tf, 2), "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
            "frac": round(tf / peaks["bf16_tflops"], 4), "traffic": None, "algorithmic_flops": flops,
            "launch_us": round(launch * 1e6, 2),
            "peak_src": peaks["src"] + " (burst dense bf16 GEMM, kernel timed alone)"}


def time_batch(q, torch, eng, args, dist, local, peaks, world):
    """One decode step of 64 sequences at their own contexts (BASELINE
    configs[4]), the same positions every step (fixed contexts), greedy
    tokens fed back through the host as the C ABI returns them."""
    pos, seqs, toks = batch_rows()
    warm = max(3, args.warmup)
    for _ in range(warm):
        toks, _ = eng.decode_batch(seqs, toks, pos)
    stream = torch.cuda.ExternalStream(eng.stream)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk = CLOCKS.begin()
    t0 = time.perf_counter()
    ev0.record(stream)
    for _ in range(args.steps):
        toks, _ = eng.decode_batch(seqs, toks, pos)
    ev1.record(stream)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    CLOCKS.end(clk)
    dev = max_over_ranks(torch, dist, ev0.elapsed_time(ev1) / 1e3) / args.steps
    wall = max_over_ranks(torch, dist, wall) / args.steps
    cfg = eng.cfg
    # bytes a step must stream per GPU: this rank's weights once, its KV heads
    # of every sequence up to its position
    kv_bytes = int(np.sum(pos.astype(np.int64) + 1)) * cfg.layers * cfg.kv_heads * cfg.head_dim * 2 * 2 // world
    w_bytes = sum(q.device_bytes(t, a, b) for _, t, a, b in q.model_tensors(cfg) if t != q.F32) // world
    step_bytes = w_bytes + kv_bytes
    gbs = step_bytes / dev / 1e9
    return {"metric": "Qwen3-4B batched decode tok/s (64 sequences, contexts uniform in [512, 4096], fp16 KV, "
                      "BASELINE configs[4])",
            "value": round(BATCH / dev, 1), "unit": "tok/s", "steps": args.steps, "warmup": warm,
            "ms_per_step": round(dev * 1e3, 3), "higher_is_better": True,
            "dtype": "fp16 tensor-core products (M=64), fp16 KV, fp32 softmax and accumulation",
            "config": {"workload": "64 sequences x 1 token per step, contexts uniform in [512, 4096] (seeded)",
                       "global_batch": BATCH, "contexts": [int(pos.min()) + 1, int(pos.max()) + 1],
                       "parallelism": f"tp{world}",
                       "l2": f"{step_bytes / 1e9:.1f} GB streamed per step per GPU (weights + 64 caches)"},
            "roofline": {"kernel": "whole batched step", "bound": "hbm", "achieved": round(gbs, 1),
                         "peak": peaks["hbm_gbs"], "unit": "GB/s", "frac": round(gbs / peaks["hbm_gbs"], 4),
                         "traffic": None, "algorithmic_bytes": step_bytes,
                         "peak_src": peaks["src"] + " (copy bandwidth)"},
            "e2e": {"value": round(BATCH / wall, 1), "unit": "tok/s", "h2d_bytes_per_step": 12 * BATCH,
                    "d2h_bytes_per_step": 4 * BATCH + 4,
                    "how": "q4k_engine_decode_batch per step, host rows in, next tokens out, host wall clock"},
            "gpu_launches": args.steps * (1 + 36 * (11 + (2 if world > 1 else 0)) + 3 + (1 if world > 1 else 0)),
            "clocks": clk}


def tp_exchange_us(recs, layers: int) -> dict:
    """Cost of the fused all-reduce of a tensor-parallel decode step, from
    traced steps (q4k_engine_trace: [launch][CTA][slot] %globaltimer ns).
    A consumer of row-parallel partial sums (the QKV product of layers 1..,
    every gate/up product, the head) records slot 1 when its dependency wait
    returns and slot 5 once its activation, summed over the ranks' words, has
    landed: the interval is the all-reduce's cost on the critical path (the
    peers' words crossing NVLink, their skew, the loads), where one GPU only
    loads the activation."""
    per = []
    consumers = [5 * l for l in range(1, layers)] + [5 * l + 3 for l in range(layers)] + [5 * layers]
    for rec in recs:
        rec = np.asarray(rec).astype(np.int64)
        for launch in consumers:
            r = rec[launch]
            ok = (r[:, 1] > 0) & (r[:, 5] > 0)
            if ok.any():
                per.append(float(np.median(r[ok, 5] - r[ok, 1])) / 1e3)
    if not per:
        return {"us_per_allreduce": None, "allreduces_per_token": 2 * layers}
    return {"us_per_allreduce": round(float(np.median(per)), 3), "allreduces_per_token": 2 * layers,
            "us_p90": round(float(np.percentile(per, 90)), 3), "launches_sampled": len(per),
            "how": "traced steps: a partial-sum consumer's dependency-wait return to its rank-summed activation "
                   "landing, median over CTAs, then over the QKV, gate/up and head launches of 3 steps (rank 0)"}


def run_decode(args, world, rank, local):
    import torch

    import q4kb200 as q

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=__import__("datetime").timedelta(seconds=300))
    peaks = load_peaks()
    # one engine for the three workloads: sequence 0 decodes (batch 1),
    # sequence 1 takes the prompt, all 64 serve the batched step
    eng, cfg = make_engine(q, torch, world, rank, local, dist, sequences=BATCH)

    stream = torch.cuda.ExternalStream(eng.stream)
    eng.generate(TOKEN0, POS, max(args.warmup, 3), advance=False, want_tokens=False)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk = CLOCKS.begin()
    ev0.record(stream)
    eng.generate(TOKEN0, POS, args.steps, advance=False, want_tokens=False)
    ev1.record(stream)
    torch.cuda.synchronize()
    CLOCKS.end(clk)
    if dist:
        dist.barrier()
    secs = max_over_ranks(torch, dist, ev0.elapsed_time(ev1) / 1e3)

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
    e2e_secs = max_over_ranks(torch, dist, time.perf_counter() - t0)

    # the fused all-reduce, as its consumer sees it: traced steps (every rank
    # takes part; rank 0's records are read)
    exchange = None
    if dist:
        recs = []
        for _ in range(3):
            dist.barrier()
            recs.append(eng.trace(TOKEN0, POS))
        exchange = tp_exchange_us(recs, cfg.layers)

    prefill = time_prefill(q, torch, eng, args, dist, local, peaks, world)
    batch = time_batch(q, torch, eng, args, dist, local, peaks, world)
    eng.close()

    result = None
    if rank == 0:
        # dominant kernel: the fused RMSNorm + gate/up + SiLU product (28 MB of
        # Q4_K weights per layer, ~40% of the step's bytes), timed alone
        torch.cuda.empty_cache()
        N = 9728 // 256 // world * 256 if world > 1 else 9728
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
        prefill["roofline"] = prefill_roofline(q, torch, peaks)
        step_bytes = (2503489024 + 36 * 2 * CTX * 8 * 128 * 2) / world
        value = args.steps / secs
        # embed, 36 x 5, head, finish (with tp the row-parallel sums travel
        # inside the products; the step's one NCCL all-gather is not counted)
        kernels_per_step = 1 + 36 * 5 + 2
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
                         "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": None,
                         "algorithmic_bytes": sw_bytes, "launch_us": round(t_sw * 1e6, 3),
                         "peak_src": peaks["src"] + " (burst copy bandwidth, kernel timed alone)"},
            "gemv": gemv,
            "e2e": {"value": round(e2e_steps / e2e_secs, 2), "unit": "tok/s", "h2d_bytes_per_step": 12,
                    "d2h_bytes_per_step": 8, "steps": e2e_steps,
                    "how": "q4k_engine_decode per token (pinned H2D of token/position/advance, graph launch, "
                           "D2H of the token and the error word, stream sync), host wall clock"},
            "gpu_launches": kernels_per_step * args.steps,
            "clocks": clk,
            "tp_exchange": exchange,
            "prefill": prefill,
            "batch": batch,
        }
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return result


def run_step(args, world, rank, local):
    """The batch-1 decode step alone, one sequence (3.1 GB on the device):
    the command the decode profiles under profiles/ are captured with. The
    driver's line is the default workload."""
    import torch

    import q4kb200 as q

    torch.cuda.set_device(local)
    eng, _ = make_engine(q, torch, 1, 0, local, None, sequences=1)
    stream = torch.cuda.ExternalStream(eng.stream)
    eng.generate(TOKEN0, POS, max(args.warmup, 3), advance=False, want_tokens=False)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    eng.generate(TOKEN0, POS, args.steps, advance=False, want_tokens=False)
    ev1.record(stream)
    torch.cuda.synchronize()
    secs = ev0.elapsed_time(ev1) / 1e3
    eng.close()
    return {"metric": METRIC_DECODE, "value": round(args.steps / secs, 2), "unit": "tok/s", "n_gpus": 1,
            "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": round(secs / args.steps * 1e3, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "data": "synthetic",
            "config": {"workload": "decode step alone, one sequence (profiling)", "seq_len": CTX,
                       "parallelism": "tp1"}, "gpu_launches": args.steps * 183}


def run_gemv(args, world, rank, local):
    import torch

    import q4kb200 as q

    torch.cuda.set_device(local)
    peaks = load_peaks()
    clk = CLOCKS.begin()
    t = time_gemv(q, torch, q.Q4_K, 2560, 9728, copies=20, reps=args.steps)
    CLOCKS.end(clk)
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
                         "frac": round(gbs / peaks["hbm_gbs"], 4), "traffic": None,
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
                         "traffic": None, "algorithmic_bytes": b},
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
    """The prefill sub-object alone, plus the reference benchmark's
    first-token latency shape (a 23-token prompt, then one decode step;
    benchmark.cpp:86-91)."""
    import torch

    import q4kb200 as q

    torch.cuda.set_device(local)
    peaks = load_peaks()
    eng, cfg = make_engine(q, torch, 1, 0, local, None, sequences=2)
    out = time_prefill(q, torch, eng, args, None, local, peaks, 1)
    rng = np.random.default_rng(SEED + 23)
    short = rng.integers(0, cfg.vocab, 23).astype(np.uint32)
    firsts = []
    for _ in range(5):
        a = time.perf_counter()
        nxt, _ = eng.prefill(short, 0)
        eng.decode(nxt, 23)
        firsts.append(time.perf_counter() - a)
    eng.close()
    out.update({"n_gpus": 1, "scaling": "weak", "vs_baseline": None, "data": "synthetic (seeded random-init Q4_K_M "
                "weights, random token ids)", "roofline": prefill_roofline(q, torch, peaks),
                "first_token_ms": round(min(firsts) * 1e3, 3),
                "first_token_note": "23-token prompt prefill + 1 decode step, host wall clock (the reference "
                                    "benchmark's 'first token' shape; the reference publishes 186.5 ms on an RTX "
                                    "4060 Laptop GPU)"})
    return out


def run_batch(args, world, rank, local):
    """The batch sub-object alone."""
    import torch

    import q4kb200 as q

    torch.cuda.set_device(local)
    peaks = load_peaks()
    eng, cfg = make_engine(q, torch, 1, 0, local, None, sequences=BATCH)
    out = time_batch(q, torch, eng, args, None, local, peaks, 1)
    eng.close()
    out.update({"n_gpus": 1, "scaling": "weak", "vs_baseline": None,
                "data": "synthetic (seeded random-init Q4_K_M weights and N(0,1) fp16 KV)"})
    return out


def cpu_steps_for(step_s: float, steps: int, budget_s: float = 150.0) -> int:
    """Steps of the CPU arm: the requested count, unless that would run
    longer than `budget_s`, then as many as fit (at least one)."""
    return max(1, min(steps, int(budget_s / max(step_s, 1e-9))))


def run_reference(args, world, rank):
    if rank != 0:
        return None
    threads = cpu_threads()
    model, kc, vc = cpu_model()
    first = cpu_decode_steps(model, kc, vc, 1, threads)
    warm = max(0, min(args.warmup, cpu_steps_for(first, args.warmup, 30.0)) - 1)
    if warm:
        cpu_decode_steps(model, kc, vc, warm, threads)
    steps = cpu_steps_for(first, args.steps)
    secs = cpu_decode_steps(model, kc, vc, steps, threads)
    value = steps / secs
    out = {"impl": "reference", "metric": METRIC_DECODE, "value": round(value, 4), "unit": "tok/s", "n_gpus": world,
           "steps": steps, "warmup": warm + 1, "ms_per_step": round(secs / steps * 1e3, 2), "higher_is_better": True,
           "scaling": "strong", "vs_baseline": None, "dtype": "fp32 activations (Q8-quantised), double accumulate",
           "data": "synthetic (the same seeded weights and KV as the GPU arm, generated by oracle/q4k_synth.c)",
           "config": {"workload": "decode batch 1 at context 4096 (BASELINE configs[2])", "model": MODEL,
                      "global_batch": 1, "seq_len": CTX, "parallelism": "cpu"},
           "cpu_baseline": {"value": round(value, 4), "unit": "tok/s", "cores": threads, "kind": "port",
                            "sample": f"{steps} full decode steps (36 layers + head, context 4096) on {threads} "
                                      "OpenMP threads; oracle/q4k_oracle.c restating MatmulReference.hpp:42-64 "
                                      "and Engine.cpp:37-114"},
           "e2e": {"value": round(value, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if steps < args.steps or warm + 1 < args.warmup:
        out["steps_cap"] = (f"{args.steps} steps / {args.warmup} warm-up requested; {steps} / {warm + 1} run to keep "
                            "the CPU arm within a few minutes (one step took "
                            f"{first:.2f} s)")
    return out


def attach_cpu_baselines(out: dict) -> None:
    """Rank 0 at N = 1: the oracle on this host's cores, bounded samples of
    the line's three workloads."""
    threads = cpu_threads()
    model, kc, vc = cpu_model()
    cpu_decode_steps(model, kc, vc, 1, threads)
    secs = cpu_decode_steps(model, kc, vc, 1, threads)
    out["cpu_baseline"] = {"value": round(1 / secs, 4), "unit": "tok/s", "cores": threads, "kind": "port",
                           "sample": f"1 full decode step (36 layers + head, context 4096) on {threads} OpenMP "
                                     "threads, oracle/q4k_oracle.c (MatmulReference.hpp:42-64 restated, OpenMP over "
                                     "output rows)"}
    if "batch" in out:
        pos, _, _ = batch_rows()
        t = 0.0
        for p in pos[:2]:
            t += cpu_decode_steps(model, kc, vc, 1, threads, pos=int(p))
        out["batch"]["cpu_baseline"] = {
            "value": round(2 / t, 4), "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"2 of the 64 sequences (contexts {int(pos[0]) + 1}, {int(pos[1]) + 1}), one decode step each, "
                      f"one after the other as separate sessions (the reference's way), on {threads} OpenMP threads"}
    del model, kc, vc
    if "prefill" in out:
        out["prefill"]["cpu_baseline"] = cpu_prefill_sample(threads)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=("decode", "step", "gemv", "swiglu", "attention", "prefill", "batch"),
                    default="decode")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    world, rank, local = dist_init()

    if args.impl == "reference":
        out = run_reference(args, world, rank)
        if out is not None:
            print(json.dumps(out), flush=True)
        return

    if rank == 0 and args.workload != "step":
        # one sampler for the job's GPUs (one process per GPU on one node:
        # rank r drives local device r), started before any model is built
        CLOCKS.devices = list(range(world)) if world > 1 else [local]
        CLOCKS.start()
    if args.workload == "decode":
        out = run_decode(args, world, rank, local)
    elif args.workload == "step":
        out = run_step(args, world, rank, local) if rank == 0 else None
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
    CLOCKS.stop()
    if rank == 0 and out is not None:
        if world == 1 and args.workload in ("decode", "prefill", "batch") and not args.no_cpu_baseline:
            if args.workload == "decode":
                attach_cpu_baselines(out)
            elif args.workload == "prefill":
                out["cpu_baseline"] = cpu_prefill_sample(cpu_threads())
            else:
                attach_cpu_baselines(tmp := {"batch": out})
                out["cpu_baseline"] = tmp["batch"]["cpu_baseline"]
        elif args.workload == "gemv" and not args.no_cpu_baseline:
            o = _oracle()
            raw = o.synth_tensor(SEED, "bench.cpu", o.Q4_K, 2560, 9728)
            x = o.synth_f32(SEED, "bench.x", 2560)
            threads = cpu_threads()
            o.matmul(x, raw, o.Q4_K, 2560, 9728, threads=threads)
            reps = 20
            t0 = time.perf_counter()
            for _ in range(reps):
                o.matmul(x, raw, o.Q4_K, 2560, 9728, threads=threads)
            t = (time.perf_counter() - t0) / reps
            b = 9728 * o.row_bytes(o.Q4_K, 2560) + 2560 * 4 + 9728 * 4
            out["cpu_baseline"] = {"value": round(b / t / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                                   "sample": f"{reps} Q4_K 9728x2560 products on {threads} OpenMP threads"}
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
