"""Tensor-parallel decomposition on CPU: two gloo ranks apply the library's
own shard plan (q4k_tp_shard) to Qwen3-4B-shaped tensors, compute their
shard with the oracle, and combine with the collectives the engine uses
(all-reduce after the row-parallel attn_output / ffn_down products,
all-gather of per-shard (logit, index) for the output head). The combined
result must equal the unsharded oracle product (K-shards are whole 256-value
super-blocks, so every Q8 group is intact and only the summation order of
the partial sums changes)."""
import os
import socket
import sys

import numpy as np
import pytest


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, paths, out):
    for p in paths:
        sys.path.insert(0, p)
    import torch
    import torch.distributed as dist

    import oracle as o
    import q4kb200 as q

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = q.qwen3_4b_config(4096)
        specs = q.model_tensors(cfg)
        idx = {s[0]: i for i, s in enumerate(specs)}
        res = {}
        # row-parallel ffn_down (Q6_K, K = 9728 = 38 super-blocks) and attn_output (Q4_K, K = 4096)
        for name in ("blk.0.ffn_down.weight", "blk.1.attn_output.weight"):
            _, t, K, N = specs[idx[name]]
            N = 64  # a slice of output rows keeps the CPU work small
            full = q.synth_tensor_host(3, name, t, K, N)
            x = q.synth_f32_host(3, name + ".x", K)
            n0, n1, b0, b1 = q.tp_shard(cfg, idx[name], rank, world)
            rb = q.gguf_row_bytes(t, K)
            bs = 144 if t == q.Q4_K else 210
            shard = full.reshape(N, rb)[:, b0 * bs:b1 * bs].copy()
            part = o.matmul(x[b0 * 256:b1 * 256], shard.ravel(), t, (b1 - b0) * 256, N).ravel()
            tens = torch.from_numpy(part.copy())
            dist.all_reduce(tens)
            want = o.matmul(x, full, t, K, N).ravel()
            res[name] = float(np.max(np.abs(tens.numpy() - want)) / np.max(np.abs(want)))
        # column-parallel attn_q rows + the vocab-sharded greedy head
        name = "blk.0.attn_q.weight"
        _, t, K, N = specs[idx[name]]
        n0, n1, b0, b1 = q.tp_shard(cfg, idx[name], rank, world)
        res["q_rows"] = (n0, n1)
        vocab = 4096
        head = q.synth_tensor_host(3, "head", q.Q6_K, 2560, vocab)
        x = q.synth_f32_host(3, "head.x", 2560)
        logits = o.matmul(x, head, q.Q6_K, 2560, vocab).ravel().astype(np.float32)
        logits[100] = logits[3000] = logits.max() + 1  # a tie across the two shards
        v0, v1 = vocab * rank // world, vocab * (rank + 1) // world
        local = int(np.argmax(logits[v0:v1]))
        cand = torch.tensor([float(logits[v0 + local]), float(v0 + local)], dtype=torch.float64)
        gathered = [torch.zeros(2, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(gathered, cand)
        best = min(((-g[0].item(), int(g[1].item())) for g in gathered))
        res["argmax"] = (best[1], o.argmax(logits))
        out.put((rank, res))
    finally:
        dist.destroy_process_group()


def test_tp_two_ranks_gloo(root):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    paths = [os.path.join(root, "qwen3-4b-q4_k_m-inference-engine_b200", "python"), os.path.join(root, "oracle")]
    procs = [ctx.Process(target=_worker, args=(r, 2, port, paths, out)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(out.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(2):
        res = results[r]
        assert res["blk.0.ffn_down.weight"] < 1e-12
        assert res["blk.1.attn_output.weight"] < 1e-12
        assert res["argmax"][0] == res["argmax"][1] == 100
    assert results[0]["q_rows"] == (0, 2048) and results[1]["q_rows"] == (2048, 4096)
