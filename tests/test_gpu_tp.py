"""Tensor parallelism on two GPUs (q4k_engine_* with tp_world = 2 over NCCL).

Each rank holds its shard of the synthetic Qwen3-4B (column-parallel
q/k/v/gate/up, row-parallel attn_output/ffn_down followed by an all-reduce,
a vocabulary-sharded head) and runs a 40-token prompt through
q4k_engine_prefill (tensor-core products, all-reduced partial rows) and four
decode steps teacher-forced on a one-GPU engine's tokens. The two ranks'
logit shards, put together, must match the one-GPU engine's logits within
the whole-step bar, and the greedy tokens agree up to near-ties. Skipped
unless two CUDA devices are visible (the host-side sharding is covered on
CPU by test_tp_gloo.py).
"""
import os
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
PROMPT = 40
STEPS = 4


def _paths():
    for p in (os.path.join(ROOT, "qwen3-4b-q4_k_m-inference-engine_b200", "python"), os.path.join(HERE, "golden"), HERE):
        if p not in sys.path:
            sys.path.insert(0, p)


def _rank(rank, world, port, prompt, forced, out):
    """One tensor-parallel rank: prefill, then decode steps on `forced` tokens;
    puts (rank, [logit shard per step]) on `out`."""
    _paths()
    import datetime

    import torch
    import torch.distributed as dist

    import q4kb200 as q
    from tiny_model import SEED

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=datetime.timedelta(seconds=120))
    try:
        cfg = q.qwen3_4b_config(1024)
        cfg.tp_rank, cfg.tp_world, cfg.device = rank, world, rank
        idt = torch.zeros(128, dtype=torch.uint8, device="cuda")
        if rank == 0:
            idt.copy_(torch.frombuffer(bytearray(q.nccl_unique_id()), dtype=torch.uint8))
        dist.broadcast(idt, 0)
        eng = q.Engine(cfg, bytes(idt.cpu().numpy().tobytes()))
        eng.load_synthetic(SEED)
        shards = []
        _, logits = eng.prefill(np.asarray(prompt, np.uint32), 0, want_logits=True)
        shards.append(logits)
        for s, tok in enumerate(forced):
            _, logits, _ = eng.decode(int(tok), PROMPT + s, want_logits=True)
            shards.append(logits)
        eng.close()  # the engine's graphs (they hold NCCL calls) go before the process group
        dist.barrier()
        out.put((rank, shards))
    finally:
        dist.destroy_process_group()


def test_tp2_prefill_and_decode_match_one_gpu(cuda):
    import torch.multiprocessing as mp

    if cuda.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")
    _paths()
    import q4kb200 as q
    from conftest import rel_l2
    from test_gpu_engine import greedy_ok
    from tiny_model import SEED

    rng = np.random.default_rng(5)
    cfg = q.qwen3_4b_config(1024)
    prompt = rng.integers(0, cfg.vocab, PROMPT).astype(np.uint32)
    one = q.Engine(cfg)
    one.load_synthetic(SEED)
    tok, logits = one.prefill(prompt, 0, want_logits=True)
    want_tokens, want_logits = [tok], [logits]
    for s in range(STEPS):
        tok, logits, _ = one.decode(tok, PROMPT + s, want_logits=True)
        want_tokens.append(tok)
        want_logits.append(logits)
    one.close()
    cuda.cuda.synchronize()

    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = 29500 + (os.getpid() % 1000)
    procs = [ctx.Process(target=_rank, args=(r, 2, port, list(prompt), want_tokens[:STEPS], out)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in procs:
        r, shards = out.get(timeout=600)
        got[r] = shards
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    worst = 0.0
    for s in range(STEPS + 1):
        full = np.concatenate([got[0][s], got[1][s]])
        e = rel_l2(full, want_logits[s])
        worst = max(worst, e)
        assert e < 5e-2, (s, e)
        assert greedy_ok(int(np.argmax(full)), want_tokens[s], want_logits[s], full), s
    print(f"tp2 vs one GPU, prefill + {STEPS} teacher-forced steps: worst logits rel-L2 {worst:.2e}")
