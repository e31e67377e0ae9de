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


ROWS, BATCH, POS1 = 64, 8, 1000


def _tp_engine(q, rank, world, dist, torch):
    cfg = q.qwen3_4b_config(1024)
    cfg.sequences = BATCH
    cfg.tp_rank, cfg.tp_world, cfg.device = rank, world, rank
    nccl_id = None
    if world > 1:
        idt = torch.zeros(128, dtype=torch.uint8, device="cuda")
        if rank == 0:
            idt.copy_(torch.frombuffer(bytearray(q.nccl_unique_id()), dtype=torch.uint8))
        dist.broadcast(idt, 0)
        nccl_id = bytes(idt.cpu().numpy().tobytes())
    return q.Engine(cfg, nccl_id)


def _layer_chain(eng, inputs, seqs, pos, batch_tokens):
    """Every layer on the given inputs (the one-GPU engine's own chain):
    prompt rows (tensor-core products), one decode token, a batched step;
    then a whole batched decode step. Returns the outputs."""
    rows_in, tok_in, bat_in = inputs
    rows = [eng.layer_rows(i, rows_in[i], 0) for i in range(len(rows_in))]
    tok = [eng.layer(i, tok_in[i], POS1) for i in range(len(tok_in))]
    bat = [eng.layer_batch(i, bat_in[i], seqs, pos) for i in range(len(bat_in))]
    nxt, logits = eng.decode_batch(seqs, batch_tokens, pos, want_logits=True)
    return rows, tok, bat, nxt, logits


def _rank_layers(rank, world, port, inputs, seqs, pos, batch_tokens, out):
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
        eng = _tp_engine(q, rank, world, dist, torch)
        eng.load_synthetic(SEED)
        eng.fill_kv_synthetic(SEED, POS1)
        res = _layer_chain(eng, inputs, seqs, pos, batch_tokens)
        eng.close()
        dist.barrier()
        out.put((rank, res))
    finally:
        dist.destroy_process_group()


def test_tp2_layers_match_one_gpu(cuda):
    """tp2 against tp1 layer by layer, on identical inputs, for the three
    forms a layer runs in: a 64-row prompt pass (tensor-core GEMM, the
    row-parallel partial sums all-reduced), one decode token (GEMV), and a
    batched step of 8 sequences; then a whole batched decode step (head
    shards merged per row). Every layer within 1e-3 relative L2 of the one-GPU
    engine's; batched greedy tokens equal."""
    import torch.multiprocessing as mp

    if cuda.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")
    _paths()
    import q4kb200 as q
    from conftest import rel_l2
    from test_gpu_engine import greedy_ok
    from tiny_model import SEED

    rng = np.random.default_rng(2)
    seqs = rng.permutation(BATCH).astype(np.int32)
    pos = rng.integers(100, POS1 + 1, BATCH).astype(np.int32)
    batch_tokens = rng.integers(0, 151936, BATCH).astype(np.uint32)
    one = _tp_engine(q, 0, 1, None, None)
    one.load_synthetic(SEED)
    one.fill_kv_synthetic(SEED, POS1)
    H, L = 2560, 36
    rows_in = [rng.standard_normal((ROWS, H)).astype(np.float32)]
    tok_in = [rng.standard_normal(H).astype(np.float32)]
    bat_in = [rng.standard_normal((BATCH, H)).astype(np.float32)]
    for i in range(L):
        rows_in.append(one.layer_rows(i, rows_in[i], 0))
        tok_in.append(one.layer(i, tok_in[i], POS1))
        bat_in.append(one.layer_batch(i, bat_in[i], seqs, pos))
    want_next, want_logits = one.decode_batch(seqs, batch_tokens, pos, want_logits=True)
    one.close()
    cuda.cuda.synchronize()
    inputs = (rows_in[:L], tok_in[:L], bat_in[:L])

    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = 29700 + (os.getpid() % 1000)
    procs = [ctx.Process(target=_rank_layers, args=(r, 2, port, inputs, seqs, pos, batch_tokens, out))
             for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    for _ in procs:
        r, res = out.get(timeout=900)
        got[r] = res
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    worst = {"rows": 0.0, "token": 0.0, "batch": 0.0}
    for r in range(2):
        rows, tok, bat, nxt, _ = got[r]
        for i in range(L):
            worst["rows"] = max(worst["rows"], rel_l2(rows[i], rows_in[i + 1]))
            worst["token"] = max(worst["token"], rel_l2(tok[i], tok_in[i + 1]))
            worst["batch"] = max(worst["batch"], rel_l2(bat[i], bat_in[i + 1]))
        assert np.array_equal(nxt, got[0][3])  # every rank returns the merged tokens
    full = np.concatenate([got[0][4], got[1][4]], axis=1)
    for b in range(BATCH):
        assert greedy_ok(int(got[0][3][b]), int(want_next[b]), want_logits[b], full[b]), b
    e = rel_l2(full, want_logits)
    print(f"tp2 vs one GPU per layer (identical inputs): prompt rows {worst['rows']:.2e}, decode token "
          f"{worst['token']:.2e}, batched step {worst['batch']:.2e}; batched logits rel-L2 {e:.2e}")
    assert max(worst.values()) < 1e-3, worst
    assert e < 5e-2
