"""Batched decode parity (q4k_engine_decode_batch, q4k_engine_prefill_seq).

One step serves n sequences, each with its own KV cache: the products run
over all n rows, attention over each token's own sequence. Every sequence
must compute what a one-sequence engine computes for it: bit for bit on the
batched GEMV path (its rows do not interact; the attention split count is
pinned to the single-token value), within the whole-step bar on the
tensor-core GEMM path (fp16 operands, test_gpu_prefill.py).
"""
import numpy as np
import pytest

import q4kb200 as q
from conftest import rel_l2
from test_gpu_engine import greedy_ok
from tiny_model import SEED, TINY, engine_config, tiny_tensors

pytestmark = pytest.mark.gpu


def tiny_engine(cap, sequences=1):
    cfg = engine_config(TINY, capacity=cap)
    cfg.sequences = sequences
    eng = q.Engine(cfg)
    for n, (t, a, b, d) in tiny_tensors().items():
        eng.set_tensor(n, t, a, b, d)
    return eng


def single_splits(cuda, kv_heads):
    return max(1, cuda.cuda.get_device_properties(0).multi_processor_count // kv_heads)


def test_tiny_batch_decode_bit_identical_to_single(cuda, monkeypatch):
    """Three of four sequences (not in index order) step together for four
    steps; each token, logit and cache row equals a one-sequence engine's."""
    monkeypatch.setenv("Q4K_BATCH_SPLITS", str(single_splits(cuda, TINY["kv_heads"])))
    cap = 32
    prompts = {0: [3, 141, 592, 653], 2: [589, 793, 238, 462, 643, 383, 279], 3: [50, 28]}
    batch = tiny_engine(cap, sequences=4)
    singles = {s: tiny_engine(cap) for s in prompts}
    nxt, pos = {}, {}
    for s, p in prompts.items():
        a, la = batch.prefill_seq(s, p, 0, want_logits=True)
        b, lb = singles[s].prefill(p, 0, want_logits=True)
        assert a == b and np.array_equal(la.view(np.uint32), lb.view(np.uint32)), s
        nxt[s], pos[s] = a, len(p)
    order = [2, 0, 3]
    for step in range(4):
        toks, logits = batch.decode_batch(order, [nxt[s] for s in order], [pos[s] for s in order], want_logits=True)
        for i, s in enumerate(order):
            t1, l1, _ = singles[s].decode(nxt[s], pos[s], want_logits=True)
            assert toks[i] == t1, (step, s)
            assert np.array_equal(logits[i].view(np.uint32), l1.view(np.uint32)), (step, s)
            nxt[s], pos[s] = t1, pos[s] + 1
    # sequence 0's cache (the one read_kv reads) holds exactly the rows its
    # own engine wrote, prompt and decoded tokens alike
    for layer in range(TINY["layers"]):
        kb, vb = batch.read_kv(layer)
        ks, vs = singles[0].read_kv(layer)
        for x, y in ((kb, ks), (vb, vs)):
            assert np.array_equal(x.reshape(-1, cap, 128)[:, : pos[0]], y.reshape(-1, cap, 128)[:, : pos[0]]), layer
    batch.close()
    for e in singles.values():
        e.close()


def test_tiny_batch_decode_gemm_path(cuda):
    """Twelve sequences in one step take the tensor-core products: every
    layer of the batched step is within 1e-3 relative L2 of a one-sequence
    engine's layer (integer-exact GEMV products) on identical inputs, and each
    sequence's logits stay within the whole-step bar (5e-2, as for the full
    model: through the layers of a random-init model the ~1e-7 product
    differences of the two paths flip Q8 codes), teacher-forced on the single
    engine's tokens for three steps."""
    cap = 24
    rng = np.random.default_rng(7)
    n = 12
    prompts = [list(rng.integers(0, TINY["vocab"], int(rng.integers(1, 9)))) for _ in range(n)]
    batch = tiny_engine(cap, sequences=n)
    singles = [tiny_engine(cap) for _ in range(n)]
    nxt, pos = [], []
    for s, p in enumerate(prompts):
        a, _ = batch.prefill_seq(s, p, 0)
        b, _ = singles[s].prefill(p, 0)
        assert a == b, s  # prompts of 1-8 tokens: the same batched-GEMV prefill
        nxt.append(b)
        pos.append(len(p))
    worst = 0.0
    for step in range(3):
        toks, logits = batch.decode_batch(list(range(n)), nxt, pos, want_logits=True)
        for s in range(n):
            t1, l1, _ = singles[s].decode(nxt[s], pos[s], want_logits=True)
            e = rel_l2(logits[s], l1)
            worst = max(worst, e)
            assert e < 5e-2, (step, s, e)
            assert greedy_ok(int(toks[s]), t1, l1, logits[s]), (step, s)
            nxt[s], pos[s] = t1, pos[s] + 1
    # every layer on identical inputs: the batched step's rows against each
    # sequence's own engine
    x = rng.standard_normal((n, TINY["hidden"])).astype(np.float32)
    layer_worst = 0.0
    for layer in range(TINY["layers"]):
        got = batch.layer_batch(layer, x, list(range(n)), pos)
        want = np.stack([singles[s].layer(layer, x[s], pos[s]) for s in range(n)])
        layer_worst = max(layer_worst, rel_l2(got, want))  # over all rows, as the full-model layer tests
        x = want
    print(f"12-sequence batch on the GEMM path: worst logits rel-L2 {worst:.2e}, worst layer {layer_worst:.2e}")
    assert layer_worst < 1e-3
    batch.close()
    for e in singles:
        e.close()


def test_batch_decode_rejects_bad_steps(cuda):
    batch = tiny_engine(8, sequences=3)
    with pytest.raises(q.InvalidArgument):
        batch.decode_batch([0, 0], [1, 2], [0, 1])  # a sequence twice
    with pytest.raises(q.OutOfRange):
        batch.decode_batch([3], [1], [0])  # no such sequence
    with pytest.raises(q.OutOfRange):
        batch.decode_batch([0, 1, 2, 0], [1, 1, 1, 1], [0, 0, 0, 0])  # more tokens than sequences
    with pytest.raises(q.OutOfRange):
        batch.decode_batch([1], [TINY["vocab"]], [0])
    with pytest.raises(q.OutOfRange):
        batch.decode_batch([1], [5], [8])
    with pytest.raises(q.OutOfRange):
        batch.prefill_seq(3, [1, 2], 0)
    t, _ = batch.decode_batch([2, 1], [5, 6], [0, 0])  # still usable
    assert t.shape == (2,)
    batch.close()


def test_full_model_batch_decode_matches_single(cuda):
    """Qwen3-4B shapes, 16 sequences over the same synthetic 4000-row
    context, each decoding a different token at a different position, one
    step: the batch (GEMM products, batched attention) against one-sequence
    decode steps (the launch sequence), run in decreasing position order so
    that the rows those steps write are never read by a later one."""
    n, ctx = 16, 4000
    cfg = q.qwen3_4b_config(4096)
    cfg.sequences = n
    batch = q.Engine(cfg)
    batch.load_synthetic(SEED)
    batch.fill_kv_synthetic(SEED, ctx)
    single = q.Engine(q.qwen3_4b_config(4096))
    single.load_synthetic(SEED)
    single.fill_kv_synthetic(SEED, ctx)
    rng = np.random.default_rng(11)
    toks = rng.integers(0, cfg.vocab, n).astype(np.uint32)
    pos = (ctx - 1 - 37 * np.arange(n)).astype(np.int32)  # 3999, 3962, ...: decreasing
    seqs = list(rng.permutation(n))
    got, logits = batch.decode_batch(seqs, toks, pos, want_logits=True)
    worst = 0.0
    for i in range(n):
        t1, l1, _ = single.decode(int(toks[i]), int(pos[i]), want_logits=True)
        e = rel_l2(logits[i], l1)
        worst = max(worst, e)
        assert e < 5e-2, (i, e)
        assert greedy_ok(int(got[i]), t1, l1, logits[i]), i
    print(f"16-sequence batch vs single decode: worst logits rel-L2 {worst:.2e}")
    batch.close()
    single.close()
