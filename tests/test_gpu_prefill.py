"""Prompt prefill parity (q4k_engine_prefill through the C ABI).

The reference runs a whole prompt through one pass of Engine::inference with
tokens = n (src/Engine.cpp:37-114): every product over n rows, causal
attention with each row stopping at its own position (attention.cu:45), the
n K/V rows appended to the cache, the head on the last row only. The engine's
prefill is compared with the CPU oracle's multi-token forward (tiny model)
and with the reference's own kernels replaying that pass (full model), with
the whole-step bars of the decode tests (see test_gpu_engine.py for why the
full model is compared at 5e-2 relative L2 plus a greedy near-tie rule).
"""
import ctypes as C

import numpy as np
import pytest

import oracle as o
import q4kb200 as q
from conftest import rel_l2
from test_gpu_engine import full_model, greedy_ok, kv_f32, oracle_model  # noqa: F401 (fixture)
from test_gpu_kernels import dev
from tiny_model import SEED, TINY, engine_config, tiny_tensors

pytestmark = pytest.mark.gpu


def upload(cuda, qt, K, N, raw):
    buf = cuda.empty(max(q.device_bytes(qt, K, N), 16), dtype=cuda.uint8, device="cuda")
    q.check(q.lib().q4k_weight_upload(qt, K, N, q.hptr(np.ascontiguousarray(raw)), buf.data_ptr(), None))
    return buf


# (types, K, output rows per weight, activation rows, epilogue, RMSNorm first)
BATCH_CASES = {
    "q4k_two_row_tiles": ([q.Q4_K], 2560, [384], 130, q.EPI_STORE, False),
    "q6k_ragged_columns": ([q.Q6_K], 2560, [200], 23, q.EPI_STORE, True),
    "q6k_down_add": ([q.Q6_K], 9728, [256], 20, q.EPI_ADD, False),
    "q4k_down_add": ([q.Q4_K], 9728, [128], 5, q.EPI_ADD, False),
    "qkv_segments": ([q.Q4_K, q.Q4_K, q.Q6_K], 2560, [512, 128, 128], 70, q.EPI_STORE, True),
    "swiglu_pairs": ([q.Q4_K, q.Q4_K], 2560, [192, 192], 129, q.EPI_SWIGLU, True),
    "one_row": ([q.Q4_K], 4096, [128], 1, q.EPI_STORE, False),
}


@pytest.mark.parametrize("case", list(BATCH_CASES))
def test_matmul_batch_matches_oracle(cuda, case):
    """q4k_matmul_batch (tensor cores) against the oracle's integer products
    (MatmulReference semantics) on the same rows: 1e-3 relative L2 per
    output, the per-layer bar; columns past each output stay untouched."""
    types, K, outs, M, epi, norm = BATCH_CASES[case]
    raws = [q.synth_tensor_host(31 + i, f"mb.{case}.{i}", t, K, n) for i, (t, n) in enumerate(zip(types, outs))]
    Ws = [upload(cuda, t, K, n, r) for t, n, r in zip(types, outs, raws)]
    x = q.synth_f32_host(5, f"mb.x.{case}", M * K)
    gamma = q.synth_tensor_host(5, f"mb.g.{case}", q.F32, K, 1) if norm else None
    xin = o.rms_norm(x, gamma, K, 1e-6) if norm else x
    prods = [o.matmul(xin, r, t, K, n).reshape(M, n).astype(np.float32) for t, n, r in zip(types, outs, raws)]
    if epi == q.EPI_SWIGLU:
        wants = [o.silu_multiply(prods[0], prods[1]).reshape(M, outs[0])]
        widths = [outs[0]]
    else:
        wants, widths = prods, outs
    ld = sum(widths) + 8
    base = q.synth_f32_host(6, f"mb.y.{case}", M * ld).reshape(M, ld)
    y = dev(cuda, base)
    offs = np.concatenate([[0], np.cumsum(widths)])[:-1]
    outs_p = [y.data_ptr() + 4 * int(off) for off in offs]
    if epi == q.EPI_SWIGLU:
        outs_p = [outs_p[0], outs_p[0]]
    n = len(types)
    q.check(q.lib().q4k_matmul_batch(dev(cuda, x).data_ptr(), dev(cuda, gamma).data_ptr() if norm else None, 1e-6, n,
                                     (C.c_void_p * n)(*[w.data_ptr() for w in Ws]), (C.c_int * n)(*types),
                                     (C.c_int64 * n)(*outs), (C.c_void_p * n)(*outs_p), ld, K, M, epi, None))
    got = y.cpu().numpy()
    for want, off, w in zip(wants, offs, widths):
        part = got[:, off : off + w]
        if epi == q.EPI_ADD:
            part = part - base[:, off : off + w]  # the product added to what was there
        e = rel_l2(part, want)
        print(f"{case}: rel-L2 {e:.2e}")
        assert e < 1e-3, (case, off, e)
    assert np.array_equal(got[:, sum(widths) :], base[:, sum(widths) :])  # columns past the outputs


def tiny_engine(cap):
    eng = q.Engine(engine_config(TINY, capacity=cap))
    for n, (t, a, b, d) in tiny_tensors().items():
        eng.set_tensor(n, t, a, b, d)
    return eng


def kv_rows(eng, layer, kv_heads, cap, n0, n1):
    """Engine cache rows [n0, n1) of one layer as fp32 [kv_heads][rows][128]."""
    k, v = eng.read_kv(layer)
    k = k.view(np.float16).astype(np.float32).reshape(kv_heads, cap, 128)[:, n0:n1]
    v = v.view(np.float16).astype(np.float32).reshape(kv_heads, cap, 128)[:, n0:n1]
    return k, v


@pytest.fixture(params=["gemm", "gemv"])
def products(request, monkeypatch):
    """Both forms of the prompt products: the tensor-core GEMM (default) and
    the batched dp4a GEMV (Q4K_PREFILL_GEMM=0)."""
    monkeypatch.setenv("Q4K_PREFILL_GEMM", "1" if request.param == "gemm" else "0")
    return request.param


def test_tiny_prefill_matches_oracle(cuda, products):
    """A 7-token prompt into an empty cache, a 3-token prompt continuing it
    (its rows attend to the first prompt's cache rows), then a decode step on
    the cache prefill wrote: logits, greedy token and every K/V row."""
    tensors = tiny_tensors()
    cap = 32
    L, KVH = TINY["layers"], TINY["kv_heads"]
    model = oracle_model(TINY, tensors)
    kc = np.zeros(L * cap * KVH * 128, np.float32)
    vc = np.zeros_like(kc)
    eng = tiny_engine(cap)
    pos = 0
    for prompt in ([3, 141, 592, 653, 589, 793, 238], [462, 643, 383]):
        want_next, want_logits, _ = model.forward(kc, vc, cap, prompt, pos, kv_round_f16=True, want_hidden=False)
        got_next, got_logits = eng.prefill(prompt, pos, want_logits=True)
        assert np.isfinite(got_logits).all()
        assert rel_l2(got_logits, want_logits) < 1e-2, pos
        assert greedy_ok(got_next, want_next, want_logits, got_logits), pos
        pos += len(prompt)
    # Layer 0's K/V rows come from the embedding through one product each: the
    # integer-exact GEMV matches to 1e-4, the GEMM's fp16 operands (3e-4 per
    # product, test_matmul_batch_matches_oracle) to 1e-3. Later layers see
    # both amplified ~40x by the Q8 code flips of the synthetic model's large
    # residual stream (the same factor on both paths): the whole-step bar.
    for layer in range(L):
        k, v = kv_rows(eng, layer, KVH, cap, 0, pos)
        ko = kc.reshape(L, cap, KVH, 128)[layer, :pos].transpose(1, 0, 2)
        vo = vc.reshape(L, cap, KVH, 128)[layer, :pos].transpose(1, 0, 2)
        bar = (1e-3 if products == "gemm" else 1e-4) if layer == 0 else 5e-2
        print(f"[{products}] layer {layer} K/V rows rel-L2 {rel_l2(k, ko):.2e} {rel_l2(v, vo):.2e}")
        assert rel_l2(k, ko) < bar and rel_l2(v, vo) < bar, layer
    # decoding continues on the rows prefill wrote
    tok = want_next
    want_next, want_logits, _ = model.forward(kc, vc, cap, [tok], pos, kv_round_f16=True, want_hidden=False)
    got_next, got_logits, _ = eng.decode(tok, pos, want_logits=True)
    assert rel_l2(got_logits, want_logits) < 1e-2
    assert greedy_ok(got_next, want_next, want_logits, got_logits)
    eng.close()


def test_tiny_prefill_passes_bit_identical(cuda, monkeypatch, products):
    """A prompt split over several prefill passes (Q4K_PREFILL_ROWS rows
    each, the last one ragged) computes what one pass does, bit for bit:
    a row's products and attention do not depend on the other rows of its
    pass, and later passes read the earlier passes' rows from the cache."""
    cap = 32
    L, KVH = TINY["layers"], TINY["kv_heads"]
    prompt = [7, 99, 250, 3, 871, 402, 16, 555, 640, 21, 998]
    out = []
    for rows in ("512", "4", "1"):
        monkeypatch.setenv("Q4K_PREFILL_ROWS", rows)
        eng = tiny_engine(cap)
        nxt, logits = eng.prefill(prompt, 2, want_logits=True)
        kv = [eng.read_kv(layer) for layer in range(L)]
        out.append((nxt, logits, kv))
        eng.close()
    monkeypatch.delenv("Q4K_PREFILL_ROWS")
    for nxt, logits, kv in out[1:]:
        assert nxt == out[0][0]
        assert np.array_equal(logits.view(np.uint32), out[0][1].view(np.uint32))
        for layer in range(L):
            for a, b in zip(kv[layer], out[0][2][layer]):
                a = a.reshape(KVH, cap, 128)[:, 2 : 2 + len(prompt)]
                b = b.reshape(KVH, cap, 128)[:, 2 : 2 + len(prompt)]
                assert np.array_equal(a, b), layer


def test_prefill_rejects_bad_prompts(cuda):
    """Errors the reference raises for a prompt (Engine.cpp:126-128 capacity,
    EmbedLookup's token range) come back as status codes, with nothing
    launched, and the engine stays usable."""
    cap = 16
    eng = tiny_engine(cap)
    with pytest.raises(q.OutOfRange):
        eng.prefill([1, 2, 3], cap - 2)  # rows cap-2 .. cap: one past the end
    with pytest.raises(q.OutOfRange):
        eng.prefill([1, TINY["vocab"], 3], 0)
    with pytest.raises(q.OutOfRange):
        eng.prefill([1], -1)
    with pytest.raises(q.InvalidArgument):
        eng.prefill([], 0)
    a, _ = eng.prefill(list(range(1, cap + 1)), 0)  # the whole capacity
    b, _ = eng.prefill(list(range(1, cap + 1)), 0)
    assert a == b
    eng.close()


def ref_prompt(c, tensors, handles, kd, vd, cap, toks, pos):
    """The reference kernels' pass over a prompt (oracle/_ref ref_forward
    with tokens = len(toks)); K/V rows rounded to fp16 like the engine's."""
    import torch

    order = [f"blk.{i}.{s}.weight" for i in range(c["layers"]) for s in o.SLOT_NAMES]
    order += ["output_norm.weight", "token_embd.weight"]
    ptrs = (C.c_void_p * len(order))(*[handles[n].h.value for n in order])
    embd = tensors["token_embd.weight"][3]
    logits = torch.empty(c["vocab"], device="cuda")
    toks = np.ascontiguousarray(toks, np.uint32)
    nxt = C.c_uint32()
    o.ref_check(o.ref().ref_forward(ptrs, c["layers"], c["hidden"], c["heads"], c["kv_heads"], c["head_dim"], c["ffn"],
                                    c["vocab"], c["eps"], c["rope_base"], embd.ctypes.data,
                                    q.gguf_row_bytes(q.Q6_K, c["hidden"]), kd.data_ptr(), vd.data_ptr(), cap,
                                    toks.ctypes.data, toks.size, pos, 1, logits.data_ptr(), None, C.byref(nxt)))
    return nxt.value, logits.cpu().numpy()


def test_full_model_prefill_matches_reference_kernels(cuda, full_model):
    """Qwen3-4B shapes: a 23-token prompt (the length of the reference's
    first-token benchmark prompt; random ids) into an empty session, and a
    64-token prompt continuing a 4000-row cache, each followed by one decode
    step on the cache prefill wrote, against the reference's own kernels."""
    import torch

    if not o.ref_available():
        pytest.fail("oracle/_ref/libq4kref.so (the reference kernels) was not built")
    cfg, c, eng, tensors, handles = full_model
    L, KVH, cap = c["layers"], c["kv_heads"], 4096
    rng = np.random.default_rng(23)
    try:
        for n, pos in ((23, 0), (64, 4000)):
            if pos:
                kc, vc = kv_f32(SEED, L, KVH, pos, cap)
                kd, vd = torch.from_numpy(kc).cuda(), torch.from_numpy(vc).cuda()
                del kc, vc
                eng.fill_kv_synthetic(SEED, pos)
            else:
                kd = torch.zeros(L * cap * KVH * 128, device="cuda")
                vd = torch.zeros_like(kd)
            prompt = rng.integers(0, c["vocab"], n).astype(np.uint32)
            want_next, want_logits = ref_prompt(c, tensors, handles, kd, vd, cap, prompt, pos)
            got_next, got_logits = eng.prefill(prompt, pos, want_logits=True)
            e = rel_l2(got_logits, want_logits)
            kerr = []
            for layer in range(L):
                k, v = kv_rows(eng, layer, KVH, cap, pos, pos + n)
                kr = kd.view(L, cap, KVH, 128)[layer, pos : pos + n].transpose(0, 1).cpu().numpy()
                vr = vd.view(L, cap, KVH, 128)[layer, pos : pos + n].transpose(0, 1).cpu().numpy()
                kerr.append(max(rel_l2(k, kr), rel_l2(v, vr)))
            print(f"prefill {n} tokens at {pos}: logits rel-L2 {e:.2e}, K/V rows rel-L2 layer 0 {kerr[0]:.2e}, "
                  f"max {max(kerr):.2e}; next token {got_next} (reference {want_next})")
            assert e < 5e-2
            assert greedy_ok(got_next, want_next, want_logits, got_logits)
            assert kerr[0] < 1e-2 and max(kerr) < 5e-2, kerr
            # one decode step after the prompt, teacher-forced on the reference's token
            want2, want2_logits = ref_prompt(c, tensors, handles, kd, vd, cap, [want_next], pos + n)
            got2, got2_logits, _ = eng.decode(want_next, pos + n, want_logits=True)
            assert rel_l2(got2_logits, want2_logits) < 5e-2
            assert greedy_ok(got2, want2, want2_logits, got2_logits)
            del kd, vd
    finally:
        eng.fill_kv_synthetic(SEED, 4095)
