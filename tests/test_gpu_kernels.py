"""Parity of every kernel entry point of include/q4k_b200.h against the CPU
oracle (and, where the prebuilt reference kernels are present, against the
reference engine's own kernels on the same device buffers).

Tolerances: dequantisation bit-exact; products per element
Catch::Approx(expected).margin(3e-5).epsilon(1e-4) against the oracle's
double accumulation (the reference's own test bar, MatmulReference.hpp:71-79)
and relative L2 <= 1e-3 against the reference kernels;
attention margin 3e-5 (AttentionTests.cpp:68)."""
import ctypes as C

import numpy as np
import pytest

import oracle as o
import q4kb200 as q
from conftest import rel_l2

pytestmark = pytest.mark.gpu


def approx_ok(actual, expected, margin=3e-5, eps=1e-4):
    """Catch::Approx(expected).margin(margin).epsilon(eps), with the margin
    taken relative to the output's RMS when that exceeds 1: the reference's
    bar was set on real-model outputs of order 0.1-1, and fp32 summation
    error grows with the magnitude of the terms."""
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    scale = max(1.0, float(np.sqrt(np.mean(e * e)))) if e.size else 1.0
    return np.abs(a - e) <= np.maximum(margin * scale, eps * np.abs(e))


_KEEP = []


@pytest.fixture(autouse=True)
def _release_device_copies():
    yield
    _KEEP.clear()


def dev(cuda, a):
    """Device copy of a host array, kept alive until the test ends: a raw
    data_ptr() of a temporary would let the caching allocator hand the same
    memory to the next copy before the kernel reads it."""
    t = cuda.from_numpy(np.ascontiguousarray(a)).cuda()
    _KEEP.append(t)
    return t


def upload(cuda, qt, K, N, raw):
    buf = cuda.empty(max(q.device_bytes(qt, K, N), 16), dtype=cuda.uint8, device="cuda")
    q.check(q.lib().q4k_weight_upload(qt, K, N, q.hptr(np.ascontiguousarray(raw)), buf.data_ptr(), None))
    return buf


def make_input(n):
    # MatmulReference.hpp:33-41
    return (np.sin(np.arange(n, dtype=np.float32) * np.float32(0.031)) * np.float32(0.1)).astype(np.float32)


# ------------------------------------------------------------------ dequant
@pytest.mark.parametrize("qt", [q.Q4_K, q.Q6_K])
def test_dequantize_embeddings_bit_exact(cuda, qt):
    rows, K = 33, 2560
    raw = q.synth_tensor_host(11, f"deq.{qt}", qt, K, rows)
    rb = q.gguf_row_bytes(qt, K)
    out = cuda.full((rows * K + 2,), 123.0, device="cuda")
    q.check(q.lib().q4k_dequantize_embeddings(dev(cuda, raw).data_ptr(), out.data_ptr() + 4, rows, K, rb, qt, None))
    got = out.cpu().numpy()
    assert got[0] == 123.0 and got[-1] == 123.0
    want = o.dequantize_rows(raw, qt, rows, K)
    assert np.array_equal(got[1:-1].view(np.uint32), want.ravel().view(np.uint32))
    if o.ref_available():
        ref_out = cuda.empty(rows * K, device="cuda")
        o.ref_check(o.ref().ref_dequantize_embeddings(dev(cuda, raw).data_ptr(), ref_out.data_ptr(), rows, K, rb, qt))
        cuda.cuda.synchronize()
        assert np.array_equal(ref_out.cpu().numpy().view(np.uint32), want.ravel().view(np.uint32))


def test_dequantize_golden_edge_blocks(cuda):
    import os

    from conftest import GOLDEN

    gg = np.load(os.path.join(GOLDEN, "dequant_gguf.npz"))
    for tag, qt in (("q4k", q.Q4_K), ("q6k", q.Q6_K)):
        blocks = gg[f"{tag}_blocks"]
        out = cuda.empty(blocks.shape[0] * 256, device="cuda")
        q.check(q.lib().q4k_dequantize_embeddings(dev(cuda, blocks).data_ptr(), out.data_ptr(), blocks.shape[0], 256,
                                                  blocks.shape[1], qt, None))
        assert np.array_equal(out.cpu().numpy().view(np.uint32), gg[f"{tag}_values"].ravel().view(np.uint32))


# ------------------------------------------------------------------- matmul
@pytest.mark.parametrize("qt", [q.Q4_K, q.Q6_K])
@pytest.mark.parametrize("K,N", [(2560, 5), (2560, 19), (4096, 37), (9728, 19)])
@pytest.mark.parametrize("rows", [1, 3, 4, 5, 101])
def test_matmul_matches_oracle(cuda, qt, K, N, rows):
    if K == 9728 and rows == 101:
        rows = 17
    raw = q.synth_tensor_host(21, f"mm.{qt}.{K}", qt, K, 64)  # 64 rows stored, the first N used
    W = upload(cuda, qt, K, 64, raw)
    x = make_input(rows * K) if rows % 2 else q.synth_f32_host(3, f"x.{rows}.{K}", rows * K)
    want = o.matmul(x, raw[: N * q.gguf_row_bytes(qt, K)], qt, K, N)
    out = cuda.full((rows * N + 2,), 123.0, device="cuda")
    xd = dev(cuda, x)
    for _ in range(2):
        q.check(q.lib().q4k_matmul(xd.data_ptr(), W.data_ptr(), qt, K, N, out.data_ptr() + 4, rows, None))
        got = out.cpu().numpy()
        assert got[0] == 123.0 and got[-1] == 123.0
        assert approx_ok(got[1:-1], want.ravel()).all()
    # a second call with zero input must overwrite the product with exact zeros
    xd.zero_()
    q.check(q.lib().q4k_matmul(xd.data_ptr(), W.data_ptr(), qt, K, N, out.data_ptr() + 4, rows, None))
    got = out.cpu().numpy()
    assert np.all(got[1:-1] == 0.0) and got[0] == 123.0 and got[-1] == 123.0


def _one_hot_q4k(K):
    """K Q4_K rows of K inputs; row r has d = 1, every 6-bit scale 1, every
    min 0 and a single code 1 at input r, so y[r] = xs[r / 32] * xq[r]
    exactly: the product exposes the activation's Q8 codes."""
    nb = K // 256
    blk = np.zeros((K, nb, 144), np.uint8)
    blk[:, :, 0:2] = np.frombuffer(np.float16(1.0).tobytes(), np.uint8)  # d; dmin stays 0
    blk[:, :, 4:8] = 1      # scales of groups 0-3 (6 bits), top bits 0
    blk[:, :, 12:16] = 1    # groups 4-7: low nibble scale 1, high nibble min 0
    r = np.arange(K)
    b, t = r // 256, r % 256
    g, i = t // 32, t % 32
    byte = 16 + 32 * (g // 2) + i
    blk[r, b, byte] = np.where(g % 2 == 0, 0x01, 0x10)
    return blk.reshape(-1)


def test_activation_codes_bit_exact(cuda):
    """The Q8 codes and scales of the activation (matmul.cu:8-22) match the
    oracle bit for bit, including values at and next to the rounding
    boundaries k + 0.5, where the kernel switches from its multiply-by-
    reciprocal path to the IEEE-division form, and groups whose maximum is
    0, subnormal or near the float range."""
    K = 2560
    rng = np.random.default_rng(7)
    x = rng.standard_normal(K).astype(np.float32)
    groups = x.reshape(-1, 32)
    deltas = [0.0, 1e-7, -1e-7, 1e-6, -1e-6, 3e-5, -3e-5, 1e-4, -1e-4, 1.9e-4, -1.9e-4, 2.1e-4, -2.1e-4, 5e-4]
    for gi in range(0, 48):
        amax = np.float32(rng.uniform(0.01, 40.0))
        ks = rng.integers(-126, 126, 31)
        d = np.array([deltas[(gi + j) % len(deltas)] for j in range(31)], np.float64)
        vals = ((ks + 0.5 + d) * float(amax) / 127.0).astype(np.float32)
        groups[gi, :31] = np.clip(vals, -amax, amax)
        groups[gi, 31] = amax if gi % 2 else -amax
    groups[50] = 0.0
    groups[51] = np.float32(1e-39) * np.sign(groups[51] + 0.5)                         # subnormal maximum
    groups[52] = (rng.uniform(-1, 1, 32) * 2e38).astype(np.float32)                     # past the fast-path range
    groups[53] = (rng.uniform(-1, 1, 32) * 3e37).astype(np.float32)                     # just inside it
    groups[54] = (rng.uniform(-1, 1, 32) * 1e-37).astype(np.float32)
    x = groups.reshape(-1)
    codes, scales = o.quantize_q8(x)
    want = (codes.astype(np.float32) * scales[np.arange(K) // 32]).astype(np.float32)
    W = upload(cuda, q.Q4_K, K, K, _one_hot_q4k(K))
    out = cuda.empty(K, device="cuda")
    q.check(q.lib().q4k_matmul(dev(cuda, x).data_ptr(), W.data_ptr(), q.Q4_K, K, K, out.data_ptr(), 1, None))
    got = out.cpu().numpy()
    bad = np.nonzero(got.view(np.uint32) != want.view(np.uint32))[0]
    assert bad.size == 0, (bad[:8], got[bad[:8]], want[bad[:8]])


def test_matmul_concurrent_streams(cuda):
    qt, K, N, rows = q.Q4_K, 2560, 1024, 3
    raw = q.synth_tensor_host(5, "mm.streams", qt, K, N)
    W = upload(cuda, qt, K, N, raw)
    x = dev(cuda, make_input(rows * K))
    a = cuda.zeros(rows * N, device="cuda")
    b = cuda.zeros(rows * N, device="cuda")
    s1, s2 = cuda.cuda.Stream(), cuda.cuda.Stream()
    q.check(q.lib().q4k_matmul(x.data_ptr(), W.data_ptr(), qt, K, N, a.data_ptr(), rows, s1.cuda_stream))
    q.check(q.lib().q4k_matmul(x.data_ptr(), W.data_ptr(), qt, K, N, b.data_ptr(), rows, s2.cuda_stream))
    s1.synchronize()
    s2.synchronize()
    want = o.matmul(make_input(rows * K), raw, qt, K, N)
    assert approx_ok(a.cpu().numpy(), want.ravel()).all()
    assert np.array_equal(a.cpu().numpy(), b.cpu().numpy())


@pytest.mark.parametrize("name,qt,K,N", [("ffn_gate", q.Q4_K, 2560, 9728), ("ffn_down", q.Q6_K, 9728, 2560),
                                         ("ffn_down_q4", q.Q4_K, 9728, 2560), ("output", q.Q6_K, 2560, 151936)])
def test_matmul_full_shapes(cuda, name, qt, K, N):
    raw = q.synth_tensor_host(0x5EED, f"full.{name}", qt, K, N)
    W = upload(cuda, qt, K, N, raw)
    x = q.synth_f32_host(0x5EED, f"full.{name}.x", K)
    out = cuda.empty(N, device="cuda")
    q.check(q.lib().q4k_matmul(dev(cuda, x).data_ptr(), W.data_ptr(), qt, K, N, out.data_ptr(), 1, None))
    got = out.cpu().numpy()
    want = o.matmul(x, raw, qt, K, N).ravel()
    assert approx_ok(got, want).all()
    assert rel_l2(got, want) < 1e-5
    if o.ref_available():
        Wr = o.RefWeight(f"full.{name}", qt, K, N, raw)
        ref_out = cuda.empty(N, device="cuda")
        o.ref_check(o.ref().ref_matmul(dev(cuda, x).data_ptr(), Wr.h, ref_out.data_ptr(), 1, None))
        cuda.cuda.synchronize()
        assert rel_l2(got, ref_out.cpu().numpy()) < 1e-3


# --------------------------------------------------------------- fused forms
def test_matmul_ex_fused_norm_qkv_segments(cuda):
    K = 2560
    segs = [("q", q.Q4_K, 4096), ("k", q.Q4_K, 1024), ("v", q.Q6_K, 1024)]
    raws = [q.synth_tensor_host(9, f"qkv.{n}", t, K, r) for n, t, r in segs]
    Ws = [upload(cuda, t, K, r, raw) for (n, t, r), raw in zip(segs, raws)]
    x = q.synth_f32_host(9, "qkv.x", K) * 3
    gamma = q.synth_tensor_host(9, "qkv.g", q.F32, K, 1)
    outs = [cuda.empty(r, device="cuda") for _, _, r in segs]
    warr = (C.c_void_p * 3)(*[w.data_ptr() for w in Ws])
    tarr = (C.c_int * 3)(*[t for _, t, _ in segs])
    rarr = (C.c_int64 * 3)(*[r for _, _, r in segs])
    oarr = (C.c_void_p * 3)(*[t.data_ptr() for t in outs])
    q.check(q.lib().q4k_matmul_ex(dev(cuda, x).data_ptr(), dev(cuda, gamma).data_ptr(), 1e-6, 3, warr, tarr, rarr,
                                  oarr, K, 1, q.EPI_STORE, None, None, None))
    normed = o.rms_norm(x, gamma, K, 1e-6)
    for (n, t, r), raw, out in zip(segs, raws, outs):
        want = o.matmul(normed, raw, t, K, r).ravel()
        got = out.cpu().numpy()
        assert rel_l2(got, want) < 1e-4, n
        assert np.mean(approx_ok(got, want, 3e-5, 1e-3)) > 0.999, n


def test_matmul_ex_swiglu_and_add(cuda):
    K, N = 2560, 9728
    rg = q.synth_tensor_host(4, "sw.gate", q.Q4_K, K, N)
    ru = q.synth_tensor_host(4, "sw.up", q.Q4_K, K, N)
    Wg, Wu = upload(cuda, q.Q4_K, K, N, rg), upload(cuda, q.Q4_K, K, N, ru)
    x = q.synth_f32_host(4, "sw.x", K)
    gamma = q.synth_tensor_host(4, "sw.g", q.F32, K, 1)
    out = cuda.empty(N, device="cuda")
    warr = (C.c_void_p * 2)(Wg.data_ptr(), Wu.data_ptr())
    tarr = (C.c_int * 2)(q.Q4_K, q.Q4_K)
    rarr = (C.c_int64 * 2)(N, N)
    oarr = (C.c_void_p * 2)(out.data_ptr(), out.data_ptr())
    q.check(q.lib().q4k_matmul_ex(dev(cuda, x).data_ptr(), dev(cuda, gamma).data_ptr(), 1e-6, 2, warr, tarr, rarr,
                                  oarr, K, 1, q.EPI_SWIGLU, None, None, None))
    n = o.rms_norm(x, gamma, K, 1e-6)
    want = o.silu_multiply(o.matmul(n, rg, q.Q4_K, K, N).astype(np.float32),
                           o.matmul(n, ru, q.Q4_K, K, N).astype(np.float32))
    assert rel_l2(out.cpu().numpy(), want) < 1e-4
    # residual add epilogue: y += W a
    rd = q.synth_tensor_host(4, "sw.down", q.Q6_K, N, K)
    Wd = upload(cuda, q.Q6_K, N, K, rd)
    act = out.clone()
    resid = dev(cuda, q.synth_f32_host(4, "sw.res", K))
    base = resid.cpu().numpy().copy()
    warr1 = (C.c_void_p * 1)(Wd.data_ptr())
    q.check(q.lib().q4k_matmul_ex(act.data_ptr(), None, 0.0, 1, warr1, (C.c_int * 1)(q.Q6_K), (C.c_int64 * 1)(K),
                                  (C.c_void_p * 1)(resid.data_ptr()), N, 1, q.EPI_ADD, None, None, None))
    want = base + o.matmul(act.cpu().numpy(), rd, q.Q6_K, N, K).ravel().astype(np.float32)
    assert rel_l2(resid.cpu().numpy(), want) < 1e-5


@pytest.mark.parametrize("qt", [q.Q4_K, q.Q6_K])
def test_gemv_ring_shapes_agree(cuda, monkeypatch, qt):
    """Every ring size the planner accepts gives the same bits for a given
    number of consumer warps (per-row arithmetic does not depend on which
    team takes a stage; the warp count changes the RMSNorm sum's order), and
    every (warps, ring) shape matches the oracle.
    The small rings put fewer slots than teams (2-3 slots of ~46-67 KB
    SwiGLU stages for 3-4 teams), where each slot must still belong to a
    single team."""
    K, N = 2560, 1000
    rg = q.synth_tensor_host(6, "ring.gate", qt, K, N)
    ru = q.synth_tensor_host(6, "ring.up", qt, K, N)
    Wg, Wu = upload(cuda, qt, K, N, rg), upload(cuda, qt, K, N, ru)
    x = dev(cuda, q.synth_f32_host(6, "ring.x", K))
    gamma = dev(cuda, q.synth_tensor_host(6, "ring.g", q.F32, K, 1))
    n = o.rms_norm(x.cpu().numpy(), gamma.cpu().numpy(), K, 1e-6)
    want = o.silu_multiply(o.matmul(n, rg, qt, K, N).astype(np.float32),
                           o.matmul(n, ru, qt, K, N).astype(np.float32))
    results = {}
    for warps, kb in [(16, 200), (16, 96), (16, 64), (12, 200), (12, 96), (8, 96), (8, 40)]:
        monkeypatch.setenv("Q4K_GEMV_WARPS", str(warps))
        monkeypatch.setenv("Q4K_GEMV_SMEM_KB", str(kb))
        out = cuda.full((N,), float("nan"), device="cuda")
        q.check(q.lib().q4k_matmul_ex(x.data_ptr(), gamma.data_ptr(), 1e-6, 2,
                                      (C.c_void_p * 2)(Wg.data_ptr(), Wu.data_ptr()), (C.c_int * 2)(qt, qt),
                                      (C.c_int64 * 2)(N, N), (C.c_void_p * 2)(out.data_ptr(), out.data_ptr()), K, 1,
                                      q.EPI_SWIGLU, None, None, None))
        cuda.cuda.synchronize()
        results[(warps, kb)] = out.cpu().numpy()
        assert rel_l2(results[(warps, kb)], want) < 1e-4, (warps, kb)
    for (warps, kb), got in results.items():
        first = next(v for (w, _), v in results.items() if w == warps)
        assert np.array_equal(got, first), (warps, kb)


@pytest.mark.parametrize("epilogue", ["store", "swiglu"])
def test_gemv_tensor_core_stages(cuda, monkeypatch, epilogue):
    """Q4K_GEMV_MMA=1: Q4_K stages of K <= 3072 run their integer dot
    products on the tensor cores (mma m16n8k32, u8 x s8); they must match
    the oracle like the dp4a path, including partial last stages."""
    monkeypatch.setenv("Q4K_GEMV_MMA", "1")
    K, N = 2560, 1000
    rg = q.synth_tensor_host(8, "mma.gate", q.Q4_K, K, N)
    ru = q.synth_tensor_host(8, "mma.up", q.Q4_K, K, N)
    Wg, Wu = upload(cuda, q.Q4_K, K, N, rg), upload(cuda, q.Q4_K, K, N, ru)
    x = dev(cuda, q.synth_f32_host(8, "mma.x", K))
    gamma = dev(cuda, q.synth_tensor_host(8, "mma.g", q.F32, K, 1))
    n = o.rms_norm(x.cpu().numpy(), gamma.cpu().numpy(), K, 1e-6)
    out = cuda.full((N,), float("nan"), device="cuda")
    if epilogue == "swiglu":
        q.check(q.lib().q4k_matmul_ex(x.data_ptr(), gamma.data_ptr(), 1e-6, 2,
                                      (C.c_void_p * 2)(Wg.data_ptr(), Wu.data_ptr()), (C.c_int * 2)(q.Q4_K, q.Q4_K),
                                      (C.c_int64 * 2)(N, N), (C.c_void_p * 2)(out.data_ptr(), out.data_ptr()), K, 1,
                                      q.EPI_SWIGLU, None, None, None))
        want = o.silu_multiply(o.matmul(n, rg, q.Q4_K, K, N).astype(np.float32),
                               o.matmul(n, ru, q.Q4_K, K, N).astype(np.float32))
    else:
        q.check(q.lib().q4k_matmul_ex(x.data_ptr(), gamma.data_ptr(), 1e-6, 1, (C.c_void_p * 1)(Wg.data_ptr()),
                                      (C.c_int * 1)(q.Q4_K), (C.c_int64 * 1)(N), (C.c_void_p * 1)(out.data_ptr()),
                                      K, 1, q.EPI_STORE, None, None, None))
        want = o.matmul(n, rg, q.Q4_K, K, N).ravel()
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    assert rel_l2(got, want) < 1e-4
    assert np.mean(approx_ok(got, want, 3e-5, 1e-3)) > 0.999


def test_matmul_ex_argmax_head(cuda):
    K, N = 2560, 151936
    raw = q.synth_tensor_host(0x5EED, "token_embd.weight", q.Q6_K, K, N)
    W = upload(cuda, q.Q6_K, K, N, raw)
    x = q.synth_f32_host(2, "head.x", K)
    gamma = q.synth_tensor_host(2, "head.g", q.F32, K, 1)
    scratch = cuda.zeros(q.lib().q4k_matmul_argmax_scratch_bytes(), dtype=cuda.uint8, device="cuda")
    token = cuda.zeros(1, dtype=cuda.int32, device="cuda")
    logits = cuda.empty(N, device="cuda")
    for _ in range(2):  # the scratch counter must reset itself
        q.check(q.lib().q4k_matmul_ex(dev(cuda, x).data_ptr(), dev(cuda, gamma).data_ptr(), 1e-6, 1,
                                      (C.c_void_p * 1)(W.data_ptr()), (C.c_int * 1)(q.Q6_K), (C.c_int64 * 1)(N),
                                      (C.c_void_p * 1)(logits.data_ptr()), K, 1, q.EPI_ARGMAX, token.data_ptr(),
                                      scratch.data_ptr(), None))
        lg = logits.cpu().numpy()
        want = o.matmul(o.rms_norm(x, gamma, K, 1e-6), raw, q.Q6_K, K, N).ravel()
        assert rel_l2(lg, want) < 1e-5
        tok = int(token.cpu().numpy()[0])
        assert tok == o.argmax(lg)
        assert want[tok] >= want.max() - 1e-4 * abs(want.max())


# ------------------------------------------------------------ other kernels
def test_rms_norm_rope_silu_residual(cuda):
    L = q.lib()
    x = q.synth_f32_host(1, "e.x", 5 * 2560)
    g = q.synth_tensor_host(1, "e.g", q.F32, 2560, 1)
    y = cuda.empty(5 * 2560, device="cuda")
    q.check(L.q4k_rms_norm(dev(cuda, x).data_ptr(), dev(cuda, g).data_ptr(), y.data_ptr(), 5, 2560, 1e-6, None))
    assert rel_l2(y.cpu().numpy(), o.rms_norm(x, g, 2560, 1e-6)) < 1e-6
    # QK-norm shape: rows of 128
    y2 = cuda.empty(5 * 2560, device="cuda")
    g2 = q.synth_tensor_host(1, "e.g2", q.F32, 128, 1)
    q.check(L.q4k_rms_norm(dev(cuda, x).data_ptr(), dev(cuda, g2).data_ptr(), y2.data_ptr(), 100, 128, 1e-6, None))
    assert rel_l2(y2.cpu().numpy(), o.rms_norm(x, g2, 128, 1e-6)) < 1e-6
    for pos in (0, 17, 4095):
        r = q.synth_f32_host(1, "e.r", 3 * 32 * 128)
        t = dev(cuda, r)
        q.check(L.q4k_rope(t.data_ptr(), 3, 32, 128, pos, 1e6, None))
        # the angle float(pos) * powf(base, -2j/d) is rounded to fp32 (as the
        # reference forms it), so the device and host libm differ by a few ulp
        # of an angle of up to 4095 rad: ~3e-5 relative at the last position
        assert rel_l2(t.cpu().numpy(), o.rope(r, 3, 32, 128, pos, 1e6)) < 1e-4
        if o.ref_available():
            t2 = dev(cuda, r)
            o.ref_check(o.ref().ref_rope(t2.data_ptr(), 3, 32, 128, pos, 1e6))
            cuda.cuda.synchronize()
            assert np.array_equal(t.cpu().numpy(), t2.cpu().numpy())
    gg = q.synth_f32_host(1, "e.gate", 9728) * 4
    uu = q.synth_f32_host(1, "e.up", 9728)
    out = cuda.empty(9728, device="cuda")
    q.check(L.q4k_silu_multiply(dev(cuda, gg).data_ptr(), dev(cuda, uu).data_ptr(), out.data_ptr(), 9728, None))
    assert rel_l2(out.cpu().numpy(), o.silu_multiply(gg, uu)) < 1e-6
    s = dev(cuda, x[:2560])
    q.check(L.q4k_residual_add(s.data_ptr(), dev(cuda, g).data_ptr(), 2560, None))
    assert np.array_equal(s.cpu().numpy(), x[:2560] + g)


@pytest.mark.parametrize("shape", [(1, 0, 1, 1, 1), (35, 0, 4, 2, 128), (3, 31, 4, 1, 33), (1, 64, 4, 2, 256),
                                   (2, 32, 2, 2, 129), (1, 4095, 32, 8, 128)])
def test_attention_f32_reference_shapes(cuda, shape):
    queries, prefix, heads, kvh, dim = shape
    cached = prefix + queries
    # AttentionTests.cpp:45-52 inputs
    qv = (np.sin(np.arange(queries * heads * dim, dtype=np.float32) * np.float32(0.13)) * 2).astype(np.float32)
    kk = (np.cos(np.arange(cached * kvh * dim, dtype=np.float32) * np.float32(0.07)) * 9).astype(np.float32)
    vv = np.sin(np.arange(cached * kvh * dim, dtype=np.float32) * np.float32(0.11)).astype(np.float32)
    want = o.attention(qv, kk, vv, queries, heads, kvh, dim, prefix)
    out = cuda.full((want.size + 2,), 123.0, device="cuda")
    for _ in range(2):
        q.check(q.lib().q4k_attention(dev(cuda, qv).data_ptr(), dev(cuda, kk).data_ptr(), dev(cuda, vv).data_ptr(),
                                      out.data_ptr() + 4, queries, heads, kvh, dim, prefix, None))
        got = out.cpu().numpy()
        assert got[0] == 123.0 and got[-1] == 123.0
        assert np.abs(got[1:-1] - want).max() <= 3e-5


@pytest.mark.parametrize("n", [1, 7, 1000, 151936])
def test_argmax(cuda, n):
    lg = q.synth_f32_host(8, f"am.{n}", n)
    if n > 10:
        lg[n // 3] = lg[n // 2] = lg.max() + 1.0  # tie: the lower index wins
        lg[5] = np.nan
    r = C.c_uint32()
    q.check(q.lib().q4k_argmax(dev(cuda, lg).data_ptr(), n, C.byref(r), None))
    assert r.value == o.argmax(lg)


# ------------------------------------------------------ decode attention
@pytest.mark.parametrize("pos,kvh", [(0, 8), (1, 8), (63, 8), (64, 8), (300, 8), (4095, 8), (777, 2), (4095, 1)])
def test_attention_decode_f16(cuda, pos, kvh):
    H, D, cap = 4 * kvh, 128, 4096
    eps, base = 1e-6, 1e6
    qkv = q.synth_f32_host(pos, "dec.qkv", (H + 2 * kvh) * D) * 2
    gq = q.synth_tensor_host(1, "dec.gq", q.F32, D, 1)
    gk = q.synth_tensor_host(1, "dec.gk", q.F32, D, 1)
    kc = np.stack([q.synth_f16_host(3, "dec.k", h * (1 << 20) * D, cap * D) for h in range(kvh)]).ravel()
    vc = np.stack([q.synth_f16_host(3, "dec.v", h * (1 << 20) * D, cap * D) for h in range(kvh)]).ravel()
    kd, vd = dev(cuda, kc.view(np.int16)), dev(cuda, vc.view(np.int16))
    posd = cuda.tensor([pos], dtype=cuda.int32, device="cuda")
    out = cuda.empty(H * D, device="cuda")
    scratch = cuda.zeros(q.lib().q4k_attention_decode_scratch_bytes(H, kvh), dtype=cuda.uint8, device="cuda")
    q.check(q.lib().q4k_attention_decode_f16(dev(cuda, qkv).data_ptr(), dev(cuda, gq).data_ptr(),
                                             dev(cuda, gk).data_ptr(), kd.data_ptr(), vd.data_ptr(), cap,
                                             posd.data_ptr(), H, kvh, D, eps, base, out.data_ptr(),
                                             scratch.data_ptr(), None))
    got = out.cpu().numpy()
    # oracle: q/k norm + rope, fp16-rounded new k/v, fp32 attention
    qn = o.rope(o.rms_norm(qkv[: H * D], gq, D, eps), 1, H, D, pos, base)
    kn = o.rope(o.rms_norm(qkv[H * D:(H + kvh) * D], gk, D, eps), 1, kvh, D, pos, base)
    vn = qkv[(H + kvh) * D:]
    K = kc.view(np.float16).astype(np.float32).reshape(kvh, cap, D)[:, : pos + 1].copy()
    V = vc.view(np.float16).astype(np.float32).reshape(kvh, cap, D)[:, : pos + 1].copy()
    K[:, pos] = kn.reshape(kvh, D).astype(np.float16).astype(np.float32)
    V[:, pos] = vn.reshape(kvh, D).astype(np.float16).astype(np.float32)
    Kt = np.ascontiguousarray(K.transpose(1, 0, 2))
    Vt = np.ascontiguousarray(V.transpose(1, 0, 2))
    want = o.attention(qn, Kt, Vt, 1, H, kvh, D, pos)
    assert np.abs(got - want).max() <= 3e-5 + 1e-4 * np.abs(want).max()
    assert rel_l2(got, want) < 1e-4
    # the new K/V row landed in the cache as fp16
    kback = kd.cpu().numpy().view(np.uint16).reshape(kvh, cap, D)
    vback = vd.cpu().numpy().view(np.uint16).reshape(kvh, cap, D)
    assert np.abs(kback[:, pos].view(np.float16).astype(np.float32) - K[:, pos]).max() <= 2e-3 * np.abs(K[:, pos]).max()
    assert np.array_equal(vback[:, pos], vn.reshape(kvh, D).astype(np.float16).view(np.uint16))
    untouched = np.ones(cap, bool)
    untouched[pos] = False
    assert np.array_equal(kback[:, untouched], kc.reshape(kvh, cap, D)[:, untouched])


def test_synth_device_matches_host(cuda):
    for qt, K, N in ((q.Q4_K, 2560, 9), (q.Q6_K, 9728, 3), (q.Q6_K, 2560, 5)):
        raw = q.synth_tensor_host(77, "sd", qt, K, N)
        a = upload(cuda, qt, K, N, raw)
        b = cuda.empty_like(a)
        q.check(q.lib().q4k_synth_tensor_device(77, b"sd", qt, K, N, b.data_ptr(), None))
        cuda.cuda.synchronize()
        assert cuda.equal(a, b)
    x = cuda.empty(10000, device="cuda")
    q.check(q.lib().q4k_synth_f32_device(5, b"sx", 10000, x.data_ptr(), None))
    assert np.array_equal(x.cpu().numpy(), q.synth_f32_host(5, "sx", 10000))
