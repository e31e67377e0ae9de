"""q4k_attention_decode_f16_static: the allocation-free decode attention.

Compared bit for bit against q4k_attention_decode_f16 (the same kernel with
caller-owned scratch) on two calls in a row, each variant on its own copy
of the caches, so that the fixed scratch's counters are shown to reset
between calls. Collected last (file name) so that it also runs after every
other GPU test in one process; it passes alone as well."""
import numpy as np
import pytest

import q4kb200 as q

pytestmark = pytest.mark.gpu

H_KV, D, CAP = 8, 128, 4096
H = 4 * H_KV


def _case(cuda, seed):
    qkv = q.synth_f32_host(seed, "noalloc.qkv", (H + 2 * H_KV) * D) * 2
    gq = q.synth_tensor_host(seed, "noalloc.gq", q.F32, D, 1)
    gk = q.synth_tensor_host(seed, "noalloc.gk", q.F32, D, 1)
    return [cuda.from_numpy(np.ascontiguousarray(a)).cuda() for a in (qkv, gq, gk)]


def _caches(cuda):
    kc = np.stack([q.synth_f16_host(5, "noalloc.k", h * (1 << 20) * D, CAP * D) for h in range(H_KV)]).ravel()
    vc = np.stack([q.synth_f16_host(5, "noalloc.v", h * (1 << 20) * D, CAP * D) for h in range(H_KV)]).ravel()
    return (cuda.from_numpy(kc.view(np.int16)).cuda(), cuda.from_numpy(vc.view(np.int16)).cuda())


def test_static_matches_regular_two_calls(cuda):
    L = q.lib()
    k_reg, v_reg = _caches(cuda)
    k_sta, v_sta = _caches(cuda)
    scratch = cuda.zeros(L.q4k_attention_decode_scratch_bytes(H, H_KV), dtype=cuda.uint8, device="cuda")
    for pos, seed in ((4095, 11), (777, 12)):
        qkv, gq, gk = _case(cuda, seed)
        posd = cuda.tensor([pos], dtype=cuda.int32, device="cuda")
        out_reg = cuda.full((H * D,), float("nan"), device="cuda")
        out_sta = cuda.full((H * D,), float("nan"), device="cuda")
        q.check(L.q4k_attention_decode_f16(qkv.data_ptr(), gq.data_ptr(), gk.data_ptr(), k_reg.data_ptr(),
                                           v_reg.data_ptr(), CAP, posd.data_ptr(), H, H_KV, D, 1e-6, 1e6,
                                           out_reg.data_ptr(), scratch.data_ptr(), None))
        q.check(L.q4k_attention_decode_f16_static(qkv.data_ptr(), gq.data_ptr(), gk.data_ptr(), k_sta.data_ptr(),
                                                  v_sta.data_ptr(), CAP, posd.data_ptr(), H, H_KV, D, 1e-6, 1e6,
                                                  out_sta.data_ptr(), None))
        cuda.cuda.synchronize()
        a, b = out_reg.cpu().numpy(), out_sta.cpu().numpy()
        assert np.isfinite(b).all()
        assert np.array_equal(a, b), pos
        assert np.array_equal(k_reg.cpu().numpy(), k_sta.cpu().numpy()), pos
        assert np.array_equal(v_reg.cpu().numpy(), v_sta.cpu().numpy()), pos


def test_static_rejects_what_does_not_fit(cuda, monkeypatch):
    L = q.lib()
    qkv, gq, gk = _case(cuda, 13)
    k, v = _caches(cuda)
    posd = cuda.tensor([10], dtype=cuda.int32, device="cuda")
    out = cuda.empty(H * D, device="cuda")
    args = (qkv.data_ptr(), gq.data_ptr(), gk.data_ptr(), k.data_ptr(), v.data_ptr(), CAP, posd.data_ptr())
    # four CTAs per SM and KV head: 32 heads x 74 splits x 520 B > 1 MiB
    monkeypatch.setenv("Q4K_ATTN_CTAS_PER_SM", "4")
    rc = L.q4k_attention_decode_f16_static(*args, H, H_KV, D, 1e-6, 1e6, out.data_ptr(), None)
    assert rc == 2 and b"static scratch holds" in L.q4k_last_error()
    monkeypatch.delenv("Q4K_ATTN_CTAS_PER_SM")
    # more KV heads than the 256-byte counter block holds
    rc = L.q4k_attention_decode_f16_static(*args, 4 * 65, 65, D, 1e-6, 1e6, out.data_ptr(), None)
    assert rc == 1
