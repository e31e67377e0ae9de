"""The C ABI without a GPU: the library loads, exports every function that
include/q4k_b200.h declares (and the C++ drop-in of include/Kernels.hpp),
host-side helpers are deterministic, and argument checks reject bad calls
before any CUDA work (the reference's std::invalid_argument cases)."""
import ctypes as C
import os
import re
import subprocess

import numpy as np
import pytest

import q4kb200 as q
from conftest import ROOT


def header_functions():
    text = open(os.path.join(ROOT, "include", "q4k_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(q4k_\w+)\s*\(", text)))


def exported_symbols():
    out = subprocess.run(["nm", "-D", "--defined-only", q.LIB_PATH], capture_output=True, text=True, check=True)
    return {line.split()[-1] for line in out.stdout.splitlines() if " T " in line}


def test_library_exports_every_declared_function():
    declared = header_functions()
    assert len(declared) >= 30
    syms = exported_symbols()
    missing = [f for f in declared if f not in syms]
    assert not missing, missing
    assert set(q.EXPORTS) == set(declared)
    q.lib()  # loads and binds every signature


def test_cpp_dropin_symbols_exported():
    syms = exported_symbols()
    for mangled in ("_ZN7kernels6matmulEPKfRK6WeightPfmP11CUstream_st", "_ZN7kernels9attentionEPKfS1_S1_Pfmmmmm",
                    "_ZN7kernels8rms_normEPKfRK6WeightPfmmf", "_ZN7kernels4ropeEPfmmmmf", "_ZN7kernels6argmaxEPKfm",
                    "_ZN7kernels21dequantize_embeddingsEPKvPfmmm9ggml_type", "_ZN7kernels10CudaStreamC1Ev"):
        assert mangled in syms, mangled


def test_abi_version_and_sizes():
    L = q.lib()
    assert L.q4k_abi_version() == 2
    assert C.sizeof(q.EngineConfig) == 14 * 4
    assert q.device_bytes(q.Q4_K, 2560, 9728) == 9728 * 1440
    assert q.device_bytes(q.Q6_K, 2560, 1024) == 1024 * (10 * 208 + 32)
    assert q.device_bytes(q.Q6_K, 9728, 2560) == 2560 * (38 * 208 + 80)
    assert q.device_bytes(q.Q4_K, 100, 5) == 0
    assert L.q4k_matmul_argmax_scratch_bytes() > 0
    assert L.q4k_attention_decode_scratch_bytes(32, 8) > 0


def test_synthetic_tensors_deterministic_and_distinct():
    a = q.synth_tensor_host(7, "blk.0.attn_q.weight", q.Q4_K, 2560, 3)
    b = q.synth_tensor_host(7, "blk.0.attn_q.weight", q.Q4_K, 2560, 3)
    c = q.synth_tensor_host(8, "blk.0.attn_q.weight", q.Q4_K, 2560, 3)
    d = q.synth_tensor_host(7, "blk.0.attn_k.weight", q.Q4_K, 2560, 3)
    assert np.array_equal(a, b) and not np.array_equal(a, c) and not np.array_equal(a, d)
    # a prefix of rows is the same tensor's first rows (block index = row * nb + b)
    e = q.synth_tensor_host(7, "blk.0.attn_q.weight", q.Q4_K, 2560, 1)
    assert np.array_equal(e, a[: e.size])


def test_synthetic_distributions():
    import oracle as o

    raw = q.synth_tensor_host(1, "dist.q4", q.Q4_K, 256, 4096).reshape(-1, 144)
    d = raw[:, 0:2].copy().view(np.float16).astype(np.float32).ravel()
    assert np.all(d >= 0) and abs(np.mean(d) / 2e-3 - np.sqrt(2 / np.pi)) < 0.05
    raw6 = q.synth_tensor_host(1, "dist.q6", q.Q6_K, 256, 4096).reshape(-1, 210)
    sc = raw6[:, 192:208].view(np.int8)
    assert sc.min() == -32 and sc.max() == 31
    g = q.synth_tensor_host(1, "dist.g", q.F32, 100000, 1)
    assert abs(g.mean() - 1) < 1e-3 and abs(g.std() - 0.02) < 1e-3
    x = q.synth_f32_host(1, "dist.x", 200000)
    assert abs(x.mean()) < 0.01 and abs(x.std() - 1) < 0.01
    # the oracle decodes generated blocks without surprises
    assert np.isfinite(o.dequantize_rows(raw6.ravel(), o.Q6_K, 4096, 256)).all()


def test_model_tensor_list():
    cfg = q.qwen3_4b_config(4096)
    ts = q.model_tensors(cfg)
    assert len(ts) == 36 * 11 + 2
    names = {t[0]: t[1:] for t in ts}
    assert names["token_embd.weight"] == (q.Q6_K, 2560, 151936)
    assert names["blk.0.attn_v.weight"] == (q.Q6_K, 2560, 1024)
    assert names["blk.0.ffn_down.weight"][0] == q.Q6_K and names["blk.1.ffn_down.weight"][0] == q.Q4_K
    assert sum(1 for n, t in names.items() if n.endswith("ffn_down.weight") and t[0] == q.Q6_K) == 18
    weight_bytes = sum(b * q.gguf_row_bytes(t, a) for _, t, a, b in ts)
    # per-token weight bytes of the decode step, norms included
    assert weight_bytes == 2503489024


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_tp_shards_partition_every_tensor(world):
    cfg = q.qwen3_4b_config(4096)
    ts = q.model_tensors(cfg)
    for i, (name, t, ne0, ne1) in enumerate(ts):
        shards = [q.tp_shard(cfg, i, r, world) for r in range(world)]
        rows = [(n0, n1) for n0, n1, _, _ in shards]
        blocks = [(b0, b1) for _, _, b0, b1 in shards]
        if all(r == (0, ne1) for r in rows) and all(b == (0, max(ne0 // 256, 0)) for b in blocks):
            continue  # replicated
        if all(b == blocks[0] for b in blocks):  # row split
            assert rows[0][0] == 0 and rows[-1][1] == ne1
            assert all(rows[k][1] == rows[k + 1][0] for k in range(world - 1)), name
        else:  # K split on super-blocks
            assert blocks[0][0] == 0 and blocks[-1][1] == ne0 // 256
            assert all(blocks[k][1] == blocks[k + 1][0] for k in range(world - 1)), name
    # ffn_down K-shards at 8 ranks: 38 blocks -> 4 or 5 each, and gate rows align with them
    i_down = [i for i, t in enumerate(ts) if t[0] == "blk.0.ffn_down.weight"][0]
    i_gate = [i for i, t in enumerate(ts) if t[0] == "blk.0.ffn_gate.weight"][0]
    for r in range(world):
        n0, n1, _, _ = q.tp_shard(cfg, i_gate, r, world)
        _, _, b0, b1 = q.tp_shard(cfg, i_down, r, world)
        assert (n0, n1) == (b0 * 256, b1 * 256)


def test_argument_validation_needs_no_gpu():
    L = q.lib()
    P = C.c_void_p
    # unsupported weight type (matmul.cu:132-133)
    assert L.q4k_matmul(P(16), P(16), 3, 2560, 4, P(16), 1, None) == q.EINVAL
    # K not a multiple of 256 (matmul.cu:134-136)
    assert L.q4k_matmul(P(16), P(16), q.Q4_K, 100, 4, P(16), 1, None) == q.EINVAL
    assert b"dimensions" in L.q4k_last_error()
    # zero rows: nothing to do
    assert L.q4k_matmul(P(16), P(16), q.Q4_K, 256, 4, P(16), 0, None) == q.OK
    # attention: heads not divisible, head_dim > 256 (attention.cu:98-102)
    assert L.q4k_attention(P(16), P(16), P(16), P(16), 1, 3, 2, 64, 0, None) == q.EINVAL
    assert L.q4k_attention(P(16), P(16), P(16), P(16), 1, 4, 2, 257, 0, None) == q.EINVAL
    assert L.q4k_attention(P(16), P(16), P(16), P(16), 0, 3, 2, 64, 0, None) == q.OK
    # rope: odd head_dim, non-positive base (rope.cu:34-35)
    assert L.q4k_rope(P(16), 1, 1, 3, 0, 1e6, None) == q.EINVAL
    assert L.q4k_rope(P(16), 1, 1, 4, 0, 0.0, None) == q.EINVAL
    # rms_norm: epsilon must be positive (rms_norm.cu:34-36)
    assert L.q4k_rms_norm(P(16), P(16), P(16), 1, 8, 0.0, None) == q.EINVAL
    # dequantize_embeddings: other storage types rejected (embedding.cu:69-70)
    assert L.q4k_dequantize_embeddings(P(16), P(16), 1, 256, 144, q.F32, None) == q.EINVAL
    # argmax: empty or oversized vocabulary (argmax.cu:73-74)
    r = C.c_uint32()
    assert L.q4k_argmax(P(16), 0, C.byref(r), None) == q.EINVAL
    assert L.q4k_argmax(None, 10, C.byref(r), None) == q.EINVAL
    # fused entry points
    assert L.q4k_attention_decode_f16(P(16), P(16), P(16), P(16), P(16), 8, P(16), 8, 4, 128, 1e-6, 1e6, P(16),
                                      P(16), None) == q.EINVAL
    # prefill without an engine, tokens or result
    assert L.q4k_engine_prefill(None, P(16), 1, 0, C.byref(r), None) == q.EINVAL
    assert L.q4k_engine_prefill_seq(None, 0, P(16), 1, 0, C.byref(r), None) == q.EINVAL
    assert L.q4k_engine_decode_batch(None, 1, P(16), P(16), P(16), P(16), None) == q.EINVAL
    # batched products: no argmax epilogue, at most 3 weights, K up to 10240
    w1, t1 = (C.c_void_p * 1)(16), (C.c_int * 1)(q.Q4_K)
    r1, o1 = (C.c_int64 * 1)(256), (C.c_void_p * 1)(16)
    assert L.q4k_matmul_batch(P(16), None, 0.0, 1, w1, t1, r1, o1, 256, 2560, 4, q.EPI_ARGMAX, None) == q.EINVAL
    assert L.q4k_matmul_batch(P(16), None, 0.0, 4, w1, t1, r1, o1, 256, 2560, 4, q.EPI_STORE, None) == q.EINVAL
    assert L.q4k_matmul_batch(P(16), None, 0.0, 1, w1, t1, r1, o1, 256, 10496, 4, q.EPI_STORE, None) == q.EINVAL
    assert L.q4k_matmul_batch(P(16), None, 0.0, 1, w1, t1, r1, o1, 128, 2560, 4, q.EPI_STORE, None) == q.EINVAL
    assert L.q4k_matmul_batch(P(16), None, 0.0, 1, w1, t1, r1, o1, 256, 2560, 0, q.EPI_STORE, None) == q.OK
    # engine configuration checks happen before any device work
    cfg = q.qwen3_4b_config(4096)
    cfg.head_dim = 64
    h = C.c_void_p()
    assert L.q4k_engine_create(C.byref(cfg), None, C.byref(h)) == q.EINVAL
    cfg = q.qwen3_4b_config(4096)
    cfg.tp_world, cfg.tp_rank = 3, 0
    assert L.q4k_engine_create(C.byref(cfg), None, C.byref(h)) == q.EINVAL
    cfg = q.qwen3_4b_config(4096)
    cfg.sequences = -1
    assert L.q4k_engine_create(C.byref(cfg), None, C.byref(h)) == q.EINVAL
