"""Generates tests/golden/ref_kernels.npz: outputs of the reference engine's
OWN CUDA kernels (oracle/_ref/libq4kref.so, compiled from the reference
sources by oracle/Makefile) on small seeded inputs, so the CPU oracle can be
pinned to the reference without a GPU.

Needs a CUDA device and the prebuilt oracle/_ref/libq4kref.so:

    python tests/golden/make_ref_golden.py [out.npz]

Cases (inputs are stored next to the outputs):
  dequant_{q4k,q6k}   kernels::dequantize_embeddings on 4 synthetic rows
  mm_{q4k,q6k}_K{2560,9728}_r{1,3,5}
                      kernels::matmul, 19 (K=2560) / 5 (K=9728) output rows,
                      N(0,1) inputs; 101 rows for one Q4_K case
  attn_{0..4}         kernels::attention on the five shapes and sin/cos
                      inputs of src/tests/AttentionTests.cpp:23-37
  rope, rms, silu     kernels::rope / rms_norm / silu_multiply
  argmax              kernels::argmax on logits with planted ties
  fwd_*               Engine::inference replay (src/Engine.cpp:37-114) of a
                      2-layer model (hidden 512, 4/1 heads of 128, ffn 768,
                      vocab 1000): a 5-token prefill then 3 decode steps
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "qwen3-4b-q4_k_m-inference-engine_b200", "python"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import oracle as o  # noqa: E402
import q4kb200 as q  # noqa: E402

sys.path.insert(0, HERE)
from tiny_model import SEED, TINY, tiny_tensors  # noqa: E402


_KEEP = []


def dev(a: np.ndarray) -> torch.Tensor:
    # kept alive for the whole run: a raw data_ptr() of a temporary could be
    # handed to the next allocation before the kernel reads it
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    _KEEP.append(t)
    return t


def main() -> None:
    out_path = sys.argv[1] if len(sys.argv) > 1 else os.path.join(HERE, "ref_kernels.npz")
    R = o.ref()
    out = {}

    # dequantize_embeddings
    for tag, qt in (("q4k", q.Q4_K), ("q6k", q.Q6_K)):
        raw = q.synth_tensor_host(SEED, f"golden.deq.{tag}", qt, 2560, 4)
        y = torch.empty(4 * 2560, device="cuda")
        o.ref_check(R.ref_dequantize_embeddings(dev(raw).data_ptr(), y.data_ptr(), 4, 2560,
                                                q.gguf_row_bytes(qt, 2560), qt))
        out[f"dequant_{tag}_raw"] = raw
        out[f"dequant_{tag}_out"] = y.cpu().numpy()

    # matmul
    cases = [(q.Q4_K, 2560, 19, (1, 3, 5, 101)), (q.Q6_K, 2560, 19, (1, 3, 5)), (q.Q4_K, 9728, 5, (1, 3)),
             (q.Q6_K, 9728, 5, (1, 3))]
    for qt, K, N, rows_list in cases:
        tag = f"{'q4k' if qt == q.Q4_K else 'q6k'}_K{K}"
        raw = q.synth_tensor_host(SEED, f"golden.mm.{tag}", qt, K, N)
        W = o.RefWeight(f"golden.mm.{tag}", qt, K, N, raw)
        out[f"mm_{tag}_w"] = raw
        for rows in rows_list:
            x = q.synth_f32_host(SEED, f"golden.mm.{tag}.x{rows}", rows * K)
            y = torch.full((rows * N,), 123.0, device="cuda")
            o.ref_check(R.ref_matmul(dev(x).data_ptr(), W.h, y.data_ptr(), rows, None))
            torch.cuda.synchronize()
            out[f"mm_{tag}_r{rows}_x"] = x
            out[f"mm_{tag}_r{rows}_y"] = y.cpu().numpy()

    # attention: src/tests/AttentionTests.cpp:23-37 shapes and inputs
    shapes = [(1, 0, 1, 1, 1), (35, 0, 4, 2, 128), (3, 31, 4, 1, 33), (1, 64, 4, 2, 256), (2, 32, 2, 2, 129)]
    for i, (queries, prefix, heads, kvh, dim) in enumerate(shapes):
        cached = prefix + queries
        qv = (np.sin(np.arange(queries * heads * dim, dtype=np.float32) * np.float32(0.13)) * 2).astype(np.float32)
        kk = (np.cos(np.arange(cached * kvh * dim, dtype=np.float32) * np.float32(0.07)) * 9).astype(np.float32)
        vv = np.sin(np.arange(cached * kvh * dim, dtype=np.float32) * np.float32(0.11)).astype(np.float32)
        y = torch.empty(queries * heads * dim, device="cuda")
        qd, kd, vd = dev(qv), dev(kk), dev(vv)  # keep the device copies alive across the call
        o.ref_check(R.ref_attention(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), y.data_ptr(),
                                    queries, heads, kvh, dim, prefix))
        torch.cuda.synchronize()
        out[f"attn_{i}_shape"] = np.array([queries, prefix, heads, kvh, dim], np.int64)
        out[f"attn_{i}_q"], out[f"attn_{i}_k"], out[f"attn_{i}_v"] = qv, kk, vv
        out[f"attn_{i}_out"] = y.cpu().numpy()

    # rope
    xr = q.synth_f32_host(SEED, "golden.rope", 3 * 4 * 128)
    t = dev(xr)
    o.ref_check(R.ref_rope(t.data_ptr(), 3, 4, 128, 4090, 1e6))
    torch.cuda.synchronize()
    out["rope_x"], out["rope_out"] = xr, t.cpu().numpy()

    # rms_norm
    xn = q.synth_f32_host(SEED, "golden.rms.x", 3 * 2560)
    gm = q.synth_tensor_host(SEED, "golden.rms.g", q.F32, 2560, 1)
    G = o.RefWeight("golden.rms.g", q.F32, 2560, 1, gm)
    y = torch.empty(3 * 2560, device="cuda")
    o.ref_check(R.ref_rms_norm(dev(xn).data_ptr(), G.h, y.data_ptr(), 3, 2560, 1e-6))
    torch.cuda.synchronize()
    out["rms_x"], out["rms_g"], out["rms_out"] = xn, gm, y.cpu().numpy()

    # silu_multiply
    g = q.synth_f32_host(SEED, "golden.silu.g", 1000) * 4
    u = q.synth_f32_host(SEED, "golden.silu.u", 1000)
    y = torch.empty(1000, device="cuda")
    gd, ud = dev(g), dev(u)
    o.ref_check(R.ref_silu_multiply(gd.data_ptr(), ud.data_ptr(), y.data_ptr(), 1000))
    torch.cuda.synchronize()
    out["silu_g"], out["silu_u"], out["silu_out"] = g, u, y.cpu().numpy()

    # argmax with ties: two maxima, the lower index must win
    lg = q.synth_f32_host(SEED, "golden.argmax", 151936)
    lg[777] = lg[150000] = 9.0
    res = o.C.c_uint32()
    o.ref_check(R.ref_argmax(dev(lg).data_ptr(), lg.size, o.C.byref(res)))
    out["argmax_logits"], out["argmax_out"] = lg, np.array([res.value], np.int64)

    # Engine::inference replay on the tiny model
    c = TINY
    tensors = tiny_tensors(c)
    handles = {n: o.RefWeight(n, t, a, b, data) for n, (t, a, b, data) in tensors.items()}
    order = [f"blk.{i}.{s}.weight" for i in range(c["layers"]) for s in o.SLOT_NAMES]
    order += ["output_norm.weight", "token_embd.weight"]
    ptrs = (o.C.c_void_p * len(order))(*[handles[n].h.value for n in order])
    cap = 16
    kvw = c["kv_heads"] * c["head_dim"]
    kc = torch.zeros(c["layers"] * cap * kvw, device="cuda")
    vc = torch.zeros_like(kc)
    tokens = [3, 141, 592, 653, 589]
    steps = []
    embd = tensors["token_embd.weight"][3]
    pos = 0
    pending = tokens
    for step in range(4):
        toks = np.array(pending, np.uint32)
        logits = torch.empty(c["vocab"], device="cuda")
        hidden = torch.empty((c["layers"] + 1) * c["hidden"], device="cuda")
        nxt = o.C.c_uint32()
        o.ref_check(R.ref_forward(ptrs, c["layers"], c["hidden"], c["heads"], c["kv_heads"], c["head_dim"], c["ffn"],
                                  c["vocab"], c["eps"], c["rope_base"], embd.ctypes.data, q.gguf_row_bytes(q.Q6_K, c["hidden"]),
                                  kc.data_ptr(), vc.data_ptr(), cap, toks.ctypes.data, toks.size, pos, 1,
                                  logits.data_ptr(), hidden.data_ptr(), o.C.byref(nxt)))
        torch.cuda.synchronize()
        out[f"fwd_{step}_tokens"] = toks
        out[f"fwd_{step}_pos"] = np.array([pos], np.int64)
        out[f"fwd_{step}_logits"] = logits.cpu().numpy()
        out[f"fwd_{step}_hidden"] = hidden.cpu().numpy()
        out[f"fwd_{step}_next"] = np.array([nxt.value], np.int64)
        steps.append(nxt.value)
        pos += toks.size
        pending = [nxt.value]
    out["fwd_kcache"] = kc.cpu().numpy()
    out["fwd_vcache"] = vc.cpu().numpy()
    np.savez_compressed(out_path, **out)
    print("wrote", out_path, len(out), "arrays; greedy tokens", steps)


if __name__ == "__main__":
    main()
