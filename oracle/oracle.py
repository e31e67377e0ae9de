"""ctypes bindings for the CPU oracle (lib/liboracle.so) and for the
reference engine's own kernels (_ref/libq4kref.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
the cpu_baseline / reference legs of bench.py as the checker. The product
package never imports this module.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "lib", "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libq4kref.so")

F32, F16, Q4_K, Q6_K = 0, 1, 12, 14
SLOTS = 11
SLOT_NAMES = ("attn_norm", "attn_q", "attn_k", "attn_v", "attn_q_norm", "attn_k_norm", "attn_output",
              "ffn_norm", "ffn_gate", "ffn_up", "ffn_down")

_lib = None
_ref = None


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            build()
        L = C.CDLL(ORACLE_SO)
        P = C.c_void_p
        L.orc_dequant_block_q4k.argtypes = [P, P]
        L.orc_dequant_block_q6k.argtypes = [P, P]
        L.orc_dequantize_rows.argtypes = [P, P, C.c_size_t, C.c_size_t, C.c_size_t, C.c_int]
        L.orc_quantize_q8.argtypes = [P, C.c_size_t, P, P]
        L.orc_matmul.argtypes = [P, P, C.c_int, C.c_size_t, C.c_size_t, C.c_size_t, P, C.c_int]
        L.orc_rms_norm.argtypes = [P, P, P, C.c_size_t, C.c_size_t, C.c_float]
        L.orc_rope.argtypes = [P, C.c_size_t, C.c_size_t, C.c_size_t, C.c_size_t, C.c_float]
        L.orc_attention.argtypes = [P, P, P, P, C.c_size_t, C.c_size_t, C.c_size_t, C.c_size_t, C.c_size_t]
        L.orc_silu_multiply.argtypes = [P, P, P, C.c_size_t]
        L.orc_residual_add.argtypes = [P, P, C.c_size_t]
        L.orc_argmax.argtypes = [P, C.c_size_t]
        L.orc_argmax.restype = C.c_uint32
        L.orc_half_to_float.argtypes = [C.c_uint16]
        L.orc_half_to_float.restype = C.c_float
        L.orc_float_to_half.argtypes = [C.c_float]
        L.orc_float_to_half.restype = C.c_uint16
        L.orc_forward.argtypes = [P, P, P, C.c_size_t, P, C.c_size_t, C.c_size_t, C.c_int, P, P, P, C.c_int]
        L.orc_layer.argtypes = [P, C.c_int, P, P, P, C.c_size_t, C.c_size_t, C.c_size_t, C.c_int, C.c_int]
        L.orc_synth_key.argtypes = [C.c_uint64, C.c_char_p]
        L.orc_synth_key.restype = C.c_uint64
        L.orc_synth_tensor.argtypes = [C.c_uint64, C.c_char_p, C.c_int, C.c_int64, C.c_int64, P]
        L.orc_synth_f16.argtypes = [C.c_uint64, C.c_char_p, C.c_uint64, C.c_size_t, P]
        L.orc_synth_f32.argtypes = [C.c_uint64, C.c_char_p, C.c_size_t, P]
        L.orc_omp_threads.argtypes = [C.c_int]
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


def row_bytes(qtype: int, K: int) -> int:
    return (K // 256) * (144 if qtype == Q4_K else 210)


# --------------------------------------------------------------------------
# The benchmark's synthetic model, built here without the product library
# (q4k_synth.c restates its seeded streams; the CPU tests compare the bytes).
# --------------------------------------------------------------------------
def qwen3_4b_config(capacity: int = 4096) -> dict:
    """Qwen3-4B shapes (Engine.cpp:49-55 metadata of the real model)."""
    return {"layers": 36, "hidden": 2560, "heads": 32, "kv_heads": 8, "head_dim": 128, "ffn": 9728,
            "vocab": 151936, "eps": 1e-6, "rope_base": 1e6, "capacity": capacity}


def model_tensors(cfg: dict):
    """(name, type, ne0, ne1) of every tensor of the synthetic Q4_K_M model
    in the engine's order: per layer the eleven Engine.cpp:82-109 tensors
    (Q6_K for attn_v and the ffn_down of even layers, Q4_K for the other
    matrices, F32 norms), then output_norm and token_embd (Q6_K, the head)."""
    qd, kvd = cfg["heads"] * cfg["head_dim"], cfg["kv_heads"] * cfg["head_dim"]
    H, F = cfg["hidden"], cfg["ffn"]
    out = []
    for i in range(cfg["layers"]):
        shapes = {"attn_norm": (F32, H, 1), "attn_q": (Q4_K, H, qd), "attn_k": (Q4_K, H, kvd),
                  "attn_v": (Q6_K, H, kvd), "attn_q_norm": (F32, cfg["head_dim"], 1),
                  "attn_k_norm": (F32, cfg["head_dim"], 1), "attn_output": (Q4_K, qd, H), "ffn_norm": (F32, H, 1),
                  "ffn_gate": (Q4_K, H, F), "ffn_up": (Q4_K, H, F),
                  "ffn_down": (Q6_K if i % 2 == 0 else Q4_K, F, H)}
        for s in SLOT_NAMES:
            t, a, b = shapes[s]
            out.append((f"blk.{i}.{s}.weight", t, a, b))
    out.append(("output_norm.weight", F32, H, 1))
    out.append(("token_embd.weight", Q6_K, H, cfg["vocab"]))
    return out


def synth_tensor(seed: int, name: str, qtype: int, ne0: int, ne1: int) -> np.ndarray:
    """Tensor `name` of the seeded synthetic model in GGUF layout (float32
    values for F32, raw super-block bytes otherwise)."""
    if qtype == F32:
        out = np.empty(ne0 * ne1, np.float32)
    else:
        out = np.empty(ne1 * row_bytes(qtype, ne0), np.uint8)
    if lib().orc_synth_tensor(seed, name.encode(), qtype, ne0, ne1, _p(out)):
        raise ValueError(f"bad synthetic tensor request {name}")
    return out


def synth_f16(seed: int, name: str, index_base: int, n: int) -> np.ndarray:
    out = np.empty(n, np.uint16)
    lib().orc_synth_f16(seed, name.encode(), index_base, n, _p(out))
    return out


def synth_f32(seed: int, name: str, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().orc_synth_f32(seed, name.encode(), n, _p(out))
    return out


def omp_threads(requested: int = 0) -> int:
    """Threads an OpenMP region of the oracle gets when asked for
    `requested` (<= 0: the OpenMP default, e.g. OMP_NUM_THREADS)."""
    return int(lib().orc_omp_threads(requested))


def dequantize_rows(packed: np.ndarray, qtype: int, rows: int, width: int, row_bytes_: int | None = None):
    rb = row_bytes(qtype, width) if row_bytes_ is None else row_bytes_
    out = np.empty((rows, width), np.float32)
    rc = lib().orc_dequantize_rows(_p(np.ascontiguousarray(packed)), _p(out), rows, width, rb, qtype)
    if rc:
        raise ValueError("unsupported type")
    return out


def quantize_q8(x: np.ndarray):
    x = np.ascontiguousarray(x, np.float32).ravel()
    codes = np.empty(x.size, np.int8)
    scales = np.empty(x.size // 32, np.float32)
    lib().orc_quantize_q8(_p(x), x.size, _p(codes), _p(scales))
    return codes, scales


def matmul(x: np.ndarray, w: np.ndarray, qtype: int, K: int, N: int, threads: int = 0) -> np.ndarray:
    """y[rows][N] in float64 (MatmulReference.hpp:42-64)."""
    x = np.ascontiguousarray(x, np.float32)
    rows = x.size // K
    y = np.empty((rows, N), np.float64)
    rc = lib().orc_matmul(_p(x), _p(np.ascontiguousarray(w)), qtype, K, N, rows, _p(y), threads)
    if rc:
        raise ValueError(f"orc_matmul failed: {rc}")
    return y


def rms_norm(x: np.ndarray, gamma: np.ndarray, width: int, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().orc_rms_norm(_p(x), _p(np.ascontiguousarray(gamma, np.float32)), _p(y), x.size // width, width, eps)
    return y


def rope(x: np.ndarray, tokens: int, heads: int, head_dim: int, pos: int, base: float) -> np.ndarray:
    y = np.array(x, np.float32, copy=True, order="C")
    lib().orc_rope(_p(y), tokens, heads, head_dim, pos, base)
    return y


def attention(q, k, v, tokens, heads, kv_heads, head_dim, offset) -> np.ndarray:
    q = np.ascontiguousarray(q, np.float32)
    out = np.empty(tokens * heads * head_dim, np.float32)
    rc = lib().orc_attention(_p(q), _p(np.ascontiguousarray(k, np.float32)), _p(np.ascontiguousarray(v, np.float32)),
                             _p(out), tokens, heads, kv_heads, head_dim, offset)
    if rc:
        raise ValueError("bad attention shape")
    return out


def silu_multiply(g, u) -> np.ndarray:
    g = np.ascontiguousarray(g, np.float32)
    out = np.empty_like(g)
    lib().orc_silu_multiply(_p(g), _p(np.ascontiguousarray(u, np.float32)), _p(out), g.size)
    return out


def argmax(logits: np.ndarray) -> int:
    logits = np.ascontiguousarray(logits, np.float32)
    return int(lib().orc_argmax(_p(logits), logits.size))


class Model:
    """Weights in GGUF layout for orc_forward; `tensors` maps GGUF names
    (blk.{i}.attn_q.weight, output_norm.weight, token_embd.weight) to
    (type, numpy bytes/float32 array)."""

    def __init__(self, cfg: dict, tensors: dict):
        self.cfg = cfg
        L = cfg["layers"]
        self.keep = []
        ptrs = (C.c_void_p * (SLOTS * L + 2))()
        types = (C.c_int * (SLOTS * L + 2))()
        for i in range(L):
            for s, nm in enumerate(SLOT_NAMES):
                t, arr = tensors[f"blk.{i}.{nm}.weight"]
                arr = np.ascontiguousarray(arr)
                self.keep.append(arr)
                ptrs[SLOTS * i + s] = arr.ctypes.data
                types[SLOTS * i + s] = t
        for j, nm in enumerate(("output_norm.weight", "token_embd.weight")):
            t, arr = tensors[nm]
            arr = np.ascontiguousarray(arr)
            self.keep.append(arr)
            ptrs[SLOTS * L + j] = arr.ctypes.data
            types[SLOTS * L + j] = t
        self.ptrs, self.types = ptrs, types

        class _M(C.Structure):
            _fields_ = [("layers", C.c_int), ("hidden", C.c_int), ("heads", C.c_int), ("kv_heads", C.c_int),
                        ("head_dim", C.c_int), ("ffn", C.c_int), ("vocab", C.c_int), ("eps", C.c_float),
                        ("rope_base", C.c_float), ("tensors", C.c_void_p), ("types", C.c_void_p)]

        self.m = _M(L, cfg["hidden"], cfg["heads"], cfg["kv_heads"], cfg["head_dim"], cfg["ffn"], cfg["vocab"],
                    cfg["eps"], cfg["rope_base"], C.cast(ptrs, C.c_void_p), C.cast(types, C.c_void_p))

    def forward(self, k_cache, v_cache, capacity, tokens, pos, kv_round_f16=True, want_logits=True,
                want_hidden=True, threads=0):
        cfg = self.cfg
        toks = np.ascontiguousarray(np.asarray(tokens, np.uint32))
        logits = np.empty(cfg["vocab"], np.float32) if want_logits else None
        hidden = np.empty((cfg["layers"] + 1, cfg["hidden"]), np.float32) if want_hidden else None
        nxt = C.c_uint32(0)
        rc = lib().orc_forward(C.byref(self.m), _p(k_cache), _p(v_cache), capacity, _p(toks), toks.size, pos,
                               int(kv_round_f16), _p(logits) if logits is not None else None,
                               _p(hidden) if hidden is not None else None, C.byref(nxt), threads)
        if rc:
            raise RuntimeError(f"orc_forward failed: {rc}")
        return int(nxt.value), logits, hidden

    def layer(self, layer, x, k_cache, v_cache, capacity, pos, kv_round_f16=True, threads=0):
        """One block (orc_layer) on rows x [tokens][hidden] at positions
        pos.. ; k_cache / v_cache: this layer's fp32 caches
        [capacity][kv_heads*head_dim] (written). Returns the new rows."""
        y = np.array(x, np.float32, copy=True, order="C")
        tokens = y.size // self.cfg["hidden"]
        rc = lib().orc_layer(C.byref(self.m), layer, _p(y), _p(k_cache), _p(v_cache), capacity, tokens, pos,
                             int(kv_round_f16), threads)
        if rc:
            raise RuntimeError(f"orc_layer failed: {rc}")
        return y


# --------------------------------------------------------------------------
# Reference kernels (GPU). Pointers are raw device addresses (ints).
# --------------------------------------------------------------------------
def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref():
    global _ref
    if _ref is None:
        if not os.path.exists(REF_SO):
            raise RuntimeError("reference kernel library was not built (oracle/_ref/libq4kref.so missing)")
        L = C.CDLL(REF_SO)
        P, S = C.c_void_p, C.c_size_t
        L.ref_last_error.restype = C.c_char_p
        L.ref_weight_create.argtypes = [C.c_char_p, C.c_int, C.c_int64, C.c_int64, P, S, C.POINTER(C.c_void_p)]
        L.ref_weight_set_rows.argtypes = [P, C.c_int64]
        L.ref_weight_data.argtypes = [P]
        L.ref_weight_data.restype = P
        L.ref_weight_destroy.argtypes = [P]
        L.ref_matmul.argtypes = [P, P, P, S, P]
        L.ref_rms_norm.argtypes = [P, P, P, S, S, C.c_float]
        L.ref_rope.argtypes = [P, S, S, S, S, C.c_float]
        L.ref_attention.argtypes = [P, P, P, P, S, S, S, S, S]
        L.ref_residual_add.argtypes = [P, P, S]
        L.ref_silu_multiply.argtypes = [P, P, P, S]
        L.ref_dequantize_embeddings.argtypes = [P, P, S, S, S, C.c_int]
        L.ref_argmax.argtypes = [P, S, C.POINTER(C.c_uint32)]
        L.ref_forward.argtypes = [P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float,
                                  C.c_float, P, S, P, P, S, P, S, S, C.c_int, P, P, C.POINTER(C.c_uint32)]
        L.ref_layer.argtypes = [P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float, C.c_float, P, P, P, S, S,
                                S, C.c_int]
        _ref = L
    return _ref


def ref_check(rc: int) -> None:
    if rc:
        raise RuntimeError(f"reference call failed ({rc}): {ref().ref_last_error().decode()}")


def ref_layer(handles: dict, cfg: dict, layer: int, x_dev: int, k_dev: int, v_dev: int, capacity: int,
              tokens: int, offset: int, kv_round_f16: bool = True) -> None:
    """One block of Engine::inference with the reference kernels (ref_layer
    in ref_shim/ref_harness.cu): x_dev [tokens][hidden] updated in place,
    k_dev / v_dev this layer's fp32 caches [capacity][kv_heads*head_dim];
    all device addresses. `handles` maps tensor names to RefWeight."""
    ws = (C.c_void_p * SLOTS)(*[handles[f"blk.{layer}.{s}.weight"].h.value for s in SLOT_NAMES])
    ref_check(ref().ref_layer(ws, cfg["hidden"], cfg["heads"], cfg["kv_heads"], cfg["head_dim"], cfg["ffn"],
                              cfg["eps"], cfg["rope_base"], x_dev, k_dev, v_dev, capacity, tokens, offset,
                              int(kv_round_f16)))


class RefWeight:
    """A reference `Weight` (src/Weight.cpp:53-61) built from GGUF-layout bytes."""

    def __init__(self, name: str, qtype: int, ne0: int, ne1: int, data: np.ndarray):
        data = np.ascontiguousarray(data)
        h = C.c_void_p()
        ref_check(ref().ref_weight_create(name.encode(), qtype, ne0, ne1, _p(data), data.nbytes, C.byref(h)))
        self.h = h

    def set_rows(self, n: int) -> None:
        ref_check(ref().ref_weight_set_rows(self.h, n))

    @property
    def data_ptr(self) -> int:
        return ref().ref_weight_data(self.h)

    def __del__(self):
        if getattr(self, "h", None) and _ref is not None:
            _ref.ref_weight_destroy(self.h)
            self.h = None
