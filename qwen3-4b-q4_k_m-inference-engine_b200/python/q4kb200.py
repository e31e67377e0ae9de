"""Python bindings (ctypes) for libq4kb200.so — the C ABI in include/q4k_b200.h.

Device buffers are passed as torch CUDA tensors (their data_ptr) or raw
integer addresses; host buffers as numpy arrays. The library must have been
built (``make -C qwen3-4b-q4_k_m-inference-engine_b200`` or
``__graft_entry__.build()``); importing this module on a machine without the
built library raises, there is no fallback path.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG_DIR, "lib", "libq4kb200.so")

OK, EINVAL, ERANGE, ECUDA, ETIMEOUT = 0, 1, 2, 3, 4
F32, F16, Q4_K, Q6_K = 0, 1, 12, 14
EPI_STORE, EPI_ADD, EPI_SWIGLU, EPI_ARGMAX = 0, 1, 2, 3

# Every symbol the C ABI exports (checked by the CPU tests against the header).
EXPORTS = (
    "q4k_last_error", "q4k_abi_version", "q4k_weight_device_bytes", "q4k_weight_upload", "q4k_synth_tensor_host",
    "q4k_synth_tensor_device", "q4k_synth_f16_host", "q4k_synth_f32_host", "q4k_synth_f32_device", "q4k_rms_norm",
    "q4k_matmul", "q4k_rope", "q4k_attention", "q4k_residual_add", "q4k_silu_multiply", "q4k_dequantize_embeddings",
    "q4k_argmax", "q4k_matmul_ex", "q4k_matmul_batch", "q4k_matmul_argmax_scratch_bytes", "q4k_attention_decode_f16",
    "q4k_attention_decode_scratch_bytes", "q4k_engine_config_qwen3_4b", "q4k_model_tensor", "q4k_nccl_unique_id",
    "q4k_engine_create", "q4k_engine_destroy", "q4k_engine_load_synthetic", "q4k_engine_set_tensor",
    "q4k_engine_fill_kv_synthetic", "q4k_engine_read_kv", "q4k_engine_decode", "q4k_engine_prefill", "q4k_engine_prefill_seq", "q4k_engine_decode_batch", "q4k_engine_generate",
    "q4k_engine_stream", "q4k_tp_shard", "q4k_engine_layer", "q4k_engine_write_kv",
    "q4k_engine_trace", "q4k_attention_decode_f16_static", "q4k_gguf_open", "q4k_gguf_close",
    "q4k_gguf_tensor_count", "q4k_gguf_tensor_info", "q4k_gguf_meta_int", "q4k_gguf_meta_float",
    "q4k_gguf_meta_string", "q4k_gguf_engine_config", "q4k_engine_load_gguf", "q4k_engine_layer_rows",
    "q4k_engine_layer_batch",
    "q4k_engine_set_limits",
    "q4k_engine_abort",
    "q4k_tp_sum_parts",
)


class Q4KError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"[{status}] {message}")
        self.status = status


class InvalidArgument(Q4KError, ValueError):
    pass


class OutOfRange(Q4KError, IndexError):
    pass


class Timeout(Q4KError, TimeoutError):
    """A bounded wait gave up (Q4K_ETIMEOUT): another rank's partial sums
    never arrived, a tensor-parallel step overran the host limit, or the
    engine was aborted."""


class EngineConfig(C.Structure):
    _fields_ = [("layers", C.c_int), ("hidden", C.c_int), ("heads", C.c_int), ("kv_heads", C.c_int),
                ("head_dim", C.c_int), ("ffn", C.c_int), ("vocab", C.c_int), ("eps", C.c_float),
                ("rope_base", C.c_float), ("capacity", C.c_int), ("tp_rank", C.c_int), ("tp_world", C.c_int),
                ("device", C.c_int), ("sequences", C.c_int)]

    def as_dict(self) -> dict:
        return {f: getattr(self, f) for f, _ in self._fields_}


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build the CUDA library first (make -C {PKG_DIR})")
        L = C.CDLL(LIB_PATH)
        P, S, I, I64, U64 = C.c_void_p, C.c_size_t, C.c_int, C.c_int64, C.c_uint64
        sig = {
            "q4k_last_error": ([], C.c_char_p),
            "q4k_abi_version": ([], I),
            "q4k_weight_device_bytes": ([I, I64, I64], S),
            "q4k_weight_upload": ([I, I64, I64, P, P, P], I),
            "q4k_synth_tensor_host": ([U64, C.c_char_p, I, I64, I64, P], I),
            "q4k_synth_tensor_device": ([U64, C.c_char_p, I, I64, I64, P, P], I),
            "q4k_synth_f16_host": ([U64, C.c_char_p, U64, S, P], I),
            "q4k_synth_f32_host": ([U64, C.c_char_p, S, P], I),
            "q4k_synth_f32_device": ([U64, C.c_char_p, S, P, P], I),
            "q4k_rms_norm": ([P, P, P, S, S, C.c_float, P], I),
            "q4k_matmul": ([P, P, I, I64, I64, P, S, P], I),
            "q4k_rope": ([P, S, S, S, S, C.c_float, P], I),
            "q4k_attention": ([P, P, P, P, S, S, S, S, S, P], I),
            "q4k_residual_add": ([P, P, S, P], I),
            "q4k_silu_multiply": ([P, P, P, S, P], I),
            "q4k_dequantize_embeddings": ([P, P, S, S, S, I, P], I),
            "q4k_argmax": ([P, S, C.POINTER(C.c_uint32), P], I),
            "q4k_matmul_ex": ([P, P, C.c_float, I, P, P, P, P, I64, S, I, P, P, P], I),
            "q4k_matmul_argmax_scratch_bytes": ([], S),
            "q4k_matmul_batch": ([P, P, C.c_float, I, P, P, P, P, I64, I64, S, I, P], I),
            "q4k_attention_decode_f16": ([P, P, P, P, P, I, P, I, I, I, C.c_float, C.c_float, P, P, P], I),
            "q4k_attention_decode_f16_static": ([P, P, P, P, P, I, P, I, I, I, C.c_float, C.c_float, P, P], I),
            "q4k_attention_decode_scratch_bytes": ([I, I], S),
            "q4k_engine_config_qwen3_4b": ([C.POINTER(EngineConfig), I], None),
            "q4k_model_tensor": ([C.POINTER(EngineConfig), I, C.c_char_p, S, C.POINTER(I), C.POINTER(I64),
                                  C.POINTER(I64)], I),
            "q4k_nccl_unique_id": ([P], I),
            "q4k_engine_create": ([C.POINTER(EngineConfig), P, C.POINTER(P)], I),
            "q4k_engine_destroy": ([P], I),
            "q4k_engine_load_synthetic": ([P, U64], I),
            "q4k_engine_set_tensor": ([P, C.c_char_p, I, I64, I64, P], I),
            "q4k_engine_fill_kv_synthetic": ([P, U64, I], I),
            "q4k_engine_read_kv": ([P, I, P, P], I),
            "q4k_engine_decode": ([P, C.c_uint32, I, C.POINTER(C.c_uint32), P, P], I),
            "q4k_engine_prefill": ([P, P, I, I, C.POINTER(C.c_uint32), P], I),
            "q4k_engine_prefill_seq": ([P, I, P, I, I, C.POINTER(C.c_uint32), P], I),
            "q4k_engine_decode_batch": ([P, I, P, P, P, P, P], I),
            "q4k_engine_generate": ([P, C.c_uint32, I, I, I, P], I),
            "q4k_engine_stream": ([P], P),
            "q4k_engine_set_limits": ([P, U64, I], I),
            "q4k_engine_abort": ([P], I),
            "q4k_tp_sum_parts": ([P, I, I64, C.c_uint32, P, P, U64, P, P], I),
            "q4k_engine_layer": ([P, I, P, I, P], I),
            "q4k_engine_layer_rows": ([P, I, I, I, I, P, P], I),
            "q4k_engine_layer_batch": ([P, I, I, P, P, P, P], I),
            "q4k_engine_write_kv": ([P, I, P, P], I),
            "q4k_engine_trace": ([P, C.c_uint32, I, P, C.c_size_t, C.POINTER(C.c_size_t)], I),
            "q4k_tp_shard": ([C.POINTER(EngineConfig), I, I, I, C.POINTER(I64), C.POINTER(I64), C.POINTER(I64),
                              C.POINTER(I64)], I),
            "q4k_gguf_open": ([C.c_char_p, C.POINTER(P)], I),
            "q4k_gguf_close": ([P], I),
            "q4k_gguf_tensor_count": ([P, C.POINTER(I64)], I),
            "q4k_gguf_tensor_info": ([P, I64, C.c_char_p, S, C.POINTER(I), C.POINTER(I64), C.POINTER(I64),
                                      C.POINTER(P)], I),
            "q4k_gguf_meta_int": ([P, C.c_char_p, C.POINTER(I64)], I),
            "q4k_gguf_meta_float": ([P, C.c_char_p, C.POINTER(C.c_double)], I),
            "q4k_gguf_meta_string": ([P, C.c_char_p, C.c_char_p, S], I),
            "q4k_gguf_engine_config": ([P, I, C.POINTER(EngineConfig)], I),
            "q4k_engine_load_gguf": ([P, P], I),
        }
        for name, (args, res) in sig.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def check(status: int) -> None:
    if status == OK:
        return
    msg = lib().q4k_last_error().decode()
    if status == EINVAL:
        raise InvalidArgument(status, msg)
    if status == ERANGE:
        raise OutOfRange(status, msg)
    if status == ETIMEOUT:
        raise Timeout(status, msg)
    raise Q4KError(status, msg)


def ptr(t) -> int | None:
    """Device address of a torch tensor (or int / None passthrough)."""
    if t is None:
        return None
    if isinstance(t, int):
        return t
    return t.data_ptr()


def hptr(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


def stream_ptr(stream) -> int | None:
    if stream is None:
        return None
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


# ------------------------------------------------------------------ helpers
def gguf_row_bytes(qtype: int, K: int) -> int:
    nb = K // 256
    return {Q4_K: nb * 144, Q6_K: nb * 210, F32: K * 4, F16: K * 2}[qtype]


def device_bytes(qtype: int, ne0: int, ne1: int) -> int:
    return int(lib().q4k_weight_device_bytes(qtype, ne0, ne1))


def synth_tensor_host(seed: int, name: str, qtype: int, ne0: int, ne1: int) -> np.ndarray:
    """GGUF-layout bytes (uint8) or float32 values of a synthetic tensor."""
    if qtype == F32:
        out = np.empty(ne0 * ne1, np.float32)
    else:
        out = np.empty(ne1 * gguf_row_bytes(qtype, ne0), np.uint8)
    check(lib().q4k_synth_tensor_host(seed, name.encode(), qtype, ne0, ne1, hptr(out)))
    return out


def synth_f16_host(seed: int, name: str, index_base: int, n: int) -> np.ndarray:
    out = np.empty(n, np.uint16)
    check(lib().q4k_synth_f16_host(seed, name.encode(), index_base, n, hptr(out)))
    return out


def synth_f32_host(seed: int, name: str, n: int) -> np.ndarray:
    out = np.empty(n, np.float32)
    check(lib().q4k_synth_f32_host(seed, name.encode(), n, hptr(out)))
    return out


def qwen3_4b_config(capacity: int = 4096) -> EngineConfig:
    cfg = EngineConfig()
    lib().q4k_engine_config_qwen3_4b(C.byref(cfg), capacity)
    return cfg


def model_tensors(cfg: EngineConfig):
    """[(name, type, ne0, ne1)] of the synthetic Q4_K_M model."""
    out = []
    i = 0
    buf = C.create_string_buffer(96)
    while True:
        t, a, b = C.c_int(), C.c_int64(), C.c_int64()
        st = lib().q4k_model_tensor(C.byref(cfg), i, buf, 96, C.byref(t), C.byref(a), C.byref(b))
        if st == ERANGE:
            break
        check(st)
        out.append((buf.value.decode(), t.value, a.value, b.value))
        i += 1
    return out


def tp_shard(cfg: EngineConfig, i: int, rank: int, world: int):
    """(n0, n1, b0, b1): rows and super-blocks of tensor i held by `rank`."""
    v = [C.c_int64() for _ in range(4)]
    check(lib().q4k_tp_shard(C.byref(cfg), i, rank, world, *[C.byref(x) for x in v]))
    return tuple(x.value for x in v)


class Gguf:
    """A GGUF model file mapped read-only (q4k_gguf_* in include/q4k_b200.h)."""

    def __init__(self, path: str):
        h = C.c_void_p()
        check(lib().q4k_gguf_open(path.encode(), C.byref(h)))
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            check(lib().q4k_gguf_close(self.h))
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def tensors(self) -> dict:
        """name -> (ggml type, ne0, ne1, address of the bytes in the mapping)."""
        n = C.c_int64()
        check(lib().q4k_gguf_tensor_count(self.h, C.byref(n)))
        out = {}
        for i in range(n.value):
            buf = C.create_string_buffer(256)
            t, a, b, d = C.c_int(), C.c_int64(), C.c_int64(), C.c_void_p()
            check(lib().q4k_gguf_tensor_info(self.h, i, buf, 256, C.byref(t), C.byref(a), C.byref(b), C.byref(d)))
            out[buf.value.decode()] = (t.value, a.value, b.value, d.value)
        return out

    def meta_int(self, key: str) -> int:
        v = C.c_int64()
        check(lib().q4k_gguf_meta_int(self.h, key.encode(), C.byref(v)))
        return v.value

    def meta_float(self, key: str) -> float:
        v = C.c_double()
        check(lib().q4k_gguf_meta_float(self.h, key.encode(), C.byref(v)))
        return v.value

    def meta_string(self, key: str) -> str:
        buf = C.create_string_buffer(4096)
        check(lib().q4k_gguf_meta_string(self.h, key.encode(), buf, 4096))
        return buf.value.decode()

    def engine_config(self, capacity: int) -> EngineConfig:
        cfg = EngineConfig()
        check(lib().q4k_gguf_engine_config(self.h, capacity, C.byref(cfg)))
        return cfg


class Engine:
    """Decode engine (q4k_engine_*)."""

    def __init__(self, cfg: EngineConfig, nccl_id: bytes | None = None):
        self.cfg = cfg
        h = C.c_void_p()
        idbuf = C.create_string_buffer(nccl_id, 128) if nccl_id is not None else None
        check(lib().q4k_engine_create(C.byref(cfg), idbuf, C.byref(h)))
        self.h = h

    def close(self):
        if getattr(self, "h", None):
            check(lib().q4k_engine_destroy(self.h))
            self.h = None

    def load_gguf(self, f: "Gguf"):
        check(lib().q4k_engine_load_gguf(self.h, f.h))

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def load_synthetic(self, seed: int):
        check(lib().q4k_engine_load_synthetic(self.h, seed))

    def set_tensor(self, name: str, qtype: int, ne0: int, ne1: int, data: np.ndarray):
        data = np.ascontiguousarray(data)
        check(lib().q4k_engine_set_tensor(self.h, name.encode(), qtype, ne0, ne1, hptr(data)))

    def fill_kv_synthetic(self, seed: int, n: int):
        check(lib().q4k_engine_fill_kv_synthetic(self.h, seed, n))

    def read_kv(self, layer: int):
        c = self.cfg
        n = (c.kv_heads // max(c.tp_world, 1)) * c.capacity * c.head_dim
        k = np.empty(n, np.uint16)
        v = np.empty(n, np.uint16)
        check(lib().q4k_engine_read_kv(self.h, layer, hptr(k), hptr(v)))
        return k, v

    def write_kv(self, layer: int, k: np.ndarray | None, v: np.ndarray | None):
        k = None if k is None else np.ascontiguousarray(k, np.uint16)
        v = None if v is None else np.ascontiguousarray(v, np.uint16)
        check(lib().q4k_engine_write_kv(self.h, layer, hptr(k), hptr(v)))

    def _vocab_rows(self) -> int:
        """Logits this rank holds: its shard of the vocabulary (all of it
        with one GPU)."""
        c = self.cfg
        world = max(c.tp_world, 1)
        return c.vocab * (c.tp_rank + 1) // world - c.vocab * c.tp_rank // world

    def decode(self, token: int, position: int, want_logits=False, want_hidden=False):
        c = self.cfg
        world = max(c.tp_world, 1)
        v0 = c.vocab * c.tp_rank // world
        v1 = c.vocab * (c.tp_rank + 1) // world
        logits = np.empty(v1 - v0, np.float32) if want_logits else None
        hidden = np.empty((c.layers + 1, c.hidden), np.float32) if want_hidden else None
        nxt = C.c_uint32()
        check(lib().q4k_engine_decode(self.h, token, position, C.byref(nxt), hptr(logits), hptr(hidden)))
        return nxt.value, logits, hidden

    def prefill(self, tokens, position: int = 0, want_logits=False):
        """A whole prompt at positions position .. position+len(tokens)-1
        (q4k_engine_prefill): returns (next token, logits of the last row)."""
        c = self.cfg
        world = max(c.tp_world, 1)
        v0 = c.vocab * c.tp_rank // world
        v1 = c.vocab * (c.tp_rank + 1) // world
        toks = np.ascontiguousarray(tokens, np.uint32)
        logits = np.empty(v1 - v0, np.float32) if want_logits else None
        nxt = C.c_uint32()
        check(lib().q4k_engine_prefill(self.h, hptr(toks), int(toks.size), position, C.byref(nxt), hptr(logits)))
        return nxt.value, logits

    def prefill_seq(self, seq: int, tokens, position: int = 0, want_logits=False):
        """q4k_engine_prefill into sequence `seq`."""
        toks = np.ascontiguousarray(tokens, np.uint32)
        logits = np.empty(self._vocab_rows(), np.float32) if want_logits else None
        nxt = C.c_uint32()
        check(lib().q4k_engine_prefill_seq(self.h, seq, hptr(toks), int(toks.size), position, C.byref(nxt),
                                           hptr(logits)))
        return nxt.value, logits

    def decode_batch(self, seqs, tokens, positions, want_logits=False):
        """One step for len(seqs) sequences (q4k_engine_decode_batch):
        returns (next tokens, logits [n][vocab] or None)."""
        sq = np.ascontiguousarray(seqs, np.int32)
        tk = np.ascontiguousarray(tokens, np.uint32)
        ps = np.ascontiguousarray(positions, np.int32)
        n = int(sq.size)
        assert tk.size == n and ps.size == n
        out = np.empty(n, np.uint32)
        logits = np.empty((n, self._vocab_rows()), np.float32) if want_logits else None
        check(lib().q4k_engine_decode_batch(self.h, n, hptr(sq), hptr(tk), hptr(ps), hptr(out), hptr(logits)))
        return out, logits

    def generate(self, token: int, position: int, steps: int, advance: bool = True, want_tokens=True):
        out = np.empty(max(steps, 1), np.uint32) if want_tokens else None
        check(lib().q4k_engine_generate(self.h, token, position, steps, int(advance), hptr(out)))
        return out[:steps] if want_tokens else None

    def layer(self, layer: int, x: np.ndarray, position: int) -> np.ndarray:
        """One block applied to residual stream x (q4k_engine_layer)."""
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty_like(x)
        check(lib().q4k_engine_layer(self.h, layer, hptr(x), position, hptr(out)))
        return out

    def layer_rows(self, layer: int, x: np.ndarray, position: int, seq: int = 0) -> np.ndarray:
        """One block of a prompt pass over rows x [n][hidden] at positions
        position .. position+n-1 of sequence seq (q4k_engine_layer_rows)."""
        x = np.ascontiguousarray(x, np.float32)
        n = x.size // self.cfg.hidden
        out = np.empty_like(x)
        check(lib().q4k_engine_layer_rows(self.h, layer, seq, n, position, hptr(x), hptr(out)))
        return out

    def layer_batch(self, layer: int, x: np.ndarray, seqs, positions) -> np.ndarray:
        """One block of a batched decode step: row i at positions[i] of
        sequence seqs[i] (q4k_engine_layer_batch)."""
        x = np.ascontiguousarray(x, np.float32)
        seqs = np.ascontiguousarray(seqs, np.int32)
        positions = np.ascontiguousarray(positions, np.int32)
        out = np.empty_like(x)
        check(lib().q4k_engine_layer_batch(self.h, layer, seqs.size, hptr(seqs), hptr(positions), hptr(x),
                                           hptr(out)))
        return out

    @property
    def stream(self) -> int:
        return lib().q4k_engine_stream(self.h)

    def set_limits(self, device_wait_ns: int = 0, host_wait_ms: int = 0):
        """Bound the in-kernel waits for other ranks' partial sums
        (device_wait_ns; 0 keeps the current 2 s) and how long a synchronous
        call waits for a tensor-parallel step (host_wait_ms; 0: unbounded).
        Either running out raises Timeout."""
        check(lib().q4k_engine_set_limits(self.h, device_wait_ns, host_wait_ms))

    def abort(self):
        """Abort the engine's communicator (safe from another thread): a call
        waiting on a step raises Timeout, and so does every later call."""
        check(lib().q4k_engine_abort(self.h))

    def trace(self, token: int, position: int) -> np.ndarray:
        """One traced decode step: [256 launches][1024 CTAs][8 slots] of
        %globaltimer ns (0 = not recorded)."""
        rec = np.zeros((256, 1024, 8), np.uint64)
        n = C.c_size_t(0)
        check(lib().q4k_engine_trace(self.h, token, position, hptr(rec), rec.size, C.byref(n)))
        return rec


def nccl_unique_id() -> bytes:
    buf = C.create_string_buffer(128)
    check(lib().q4k_nccl_unique_id(buf))
    return buf.raw


class PeerLost(RuntimeError):
    """Another tensor-parallel rank left or stopped beating (PeerWatch)."""


class PeerWatch:
    """Host-side liveness of the tensor-parallel ranks over a key-value store
    (a torch.distributed Store: TCPStore, FileStore, ...). No counterpart in
    the reference, which runs on one GPU.

    Every rank calls beat() before it launches a step and check() before its
    next launch: check() raises PeerLost when another rank said it left
    (leave(), called between steps) or when its beat has not changed for
    `timeout_s` seconds of this process's monotonic clock (a rank that
    crashed or hangs). With `engine` given, a lost peer also aborts that
    engine's communicator, so that a call still waiting on a collective
    returns (Timeout) instead of blocking for good. Beats are step counters,
    not wall-clock times, so ranks on different hosts need no common clock."""

    def __init__(self, store, rank: int, world: int, timeout_s: float = 10.0, engine=None, prefix: str = "q4k/peer"):
        import time

        self._time = time.monotonic
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s, self.engine, self.prefix = timeout_s, engine, prefix
        self.step = 0
        now = self._time()
        self._seen = {r: (None, now) for r in range(world) if r != rank}
        self.store.set(self._key(rank), "0")

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def beat(self):
        self.step += 1
        self.store.set(self._key(self.rank), str(self.step))

    def leave(self):
        self.store.set(self._key(self.rank), "left")

    def _lost(self, why: str):
        if self.engine is not None:
            try:
                self.engine.abort()
            except Exception:  # noqa: BLE001 - the peer is gone either way
                pass
        raise PeerLost(why)

    def check(self):
        now = self._time()
        for r, (last, since) in list(self._seen.items()):
            key = self._key(r)
            value = self.store.get(key).decode() if self.store.check([key]) else None
            if value == "left":
                self._lost(f"rank {r} left")
            if value != last:
                self._seen[r] = (value, now)
            elif now - since > self.timeout_s:
                self._lost(f"rank {r} has not beaten for {now - since:.1f} s (last beat {last})")
