"""GGUF reader (include/q4k_b200.h q4k_gguf_*; host code, no GPU): files
written by the ggml project's own `gguf` Python package (0.19.0) are read
back with the same metadata, tensor directory and bytes, the engine
configuration comes out of the metadata the reference reads
(src/Engine.cpp:49-55), and malformed files are rejected rather than read
out of bounds."""
import ctypes as C

import numpy as np
import pytest

import q4kb200 as q
from tiny_model import TINY, tiny_tensors

gguf = pytest.importorskip("gguf")


def write_model(path, tensors, c=TINY, arch="qwen3", extra_meta=True, drop=()):
    w = gguf.GGUFWriter(path, arch)
    if "block_count" not in drop:
        w.add_block_count(c["layers"])
    w.add_embedding_length(c["hidden"])
    w.add_head_count(c["heads"])
    w.add_head_count_kv(c["kv_heads"])
    w.add_key_length(c["head_dim"])
    w.add_feed_forward_length(c["ffn"])
    w.add_layer_norm_rms_eps(c["eps"])
    w.add_rope_freq_base(c["rope_base"])
    if extra_meta:
        # keys the engine does not read, of every container kind, to be skipped
        w.add_array("tokenizer.ggml.tokens", [f"tok{i}" for i in range(50)])
        w.add_array("tokenizer.ggml.scores", [float(i) for i in range(50)])
        w.add_uint64("test.u64", 1 << 40)
        w.add_int8("test.i8", -5)
        w.add_bool("test.flag", True)
        w.add_string("test.text", "gguf reader")
    for name, (t, a, b, d) in tensors.items():
        if t == q.F32:
            w.add_tensor(name, np.asarray(d, np.float32).reshape(b, a) if b > 1 else np.asarray(d, np.float32))
        else:
            qt = gguf.GGMLQuantizationType.Q4_K if t == q.Q4_K else gguf.GGMLQuantizationType.Q6_K
            w.add_tensor(name, np.asarray(d, np.uint8).reshape(b, -1), raw_dtype=qt)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


@pytest.fixture(scope="module")
def tiny_file(tmp_path_factory):
    tensors = tiny_tensors()
    path = str(tmp_path_factory.mktemp("gguf") / "tiny.gguf")
    write_model(path, tensors)
    return path, tensors


def test_reads_back_what_gguf_wrote(tiny_file):
    path, tensors = tiny_file
    f = q.Gguf(path)
    got = f.tensors()
    assert set(got) == set(tensors)
    for name, (t, a, b, d) in tensors.items():
        gt, ga, gb, addr = got[name]
        assert (gt, ga, gb) == (t, a, b), name
        raw = np.frombuffer(np.ascontiguousarray(d).tobytes(), np.uint8)
        assert C.string_at(addr, raw.size) == raw.tobytes(), name
    assert f.meta_string("general.architecture") == "qwen3"
    assert f.meta_int("qwen3.block_count") == TINY["layers"]
    assert f.meta_int("test.u64") == 1 << 40
    assert f.meta_int("test.i8") == -5
    assert f.meta_float("qwen3.rope.freq_base") == pytest.approx(1e6)
    assert f.meta_string("test.text") == "gguf reader"
    with pytest.raises(q.OutOfRange):
        f.meta_int("no.such.key")
    with pytest.raises(q.OutOfRange):
        f.meta_int("test.text")  # a string, not an integer
    f.close()


def test_engine_config_from_metadata(tiny_file):
    path, _ = tiny_file
    cfg = q.Gguf(path).engine_config(64)
    for k in ("layers", "hidden", "heads", "kv_heads", "head_dim", "ffn", "vocab"):
        assert getattr(cfg, k) == TINY[k], k
    assert cfg.eps == pytest.approx(TINY["eps"]) and cfg.rope_base == pytest.approx(TINY["rope_base"])
    assert (cfg.capacity, cfg.tp_rank, cfg.tp_world) == (64, 0, 1)


def test_missing_metadata_is_an_error(tmp_path):
    path = str(tmp_path / "nolayers.gguf")
    write_model(path, tiny_tensors(), drop=("block_count",))
    with pytest.raises(q.InvalidArgument, match="block_count"):
        q.Gguf(path).engine_config(16)


def test_malformed_files_are_rejected(tiny_file, tmp_path):
    path, _ = tiny_file
    blob = open(path, "rb").read()
    cases = {
        "empty": b"",
        "magic": b"GGUX" + blob[4:],
        "version": blob[:4] + (7).to_bytes(4, "little") + blob[8:],
        "header_only": blob[:40],
        "truncated_metadata": blob[: len(blob) // 50],
        "truncated_data": blob[: len(blob) - 1000],
        "huge_count": blob[:8] + (1 << 40).to_bytes(8, "little") + blob[16:],
    }
    for tag, data in cases.items():
        p = tmp_path / f"{tag}.gguf"
        p.write_bytes(data)
        with pytest.raises(q.InvalidArgument):
            q.Gguf(str(p))
    with pytest.raises(q.InvalidArgument):
        q.Gguf(str(tmp_path / "does_not_exist.gguf"))
