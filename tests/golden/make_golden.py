"""Generates tests/golden/dequant_gguf.npz: Q4_K / Q6_K super-blocks and
their fp32 dequantisation by the `gguf` Python package (0.19.0, the ggml
project's own restatement of `ggml_get_type_traits(type)->to_float`, which the
reference's tests use as their CPU oracle: src/tests/reference/
MatmulReference.hpp:47,54 and src/tests/EmbedLookupTests.cpp:26,45).

Blocks: seeded synthetic rows from this library's generator plus hand-built
edge cases (zero scales, all-max fields, fp16 subnormal and large d/dmin,
negative d). Run in a container that has the `gguf` package:

    python tests/golden/make_golden.py
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "qwen3-4b-q4_k_m-inference-engine_b200", "python"))

import gguf  # noqa: E402
from gguf import quants  # noqa: E402

import q4kb200 as q  # noqa: E402


def edge_blocks_q4k() -> np.ndarray:
    blocks = []
    rng = np.random.default_rng(7)
    for d, dmin in [(0x0000, 0x0000), (0x3C00, 0x3C00), (0x0001, 0x03FF), (0x7BFF, 0x7BFF), (0xBC00, 0x3800),
                    (0x1400, 0x0C00)]:
        for fill in ("zero", "max", "rand"):
            b = np.zeros(144, np.uint8)
            b[0:2] = np.frombuffer(np.uint16(d).tobytes(), np.uint8)
            b[2:4] = np.frombuffer(np.uint16(dmin).tobytes(), np.uint8)
            if fill == "max":
                b[4:] = 0xFF
            elif fill == "rand":
                b[4:] = rng.integers(0, 256, 140, dtype=np.uint8)
            blocks.append(b)
    return np.stack(blocks)


def edge_blocks_q6k() -> np.ndarray:
    blocks = []
    rng = np.random.default_rng(8)
    for d in (0x0000, 0x3C00, 0x0001, 0x7BFF, 0xBC00):
        for fill in ("zero", "max", "min", "rand"):
            b = np.zeros(210, np.uint8)
            if fill == "max":
                b[:192] = 0xFF
                b[192:208] = 127
            elif fill == "min":
                b[192:208] = np.uint8(0x80)  # int8 -128
            elif fill == "rand":
                b[:208] = rng.integers(0, 256, 208, dtype=np.uint8)
            b[208:210] = np.frombuffer(np.uint16(d).tobytes(), np.uint8)
            blocks.append(b)
    return np.stack(blocks)


def main() -> None:
    out = {}
    for tag, qt, gq, edges in (("q4k", q.Q4_K, gguf.GGMLQuantizationType.Q4_K, edge_blocks_q4k()),
                               ("q6k", q.Q6_K, gguf.GGMLQuantizationType.Q6_K, edge_blocks_q6k())):
        synth = q.synth_tensor_host(0x5EED, f"golden.{tag}", qt, 2560, 4).reshape(4, -1)
        bsize = 144 if qt == q.Q4_K else 210
        blocks = np.concatenate([synth.reshape(-1, bsize), edges], axis=0)
        deq = quants.dequantize(blocks, gq).astype(np.float32).reshape(blocks.shape[0], 256)
        out[f"{tag}_blocks"] = blocks
        out[f"{tag}_values"] = deq
    np.savez_compressed(os.path.join(HERE, "dequant_gguf.npz"), **out)
    print({k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
