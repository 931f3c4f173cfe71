"""Generates the committed golden vectors under tests/golden/ (run from the repo root:
`python tests/golden/make_golden.py`).

For each GGUF block type (q8_0, q4_k, q6_k) one seeded fp32 weight matrix with
the edge rows the quantizers must handle (all-zero, constant, one-signed,
outliers, tiny values) is quantized by the C oracle (the restatement of
src/torch2vk/quantize/vulkan.py:91-637); the file stores the input, the
packed bytes, the dequantized floats, a seeded fp16 x and the double-precision
product.  Before writing, the packed bytes are decoded by gguf-py (the
llama.cpp reference decoders) and must equal the oracle's decode bit for bit,
and the Q8_0 bytes must equal gguf-py's Q8_0 quantizer.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from oracle import oracle  # noqa: E402

SHAPES = {"q8_0": (12, 256), "q4_k": (12, 512), "q6_k": (12, 512)}


def weights(kind: str) -> np.ndarray:
    n, k = SHAPES[kind]
    rng = np.random.default_rng({"q8_0": 101, "q4_k": 102, "q6_k": 103}[kind])
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    w[0] = 0.0
    w[1] = 0.013
    w[2, : k // 2] = -0.5
    w[3] = np.abs(w[3])
    w[4, ::7] = 3.0
    w[5] *= 1e-7
    w[6] = -np.abs(w[6])
    w[7, 5] = 40.0
    return w


def gguf_py_check(kind: str, packed: np.ndarray, deq: np.ndarray, w: np.ndarray) -> None:
    from gguf import GGMLQuantizationType as Q
    from gguf import quants

    qt = {"q8_0": Q.Q8_0, "q4_k": Q.Q4_K, "q6_k": Q.Q6_K}[kind]
    ref = quants.dequantize(packed, qt)
    assert np.array_equal(ref.view(np.uint32), deq.view(np.uint32)), f"{kind}: gguf-py decode differs"
    if kind == "q8_0":
        assert np.array_equal(quants.quantize(w, qt), packed), "q8_0: gguf-py quantize differs"


def main() -> None:
    oracle.build()
    for kind, (n, k) in SHAPES.items():
        w = weights(kind)
        packed = oracle.quantize(w, kind)
        deq = oracle.dequantize(packed, kind, k)
        gguf_py_check(kind, packed, deq, w)
        x = np.random.default_rng(7).standard_normal((3, k)).astype(np.float16)
        y = oracle.matvec(packed, kind, x)
        np.savez_compressed(HERE / f"{kind}.npz", w=w, packed=packed, deq=deq, x=x, y=y)
        print(kind, packed.shape, packed.nbytes)


if __name__ == "__main__":
    main()
