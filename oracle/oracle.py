"""CPU oracle for the torch2vk quantized hot path (TEST INFRASTRUCTURE ONLY).

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` leg of
``bench.py`` import this module, and only as the checker.  The product
package ``torch2vk_b200`` never imports it.

It wraps the plain-C restatement in ``gguf_quant_ref.c`` (quantizers and
decoders of the reference's GGUF Q8_0 / Q4_K / Q6_K blocks) through ctypes and
adds vectorised numpy decoders for large matrices.  Citations (paths inside
the torch2vk project):

* quantizers: ``src/torch2vk/quantize/vulkan.py:91-637``
* decoders:   ``src/models/quantized_qwen3/shaders/embedding_q4_k_f32.py:96-110``,
  ``linear_nobias_q6_k_matvec_f32.py:116-156``, ``linear_nobias_q8_0_matvec_f32.py:84-95``
* Q4_K_M topology: ``src/torch2vk/quantize/gguf.py:54-161``

Pins: gguf-py 0.19.0 dequantizers (bit-exact), the reference GGUF reader, and
the committed golden fixtures under ``tests/golden``.  The Q4_K/Q6_K scale
search is "parity unpinned" beyond those (no runnable reference quantizer).
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
LIB_PATH = ORACLE_DIR / "_build" / "libt2c_oracle.so"

BLOCK = {"q4_k": (256, 144), "q6_k": (256, 210), "q8_0": (32, 34)}
_TYPE_ID = {"q4_k": 0, "q6_k": 1, "q8_0": 2}

_lib: ctypes.CDLL | None = None


def build() -> Path:
    """Compile the C restatement (make in oracle/)."""
    subprocess.run(["make", "-C", str(ORACLE_DIR)], check=True, capture_output=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        handle = ctypes.CDLL(str(LIB_PATH))
        f32p = ctypes.POINTER(ctypes.c_float)
        u8p = ctypes.POINTER(ctypes.c_uint8)
        u16p = ctypes.POINTER(ctypes.c_uint16)
        i64 = ctypes.c_int64
        for kind in ("q8_0", "q4_k", "q6_k"):
            q = getattr(handle, f"t2c_oracle_quantize_{kind}")
            q.argtypes = [f32p, i64, i64, u8p]
            q.restype = ctypes.c_int
            d = getattr(handle, f"t2c_oracle_dequantize_{kind}")
            d.argtypes = [u8p, i64, i64, f32p]
            d.restype = ctypes.c_int
        handle.t2c_oracle_matvec.argtypes = [ctypes.c_int, u8p, u16p, i64, i64, i64, f32p, i64, i64]
        handle.t2c_oracle_matvec.restype = ctypes.c_int
        handle.t2c_oracle_f32_to_f16.argtypes = [ctypes.c_float]
        handle.t2c_oracle_f32_to_f16.restype = ctypes.c_uint16
        _lib = handle
    return _lib


def _ptr(array: np.ndarray, ctype):
    return array.ctypes.data_as(ctypes.POINTER(ctype))


def row_bytes(kind: str, k: int) -> int:
    block, nbytes = BLOCK[kind]
    if k % block:
        raise ValueError(f"{kind} needs K % {block} == 0, got {k}")
    return k // block * nbytes


def quantize(x: np.ndarray, kind: str, threads: int | None = None) -> np.ndarray:
    """fp32 [R, K] -> packed uint8 [R, row_bytes]; rows are split over threads."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if x.ndim != 2:
        raise ValueError(f"quantize expects rank 2, got {x.shape}")
    rows, k = x.shape
    out = np.empty((rows, row_bytes(kind, k)), dtype=np.uint8)
    fn = getattr(lib(), f"t2c_oracle_quantize_{kind}")
    threads = threads or min(os.cpu_count() or 1, max(1, rows // 64))

    def work(lo: int, hi: int) -> None:
        if hi > lo:
            rc = fn(_ptr(x[lo:hi], ctypes.c_float), hi - lo, k, _ptr(out[lo:hi], ctypes.c_uint8))
            if rc != 0:
                raise ValueError(f"oracle quantize {kind} failed rc={rc}")

    bounds = np.linspace(0, rows, threads + 1).astype(int)
    if threads == 1:
        work(0, rows)
    else:
        with ThreadPoolExecutor(threads) as pool:
            list(pool.map(lambda i: work(bounds[i], bounds[i + 1]), range(threads)))
    return out


def dequantize(packed: np.ndarray, kind: str, k: int) -> np.ndarray:
    """packed uint8 [R, row_bytes] -> fp32 [R, K] via the C restatement."""
    packed = np.ascontiguousarray(packed).view(np.uint8).reshape(packed.shape[0], -1)
    rows = packed.shape[0]
    if packed.shape[1] != row_bytes(kind, k):
        raise ValueError(f"{kind} row bytes {packed.shape[1]} != {row_bytes(kind, k)}")
    out = np.empty((rows, k), dtype=np.float32)
    rc = getattr(lib(), f"t2c_oracle_dequantize_{kind}")(_ptr(packed, ctypes.c_uint8), rows, k, _ptr(out, ctypes.c_float))
    if rc != 0:
        raise ValueError(f"oracle dequantize {kind} failed rc={rc}")
    return out


def dequantize_np(packed: np.ndarray, kind: str, k: int) -> np.ndarray:
    """Vectorised numpy decoder with the same fp32 evaluation order as the C one."""
    packed = np.ascontiguousarray(packed).view(np.uint8)
    rows = packed.shape[0]
    block, nbytes = BLOCK[kind]
    blocks = packed.reshape(rows * (k // block), nbytes)
    if kind == "q8_0":
        d = blocks[:, :2].copy().view(np.float16).astype(np.float32)
        q = blocks[:, 2:].view(np.int8).astype(np.float32)
        return (d * q).reshape(rows, k)
    if kind == "q4_k":
        d = blocks[:, 0:2].copy().view(np.float16).astype(np.float32)
        dmin = blocks[:, 2:4].copy().view(np.float16).astype(np.float32)
        s = blocks[:, 4:16].astype(np.uint32)
        sc = np.empty((blocks.shape[0], 8), dtype=np.uint32)
        mn = np.empty((blocks.shape[0], 8), dtype=np.uint32)
        sc[:, :4] = s[:, 0:4] & 63
        mn[:, :4] = s[:, 4:8] & 63
        sc[:, 4:] = (s[:, 8:12] & 15) | ((s[:, 0:4] >> 6) << 4)
        mn[:, 4:] = (s[:, 8:12] >> 4) | ((s[:, 4:8] >> 6) << 4)
        qb = blocks[:, 16:].reshape(-1, 4, 32)
        q = np.stack([qb & 15, qb >> 4], axis=2).reshape(-1, 8, 32).astype(np.float32)
        ds = (d * sc.astype(np.float32))[:, :, None]
        dm = (dmin * mn.astype(np.float32))[:, :, None]
        return (ds * q - dm).reshape(rows, k)
    if kind == "q6_k":
        d = blocks[:, 208:210].copy().view(np.float16).astype(np.float32)
        sc = blocks[:, 192:208].view(np.int8).astype(np.float32)
        ql = blocks[:, 0:128].reshape(-1, 2, 2, 32)  # [blk, s, c&1, l]
        qh = blocks[:, 128:192].reshape(-1, 2, 32)  # [blk, s, l]
        lo = np.stack([ql & 15, ql >> 4], axis=2)  # [blk, s, c>>1, c&1, l]
        lo = lo.reshape(-1, 2, 4, 32)  # c = 2*(c>>1) + (c&1)
        hi = np.stack([(qh >> (2 * c)) & 3 for c in range(4)], axis=2)  # [blk, s, c, l]
        level = (lo.astype(np.int32) | (hi.astype(np.int32) << 4)) - 32
        level = level.reshape(-1, 16, 16).astype(np.float32)
        return ((d * sc)[:, :, None] * level).reshape(rows, k)
    raise ValueError(kind)


def matvec(packed: np.ndarray, kind: str, x: np.ndarray, threads: int | None = None) -> np.ndarray:
    """Direct block matvec: fp16 x [M, K] times deq(W)^T -> fp32 [M, N] (double accumulate)."""
    x16 = np.ascontiguousarray(x, dtype=np.float16)
    m, k = x16.shape
    packed = np.ascontiguousarray(packed).view(np.uint8)
    n = packed.shape[0]
    y = np.empty((m, n), dtype=np.float32)
    threads = threads or (os.cpu_count() or 1)
    bounds = np.linspace(0, n, threads + 1).astype(int)
    fn = lib().t2c_oracle_matvec

    def work(i: int) -> None:
        rc = fn(_TYPE_ID[kind], _ptr(packed, ctypes.c_uint8), _ptr(x16.view(np.uint16), ctypes.c_uint16),
                m, n, k, _ptr(y, ctypes.c_float), int(bounds[i]), int(bounds[i + 1]))
        if rc != 0:
            raise ValueError(f"oracle matvec failed rc={rc}")

    with ThreadPoolExecutor(threads) as pool:
        list(pool.map(work, range(threads)))
    return y


def gguf_physical(packed: np.ndarray, kind: str) -> np.ndarray:
    """View packed bytes as the reference's physical tensor dtype (checkpoints/gguf.py:306-326)."""
    packed = np.ascontiguousarray(packed).view(np.uint8)
    return packed.view(np.uint32) if kind == "q4_k" else packed.view(np.uint16)


def q4_k_m_more_bits_layer_indices(num_layers: int) -> tuple[int, ...]:
    """Layers whose v_proj/down_proj are Q6_K under Q4_K_M (quantize/gguf.py:150-161)."""
    first = num_layers // 8
    last = (7 * num_layers) // 8
    return tuple(i for i in range(num_layers) if i < first or i >= last or (i - first) % 3 == 2)
