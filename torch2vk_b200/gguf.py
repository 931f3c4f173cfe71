"""GGUF v3 files: read (mmap, physical tensor views) and write Q4_K_M-quantized checkpoints.

Format rules followed (so that the reference reader torch2vk.checkpoints.gguf
parses these files and the reference writer's files load here):
  * header: magic "GGUF", version 3, tensor count, metadata count (u64);
  * metadata key/value pairs; general.alignment (default 32) aligns the data;
  * tensor infos: name, n_dims, dims in reversed (fastest-first) order, ggml
    type, data offset relative to the aligned data section;
  * physical views (src/torch2vk/checkpoints/gguf.py:265-326): Q4_K rows as
    uint32 [N, K/256*36], Q6_K as uint16 [N, K/256*105], Q8_0 as uint16
    [N, K/32*17], F16 / F32 as their logical shape.
The Q4_K_M type topology is src/torch2vk/quantize/gguf.py:54-161; quantization
runs on the GPU with this repo's bit-exact quantizer kernels.
"""

from __future__ import annotations

import mmap
import struct
from dataclasses import dataclass
from enum import IntEnum
from pathlib import Path
from typing import BinaryIO

import numpy as np

GGUF_MAGIC = 0x46554747
GGUF_VERSION = 3
DEFAULT_ALIGNMENT = 32
FILE_TYPE_MOSTLY_Q4_K_M = 15


class GGMLType(IntEnum):
    F32 = 0
    F16 = 1
    Q8_0 = 8
    Q4_K = 12
    Q6_K = 14
    I32 = 26
    I64 = 27
    BF16 = 30


class ValueType(IntEnum):
    UINT8 = 0
    INT8 = 1
    UINT16 = 2
    INT16 = 3
    UINT32 = 4
    INT32 = 5
    FLOAT32 = 6
    BOOL = 7
    STRING = 8
    ARRAY = 9
    UINT64 = 10
    INT64 = 11
    FLOAT64 = 12


# type -> (values per block, bytes per block, physical numpy dtype, physical words per block)
_BLOCKS = {
    GGMLType.Q4_K: (256, 144, np.uint32, 36),
    GGMLType.Q6_K: (256, 210, np.uint16, 105),
    GGMLType.Q8_0: (32, 34, np.uint16, 17),
}
_PLAIN = {GGMLType.F32: np.float32, GGMLType.F16: np.float16, GGMLType.BF16: np.uint16, GGMLType.I32: np.int32,
          GGMLType.I64: np.int64}
KIND_TO_TYPE = {"q4_k": GGMLType.Q4_K, "q6_k": GGMLType.Q6_K, "q8_0": GGMLType.Q8_0}
TYPE_TO_KIND = {v: k for k, v in KIND_TO_TYPE.items()}

_SCALAR = {ValueType.UINT8: "<B", ValueType.INT8: "<b", ValueType.UINT16: "<H", ValueType.INT16: "<h",
           ValueType.UINT32: "<I", ValueType.INT32: "<i", ValueType.FLOAT32: "<f", ValueType.BOOL: "<?",
           ValueType.UINT64: "<Q", ValueType.INT64: "<q", ValueType.FLOAT64: "<d"}


@dataclass(frozen=True)
class TensorEntry:
    name: str
    ggml_type: GGMLType
    logical_shape: tuple[int, ...]
    offset: int   # absolute file offset
    nbytes: int

    @property
    def physical(self) -> tuple[np.dtype, tuple[int, ...]]:
        if self.ggml_type in _BLOCKS:
            values, nbytes, dtype, words = _BLOCKS[self.ggml_type]
            rows = 1
            for d in self.logical_shape[:-1]:
                rows *= d
            return np.dtype(dtype), (rows, self.logical_shape[-1] // values * words)
        return np.dtype(_PLAIN[self.ggml_type]), self.logical_shape


def _read(fmt: str, h: BinaryIO):
    size = struct.calcsize(fmt)
    data = h.read(size)
    if len(data) != size:
        raise ValueError("truncated GGUF file")
    return struct.unpack(fmt, data)[0]


def _read_str(h: BinaryIO) -> str:
    n = _read("<Q", h)
    raw = h.read(n)
    if len(raw) != n:
        raise ValueError("truncated GGUF string")
    return raw.decode("utf-8")


def _read_value(h: BinaryIO, vt: ValueType):
    if vt is ValueType.STRING:
        return _read_str(h)
    if vt is ValueType.ARRAY:
        et = ValueType(_read("<I", h))
        n = _read("<Q", h)
        return [_read_value(h, et) for _ in range(n)]
    return _read(_SCALAR[vt], h)


class GGUFFile:
    """Read-only mmap of a GGUF v3 file with physical numpy views of its tensors."""

    def __init__(self, path: str | Path) -> None:
        self.path = Path(path)
        with self.path.open("rb") as h:
            if _read("<I", h) != GGUF_MAGIC:
                raise ValueError(f"{path}: not a GGUF file")
            version = _read("<I", h)
            if version != GGUF_VERSION:
                raise ValueError(f"{path}: GGUF version {version} unsupported")
            n_tensors = _read("<Q", h)
            n_kv = _read("<Q", h)
            self.metadata: dict[str, object] = {}
            for _ in range(n_kv):
                key = _read_str(h)
                self.metadata[key] = _read_value(h, ValueType(_read("<I", h)))
            infos = []
            for _ in range(n_tensors):
                name = _read_str(h)
                n_dims = _read("<I", h)
                dims = tuple(_read("<Q", h) for _ in range(n_dims))
                gt = GGMLType(_read("<I", h))
                off = _read("<Q", h)
                infos.append((name, tuple(reversed(dims)), gt, off))
            align = int(self.metadata.get("general.alignment", DEFAULT_ALIGNMENT))
            pos = h.tell()
            data_start = (pos + align - 1) // align * align
        self._file = self.path.open("rb")
        self._mm = mmap.mmap(self._file.fileno(), 0, access=mmap.ACCESS_READ)
        self.tensors: dict[str, TensorEntry] = {}
        for name, shape, gt, off in infos:
            if gt in _BLOCKS:
                values, nbytes, _, _ = _BLOCKS[gt]
                rows = int(np.prod(shape[:-1])) if len(shape) > 1 else 1
                size = rows * (shape[-1] // values) * nbytes
            else:
                size = int(np.prod(shape)) * np.dtype(_PLAIN[gt]).itemsize
            self.tensors[name] = TensorEntry(name, gt, shape, data_start + off, size)

    def array(self, name: str) -> np.ndarray:
        """Physical view (no copy) of one tensor."""
        e = self.tensors[name]
        dtype, shape = e.physical
        return np.frombuffer(self._mm, dtype=dtype, count=e.nbytes // dtype.itemsize, offset=e.offset).reshape(shape)

    def close(self) -> None:
        """Closes the file; the mapping stays alive while array() views of it exist."""
        try:
            self._mm.close()
        except BufferError:
            pass
        self._file.close()

    def __enter__(self) -> "GGUFFile":
        return self

    def __exit__(self, *exc) -> None:
        self.close()


@dataclass(frozen=True)
class WriteTensor:
    name: str
    data: np.ndarray        # packed bytes (block types) or plain values
    ggml_type: GGMLType
    logical_shape: tuple[int, ...]


def _w_str(h: BinaryIO, s: str) -> None:
    raw = s.encode("utf-8")
    h.write(struct.pack("<Q", len(raw)))
    h.write(raw)


def pad_to_alignment(h: BinaryIO, align: int = DEFAULT_ALIGNMENT) -> None:
    rem = h.tell() % align
    if rem:
        h.write(bytes(align - rem))


def write_header(h: BinaryIO, tensors: list[WriteTensor], *, arch: str = "qwen3", name: str = "Qwen3",
                 file_type: int = FILE_TYPE_MOSTLY_Q4_K_M, extra_u32: tuple[tuple[str, int], ...] = ()) -> None:
    """Header, metadata (keys of quantize/gguf.py:349-360) and tensor infos, padded to the
    32-byte data section; each tensor's offset assumes its payload padded to 32 bytes."""
    meta: list[tuple[str, ValueType, object]] = [
        ("general.architecture", ValueType.STRING, arch), ("general.name", ValueType.STRING, name),
        ("general.type", ValueType.STRING, "model"), ("general.file_type", ValueType.UINT32, file_type),
        ("general.quantization_version", ValueType.UINT32, 2)]
    meta += [(k, ValueType.UINT32, v) for k, v in extra_u32]
    offsets, cur = [], 0
    for t in tensors:
        offsets.append(cur)
        cur += (t.data.nbytes + DEFAULT_ALIGNMENT - 1) // DEFAULT_ALIGNMENT * DEFAULT_ALIGNMENT
    h.write(struct.pack("<IIQQ", GGUF_MAGIC, GGUF_VERSION, len(tensors), len(meta)))
    for key, vt, value in meta:
        _w_str(h, key)
        h.write(struct.pack("<I", int(vt)))
        if vt is ValueType.STRING:
            _w_str(h, str(value))
        else:
            h.write(struct.pack(_SCALAR[vt], value))
    for t, off in zip(tensors, offsets):
        _w_str(h, t.name)
        h.write(struct.pack("<I", len(t.logical_shape)))
        for d in reversed(t.logical_shape):
            h.write(struct.pack("<Q", d))
        h.write(struct.pack("<IQ", int(t.ggml_type), off))
    pad_to_alignment(h)


def write_gguf(path: str | Path, tensors: list[WriteTensor], *, arch: str = "qwen3", name: str = "Qwen3",
               file_type: int = FILE_TYPE_MOSTLY_Q4_K_M, extra_u32: tuple[tuple[str, int], ...] = ()) -> Path:
    """Writes a GGUF v3 file: header, then each payload padded to 32 bytes."""
    path = Path(path)
    with path.open("wb") as h:
        write_header(h, tensors, arch=arch, name=name, file_type=file_type, extra_u32=extra_u32)
        for t in tensors:
            h.write(np.ascontiguousarray(t.data).tobytes())
            pad_to_alignment(h)
    return path


def q4_k_m_type(name: str, shape: tuple[int, ...], num_layers: int, *, f16_names: tuple[str, ...] = ()) -> GGMLType:
    """Q4_K_M tensor type for a Qwen3 checkpoint key (quantize/gguf.py:54-83 with the
    models/quantized_qwen3/quantization.py:17-23 Q6_K names)."""
    first, last = num_layers // 8, (7 * num_layers) // 8
    more_bits = {i for i in range(num_layers) if i < first or i >= last or (i - first) % 3 == 2}
    if name in f16_names:
        return GGMLType.F16
    if len(shape) >= 2:
        if name == "lm_head.weight":
            return GGMLType.Q6_K
        parts = name.split(".")
        if len(parts) > 2 and parts[0] == "model" and parts[1] == "layers" and int(parts[2]) in more_bits and (
                name.endswith("self_attn.v_proj.weight") or name.endswith("mlp.down_proj.weight")):
            return GGMLType.Q6_K
    if len(shape) != 2:
        return GGMLType.F32
    if shape[-1] % 256 == 0:
        return GGMLType.Q4_K
    if shape[-1] % 32 == 0:
        return GGMLType.Q8_0
    return GGMLType.F32
