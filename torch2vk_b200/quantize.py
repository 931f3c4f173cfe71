"""Q4_K_M GGUF export with the sm_100a quantizers (the torch2vk.quantize surface:
src/torch2vk/quantize/gguf.py:31-247 and quantize/vulkan.py:39-50 wrappers).

Q4KMQuantizationConfig keeps the reference's fields and type rules (forced
F16 names / prefixes, forced Q8_0 / Q6_K names / prefixes, rank != 2 -> F32,
cols % 256 -> Q4_K, cols % 32 -> Q8_0, else F32).  export_q4_k_m_gguf streams
safetensors tensors through the GPU quantizer kernels (bit-exact with the CPU
oracle restatement of the reference quantizers) into a GGUF v3 file with the
reference's metadata keys and 32-byte alignment, header first (payload sizes
come from the checkpoint headers).
"""

from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

from torch2vk_b200 import gguf
from torch2vk_b200.gguf import GGMLType as GGUFTensorType

GGUF_FILE_TYPE_MOSTLY_Q4_K_M = gguf.FILE_TYPE_MOSTLY_Q4_K_M


def _checkpoint_float_dtype(dtype: str) -> str:
    if dtype in {"float32", "float16", "bfloat16"} or dtype.startswith("float8"):
        return "float32"
    return dtype


def _matrix_shape(shape: tuple[int, ...]) -> tuple[int, int]:
    cols = 1
    for d in shape[1:]:
        cols *= d
    return shape[0], cols


def _round_up(value: int, multiple: int) -> int:
    return (value + multiple - 1) // multiple * multiple


@dataclass(frozen=True, slots=True)
class _WeightDeclaration:
    gguf_type: GGUFTensorType
    dtype: str
    shape: tuple[int, ...]
    layout_source: str


@dataclass(frozen=True, slots=True)
class Q4KMQuantizationConfig:
    model_name: str
    gguf_arch: str
    f16_tensor_names: tuple[str, ...] = ()
    f16_tensor_prefixes: tuple[str, ...] = ()
    q6_tensor_names: tuple[str, ...] = ()
    q6_tensor_prefixes: tuple[str, ...] = ()
    q8_tensor_names: tuple[str, ...] = ()
    q8_tensor_prefixes: tuple[str, ...] = ()
    safetensor_subdirs: tuple[str, ...] = ()
    extra_uint32_metadata: tuple[tuple[str, int], ...] = ()

    @property
    def has_q6(self) -> bool:
        return bool(self.q6_tensor_names or self.q6_tensor_prefixes)

    def _preserve_f16(self, key: str) -> bool:
        return key in self.f16_tensor_names or key.startswith(self.f16_tensor_prefixes)

    def gguf_type(self, *, checkpoint_key: str, shape: tuple[int, ...], dtype: str = "float32") -> GGUFTensorType:
        if self._preserve_f16(checkpoint_key):
            return GGUFTensorType.F16
        if _checkpoint_float_dtype(dtype) != "float32":
            return GGUFTensorType.F32
        rank2 = len(shape) >= 2
        if rank2 and (checkpoint_key in self.q8_tensor_names or checkpoint_key.startswith(self.q8_tensor_prefixes)):
            return GGUFTensorType.Q8_0
        if rank2 and (checkpoint_key in self.q6_tensor_names or checkpoint_key.startswith(self.q6_tensor_prefixes)):
            return GGUFTensorType.Q6_K
        if len(shape) != 2:
            return GGUFTensorType.F32
        if shape[-1] % 256 == 0:
            return GGUFTensorType.Q4_K
        if shape[-1] % 32 == 0:
            return GGUFTensorType.Q8_0
        return GGUFTensorType.F32

    def declare_weight(self, *, checkpoint_key: str, dtype: str, shape: tuple[int, ...]) -> _WeightDeclaration:
        """Physical dtype / shape / layout expression of one checkpoint tensor in the GGUF."""
        if self._preserve_f16(checkpoint_key):
            return _WeightDeclaration(GGUFTensorType.F16, "float16", shape, "CONTIGUOUS_LAYOUT")
        dtype = _checkpoint_float_dtype(dtype)
        t = self.gguf_type(checkpoint_key=checkpoint_key, dtype=dtype, shape=shape)
        if t is GGUFTensorType.Q6_K:
            n, k = _matrix_shape(shape)
            if k % 256:
                raise ValueError(f"Q6_K tensor {checkpoint_key} requires K to be divisible by 256, got {k}")
            return _WeightDeclaration(t, "uint16", (n, k // 256 * 105), f"q6_k_halfwords_layout(logical_k={k})")
        if t is GGUFTensorType.Q8_0:
            n, k = _matrix_shape(shape)
            return _WeightDeclaration(t, "uint16", (n, _round_up(k, 32) // 32 * 17),
                                      f"q8_0_halfwords_layout(logical_k={k})")
        if t is GGUFTensorType.Q4_K:
            n, k = shape
            return _WeightDeclaration(t, "uint32", (n, k // 256 * 36), f"q4_k_words_layout(logical_k={k})")
        return _WeightDeclaration(t, dtype, shape, "CONTIGUOUS_LAYOUT")


def q4_k_m_more_bits_layer_indices(num_layers: int) -> tuple[int, ...]:
    """Layers whose v_proj / down_proj stay Q6_K under Q4_K_M (quantize/gguf.py:150-161)."""
    if num_layers <= 0:
        raise ValueError(f"num_layers must be positive, got {num_layers}")
    first, last = num_layers // 8, (7 * num_layers) // 8
    return tuple(i for i in range(num_layers) if i < first or i >= last or (i - first) % 3 == 2)


# ------------------------------------------------------------------ GPU quantizers
def _gpu_quantize(array: np.ndarray, kind: str, device: int | torch.device = 0) -> np.ndarray:
    from torch2vk_b200 import kernels

    if array.ndim != 2:
        raise ValueError(f"quantize expects a 2-D float32 array, got shape {array.shape}")
    x = torch.from_numpy(np.ascontiguousarray(array, dtype=np.float32)).to(device)
    packed = kernels.quantize(x, kind)
    return packed.cpu().numpy() if packed.dtype != torch.uint32 else packed.view(torch.int32).cpu().numpy().view(np.uint32)


def quantize_q4_k(array: np.ndarray, *, device: int = 0) -> np.ndarray:
    """fp32 [R, K] -> uint32 [R, K/256*36] on the GPU."""
    return _gpu_quantize(array, "q4_k", device)


def quantize_q6_k(array: np.ndarray, *, device: int = 0) -> np.ndarray:
    """fp32 [R, K] -> uint16 [R, K/256*105] on the GPU."""
    return _gpu_quantize(array, "q6_k", device)


def quantize_q8_0(array: np.ndarray, *, device: int = 0) -> np.ndarray:
    """fp32 [R, K] -> uint16 [R, K/32*17] on the GPU."""
    return _gpu_quantize(array, "q8_0", device)


def quantize_q4_k_vulkan(rt, array: np.ndarray, *, name: str = "") -> np.ndarray:
    """Reference-named entry (quantize/vulkan.py:39-50); runs the sm_100a quantizer on rt's device."""
    return quantize_q4_k(array, device=getattr(rt, "device", 0))


def quantize_q6_k_vulkan(rt, array: np.ndarray, *, name: str = "") -> np.ndarray:
    return quantize_q6_k(array, device=getattr(rt, "device", 0))


def quantize_q8_0_vulkan(rt, array: np.ndarray, *, name: str = "") -> np.ndarray:
    return quantize_q8_0(array, device=getattr(rt, "device", 0))


# ------------------------------------------------------------------ export
def _safetensor_files(model_dir: Path, subdirs: tuple[str, ...]) -> list[Path]:
    files: list[Path] = []
    for source in (model_dir, *(model_dir / s for s in subdirs)):
        found = sorted(source.glob("*.safetensors"))
        if not found:
            raise FileNotFoundError(f"No safetensors files found in {source}")
        files += found
    return files


@dataclass(frozen=True, slots=True)
class _PlannedTensor:
    """One checkpoint tensor as it will sit in the GGUF file: where it comes from, its type, its logical
    shape there and the size of its payload (known from the checkpoint header alone)."""
    name: str
    source: Path
    ggml_type: GGUFTensorType
    logical_shape: tuple[int, ...]
    nbytes: int


def _payload_plan(name: str, shape: tuple[int, ...], dtype: str,
                  config: "Q4KMQuantizationConfig") -> tuple[GGUFTensorType, tuple[int, ...], int]:
    """GGUF type, logical shape and payload bytes of a checkpoint tensor, from its shape and dtype."""
    t = config.gguf_type(checkpoint_key=name, dtype=dtype, shape=shape)
    count = int(np.prod(shape)) if shape else 1
    if t is GGUFTensorType.F16:
        return t, shape, 2 * count
    if t is GGUFTensorType.F32:
        return t, shape, 4 * count
    rows, cols = _matrix_shape(shape)
    if t is GGUFTensorType.Q8_0:
        padded = _round_up(cols, 32)
        return t, (rows, padded), rows * (padded // 32) * 34
    if t is GGUFTensorType.Q6_K:
        return t, (rows, cols), rows * (cols // 256) * 210
    return t, shape, rows * (cols // 256) * 144


def tensor_to_gguf(name: str, tensor: torch.Tensor, config: Q4KMQuantizationConfig,
                   device: int = 0) -> gguf.WriteTensor:
    """One checkpoint tensor -> its GGUF payload (quantize/gguf.py:284-342 type and shape rules)."""
    array = tensor.float().numpy() if tensor.is_floating_point() else tensor.numpy()
    shape = tuple(int(d) for d in array.shape)
    t = config.gguf_type(checkpoint_key=name, dtype=str(tensor.dtype).removeprefix("torch."), shape=shape)
    if t is GGUFTensorType.Q6_K:
        rows, cols = _matrix_shape(shape)
        if cols % 256:
            raise ValueError(f"Q6_K tensor {name} requires K to be divisible by 256, got {cols}")
        return gguf.WriteTensor(name, quantize_q6_k(array.reshape(rows, cols), device=device), t, (rows, cols))
    if t is GGUFTensorType.Q8_0:
        rows, cols = _matrix_shape(shape)
        padded = _round_up(cols, 32)
        f32 = np.zeros((rows, padded), np.float32)
        f32[:, :cols] = array.reshape(rows, cols)
        return gguf.WriteTensor(name, quantize_q8_0(f32, device=device), t, (rows, padded))
    if t is GGUFTensorType.F32:
        return gguf.WriteTensor(name, np.asarray(array, dtype=np.float32), t, shape)
    if t is GGUFTensorType.F16:
        if not tensor.is_floating_point():
            raise TypeError(f"F16 GGUF tensor {name} requires floating point source")
        return gguf.WriteTensor(name, tensor.to(torch.float16).numpy(), t, shape)
    if t is not GGUFTensorType.Q4_K:
        raise ValueError(f"Unsupported GGUF tensor type for {name}: {t}")
    return gguf.WriteTensor(name, quantize_q4_k(array, device=device), t, shape)


def gguf_matches_quantization(path: Path, config: Q4KMQuantizationConfig) -> bool:
    with gguf.GGUFFile(path) as f:
        if f.metadata.get("general.file_type") != GGUF_FILE_TYPE_MOSTLY_Q4_K_M:
            return False
        for key, value in config.extra_uint32_metadata:
            if f.metadata.get(key) != value:
                return False
        return all(e.ggml_type is config.gguf_type(checkpoint_key=n, shape=e.logical_shape)
                   for n, e in f.tensors.items())


def export_q4_k_m_gguf(*, model_dir: str | Path, output: str | Path, config: Q4KMQuantizationConfig,
                       overwrite: bool = False, device: int = 0) -> Path:
    """safetensors checkpoint -> Q4_K_M GGUF v3 file (the reference's export entry point,
    src/torch2vk/quantize/gguf.py:191-247: same arguments, type plan and metadata keys; an existing file
    whose tensor types already follow `config` is kept unless `overwrite`).

    The file is produced header first: every tensor's GGUF type and payload size follow from the
    checkpoint's own headers (names, shapes, dtypes), so the header with all tensor offsets is written
    before any weight is read; then each tensor is loaded, quantized on the GPU and written at its offset
    (payloads 32-byte aligned).  The file is assembled under a temporary name beside `output` and renamed
    into place only when complete.
    """
    from safetensors import safe_open

    out = Path(output).expanduser().resolve()
    if out.exists() and not overwrite and gguf_matches_quantization(out, config):
        return out
    plan: list[_PlannedTensor] = []
    names: set[str] = set()
    for path in _safetensor_files(Path(model_dir).expanduser().resolve(), config.safetensor_subdirs):
        with safe_open(path, framework="pt", device="cpu") as ck:
            for name in ck.keys():
                if name in names:
                    raise ValueError(f"tensor {name} appears twice in the checkpoint ({path})")
                names.add(name)
                sl = ck.get_slice(name)
                shape = tuple(int(d) for d in sl.get_shape())
                dtype = {"F32": "float32", "F16": "float16", "BF16": "bfloat16"}.get(sl.get_dtype(),
                                                                                  sl.get_dtype().lower())
                t, logical, nbytes = _payload_plan(name, shape, dtype, config)
                plan.append(_PlannedTensor(name, path, t, logical, nbytes))
    out.parent.mkdir(parents=True, exist_ok=True)
    partial = out.parent / f".{out.name}.partial"
    try:
        with partial.open("wb") as h:
            # the header only needs each payload's size: stand-in arrays of that many bytes
            gguf.write_header(h, [gguf.WriteTensor(p.name, np.empty(p.nbytes, np.uint8), p.ggml_type,
                                                   p.logical_shape) for p in plan],
                              arch=config.gguf_arch, name=config.model_name, extra_u32=config.extra_uint32_metadata)
            open_file, handle = None, None
            try:
                for p in plan:
                    if p.source != open_file:
                        if handle is not None:
                            handle.__exit__(None, None, None)
                        handle = safe_open(p.source, framework="pt", device="cpu")
                        handle.__enter__()
                        open_file = p.source
                    wt = tensor_to_gguf(p.name, handle.get_tensor(p.name), config, device)
                    payload = np.ascontiguousarray(wt.data)
                    if payload.nbytes != p.nbytes or wt.ggml_type is not p.ggml_type:
                        raise RuntimeError(f"{p.name}: planned {p.ggml_type.name} {p.nbytes} bytes, "
                                           f"produced {wt.ggml_type.name} {payload.nbytes}")
                    h.write(payload.tobytes())
                    gguf.pad_to_alignment(h)
            finally:
                if handle is not None:
                    handle.__exit__(None, None, None)
        partial.replace(out)
    finally:
        if partial.exists():
            partial.unlink()
    return out
