"""Q4_K_M GGUF export with the sm_100a quantizers (the torch2vk.quantize surface:
src/torch2vk/quantize/gguf.py:31-247 and quantize/vulkan.py:39-50 wrappers).

Q4KMQuantizationConfig keeps the reference's fields and type rules (forced
F16 names / prefixes, forced Q8_0 / Q6_K names / prefixes, rank != 2 -> F32,
cols % 256 -> Q4_K, cols % 32 -> Q8_0, else F32).  export_q4_k_m_gguf streams
safetensors tensors through the GPU quantizer kernels (bit-exact with the CPU
oracle restatement of the reference quantizers) into a GGUF v3 file with the
reference's metadata keys, tensor order and 32-byte alignment.
"""

from __future__ import annotations

import shutil
from collections.abc import Iterator
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
def _iter_safetensors(model_dir: Path, subdirs: tuple[str, ...]) -> Iterator[tuple[str, torch.Tensor]]:
    from safetensors import safe_open

    for source in (model_dir, *(model_dir / s for s in subdirs)):
        paths = sorted(source.glob("*.safetensors"))
        if not paths:
            raise FileNotFoundError(f"No safetensors files found in {source}")
        for p in paths:
            with safe_open(p, framework="pt", device="cpu") as ck:
                for name in ck.keys():
                    yield name, ck.get_tensor(name)


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
    """safetensors checkpoint -> Q4_K_M GGUF (quantize/gguf.py:191-247); an existing file with
    the same type plan is kept unless overwrite."""
    out = Path(output).expanduser().resolve()
    if out.exists() and not overwrite and gguf_matches_quantization(out, config):
        return out
    out.parent.mkdir(parents=True, exist_ok=True)
    if out.exists():
        out.unlink()
    data_path = out.with_name(f"{out.name}.data.tmp")
    final_path = out.with_name(f"{out.name}.tmp")
    infos: list[gguf.WriteTensor] = []
    seen: set[str] = set()
    try:
        with data_path.open("wb") as data:
            for name, tensor in _iter_safetensors(Path(model_dir).expanduser().resolve(), config.safetensor_subdirs):
                if name in seen:
                    raise ValueError(f"Duplicate safetensor tensor name while writing GGUF: {name}")
                seen.add(name)
                wt = tensor_to_gguf(name, tensor, config, device)
                data.write(np.ascontiguousarray(wt.data).tobytes())
                gguf.pad_to_alignment(data)
                infos.append(gguf.WriteTensor(wt.name, np.empty(wt.data.nbytes, np.uint8), wt.ggml_type,
                                              wt.logical_shape))
        with final_path.open("wb") as h:
            gguf.write_header(h, infos, arch=config.gguf_arch, name=config.model_name,
                              extra_u32=config.extra_uint32_metadata)
            with data_path.open("rb") as data:
                shutil.copyfileobj(data, h, length=16 << 20)
        final_path.replace(out)
    finally:
        for p in (data_path, final_path):
            if p.exists():
                p.unlink()
    return out
