"""ctypes binding of libt2c_sm100.so (the C ABI declared in include/t2c_sm100.h).

The library is loaded from the package directory (built in-tree by
``torch2vk_b200.build``).  There is no fallback: if the library or a CUDA
device is missing, calls raise.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libt2c_sm100.so"
# Alternative build of the same library (for A/B timing of kernel variants); default: the in-tree build.
if os.environ.get("T2C_LIBRARY"):
    LIB_PATH = Path(os.environ["T2C_LIBRARY"]).resolve()

T2C_OK = 0
STATUS_NAMES = {1: "EINVAL", 2: "EUNSUPPORTED", 3: "ECUDA", 4: "ETIMEOUT", 5: "ESCRATCH"}

Q8_0 = 8
Q4_K = 12
Q6_K = 14
F16 = 1
F32 = 0
WTYPE_BY_NAME = {"q8_0": Q8_0, "q4_k": Q4_K, "q6_k": Q6_K, "f16": F16}

_c = ctypes
_vp = _c.c_void_p
_i64 = _c.c_int64
_i32 = _c.c_int
_f32 = _c.c_float

# name -> argtypes (all return int status unless listed in _RESTYPES)
_SIGNATURES: dict[str, list] = {
    "t2c_abi_version": [],
    "t2c_device_sm_count": [],
    "t2c_linear": [_i32, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp],
    "t2c_linear_multi": [_i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _f32, _i64, _i64, _vp],
    "t2c_linear_swiglu": [_i32, _vp, _vp, _vp, _vp, _vp, _f32, _i64, _i64, _i64, _vp],
    "t2c_quantize": [_i32, _vp, _vp, _i64, _i64, _vp],
    "t2c_dequantize": [_i32, _vp, _vp, _i64, _i64, _vp],
    "t2c_device_status": [_vp, _i32, _vp],
    "t2c_lm_head_argmax": [_i32, _vp, _vp, _vp, _vp, _vp, _f32, _i64, _i64, _i64, _vp],
    "t2c_token_select": [_vp, _vp, _i64, _i64, _vp, _i64, _vp, _vp, _vp],
    "t2c_token_store": [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _c.c_int32, _vp, _i32, _vp],
    "t2c_rms_norm": [_vp, _vp, _vp, _i64, _i64, _f32, _vp],
    "t2c_qk_norm_rope_cache": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64,
                               _i64, _i64, _i64, _vp, _f32, _vp],
    "t2c_attn_decode": [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp,
                        _i64, _vp],
    "t2c_attn_decode_fused": [_vp, _vp, _vp, _i64, _i64, _i64, _vp, _vp, _vp, _c.c_float, _vp, _vp, _i64, _i64,
                              _i64, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _i64, _vp],
    "t2c_attn_decode_fused_workspace": [_i64, _i64, _i64, _i64, _i64],
    "t2c_allreduce_buffer_bytes": [_i64],
    "t2c_ipc_get_handle": [_vp, _vp, _vp],
    "t2c_ipc_open_handle": [_vp, _vp],
    "t2c_ipc_close_handle": [_vp],
    "t2c_allreduce_sum_f16": [_vp, _i64, _vp, _c.c_int, _c.c_int, _vp, _i64, _vp],
    "t2c_linear_allreduce_buffer_bytes": [_i64],
    "t2c_linear_allreduce": [_c.c_int, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _c.c_int, _c.c_int, _vp, _i64, _vp],
    "t2c_attn_prefill": [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                         _i64, _i64, _i64, _i64, _vp],
    "t2c_copy4d": [_i32, _vp, _vp, _vp, _vp, _vp, _vp],
    "t2c_elementwise4d": [_i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp],
    "t2c_rope_table": [_vp, _vp, _i64, _i64, _i64, _f32, _i64, _f32, _vp],
    "t2c_rms_norm_rope": [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _vp],
    "t2c_kv_cache_write": [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                           _vp],
    "t2c_token_select_chunks": [_vp, _vp, _i64, _vp, _vp, _vp],
    "t2c_linear_q8_0_bias": [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i32, _vp],
    "t2c_conv2d_q8_0": [_vp, _vp, _vp, _vp] + [_i64] * 13 + [_i32, _vp],
    "t2c_conv2d_q8_0_nhwc": [_vp, _vp, _vp, _vp] + [_i64] * 13 + [_i32, _vp],
    "t2c_im2col_f16": [_vp, _vp] + [_i64] * 13 + [_vp, _i32, _vp],
    "t2c_layer_norm": [_vp, _vp, _vp, _vp, _i64, _i64, _f32, _vp],
    "t2c_layer_norm_padded": [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _f32, _vp],
    "t2c_gelu": [_vp, _vp, _i64, _vp],
    "t2c_index_rows": [_vp, _vp, _vp, _i64, _i64, _i64, _vp],
    "t2c_attn_masked": [_vp] * 5 + [_i64] * 5 + [_vp] * 5 + [_f32, _vp],
    "t2c_embedding": [_i32, _vp, _vp, _vp, _i64, _i64, _i64, _vp],
    "t2c_add": [_vp, _vp, _vp, _i64, _vp],
    "t2c_swiglu": [_vp, _vp, _vp, _i64, _vp],
    "t2c_advance_positions": [_vp, _i64, _vp, _vp],
    "t2c_attn_masked_gqa": [_vp] * 5 + [_i64] * 6 + [_vp] * 3 + [_i64] * 2 + [_f32, _vp],
    "t2c_omnivoice_input_embed": [_vp] * 5 + [_i64] * 6 + [_vp],
    "t2c_attn_decode_paged": [_vp] * 6 + [_i64] * 11 + [_vp, _i64, _vp],
    "t2c_kv_cache_write_paged": [_vp, _vp, _i64, _i64, _vp, _vp] + [_i64] * 10 + [_vp],
    "t2c_attn_decode_static": [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp],
    "t2c_linear_f32_scratch_bytes": [_i64, _i64, _i64],
    "t2c_linear_f32": [_i32, _vp, _vp, _vp, _i64, _i64, _i64, _vp, _i64, _vp],
    "t2c_rms_norm_f32": [_vp, _vp, _vp, _i64, _i64, _f32, _vp],
    "t2c_rms_norm_rope_f32": [_vp, _vp, _vp, _vp, _vp, _i32, _i64, _i64, _i64, _i64, _f32, _vp],
    "t2c_binary_f32": [_i32, _vp, _vp, _vp, _i64, _vp],
    "t2c_cast": [_vp, _i32, _vp, _i32, _i64, _vp],
    "t2c_slice_last_f32_to_f16": [_vp, _vp, _i64, _i64, _i64, _vp],
    "t2c_value_cache_write_f32": [_vp, _vp, _i32, _vp, _vp, _i64, _i64, _i64, _i64, _vp],
    "t2c_fa_mask_opt": [_vp, _vp, _i64, _i64, _i64, _i64, _vp],
    "t2c_attn_prefill_masked_f32": [_vp, _vp, _vp, _vp, _vp, _vp] + [_i64] * 8 + [_f32, _vp],
    "t2c_embedding_f32": [_i32, _vp, _vp, _vp, _i64, _i64, _i64, _vp],
    "t2c_rope_table_f32": [_vp, _vp, _i64, _i64, _i64, _f32, _i64, _f32, _vp],
    "t2c_rope_table_dev": [_vp, _vp, _i64, _i64, _i64, _f32, _vp, _f32, _i32, _vp],
    "t2c_index_copy_rows": [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp],
    "t2c_embedding_q8_0": [_vp, _vp, _vp, _i64, _i64, _i64, _vp],
    "t2c_ew_misc": [_i32, _vp, _i32, _vp, _i32, _vp, _i32, _i64, _i64, _f32, _vp],
    "t2c_row_mean_f32": [_vp, _vp, _i64, _i64, _vp],
}
_RESTYPES = {"t2c_last_error": _c.c_char_p, "t2c_attn_decode_fused_workspace": _c.c_int64,
             "t2c_allreduce_buffer_bytes": _c.c_int64, "t2c_linear_f32_scratch_bytes": _c.c_int64,
             "t2c_linear_allreduce_buffer_bytes": _c.c_int64}


class T2CError(RuntimeError):
    """A libt2c_sm100 entry point returned a non-zero status."""

    def __init__(self, function: str, status: int, message: str) -> None:
        super().__init__(f"{function} failed ({STATUS_NAMES.get(status, status)}): {message}")
        self.function = function
        self.status = status


class _Library:
    def __init__(self, path: Path) -> None:
        if not path.exists():
            raise FileNotFoundError(
                f"{path} is missing: build it with `python -m torch2vk_b200.build` (nvcc, sm_100a)"
            )
        self.handle = ctypes.CDLL(str(path))
        self.handle.t2c_last_error.argtypes = []
        self.handle.t2c_last_error.restype = _c.c_char_p
        for name, argtypes in _SIGNATURES.items():
            fn = getattr(self.handle, name)
            fn.argtypes = argtypes
            fn.restype = _RESTYPES.get(name, _c.c_int)

    def call(self, name: str, *args) -> None:
        status = getattr(self.handle, name)(*args)
        if status != T2C_OK:
            raise T2CError(name, status, self.handle.t2c_last_error().decode(errors="replace"))

    def raw(self, name: str):
        return getattr(self.handle, name)


_LIB: _Library | None = None


def lib() -> _Library:
    global _LIB
    if _LIB is None:
        _LIB = _Library(LIB_PATH)
    return _LIB


def exported_symbols() -> list[str]:
    return ["t2c_last_error", *_SIGNATURES.keys()]


def ptr(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("libt2c_sm100 operands must be CUDA tensors")
    return t.data_ptr()


def stream_ptr(stream: torch.cuda.Stream | None = None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def ptr_array(values) -> ctypes.Array:
    arr = (_vp * len(values))()
    for i, v in enumerate(values):
        arr[i] = v
    return arr


def int_array(values) -> ctypes.Array:
    arr = (_i32 * len(values))()
    for i, v in enumerate(values):
        arr[i] = v
    return arr


def i64_array(values) -> ctypes.Array:
    arr = (_i64 * len(values))()
    for i, v in enumerate(values):
        arr[i] = v
    return arr
