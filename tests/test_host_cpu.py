"""Host-side checks that need no GPU: the C-ABI library loads and exports every
symbol include/t2c_sm100.h declares (no compute calls), the ctypes signature
table covers the header, and the tensor wrappers reject bad arguments before
any launch."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch

REPO = Path(__file__).resolve().parents[1]
HEADER = REPO / "include" / "t2c_sm100.h"


def header_symbols() -> set[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    text = re.sub(r"//[^\n]*", "", text)
    return set(re.findall(r"\b(t2c_[a-z0-9_]+)\s*\(", text))


def _built_lib() -> Path:
    from torch2vk_b200 import build

    path = build.LIB_PATH
    if not path.exists():
        build.build()
    return path


def test_library_exports_every_header_symbol():
    syms = header_symbols()
    assert len(syms) >= 25
    lib = ctypes.CDLL(str(_built_lib()))
    missing = [s for s in sorted(syms) if not hasattr(lib, s)]
    assert not missing, missing
    lib.t2c_abi_version.restype = ctypes.c_int
    assert lib.t2c_abi_version() == 1
    lib.t2c_last_error.restype = ctypes.c_char_p
    assert isinstance(lib.t2c_last_error(), bytes)


def test_ctypes_table_covers_header():
    from torch2vk_b200 import _lib

    assert header_symbols() == set(_lib.exported_symbols()), header_symbols() ^ set(_lib.exported_symbols())


def test_wrappers_reject_bad_arguments_without_launching():
    from torch2vk_b200 import kernels

    x = torch.zeros(2, 256, dtype=torch.float16)
    w = torch.zeros(4, 36, dtype=torch.int32)
    with pytest.raises(ValueError, match="CUDA"):
        kernels.linear(x, w, "q4_k", 256)
    with pytest.raises(ValueError, match="multiple of 256"):
        kernels.row_bytes(kernels.wtype_of("q4_k"), 300)
    with pytest.raises(ValueError):
        kernels.quantize(torch.zeros(2, 256), "q8_0")
    with pytest.raises(ValueError, match="token_major|head_major|bogus"):
        kernels.cache_strides(torch.zeros(1, 2, 3, 4), "bogus")


def test_session_requires_cuda():
    from torch2vk_b200.runtime.session import RuntimeSession

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        RuntimeSession.open()
