"""Host-side checks that need no GPU: the C-ABI library loads and exports every
symbol include/t2c_sm100.h declares (no compute calls), the ctypes signature
table covers the header, and the tensor wrappers reject bad arguments before
any launch."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import numpy as np
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


def test_replay_push_slots_and_guards():
    """Captured replay plans: a DynamicPush hands ops device slots that are rewritten from each step's
    value, records guards, and bakes any host use of the value behind an equality guard."""
    import numpy as np

    from torch2vk_b200.runtime.replay import DynamicPush, PushSlots

    slots = PushSlots(torch.device("cpu"))
    pos = DynamicPush(slots, "cache_position", 300)
    a = pos.device(torch.int64, 3, ramp=True)
    b = pos.device(torch.int32, 4, clamp_max=301)
    assert pos.device(torch.int64, 3, ramp=True).data_ptr() == a.data_ptr()  # shared slot
    assert a.data_ptr() % 16 == 0 and b.data_ptr() % 16 == 0
    pos.guard(0, 640)
    theta = DynamicPush(slots, "theta", 1e6)
    assert float(theta) == 1e6 and theta == 1e6
    slots.names = frozenset({"cache_position", "theta"})
    img = slots.host_image({"cache_position": 305, "theta": 1e6})
    off_a, _ = slots.slots[("cache_position", torch.int64, 3, True, None)]
    off_b, _ = slots.slots[("cache_position", torch.int32, 4, False, 301)]
    assert np.frombuffer(img[off_a:off_a + 24].tobytes(), np.int64).tolist() == [305, 306, 307]
    assert np.frombuffer(img[off_b:off_b + 16].tobytes(), np.int32).tolist() == [301] * 4
    assert slots.admits({"cache_position": 639, "theta": 1e6})
    assert not slots.admits({"cache_position": 640, "theta": 1e6})  # outside the range guard
    assert not slots.admits({"cache_position": 5, "theta": 1e4})  # baked value changed
    assert not slots.admits({"cache_position": 5})  # another set of names than the capture's
    # why a value set is not served: a range miss runs directly, an equality or name-set miss recaptures
    assert slots.rejection({"cache_position": 640, "theta": 1e6}) == "range"
    assert slots.rejection({"cache_position": 5, "theta": 1e4}) == "eq"
    assert slots.rejection({"cache_position": 5}) == "names"
    assert slots.rejection({"cache_position": 5, "theta": 1e6}) is None
    assert int(DynamicPush(slots, "token_index", 7)) + 1 == 8
    assert ("token_index", "eq", 7, None) in slots.guards


def test_decode_ops_read_dynamic_push_constants_from_slots(monkeypatch):
    """While a replay plan is captured, the decode ops hand the kernels device slots instead of host
    values: attention lengths (cache_position clamped to S - 1), the cache-write row, the rope-table
    start and the token index; their guards bound the steps the graph serves."""
    from types import SimpleNamespace

    from torch2vk_b200.runtime import optable
    from torch2vk_b200.runtime.replay import DynamicPush, PushSlots

    calls = []
    for name in ("attn_decode", "kv_cache_write", "rope_table", "token_store"):
        monkeypatch.setattr(optable.kernels, name, lambda *a, _n=name, **k: calls.append((_n, a, k)))
    slots = PushSlots(torch.device("cpu"))
    B, NH, NK, S, D = 2, 4, 2, 64, 128
    v = SimpleNamespace(name="v")
    f16 = lambda *shape: torch.zeros(*shape, dtype=torch.float16)  # noqa: E731
    b = {"q": f16(B, NH, 1, D), "new_k": f16(B, NK, 1, D), "new_v": f16(B, 1, NK, D), "k_cache": f16(B, S, NK, D),
         "v_cache": f16(B, S, NK, D), "output": f16(B, NH, 1, D)}
    s = {"B": B, "NH": NH, "NK": NK, "S": S, "D": D, "T": 1}
    optable.OPS["SdpaDecodeCacheWriteF32Program"](None, v, b, s, {"cache_position": DynamicPush(slots, "cache_position", 9)})
    optable.OPS["RopeTableF32Program"](None, v, {"cos": f16(1, 1, D), "sin": f16(1, 1, D)}, {},
                                       {"theta": DynamicPush(slots, "theta", 1e6),
                                        "start_position": DynamicPush(slots, "start_position", 9)})
    optable.OPS["Qwen3TokenStoreEosProgram"](None, v, {"next_token": torch.zeros(1, 1, dtype=torch.int64),
                                                      "done": torch.zeros(1, dtype=torch.int32),
                                                      "generated_tokens": torch.zeros(1, 8, dtype=torch.int64),
                                                      "generated_length": torch.zeros(1, dtype=torch.int32),
                                                      "stopped": torch.zeros(1, dtype=torch.int32)}, {},
                                             {"token_index": DynamicPush(slots, "token_index", 3)})
    names = [c[0] for c in calls]
    assert names == ["kv_cache_write", "kv_cache_write", "attn_decode", "rope_table", "token_store"]
    push = {"cache_position": 70, "start_position": 70, "theta": 1e6, "token_index": 5}
    slots.names = frozenset(push)
    slots.buffer.copy_(torch.from_numpy(np.pad(slots.host_image(push), (0, slots.buffer.numel() - max(slots.used, 16)))))
    assert calls[0][2]["positions"].tolist() == [70] and calls[0][2]["position"] == 0
    assert calls[2][1][3].tolist() == [S - 1] * B and calls[2][2]["splits"] == optable._decode_splits(S)
    assert calls[3][2]["start_position_dev"].tolist() == [70]
    assert calls[4][2]["token_index_dev"].tolist() == [5]
    assert not slots.admits(push)  # the cache write's guard: 0 <= cache_position < S
    assert slots.admits({**push, "cache_position": 63}) and not slots.admits({**push, "theta": 1e4})
