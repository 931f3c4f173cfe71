"""Peer-memory all-reduce for tensor-parallel decode (wraps t2c_allreduce_sum_f16).

Every rank allocates one buffer (flags + two fp16 regions), publishes its CUDA
IPC handle through the process group, and maps the buffers of its peers; a
reduction is then one kernel on the caller's stream that reads the peers'
regions over NVLink (no NCCL call, no multicast), so it captures into CUDA
graphs.  Tensors larger than the buffer go to NCCL.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from torch2vk_b200 import _lib


class PeerAllReduce:
    def __init__(self, group=None, *, max_elems: int = 1 << 16, device: torch.device | None = None) -> None:
        self.group = group
        self.rank = dist.get_rank(group)
        self.tp = dist.get_world_size(group)
        if self.tp > 8:
            raise ValueError("peer all-reduce supports up to 8 ranks")
        self.max_elems = (max_elems + 7) // 8 * 8
        device = device or torch.device("cuda", torch.cuda.current_device())
        lib = _lib.lib()
        nbytes = int(lib.raw("t2c_allreduce_buffer_bytes")(self.max_elems))
        # a dedicated allocation (its own IPC handle); zeroed flags
        self._buf = torch.zeros(nbytes + 256, dtype=torch.uint8, device=device)
        base = self._buf.data_ptr()
        self._local = (base + 255) // 256 * 256
        handle = (ctypes.c_uint8 * 64)()
        offset = ctypes.c_int64(0)
        lib.call("t2c_ipc_get_handle", ctypes.c_void_p(self._local), handle, ctypes.byref(offset))
        mine = (bytes(handle), int(offset.value))
        everyone: list = [None] * self.tp
        dist.all_gather_object(everyone, mine, group=group)
        self._opened: list[int] = []
        ptrs = []
        for p, (h, off) in enumerate(everyone):
            if p == self.rank:
                ptrs.append(self._local)
                continue
            out = ctypes.c_void_p(0)
            lib.call("t2c_ipc_open_handle", (ctypes.c_uint8 * 64).from_buffer_copy(h), ctypes.byref(out))
            self._opened.append(out.value)
            ptrs.append(out.value + off)
        self._ptrs = (ctypes.c_void_p * self.tp)(*ptrs)
        self._counter = torch.zeros(2, dtype=torch.int32, device=device)
        dist.barrier(group=group)

    def __call__(self, x: torch.Tensor) -> None:
        """In-place sum of x (fp16, contiguous) over the ranks."""
        n = x.numel()
        if x.dtype != torch.float16 or not x.is_contiguous() or n > self.max_elems or n % 8:
            dist.all_reduce(x, group=self.group)
            return
        _lib.lib().call("t2c_allreduce_sum_f16", _lib.ptr(x), n, self._ptrs, self.rank, self.tp,
                        _lib.ptr(self._counter), self.max_elems, _lib.stream_ptr())

    def close(self) -> None:
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for p in self._opened:
            _lib.lib().call("t2c_ipc_close_handle", ctypes.c_void_p(p))
        self._opened = []
