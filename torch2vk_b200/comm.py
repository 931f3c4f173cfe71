"""Peer-memory all-reduce for tensor-parallel decode (wraps t2c_allreduce_sum_f16 and the fused
row-parallel linear t2c_linear_allreduce).

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


def _exchange_buffers(group, rank: int, tp: int, nbytes: int, device: torch.device):
    """A zeroed, 256-byte aligned device buffer of nbytes in its own allocation, mapped into every
    rank: (owning tensor, the tp addresses as seen by this rank, the peer mappings to close)."""
    lib = _lib.lib()
    buf = torch.zeros(nbytes + 256, dtype=torch.uint8, device=device)
    local = (buf.data_ptr() + 255) // 256 * 256
    handle = (ctypes.c_uint8 * 64)()
    offset = ctypes.c_int64(0)
    lib.call("t2c_ipc_get_handle", ctypes.c_void_p(local), handle, ctypes.byref(offset))
    everyone: list = [None] * tp
    dist.all_gather_object(everyone, (bytes(handle), int(offset.value)), group=group)
    opened: list[int] = []
    ptrs = []
    for p, (h, off) in enumerate(everyone):
        if p == rank:
            ptrs.append(local)
            continue
        out = ctypes.c_void_p(0)
        lib.call("t2c_ipc_open_handle", (ctypes.c_uint8 * 64).from_buffer_copy(h), ctypes.byref(out))
        opened.append(out.value)
        ptrs.append(out.value + off)
    return buf, (ctypes.c_void_p * tp)(*ptrs), opened


class PeerAllReduce:
    """linear_rows > 0 also sets up the buffer of the fused row-parallel linear (`linear`):
    outputs of up to linear_rows rows at one token."""

    def __init__(self, group=None, *, max_elems: int = 1 << 16, device: torch.device | None = None,
                 linear_rows: int = 0) -> None:
        self.group = group
        self.rank = dist.get_rank(group)
        self.tp = dist.get_world_size(group)
        if self.tp > 8:
            raise ValueError("peer all-reduce supports up to 8 ranks")
        self.max_elems = (max_elems + 7) // 8 * 8
        device = device or torch.device("cuda", torch.cuda.current_device())
        lib = _lib.lib()
        nbytes = int(lib.raw("t2c_allreduce_buffer_bytes")(self.max_elems))
        self._buf, self._ptrs, self._opened = _exchange_buffers(group, self.rank, self.tp, nbytes, device)
        self._counter = torch.zeros(2, dtype=torch.int32, device=device)
        self.linear_rows = int(linear_rows)
        if self.linear_rows > 0:
            lbytes = int(lib.raw("t2c_linear_allreduce_buffer_bytes")(self.linear_rows))
            self._lbuf, self._lptrs, opened = _exchange_buffers(group, self.rank, self.tp, lbytes, device)
            self._opened += opened
            self._lcounter = torch.zeros(2, dtype=torch.int32, device=device)
        dist.barrier(group=group)

    def __call__(self, x: torch.Tensor) -> None:
        """In-place sum of x (fp16, contiguous) over the ranks."""
        n = x.numel()
        if x.dtype != torch.float16 or not x.is_contiguous() or n > self.max_elems or n % 8:
            dist.all_reduce(x, group=self.group)
            return
        _lib.lib().call("t2c_allreduce_sum_f16", _lib.ptr(x), n, self._ptrs, self.rank, self.tp,
                        _lib.ptr(self._counter), self.max_elems, _lib.stream_ptr())

    def linear(self, x: torch.Tensor, w: torch.Tensor, kind: str | int, k: int, *, residual: torch.Tensor,
               out: torch.Tensor) -> bool:
        """out = residual + the sum over the ranks of x @ W_rank^T (each rank: its K-slice of a
        row-parallel weight), one fused launch; False (nothing launched) where the fused kernel does
        not serve the call, so the caller runs linear + all-reduce."""
        from torch2vk_b200 import kernels

        m = x.numel() // k
        n = out.numel() // max(1, m)
        if (self.linear_rows <= 0 or m != 1 or kernels.wtype_of(kind) != kernels.wtype_of("q4_k")
                or n % 16 or n > self.linear_rows or k % 512):
            return False
        _lib.lib().call("t2c_linear_allreduce", kernels.wtype_of(kind), _lib.ptr(x), _lib.ptr(w), _lib.ptr(residual),
                        _lib.ptr(out), 1, n, k, self._lptrs, self.rank, self.tp, _lib.ptr(self._lcounter),
                        self.linear_rows, _lib.stream_ptr())
        return True

    def close(self) -> None:
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for p in self._opened:
            _lib.lib().call("t2c_ipc_close_handle", ctypes.c_void_p(p))
        self._opened = []
