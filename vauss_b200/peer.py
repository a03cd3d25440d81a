"""Device buffers shared by the GPUs of one node (one process per GPU).

Each rank allocates its buffers with ``vs_peer_alloc`` (plain cudaMalloc),
the ranks exchange the CUDA IPC handles, and every rank maps the others'
buffers with ``vs_peer_open``.  The kernels of this library then read and
write those buffers directly over NVLink; torch only ever sees a rank's own
buffers (as tensors through the CUDA array interface), never a peer's.
``barrier`` is the stream-ordered device barrier over the ranks' flag arrays.
"""
from __future__ import annotations

import ctypes
from typing import Callable, Sequence

import torch

from . import _native as N
from . import ops

_TYPESTR = {torch.float32: "<f4", torch.uint32: "<u4", torch.int32: "<i4", torch.uint8: "|u1"}


class _DeviceArray:
    """A raw device allocation exposed through __cuda_array_interface__."""

    def __init__(self, ptr: int, numel: int, dtype: torch.dtype):
        self.__cuda_array_interface__ = {"shape": (numel,), "typestr": _TYPESTR[dtype], "data": (ptr, False),
                                         "version": 3, "strides": None}


def gather_bytes_nccl(data: bytes, device) -> list[bytes]:
    """All-gather one small byte string per rank (torch.distributed, default group)."""
    import torch.distributed as dist
    world = dist.get_world_size()
    mine = torch.tensor(list(data), dtype=torch.uint8, device=device)
    out = torch.empty(world * len(data), dtype=torch.uint8, device=device)
    dist.all_gather_into_tensor(out, mine)
    flat = bytes(out.cpu().tolist())
    return [flat[i * len(data):(i + 1) * len(data)] for i in range(world)]


class PeerGroup:
    """Buffers of `world` ranks mapped into every rank; `gather` exchanges
    each rank's 64-byte IPC handle (one entry per rank, in rank order)."""

    def __init__(self, device, world: int, rank: int, gather: Callable[[bytes], Sequence[bytes]]):
        if not 1 <= world <= N.PEER_MAX:
            raise ValueError(f"peer group of {world} ranks (at most {N.PEER_MAX})")
        self.device = torch.device(device)
        self.world, self.rank = world, rank
        self.ctx = ops.context(self.device)
        self.gather = gather
        self._own: list[int] = []
        self._opened: list[int] = []
        self.epoch = 0
        self.flags = self.alloc(64, torch.int32, zero=True)  # zeroed before any rank can signal
        self._flag_ptrs = (ctypes.c_void_p * N.PEER_MAX)(*self.flags, *([None] * (N.PEER_MAX - world)))

    def alloc(self, numel: int, dtype: torch.dtype, zero: bool = False) -> list[int]:
        """Allocates `numel` elements on every rank (zeroed if asked, before
        the handles are exchanged); returns the device addresses of all
        ranks' buffers as seen from this rank."""
        nbytes = max(numel, 1) * torch.tensor([], dtype=dtype).element_size()
        ptr = ctypes.c_void_p()
        h = N.IpcHandle()
        self.ctx.check(self.ctx.lib.vs_peer_alloc(self.ctx.h, nbytes, ctypes.byref(ptr), ctypes.byref(h)))
        self._own.append(ptr.value)
        if zero:
            torch.as_tensor(_DeviceArray(ptr.value, max(numel, 1), dtype), device=self.device).zero_()
            torch.cuda.synchronize(self.device)
        handles = self.gather(bytes(h.bytes))
        addrs = []
        for r, hb in enumerate(handles):
            if r == self.rank:
                addrs.append(ptr.value)
                continue
            ph = N.IpcHandle()
            ctypes.memmove(ph.bytes, hb, 64)
            peer = ctypes.c_void_p()
            self.ctx.check(self.ctx.lib.vs_peer_open(self.ctx.h, ctypes.byref(ph), ctypes.byref(peer)))
            self._opened.append(peer.value)
            addrs.append(peer.value)
        return addrs

    def local(self, addrs: Sequence[int], numel: int, dtype: torch.dtype) -> torch.Tensor:
        """This rank's buffer of `addrs` as a torch tensor (no copy)."""
        return torch.as_tensor(_DeviceArray(addrs[self.rank], numel, dtype), device=self.device)

    def barrier(self):
        """Device barrier of all ranks on the current stream."""
        self.epoch += 1
        self.ctx.bind()  # ordered after the work already queued on the current stream
        self.ctx.check(self.ctx.lib.vs_peer_barrier(self.ctx.h, self._flag_ptrs, self.world, self.rank,
                                                    self.epoch & 0xFFFFFFFF))

    def check(self):
        """Raises if a device wait of this rank gave up (synchronises)."""
        self.ctx.bind()
        self.ctx.check(self.ctx.lib.vs_ctx_check(self.ctx.h))

    def close(self):
        """Unmaps the peers' buffers and frees this rank's.  Call on every
        rank after a final synchronisation and a host-side barrier, so that no
        kernel of any rank still touches them."""
        for p in self._opened:
            self.ctx.lib.vs_peer_close(self.ctx.h, ctypes.c_void_p(p))
        for p in self._own:
            self.ctx.lib.vs_peer_free(self.ctx.h, ctypes.c_void_p(p))
        self._opened, self._own = [], []
