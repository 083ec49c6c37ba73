"""Tensor-parallel all-reduce over NVLink peer memory (hyq_peer_allreduce).

Each rank allocates one peer region through the library, the CUDA IPC
handles are exchanged over a torch.distributed group (any backend: the
group only carries the 64-byte handles and a barrier), and every rank maps
the others' regions.  A row-parallel product writes its partial output into
`partial`; `allreduce(out)` leaves the sum over all ranks in `out`, in rank
order, on every rank.  No multicast object is involved.
"""
import ctypes as C

import torch

from ._native import check, lib

PEER_DATA_OFFSET = 1024  # HYQ_PEER_DATA_OFFSET


class _DeviceArray:
    """__cuda_array_interface__ over a raw device pointer (zero-copy view)."""

    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 3}


class PeerAllReduce:
    def __init__(self, n, group=None, device=None):
        import torch.distributed as dist

        self.n = int(n)
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        region = C.c_void_p()
        handle = (C.c_char * 64)()
        check(lib.hyq_peer_alloc(4 * self.n, C.byref(region), handle))
        self._own = region
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self._opened = []
        ptrs = []
        for q, h in enumerate(handles):
            if q == self.rank:
                ptrs.append(region.value)
                continue
            p = C.c_void_p()
            check(lib.hyq_peer_open((C.c_char * 64).from_buffer_copy(h), C.byref(p)))
            self._opened.append(p)
            ptrs.append(p.value)
        self._regions = (C.c_uint64 * self.world)(*ptrs)
        self.partial = torch.as_tensor(_DeviceArray(region.value + PEER_DATA_OFFSET, self.n), device=self.device)
        dist.barrier(group)

    def allreduce(self, out):
        """out (float32, n, on this rank's device) = sum of every rank's
        `partial`.  Ordered on the current stream; every rank must call."""
        if out.numel() != self.n or out.dtype != torch.float32:
            raise ValueError("allreduce: out must be float32 with n elements")
        check(lib.hyq_peer_allreduce(self._regions, self.rank, self.world, self.n, C.c_void_p(out.data_ptr()),
                                     C.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)))
        return out

    def close(self):
        import torch.distributed as dist

        torch.cuda.synchronize(self.device)
        dist.barrier(self.group)
        for p in self._opened:
            check(lib.hyq_peer_close(p))
        self._opened = []
        dist.barrier(self.group)
        if self._own is not None:
            self.partial = None
            check(lib.hyq_peer_free(self._own))
            self._own = None
