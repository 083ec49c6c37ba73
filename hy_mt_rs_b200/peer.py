"""Tensor-parallel all-reduce (hyq_peer_allreduce) and the expert-parallel
row exchange (hyq_peer_exchange) over NVLink peer memory.

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


class PeerExchange:
    """Expert-parallel exchange over NVLink peer memory (hyq_peer_exchange):
    each rank pushes its block for rank q -- `rows` rows of `row_floats`
    floats, of which the first valid[q] are sent (plus, with last_row, the
    block's last row) -- straight into q's region, slot = this rank.  After
    exchange(), `recv(rows, row_floats)` views this rank's region as
    [world * slot_rows, row_floats] rows: source s's block starts at row
    s * slot_rows.  One region per rank, sized for `slot_floats` floats per
    source; every rank must make the same calls in the same order."""

    def __init__(self, slot_floats, group=None, device=None):
        import torch.distributed as dist

        self.slot = int(slot_floats)
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.data_bytes = 4 * self.world * self.slot
        region = C.c_void_p()
        handle = (C.c_char * 64)()
        check(lib.hyq_peer_alloc(self.data_bytes, C.byref(region), handle))
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
        self._data = torch.as_tensor(_DeviceArray(region.value + PEER_DATA_OFFSET, self.world * self.slot),
                                     device=self.device)
        dist.barrier(group)

    def exchange(self, send, rows, valid=None, last_row=False):
        """send: float32 [world * rows, row_floats] (block q for rank q);
        valid: int32 [world] rows of each block to send (None: all).
        Ordered on the current stream."""
        if send.dtype != torch.float32 or not send.is_contiguous() or send.dim() != 2:
            raise ValueError("exchange: send must be a contiguous float32 matrix")
        if send.shape[0] != self.world * rows:
            raise ValueError("exchange: send must hold world * rows rows")
        if valid is not None and (valid.dtype != torch.int32 or valid.numel() != self.world or
                                  not valid.is_contiguous()):
            raise ValueError("exchange: valid must be int32 [world]")
        check(lib.hyq_peer_exchange(self._regions, self.rank, self.world, self.data_bytes,
                                    C.c_void_p(send.data_ptr()), rows, send.shape[1],
                                    C.c_void_p(valid.data_ptr()) if valid is not None else None,
                                    1 if last_row else 0, self.slot,
                                    C.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)))

    def recv(self, slot_rows, row_floats):
        """This rank's region as [world * slot_rows, row_floats] rows (a view)."""
        if slot_rows * row_floats != self.slot:
            raise ValueError("recv: slot_rows * row_floats must equal the slot size")
        return self._data.view(self.world * slot_rows, row_floats)

    def close(self):
        import torch.distributed as dist

        torch.cuda.synchronize(self.device)
        dist.barrier(self.group)
        for p in self._opened:
            check(lib.hyq_peer_close(p))
        self._opened = []
        dist.barrier(self.group)
        if self._own is not None:
            self._data = None
            check(lib.hyq_peer_free(self._own))
            self._own = None
