"""Multi-GPU reduce-sum fused with its all-reduce (opl_team_* in the C-ABI).

One ``ReduceTeam`` per rank (one process per GPU, ``torch.distributed``
initialised): construction creates this GPU's team buffer, exchanges the CUDA
IPC handles of all ranks with ``all_gather_object`` and opens the peers'
buffers.  ``reduce_sum_into(x, out)`` then sums this rank's chunk ``x`` and
combines the partials of all ranks over NVLink inside the same launch
sequence; every rank receives the same total.  All ranks must call it the
same number of times, in the same order.
"""
from __future__ import annotations

import ctypes


class ReduceTeam:
    HANDLE_BYTES = 64

    def __init__(self, rank: int, world: int, group=None):
        import torch.distributed as dist

        from . import capi, check

        self._lib = capi()
        self.rank, self.world = rank, world
        self._team = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(self.HANDLE_BYTES)
        check("team_create", self._lib.opl_team_create(rank, world, ctypes.byref(self._team),
                                                       handle))
        handles = [None] * world
        dist.all_gather_object(handles, handle.raw, group=group)
        check("team_connect", self._lib.opl_team_connect(self._team, b"".join(handles)))
        dist.barrier(group=group)

    def reduce_sum_into(self, x, out, stream=None) -> None:
        import torch

        from . import check

        s = stream if stream is not None else torch.cuda.current_stream(x.device)
        check("team_reduce_sum", self._lib.opl_team_reduce_sum_f32(
            self._team, x.data_ptr(), out.data_ptr(), x.numel(), s.cuda_stream))

    def launch(self, x, out, stream_handle) -> int:
        """Raw C-ABI call on a given stream handle (for graph capture)."""
        return self._lib.opl_team_reduce_sum_f32(self._team, x.data_ptr(), out.data_ptr(),
                                                 x.numel(), stream_handle)

    def close(self) -> None:
        if self._team:
            self._lib.opl_team_destroy(self._team)
            self._team = ctypes.c_void_p()
