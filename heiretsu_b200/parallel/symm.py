"""Symmetric peer-memory buffers over NVLink (CUDA IPC) for the fused collectives.

A ``SymmetricBuffer`` is one device allocation of the same size on every
rank of a process group; each rank holds device pointers to all the others'
copies (``ptrs``), exchanged once over torch.distributed. Kernels in
heiretsu_b200/csrc/comm.cu read and write peers' copies directly with loads
and stores over NVLink. Each buffer comes with a signal pad (per-block,
epoch-tagged flags) and a local epoch counter used by the kernels' bounded
barriers.
"""
from __future__ import annotations

import os
from typing import List, Optional

import torch
import torch.distributed as dist

from ..ops._C import load

SIGNAL_BYTES = 8 * 1024 * 4  # uint32 [8 ranks][1024 blocks]


class CommTimeoutError(RuntimeError):
    """A peer did not arrive at a device-side barrier within the bounded wait."""


def _exchange(group, local_bytes: bytes) -> List[bytes]:
    world = dist.get_world_size(group)
    out: List[Optional[bytes]] = [None] * world
    dist.all_gather_object(out, local_bytes, group=group)
    return out  # type: ignore[return-value]


class SymmetricBuffer:
    def __init__(self, group, nbytes: int, device: torch.device, local_ptr: Optional[int] = None):
        """Allocate (or, with ``local_ptr``, share an existing raw allocation of
        this rank) and map every peer's copy in ``group``."""
        ext = load()
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > 8:
            raise ValueError("symmetric buffers support at most 8 ranks per group (one NVSwitch node)")
        per_node = int(os.environ.get("LOCAL_WORLD_SIZE", dist.get_world_size()) or dist.get_world_size())
        if len({r // per_node for r in dist.get_process_group_ranks(group)}) > 1:
            raise ValueError("symmetric buffers map peers through CUDA IPC, which needs every rank of the group "
                             "on one node; this group spans nodes")
        self.device = device
        self.nbytes = nbytes
        with torch.cuda.device(device):
            self.local_ptr = ext.raw_malloc(nbytes) if local_ptr is None else local_ptr
            self.signal_ptr = ext.raw_malloc(SIGNAL_BYTES)
            handles = _exchange(group, ext.ipc_handle(self.local_ptr))
            sig_handles = _exchange(group, ext.ipc_handle(self.signal_ptr))
            self.ptrs = [self.local_ptr if i == self.rank else ext.ipc_open(h) for i, h in enumerate(handles)]
            self.signal_ptrs = [self.signal_ptr if i == self.rank else ext.ipc_open(h)
                                for i, h in enumerate(sig_handles)]
            self.counter = torch.zeros(1024, dtype=torch.int32, device=device)
        dist.barrier(group=group)

    def tensor(self, dtype: torch.dtype, numel: Optional[int] = None, offset_bytes: int = 0) -> torch.Tensor:
        """This rank's copy viewed as a 1-D tensor (no copy)."""
        esz = torch.empty((), dtype=dtype).element_size()
        if numel is None:
            numel = (self.nbytes - offset_bytes) // esz
        return load().tensor_from_ptr(self.local_ptr + offset_bytes, numel, dtype, self.device.index)

    def barrier(self) -> None:
        """Device-side barrier of the group (bounded wait), ordered on the current stream."""
        load().group_barrier(self.ptrs, self.signal_ptrs, self.rank, self.counter)

    def sum_range(self, start_elem: int, n_elem: int, scale: float = 1.0, threads: int = 512, blocks: int = 0) -> None:
        """In place over the group: fp32 elements [start, start+n) <- scale * sum over ranks (NVLink, one kernel).

        ``threads`` = 64 gives a footprint small enough to run beside compute kernels;
        ``blocks`` > 0 caps the grid (0: one CTA per SM). Every rank must pass the same values."""
        if self.world == 1 or n_elem == 0:
            return
        if start_elem % 4 or n_elem % 4:
            raise ValueError(f"sum_range: start ({start_elem}) and count ({n_elem}) must be multiples of 4 "
                             "(the kernel moves float4 vectors)")
        off = start_elem * 4
        load().dp_allreduce([p + off for p in self.ptrs], self.signal_ptrs, self.rank, n_elem, scale, self.counter,
                            threads, blocks)


def check_comm_status(device: int) -> None:
    code = int(load().read_and_clear_status(device))
    if code & 0xFF == 2:
        raise CommTimeoutError(f"device {device}: peer did not arrive (site {code >> 8})")
    if code:
        raise RuntimeError(f"device {device}: kernel status {code:#x}")
