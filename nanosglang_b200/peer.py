"""One-shot all-reduce over NVLink peer memory (libnsq's nsq_peer_allreduce)
for the small row-parallel outputs of tensor-parallel decode.

The reference reduces every row-parallel output with ``dist.all_reduce``
(nano_sglang/distributed/tensor_parallel.py:134-140). For decode-sized
outputs (a Llama-3-8B layer at 64 tokens: [64, 4096] bf16 = 512 KB, twice per
layer) NCCL's per-call latency dominates; this path stores every rank's
partial straight into every other rank's workspace over NVLink and sums
locally, in rank order, so all ranks hold identical results.
"""

from __future__ import annotations

import ctypes
from typing import Optional

import torch
import torch.distributed as dist

from . import _lib

_CODES = {torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_F16, torch.float32: _lib.DTYPE_F32}


class PeerAllReduce:
    """Set up once per process group (collective: every rank must construct
    it); then ``reduce_(t)`` sums ``t`` over the ranks in place and returns
    True, or returns False without touching ``t`` when it does not apply
    (size above ``max_bytes``, dtype, alignment), so the caller falls back to
    ``dist.all_reduce``."""

    def __init__(self, max_bytes: int = 4 << 20, group=None, device: Optional[torch.device] = None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.max_bytes = (int(max_bytes) + 15) // 16 * 16
        lib = _lib.load()
        size = lib.nsq_peer_workspace_size(self.world, self.max_bytes)
        if size == 0:
            raise ValueError(f"peer all-reduce supports 1..8 ranks (got {self.world})")
        if device is not None:
            torch.cuda.set_device(device)
        ws = ctypes.c_void_p()
        _lib.check(lib.nsq_peer_workspace_alloc(size, ctypes.byref(ws)), "nsq_peer_workspace_alloc")
        self._own = ws.value
        handle = ctypes.create_string_buffer(64)
        _lib.check(lib.nsq_ipc_handle(self._own, handle), "nsq_ipc_handle")
        handles = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        ptrs, self._opened = [], []
        for q, h in enumerate(handles):
            if q == self.rank:
                ptrs.append(self._own)
                continue
            p = ctypes.c_void_p()
            _lib.check(lib.nsq_ipc_open(ctypes.create_string_buffer(h, 64), ctypes.byref(p)), "nsq_ipc_open")
            ptrs.append(p.value)
            self._opened.append(p.value)
        self._ptrs = (ctypes.c_void_p * self.world)(*ptrs)
        dist.barrier(group=group)  # every rank mapped every workspace before the first call

    def reduce_(self, t: torch.Tensor) -> bool:
        if t.dtype not in _CODES or not t.is_cuda or not t.is_contiguous():
            return False
        nbytes = t.numel() * t.element_size()
        if nbytes > self.max_bytes or nbytes % 16 != 0 or t.data_ptr() % 16 != 0:
            return False
        rc = _lib.load().nsq_peer_allreduce(self._ptrs, self.rank, self.world, self.max_bytes, t.data_ptr(),
                                            t.data_ptr(), t.numel(), _CODES[t.dtype],
                                            torch.cuda.current_stream(t.device).cuda_stream)
        _lib.check(rc, "nsq_peer_allreduce")
        return True

    def close(self):
        """Unmap the peers' workspaces and free this rank's (collective)."""
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        lib = _lib.load()
        for p in self._opened:
            lib.nsq_ipc_close(p)
        self._opened = []
        dist.barrier(group=self.group)
        if self._own:
            lib.nsq_peer_workspace_free(self._own)
            self._own = None
