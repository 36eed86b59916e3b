"""The sum of the partial d_hidden over a vocabulary-sharded group, over NVLink
peer memory (``sparton_hidden_allreduce`` of the C ABI).

Every rank of the group is one process driving one GPU of the same node. Each
rank allocates three buffers: its fp32 partial d_hidden (written by its own
backward), its reduced-row buffer and its flag words. At set-up the ranks
exchange CUDA IPC handles of those buffers through the process group (once,
for a given capacity) and map each other's; from then on a reduction is four
kernel launches and no host synchronisation, on the instance's own stream at the
device's highest priority (ordered after the calling stream's work so far and
before its later work), so that they are not queued behind kernels the caller
runs beside them:

* only the packed rows (positions before each batch row's extent, counted on
  the device by the forward) cross NVLink, where a library collective would
  move all B*S rows because it needs its count on the host;
* rank q sums rows [T q / N, T (q+1) / N) of every partial in fp32, in rank
  order, and rounds once to hidden's dtype; every rank then copies every row
  from its owner. The result equals an fp32 all-reduce followed by a cast.

The buffers live as long as the process (a module-level cache keyed by the
group, device, hidden size and dtype; the capacity grows with B*S, which every
rank sees alike).
"""
from __future__ import annotations

import ctypes
import socket
from typing import Dict, Tuple

import torch
import torch.distributed as dist

from . import _lib

MAX_PEERS = 8


def _export(t: torch.Tensor) -> Tuple[bytes, int]:
    handle = ctypes.create_string_buffer(64)
    off = ctypes.c_uint64(0)
    _lib.check(_lib.load().sparton_ipc_export(t.data_ptr(), handle, ctypes.byref(off)),
               "sparton_ipc_export")
    return handle.raw, int(off.value)


def _open(handle: bytes, offset: int) -> int:
    ptr = ctypes.c_void_p(0)
    _lib.check(_lib.load().sparton_ipc_open(handle, offset, ctypes.byref(ptr)),
               "sparton_ipc_open")
    return int(ptr.value)


class PeerHiddenReduce:
    """Peer buffers of one rank of a group, and the reduction over them."""

    _cache: Dict[tuple, "PeerHiddenReduce"] = {}

    @classmethod
    def get(cls, group, device: torch.device, rows: int, D: int,
            out_dtype: torch.dtype) -> "PeerHiddenReduce":
        """The instance for (group, device, D, dtype) with room for ``rows``
        rows of d_hidden; every rank must call it with the same arguments (it
        may run a collective to exchange handles)."""
        key = (id(group), device.index, D, out_dtype)
        inst = cls._cache.get(key)
        if inst is None or inst.rows < rows:
            inst = cls(group, device, max(rows, inst.rows * 2 if inst else rows), D, out_dtype)
            cls._cache[key] = inst
        return inst

    @staticmethod
    def usable(group, hidden: torch.Tensor) -> bool:
        """All ranks on this node's GPUs, at most 8 of them, CUDA tensors."""
        if not hidden.is_cuda or group is None:
            return False
        world = dist.get_world_size(group)
        if world < 2 or world > MAX_PEERS:
            return False
        key = ("node", id(group))
        same = PeerHiddenReduce._cache.get(key)
        if same is None:
            hosts = [None] * world
            dist.all_gather_object(hosts, socket.gethostname(), group=group)
            same = len(set(hosts)) == 1
            PeerHiddenReduce._cache[key] = same
        return bool(same)

    def __init__(self, group, device: torch.device, rows: int, D: int, out_dtype: torch.dtype):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.rows, self.D, self.out_dtype = rows, D, out_dtype
        self.device = device
        with torch.cuda.device(device):
            self.part = torch.empty(rows * D, dtype=torch.float32, device=device)
            self.red = torch.empty(rows * D, dtype=out_dtype, device=device)
            self.flags = torch.zeros(2 * MAX_PEERS, dtype=torch.int32, device=device)
            self.status = torch.zeros(1, dtype=torch.int32, device=device)
            torch.cuda.synchronize(device)  # flags are zero before any peer can write them
            mine = (_export(self.part), _export(self.red), _export(self.flags))
            everyone = [None] * self.world
            dist.all_gather_object(everyone, mine, group=group)
            ptrs = []
            for r, bufs in enumerate(everyone):
                if r == self.rank:
                    ptrs.append((self.part.data_ptr(), self.red.data_ptr(),
                                 self.flags.data_ptr()))
                else:
                    ptrs.append(tuple(_open(h, off) for h, off in bufs))
        # The reduction's own stream, at the device's highest priority: its
        # short kernels get SMs ahead of the d_weight blocks queued beside it.
        self.stream = torch.cuda.Stream(device=device, priority=-1)
        arr = ctypes.c_void_p * self.world
        self._parts = arr(*[p[0] for p in ptrs])
        self._reds = arr(*[p[1] for p in ptrs])
        self._flags = arr(*[p[2] for p in ptrs])
        self.epoch = 0

    def partial(self, B: int, S: int) -> torch.Tensor:
        """This rank's fp32 partial d_hidden [B, S, D] (a view of its buffer)."""
        return self.part[: B * S * self.D].view(B, S, self.D)

    def reduce(self, fwd_workspace: torch.Tensor, B: int, S: int, out: torch.Tensor) -> None:
        """out [B, S, D] (hidden's dtype) = sum over the ranks of their partials,
        ordered after the current stream's work and before its later work (the
        kernels run on the reduction's high-priority stream); every rank calls
        it once per backward."""
        self.epoch += 1
        lib = _lib.load()
        cur = torch.cuda.current_stream(self.device)
        self.stream.wait_stream(cur)
        with torch.cuda.device(self.device):
            st = lib.sparton_hidden_allreduce(ctypes.cast(self._parts, ctypes.c_void_p),
                                              ctypes.cast(self._reds, ctypes.c_void_p),
                                              ctypes.cast(self._flags, ctypes.c_void_p),
                                              self.rank,
                                              self.world, self.epoch, fwd_workspace.data_ptr(),
                                              B, S, self.D, out.data_ptr(),
                                              _lib.DTYPE[out.dtype], self.status.data_ptr(),
                                              self.stream.cuda_stream)
        _lib.check(st, "sparton_hidden_allreduce")
        out.record_stream(self.stream)
        fwd_workspace.record_stream(self.stream)
        cur.wait_stream(self.stream)

    def device_status(self) -> int:
        """SPARTON_DEV_TIMEOUT_PEER (0x105) if a wait on a peer gave up (synchronises)."""
        return int(self.status.item())
