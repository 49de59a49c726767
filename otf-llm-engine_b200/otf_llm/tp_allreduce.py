"""Tensor-parallel peer all-reduce over NVLink, fused into the 2-bit GEMV launches.

One process per GPU.  Each rank allocates a receive region in its own HBM (two buffers
of world x max_elems fp32 slots and their arrival counters) and maps every peer's region
through CUDA IPC; the handles travel over the process group once, at construction.

The decoder stack uses it without any all-reduce launch of its own:

* a row-parallel o_proj / down_proj runs with ``ar_mode=OTF_AR_PRODUCE``: its finishing
  CTAs store the fp32 rows straight into every rank's buffer over NVLink and bump each
  rank's arrival counter;
* the next grouped launch (RMSNorm + gate/up, or RMSNorm + the next layer's q/k/v) runs
  with ``ar_mode=OTF_AR_CONSUME``: while staging its activation it waits for all ranks'
  rows, sums them in rank order (bit-identical on every rank) and writes the fp16 sum
  once (``ar_out``) for the residual path;
* the last exchange of a step ends in ``finish`` (wait, sum, write).

Consecutive exchanges alternate buffers 0 and 1.  Every wait is bounded: a peer that
never delivers raises the library's device error flag instead of hanging the GPU.
This replaces the NCCL all_reduce after o_proj / down_proj (one 8-16 KB collective per
projection at batch 1).
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch
import torch.distributed as dist

from . import _native


class PeerAllReduce:
    """Receive buffers of this rank, mapped by every rank of ``group``."""

    def __init__(self, max_elems: int, group=None, device: Optional[torch.device] = None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.max_elems = int(max_elems)
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        L = _native.lib()
        handle = ctypes.create_string_buffer(_native.OTF_AR_HANDLE_BYTES)
        ptr = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _native._check(L.otf_ar_create(self.rank, self.world, self.max_elems, handle, ctypes.byref(ptr)),
                           "otf_ar_create")
        self.handle = ptr.value
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle.raw), group=group)
        blob = b"".join(handles)
        with torch.cuda.device(self.device):
            _native._check(L.otf_ar_open(ctypes.c_void_p(self.handle), blob), "otf_ar_open")
        dist.barrier(group=group)        # every rank has mapped every region before first use
        self._next = 0

    # -- buffers ---------------------------------------------------------------------------
    def next_buffer(self) -> int:
        """The buffer of the next exchange (0, 1, 0, ...)."""
        b = self._next
        self._next ^= 1
        return b

    # -- standalone exchange ---------------------------------------------------------------
    def push(self, x: torch.Tensor, buf: int) -> None:
        """This rank's fp16 partial x [n] into buffer ``buf`` of every rank."""
        _native._need_cuda(x, "x")
        if x.dtype != torch.float16 or not x.is_contiguous():
            raise ValueError("x must be contiguous fp16")
        with torch.cuda.device(x.device):
            _native._check(_native.lib().otf_ar_push(ctypes.c_void_p(self.handle), buf, _native._ptr(x), x.numel(),
                                                     _native._stream(x.device)), "otf_ar_push")

    def finish(self, out: torch.Tensor, buf: int) -> torch.Tensor:
        """Wait for every rank's rows of buffer ``buf`` and write their fp16 sum to ``out``."""
        _native._need_cuda(out, "out")
        if out.dtype != torch.float16 or not out.is_contiguous():
            raise ValueError("out must be contiguous fp16")
        with torch.cuda.device(out.device):
            _native._check(_native.lib().otf_ar_finish(ctypes.c_void_p(self.handle), buf, _native._ptr(out),
                                                       out.numel(), _native._stream(out.device)), "otf_ar_finish")
        return out

    def all_reduce(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """fp16 sum over ranks of x (one push, one finish)."""
        b = self.next_buffer()
        self.push(x.reshape(-1), b)
        if out is None:
            out = torch.empty_like(x)
        self.finish(out.view(-1), b)
        return out

    def close(self) -> None:
        if self.handle:
            with torch.cuda.device(self.device):
                _native.lib().otf_ar_destroy(ctypes.c_void_p(self.handle))
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
