"""Device buffers mapped into every rank of a process group (CUDA IPC over NVLink).

Each rank allocates one buffer with ``wfattn_peer_alloc`` (plain ``cudaMalloc``
memory), the 64-byte handles are exchanged with ``all_gather_object`` over the
process group, and every rank maps the other ranks' buffers with
``wfattn_peer_open``.  A mapped buffer is an ordinary peer mapping: kernels on
this GPU load from and store to it over NVLink.  No multicast object is made.

Setup and ``close`` are collective: every rank of the group calls them in the
same order.  A rank whose allocation or mapping fails still takes every
collective step, and then all ranks raise ``PeerSetupError`` together after
releasing what they set up, so a caller can fall back on every rank at once.
"""

from __future__ import annotations

import contextlib
import ctypes
import math

import torch
import torch.distributed as dist

from . import _lib

_TYPESTR = {1: "|u1", 2: "<i2", 4: "<i4", 8: "<i8"}


class PeerSetupError(RuntimeError):
    """Some rank could not allocate or map its peer buffers (raised on every rank)."""


class _DeviceArray:
    """A raw device allocation seen by torch through ``__cuda_array_interface__``."""

    def __init__(self, ptr: int, shape: tuple[int, ...], itemsize: int) -> None:
        self.__cuda_array_interface__ = {
            "shape": tuple(shape), "typestr": _TYPESTR[itemsize], "data": (ptr, False),
            "strides": None, "version": 2}


class PeerBuffer:
    """A contiguous ``shape``/``dtype`` buffer on ``device``, mapped on every rank.

    ``tensor`` is this rank's buffer as a torch tensor; ``ptrs[r]`` is the
    device address of rank r's buffer as mapped on this GPU (``ptrs[rank]`` is
    this rank's own).  The memory lives until ``close()`` (collective) or the
    process exits.
    """

    def __init__(self, shape: tuple[int, ...], dtype: torch.dtype, device: torch.device,
                 group=None) -> None:
        self.group = group
        self.device = torch.device(device)
        self.index = self.device.index if self.device.index is not None else 0
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.shape = tuple(int(s) for s in shape)
        itemsize = torch.empty((), dtype=dtype).element_size()
        nbytes = math.prod(self.shape) * itemsize
        self._own: int | None = None
        self._opened: list[int] = []
        self.ptrs: list[int] = []
        handle = _lib.PeerHandle()
        err = ""
        ptr = ctypes.c_void_p()
        lib = None
        try:  # a failure here still takes part in the collectives below
            lib = _lib.load()
            _lib.check(lib.wfattn_peer_alloc(nbytes, self.index, ctypes.byref(ptr),
                                             ctypes.byref(handle)))
            self._own = ptr.value
        except _lib.WfattnError as e:
            err = str(e)
        with self._on_device():
            handles: list = [None] * self.world
            dist.all_gather_object(handles, None if err else bytes(handle.bytes), group=group)
            if not err and any(h is None for h in handles):
                err = "another rank could not allocate its buffer"
            if not err:
                try:
                    for r, hb in enumerate(handles):
                        if r == self.rank:
                            self.ptrs.append(self._own)
                            continue
                        other = _lib.PeerHandle.from_buffer_copy(hb)
                        mapped = ctypes.c_void_p()
                        _lib.check(lib.wfattn_peer_open(ctypes.byref(other), self.index,
                                                        ctypes.byref(mapped)))
                        self._opened.append(mapped.value)
                        self.ptrs.append(mapped.value)
                except _lib.WfattnError as e:
                    err = str(e)
            errors: list = [None] * self.world
            dist.all_gather_object(errors, err, group=group)
        bad = [(r, e) for r, e in enumerate(errors) if e]
        if bad:
            if lib is not None:
                self._release(lib)
            raise PeerSetupError("; ".join(f"rank {r}: {e}" for r, e in bad))
        self.tensor = torch.as_tensor(_DeviceArray(self._own, self.shape, itemsize),
                                      device=self.device).view(dtype)

    def _on_device(self):
        # the NCCL object collectives stage through the current device
        return torch.cuda.device(self.index) if torch.cuda.is_available() \
            else contextlib.nullcontext()

    def _release(self, lib) -> None:
        for p in self._opened:
            lib.wfattn_peer_close(p, self.index)
        self._opened = []
        if self._own is not None:
            lib.wfattn_peer_free(self._own, self.index)
            self._own = None
        self.ptrs = []

    def _barrier(self) -> None:
        with self._on_device():
            torch.cuda.synchronize()
            dist.barrier(group=self.group)
            torch.cuda.synchronize()

    def close(self) -> None:
        """Collective: waits until no rank's work touches the buffers, unmaps the other
        ranks' buffers, waits until every rank has done so, then frees this rank's."""
        if self._own is None:
            return
        lib = _lib.load()
        self._barrier()
        for p in self._opened:
            _lib.check(lib.wfattn_peer_close(p, self.index))
        self._opened = []
        self._barrier()
        self.tensor = None
        _lib.check(lib.wfattn_peer_free(self._own, self.index))
        self._own = None
        self.ptrs = []
