"""Peer-memory all-reduce for tensor parallelism (libswq's swq_allreduce_*).

`PeerAllReduce(max_elems, group)` creates this rank's buffer, all-gathers
the CUDA IPC handles over `group` (any torch.distributed backend; the handle
bytes travel as a uint8 tensor on the group's device type) and maps the
peers' buffers.  Calling it on an fp32 tensor sums that tensor across the
group in place on the given stream: one kernel launch, no NCCL, capturable in
a CUDA graph.  Every rank must make the same calls in the same order.
"""
from __future__ import annotations

import ctypes

from .lib import _raise, lib, _ptr, _stream

HANDLE_BYTES = 64


_SHARED: dict = {}


def shared_peer_allreduce(max_elems: int, group=None, device=None) -> "PeerAllReduce":
    """One PeerAllReduce per (group, device), grown when a caller needs more
    elements and never freed while the process runs: buffers that other
    processes have mapped are not released and re-allocated between decoders
    (a new allocation could reuse an address a peer still maps).  Every rank
    must make the same calls in the same order."""
    import torch
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    key = (id(group), dev.index)
    ar = _SHARED.get(key)
    if ar is None or ar.max_elems < max_elems:
        ar = PeerAllReduce(max_elems, group=group, device=dev)
        _SHARED.setdefault(("retired", key), []).append(_SHARED.get(key))
        _SHARED[key] = ar
    return ar


class PeerAllReduce:
    def __init__(self, max_elems: int, group=None, device=None):
        import torch
        import torch.distributed as dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.max_elems = int(max_elems)
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        handle = ctypes.create_string_buffer(HANDLE_BYTES)
        self._ar = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _raise(lib().swq_allreduce_create(self.max_elems, self.rank, self.world, ctypes.byref(self._ar), handle))
        mine = torch.frombuffer(bytearray(handle.raw), dtype=torch.uint8)
        gdev = self.device if dist.get_backend(group) == "nccl" else torch.device("cpu")
        parts = [torch.empty(HANDLE_BYTES, dtype=torch.uint8, device=gdev) for _ in range(self.world)]
        dist.all_gather(parts, mine.to(gdev), group=group)
        allh = b"".join(bytes(p.cpu().numpy().tobytes()) for p in parts)
        with torch.cuda.device(self.device):
            _raise(lib().swq_allreduce_open(self._ar, allh))

    def __call__(self, t, stream=None) -> None:
        import torch
        if t.dtype != torch.float32 or not t.is_contiguous():
            raise ValueError("PeerAllReduce sums contiguous float32 tensors")
        if stream is None:
            stream = torch.cuda.current_stream(self.device)
        _raise(lib().swq_allreduce_sum(self._ar, _ptr(t), t.numel(), _stream(stream)))

    def reset(self, stream=None, group=None) -> None:
        """Bring the group back after a sum timed out (swq_check raised
        SwqError with SWQ_ERR_TIMEOUT on some rank): every rank calls reset()
        between steps.  Waits until no kernel of this rank is in flight
        (every wait is bounded, so this ends), meets the other ranks at a host
        barrier, zeroes this rank's flag words and epoch counters, and meets
        them again so that no rank publishes a new epoch while a peer still
        shows its old flags.  `group` is the process group for the two
        barriers (default: the one the handles were exchanged over); a gloo
        group keeps them off the GPU."""
        import torch
        import torch.distributed as dist
        g = self.group if group is None else group
        torch.cuda.synchronize(self.device)
        dist.barrier(group=g)
        if stream is None:
            stream = torch.cuda.current_stream(self.device)
        with torch.cuda.device(self.device):
            _raise(lib().swq_allreduce_reset(self._ar, _stream(stream)))
        dist.barrier(group=g)

    def close(self) -> None:
        if self._ar:
            lib().swq_allreduce_destroy(self._ar)
            self._ar = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 -- interpreter shutdown
            pass
