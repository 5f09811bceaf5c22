"""Mixture-of-experts FFN on the device (libswq's swq_moe_* and swq_ep_*).

The reference has no MoE forward (its FFN is dense, src/model.h:520-528; the
GGUF expert tensor names `ffn_gate_inp`, `ffn_{gate,up,down}_exps` and
`ffn_*_shexp` appear only at src/hf_loader.h:474-493).  `MoEFFN` runs the
MoE FFN of the MoE decoder shape with every step in libswq kernels and no
host synchronisation:

  router GEMV (fp32) + top-k + softmax over the k      swq_moe_router
  rows to the ranks that own their experts             swq_ep_dispatch
  gate|up of every routed row, grouped by expert        swq_grouped_matmul_stacked
  silu(gate) * up                                       swq_silu_mul
  down, grouped by expert                               swq_grouped_matmul_stacked
  weighted sum back in token order (+ shared expert)    swq_ep_combine

`ExpertParallel` owns the peer-memory buffers of the dispatch and combine
(one per rank of a process group, mapped by every other rank over CUDA IPC);
with one rank it runs on one GPU without peers.  Every rank makes the same
calls in the same order.
"""
from __future__ import annotations

import ctypes
import math
from typing import Sequence

import numpy as np

from .lib import _ptr, _raise, _stream, grouped_matmul, grouped_matmul_stacked, lib, moe_router, silu_mul

HANDLE_BYTES = 64


def _group_rank_world(group):
    """(rank, size) of `group`; None is this process alone, whatever process
    groups exist."""
    if group is None:
        return 0, 1
    import torch.distributed as dist
    return dist.get_rank(group), dist.get_world_size(group)


class ExpertParallel:
    """swq_ep_* of this rank: at most max_tokens tokens per call, top_k slots
    each, n_experts split evenly over `group` (None: this process alone),
    hidden size H."""

    def __init__(self, max_tokens: int, top_k: int, n_experts: int, hidden: int, group=None, device=None):
        import torch
        self.group = group
        self.rank, self.world = _group_rank_world(group)
        self.max_tokens, self.k, self.E, self.H = int(max_tokens), int(top_k), int(n_experts), int(hidden)
        self.el = self.E // self.world
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        handle = ctypes.create_string_buffer(HANDLE_BYTES)
        self._ep = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _raise(lib().swq_ep_create(self.max_tokens, self.k, self.E, self.H, self.rank, self.world,
                                       ctypes.byref(self._ep), handle))
        if self.world > 1:
            import torch.distributed as dist
            mine = torch.frombuffer(bytearray(handle.raw), dtype=torch.uint8)
            gdev = self.device if dist.get_backend(group) == "nccl" else torch.device("cpu")
            parts = [torch.empty(HANDLE_BYTES, dtype=torch.uint8, device=gdev) for _ in range(self.world)]
            dist.all_gather(parts, mine.to(gdev), group=group)
            allh = b"".join(bytes(p.cpu().numpy().tobytes()) for p in parts)
            with torch.cuda.device(self.device):
                _raise(lib().swq_ep_open(self._ep, allh))
        x, off, cap = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_int()
        _raise(lib().swq_ep_received(self._ep, ctypes.byref(x), ctypes.byref(off), ctypes.byref(cap)))
        self.recv_ptr, self.offsets_ptr, self.capacity = int(x.value), int(off.value), int(cap.value)

    def dispatch(self, X, ids, T: int, stream=None) -> None:
        """Send the T token rows of X [T, H] to the ranks owning their experts
        (ids [T, k] int32, global expert ids)."""
        _raise(lib().swq_ep_dispatch(self._ep, _ptr(X), _ptr(ids), int(T), _stream(stream)))

    def combine(self, Y_recv, w, Y, accumulate: bool = False, stream=None) -> None:
        """Y [T, H] (+)= sum_j w[t, j] * expert output of pair (t, j); Y_recv
        holds the outputs of the received rows (capacity x H)."""
        _raise(lib().swq_ep_combine(self._ep, _ptr(Y_recv), _ptr(w), _ptr(Y), 1 if accumulate else 0,
                                    _stream(stream)))

    def reset(self, stream=None) -> None:
        """After a timed-out call: every rank calls reset() between steps
        (device idle, barrier, zero this rank's flags, barrier)."""
        import torch
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            _raise(lib().swq_ep_reset(self._ep, _stream(stream)))
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier(group=self.group)

    def close(self) -> None:
        if self._ep:
            lib().swq_ep_destroy(self._ep)
            self._ep = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 -- interpreter shutdown
            pass


def _to_dev(a, device):
    import torch
    if isinstance(a, torch.Tensor):
        return a.reshape(-1).to(device=device, dtype=torch.uint8).contiguous()
    return torch.from_numpy(np.ascontiguousarray(a).reshape(-1).view(np.uint8)).to(device)


class MoEFFN:
    """SwiGLU mixture-of-experts FFN, experts sharded over `group` (None: all
    experts in this process).

    experts: n_experts triples (gate [F x H], up [F x H], down [H x F]) of GGUF
      block arrays (numpy or torch uint8); only this rank's are read (the
      others may be None).  types: GGML types of gate, up, down.
    router_w: [n_experts, H] fp32 (replicated on every rank).
    shared: optional (gate, up, down) of a shared expert of intermediate size
      shared_F (types `shared_types`), computed on every rank for its own
      tokens and added to the routed sum.
    max_tokens: the most tokens one call takes (buffers are sized for it).
    scratch_from: another MoEFFN of the same shape whose dispatch buffers and
      activations this one reuses (the layers of a decoder run one at a time).
    Call: y = ffn(x [T, H] fp32 device tensor) -> [T, H]; no host sync."""

    def __init__(self, experts: Sequence | None, types: tuple[int, int, int], H: int, F: int, router_w, top_k: int,
                 max_tokens: int, group=None, device=None, shared=None, shared_types=None, shared_F: int = 0,
                 scratch_from: "MoEFFN | None" = None, n_experts: int = 0, device_blocks=None):
        import torch
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.rank, self.world = _group_rank_world(group)
        self.E = len(experts) if experts is not None else int(n_experts)
        self.H, self.F, self.k, self.types = int(H), int(F), int(top_k), tuple(types)
        if self.E % self.world:
            raise ValueError(f"{self.E} experts do not split over {self.world} ranks")
        self.el = self.E // self.world
        self.e0 = self.rank * self.el
        self.max_tokens = int(max_tokens)
        dev = self.device
        if device_blocks is not None:
            self._weights_from_device(*device_blocks)
        else:
            self._weights_from_experts(experts[self.e0:self.e0 + self.el])
        rw = router_w if isinstance(router_w, torch.Tensor) else torch.from_numpy(np.asarray(router_w, np.float32))
        self.router_w = rw.to(device=dev, dtype=torch.float32).contiguous()
        self.shared = None
        if shared is not None:
            st = tuple(shared_types or types)
            self.shared_types, self.shared_F = st, int(shared_F or F)
            self.shared = True
            sg, su, sd = (_to_dev(a, dev) for a in shared)
            self.sh_fused = st[0] == st[1]
            if self.sh_fused:
                self.sh_gu_w = torch.cat([sg, su])
            else:
                self.sh_g, self.sh_u = sg, su
            self.sh_d = sd
        self._alloc(scratch_from, group)

    def _weights_from_experts(self, own) -> None:
        """Stack this rank's experts into one tensor per projection (the GGUF
        expert-tensor layout) when every expert matrix keeps a 16-byte
        boundary there; else one allocation per expert with a pointer table."""
        import torch
        from .synth import row_bytes
        dev = self.device
        self.fused = self.types[0] == self.types[1]
        gu_sz = (2 if self.fused else 1) * self.F * row_bytes(self.types[0], self.H)
        d_sz = self.H * row_bytes(self.types[2], self.F)
        u_sz = self.F * row_bytes(self.types[1], self.H)
        self.stacked = gu_sz % 16 == 0 and d_sz % 16 == 0 and (self.fused or u_sz % 16 == 0)
        if self.fused:  # gate rows then up rows: one [2F x H] matrix per expert
            gu = [torch.cat([_to_dev(g, dev), _to_dev(u, dev)]) for g, u, _ in own]
            parts = {"gu": gu}
        else:
            parts = {"g": [_to_dev(g, dev) for g, _, _ in own], "u": [_to_dev(u, dev) for _, u, _ in own]}
        parts["d"] = [_to_dev(d, dev) for _, _, d in own]
        for name, mats in parts.items():
            if self.stacked:
                setattr(self, name + "_all", torch.cat(mats))
            else:
                setattr(self, name, mats)
                setattr(self, name + "_tab", torch.tensor([t.data_ptr() for t in mats], dtype=torch.int64,
                                                          device=dev))

    def _weights_from_device(self, gu_all, d_all) -> None:
        """gu_all: this rank's experts' fused gate|up matrices back to back
        (el x [2F x H] GGUF rows, one device uint8 tensor); d_all: their down
        matrices (el x [H x F])."""
        from .synth import row_bytes
        if self.types[0] != self.types[1]:
            raise ValueError("device blocks hold fused gate|up matrices: gate and up need one type")
        self.fused, self.stacked = True, True
        gu_sz = 2 * self.F * row_bytes(self.types[0], self.H)
        d_sz = self.H * row_bytes(self.types[2], self.F)
        if gu_all.numel() != self.el * gu_sz or d_all.numel() != self.el * d_sz:
            raise ValueError("device blocks do not hold el experts of this shape")
        if gu_sz % 16 or d_sz % 16:
            raise ValueError("stacked expert matrices must keep 16-byte boundaries")
        self.gu_all, self.d_all = gu_all, d_all

    def _gmm(self, name: str, type_id: int, offs, X, Y, rows: int, N: int, K: int, mean: int, stream) -> None:
        if self.stacked:
            grouped_matmul_stacked(type_id, getattr(self, name + "_all"), offs, X, Y, self.el, rows, N, K, mean,
                                   stream=stream)
        else:
            grouped_matmul(type_id, getattr(self, name + "_tab"), offs, X, Y, self.el, rows, N, K, mean,
                           stream=stream)

    def _alloc(self, other: "MoEFFN | None", group) -> None:
        import torch
        dev = self.device
        Fs = self.shared_F if self.shared else 0
        if other is not None:
            same = (other.E, other.H, other.F, other.k, other.max_tokens, other.world, Fs) == \
                   (self.E, self.H, self.F, self.k, self.max_tokens, self.world, other.shared_F if other.shared else 0)
            if not same:
                raise ValueError("scratch_from needs a MoEFFN of the same shape")
            for name in ("ep", "logits", "ids", "w", "gu_out", "h", "y_recv", "y", "sh_gu", "sh_h"):
                setattr(self, name, getattr(other, name, None))
            return
        self.ep = ExpertParallel(self.max_tokens, self.k, self.E, self.H, group=group, device=dev)
        cap = self.ep.capacity
        self.logits = torch.empty(self.max_tokens, self.E, device=dev)
        self.ids = torch.zeros(self.max_tokens, self.k, dtype=torch.int32, device=dev)
        self.w = torch.zeros(self.max_tokens, self.k, device=dev)
        self.gu_out = torch.empty(cap, 2 * self.F, device=dev)
        self.h = torch.empty(cap, self.F, device=dev)
        self.y_recv = torch.empty(cap, self.H, device=dev)
        self.y = torch.empty(self.max_tokens, self.H, device=dev)
        self.sh_gu = torch.empty(self.max_tokens, 2 * Fs, device=dev) if Fs else None
        self.sh_h = torch.empty(self.max_tokens, Fs, device=dev) if Fs else None

    def route(self, x, T: int, stream=None) -> None:
        moe_router(self.router_w, x, T, self.E, self.H, self.k, self.logits, self.ids, self.w, stream=stream)

    def _shared_ffn(self, x, T: int, y, stream) -> None:
        """y[:T] = the shared expert's SwiGLU FFN of x (written, not added)."""
        from .lib import ACT_SWIGLU, gemm, gemm_act
        Fs, H = self.shared_F, self.H
        if self.sh_fused:
            gemm(self.shared_types[0], self.sh_gu_w, x, self.sh_gu, T, 2 * Fs, H, stream=stream)
            gemm_act(self.shared_types[2], self.sh_d, self.sh_gu, y, T, H, Fs, kind=ACT_SWIGLU, ld=2 * Fs,
                     stream=stream)
        else:
            gemm(self.shared_types[0], self.sh_g, x, self.sh_h, T, Fs, H, stream=stream)
            gemm(self.shared_types[1], self.sh_u, x, self.sh_gu, T, Fs, H, stream=stream)
            silu_mul(self.sh_h, self.sh_h, self.sh_gu, Fs, rows=T, ld=Fs, stream=stream)
            gemm(self.shared_types[2], self.sh_d, self.sh_h, y, T, H, Fs, stream=stream)

    def experts(self, T: int, peer_tokens: int | None = None, stream=None) -> None:
        """The grouped expert FFN on the rows this rank received (after
        ep.dispatch) into y_recv.  peer_tokens: the most tokens any rank
        dispatched in this call (default max_tokens), bounding the rows."""
        F, H = self.F, self.H
        mean = max(1, math.ceil(T * self.k / self.E))
        pt = self.max_tokens if peer_tokens is None else int(peer_tokens)
        rows = min(self.ep.capacity, self.world * pt * self.k)
        xr, offs = self.ep.recv_ptr, self.ep.offsets_ptr
        if self.fused:
            self._gmm("gu", self.types[0], offs, xr, self.gu_out, rows, 2 * F, H, mean, stream)
            silu_mul(self.h, self.gu_out, self.gu_out.data_ptr() + 4 * F, F, rows=rows, ld=2 * F, stream=stream)
        else:
            self._gmm("g", self.types[0], offs, xr, self.h, rows, F, H, mean, stream)
            self._gmm("u", self.types[1], offs, xr, self.gu_out, rows, F, H, mean, stream)
            silu_mul(self.h, self.h, self.gu_out, F, rows=rows, ld=F, stream=stream)
        self._gmm("d", self.types[2], offs, self.h, self.y_recv, rows, H, F, mean, stream)

    def __call__(self, x, T: int | None = None, ids=None, w=None, out=None, peer_tokens: int | None = None,
                 stream=None):
        """y [T, H] for x [T, H] (fp32, device), into `out` when given.
        ids/w override the router (int32 [T, k] global expert ids and fp32
        [T, k] weights)."""
        T = int(x.shape[0]) if T is None else int(T)
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens above max_tokens={self.max_tokens}")
        if ids is None:
            self.route(x, T, stream)
            ids, w = self.ids, self.w
        y = self.y if out is None else out
        self.ep.dispatch(x, ids, T, stream=stream)
        self.experts(T, peer_tokens, stream=stream)
        acc = False
        if self.shared is not None:
            self._shared_ffn(x, T, y, stream)
            acc = True
        self.ep.combine(self.y_recv, w, y, accumulate=acc, stream=stream)
        return y[:T]
