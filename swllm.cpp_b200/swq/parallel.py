"""Tensor and expert parallelism for the quantized projections (one process per GPU).

Dense tensor parallelism for a Llama decoder layer's projections:

* column parallel (q/k/v split by heads, gate/up): rank r of G holds rows
  [r N/G, (r+1) N/G) of W -- whole GGUF rows -- and produces that slice of Y.
  No exchange.
* row parallel (o_proj, down_proj): rank r holds, of every row, the blocks that
  cover columns [r K/G, (r+1) K/G) (K/G a multiple of the block size, so the
  shard is still a valid GGUF matrix) and multiplies them with the same slice
  of X.  One all-reduce (sum) of the M x N partial products gives Y.

Expert parallelism for a mixture-of-experts FFN (SwiGLU experts):

* rank r owns experts [r E/G, (r+1) E/G).  Every (token, top-k slot) pair is
  sent to the owner of its expert (all-to-all), the owner runs gate/up, SwiGLU
  and down for all pairs it received with the grouped GEMM, and the outputs
  travel back (all-to-all) to be weighted by the routing weights and summed.

The reference runs one process and has no MoE path; each parallel layer is
checked against the same layer computed whole by one process.  The matmul
functions are parameters so the exchange logic can run on CPU ranks (gloo)
with a CPU stand-in for the kernels; by default they are libswq's CUDA
kernels and every tensor lives on the rank's GPU.
"""
from __future__ import annotations

from typing import Callable, Sequence

import numpy as np

from .lib import gemm as _swq_gemm, grouped_gemm as _swq_grouped_gemm, grouped_gemv as _swq_grouped_gemv
from .lib import grouped_matmul as _swq_grouped_matmul
from .synth import block_geometry


# ---------------------------------------------------------------- sharding
def split_rows(blocks: np.ndarray, N: int, rank: int, world: int) -> tuple[np.ndarray, int, int]:
    """Column-parallel shard: rows [n0, n1) of an [N, row_bytes] block matrix."""
    if N % world:
        raise ValueError(f"N={N} is not divisible by {world} ranks")
    n = N // world
    b = np.asarray(blocks).reshape(N, -1)
    return np.ascontiguousarray(b[rank * n:(rank + 1) * n]), rank * n, (rank + 1) * n


def split_k(blocks: np.ndarray, type_id: int, N: int, K: int, rank: int, world: int) -> tuple[np.ndarray, int, int]:
    """Row-parallel shard: of every row, the blocks covering columns [k0, k1)."""
    qk, bb = block_geometry(type_id)
    if K % (world * qk):
        raise ValueError(f"K={K} does not split into {world} shards of whole {qk}-element blocks")
    kl = K // world
    nb = kl // qk
    b = np.asarray(blocks).reshape(N, -1)
    return np.ascontiguousarray(b[:, rank * nb * bb:(rank + 1) * nb * bb]), rank * kl, (rank + 1) * kl


def _world(group) -> tuple[int, int]:
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(group), dist.get_world_size(group)
    return 0, 1


def _default_gemm(type_id, W, X, Y, M, N, K):
    _swq_gemm(type_id, W, X, Y, M, N, K)


# ---------------------------------------------------------------- dense TP
class ColumnParallelLinear:
    """y_local[M, N/G] = x[M, K] . W[rows of this rank]^T."""

    def __init__(self, blocks: np.ndarray, type_id: int, N: int, K: int, device=None, group=None,
                 gemm: Callable | None = None):
        import torch
        self.rank, self.world = _world(group)
        shard, self.n0, self.n1 = split_rows(blocks, N, self.rank, self.world)
        self.type_id, self.N, self.K, self.group = type_id, N, K, group
        self.W = torch.from_numpy(shard.reshape(-1)).to(device)
        self.gemm = gemm or _default_gemm

    def __call__(self, x):
        import torch
        M = x.shape[0]
        y = torch.empty((M, self.n1 - self.n0), dtype=torch.float32, device=x.device)
        self.gemm(self.type_id, self.W, x, y, M, self.n1 - self.n0, self.K)
        return y

    def gather(self, y_local):
        """All ranks' slices side by side: y[M, N]."""
        import torch
        import torch.distributed as dist
        if self.world == 1:
            return y_local
        parts = [torch.empty_like(y_local) for _ in range(self.world)]
        dist.all_gather(parts, y_local.contiguous(), group=self.group)
        return torch.cat(parts, dim=1)


class RowParallelLinear:
    """y[M, N] = sum over ranks of x[:, K slice] . W[:, K slice]^T (one all-reduce)."""

    def __init__(self, blocks: np.ndarray, type_id: int, N: int, K: int, device=None, group=None,
                 gemm: Callable | None = None):
        import torch
        self.rank, self.world = _world(group)
        shard, self.k0, self.k1 = split_k(blocks, type_id, N, K, self.rank, self.world)
        self.type_id, self.N, self.K, self.group = type_id, N, K, group
        self.W = torch.from_numpy(shard.reshape(-1)).to(device)
        self.gemm = gemm or _default_gemm

    def local_input(self, x):
        """This rank's columns of a full activation x[M, K]."""
        return x[:, self.k0:self.k1].contiguous()

    def __call__(self, x_local):
        import torch
        import torch.distributed as dist
        M = x_local.shape[0]
        y = torch.empty((M, self.N), dtype=torch.float32, device=x_local.device)
        self.gemm(self.type_id, self.W, x_local, y, M, self.N, self.k1 - self.k0)
        if self.world > 1:
            dist.all_reduce(y, op=dist.ReduceOp.SUM, group=self.group)
        return y


# ---------------------------------------------------------------- MoE EP
def route_topk(logits, k: int):
    """Router output -> (expert ids [T, k], weights [T, k]): the k largest logits
    per token, weights = softmax over those k logits (fp32)."""
    import torch
    vals, ids = torch.topk(logits.float(), k, dim=-1)
    return ids.to(torch.int32), torch.softmax(vals, dim=-1)


class _GroupedCUDA:
    """Expert matmuls through libswq: one device table of the local experts'
    weight addresses per projection.  A few rows per expert (decode, at most
    `gemv_rows` on average) take swq_grouped_gemv, more take the tensor-core
    swq_grouped_gemm.  The expert weights are separate torch allocations, so
    they start on the 16-byte boundary the GEMV path needs."""

    def __init__(self, device, gemv_rows: int = 4):
        self.device = device
        self.gemv_rows = gemv_rows
        self.mean_rows = 0  # expected rows per expert, set by the caller (0: rows / experts)

    def table(self, weights: Sequence):
        import torch
        return torch.tensor([w.data_ptr() for w in weights], dtype=torch.int64, device=self.device)

    def __call__(self, type_id, weights, table, offsets, X, Y, N, K):
        rows, E = X.shape[0], len(weights)
        if self.mean_rows > 0:  # the same kernel on every rank, whatever its share of the rows
            _swq_grouped_matmul(type_id, table, offsets, X, Y, E, rows, N, K, self.mean_rows)
            return
        fn = _swq_grouped_gemv if rows <= self.gemv_rows * E else _swq_grouped_gemm
        fn(type_id, table, offsets, X, Y, E, rows, N, K)


class ExpertParallelMoE:
    """A SwiGLU mixture-of-experts FFN with experts sharded over ranks.

    experts: E triples (gate, up, down) of GGUF block arrays, gate/up [F x H]
    and down [H x F] (only this rank's experts are kept; each may also be a
    torch uint8 tensor already on the device, and the other ranks' entries
    may be None).  types: the GGML type
    of gate, up and down.  grouped: expert matmul (type, weights, table,
    offsets, X, Y, N, K) over rows grouped by local expert; default libswq."""

    def __init__(self, experts: Sequence[tuple[np.ndarray, np.ndarray, np.ndarray]], types: tuple[int, int, int],
                 H: int, F: int, device=None, group=None, grouped: Callable | None = None):
        import torch
        self.rank, self.world = _world(group)
        self.E = len(experts)
        if self.E % self.world:
            raise ValueError(f"{self.E} experts do not split over {self.world} ranks")
        self.el = self.E // self.world
        self.e0 = self.rank * self.el
        self.H, self.F, self.types, self.group, self.device = H, F, types, group, device
        own = experts[self.e0:self.e0 + self.el]
        def to_dev(a):
            if isinstance(a, torch.Tensor):
                return a.reshape(-1).to(device)
            return torch.from_numpy(np.ascontiguousarray(a).reshape(-1)).to(device)
        self.gate = [to_dev(g) for g, _, _ in own]
        self.up = [to_dev(u) for _, u, _ in own]
        self.down = [to_dev(d) for _, _, d in own]
        self.grouped = grouped or _GroupedCUDA(device)
        tab = getattr(self.grouped, "table", None)
        self.tables = [tab(w) if tab else None for w in (self.gate, self.up, self.down)]

    def _a2a(self, x, send_counts, recv_counts):
        import torch
        import torch.distributed as dist
        out = torch.empty((int(sum(recv_counts)),) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
        if self.world == 1:
            out.copy_(x)
        else:
            dist.all_to_all_single(out, x.contiguous(), list(recv_counts), list(send_counts), group=self.group)
        return out

    def experts_forward(self, xr, er):
        """Rows xr [R, H] for local experts er [R] (0 .. el-1) -> [R, H]."""
        import torch
        order = torch.argsort(er, stable=True)
        xs = xr[order].contiguous()
        counts = torch.bincount(er.long(), minlength=self.el)
        offs = torch.zeros(self.el + 1, dtype=torch.int32, device=xr.device)
        offs[1:] = torch.cumsum(counts, 0).to(torch.int32)
        R = xs.shape[0]
        g = torch.empty((R, self.F), dtype=torch.float32, device=xr.device)
        u = torch.empty_like(g)
        self.grouped(self.types[0], self.gate, self.tables[0], offs, xs, g, self.F, self.H)
        self.grouped(self.types[1], self.up, self.tables[1], offs, xs, u, self.F, self.H)
        h = (torch.nn.functional.silu(g) * u).contiguous()
        ys = torch.empty((R, self.H), dtype=torch.float32, device=xr.device)
        self.grouped(self.types[2], self.down, self.tables[2], offs, h, ys, self.H, self.F)
        out = torch.empty_like(ys)
        out[order] = ys
        return out

    def __call__(self, x, topk_ids, topk_w):
        """x [T, H] fp32, topk_ids [T, k] int, topk_w [T, k] -> [T, H]."""
        import torch
        import torch.distributed as dist
        T, k = topk_ids.shape
        if hasattr(self.grouped, "mean_rows"):
            self.grouped.mean_rows = max(1, -(-T * k // self.E))
        eid = topk_ids.reshape(-1).long()                       # pair p = t*k + j
        owner = torch.div(eid, self.el, rounding_mode="floor")
        order = torch.argsort(owner, stable=True)                # send order
        send_counts = torch.bincount(owner, minlength=self.world)
        recv_counts = torch.empty_like(send_counts)
        if self.world > 1:
            dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        else:
            recv_counts.copy_(send_counts)
        sc, rc = send_counts.tolist(), recv_counts.tolist()
        tok = torch.div(order, k, rounding_mode="floor")
        xr = self._a2a(x[tok], sc, rc)
        er = self._a2a((eid[order] - owner[order] * self.el).to(torch.int32), sc, rc)
        yr = self.experts_forward(xr, er) if xr.shape[0] else xr.new_zeros((0, self.H))
        yb = self._a2a(yr, rc, sc)                               # back in send order
        y_pairs = torch.empty_like(yb)
        y_pairs[order] = yb
        w = topk_w.reshape(-1, 1).to(y_pairs.dtype)
        return (y_pairs * w).reshape(T, k, self.H).sum(dim=1)
