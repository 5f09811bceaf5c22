"""Tensor- and expert-parallel layers (swq.parallel) on CPU ranks (gloo, world 2).

The exchange logic (sharding, all-reduce, all-to-all dispatch and combine) runs
in two processes; the quantized matmuls are the oracle's CPU products, so the
parallel result must match one process computing the whole layer with the same
products (fp32, up to summation order).
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from swq import parallel, synth

TOL = 1e-5


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def cpu_gemm(type_id, W, X, Y, M, N, K):
    import oracle
    y = oracle.gemm(type_id, W.numpy().reshape(N, -1), X.numpy(), M, N, K)
    Y.copy_(torch.from_numpy(y))


class CpuGrouped:
    def __call__(self, type_id, weights, table, offsets, X, Y, N, K):
        offs = offsets.tolist()
        for e, w in enumerate(weights):
            a, b = offs[e], offs[e + 1]
            if b > a:
                cpu_gemm(type_id, w, X[a:b].contiguous(), Y[a:b], b - a, N, K)


def _init(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)


def _tp_worker(rank, world, port):
    _init(rank, world, port)
    try:
        t1, t2 = synth.Q4_K, synth.Q6_K
        M, K, N1, N2 = 5, 512, 512, 256
        W1 = synth.random_blocks(t1, N1, K, seed=31)
        W2 = synth.random_blocks(t2, N2, N1, seed=32)
        x = torch.from_numpy(synth.random_activations(M, K, seed=33))
        col = parallel.ColumnParallelLinear(W1, t1, N1, K, gemm=cpu_gemm)
        row = parallel.RowParallelLinear(W2, t2, N2, N1, gemm=cpu_gemm)
        h_local = col(x)
        assert h_local.shape == (M, N1 // world)
        y = row(h_local)  # the column shard of h is exactly the row shard's K slice
        h_full = torch.empty((M, N1))
        cpu_gemm(t1, torch.from_numpy(W1.reshape(-1)), x, h_full, M, N1, K)
        want = torch.empty((M, N2))
        cpu_gemm(t2, torch.from_numpy(W2.reshape(-1)), h_full, want, M, N2, N1)
        err = float(torch.linalg.norm(y - want) / torch.linalg.norm(want))
        assert err <= TOL, err
        assert torch.allclose(col.gather(h_local), h_full)
    finally:
        dist.destroy_process_group()


def _moe_reference(experts, types, x, ids, w, H, F):
    T, k = ids.shape
    y = torch.zeros((T, H))
    for t in range(T):
        for j in range(k):
            g_b, u_b, d_b = experts[int(ids[t, j])]
            xt = x[t:t + 1]
            g, u = torch.empty((1, F)), torch.empty((1, F))
            cpu_gemm(types[0], torch.from_numpy(g_b.reshape(-1)), xt, g, 1, F, H)
            cpu_gemm(types[1], torch.from_numpy(u_b.reshape(-1)), xt, u, 1, F, H)
            h = torch.nn.functional.silu(g) * u
            o = torch.empty((1, H))
            cpu_gemm(types[2], torch.from_numpy(d_b.reshape(-1)), h, o, 1, H, F)
            y[t] += w[t, j] * o[0]
    return y


def _moe_worker(rank, world, port):
    _init(rank, world, port)
    try:
        E, H, F, T, k = 4, 256, 512, 9, 2
        types = (synth.Q4_K, synth.Q4_K, synth.Q6_K)
        experts = [(synth.random_blocks(types[0], F, H, seed=40 + 3 * e),
                    synth.random_blocks(types[1], F, H, seed=41 + 3 * e),
                    synth.random_blocks(types[2], H, F, seed=42 + 3 * e)) for e in range(E)]
        # every rank sees the same tokens and routing (router replicated)
        g = torch.Generator().manual_seed(7)
        x = torch.randn(T, H, generator=g)
        logits = torch.randn(T, E, generator=g)
        ids, w = parallel.route_topk(logits, k)
        moe = parallel.ExpertParallelMoE(experts, types, H, F, grouped=CpuGrouped())
        assert moe.el == E // world
        y = moe(x, ids, w)
        want = _moe_reference(experts, types, x, ids, w, H, F)
        err = float(torch.linalg.norm(y - want) / torch.linalg.norm(want))
        assert err <= TOL, err
    finally:
        dist.destroy_process_group()


def _decoder_worker(rank, world, port):
    """The tensor-parallel LlamaDecoder's host path on real ranks: its device
    operations are recorded, not run (no GPU here), but every collective of a
    decode step and of a prefill goes through gloo, so both ranks must issue
    the same ones in the same order.  (gloo's tensor all-gather wants equal
    chunk shapes; the logits gather uses its list form, the same exchange.)"""
    import contextlib

    import swq.model as M
    from test_gpu_model import _small, _weights

    class _S:
        def synchronize(self):
            pass

    _init(rank, world, port)
    try:
        for name in ("embed", "rmsnorm", "add_rmsnorm", "gemm_act_ws", "rope_kv", "attention_decode", "silu_mul",
                     "argmax", "decode_advance", "rope_kv_prefill", "attention_prefill", "add", "qkv_bias_norm"):
            setattr(M, name, lambda *a, **k: None)
        M.gemm_workspace_bytes = lambda *a: 0
        torch.cuda.Stream = lambda device=None: _S()
        torch.cuda.stream = lambda st: contextlib.nullcontext()
        cfg = _small()
        dec = M.LlamaDecoder(cfg, rows=2, device="cpu", weights=_weights(cfg, seed=9), group=dist.group.WORLD,
                             collective="nccl")
        assert (dec.rank, dec.world) == (rank, world)
        seen = []
        orig = dec._nccl_all_reduce

        def counted(t):
            seen.append(("sum", tuple(t.shape)))
            orig(t)

        def gather():
            parts = [torch.empty_like(dec.logits_l) for _ in range(world)]
            dist.all_gather(parts, dec.logits_l, group=dec.group)
            dec.logits.view(dec.rows, world, dec.vocab).copy_(torch.stack(parts).transpose(0, 1))
            seen.append(("gather",))

        dec.all_reduce = dec._nccl_all_reduce = counted
        dec._gather_logits = gather
        dec.logits_l.fill_(float(rank))
        dec.step()
        assert [tuple(dec.logits[0, i * dec.vocab:(i + 1) * dec.vocab].unique().tolist()) for i in range(world)] == \
            [(float(i),) for i in range(world)]  # each rank's slice in rank order
        dec.prefill([[1, 2, 3], [4, 5, 6]])
        per = [("sum", (2, cfg.dim))] * (2 * cfg.n_layers) + [("gather",)]
        per_prefill = [("sum", (6, cfg.dim))] * (2 * cfg.n_layers) + [("gather",)]
        assert seen == per + per_prefill, seen
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("worker", [_tp_worker, _moe_worker, _decoder_worker],
                         ids=["tensor_parallel", "expert_parallel", "decoder"])
def test_two_ranks(worker):
    mp.spawn(worker, args=(2, _free_port()), nprocs=2, join=True)


def test_route_topk():
    logits = torch.tensor([[0.0, 3.0, 1.0, 2.0]])
    ids, w = parallel.route_topk(logits, 2)
    assert ids.tolist() == [[1, 3]]
    assert torch.allclose(w, torch.softmax(torch.tensor([[3.0, 2.0]]), dim=-1))


def test_shards_are_valid_matrices():
    t = synth.Q4_K
    N, K = 8, 1024
    b = synth.random_blocks(t, N, K, seed=50)
    rows = [parallel.split_rows(b, N, r, 4)[0] for r in range(4)]
    assert np.array_equal(np.concatenate(rows), b.reshape(N, -1))
    cols = [parallel.split_k(b, t, N, K, r, 4)[0] for r in range(4)]
    assert np.array_equal(np.concatenate(cols, axis=1), b.reshape(N, -1))
    with pytest.raises(ValueError):
        parallel.split_k(b, t, N, K, 0, 8)  # 128-column shards are not whole blocks


def test_decoder_shards_reassemble():
    """The decoder's weight shards: rows of a column-parallel matrix and the
    whole blocks of a row-parallel one, which put back together give the
    matrix (and match the parallel-layer split functions)."""
    from swq.model import _shard
    from swq.parallel import split_k, split_rows
    for t, N, K in ((synth.Q4_K, 64, 1024), (synth.Q6_K, 32, 2048), (synth.Q8_0, 16, 256)):
        b = synth.random_blocks(t, N, K, seed=t)
        rows = [_shard(b, t, N, K, (r * N // 4, (r + 1) * N // 4), None) for r in range(4)]
        assert np.array_equal(np.concatenate(rows), b.reshape(N, -1))
        assert np.array_equal(rows[1], split_rows(b, N, 1, 4)[0])
        cols = [_shard(b, t, N, K, None, (r * K // 2, (r + 1) * K // 2)) for r in range(2)]
        assert np.array_equal(np.concatenate(cols, axis=1), b.reshape(N, -1))
        assert np.array_equal(cols[1], split_k(b, t, N, K, 1, 2)[0])


# ------------------------------------------- peer all-reduce recovery (host)
def _reset_worker(rank, world, port, path):
    """PeerAllReduce.reset's host ordering with the device calls faked: no
    rank may zero its flags before every rank has stopped its kernels
    (first barrier), and no rank may return -- and so launch the next sum --
    before every rank has zeroed them (second barrier).  Rank 1 arrives late."""
    import contextlib
    import time
    from swq import comm
    _init(rank, world, port)
    try:
        log = {}

        class FakeLib:
            def swq_allreduce_reset(self, ar, stream):
                log["reset"] = time.time()
                return 0

        comm.lib = lambda: FakeLib()
        comm._stream = lambda s: None
        torch.cuda.synchronize = lambda device=None: log.setdefault("sync", time.time())
        torch.cuda.device = lambda device: contextlib.nullcontext()
        ar = object.__new__(comm.PeerAllReduce)
        ar.group, ar.device, ar._ar = None, None, object()
        if rank == 1:
            time.sleep(0.5)
        log["enter"] = time.time()
        ar.reset(stream=object())
        log["return"] = time.time()
        np.save(f"{path}.{rank}.npy", np.array([log["enter"], log["sync"], log["reset"], log["return"]]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_peer_allreduce_reset_barriers(tmp_path):
    path = str(tmp_path / "reset")
    mp.spawn(_reset_worker, args=(2, _free_port(), path), nprocs=2, join=True)
    enter, sync, reset, ret = np.stack([np.load(f"{path}.{r}.npy") for r in range(2)]).T
    assert np.all(sync <= reset)                 # own kernels done before zeroing
    assert reset.min() >= sync.max()             # nobody zeroes before everyone stopped
    assert ret.min() >= reset.max()              # nobody resumes before everyone zeroed
    assert reset[0] >= enter[1]                  # the early rank waited for the late one
