"""Tensor-parallel decode (swq.model.LlamaDecoder with a process group): two
ranks over NCCL against the same model decoded by one GPU.

A 2-layer Llama-shaped model (dim 512, 8 query / 2 kv heads of 64, FFN 1024,
vocab 1000, Q4_K_M mix) with host weights; both runs get the same token at
each position (teacher-forced) and the step runs from a captured CUDA graph
that holds the all-reduces and the logits all-gather.  The rank's partial
products are summed in a different order than one GPU's, so the logits agree
to fp32 rounding (relative L2 1e-4).  Needs two GPUs (skipped otherwise).
"""
import os
import socket
import tempfile

import numpy as np
import pytest

from conftest import rel_l2

pytestmark = pytest.mark.gpu

TOKENS = [5, 811, 42, 300, 7]
TOL = 1e-4


def _cfg():
    from swq.model import LlamaConfig
    return LlamaConfig(n_layers=2, dim=512, n_heads=8, n_kv_heads=2, head_dim=64, ffn=1024, vocab=1000, max_seq=32)


def _run(dec, graph: bool):
    out = []
    if graph:
        dec.reset([TOKENS[0]], 0)
        dec.capture()
    for pos, tok in enumerate(TOKENS):
        dec.reset([tok], pos)
        dec.generate(1)
        dec.stream.synchronize()
        out.append(dec.logits[0].cpu().numpy().copy())
    return np.stack(out)


def _rank(rank, world, port, path, graph, collective="peer"):
    import datetime

    import torch
    import torch.distributed as dist
    from test_gpu_model import _weights
    from swq.model import LlamaDecoder
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        dec = LlamaDecoder(_cfg(), rows=1, weights=_weights(_cfg(), seed=11), device=f"cuda:{rank}",
                           collective=collective, group=dist.group.WORLD)
        assert dec.world == world and dec.nh == 8 // world
        logits = _run(dec, graph)
        dec.graph = None
        if rank == 0:
            np.save(path, logits)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("collective", ["peer", "nccl"])
@pytest.mark.parametrize("graph", [False, True], ids=["eager", "graph"])
def test_tp2_matches_one_gpu(cuda, graph, collective):
    torch = cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    from test_gpu_model import _weights
    from swq.model import LlamaDecoder
    want = _run(LlamaDecoder(_cfg(), rows=1, weights=_weights(_cfg(), seed=11)), graph)
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "logits.npy")
        mp.start_processes(_rank, args=(2, _free_port(), path, graph, collective), nprocs=2, join=True,
                           start_method="spawn")
        got = np.load(path)
    for pos in range(len(TOKENS)):
        assert rel_l2(got[pos], want[pos]) <= TOL, (pos, rel_l2(got[pos], want[pos]))


# ---------------------------------------------------------------- all-reduce
SIZES = [1, 3, 1000, 8192, 65536 * 4 + 3]


def _ar_rank(rank, world, port, path):
    import datetime

    import torch
    import torch.distributed as dist
    from swq.comm import PeerAllReduce
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        ar = PeerAllReduce(max(SIZES), device=f"cuda:{rank}")
        out = {}
        for n in SIZES:
            for rep in range(3):  # epochs advance; both data halves get used
                g = torch.Generator().manual_seed(1000 * n + 10 * rep + rank)
                x = torch.randn(n, generator=g).cuda()
                ar(x)
                torch.cuda.synchronize()
                out[f"{n}_{rep}"] = x.cpu().numpy()
        # inside a CUDA graph, replayed: the epochs live on the device
        s = torch.cuda.Stream()
        x = torch.ones(8192, device="cuda") * (rank + 1)
        with torch.cuda.stream(s):
            ar(x, stream=s)
        s.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            x.mul_(0.5)
            ar(x, stream=s)
        with torch.cuda.stream(s):
            for _ in range(5):
                graph.replay()
        s.synchronize()
        out["graph"] = x.cpu().numpy()
        import swq
        swq.check()
        np.savez(f"{path}.{rank}.npz", **out)
        del graph
        ar.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_peer_allreduce_two_ranks(cuda):
    torch = cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "ar")
        mp.start_processes(_ar_rank, args=(2, _free_port(), path), nprocs=2, join=True, start_method="spawn")
        got = [dict(np.load(f"{path}.{r}.npz")) for r in range(2)]
    for n in SIZES:
        for rep in range(3):
            xs = [torch.randn(n, generator=torch.Generator().manual_seed(1000 * n + 10 * rep + r)).numpy()
                  for r in range(2)]
            want = (xs[0] + xs[1]).astype(np.float32)  # rank order, fp32
            key = f"{n}_{rep}"
            assert np.array_equal(got[0][key], got[1][key]), key   # same bits on every rank
            assert np.array_equal(got[0][key], want), key
    # graph: x <- (x * 0.5) summed over 2 ranks, 1 eager + 5 replays from (1, 2) -> sum 3 * (0.5 * 2)^k ...
    v = 3.0  # after the eager call every rank holds 1 + 2
    for _ in range(5):
        v = 2 * (0.5 * v)
    assert np.all(got[0]["graph"] == v) and np.all(got[1]["graph"] == v)


# ------------------------------------------------------ failure and recovery
def _ar_fail_rank(rank, world, port, path):
    """Rank 1 skips one sum; rank 0's bounded wait gives up (SWQ_ERR_TIMEOUT
    from swq_check), both ranks reset between steps, and the next matched
    sums are exact again.  The process group is gloo: the handle exchange and
    the reset barriers stay on the host, no NCCL kernel is in flight."""
    import datetime
    import time

    import torch
    import torch.distributed as dist
    import swq
    from swq.comm import PeerAllReduce
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    try:
        ar = PeerAllReduce(4096, device=f"cuda:{rank}")
        s = torch.cuda.Stream()
        out = {}

        def matched(tag, n):
            x = torch.full((n,), float(rank + 1), device="cuda") * (1 + torch.arange(n, device="cuda"))
            torch.cuda.synchronize()
            dist.barrier()      # launch within the 50 ms bound of each other
            with torch.cuda.stream(s):
                ar(x, stream=s)
            swq.check(s)
            out[tag] = x.cpu().numpy()

        matched("before", 4096)
        # the failure: rank 1 does not make this call
        status = 0
        if rank == 0:
            x = torch.ones(4096, device="cuda")
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            with torch.cuda.stream(s):
                ar(x, stream=s)
            try:
                swq.check(s)
            except swq.SwqError as e:
                status = int(e.status)
            out["wait_s"] = np.array(time.perf_counter() - t0)
        out["status"] = np.array(status)
        ar.reset(stream=s)
        swq.check(s)            # the status word was read and cleared above
        for i in range(3):      # both data halves after the reset
            matched(f"after{i}", 4096 - 1000 * i)
        np.savez(f"{path}.{rank}.npz", **out)
        ar.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_peer_allreduce_timeout_and_reset(cuda):
    torch = cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    from swq.lib import Status
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "arf")
        mp.start_processes(_ar_fail_rank, args=(2, _free_port(), path), nprocs=2, join=True, start_method="spawn")
        got = [dict(np.load(f"{path}.{r}.npz")) for r in range(2)]
    assert int(got[0]["status"]) == int(Status.TIMEOUT)
    assert int(got[1]["status"]) == 0
    assert 0.04 <= float(got[0]["wait_s"]) < 5.0   # the 50 ms bound, not a hang
    for tag, n in [("before", 4096), ("after0", 4096), ("after1", 3096), ("after2", 2096)]:
        want = (3.0 * (1 + np.arange(n))).astype(np.float32)
        for r in range(2):
            assert np.array_equal(got[r][tag], want), (tag, r)


# ------------------------------------------------------ expert parallel (peer memory)
EP_E, EP_H, EP_F, EP_K = 16, 1024, 256, 4
EP_T = [(11, 3), (40, 37)]  # tokens of rank 0 and rank 1, per case (decode-like, then TC-sized)


def _ep_inputs(rank, T):
    from swq import synth
    g = torch_gen(100 + 7 * rank + T)
    x = g.standard_normal((T, EP_H)).astype(np.float32)
    experts = [(synth.random_blocks(synth.Q4_K, EP_F, EP_H, seed=300 + 3 * e),
                synth.random_blocks(synth.Q4_K, EP_F, EP_H, seed=301 + 3 * e),
                synth.random_blocks(synth.Q6_K, EP_H, EP_F, seed=302 + 3 * e)) for e in range(EP_E)]
    router = (np.random.default_rng(9).standard_normal((EP_E, EP_H)) * 0.02).astype(np.float32)
    return x, experts, router


def torch_gen(seed):
    return np.random.default_rng(seed)


def _ep_rank(rank, world, port, path):
    import datetime

    import torch
    import torch.distributed as dist
    import swq
    from swq.moe import MoEFFN
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        out = {}
        for case, Ts in enumerate(EP_T):
            T = Ts[rank]
            x, experts, router = _ep_inputs(rank, T)
            moe = MoEFFN([e if (i // (EP_E // world)) == rank else None for i, e in enumerate(experts)],
                         (swq.Q4_K, swq.Q4_K, swq.Q6_K), EP_H, EP_F, router, EP_K, max_tokens=64,
                         group=dist.group.WORLD)
            xd = torch.from_numpy(x).cuda()
            for rep in range(2):
                dist.barrier()  # launch within the 50 ms bound of each other
                y = moe(xd, T)
                swq.check()
                out[f"y{case}_{rep}"] = y.cpu().numpy()
            out[f"ids{case}"] = moe.ids[:T].cpu().numpy()
            from test_gpu_moe import d2h
            loff = d2h(moe.ep.offsets_ptr, (EP_E // world + 1,), np.int32)
            out[f"loff{case}"] = loff
            out[f"recv{case}"] = d2h(moe.ep.recv_ptr, (int(loff[-1]), EP_H), np.float32)
            dist.barrier()
            moe.ep.close()
        np.savez(f"{path}.{rank}.npz", **out)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_expert_parallel_two_ranks(cuda, oracle_mod):
    """MoEFFN over two GPUs (8 experts each, rows moved by peer stores) against
    the same layer on one GPU: the same routing, the rows each rank receives
    in the oracle's layout, and the layer output within 1e-6 (the GEMV form
    is bit-equal: a row's result does not depend on the other rows)."""
    torch = cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    import swq
    from swq.moe import MoEFFN
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "ep")
        mp.start_processes(_ep_rank, args=(2, _free_port(), path), nprocs=2, join=True, start_method="spawn")
        got = [dict(np.load(f"{path}.{r}.npz")) for r in range(2)]
    for case, Ts in enumerate(EP_T):
        ids = [got[r][f"ids{case}"] for r in range(2)]
        lay = oracle_mod.ep_layout(ids, EP_E, 2)
        xs = [_ep_inputs(r, Ts[r])[0] for r in range(2)]
        sorts = [oracle_mod.moe_sort(i, EP_E) for i in ids]
        for d in range(2):
            assert np.array_equal(got[d][f"loff{case}"], lay[d]["loff"]), (case, d)
            want = np.stack([xs[s][sorts[s][1][i] // EP_K] for s, i in lay[d]["tags"]])
            assert np.array_equal(got[d][f"recv{case}"], want), (case, d)
        for r in range(2):
            x, experts, router = _ep_inputs(r, Ts[r])
            one = MoEFFN(experts, (swq.Q4_K, swq.Q4_K, swq.Q6_K), EP_H, EP_F, router, EP_K, max_tokens=64)
            y1 = one(torch.from_numpy(x).cuda(), Ts[r]).cpu().numpy()
            assert np.array_equal(one.ids[:Ts[r]].cpu().numpy(), ids[r])
            assert rel_l2(got[r][f"y{case}_0"], y1) <= 1e-6, (case, r)
            assert np.array_equal(got[r][f"y{case}_0"], got[r][f"y{case}_1"])
            if max(Ts) * EP_K <= 4 * EP_E:  # both on the GEMV form
                assert np.array_equal(got[r][f"y{case}_0"], y1), (case, r)
            one.ep.close()
