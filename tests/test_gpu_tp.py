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
