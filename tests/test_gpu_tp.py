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


def _rank(rank, world, port, path, graph):
    import datetime

    import torch
    import torch.distributed as dist
    from test_gpu_model import _weights
    from swq.model import LlamaDecoder
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        dec = LlamaDecoder(_cfg(), rows=1, weights=_weights(_cfg(), seed=11), device=f"cuda:{rank}")
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


@pytest.mark.parametrize("graph", [False, True], ids=["eager", "graph"])
def test_tp2_matches_one_gpu(cuda, graph):
    torch = cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    from test_gpu_model import _weights
    from swq.model import LlamaDecoder
    want = _run(LlamaDecoder(_cfg(), rows=1, weights=_weights(_cfg(), seed=11)), graph)
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "logits.npy")
        mp.start_processes(_rank, args=(2, _free_port(), path, graph), nprocs=2, join=True, start_method="spawn")
        got = np.load(path)
    for pos in range(len(TOKENS)):
        assert rel_l2(got[pos], want[pos]) <= TOL, (pos, rel_l2(got[pos], want[pos]))
