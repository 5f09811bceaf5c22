"""swq.parallel on GPUs: the MoE layer through the CUDA grouped GEMM (1 GPU),
and tensor/expert parallelism over NCCL (2 GPUs, skipped with fewer).

Tolerance: relative L2 <= 1e-3 against the oracle (fp16-operand kernels), and
<= 1e-5 between the parallel and the 1-GPU results of the same kernels (they
differ only by the order of the all-reduce sum and by row grouping).
"""
import os
import socket
import tempfile

import numpy as np
import pytest
import torch

from conftest import REL_L2_TOL, rel_l2
from swq import parallel, synth

pytestmark = pytest.mark.gpu


def _experts(E, H, F, types, seed):
    return [(synth.random_blocks(types[0], F, H, seed=seed + 3 * e),
             synth.random_blocks(types[1], F, H, seed=seed + 3 * e + 1),
             synth.random_blocks(types[2], H, F, seed=seed + 3 * e + 2)) for e in range(E)]


def _moe_oracle(oracle_mod, experts, types, x, ids, w, H, F):
    T, k = ids.shape
    y = np.zeros((T, H), np.float32)
    for t in range(T):
        for j in range(k):
            g_b, u_b, d_b = experts[int(ids[t, j])]
            g = oracle_mod.gemm(types[0], g_b, x[t:t + 1], 1, F, H)
            u = oracle_mod.gemm(types[1], u_b, x[t:t + 1], 1, F, H)
            h = (g / (1.0 + np.exp(-g)) * u).astype(np.float32)
            y[t] += w[t, j] * oracle_mod.gemm(types[2], d_b, h, 1, H, F)[0]
    return y


def test_moe_layer_one_gpu(cuda, oracle_mod):
    """16 experts (gate/up 512x2048 Q4_K, down 2048x512 Q6_K), 24 tokens, top-4."""
    E, H, F, T, k = 16, 2048, 512, 24, 4
    types = (synth.Q4_K, synth.Q4_K, synth.Q6_K)
    experts = _experts(E, H, F, types, seed=5000)
    g = torch.Generator().manual_seed(9)
    x = torch.randn(T, H, generator=g)
    ids, w = parallel.route_topk(torch.randn(T, E, generator=g), k)
    moe = parallel.ExpertParallelMoE(experts, types, H, F, device="cuda")
    y = moe(x.cuda(), ids.cuda(), w.cuda()).cpu().numpy()
    want = _moe_oracle(oracle_mod, experts, types, x.numpy(), ids.numpy(), w.numpy(), H, F)
    assert rel_l2(y, want) <= REL_L2_TOL


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, path):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        # tensor parallel: column (gate-like) then row (down-like) projection
        t1, t2 = synth.Q4_K, synth.Q6_K
        M, K, N1, N2 = 7, 2048, 1024, 2048
        W1 = synth.random_blocks(t1, N1, K, seed=61)
        W2 = synth.random_blocks(t2, N2, N1, seed=62)
        x = torch.from_numpy(synth.random_activations(M, K, seed=63)).cuda()
        col = parallel.ColumnParallelLinear(W1, t1, N1, K, device="cuda")
        row = parallel.RowParallelLinear(W2, t2, N2, N1, device="cuda")
        y_tp = row(col(x))
        # expert parallel MoE
        E, H, F, T, k = 8, 2048, 512, 12, 2
        types = (synth.Q4_K, synth.Q4_K, synth.Q6_K)
        experts = _experts(E, H, F, types, seed=6000)
        g = torch.Generator().manual_seed(10)
        xm = torch.randn(T, H, generator=g).cuda()
        ids, w = parallel.route_topk(torch.randn(T, E, generator=g), k)
        moe = parallel.ExpertParallelMoE(experts, types, H, F, device="cuda")
        y_ep = moe(xm, ids.cuda(), w.cuda())
        torch.cuda.synchronize()
        if rank == 0:
            # through a file: a queue's pipe holds 64 KB, and a larger put()
            # would block until the parent reads, which it does only after join
            np.savez(path, y_tp=y_tp.cpu().numpy(), y_ep=y_ep.cpu().numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_tensor_and_expert_parallel(cuda):
    import torch.multiprocessing as mp
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "results.npz")
        mp.start_processes(_nccl_worker, args=(2, _free_port(), path), nprocs=2, join=True, start_method="spawn")
        got = np.load(path)
        y_tp, y_ep = got["y_tp"], got["y_ep"]
    # the same layers on one GPU
    t1, t2 = synth.Q4_K, synth.Q6_K
    M, K, N1, N2 = 7, 2048, 1024, 2048
    W1 = synth.random_blocks(t1, N1, K, seed=61)
    W2 = synth.random_blocks(t2, N2, N1, seed=62)
    x = torch.from_numpy(synth.random_activations(M, K, seed=63)).cuda()
    h = parallel.ColumnParallelLinear(W1, t1, N1, K, device="cuda")(x)
    y1 = parallel.RowParallelLinear(W2, t2, N2, N1, device="cuda")(h).cpu().numpy()
    assert rel_l2(y_tp, y1) <= 1e-5
    E, H, F, T, k = 8, 2048, 512, 12, 2
    types = (synth.Q4_K, synth.Q4_K, synth.Q6_K)
    experts = _experts(E, H, F, types, seed=6000)
    g = torch.Generator().manual_seed(10)
    xm = torch.randn(T, H, generator=g).cuda()
    ids, w = parallel.route_topk(torch.randn(T, E, generator=g), k)
    y2 = parallel.ExpertParallelMoE(experts, types, H, F, device="cuda")(xm, ids.cuda(), w.cuda()).cpu().numpy()
    assert rel_l2(y_ep, y2) <= 1e-5
