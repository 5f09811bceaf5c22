"""MoE routing, sort, gather, combine and the expert-parallel dispatch on one
GPU (libswq's swq_moe_*, swq_ep_* with one rank, swq_grouped_matmul and
swq.moe.MoEFFN) against the C oracle (oracle/moe_oracle.c).

The reference has no MoE forward, so parity for routing is unpinned by it:
the oracle states the routing as libswq defines it.  Exact (bit-equal): top-k
ids, sort, gather, combine (one fmaf per slot in both), dispatch layout.
Router logits: fp32 sums in another order than the oracle's double sums,
relative error <= 1e-5 of the row's largest |logit|; softmax weights: CUDA's
expf against the C library's, <= 1e-6 relative.
"""
import ctypes
import math
import os

import numpy as np
import pytest
import torch

from conftest import REL_L2_TOL, rel_l2
from swq import synth

pytestmark = pytest.mark.gpu


def _cudart():
    import nvidia.cuda_runtime as cr
    lib = ctypes.CDLL(os.path.join(list(cr.__path__)[0], "lib", "libcudart.so.12"))
    lib.cudaMemcpy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int]
    return lib


def d2h(ptr: int, shape, dtype) -> np.ndarray:
    """Copy device memory at a raw address (libswq-owned) to a numpy array."""
    out = np.empty(shape, dtype=dtype)
    torch.cuda.synchronize()
    assert _cudart().cudaMemcpy(out.ctypes.data, ptr, out.nbytes, 2) == 0  # cudaMemcpyDeviceToHost
    return out


# ---------------------------------------------------------------- router
@pytest.mark.parametrize("T,E,H,k", [(1, 8, 64, 1), (5, 256, 2048, 8), (33, 64, 130, 4), (9, 1024, 512, 32),
                                     (17, 256, 4096, 8)])
def test_router(cuda, oracle_mod, T, E, H, k):
    import swq
    g = torch.Generator().manual_seed(T * 1000 + E)
    W = (torch.randn(E, H, generator=g) * 0.02).float()
    X = torch.randn(T, H, generator=g).float()
    logits = torch.empty(T, E, device="cuda")
    ids = torch.empty(T, k, dtype=torch.int32, device="cuda")
    w = torch.empty(T, k, device="cuda")
    swq.moe_router(W.cuda(), X.cuda(), T, E, H, k, logits, ids, w)
    swq.check()
    got_l = logits.cpu().numpy()
    want_l = oracle_mod.moe_router_logits(W.numpy(), X.numpy())
    scale = np.abs(want_l).max(axis=1, keepdims=True)
    assert np.all(np.abs(got_l - want_l) <= 1e-5 * scale)
    # selection and weights exactly as the oracle states them, on the GPU's logits
    want_ids, want_w = oracle_mod.moe_topk_softmax(got_l, k)
    assert np.array_equal(ids.cpu().numpy(), want_ids)
    np.testing.assert_allclose(w.cpu().numpy(), want_w, rtol=1e-6, atol=1e-7)
    # and the same experts as the exact logits pick, up to near-ties
    ex_ids, _ = oracle_mod.moe_topk_softmax(want_l.astype(np.float32), k)
    assert (ids.cpu().numpy() == ex_ids).mean() > 0.95


def test_router_ties_and_nan(cuda, oracle_mod):
    """Equal logits select the lower expert id first; a NaN token ranks every
    expert as -inf (ids 0 .. k-1 in order, NaN weights)."""
    import swq
    T, E, H, k = 3, 16, 32, 4
    W = torch.randn(E, H).float()
    W[5] = W[3]
    W[9] = W[3]
    X = torch.randn(T, H).float()
    X[0] = W[3] * 10  # experts 3, 5, 9 tie at the top for token 0
    X[2, 7] = float("nan")
    logits = torch.empty(T, E, device="cuda")
    ids = torch.empty(T, k, dtype=torch.int32, device="cuda")
    w = torch.empty(T, k, device="cuda")
    swq.moe_router(W.cuda(), X.cuda(), T, E, H, k, logits, ids, w)
    swq.check()
    got = ids.cpu().numpy()
    assert list(got[0, :3]) == [3, 5, 9]
    assert list(got[2]) == [0, 1, 2, 3]
    want_ids, want_w = oracle_mod.moe_topk_softmax(logits.cpu().numpy(), k)
    assert np.array_equal(got, want_ids)
    gw = w.cpu().numpy()
    assert np.array_equal(np.isnan(gw), np.isnan(want_w)) and np.isnan(gw[2]).all()


def test_router_shape_errors(cuda):
    import swq
    t = torch.empty(64, device="cuda")
    i = torch.empty(64, dtype=torch.int32, device="cuda")
    with pytest.raises(swq.SwqError):
        swq.moe_router(t, t, 1, 8, 8, 9, t, i, t)       # k > E
    with pytest.raises(swq.SwqError):
        swq.moe_router(t, t, 1, 2048, 8, 8, t, i, t)    # E above the limit
    with pytest.raises(swq.SwqError):
        swq.moe_router(t, t, 1, 8, 8, 33, t, i, t)      # k above the limit


# ---------------------------------------------------------------- sort / gather / combine
def _sort(ids_np, E):
    import swq
    P = ids_np.size
    ids = torch.from_numpy(ids_np.reshape(-1).astype(np.int32)).cuda()
    offs = torch.empty(E + 1, dtype=torch.int32, device="cuda")
    srt = torch.full((max(P, 1),), -7, dtype=torch.int32, device="cuda")
    prow = torch.empty(max(P, 1), dtype=torch.int32, device="cuda")
    swq.moe_sort(ids, P, E, offs, srt, prow)
    return offs, srt, prow


@pytest.mark.parametrize("P,E", [(0, 4), (1, 1), (31, 7), (33, 256), (1000, 256), (8192, 256), (70001, 1024),
                                 (4096, 1)])
def test_sort(cuda, oracle_mod, P, E):
    import swq
    rng = np.random.default_rng(P + E)
    ids = rng.integers(0, E, size=P).astype(np.int32)
    if P > 100:
        ids[: P // 3] = ids[0]  # a hot expert
    offs, srt, prow = _sort(ids, E)
    swq.check()
    w_off, w_srt, w_prow, bad = oracle_mod.moe_sort(ids, E)
    assert bad == 0
    assert np.array_equal(offs.cpu().numpy(), w_off)
    assert np.array_equal(srt.cpu().numpy()[: w_off[-1]], w_srt)
    assert np.array_equal(prow.cpu().numpy()[:P], w_prow)


def test_sort_bad_ids(cuda, oracle_mod):
    import swq
    ids = np.array([3, 9, -1, 2, 3, 100, 0], dtype=np.int32)
    offs, srt, prow = _sort(ids, 8)
    with pytest.raises(swq.SwqError) as ei:
        swq.check()
    assert ei.value.status == swq.Status.BAD_ARG
    w_off, w_srt, w_prow, bad = oracle_mod.moe_sort(ids, 8)
    assert bad == 3
    assert np.array_equal(offs.cpu().numpy(), w_off)
    assert np.array_equal(prow.cpu().numpy()[:7], w_prow)
    swq.check()  # the status word was cleared


@pytest.mark.parametrize("T,k,E,H,acc", [(1, 1, 1, 4, False), (37, 8, 64, 2048, False), (5, 3, 16, 130, True)])
def test_gather_combine(cuda, oracle_mod, T, k, E, H, acc):
    import swq
    rng = np.random.default_rng(T * k + H)
    ids = rng.integers(0, E, size=(T, k)).astype(np.int32)
    X = rng.standard_normal((T, H)).astype(np.float32)
    offs, srt, prow = _sort(ids, E)
    P = T * k
    Xs = torch.full((P, H), float("nan"), device="cuda")
    swq.moe_gather(torch.from_numpy(X).cuda(), srt, offs, E, P, k, H, Xs)
    w_off, w_srt, w_prow, _ = oracle_mod.moe_sort(ids, E)
    assert np.array_equal(Xs.cpu().numpy(), X[w_srt // k])
    Ys = rng.standard_normal((P, H)).astype(np.float32)
    w = rng.random((T, k)).astype(np.float32)
    Y0 = rng.standard_normal((T, H)).astype(np.float32)
    Y = torch.from_numpy(Y0.copy()).cuda()
    swq.moe_combine(torch.from_numpy(Ys).cuda(), prow, torch.from_numpy(w).cuda(), T, k, H, Y, accumulate=acc)
    swq.check()
    want = oracle_mod.moe_combine(Ys, w_prow, w, T, k, H, Y0 if acc else None)
    assert np.array_equal(Y.cpu().numpy(), want)


# ---------------------------------------------------------------- grouped matmul
@pytest.mark.parametrize("mean", [1, 32])
def test_grouped_matmul_live_rows(cuda, oracle_mod, mean):
    """Rows past expert_offsets[E] (NaN here) are not read, and every routed
    row matches the oracle (GEMV form: the single-row fixed-point tolerance;
    tensor-core form: fp16 operands)."""
    import swq
    E, N, K = 6, 512, 2048
    t = synth.Q4_K
    Ws = [synth.random_blocks(t, N, K, seed=700 + e) for e in range(E)]
    dW = [torch.from_numpy(w.reshape(-1)).cuda() for w in Ws]
    tab = torch.tensor([d.data_ptr() for d in dW], dtype=torch.int64, device="cuda")
    counts = [0, mean, 2 * mean + 1, 1, 0, mean + 3]
    offs = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    R = int(offs[-1])
    cap = R + 40
    X = np.full((cap, K), np.nan, np.float32)
    X[:R] = synth.random_activations(R, K, seed=71)
    Y = torch.full((cap, N), 7.0, device="cuda")
    swq.grouped_matmul(t, tab, torch.from_numpy(offs).cuda(), torch.from_numpy(X).cuda(), Y, E, cap, N, K, mean)
    swq.check()
    got = Y.cpu().numpy()
    assert np.all(got[R:] == 7.0)
    for e in range(E):
        a, b = offs[e], offs[e + 1]
        if b > a:
            want = oracle_mod.gemm(t, Ws[e], X[a:b], b - a, N, K)
            assert rel_l2(got[a:b], want) <= REL_L2_TOL, e


def test_grouped_matmul_rows_independent(cuda):
    """The GEMV form's result for a row does not depend on the other rows of
    its expert (passes of 4, 2 or 1): the same rows alone give the same bits."""
    import swq
    E, N, K, t = 3, 256, 1024, synth.Q6_K
    Ws = [torch.from_numpy(synth.random_blocks(t, N, K, seed=90 + e).reshape(-1)).cuda() for e in range(E)]
    tab = torch.tensor([w.data_ptr() for w in Ws], dtype=torch.int64, device="cuda")
    X = torch.from_numpy(synth.random_activations(7, K, seed=91)).cuda()
    offs = torch.tensor([0, 3, 5, 7], dtype=torch.int32, device="cuda")
    Y = torch.empty(7, N, device="cuda")
    swq.grouped_matmul(t, tab, offs, X, Y, E, 7, N, K, 2)
    for r in range(7):
        e = 0 if r < 3 else (1 if r < 5 else 2)
        y1 = torch.empty(1, N, device="cuda")
        one = torch.tensor([0, 0, 0, 0], dtype=torch.int32, device="cuda")
        one[e + 1:] = 1
        swq.grouped_matmul(t, tab, one, X[r:r + 1].contiguous(), y1, E, 1, N, K, 1)
        assert torch.equal(y1[0], Y[r]), r
    swq.check()


# ---------------------------------------------------------------- expert parallel, one rank
def test_ep_one_rank(cuda, oracle_mod):
    from swq.moe import ExpertParallel
    T, k, E, H = 29, 4, 12, 256
    rng = np.random.default_rng(5)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
    X = rng.standard_normal((T, H)).astype(np.float32)
    ep = ExpertParallel(40, k, E, H)
    assert ep.capacity == 40 * k
    for rep in range(3):  # epochs advance
        ep.dispatch(torch.from_numpy(X).cuda(), torch.from_numpy(ids).cuda(), T)
        lay = oracle_mod.ep_layout([ids], E, 1)[0]
        R = len(lay["tags"])
        xr = d2h(ep.recv_ptr, (R, H), np.float32)
        loff = d2h(ep.offsets_ptr, (E + 1,), np.int32)
        assert np.array_equal(loff, lay["loff"])
        _, w_srt, w_prow, _ = oracle_mod.moe_sort(ids, E)
        assert np.array_equal(xr, X[np.array([w_srt[i] for _, i in lay["tags"]]) // k])
        Yr = rng.standard_normal((ep.capacity, H)).astype(np.float32)
        w = rng.random((T, k)).astype(np.float32)
        Y = torch.empty(T, H, device="cuda")
        ep.combine(torch.from_numpy(Yr).cuda(), torch.from_numpy(w).cuda(), Y)
        import swq
        swq.check()
        # the output of sorted slot i is the received row that carries tag (0, i)
        ret = np.zeros((T * k, H), np.float32)
        for r, (_, i) in enumerate(lay["tags"]):
            ret[i] = Yr[r]
        assert np.array_equal(Y.cpu().numpy(), oracle_mod.moe_combine(ret, w_prow, w, T, k, H)), rep
    ep.close()


# ---------------------------------------------------------------- MoE FFN
def _experts(E, H, F, types, seed):
    return [(synth.random_blocks(types[0], F, H, seed=seed + 3 * e),
             synth.random_blocks(types[1], F, H, seed=seed + 3 * e + 1),
             synth.random_blocks(types[2], H, F, seed=seed + 3 * e + 2)) for e in range(E)]


def _ffn_oracle(oracle_mod, experts, types, x, ids, w, H, F, shared=None, shared_types=None, Fs=0):
    T, k = ids.shape
    y = np.zeros((T, H), np.float32)

    def swiglu(g_b, u_b, d_b, ts, xt, f):
        g = oracle_mod.gemm(ts[0], g_b, xt, 1, f, H)
        u = oracle_mod.gemm(ts[1], u_b, xt, 1, f, H)
        h = (g / (1.0 + np.exp(-g.astype(np.float64))) * u).astype(np.float32)
        return oracle_mod.gemm(ts[2], d_b, h, 1, H, f)[0]

    for t in range(T):
        if shared is not None:
            y[t] = swiglu(*shared, shared_types, x[t:t + 1], Fs)
        for j in range(k):
            y[t] += w[t, j] * swiglu(*experts[int(ids[t, j])], types, x[t:t + 1], F)
    return y


@pytest.mark.parametrize("T,shared", [(4, False), (24, True), (300, False)])
def test_moe_ffn_one_gpu(cuda, oracle_mod, T, shared):
    """16 experts (gate/up 512x2048 Q4_K, down 2048x512 Q6_K), top-4, the
    fp32 router on the device; decode-sized T takes the grouped GEMV, T=300
    the tensor-core grouped GEMM."""
    from swq.moe import MoEFFN
    E, H, F, k = 16, 2048, 512, 4
    types = (synth.Q4_K, synth.Q4_K, synth.Q6_K)
    experts = _experts(E, H, F, types, seed=5000)
    g = torch.Generator().manual_seed(9)
    router = (torch.randn(E, H, generator=g) * 0.02).float()
    x = torch.randn(T, H, generator=g).float()
    sh = None
    if shared:
        sh = (synth.random_blocks(types[0], 1024, H, seed=11), synth.random_blocks(types[1], 1024, H, seed=12),
              synth.random_blocks(types[2], H, 1024, seed=13))
    moe = MoEFFN(experts, types, H, F, router, k, max_tokens=max(T, 8), shared=sh, shared_types=types,
                 shared_F=1024)
    y = moe(x.cuda()).cpu().numpy()
    import swq
    swq.check()
    ids = moe.ids[:T].cpu().numpy()
    w = moe.w[:T].cpu().numpy()
    want_ids, _ = oracle_mod.moe_topk_softmax(moe.logits[:T].cpu().numpy(), k)
    assert np.array_equal(ids, want_ids)
    rows = slice(0, min(T, 40))
    want = _ffn_oracle(oracle_mod, experts, types, x.numpy()[rows], ids[rows], w[rows], H, F, sh, types, 1024)
    assert rel_l2(y[rows], want) <= REL_L2_TOL
    # a second call (epochs advance) gives the same bits
    y2 = moe(x.cuda()).cpu().numpy()
    assert np.array_equal(y, y2)
    moe.ep.close()


def test_moe_ffn_graph(cuda):
    """The whole layer captured in a CUDA graph and replayed: no host sync
    inside, and replays give the eager bits."""
    from swq.moe import MoEFFN
    E, H, F, k, T = 8, 1024, 256, 2, 6
    types = (synth.Q4_K, synth.Q4_K, synth.Q4_K)
    experts = _experts(E, H, F, types, seed=44)
    router = (torch.randn(E, H, generator=torch.Generator().manual_seed(1)) * 0.02).float()
    moe = MoEFFN(experts, types, H, F, router, k, max_tokens=T)
    x = torch.randn(T, H, generator=torch.Generator().manual_seed(2)).cuda()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        eager = moe(x, stream=s).clone()
    s.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        moe(x, stream=s)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(moe.y[:T], eager)
    del graph
    moe.ep.close()


@pytest.mark.parametrize("t,N,mean", [(synth.Q4_K, 512, 1), (synth.Q4_K, 300, 32), (synth.Q6_K, 256, 32),
                                      (synth.Q4_0, 384, 40)])
def test_grouped_matmul_stacked(cuda, t, N, mean):
    """Experts stacked in one tensor (expert e at rows e*N ..) give the same
    bits as the same matrices behind a pointer table, in both forms (for the
    tensor-core form: one tensor-map box per stage against one copy per row;
    a ragged N reads past an expert's last row and must mask it)."""
    import swq
    E, K = 5, 2048
    Ws = [synth.random_blocks(t, N, K, seed=800 + e) for e in range(E)]
    W_all = torch.from_numpy(np.concatenate([w.reshape(-1) for w in Ws])).cuda()
    dW = [torch.from_numpy(w.reshape(-1)).cuda() for w in Ws]
    tab = torch.tensor([d.data_ptr() for d in dW], dtype=torch.int64, device="cuda")
    counts = [mean, 0, 2 * mean + 1, mean + 5, 3]
    offs = torch.tensor(np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)).cuda()
    R = int(sum(counts))
    X = torch.from_numpy(synth.random_activations(R, K, seed=81)).cuda()
    Y1 = torch.empty(R, N, device="cuda")
    Y2 = torch.empty(R, N, device="cuda")
    swq.grouped_matmul(t, tab, offs, X, Y1, E, R, N, K, mean)
    swq.grouped_matmul_stacked(t, W_all, offs, X, Y2, E, R, N, K, mean)
    swq.check()
    assert torch.equal(Y1, Y2)
