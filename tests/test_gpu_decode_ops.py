"""The decode-step kernels one by one against numpy restatements of the
reference's Compute helpers (src/tensor.h:1028-1180) and attention loop
(src/model.h:329-361): RMSNorm (alone and fused with the residual add), RoPE +
KV append, split-context attention (contexts below, at and above the split
size; GQA group sizes 1, 4, 8; head dims 64, 128, 256; several sequences),
SiLU-mul, embedding and argmax.  fp32 throughout; tolerances are fp32
rounding of differently ordered sums."""
import numpy as np
import pytest

import swq
from conftest import rel_l2

pytestmark = pytest.mark.gpu

F32 = np.float32


def _t(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _attention_ref(q, kc, vc, n_ctx, nh, nkv, hd):
    out = np.zeros(nh * hd, np.float64)
    mul = nh // nkv
    for h in range(nh):
        kvh = h // mul
        qh = q[h * hd:(h + 1) * hd].astype(np.float64)
        ks = kc[:n_ctx, kvh * hd:(kvh + 1) * hd].astype(np.float64)
        vs = vc[:n_ctx, kvh * hd:(kvh + 1) * hd].astype(np.float64)
        s = ks @ qh / np.sqrt(hd)
        p = np.exp(s - s.max())
        out[h * hd:(h + 1) * hd] = (p / p.sum()) @ vs
    return out


@pytest.mark.parametrize("nh,nkv,hd", [(8, 2, 64), (32, 8, 128), (8, 8, 128), (16, 2, 128), (4, 1, 256)])
@pytest.mark.parametrize("pos", [0, 1, 63, 64, 65, 511, 1000, 1023])
def test_attention(cuda, nh, nkv, hd, pos):
    torch = cuda
    rows, max_seq = 3, 1024
    rng = np.random.default_rng(pos * 7 + nh)
    kv_dim = nkv * hd
    kc = rng.standard_normal((rows, max_seq, kv_dim)).astype(F32)
    vc = rng.standard_normal((rows, max_seq, kv_dim)).astype(F32)
    q = (2.0 * rng.standard_normal((rows, nh * hd))).astype(F32)
    ws_bytes = swq.attention_workspace_bytes(nh, nkv, hd, rows, max_seq)
    ws = torch.zeros(ws_bytes // 4 + 1, dtype=torch.float32, device="cuda")
    d_out = torch.full((rows, nh * hd), float("nan"), device="cuda")
    d_pos = torch.tensor([pos], dtype=torch.int32, device="cuda")
    d_q, d_k, d_v = _t(torch, q), _t(torch, kc), _t(torch, vc)
    for _ in range(2):  # the second call reuses the workspace counters
        swq.attention_decode(d_out, d_q, d_k, d_v, d_pos, ws, ws_bytes, nh, nkv, hd, rows, max_seq)
        swq.check()
        got = d_out.cpu().numpy()
        for b in range(rows):
            want = _attention_ref(q[b], kc[b], vc[b], pos + 1, nh, nkv, hd)
            assert rel_l2(got[b], want) <= 2e-6, (b, rel_l2(got[b], want))


def test_attention_position_moves_inside_one_workspace(cuda):
    """Consecutive positions through the same workspace (as graph replays do)."""
    torch = cuda
    nh, nkv, hd, rows, max_seq = 32, 8, 128, 1, 256
    rng = np.random.default_rng(5)
    kc = rng.standard_normal((rows, max_seq, nkv * hd)).astype(F32)
    vc = rng.standard_normal((rows, max_seq, nkv * hd)).astype(F32)
    q = rng.standard_normal((rows, nh * hd)).astype(F32)
    ws_bytes = swq.attention_workspace_bytes(nh, nkv, hd, rows, max_seq)
    ws = torch.zeros(ws_bytes // 4 + 1, dtype=torch.float32, device="cuda")
    d_out = torch.empty((rows, nh * hd), device="cuda")
    d_q, d_k, d_v = _t(torch, q), _t(torch, kc), _t(torch, vc)
    for pos in (3, 70, 71, 140, 200, 255, 10):
        d_pos = torch.tensor([pos], dtype=torch.int32, device="cuda")
        swq.attention_decode(d_out, d_q, d_k, d_v, d_pos, ws, ws_bytes, nh, nkv, hd, rows, max_seq)
        swq.check()
        want = _attention_ref(q[0], kc[0], vc[0], pos + 1, nh, nkv, hd)
        assert rel_l2(d_out[0].cpu().numpy(), want) <= 2e-6, pos


@pytest.mark.parametrize("n,rows", [(4096, 1), (8192, 3), (1000, 2)])
def test_rmsnorm_and_add_rmsnorm(cuda, n, rows):
    torch = cuda
    rng = np.random.default_rng(n + rows)
    x = rng.standard_normal((rows, n)).astype(F32)
    y = rng.standard_normal((rows, n)).astype(F32)
    w = (1 + 0.01 * rng.standard_normal(n)).astype(F32)
    eps = 1e-5

    def ref(v):
        v = v.astype(np.float64)
        return v / np.sqrt((v * v).mean(axis=1, keepdims=True) + eps) * w

    d_x, d_y, d_w = _t(torch, x), _t(torch, y), _t(torch, w)
    out = torch.empty((rows, n), device="cuda")
    swq.rmsnorm(out, d_x, d_w, n, eps, rows)
    swq.check()
    assert rel_l2(out.cpu().numpy(), ref(x)) <= 1e-6
    swq.add_rmsnorm(out, d_x, d_y, d_w, n, eps, rows)  # x += y; out = norm(x)
    swq.check()
    assert np.array_equal(d_x.cpu().numpy(), (x + y).astype(F32))
    assert rel_l2(out.cpu().numpy(), ref(x + y)) <= 1e-6


def test_silu_mul_embed_argmax(cuda):
    torch = cuda
    rng = np.random.default_rng(9)
    rows, n = 3, 5000
    gu = rng.standard_normal((rows, 2 * n)).astype(F32) * 4
    d_gu = _t(torch, gu)
    h = torch.empty((rows, n), device="cuda")
    swq.silu_mul(h, d_gu, d_gu[:, n:], n, rows, 2 * n)
    swq.check()
    g, u = gu[:, :n].astype(np.float64), gu[:, n:].astype(np.float64)
    assert rel_l2(h.cpu().numpy(), g / (1 + np.exp(-g)) * u) <= 1e-6

    vocab, dim = 777, 96
    table = rng.standard_normal((vocab, dim)).astype(F32)
    toks = np.array([0, 776, 123], np.int32)
    x = torch.empty((rows, dim), device="cuda")
    swq.embed(x, _t(torch, table), _t(torch, toks), dim, vocab, rows)
    swq.check()
    assert np.array_equal(x.cpu().numpy(), table[toks])

    logits = rng.standard_normal((rows, 128256)).astype(F32)
    logits[1, 128255] = 100.0
    d_tok = torch.zeros(rows, dtype=torch.int32, device="cuda")
    swq.argmax(_t(torch, logits), 128256, rows, d_tok)
    swq.check()
    assert d_tok.cpu().numpy().tolist() == np.argmax(logits, axis=1).tolist()


@pytest.mark.parametrize("neox", [False, True], ids=["interleaved", "neox"])
def test_rope_kv(cuda, neox):
    """q rotated in place, rotated k and v appended at pos (rows 0..B-1)."""
    torch = cuda
    rng = np.random.default_rng(3)
    nh, nkv, hd, rows, max_seq, pos = 8, 2, 64, 2, 16, 9
    q_dim, kv_dim = nh * hd, nkv * hd
    freqs = (1.0 / np.power(F32(5e5), np.arange(0, hd, 2, dtype=F32) / F32(hd))).astype(F32)
    q = rng.standard_normal((rows, q_dim)).astype(F32)
    k = rng.standard_normal((rows, kv_dim)).astype(F32)
    v = rng.standard_normal((rows, kv_dim)).astype(F32)
    d_q, d_k, d_v = _t(torch, q), _t(torch, k), _t(torch, v)
    kc = torch.zeros((rows, max_seq, kv_dim), device="cuda")
    vc = torch.zeros_like(kc)
    swq.rope_kv(d_q, d_k, d_v, kc, vc, torch.tensor([pos], dtype=torch.int32, device="cuda"), _t(torch, freqs),
                q_dim, kv_dim, hd, hd, neox, rows, max_seq)
    swq.check()

    def rot(a):
        a = a.astype(np.float64).reshape(rows, -1, hd)
        ang = pos * freqs.astype(np.float64)
        c, s = np.cos(ang), np.sin(ang)
        if neox:
            x0, x1 = a[..., :hd // 2], a[..., hd // 2:]
            return np.concatenate([x0 * c - x1 * s, x0 * s + x1 * c], -1).reshape(rows, -1)
        x0, x1 = a[..., 0::2], a[..., 1::2]
        out = np.empty_like(a)
        out[..., 0::2], out[..., 1::2] = x0 * c - x1 * s, x0 * s + x1 * c
        return out.reshape(rows, -1)

    assert rel_l2(d_q.cpu().numpy(), rot(q)) <= 1e-6
    kcn, vcn = kc.cpu().numpy(), vc.cpu().numpy()
    assert rel_l2(kcn[:, pos], rot(k)) <= 1e-6
    assert np.array_equal(vcn[:, pos], v)
    assert not kcn[:, :pos].any() and not kcn[:, pos + 1:].any()
