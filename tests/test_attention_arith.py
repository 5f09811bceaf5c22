"""The operand representation of the tensor-core causal prefill attention
(prefill.cu, SWQ_OPT_PREFILL_ATTENTION 3 and 2), restated in numpy on the CPU
against float64 attention (softmax(q k^T / sqrt(hd)) v per head, the causal
mask of the reference's per-token forward, src/model.h:329-361).

The kernel splits operands into pairs of fp16 numbers (stage_row, split2):
* each q and k row scaled by 2^(13 - E) (E its largest binary exponent,
  E >= -100) and split x = h + l; S = h.h + h.l + l.h with exact products,
  then the row factors and 1/sqrt(hd) in fp32;
* the softmax weights P = exp(S - max) in (0, 1], split unscaled;
* each V row unscaled (scaled down only from 2^15 up, the factor taken back
  by P), split the same way; O = (ph.vh + ph.vl + pl.vh) / sum P.
Here the same splits are made (the softmax over a row's whole context at once;
the kernel's online rescaling only changes which maximum P is taken against)
and everything else is float64: the error left is the representation's.

Results: about 1e-7 relative L2 with q, k, v of order one and with q / k
rows over many decades; V is the limit -- its pairs lose bits once values
fall below fp16's normal range relative to nothing (no scale-up), about
1.7e-8 / |V| (1.7e-5 at 1e-3, 1.7e-4 at 1e-4), where the GPU tests' 1e-5 no
longer holds; the fp32 forms (1, 0) have no such floor."""
import numpy as np
import pytest

from conftest import rel_l2

F16, F32, F64 = np.float16, np.float32, np.float64


def split_rows(x: np.ndarray, to_top: bool):
    """stage_row: per row the fp16 pair (h, l) as float64 and the factor back."""
    x = np.asarray(x, F32)
    mx = np.abs(x).max(axis=-1).astype(F32)
    E = np.maximum(((mx.view(np.int32) >> 23) & 0xFF) - 126, -100)
    if to_top:
        up, back = np.ldexp(F32(1), 13 - E).astype(F32), np.ldexp(1.0, E - 13)
    else:
        k = np.maximum(E - 15, 0)
        up, back = np.ldexp(F32(1), -k).astype(F32), np.ldexp(1.0, k)
    u = (x * up[..., None]).astype(F32)
    h = u.astype(F16)
    l = (u - h.astype(F32)).astype(F16)
    return h.astype(F64), l.astype(F64), back


def split_vals(p: np.ndarray):
    u = np.asarray(p, F32)
    h = u.astype(F16)
    return h.astype(F64), (u - h.astype(F32)).astype(F16).astype(F64)


def attention_ref(q, k, v, pos0):
    """float64 causal attention of P query rows at positions pos0 .. over
    pos0 + P keys; q [P, hd], k / v [pos0 + P, hd] (one head)."""
    P, hd = q.shape
    S = (q.astype(F64) @ k.astype(F64).T) / np.sqrt(hd)
    S[np.arange(k.shape[0])[None, :] > (pos0 + np.arange(P))[:, None]] = -np.inf
    W = np.exp(S - S.max(axis=1, keepdims=True))
    return (W @ v.astype(F64)) / W.sum(axis=1, keepdims=True)


def attention_pairs(q, k, v, pos0):
    P, hd = q.shape
    qh, ql, qb = split_rows(q, True)
    kh, kl, kb = split_rows(k, True)
    vh, vl, vb = split_rows(v, False)
    S = (qh @ kh.T + qh @ kl.T + ql @ kh.T) * qb[:, None] * kb[None, :] / np.sqrt(hd)
    S[np.arange(k.shape[0])[None, :] > (pos0 + np.arange(P))[:, None]] = -np.inf
    W = np.exp(S - S.max(axis=1, keepdims=True))
    ph, pl = split_vals(W * vb[None, :])
    O = ph @ vh + ph @ vl + pl @ vh
    return O / W.sum(axis=1, keepdims=True)


def _case(seed, hd=128, P=96, pos0=40, qk_decades=0.0, v_scale=1.0):
    rng = np.random.default_rng(seed)
    n = pos0 + P
    q = rng.standard_normal((P, hd)) * 10.0 ** rng.uniform(-qk_decades, 0, (P, 1))
    k = rng.standard_normal((n, hd)) * 10.0 ** rng.uniform(-qk_decades, 0, (n, 1))
    v = rng.standard_normal((n, hd)) * v_scale
    return q.astype(F32), k.astype(F32), v.astype(F32), pos0


@pytest.mark.parametrize("hd", [64, 128])
def test_pairs_representation_order_one(hd):
    q, k, v, pos0 = _case(1, hd=hd)
    assert rel_l2(attention_pairs(q, k, v, pos0), attention_ref(q, k, v, pos0)) <= 3e-7


def test_pairs_representation_qk_over_decades():
    """Each q / k row carries its own scale: rows spread over five decades
    keep their 22 bits."""
    q, k, v, pos0 = _case(2, qk_decades=5.0)
    assert rel_l2(attention_pairs(q, k, v, pos0), attention_ref(q, k, v, pos0)) <= 3e-7


def test_pairs_large_v_scaled_down():
    """V rows up to 1e6: scaled below fp16's range, the factor taken back by P."""
    q, k, v, pos0 = _case(3)
    v = (v * (10.0 ** np.random.default_rng(4).uniform(0, 6, (v.shape[0], 1)))).astype(F32)
    assert rel_l2(attention_pairs(q, k, v, pos0), attention_ref(q, k, v, pos0)) <= 3e-7


@pytest.mark.parametrize("v_scale,lo,hi", [(1e-2, 5e-7, 5e-6), (1e-3, 5e-6, 5e-5), (1e-4, 5e-5, 5e-4)])
def test_pairs_small_v_floor(v_scale, lo, hi):
    """Unscaled V: the low fp16 part of small values turns subnormal (spacing
    2^-24), so the error grows as about 1.7e-8 / |V|."""
    q, k, v, pos0 = _case(5, v_scale=v_scale)
    err = rel_l2(attention_pairs(q, k, v, pos0), attention_ref(q, k, v, pos0))
    assert lo <= err <= hi, err
