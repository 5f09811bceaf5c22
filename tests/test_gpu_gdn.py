"""swq_gdn_step -- one GatedDeltaNet decode step on the device -- against the
restatement of the reference's loops (oracle/model_ref.py gdn_step,
src/model.h:421-504), over several steps so the recurrent state and the conv
history carry over.

Both round every product and sum as the reference's loops do, except the
per-head norm's sum of squares (a tree on the device); outputs agree to
1e-5 relative L2 and the state to 1e-5."""
import numpy as np
import pytest

import swq
from conftest import rel_l2

pytestmark = pytest.mark.gpu

F32 = np.float32


def _case(rng, rows, n_k, n_v, k_hd, v_hd, cw, optional):
    kd, vd = n_k * k_hd, n_v * v_hd
    qkv = (0.3 * rng.standard_normal((rows, 2 * kd + vd))).astype(F32)
    z = rng.standard_normal((rows, vd)).astype(F32) if optional else None
    gates = [rng.standard_normal((rows, n_v)).astype(F32) if optional else None for _ in range(3)]
    a = (0.5 * rng.standard_normal(n_v)).astype(F32) if optional else None
    conv_w = (0.5 * rng.standard_normal((vd, cw))).astype(F32) if optional and cw else None
    norm_w = (1 + 0.1 * rng.standard_normal(vd)).astype(F32) if optional else None
    return qkv, z, gates, a, conv_w, norm_w


@pytest.mark.parametrize("rows,n_k,n_v,k_hd,v_hd,cw,optional", [
    (1, 2, 4, 32, 32, 4, True),      # the tiny hybrid model's layer
    (3, 4, 8, 64, 128, 4, True),     # several rows, GQA-style key head sharing
    (1, 16, 32, 128, 128, 4, True),  # Qwen3.5-sized heads
    (2, 2, 2, 16, 48, 3, False),     # no gate / beta / alpha / dt / conv / norm: the reference's defaults
    (1, 1, 1, 8, 1000, 2, True),     # value heads wider than a warp multiple
])
def test_gdn_step_matches_restatement(cuda, rows, n_k, n_v, k_hd, v_hd, cw, optional):
    from oracle.model_ref import gdn_step
    torch = cuda
    rng = np.random.default_rng(rows * 1000 + v_hd)
    kd, vd = n_k * k_hd, n_v * v_hd
    S_ref = np.zeros((rows, n_v, k_hd, v_hd), F32)
    conv_ref = np.zeros((rows, vd, max(1, cw)), F32)
    d_S = torch.zeros((rows, n_v, k_hd, v_hd), device="cuda")
    d_conv = torch.zeros((rows, vd, max(1, cw)), device="cuda")
    d_y = torch.full((rows, vd), float("nan"), device="cuda")
    dev = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    for step in range(4):
        qkv, z, gates, a, conv_w, norm_w = _case(rng, rows, n_k, n_v, k_hd, v_hd, cw, optional)
        swq.gdn_step(dev(qkv), dev(z), dev(gates[0]), dev(gates[1]), dev(gates[2]), dev(a), dev(conv_w),
                     dev(norm_w), d_S, d_conv, d_y, rows, n_k, n_v, k_hd, v_hd, cw if conv_w is not None else 0)
        swq.check()
        want = np.stack([
            gdn_step(qkv[r], None if z is None else z[r], *(None if gt is None else gt[r] for gt in gates), a,
                     conv_w, norm_w, S_ref[r], conv_ref[r], n_k, n_v, k_hd, v_hd,
                     cw if conv_w is not None else 0) for r in range(rows)])
        assert rel_l2(d_y.cpu().numpy(), want) <= 1e-5, step
        assert rel_l2(d_S.cpu().numpy(), S_ref) <= 1e-5, step
        if conv_w is not None:
            assert np.array_equal(d_conv.cpu().numpy(), conv_ref), step


def test_gdn_step_rejects_bad_shapes(cuda):
    torch = cuda
    buf = torch.zeros(4096, device="cuda")
    with pytest.raises(swq.SwqError):  # value head wider than the kernel's 1024 threads
        swq.gdn_step(buf, None, None, None, None, None, None, None, buf, buf, buf, 1, 1, 1, 8, 2048, 0)
    with pytest.raises(swq.SwqError):  # q/k/v stride below its row
        swq.gdn_step(buf, None, None, None, None, None, None, None, buf, buf, buf, 1, 1, 1, 8, 8, 0, ld_qkv=16)
    with pytest.raises(swq.SwqError):
        swq.gdn_step(None, None, None, None, None, None, None, None, buf, buf, buf, 1, 1, 1, 8, 8, 0)
