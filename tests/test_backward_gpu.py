"""Training path (one layer step of the reference's backward) against the
reference's own backward kernels, through the C ABI.

Fixtures (tests/golden/backward_*.npz, made by make_golden.py on a B200 from
the reference's kernels): per case the gradients, the two square sums of the
clip, the updated fp32 masters / biases and the re-quantised weights.

Gradients must be bit-identical. The square sums are compared with a relative
tolerance of 1e-6: the reference adds its per-block sums with atomics in
arrival order, this build in block order, so the clip factor (and through it
the updated masters) may differ in the last bit; the updated masters are
compared within 2 ulp and the re-quantised codes within a flip budget.
"""
import sys

import numpy as np
import pytest
import torch

import aicortex_b200 as A
from aicortex_b200 import fmt
from conftest import GOLDEN

sys.path.insert(0, str(GOLDEN))
import golden_specs as S  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def h(x):
    torch.cuda.synchronize()
    return x.cpu().numpy()


def ulp_close(a, b, ulps=2, what=""):
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    ia, ib = a.view(np.int32).astype(np.int64), b.view(np.int32).astype(np.int64)
    d = np.abs(ia - ib)
    assert (d <= ulps).all(), f"{what}: {int((d > ulps).sum())} values differ by more than {ulps} ulp (max {d.max()})"


def sum_sq_f32(g):
    return float(np.sum(np.asarray(g, np.float64) ** 2))


def clip_f32(sum_sq):
    """clip_op (conv_layer.h:209-213) in fp32."""
    norm = np.sqrt(np.float32(sum_sq) + np.float32(1.0 / 8192.0), dtype=np.float32)
    return np.float32(1.0) / norm if norm > np.float32(1.0) else np.float32(1.0)


def check_update(ours, ref, master0, grad, ref_sum, penalty, what):
    """The update kernel with the reference's clip factor reproduces the
    reference's parameters bit for bit; the layer's own step (its factor from
    a block-order square sum) stays within the rounding of that factor."""
    f = clip_f32(ref_sum)
    d = t(master0)
    A.sgd_update(d, t(grad), t(np.array([f, ref_sum], np.float32)), S.TRAIN_LR, penalty)
    np.testing.assert_array_equal(h(d), ref, err_msg=f"{what}: update with the reference's clip factor")
    # the factor is 1 / sqrt(sum): a sum that is off by r moves it by r / 2 (r <= 4e-6 for
    # these sizes: fp32 sums over up to 1604 blocks, added in two different orders)
    tol = np.abs(grad.astype(np.float64)) * S.TRAIN_LR * float(f) * 2e-6 + np.abs(ref.astype(np.float64)) * 2.4e-7
    err = np.abs(np.asarray(ours, np.float64) - ref)
    assert (err <= tol).all(), f"{what}: {int((err > tol).sum())} updated values beyond the clip-factor rounding"


@pytest.mark.parametrize("case", [c[0] for c in S.CONV_BWD_CASES])
def test_conv_layer_backward_vs_reference(golden, case):
    g = golden("backward_conv")
    _, cin, cout, k, st, din, dout, act = next(c for c in S.CONV_BWD_CASES if c[0] == case)
    master, bias, _, gout = S.conv_bwd_case(case)
    layer = A.ConvLayer(cin, cout, k, st, din, dout, disable_activation=not act)
    layer.load_weights(t(master), t(bias))
    layer.train_bind(t(master), S.TRAIN_LR, S.TRAIN_PENALTY)
    gi = torch.zeros(din * din * cin, dtype=torch.float32, device=DEV)
    layer.backward(t(gout), t(g[f"{case}_xw"].view(np.int32)), t(g[f"{case}_xs"]), gi)
    m, gw, gb = layer.train_views()
    np.testing.assert_array_equal(h(gw), g[f"{case}_gw"], err_msg=f"{case}: weight gradient")
    np.testing.assert_array_equal(h(gb), g[f"{case}_gb"], err_msg=f"{case}: bias gradient")
    np.testing.assert_array_equal(h(gi), g[f"{case}_gi"], err_msg=f"{case}: input gradient")
    sw, sb = g[f"{case}_sums"]
    assert abs(sum_sq_f32(h(gw)) - sw) <= 1e-5 * max(sw, 1e-30) and abs(sum_sq_f32(h(gb)) - sb) <= 1e-5 * max(sb, 1e-30)
    check_update(h(m), g[f"{case}_master"], master, g[f"{case}_gw"], sw, S.TRAIN_PENALTY, f"{case}: masters")
    check_update(h(layer.packed()[2]), g[f"{case}_bias"], bias, g[f"{case}_gb"], sb, 0.0, f"{case}: bias")
    w, s, _ = layer.packed()
    cw, cr = fmt.codes(h(w).view(np.uint32).reshape(-1)), fmt.codes(g[f"{case}_w"].reshape(-1))
    # stochastic re-quantisation of masters that differ in the last bits: rare code flips
    assert np.mean(h(s) != g[f"{case}_s"]) <= 1e-3 and np.mean(cw != cr) <= 1e-3, f"{case}: re-quantised weights"


@pytest.mark.parametrize("out_c,act", S.MB_BWD_CASES)
def test_mamba_layer_backward_vs_reference(golden, out_c, act):
    g = golden("backward_mamba_N128")
    tag = f"o{out_c}_a{act}"
    blob, bias, _, gout = S.mamba_bwd_case(out_c, act)
    layer = A.MambaLayer(S.SSM_D, 128, out_c, act)
    layer.set_mode(A.AIC_MAMBA_EXACT)
    layer.load_weights(t(blob), t(bias))
    layer.bind_state(1)
    layer.bind_traces()
    layer.train_bind(t(blob), S.TRAIN_LR, S.TRAIN_PENALTY)
    xw, xs = t(g[f"{tag}_xw"].view(np.int32)), t(g[f"{tag}_xs"])
    out = torch.empty(S.MB_BWD_T, out_c, dtype=torch.float32, device=DEV)
    layer.forward(xw, xs, out, 1, S.MB_BWD_T)
    gi = torch.empty(S.SSM_D, dtype=torch.float32, device=DEV)
    layer.backward(t(gout), xw[-1:], xs[-1:], gi)
    m, gw, gb = layer.train_views()
    np.testing.assert_array_equal(h(gw), g[f"{tag}_gw"], err_msg=f"{tag}: blob gradient")
    np.testing.assert_array_equal(h(gb), g[f"{tag}_gb"], err_msg=f"{tag}: bias gradient")
    np.testing.assert_array_equal(h(gi), g[f"{tag}_gi"], err_msg=f"{tag}: input gradient")
    sw, sb = g[f"{tag}_sums"]
    assert abs(sum_sq_f32(h(gw)) - sw) <= 1e-5 * max(sw, 1e-30) and abs(sum_sq_f32(h(gb)) - sb) <= 1e-5 * max(sb, 1e-30)
    check_update(h(m), g[f"{tag}_master"], blob, g[f"{tag}_gw"], sw, S.TRAIN_PENALTY, f"{tag}: blob")
    check_update(h(layer.train_bias()), g[f"{tag}_bias"], bias, g[f"{tag}_gb"], sb, 0.0, f"{tag}: bias")


def test_critic_backward_vs_reference(golden):
    g = golden("backward_critic")
    w1, w2, wl, x = S.critic_case()
    c = A.Critic(32, 128, 1)
    c.load_weights(t(w1), t(w2), t(wl))
    c.bind_state(1)
    c.bind_traces()
    c.train_bind(S.TRAIN_LR, S.TRAIN_PENALTY)
    score = torch.empty(x.shape[0], dtype=torch.float32, device=DEV)
    c.forward_pooled(t(x), score, 1, x.shape[0])
    assert h(score)[-1] == g["pred"][0]
    c.backward(score[-1:], S.CRITIC_BWD_REAL)
    g1, g2, gl = c.train_views()
    for name, a in (("gw1", g1), ("gw2", g2), ("gl", gl)):
        np.testing.assert_array_equal(h(a), g[name], err_msg=name)
    for name, a, w0, gname, k in zip(("w1_after", "w2_after", "wl_after"), c.weights(), (w1, w2, wl),
                                     ("gw1", "gw2", "gl"), range(3)):
        check_update(h(a), g[name], w0, g[gname], g["sums"][k], S.TRAIN_PENALTY, name)


def test_residual_backward():
    """grad_res = grad_next, grad_next *= survival_prob_inv * residual_factor (kernels.h:1056-1079)."""
    rng = np.random.default_rng(5)
    gn = rng.standard_normal(4096).astype(np.float32)
    a, b = t(gn), torch.empty(4096, dtype=torch.float32, device=DEV)
    A.residual_backward(a, b, 1.25, 0.75)
    np.testing.assert_array_equal(h(b), gn)
    np.testing.assert_array_equal(h(a), gn * (np.float32(1.25) * np.float32(0.75)))


def test_sgd_update_matches_formula():
    """updateParamsKernel: d = fma(g, -lr * f, d * (1 - lr * penalty)) on whole uint4 only."""
    rng = np.random.default_rng(6)
    n = 1030  # two trailing elements are left alone, as in the reference
    d, gr = rng.standard_normal(n).astype(np.float32), rng.standard_normal(n).astype(np.float32)
    dd, gg = t(d), t(gr)
    factor = A.grad_clip_factor(gg)
    f = float(h(factor)[0])
    A.sgd_update(dd, gg, factor, 0.01, 1e-3)
    c_grad = np.float32(-0.01) * np.float32(f)
    c_data = np.float32(np.float64(np.float32(-0.01)) * np.float64(np.float32(1e-3)) + 1.0)
    want = d.copy()
    m = (n // 4) * 4
    want[:m] = (gr[:m].astype(np.float64) * np.float64(c_grad) +
                (d[:m] * c_data).astype(np.float64)).astype(np.float32)
    # float64 emulation of the fma: within 1 ulp (double rounding), the tail untouched
    ulp_close(h(dd)[:m], want[:m], ulps=1, what="sgd update")
    np.testing.assert_array_equal(h(dd)[m:], d[m:])
    norm = np.sqrt(np.float32(np.sum(gr.astype(np.float64) ** 2)) + np.float32(1 / 8192), dtype=np.float32)
    assert abs(f - float(np.float32(1) / norm)) <= 2e-7 * f
