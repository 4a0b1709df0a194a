"""The CPU oracle pinned against the reference: the golden fixtures hold the
outputs of the reference's own CUDA kernels (tests/golden/make_golden.py) on
the inputs of tests/golden/golden_specs.py.

Bit-exact: packing (hash + nibble layout), exponents, codes, action bits.
The reference is built with --use_fast_math, so its __expf/__logf/__log2f/
sqrt.approx differ from libm in the last bits; where that reaches a packed
output it can flip an exponent or a code at a rounding boundary, which is
counted and bounded. fp32 outputs agree to ~1e-6 relative.
"""
import sys

import numpy as np
import pytest

from conftest import GOLDEN

sys.path.insert(0, str(GOLDEN))
import golden_specs as S  # noqa: E402
import oracle as O  # noqa: E402
from aicortex_b200 import fmt  # noqa: E402


def check_f(w_a, s_a, w_b, s_b, flip_rate=2e-3, what=""):
    ca = fmt.codes(np.ascontiguousarray(w_a).view(np.uint32).reshape(-1))
    cb = fmt.codes(np.ascontiguousarray(w_b).view(np.uint32).reshape(-1))
    sa, sb = np.asarray(s_a).reshape(-1), np.asarray(s_b).reshape(-1)
    exp_rate = np.mean(sa != sb)
    diff = np.abs(ca.astype(np.int32) - cb.astype(np.int32))
    same = np.repeat(sa == sb, 32)
    assert exp_rate <= flip_rate, f"{what}: exponent mismatch rate {exp_rate}"
    assert diff[same].max(initial=0) <= 1, f"{what}: code off by {diff[same].max()}"
    assert np.mean(diff > 0) <= flip_rate, f"{what}: code flip rate {np.mean(diff > 0)}"


def close(a, b, rtol, what=""):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    scale = max(np.abs(b).max(), 1e-30)
    err = np.abs(a - b).max() / scale
    assert np.isfinite(a).all() and err <= rtol, f"{what}: error {err:.3e}"


def test_hash_uniform_ceiling():
    """The reference's factor 1/0xFFFFFFFFf is 2^-36 (hex integer literal), so
    its 'uniform' never reaches 1/16 (kernels.h:41)."""
    vals = np.array([O.lib.orc_uniform(O.lib.orc_unique_seed(i, i * 7), 1.0) for i in range(20000)])
    assert vals.max() < 1.0 / 16 and vals.max() > 0.06


def test_unique_seed_matches_definition():
    def seed(tid, sample):  # kernels.h:21-37, written independently in Python
        s = (tid + (sample & 0xFFFFFFFF) * 2654435761) & 0xFFFFFFFF
        s = (s ^ 61) ^ (s >> 16)
        s = (s * 9) & 0xFFFFFFFF
        s ^= s >> 4
        s = (s * 668265261) & 0xFFFFFFFF
        s ^= s >> 15
        return 123456789 if s == 0 else s
    for tid, sample in [(0, 0), (5, 12345), (1 << 20, -7), (255, 2**31 - 1)]:
        assert O.lib.orc_unique_seed(tid, sample) == seed(tid, sample)


def test_format_round_trip():
    rng = np.random.default_rng(0)
    x = (rng.standard_normal(32 * 64) * rng.uniform(0.01, 10, size=32 * 64)).astype(np.float32)
    w, s = O.pack_f32(x)
    q = fmt.codes(w.reshape(64, 4)).reshape(-1).astype(np.float64)
    amax = np.abs(x.reshape(64, 32)).max(axis=1).repeat(32).astype(np.float64)
    # codes are rn(x * 7 / absmax), but the stored exponent is rn(log2 absmax):
    # the format dequantises with 2^s/7, not absmax/7 (kernels.h:68-70)
    assert np.all(np.abs(q - x * 7.0 / amax) <= 0.5 + 1e-5)
    np.testing.assert_array_equal(s, np.rint(np.log2(amax[::32])).astype(np.int8))
    v = fmt.dequant(w.reshape(64, 4), s.reshape(64, 1)).reshape(-1)
    np.testing.assert_allclose(v, q * np.ldexp(1.0, s.astype(int)).repeat(32) / 7.0, rtol=1e-6)
    z, zs = O.pack_f32(np.zeros(32, np.float32))
    assert zs[0] == 0 and np.all(z == 0)


def test_oracle_pack(golden):
    g = golden("pack")
    master, acts = S.pack_master()
    assert S.sha(master) == str(g["master_sha"]) and S.sha(acts) == str(g["acts_sha"])
    w, s = O.pack_f32(master, stochastic=True, add_idx=master.size)
    np.testing.assert_array_equal(w, g["w"])
    np.testing.assert_array_equal(s, g["s"])
    w, s = O.pack_f32(acts)
    check_f(w, s, g["acts_w"], g["acts_s"], flip_rate=0.0, what="rn pack")


def test_oracle_stem(golden):
    g = golden("stem")
    planes = S.stem_case()
    assert S.sha(planes) == str(g["planes_sha"])
    w, s = O.stem_pack(planes[None], 32)
    check_f(w, s, g["w"], g["s"], flip_rate=1e-3, what="stem")


@pytest.mark.parametrize("name", sorted(S.CONV_CASES))
def test_oracle_conv(golden, name):
    g = golden(f"conv_{name}")
    cin, cout, k, st, din, dout, act = S.CONV_CASES[name]
    master, bias, _ = S.conv_case(name)
    assert S.sha(master) == str(g["master_sha"]) and S.sha(bias) == str(g["bias_sha"])
    ww, ws = O.pack_f32(master, True, master.size)
    assert S.sha(ww) == str(g["w_sha"]) and S.sha(ws) == str(g["s_sha"])
    ow, os_ = O.conv(g["x_w"], g["x_s"], ww, ws, bias, 1, cin, cout, k, st, din, dout, act)
    check_f(ow, os_, g["out_w"], g["out_s"], flip_rate=2e-3, what=name)


@pytest.mark.parametrize("name", sorted(S.RES_CASES))
def test_oracle_residual(golden, name):
    g = golden(name)
    pos, ch, dim, rf = S.RES_CASES[name]
    ow, os_ = O.residual(g["main_w"], g["main_s"], g["res_w"], g["res_s"], pos, ch, rf, False)
    check_f(ow, os_, g["out_w"], g["out_s"], flip_rate=0.0, what=name)


def test_oracle_gap(golden):
    g = golden("gap")
    close(O.gap_f32(g["x_w"], g["x_s"], 1, 64, 256)[0], g["out"], 1e-6, "gap f32")
    oh = O.gap_f16(g["c_w"], g["c_s"], 1, 16, 32)[0].astype(np.float32)
    close(oh, g["c_out"].astype(np.float32), 2e-3, "gap f16")


@pytest.mark.parametrize("n", [32, 128, 512])
def test_oracle_ssm(golden, n):
    g = golden(f"ssm_N{n}")
    blob, _ = S.ssm_case(n)
    assert S.sha(blob) == str(g["blob_sha"])
    layer = O.MambaLayerRef(S.SSM_D, n, S.SSM_D, 1, blob, np.zeros(S.SSM_D, np.float32), 1)
    assert S.sha(layer.w) == str(g["w_sha"]) and S.sha(layer.s) == str(g["s_sha"])
    y = O.ssm_scan(g["x_w"], g["x_s"], layer.w, layer.s, S.SSM_D, n, S.SSM_D, layer.h, 1, S.SSM_T)
    close(y, g["y"], 2e-5, f"scan y N={n}")
    close(layer.h[0], g["h"], 2e-5, f"scan state N={n}")
    # training-mode traces (kernels.h:1158-1170), from a zero state as in the fixture
    h = np.zeros_like(layer.h)
    tr = np.zeros((3,) + layer.h.shape, np.float32)
    y2 = O.ssm_scan(g["x_w"], g["x_s"], layer.w, layer.s, S.SSM_D, n, S.SSM_D, h, 1, S.SSM_T, traces=tr)
    np.testing.assert_array_equal(y2, y)  # the traces do not feed back into y or h
    for k, name in enumerate(("trace_A", "trace_B", "trace_Delta")):
        close(tr[k, 0], g["traces"][k], 1e-4, f"{name} N={n}")
    for out_c, act in S.OUTPROJ_CASES:
        blob_o, bias_o, yin = S.outproj_case(n, out_c, act)
        assert S.sha(blob_o) == str(g[f"op{out_c}_{act}_sha"])
        bw, bs = O.pack_f32(blob_o, True, blob_o.size)
        o = O.outproj(yin[None], bw, bs, bias_o, S.SSM_D, n, out_c, act)[0]
        close(o, g[f"op{out_c}_{act}_out"], 2e-6, f"outproj {out_c}/{act}")


def test_oracle_mamba_block(golden):
    g = golden("mamba_block_N128")
    blobs, biases, _ = S.mamba_block_case()
    assert [S.sha(b) for b in blobs] == [str(v) for v in g["blob_sha"]]
    D, N = S.MB_D, S.MB_N
    layers = [O.MambaLayerRef(D, N, D, 1, blobs[0], biases[0], 1), O.MambaLayerRef(D, N, D, 1, blobs[1], biases[1], 1),
              O.MambaLayerRef(D, N, S.MB_OUT, 2, blobs[2], biases[2], 1)]
    outs = []
    for t in range(S.MB_T):
        xw, xs = g["x_w"][t:t + 1], g["x_s"][t:t + 1]
        o0 = layers[0].forward(xw, xs, 1, 1)
        aw, as_ = O.pack_f32(o0)
        bw, bs = O.residual(aw, as_, xw, xs, 1, D, 1.0, False)
        o1 = layers[1].forward(bw, bs, 1, 1)
        aw, as_ = O.pack_f32(o1)
        outs.append(layers[2].forward(aw.reshape(1, -1), as_.reshape(1, -1), 1, 1)[0])
    close(np.stack(outs), g["out"], 1e-4, "mamba block")


def test_oracle_conv_block(golden):
    g = golden("conv_block")
    masters, biases, _ = S.conv_block_case()
    assert [S.sha(m) for m in masters] == [str(v) for v in g["master_sha"]]
    layers = [O.pack_conv_layer(m, b) for m, b in zip(masters, biases)]
    ow, os_ = O.conv_block(g["x_w"], g["x_s"], layers, 1, S.CB_GEO, main_mult=S.CB_RF)
    check_f(ow, os_, g["out_w"], g["out_s"], flip_rate=5e-3, what="conv block")


def test_oracle_mamba_block_train(golden):
    """Training-mode block (stochastic requants seeded by add_seed, survival
    scaling, one skipped step) against the reference kernels' fixture."""
    g = golden("mamba_block_train_N128")
    blobs, biases, _ = S.mamba_block_case()
    assert [S.sha(b) for b in blobs] == [str(v) for v in g["blob_sha"]]
    D, N = S.MB_D, S.MB_N
    layers = [O.MambaLayerRef(D, N, D, 1, blobs[0], biases[0], 1), O.MambaLayerRef(D, N, D, 1, blobs[1], biases[1], 1),
              O.MambaLayerRef(D, N, S.MB_OUT, 2, blobs[2], biases[2], 1)]
    surv_inv = np.float32(1.0) / np.float32(S.MB_TRAIN_SURV)
    outs = []
    for t in range(S.MB_T):
        survived = t not in S.MB_TRAIN_SKIPPED
        xw, xs = g["x_w"][t:t + 1], g["x_s"][t:t + 1]
        o0 = layers[0].forward(xw, xs, 1, 1)
        aw, as_ = O.pack_f32(o0, True, S.MB_TRAIN_SEED)
        bw, bs = O.residual(aw, as_, xw, xs, 1, D, float(surv_inv) if survived else 1.0, not survived)
        o1 = layers[1].forward(bw, bs, 1, 1)
        aw, as_ = O.pack_f32(o1, True, S.MB_TRAIN_SEED)
        outs.append(layers[2].forward(aw.reshape(1, -1), as_.reshape(1, -1), 1, 1)[0])
    close(np.stack(outs), g["out"], 1e-4, "mamba block, training mode")


def test_oracle_conv_block_train(golden):
    g = golden("conv_block_train")
    masters, biases, _ = S.conv_block_case()
    assert [S.sha(m) for m in masters] == [str(v) for v in g["master_sha"]]
    layers = [O.pack_conv_layer(m, b) for m, b in zip(masters, biases)]
    surv_inv = np.float32(1.0) / np.float32(S.CB_TRAIN_SURV)
    for name, survived in (("survived", True), ("skipped", False)):
        mult = float(np.float32(S.CB_RF) * surv_inv) if survived else S.CB_RF
        ow, os_ = O.conv_block(g["x_w"], g["x_s"], layers, 1, S.CB_GEO, main_mult=mult, skipped=not survived)
        check_f(ow, os_, g[f"{name}_w"], g[f"{name}_s"], flip_rate=5e-3, what=f"conv block, training mode, {name}")


def test_oracle_critic(golden):
    g = golden("critic")
    w1, w2, wl, x = S.critic_case()
    assert [S.sha(a) for a in (w1, w2, wl, x)] == [str(v) for v in g["w_sha"]]
    h = np.zeros((1, 128, 2), np.float32)
    score = O.critic(x, w1, wl, w2, 32, 128, h, 1, x.shape[0])
    close(score, g["score"], 1e-5, "critic score")
    close(h.reshape(-1), g["h"], 1e-5, "critic state")
    # training-mode traces (kernels.h:1731-1751)
    h2 = np.zeros((1, 128, 2), np.float32)
    tw, tl = np.zeros((1, 32, 128, 2), np.float32), np.zeros((1, 128, 32, 2), np.float32)
    score2 = O.critic(x, w1, wl, w2, 32, 128, h2, 1, x.shape[0], traces=(tw, tl))
    np.testing.assert_array_equal(score2, score)
    close(tw.reshape(-1), g["trace_w1"], 1e-4, "critic trace_w1")
    close(tl.reshape(-1), g["trace_lambda"], 1e-4, "critic trace_lambda")


def test_oracle_actions(golden):
    g = golden("actions")
    probs = S.actions_case()
    assert S.sha(probs) == str(g["probs_sha"])
    np.testing.assert_array_equal(O.set_actions(probs[None])[0], g["words"])


def audio_stats(out, ref):
    """Per plane: share of fp16 values that differ, and the largest difference
    (magnitude relative to the plane's max; phase modulo 2 pi, in radians)."""
    out, ref = np.asarray(out, np.float64), np.asarray(ref, np.float64)
    mag_err = np.abs(out[:, 0] - ref[:, 0]).max() / max(np.abs(ref[:, 0]).max(), 1e-30)
    d = np.abs(out[:, 1] - ref[:, 1])
    ph_err = np.minimum(d, np.abs(d - 2 * np.pi)).max()
    return np.mean(out != ref), mag_err, ph_err


def test_oracle_audio(golden):
    g = golden("audio")
    pcm = S.audio_case()
    assert S.sha(pcm) == str(g["pcm_sha"])
    out = np.stack([O.audio_frontend(w, S.AUDIO_DIM)[1] for w in pcm])
    diff_rate, mag_err, ph_err = audio_stats(out, g["out"])
    # Twiddles and phase come from libm sin/cos/atan2 here and from the GPU's
    # __sincosf/atan2f there; both round to fp16, so a handful of values sit
    # one fp16 step apart (measured: 4 of 131072, magnitudes identical).
    assert diff_rate <= 1e-3 and mag_err <= 1e-3 and ph_err <= 2e-3, (diff_rate, mag_err, ph_err)


def test_oracle_screen(golden):
    g = golden("screen")
    bgra = S.screen_case()
    assert S.sha(bgra) == str(g["bgra_sha"])
    plain = O.screen_frontend(bgra)
    train = O.screen_frontend(bgra, True, S.SCREEN_SEED, *S.SCREEN_AUG)
    np.testing.assert_array_equal(plain.view(np.uint16), g["out"][0].view(np.uint16))
    np.testing.assert_array_equal(train.view(np.uint16), g["out"][1].view(np.uint16))


# ---------------------------------------------------------------- training path

def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.mark.parametrize("case", [c[0] for c in S.CONV_BWD_CASES])
def test_oracle_conv_backward(golden, case):
    """The oracle's ConvLayer::backward against the reference's own backward
    kernels (fixture backward_conv): gradients within 1e-5 of their largest
    value (libm in place of the fast-math rsqrt and exp), and the update with
    the reference's square sums reproduces its masters."""
    g = golden("backward_conv")
    _, cin, cout, k, st, din, dout, act = next(c for c in S.CONV_BWD_CASES if c[0] == case)
    master, bias, _, gout = S.conv_bwd_case(case)
    w, s, b = O.pack_conv_layer(master, bias)
    gw, gb, gi = O.conv_backward(g[f"{case}_xw"], g[f"{case}_xs"], w, s, b, master, gout, cin, cout, k, st, din,
                                 dout, act)
    for name, got in (("gw", gw), ("gb", gb), ("gi", gi)):
        ref = g[f"{case}_{name}"]
        assert _rel(got, ref) <= 1e-5, (case, name, _rel(got, ref))
    sw, sb = g[f"{case}_sums"]
    for data, grad, ssum, pen, name in ((master, g[f"{case}_gw"], sw, S.TRAIN_PENALTY, "master"),
                                        (bias, g[f"{case}_gb"], sb, 0.0, "bias")):
        norm = np.sqrt(np.float32(ssum) + np.float32(1 / 8192), dtype=np.float32)
        f = np.float32(1) / norm if norm > 1 else np.float32(1)
        np.testing.assert_array_equal(O.sgd_update(data, grad, f, S.TRAIN_LR, pen), g[f"{case}_{name}"])


@pytest.mark.parametrize("out_c,act", S.MB_BWD_CASES)
def test_oracle_mamba_backward(golden, out_c, act):
    """The oracle's MambaLayer::backward after the fixture's training-mode
    steps (state and traces from the oracle's own forward) against the
    reference's backward kernels."""
    g = golden("backward_mamba_N128")
    tag = f"o{out_c}_a{act}"
    blob, bias, _, gout = S.mamba_bwd_case(out_c, act)
    D, N = S.SSM_D, 128
    E, P = 2 * D, N // 32
    bw, bs = O.pack_f32(blob, True, blob.size)
    h = np.zeros((1, E, P, 2), np.float32)
    tr = np.zeros((3, 1, E, P, 2), np.float32)
    xw, xs = g[f"{tag}_xw"], g[f"{tag}_xs"]
    O.ssm_scan(xw, xs, bw, bs, D, N, out_c, h, 1, S.MB_BWD_T, traces=tr)
    gw, gb, gi = O.mamba_backward(xw[-1:], xs[-1:], h[0], tr[:, 0], blob, bias, gout, D, N, out_c, act)
    for name, got in (("gw", gw), ("gb", gb), ("gi", gi)):
        ref = g[f"{tag}_{name}"]
        assert _rel(got, ref) <= 1e-4, (tag, name, _rel(got, ref))


def test_oracle_critic_backward(golden):
    g = golden("backward_critic")
    w1, w2, wl, x = S.critic_case()
    units, cin = 128, 32
    h = np.zeros((1, units, 2), np.float32)
    tw = np.zeros((1, cin, units, 2), np.float32)
    tl = np.zeros((1, units, cin, 2), np.float32)
    score = O.critic(x, w1, wl, w2, cin, units, h, 1, x.shape[0], traces=(tw, tl))
    assert abs(score[-1] - g["pred"][0]) <= 1e-5 * abs(g["pred"][0])
    gw1, gl, gw2 = O.critic_backward(w2, tw, tl, h, g["pred"][0], S.CRITIC_BWD_REAL, units, cin)
    for name, got in (("gw1", gw1), ("gl", gl), ("gw2", gw2)):
        assert _rel(got, g[name]) <= 1e-4, (name, _rel(got, g[name]))


def test_oracle_clip_factor_block_order():
    """The square sum over one block equals the reference's (no atomics to order)."""
    rng = np.random.default_rng(3)
    gsmall = rng.standard_normal(200).astype(np.float32)
    f, s = O.clip_factor(gsmall, 1)
    assert abs(s - float(np.sum(gsmall.astype(np.float64) ** 2))) <= 1e-5 * s
    assert f == pytest.approx(1.0 / np.sqrt(s + 1 / 8192), rel=1e-6)
