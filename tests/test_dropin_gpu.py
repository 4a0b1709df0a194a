"""The compiled drop-in boundary: include/aicortex_layers.hpp keeps the
reference's ConvBlock / MambaBlock / Critic constructors, initData, forward and
loadFromFile signatures over the C ABI. tests/dropin/dropin_main.cpp drives
them the way the reference's Cortex does (count arena bytes, allocate once,
carve with initData from reference-format checkpoint trees, one environment
step per forward call). Its outputs are compared with the reference kernels'
golden outputs bit for bit (ConvBlock; MambaBlock over 6 successive calls with
the state carried) and with the CPU oracle for the critic (1e-4 relative: the
oracle uses libm where the kernels use fast-math intrinsics).
"""
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from conftest import GOLDEN, ROOT

sys.path.insert(0, str(GOLDEN))
import golden_specs as S  # noqa: E402

pytestmark = pytest.mark.gpu

CUDA = Path("/usr/local/cuda")


def build_driver(out: Path, d_model: int, d_state: int) -> Path:
    exe = out / "dropin_main"
    cmd = ["g++", "-std=c++17", "-O2", f"-DAIC_LAYERS_D_MODEL={d_model}", f"-DAIC_LAYERS_D_STATE={d_state}",
           "-I", str(ROOT / "include"), "-I", str(CUDA / "include"), str(ROOT / "tests" / "dropin" / "dropin_main.cpp"),
           "-L", str(ROOT / "aicortex_b200"), "-laicortex_b200", "-L", str(CUDA / "lib64"), "-lcudart",
           f"-Wl,-rpath,{ROOT / 'aicortex_b200'}", "-o", str(exe)]
    subprocess.run(cmd, check=True)
    return exe


def write_bin(path: Path, *arrays):
    path.parent.mkdir(parents=True, exist_ok=True)
    with open(path, "wb") as f:
        for a in arrays:
            f.write(np.ascontiguousarray(a, dtype="<f4").tobytes())


def test_dropin_layer_classes(golden, tmp_path):
    import oracle as O
    gc, gm = golden("conv_block"), golden("mamba_block_N128")
    # ConvBlock tree (conv_block.h:18-21) and input frame
    masters, biases, _ = S.conv_block_case()
    for name, m, b in zip(("depthwise_layer.bin", "conv_layer1.bin", "conv_layer2.bin", "residual_layer.bin"),
                          masters, biases):
        write_bin(tmp_path / "conv_block" / name, m, b)
    gc["x_w"].astype("<u4").tofile(tmp_path / "conv_in_w.bin")
    gc["x_s"].astype(np.int8).tofile(tmp_path / "conv_in_s.bin")
    # MambaBlock tree (mamba_block.h:18-20) and its steps
    blobs, mbiases, _ = S.mamba_block_case()
    for name, m, b in zip(("mamba_strategist.bin", "mamba_tactic.bin", "mamba_executor.bin"), blobs, mbiases):
        write_bin(tmp_path / "mamba_block" / name, m, b)
    gm["x_w"].astype("<u4").tofile(tmp_path / "mamba_in_w.bin")
    gm["x_s"].astype(np.int8).tofile(tmp_path / "mamba_in_s.bin")
    # Critic file (critic.h:36-38) and F input frames of 2 x 2 pixels
    w1, w2, wl, _ = S.critic_case()
    write_bin(tmp_path / "critic.bin", w1, w2, wl)
    c_in, units, dim, steps = 32, 128, 2, 5
    rng = np.random.default_rng(910)
    cw, cs = O.pack_f32(rng.standard_normal(steps * dim * dim * c_in).astype(np.float32))
    cw.astype("<u4").tofile(tmp_path / "critic_in_w.bin")
    cs.astype(np.int8).tofile(tmp_path / "critic_in_s.bin")
    cin, mid, cout, st, din, dout, k = S.CB_GEO
    (tmp_path / "spec.txt").write_text(f"conv {cin} {mid} {cout} {st} {din} {dout} {k} {S.CB_RF}\n"
                                       f"mamba {S.MB_T} {S.MB_OUT} 2\n"
                                       f"critic {c_in} {units} {dim} {steps}\n")
    # training (conv_layer.h:150, mamba_layer.h:146): one pointwise-conv frame and
    # one Mamba step through the classes' backward, against the reference kernels
    gbc, gbm = golden("backward_conv"), golden("backward_mamba_N128")
    case = "pw_silu"
    _, tci, tco, tk, tst, tdi, tdo, tact = next(c for c in S.CONV_BWD_CASES if c[0] == case)
    cm, cb, _, cgo = S.conv_bwd_case(case)
    write_bin(tmp_path / "train_conv.bin", cm, cb)
    gbc[f"{case}_xw"].astype("<u4").tofile(tmp_path / "train_conv_in_w.bin")
    gbc[f"{case}_xs"].astype(np.int8).tofile(tmp_path / "train_conv_in_s.bin")
    cgo.astype("<f4").tofile(tmp_path / "train_conv_gout.bin")
    mo, ma = S.MB_BWD_CASES[0]
    mblob, mbias, _, mgo = S.mamba_bwd_case(mo, ma)
    write_bin(tmp_path / "train_mamba.bin", mblob, mbias)
    tag = f"o{mo}_a{ma}"
    gbm[f"{tag}_xw"].astype("<u4").tofile(tmp_path / "train_mamba_in_w.bin")
    gbm[f"{tag}_xs"].astype(np.int8).tofile(tmp_path / "train_mamba_in_s.bin")
    mgo.astype("<f4").tofile(tmp_path / "train_mamba_gout.bin")
    (tmp_path / "train_spec.txt").write_text(
        f"convtrain {tci} {tco} {tk} {tst} {tdi} {tdo} {tact} {S.TRAIN_LR} {S.TRAIN_PENALTY}\n"
        f"mambatrain {S.MB_BWD_T} {mo} {ma} {S.TRAIN_LR} {S.TRAIN_PENALTY}\n")
    exe = build_driver(tmp_path, S.MB_D, S.MB_N)
    res = subprocess.run([str(exe), str(tmp_path)], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stdout + res.stderr
    np.testing.assert_array_equal(np.fromfile(tmp_path / "conv_out_w.bin", dtype="<u4"), gc["out_w"],
                                  err_msg="ConvBlock words")
    np.testing.assert_array_equal(np.fromfile(tmp_path / "conv_out_s.bin", dtype=np.int8), gc["out_s"],
                                  err_msg="ConvBlock exponents")
    np.testing.assert_array_equal(np.fromfile(tmp_path / "mamba_out.bin", dtype="<f4").reshape(S.MB_T, S.MB_OUT),
                                  gm["out"], err_msg="MambaBlock over successive calls")
    pooled = O.gap_f16(cw, cs, steps, dim * dim, c_in)
    ref = O.critic(pooled, w1, wl, w2, c_in, units, np.zeros((1, units, 2), np.float32), 1, steps)
    got = np.fromfile(tmp_path / "critic_out.bin", dtype="<f4")
    assert np.abs(got - ref).max() <= 1e-4 * np.abs(ref).max(), (got, ref)
    # training through the drop-in classes: input gradients bit for bit, host
    # masters updated within the clip factor's rounding (the reference adds its
    # square-sum blocks in arrival order)
    np.testing.assert_array_equal(np.fromfile(tmp_path / "train_conv_gin.bin", dtype="<f4"), gbc[f"{case}_gi"],
                                  err_msg="ConvLayer::backward input gradient")
    np.testing.assert_array_equal(np.fromfile(tmp_path / "train_mamba_gin.bin", dtype="<f4"), gbm[f"{tag}_gi"],
                                  err_msg="MambaLayer::backward input gradient")
    for name, got_path, ref, grad in (("conv", "train_conv_master.bin", gbc[f"{case}_master"], gbc[f"{case}_gw"]),
                                      ("mamba", "train_mamba_master.bin", gbm[f"{tag}_master"], gbm[f"{tag}_gw"])):
        got = np.fromfile(tmp_path / got_path, dtype="<f4").astype(np.float64)
        tol = np.abs(grad.astype(np.float64)) * S.TRAIN_LR * 2e-6 + np.abs(ref.astype(np.float64)) * 2.4e-7
        assert (np.abs(got - ref) <= tol).all(), f"{name}: host masters after backward"
