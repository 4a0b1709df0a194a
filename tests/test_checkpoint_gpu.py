"""Checkpoint loading (the reference's .bin format) through the C ABI.

The reference saves each layer as raw little-endian fp32: the master weights,
then the bias (ConvLayer conv_layer.h:15-44, MambaLayer mamba_layer.h:24-53);
the critic as W1, W2, Wlambda (critic.h:23-57); blocks as directories of
those files (conv_block.h:18-21, mamba_block.h:18-20). Here the golden masters
are written in that format, loaded with aic_*_load_file_sync /
aic_*_load_dir_sync, and the packed weights are compared bit for bit with the
reference packer's output (the sha256 of the packed words and exponents the
reference's quantizeKernel produced, stored in the golden fixtures), and the
forwards with the reference kernels' outputs.
"""
import sys

import numpy as np
import pytest
import torch

import aicortex_b200 as A
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


def write_bin(path, *arrays):
    with open(path, "wb") as f:
        for a in arrays:
            f.write(np.ascontiguousarray(a, dtype="<f4").tobytes())


@pytest.mark.parametrize("case", sorted(S.CONV_CASES))
def test_conv_layer_checkpoint_packs_like_the_reference(golden, case, tmp_path):
    g = golden(f"conv_{case}")
    cin, cout, k, st, din, dout, act = S.CONV_CASES[case]
    master, bias, _ = S.conv_case(case)
    write_bin(tmp_path / "layer.bin", master, bias)
    layer = A.ConvLayer(cin, cout, k, st, din, dout, disable_activation=not act)
    layer.load_file(str(tmp_path / "layer.bin"))
    pw, ps, pb = layer.packed()
    assert S.sha(h(pw).view(np.uint32)) == str(g["w_sha"]), "packed words differ from the reference packer"
    assert S.sha(h(ps)) == str(g["s_sha"]), "packed exponents differ from the reference packer"
    np.testing.assert_array_equal(h(pb), bias)


@pytest.mark.parametrize("n", [32, 128, 512])
def test_mamba_layer_checkpoint_packs_like_the_reference(golden, n, tmp_path):
    g = golden(f"ssm_N{n}")
    D = S.SSM_D
    blob, _ = S.ssm_case(n)
    write_bin(tmp_path / "mamba.bin", blob, np.zeros(D, np.float32))
    layer = A.MambaLayer(D, n, D, 1)
    layer.load_file(str(tmp_path / "mamba.bin"))
    pw, ps, _ = layer.packed()
    assert S.sha(h(pw).view(np.uint32)) == str(g["w_sha"]) and S.sha(h(ps)) == str(g["s_sha"])


def test_conv_block_checkpoint_dir(golden, tmp_path):
    """A ConvBlock directory tree loads and runs bit-identically to the reference kernels."""
    g = golden("conv_block")
    masters, biases, _ = S.conv_block_case()
    for name, m, b in zip(A.ConvBlock.LAYER_FILES, masters, biases):
        write_bin(tmp_path / name, m, b)
    cin, mid, cout, st, din, dout, k = S.CB_GEO
    blk = A.ConvBlock(cin, mid, cout, st, din, dout, k, 1.0, S.CB_RF)
    blk.load_dir(str(tmp_path))
    ow, os_ = A.empty_f(dout * dout, cout)
    blk.forward(t(g["x_w"]), t(g["x_s"]), ow, os_, 1)
    np.testing.assert_array_equal(h(ow).view(np.uint32).reshape(-1), g["out_w"])
    np.testing.assert_array_equal(h(os_).reshape(-1), g["out_s"])


def test_mamba_block_checkpoint_dir(golden, tmp_path):
    g = golden("mamba_block_N128")
    blobs, biases, _ = S.mamba_block_case()
    for name, m, b in zip(A.MambaBlock.LAYER_FILES, blobs, biases):
        write_bin(tmp_path / name, m, b)
    blk = A.MambaBlock(S.MB_D, S.MB_N, S.MB_OUT, activation=2)
    blk.load_dir(str(tmp_path))
    blk.set_mode(A.AIC_MAMBA_EXACT)
    blk.bind_state(1)
    out = torch.empty(S.MB_T, S.MB_OUT, dtype=torch.float32, device=DEV)
    blk.forward(t(g["x_w"]), t(g["x_s"]), out, 1, S.MB_T)
    np.testing.assert_array_equal(h(out), g["out"])


def test_critic_checkpoint(golden, tmp_path):
    g = golden("critic")
    w1, w2, wl, x = S.critic_case()
    write_bin(tmp_path / "critic.bin", w1, w2, wl)
    c = A.Critic(32, 128, 1)
    c.load_file(str(tmp_path / "critic.bin"))
    c.bind_state(1)
    score = torch.empty(x.shape[0], dtype=torch.float32, device=DEV)
    c.forward_pooled(t(x), score, 1, x.shape[0])
    np.testing.assert_array_equal(h(score), g["score"])


def test_checkpoint_errors(tmp_path):
    """A missing file and a short file fail with AIC_ERR_IO before any device work."""
    layer = A.ConvLayer(32, 64, 1, 1, 8, 8, disable_activation=True)
    with pytest.raises(A.AicError) as e:
        layer.load_file(str(tmp_path / "missing.bin"))
    assert e.value.status == A._lib.AIC_ERR_IO
    write_bin(tmp_path / "short.bin", np.zeros(32 * 64 - 1, np.float32))
    with pytest.raises(A.AicError) as e:
        layer.load_file(str(tmp_path / "short.bin"))
    assert e.value.status == A._lib.AIC_ERR_IO
