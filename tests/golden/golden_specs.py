"""Deterministic inputs of the golden fixtures.

Weight masters are regenerated from these specs (numpy PCG64 seeds) instead of
being stored; each fixture records the sha256 of every regenerated array, so
a change of generator is detected rather than silently compared. Used by
make_golden.py (on a GPU box, with the reference kernels) and by the tests.
"""
from __future__ import annotations

import hashlib

import numpy as np

from aicortex_b200 import workloads as W


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


CONV_CASES = {  # name: (in, out, k, stride, din, dout, act)
    "pw_64_128_silu": (64, 128, 1, 1, 16, 16, 1),
    "pw_128_64": (128, 64, 1, 1, 16, 16, 0),
    "pw_64_512_silu": (64, 512, 1, 1, 8, 8, 1),
    "pw_96_96": (96, 96, 1, 1, 8, 8, 0),
    "dense_k2_64_128": (64, 128, 2, 2, 16, 8, 0),
    "dense_k4_32_64": (32, 64, 4, 4, 32, 8, 0),
    "dense_k2_160_288": (160, 288, 2, 2, 8, 4, 0),
    "dw_k3_s2_64": (64, 64, 3, 2, 16, 8, 0),
    "dw_k5_s1_32": (32, 32, 5, 1, 8, 8, 0),
    "dw_k7_s2_96": (96, 96, 7, 2, 16, 8, 0),
}


def pack_master():
    rng = np.random.default_rng(100)
    master = W.conv_weights(rng, 64, 128, 1, False)
    acts = (rng.standard_normal(4096) * 3).astype(np.float32)
    acts[:32] = 0.0          # all-zero group: absmax < eps, scale 1
    acts[32:64] *= 1e-4      # tiny group: clamped dequantisation
    return master, acts


def conv_case(name: str):
    cin, cout, k, st, din, dout, act = CONV_CASES[name]
    seed = 200 + sorted(CONV_CASES).index(name)
    rng = np.random.default_rng(seed)
    dw = k > 1 and k % 2 == 1
    master = W.conv_weights(rng, cin, cout, k, dw)
    bias = W.bias(rng, cout)
    x = rng.standard_normal((din * din, cin)).astype(np.float32)
    return master, bias, x


SSM_D = 256
SSM_T = 8
OUTPROJ_CASES = ((256, 1), (64, 0), (256, 2))


def ssm_case(d_state: int):
    rng = np.random.default_rng(300 + d_state)
    blob = W.mamba_blob(rng, SSM_D, d_state, SSM_D, a_im=None)
    x = rng.standard_normal((SSM_T, SSM_D)).astype(np.float32)
    return blob, x


def outproj_case(d_state: int, out_c: int, act: int):
    rng = np.random.default_rng(400 + d_state + 7 * out_c + act)
    blob = W.mamba_blob(rng, SSM_D, d_state, out_c, a_im=None)
    bias = W.bias(rng, out_c)
    y = (rng.standard_normal(2 * SSM_D) * 2).astype(np.float32)
    return blob, bias, y


MB_D, MB_N, MB_T, MB_OUT = 256, 128, 6, 128


def mamba_block_case():
    rng = np.random.default_rng(500)
    blobs = [W.mamba_blob(rng, MB_D, MB_N, MB_D, a_im=None), W.mamba_blob(rng, MB_D, MB_N, MB_D, a_im=None),
             W.mamba_blob(rng, MB_D, MB_N, MB_OUT, a_im=None)]
    biases = [W.bias(rng, MB_D), W.bias(rng, MB_D), W.bias(rng, MB_OUT)]
    x = rng.standard_normal((MB_T, MB_D)).astype(np.float32)
    return blobs, biases, x


# training-mode forward (mamba_block.h:58-72 with on_training): stochastic
# requant seeded by add_seed, survival scaling 1/p, and one skipped step
MB_TRAIN_SEED, MB_TRAIN_SURV = 4321, 0.8
MB_TRAIN_SKIPPED = (2,)  # time steps run with is_survived = false

CB_GEO = (64, 256, 128, 2, 32, 16, 3)  # in, mid, out, stride, din, dout, dw k
CB_TRAIN_SURV = 0.75  # ConvBlock survival probability in the training-mode fixture
CB_RF = 0.75


def conv_block_case():
    rng = np.random.default_rng(600)
    cin, mid, cout, st, din, dout, k = CB_GEO
    geo = [(cin, cin, k, True), (cin, mid, 1, False), (mid, cout, 1, False), (cin, cout, 2, False)]
    masters = [W.conv_weights(rng, a, b, kk, dw) for (a, b, kk, dw) in geo]
    biases = [W.bias(rng, b) for (_, b, _, _) in geo]
    x = rng.standard_normal((din * din, cin)).astype(np.float32)
    return masters, biases, x


def critic_case():
    rng = np.random.default_rng(700)
    w1, w2, wl = W.critic_weights(rng, 32, 128)
    x = (rng.standard_normal((5, 32)) * 0.5).astype(np.float16)
    return w1, w2, wl, x


def actions_case():
    rng = np.random.default_rng(800)
    probs = rng.random(98).astype(np.float32)
    probs[:8] = rng.random(8).astype(np.float32) * 0.06  # below the 1/16 ceiling of the hash uniform
    return probs


def gap_case():
    rng = np.random.default_rng(900)
    return (rng.standard_normal((64, 256)).astype(np.float32),
            (rng.standard_normal((16, 32)) * 0.7).astype(np.float32))


def residual_case(name: str):
    rng = np.random.default_rng(1000 + (0 if name == "res_160" else 1))
    pos, ch = (64, 160) if name == "res_160" else (1, 256)
    return (rng.standard_normal((pos, ch)).astype(np.float32),
            (rng.standard_normal((pos, ch)) * 0.5).astype(np.float32))


RES_CASES = {"res_160": (64, 160, 8, 0.625), "res_mamba_256": (1, 256, 1, 1.0)}


def stem_case():
    rng = np.random.default_rng(1100)
    return rng.random((3, 64, 64), dtype=np.float32).astype(np.float16)


AUDIO_DIM = 256  # img_resolution of the frames the audio planes are written into


def audio_case():
    """Two 2048-sample int16 windows (1024 stereo frames): a seeded noisy one
    and one with both extremes of int16 at the samples the front-end reads."""
    rng = np.random.default_rng(1200)
    a = np.clip(rng.standard_normal(2048) * 6000, -32768, 32767).astype(np.int16)
    b = rng.integers(-32768, 32768, 2048).astype(np.int16)
    b[0], b[1] = -32768, 32767
    return np.stack([a, b])


SCREEN_DIM = 64
SCREEN_SEED = 0x9E3779B9          # frame seed of the training-mode case (the reference draws it per frame)
SCREEN_AUG = (0.0732421875, 1.1484375)  # brightness, contrast (in the reference's +-0.15 and 1 +- 0.2 ranges)


def screen_case():
    """A seeded BGRA8 frame of SCREEN_DIM^2 pixels."""
    rng = np.random.default_rng(1300)
    return rng.integers(0, 256, (SCREEN_DIM, SCREEN_DIM, 4), dtype=np.uint8)


# ---- training path (one layer step of ConvLayer / MambaLayer / Critic ::backward)
TRAIN_LR, TRAIN_PENALTY = 0.01, 1e-4
# (name, in, out, k, stride, dim_in, dim_out, act). Shapes on which the
# reference's backward kernels stay inside their buffers: pointwise with 256 or
# 512 output channels (fewer read unwritten shared memory and past the master
# weights), depthwise with 256 channels (fewer write past the gradients).
CONV_BWD_CASES = (
    ("pw_silu", 128, 256, 1, 1, 8, 8, 1),
    ("pw_512", 256, 512, 1, 1, 8, 8, 0),
    ("dense_k2", 64, 128, 2, 2, 16, 8, 0),
    ("dense_k2_silu", 64, 256, 2, 2, 8, 4, 1),
    ("dw_k3", 256, 256, 3, 2, 16, 8, 0),
)


def conv_bwd_case(name):
    spec = next(c for c in CONV_BWD_CASES if c[0] == name)
    _, cin, cout, k, st, din, dout, act = spec
    rng = np.random.default_rng(900 + cin + 3 * cout + 7 * k)
    dw = k > 1 and k % 2 == 1
    master = W.conv_weights(rng, cin, cout, k, dw)
    bias = W.bias(rng, cout)
    x = rng.standard_normal((din * din, cin)).astype(np.float32)
    grad_out = (rng.standard_normal((dout * dout, cout)) * 0.1).astype(np.float32)
    return master, bias, x, grad_out


MB_BWD_CASES = ((256, 1), (128, 2))  # (out channels, activation) of the Mamba layer step
MB_BWD_T = 3


def mamba_bwd_case(out_c, act):
    rng = np.random.default_rng(1000 + out_c + act)
    blob = W.mamba_blob(rng, SSM_D, 128, out_c, a_im=None)
    bias = W.bias(rng, out_c)
    x = rng.standard_normal((MB_BWD_T, SSM_D)).astype(np.float32)
    grad_out = (rng.standard_normal(out_c) * 0.1).astype(np.float32)
    return blob, bias, x, grad_out


CRITIC_BWD_REAL = 0.5
