"""GPU parity at the benchmarked sizes, through the C ABI, against the CPU oracle.

  * the full cortex at the benchmark architecture's real dimensions (128x128
    frames, 4 blocks 32-64-128-256-256, 16 states per channel = reference
    d_state 512, 4 Mamba units, actor 64, critic 128) on B=4 x T=8;
  * one Mamba unit (layer D=256 -> requant -> residual, mamba_block.h:60-65)
    over B=1 x T=64 steps from zero state, the single-block configuration;
  * one D=1024 Mamba layer (E=2048) over B=2 x T=256, a sample of the
    long-sequence scan configuration (bf16-rounded N(0,1) inputs).

Tolerance: fp32 outputs within max-abs 1e-3 relative to the tensor's maximum
(the oracle uses libm where the kernels use fast-math intrinsics); packed
outputs as codes + exponents with rare one-step flips at rounding boundaries.
"""
import numpy as np
import pytest
import torch

import aicortex_b200 as A
from aicortex_b200 import fmt, workloads as W

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")
RTOL = 1e-3


def t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def h(x):
    torch.cuda.synchronize()
    return x.cpu().numpy()


def max_rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    assert np.isfinite(a).all() and np.isfinite(b).all()
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def f_mismatch(w_a, s_a, w_b, s_b):
    """(code flip rate, largest code step, exponent mismatch rate) of two packed tensors."""
    ca = fmt.codes(np.ascontiguousarray(w_a).view(np.uint32).reshape(-1)).astype(np.int32)
    cb = fmt.codes(np.ascontiguousarray(w_b).view(np.uint32).reshape(-1)).astype(np.int32)
    sa, sb = np.asarray(s_a).reshape(-1), np.asarray(s_b).reshape(-1)
    same = np.repeat(sa == sb, 32)
    d = np.abs(ca - cb)
    return float(np.mean(d > 0)), int(d[same].max(initial=0)), float(np.mean(sa != sb))


def test_cortex_benchmark_architecture_vs_oracle():
    import oracle as O
    B, T = 4, 8
    desc = W.cortex_desc(batch_chunk=16)
    wts = W.cortex_weights(4)
    planes = W.planes_u01(np.random.default_rng(40), B * T)
    cx = A.Cortex(desc)
    for blk, layers in zip(cx.blocks, wts["blocks"]):
        for lay, (m, b) in zip(blk.layers, layers):
            lay.load_weights(t(m), t(b))
    for u, (m, b) in zip(cx.units, wts["units"]):
        u.load_weights(t(m), t(b))
    cx.actor.load_weights(t(wts["actor"][0]), t(wts["actor"][1]))
    cx.critic.load_weights(*(t(a) for a in wts["critic"]))
    cx.bind_state(B)
    a_ref, c_ref, (frw, frs) = O.cortex_forward(wts, planes, B, T, W.cfg2_blocks(128), 256, W.D_STATE, 64, 128)
    outs = {}
    for mode in (A.AIC_CONV_ORDERED, A.AIC_CONV_SIMT):
        cx.set_conv_mode(mode)
        cx.reset()
        actor = torch.empty(B * T, 64, dtype=torch.float32, device=DEV)
        critic = torch.empty(B * T, dtype=torch.float32, device=DEV)
        fw, fs = A.empty_f(B * T, 256)
        cx.forward(t(planes), B, T, actor, critic, features=(fw, fs))
        outs[mode] = (h(fw), h(fs), h(actor), h(critic))
    fw, fs, actor, critic = outs[A.AIC_CONV_ORDERED]
    flips, step, exps = f_mismatch(fw, fs, frw, frs)
    assert flips <= 1e-2 and step <= 1 and exps <= 1e-2, (flips, step, exps)
    assert max_rel(actor, a_ref) <= RTOL, max_rel(actor, a_ref)
    assert max_rel(critic, c_ref.reshape(critic.shape)) <= RTOL
    for x, y, name in zip(outs[A.AIC_CONV_ORDERED], outs[A.AIC_CONV_SIMT], ("words", "exponents", "actor", "critic")):
        assert np.array_equal(x, y), f"tensor cores (reference order) vs CUDA cores: {name} differ"


def _layer_case(D, B, T, seed, bf16_inputs=False):
    import oracle as O
    rng = np.random.default_rng(seed)
    blob = W.mamba_blob(rng, D, W.D_STATE, D)  # the configuration's W_delta range U(0.001, 0.01)
    bias = W.bias(rng, D)
    x = rng.standard_normal((B * T, D)).astype(np.float32)
    if bf16_inputs:
        x = torch.from_numpy(x).bfloat16().float().numpy()
    xw, xs = O.pack_f32(x)
    xw, xs = xw.reshape(B * T, -1), xs.reshape(B * T, -1)
    ref = O.MambaLayerRef(D, W.D_STATE, D, 1, blob, bias, B)
    layer = A.MambaLayer(D, W.D_STATE, D, 1)
    layer.load_weights(t(blob), t(bias))
    layer.bind_state(B)
    return ref, layer, xw, xs


def test_mamba_unit_single_block_configuration_vs_oracle():
    """D=256 unit, B=1, T=64 from zero state: layer output, carried state and
    the unit output (requant + residual with the unit input)."""
    import oracle as O
    D, B, T = 256, 1, 64
    ref, layer, xw, xs = _layer_case(D, B, T, 0)
    o_ref = ref.forward(xw, xs, B, T)
    out = torch.empty(B * T, D, dtype=torch.float32, device=DEV)
    layer.forward(t(xw.view(np.int32)), t(xs), out, B, T)
    o = h(out)
    assert max_rel(o, o_ref) <= RTOL, max_rel(o, o_ref)
    assert max_rel(h(layer.state_tensor()), ref.h) <= RTOL
    qw, qs = A.pack_f32(out)
    uw, us = A.residual_add(qw, qs, t(xw.view(np.int32)), t(xs), B * T, D)
    rqw, rqs = O.pack_f32(o_ref)
    ruw, rus = O.residual(rqw, rqs, xw, xs, B * T, D, 1.0, False)
    flips, step, exps = f_mismatch(h(uw), h(us), ruw, rus)
    assert flips <= 1e-2 and step <= 1 and exps <= 1e-2, (flips, step, exps)


def test_mamba_layer_long_sequence_sample_vs_oracle():
    """D=1024 (E=2048) layer over B=2 x T=256 steps."""
    D, B, T = 1024, 2, 256
    ref, layer, xw, xs = _layer_case(D, B, T, 3, bf16_inputs=True)
    o_ref = ref.forward(xw, xs, B, T)
    out = torch.empty(B * T, D, dtype=torch.float32, device=DEV)
    layer.forward(t(xw.view(np.int32)), t(xs), out, B, T)
    assert max_rel(h(out), o_ref) <= RTOL, max_rel(h(out), o_ref)
    assert max_rel(h(layer.state_tensor()), ref.h) <= RTOL


def test_cortex_multi_tile_ctas_vs_cuda_cores():
    """The full cortex at its real dimensions in 256-frame conv chunks (B=8 x
    T=32), so that every tensor-core conv CTA runs a long run of row tiles
    (2 to 14 per CTA) as in the benchmark's large launches: features, actor
    and critic of AIC_CONV_ORDERED bit-identical to AIC_CONV_SIMT. Rare
    one-step code flips only show up over this many outputs."""
    B, T = 8, 32
    desc = W.cortex_desc(batch_chunk=256)
    wts = W.cortex_weights(5)
    planes = W.planes_u01(np.random.default_rng(41), B * T)
    cx = A.Cortex(desc)
    for blk, layers in zip(cx.blocks, wts["blocks"]):
        for lay, (m, b) in zip(blk.layers, layers):
            lay.load_weights(t(m), t(b))
    for u, (m, b) in zip(cx.units, wts["units"]):
        u.load_weights(t(m), t(b))
    cx.actor.load_weights(t(wts["actor"][0]), t(wts["actor"][1]))
    cx.critic.load_weights(*(t(a) for a in wts["critic"]))
    cx.bind_state(B)
    outs = {}
    for mode in (A.AIC_CONV_ORDERED, A.AIC_CONV_SIMT):
        cx.set_conv_mode(mode)
        cx.reset()
        actor = torch.empty(B * T, 64, dtype=torch.float32, device=DEV)
        critic = torch.empty(B * T, dtype=torch.float32, device=DEV)
        fw, fs = A.empty_f(B * T, 256)
        cx.forward(t(planes), B, T, actor, critic, features=(fw, fs))
        outs[mode] = (h(fw), h(fs), h(actor), h(critic))
    for x, y, name in zip(outs[A.AIC_CONV_ORDERED], outs[A.AIC_CONV_SIMT], ("words", "exponents", "actor", "critic")):
        assert np.array_equal(x, y), f"tensor cores (reference order) vs CUDA cores over multi-tile CTAs: {name} differ"
