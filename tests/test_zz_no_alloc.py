"""aic_mamba_layer_forward_noalloc: the Mamba layer forward for callers that
cannot allocate device memory (a real-time loop that must not call cudaMalloc,
or a plugin whose host owns all device memory). Its scratch is a fixed 4 MiB
array inside the library instead of a caller-provided workspace.

Checked through the C ABI against aic_mamba_layer_forward (same kernels, so
the outputs must be identical) on two calls in a row, the second continuing
from the recurrent state the first one left. Kept in a file of its own,
collected last.
"""
import ctypes as C

import numpy as np
import pytest
import torch

import aicortex_b200 as A
from aicortex_b200 import workloads as W
from aicortex_b200._lib import AIC_ERR_INVALID, AIC_ERR_STATE, lib

pytestmark = pytest.mark.gpu


def _vp(t):
    return C.c_void_p(t.data_ptr())


def test_noalloc_forward_matches_workspace_forward():
    dev = torch.device("cuda")
    D, N, OUT, B, T = 256, 128, 256, 3, 5
    rng = np.random.default_rng(77)
    blob = torch.from_numpy(W.mamba_blob(rng, D, N, OUT, a_im=None)).to(dev)
    bias = torch.from_numpy(W.bias(rng, OUT)).to(dev)
    ref = A.MambaLayer(D, N, OUT, 1)
    fix = A.MambaLayer(D, N, OUT, 1)
    for layer in (ref, fix):
        layer.load_weights(blob, bias)
        layer.bind_state(B)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call in range(2):
        xw, xs = A.pack_f32(torch.randn(B * T * D, device=dev))
        out_ref = torch.empty(B * T, OUT, dtype=torch.float32, device=dev)
        out_fix = torch.full((B * T, OUT), float("nan"), dtype=torch.float32, device=dev)
        ref.forward(xw, xs, out_ref, B, T)
        st = lib.aic_mamba_layer_forward_noalloc(fix.h, _vp(xw), _vp(xs), _vp(out_fix), B, T, stream)
        assert st == 0, lib.aic_last_error()
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out_fix.cpu().numpy(), out_ref.cpu().numpy(), err_msg=f"call {call}")
        np.testing.assert_array_equal(fix.state_tensor().cpu().numpy(), ref.state_tensor().cpu().numpy())


def test_noalloc_forward_rejects_oversize():
    layer = A.MambaLayer(256, 32, 256, 1)
    layer.bind_state(1)
    # 1 * 4096 rows * 512 channels = 2,097,152 floats > 1,048,576
    st = lib.aic_mamba_layer_forward_noalloc(layer.h, None, None, None, 1, 4096, None)
    assert st == AIC_ERR_INVALID
    assert b"exceeds the fixed scratch" in lib.aic_last_error()


def test_noalloc_forward_at_the_limit():
    """Exactly the 1,048,576-float limit (B=1, T=2048, d_model 256) runs and
    matches the workspace forward; one row more is rejected before any launch."""
    dev = torch.device("cuda")
    D, N, OUT, B, T = 256, 32, 256, 1, 2048
    rng = np.random.default_rng(78)
    blob = torch.from_numpy(W.mamba_blob(rng, D, N, OUT, wd_scale=W.WD_SCALE)).to(dev)
    bias = torch.from_numpy(W.bias(rng, OUT)).to(dev)
    ref = A.MambaLayer(D, N, OUT, 1)
    fix = A.MambaLayer(D, N, OUT, 1)
    for layer in (ref, fix):
        layer.load_weights(blob, bias)
        layer.bind_state(B)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    xw, xs = A.pack_f32(torch.randn(B * T * D, device=dev))
    out_ref = torch.empty(B * T, OUT, dtype=torch.float32, device=dev)
    out_fix = torch.full((B * T, OUT), float("nan"), dtype=torch.float32, device=dev)
    ref.forward(xw, xs, out_ref, B, T)
    assert B * T * 2 * D == 1 << 20
    st = lib.aic_mamba_layer_forward_noalloc(fix.h, _vp(xw), _vp(xs), _vp(out_fix), B, T, stream)
    assert st == 0, lib.aic_last_error()
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out_fix.cpu().numpy(), out_ref.cpu().numpy())
    st = lib.aic_mamba_layer_forward_noalloc(fix.h, _vp(xw), _vp(xs), _vp(out_fix), B, T + 1, stream)
    assert st == AIC_ERR_INVALID


def test_noalloc_forward_checks_like_the_workspace_forward():
    """Unbound state and a batch that differs from the bound one fail the same
    way on both entry points, empty extents included."""
    layer = A.MambaLayer(256, 32, 256, 1)
    st = lib.aic_mamba_layer_forward_noalloc(layer.h, None, None, None, 1, 4, None)
    assert st == AIC_ERR_STATE, lib.aic_last_error()
    layer.bind_state(3)
    for batch, seq in ((0, 4), (2, 0)):
        st_ws = lib.aic_mamba_layer_forward(layer.h, None, None, None, batch, seq, None, None)
        st_na = lib.aic_mamba_layer_forward_noalloc(layer.h, None, None, None, batch, seq, None)
        assert st_ws == st_na == AIC_ERR_INVALID, (batch, seq, st_ws, st_na)
    st = lib.aic_mamba_layer_forward_noalloc(layer.h, None, None, None, 3, 0, None)
    assert st == 0, lib.aic_last_error()
