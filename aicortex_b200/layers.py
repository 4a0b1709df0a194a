"""Python mirror of the reference's layer classes over the C ABI.

ConvLayer, ConvBlock, MambaLayer, MambaBlock and Critic keep the reference's
construction (dimensions in the constructor, weights loaded from fp32 masters
or the reference's .bin checkpoint files) and forward() signatures, with
batch and sequence extents added. Device memory (parameters, recurrent state,
workspace) is allocated here with torch and bound to the C handles; all
compute runs in libaicortex_b200.so on the caller's current CUDA stream.

Activation tensors use the packed int4 layout of the reference: words as an
int32 tensor [rows, C // 8] and exponents as an int8 tensor [rows, C // 32].
"""
from __future__ import annotations

import ctypes as C
from typing import Optional, Sequence

import torch

from . import _lib
from ._lib import call

_ALIGN = 256


def _vp(t: Optional[torch.Tensor]) -> Optional[C.c_void_p]:
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream(stream: Optional[torch.cuda.Stream] = None) -> C.c_void_p:
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


class _Arena:
    """A 256-byte aligned device byte buffer owned by torch."""

    def __init__(self, nbytes: int, device: torch.device):
        self.nbytes = int(nbytes)
        self.raw = torch.empty(max(self.nbytes, 1) + _ALIGN, dtype=torch.uint8, device=device)
        self.offset = (-self.raw.data_ptr()) % _ALIGN
        self.ptr = self.raw.data_ptr() + self.offset

    def view(self, ptr: int, count: int, dtype: torch.dtype) -> torch.Tensor:
        """Tensor view of `count` elements at device address `ptr` inside the arena."""
        start = ptr - self.raw.data_ptr()
        nb = count * torch.tensor([], dtype=dtype).element_size()
        assert 0 <= start and start + nb <= self.raw.numel(), "view outside arena"
        return self.raw[start:start + nb].view(dtype)


def _size_out() -> C.c_size_t:
    return C.c_size_t(0)


def _train_views(fn: str, h, arena: "_Arena", counts) -> list:
    """fp32 device views of the pointers a *_train_views entry point returns."""
    ptrs = [C.c_void_p() for _ in counts]
    call(fn, h, *[C.byref(p) for p in ptrs])
    out = []
    for p, n in zip(ptrs, counts):
        if arena is not None and arena.raw.data_ptr() <= p.value < arena.raw.data_ptr() + arena.raw.numel():
            out.append(arena.view(p.value, n, torch.float32))
        else:
            out.append(p.value)
    return out


def empty_f(rows: int, channels: int, device="cuda") -> tuple[torch.Tensor, torch.Tensor]:
    """Uninitialised packed int4 activation tensor pair for rows x channels."""
    return (torch.empty(rows, channels // 8, dtype=torch.int32, device=device),
            torch.empty(rows, channels // 32, dtype=torch.int8, device=device))


class _Handle:
    _destroy = ""

    def __init__(self, handle: C.c_void_p, owned: bool):
        self.h = handle
        self.owned = owned

    def __del__(self):
        if getattr(self, "owned", False) and self.h:
            try:
                getattr(_lib.lib, self._destroy)(self.h)
            except Exception:
                pass
            self.h = None


class ConvLayer(_Handle):
    """ConvLayer (conv_layer.h): depthwise / dense / pointwise quantized conv."""
    _destroy = "aic_conv_layer_destroy"

    def __init__(self, in_channels, out_channels, kernel_size, stride, dim_in, dim_out, disable_activation=False,
                 device="cuda", _handle: Optional[C.c_void_p] = None):
        self.desc = _lib.ConvLayerDesc(in_channels, out_channels, kernel_size, stride, dim_in, dim_out,
                                       int(disable_activation))
        self.device = torch.device(device)
        if _handle is None:
            h = C.c_void_p()
            call("aic_conv_layer_create", C.byref(self.desc), C.byref(h))
            super().__init__(h, True)
            self.params = _Arena(self._param_bytes(), self.device)
            call("aic_conv_layer_bind", self.h, C.c_void_p(self.params.ptr))
        else:
            super().__init__(_handle, False)
            self.params = None
        we, be = C.c_int64(), C.c_int64()
        call("aic_conv_layer_sizes", self.h, C.byref(we), C.byref(be), None)
        self.weight_elems, self.bias_elems = we.value, be.value

    def _param_bytes(self) -> int:
        nb = _size_out()
        call("aic_conv_layer_sizes", self.h, None, None, C.byref(nb))
        return nb.value

    def load_weights(self, master: torch.Tensor, bias: torch.Tensor, stream=None) -> None:
        assert master.dtype == torch.float32 and master.numel() == self.weight_elems and master.is_contiguous()
        assert bias.dtype == torch.float32 and bias.numel() == self.bias_elems
        call("aic_conv_layer_load_weights", self.h, _vp(master), _vp(bias), _stream(stream))

    def load_file(self, path: str, stream=None) -> None:
        call("aic_conv_layer_load_file_sync", self.h, str(path).encode(), _stream(stream))

    def packed(self, arena: Optional[_Arena] = None):
        """(words int32, exponents int8, bias fp32) device views of the bound parameters."""
        arena = arena or self.params
        w, s, b = C.c_void_p(), C.c_void_p(), C.c_void_p()
        call("aic_conv_layer_param_ptrs", self.h, C.byref(w), C.byref(s), C.byref(b))
        g = self.weight_elems // 32
        return (arena.view(w.value, 4 * g, torch.int32), arena.view(s.value, g, torch.int8),
                arena.view(b.value, self.bias_elems, torch.float32))

    def forward(self, x, x_s, out, out_s, frames: int, stream=None) -> None:
        call("aic_conv_layer_forward", self.h, _vp(x), _vp(x_s), _vp(out), _vp(out_s), int(frames), _stream(stream))

    def set_mode(self, mode: int) -> None:
        """AIC_CONV_ORDERED (default, tensor cores, reference order), AIC_CONV_FAST
        (tensor cores, MMA summation order) or AIC_CONV_SIMT (CUDA cores, reference order)."""
        call("aic_conv_layer_set_mode", self.h, int(mode))

    def forward_exact(self, x, x_s, out, out_s, frames: int, stream=None) -> None:
        """Reference accumulation order on CUDA cores (bit-exact with the reference)."""
        call("aic_conv_layer_forward_exact", self.h, _vp(x), _vp(x_s), _vp(out), _vp(out_s), int(frames),
             _stream(stream))

    def train_bind(self, master: torch.Tensor, learning_rate: float, penalty: float, stream=None) -> None:
        """Training state (ConvLayer::backward): fp32 masters, gradients, SGD settings."""
        assert master.dtype == torch.float32 and master.numel() == self.weight_elems and master.is_contiguous()
        nb = _size_out()
        call("aic_conv_layer_train_bytes", self.h, C.byref(nb))
        self.train_state = _Arena(nb.value, self.device)
        call("aic_conv_layer_train_bind", self.h, C.c_void_p(self.train_state.ptr), _vp(master), float(learning_rate),
             float(penalty), _stream(stream))

    def backward(self, grad_out: torch.Tensor, x, x_s, grad_in: Optional[torch.Tensor] = None, stream=None) -> None:
        """One frame: gradients, clipped SGD on masters and biases, re-quantised weights.
        grad_in (fp32 [dim_in^2 * in]) is added to (dense / pointwise) or written (depthwise)."""
        call("aic_conv_layer_backward", self.h, _vp(grad_out), _vp(x), _vp(x_s),
             _vp(grad_in) if grad_in is not None else None, _stream(stream))

    def train_views(self):
        """(master, grad_w, grad_b) fp32 device views and the bias pointer."""
        m, gw, gb, b = _train_views("aic_conv_layer_train_views", self.h, self.train_state,
                                    (self.weight_elems, self.weight_elems, self.bias_elems, self.bias_elems))
        return m, gw, gb


class ConvBlock(_Handle):
    """ConvBlock (conv_block.h): dw -> pw1 (SiLU) -> pw2, shortcut, residual add."""
    _destroy = "aic_conv_block_destroy"
    LAYER_FILES = ("depthwise_layer.bin", "conv_layer1.bin", "conv_layer2.bin", "residual_layer.bin")

    def __init__(self, in_channels, mid_channels, out_channels, stride, dim_in, dim_out, dw_kernel,
                 survival_probability=1.0, residual_factor=1.0, device="cuda", _handle=None, _arena=None):
        self.desc = _lib.ConvBlockDesc(in_channels, mid_channels, out_channels, stride, dim_in, dim_out, dw_kernel,
                                       survival_probability, residual_factor)
        self.device = torch.device(device)
        if _handle is None:
            h = C.c_void_p()
            call("aic_conv_block_create", C.byref(self.desc), C.byref(h))
            super().__init__(h, True)
            nb = _size_out()
            call("aic_conv_block_param_bytes", self.h, C.byref(nb))
            self.params = _Arena(nb.value, self.device)
            call("aic_conv_block_bind", self.h, C.c_void_p(self.params.ptr))
        else:
            super().__init__(_handle, False)
            self.params = _arena
        stride1 = stride if dim_in != dim_out else 1
        geo = [(in_channels, in_channels, dw_kernel, stride1, dim_in, dim_out, True),
               (in_channels, mid_channels, 1, 1, dim_out, dim_out, False),
               (mid_channels, out_channels, 1, 1, dim_out, dim_out, True),
               (in_channels, out_channels, stride1, stride1, dim_in, dim_out, True)]
        self.layers = []
        for i, g in enumerate(geo):
            lh = C.c_void_p()
            call("aic_conv_block_layer", self.h, i, C.byref(lh))
            layer = ConvLayer(*g, device=device, _handle=lh)
            layer.params = self.params
            self.layers.append(layer)
        self._ws = None

    def workspace(self, frames: int) -> _Arena:
        nb = _size_out()
        call("aic_conv_block_workspace_bytes", self.h, int(frames), C.byref(nb))
        if self._ws is None or self._ws.nbytes < nb.value:
            self._ws = _Arena(nb.value, self.device)
        return self._ws

    def load_dir(self, path: str, stream=None) -> None:
        call("aic_conv_block_load_dir_sync", self.h, str(path).encode(), _stream(stream))

    def forward(self, x, x_s, out, out_s, frames: int, train_mode=False, is_survived=True, stream=None) -> None:
        ws = self.workspace(frames)
        call("aic_conv_block_forward", self.h, _vp(x), _vp(x_s), _vp(out), _vp(out_s), int(frames), int(train_mode),
             int(is_survived), C.c_void_p(ws.ptr), _stream(stream))


class MambaLayer(_Handle):
    """MambaLayer (mamba_layer.h): SSM step + out-proj + RMSNorm + bias + activation."""
    _destroy = "aic_mamba_layer_destroy"

    def __init__(self, d_model, d_state, out_channels, activation, device="cuda", _handle=None, _arena=None):
        self.desc = _lib.MambaLayerDesc(d_model, d_state, out_channels, activation)
        self.device = torch.device(device)
        if _handle is None:
            h = C.c_void_p()
            call("aic_mamba_layer_create", C.byref(self.desc), C.byref(h))
            super().__init__(h, True)
            nb = _size_out()
            call("aic_mamba_layer_sizes", self.h, None, None, C.byref(nb))
            self.params = _Arena(nb.value, self.device)
            call("aic_mamba_layer_bind", self.h, C.c_void_p(self.params.ptr))
        else:
            super().__init__(_handle, False)
            self.params = _arena
        we, be = C.c_int64(), C.c_int64()
        call("aic_mamba_layer_sizes", self.h, C.byref(we), C.byref(be), None)
        self.weight_elems, self.bias_elems = we.value, be.value
        self.state = None
        self.batch = None
        self._ws = None

    def load_weights(self, master: torch.Tensor, bias: torch.Tensor, stream=None) -> None:
        assert master.dtype == torch.float32 and master.numel() == self.weight_elems and master.is_contiguous()
        assert bias.dtype == torch.float32 and bias.numel() == self.bias_elems
        call("aic_mamba_layer_load_weights", self.h, _vp(master), _vp(bias), _stream(stream))

    def load_file(self, path: str, stream=None) -> None:
        call("aic_mamba_layer_load_file_sync", self.h, str(path).encode(), _stream(stream))

    def packed(self):
        w, s, b = C.c_void_p(), C.c_void_p(), C.c_void_p()
        call("aic_mamba_layer_param_ptrs", self.h, C.byref(w), C.byref(s), C.byref(b))
        g = self.weight_elems // 32
        return (self.params.view(w.value, 4 * g, torch.int32), self.params.view(s.value, g, torch.int8),
                self.params.view(b.value, self.bias_elems, torch.float32))

    def bind_state(self, batch: int, stream=None) -> None:
        nb = _size_out()
        call("aic_mamba_layer_state_bytes", self.h, int(batch), C.byref(nb))
        self.state = _Arena(nb.value, self.device)
        self.batch = int(batch)
        call("aic_mamba_layer_bind_state", self.h, C.c_void_p(self.state.ptr), int(batch))
        self.reset(stream)

    def state_tensor(self) -> torch.Tensor:
        """Recurrent state view [batch, 2*d_model, d_state // 32, 2] fp32."""
        E, Pn = 2 * self.desc.d_model, self.desc.d_state // 32
        n = self.batch * E * Pn * 2
        return self.state.view(self.state.ptr, n, torch.float32).view(self.batch, E, Pn, 2)

    def bind_traces(self, stream=None) -> None:
        """Training-mode forward: every forward also advances trace_A, trace_B and
        trace_Delta (kernels.h:1158-1170); reset zeroes them with the state."""
        nb = _size_out()
        call("aic_mamba_layer_trace_bytes", self.h, self.batch, C.byref(nb))
        self.traces = _Arena(nb.value, self.device)
        call("aic_mamba_layer_bind_traces", self.h, C.c_void_p(self.traces.ptr), self.batch)
        self.reset(stream)

    def unbind_traces(self) -> None:
        call("aic_mamba_layer_bind_traces", self.h, None, self.batch)
        self.traces = None

    def trace_tensor(self) -> torch.Tensor:
        """[3 (A, B, Delta), batch, 2*d_model, d_state // 32, 2] fp32."""
        E, Pn = 2 * self.desc.d_model, self.desc.d_state // 32
        n = 3 * self.batch * E * Pn * 2
        return self.traces.view(self.traces.ptr, n, torch.float32).view(3, self.batch, E, Pn, 2)

    def train_bind(self, master: torch.Tensor, learning_rate: float, penalty: float, stream=None) -> None:
        """Training state (MambaLayer::backward): fp32 master blob, gradients, SGD settings."""
        assert master.dtype == torch.float32 and master.is_contiguous()
        nb = _size_out()
        call("aic_mamba_layer_train_bytes", self.h, C.byref(nb))
        self.train_state = _Arena(nb.value, self.device)
        self.blob_elems = master.numel()
        call("aic_mamba_layer_train_bind", self.h, C.c_void_p(self.train_state.ptr), _vp(master),
             float(learning_rate), float(penalty), _stream(stream))

    def backward(self, grad_out: torch.Tensor, x, x_s, grad_in: torch.Tensor, stream=None) -> None:
        """The step just run (batch 1, traces bound): gradients, clipped SGD, re-quantised blob."""
        call("aic_mamba_layer_backward", self.h, _vp(grad_out), _vp(x), _vp(x_s), _vp(grad_in), _stream(stream))

    def train_views(self):
        """(master blob, grad blob, grad bias) fp32 device views."""
        m, gw, gb, _ = _train_views("aic_mamba_layer_train_views", self.h, self.train_state,
                                    (self.blob_elems, self.blob_elems, self.desc.out_channels, 0))
        return m, gw, gb

    def train_bias(self) -> torch.Tensor:
        """The fp32 bias the backward updates, as a device view."""
        b = C.c_void_p()
        call("aic_mamba_layer_train_views", self.h, None, None, None, C.byref(b))
        return self.params.view(b.value, self.desc.out_channels, torch.float32)

    def reset(self, stream=None) -> None:
        call("aic_mamba_layer_reset_state", self.h, _stream(stream))

    def workspace(self, rows: int) -> _Arena:
        nb = _size_out()
        call("aic_mamba_layer_workspace_bytes", self.h, int(rows), C.byref(nb))
        if self._ws is None or self._ws.nbytes < nb.value:
            self._ws = _Arena(nb.value, self.device)
        return self._ws

    def outproj(self, y: torch.Tensor, out: torch.Tensor, rows: int, stream=None) -> None:
        call("aic_mamba_layer_outproj", self.h, _vp(y), _vp(out), int(rows), _stream(stream))

    def set_mode(self, mode: int) -> None:
        """AIC_MAMBA_TENSOR (default) or AIC_MAMBA_EXACT out-projection."""
        call("aic_mamba_layer_set_mode", self.h, int(mode))

    def scan(self, x, x_s, y, batch: int, seq: int, split: bool = False, stream=None) -> None:
        """The SSM scan alone into y (256-byte aligned, batch*seq*2*d_model*4 bytes)."""
        call("aic_mamba_layer_scan", self.h, _vp(x), _vp(x_s), _vp(y), int(batch), int(seq), int(split),
             _stream(stream))

    def outproj_split(self, y_planes, out: torch.Tensor, rows: int, stream=None) -> None:
        """The tensor-core out-projection of split-bf16 y planes (as scan(split=True) writes them)."""
        call("aic_mamba_layer_outproj_split", self.h, _vp(y_planes), _vp(out), int(rows), _stream(stream))

    def forward(self, x, x_s, out, batch: int, seq: int, stream=None) -> None:
        ws = self.workspace(batch * seq)
        call("aic_mamba_layer_forward", self.h, _vp(x), _vp(x_s), _vp(out), int(batch), int(seq), C.c_void_p(ws.ptr),
             _stream(stream))


class MambaBlock(_Handle):
    """MambaBlock (mamba_block.h): strategist -> requant -> residual -> tactic -> requant -> executor."""
    _destroy = "aic_mamba_block_destroy"
    LAYER_FILES = ("mamba_strategist.bin", "mamba_tactic.bin", "mamba_executor.bin")

    def __init__(self, d_model, d_state, out_channels, activation=2, survival_probability=1.0, residual_factor=1.0,
                 device="cuda"):
        self.desc = _lib.MambaBlockDesc(d_model, d_state, out_channels, activation, survival_probability,
                                        residual_factor)
        self.device = torch.device(device)
        h = C.c_void_p()
        call("aic_mamba_block_create", C.byref(self.desc), C.byref(h))
        super().__init__(h, True)
        nb = _size_out()
        call("aic_mamba_block_param_bytes", self.h, C.byref(nb))
        self.params = _Arena(nb.value, self.device)
        call("aic_mamba_block_bind", self.h, C.c_void_p(self.params.ptr))
        outs = (d_model, d_model, out_channels)
        acts = (1, 1, activation)
        self.layers = []
        for i in range(3):
            lh = C.c_void_p()
            call("aic_mamba_block_layer", self.h, i, C.byref(lh))
            self.layers.append(MambaLayer(d_model, d_state, outs[i], acts[i], device=device, _handle=lh,
                                          _arena=self.params))
        self.state = None
        self.batch = None
        self._ws = None

    def bind_state(self, batch: int, stream=None) -> None:
        nb = _size_out()
        call("aic_mamba_block_state_bytes", self.h, int(batch), C.byref(nb))
        self.state = _Arena(nb.value, self.device)
        self.batch = int(batch)
        call("aic_mamba_block_bind_state", self.h, C.c_void_p(self.state.ptr), int(batch))
        self.reset(stream)

    def bind_traces(self, stream=None) -> None:
        """Training-mode forward for all three layers (their traces carved in order)."""
        nb = _size_out()
        call("aic_mamba_block_trace_bytes", self.h, self.batch, C.byref(nb))
        self.traces = _Arena(nb.value, self.device)
        call("aic_mamba_block_bind_traces", self.h, C.c_void_p(self.traces.ptr), self.batch)
        self.reset(stream)

    def reset(self, stream=None) -> None:
        call("aic_mamba_block_reset_state", self.h, _stream(stream))

    def set_mode(self, mode: int) -> None:
        """AIC_MAMBA_TENSOR (default) or AIC_MAMBA_EXACT for the three layers."""
        call("aic_mamba_block_set_mode", self.h, int(mode))

    def load_dir(self, path: str, stream=None) -> None:
        call("aic_mamba_block_load_dir_sync", self.h, str(path).encode(), _stream(stream))

    def forward(self, x, x_s, out, batch: int, seq: int, on_training=False, add_seed=0, is_survived=True,
                stream=None) -> None:
        nb = _size_out()
        call("aic_mamba_block_workspace_bytes", self.h, int(batch * seq), C.byref(nb))
        if self._ws is None or self._ws.nbytes < nb.value:
            self._ws = _Arena(nb.value, self.device)
        call("aic_mamba_block_forward", self.h, _vp(x), _vp(x_s), _vp(out), int(batch), int(seq), int(on_training),
             int(add_seed), int(is_survived), C.c_void_p(self._ws.ptr), _stream(stream))


class Critic(_Handle):
    """Critic (critic.h): pooled fp16 features -> gated leaky complex cell -> score."""
    _destroy = "aic_critic_destroy"

    def __init__(self, in_channels, units, dim_in, device="cuda", _handle=None, _arena=None):
        self.desc = _lib.CriticDesc(in_channels, units, dim_in)
        self.device = torch.device(device)
        if _handle is None:
            h = C.c_void_p()
            call("aic_critic_create", C.byref(self.desc), C.byref(h))
            super().__init__(h, True)
            nb = _size_out()
            call("aic_critic_param_bytes", self.h, C.byref(nb))
            self.params = _Arena(nb.value, self.device)
            call("aic_critic_bind", self.h, C.c_void_p(self.params.ptr))
        else:
            super().__init__(_handle, False)
            self.params = _arena
        self.state = None
        self.batch = None
        self._ws = None

    def load_weights(self, w1: torch.Tensor, w2: torch.Tensor, wl: torch.Tensor, stream=None) -> None:
        call("aic_critic_load_weights", self.h, _vp(w1), _vp(w2), _vp(wl), _stream(stream))

    def load_file(self, path: str, stream=None) -> None:
        call("aic_critic_load_file_sync", self.h, str(path).encode(), _stream(stream))

    def bind_state(self, batch: int, stream=None) -> None:
        nb = _size_out()
        call("aic_critic_state_bytes", self.h, int(batch), C.byref(nb))
        self.state = _Arena(nb.value, self.device)
        self.batch = int(batch)
        call("aic_critic_bind_state", self.h, C.c_void_p(self.state.ptr), int(batch))
        self.reset(stream)

    def bind_traces(self, stream=None) -> None:
        """Training-mode forward: every step also advances the eligibility traces of
        W1 and Wlambda (kernels.h:1731-1751); reset zeroes them with the state."""
        nb = _size_out()
        call("aic_critic_trace_bytes", self.h, self.batch, C.byref(nb))
        self.traces = _Arena(nb.value, self.device)
        call("aic_critic_bind_traces", self.h, C.c_void_p(self.traces.ptr), self.batch)
        self.reset(stream)

    def trace_tensors(self):
        """(trace_w1 [batch, in, units, 2], trace_lambda [batch, units, in, 2]) fp32 views."""
        cin, units = self.desc.in_channels, self.desc.units
        n = self.batch * cin * units * 2
        t = self.traces.view(self.traces.ptr, 2 * n, torch.float32)
        return t[:n].view(self.batch, cin, units, 2), t[n:].view(self.batch, units, cin, 2)

    def reset(self, stream=None) -> None:
        call("aic_critic_reset_state", self.h, _stream(stream))

    def _workspace(self, rows: int) -> _Arena:
        nb = _size_out()
        call("aic_critic_workspace_bytes", self.h, int(rows), C.byref(nb))
        if self._ws is None or self._ws.nbytes < nb.value:
            self._ws = _Arena(nb.value, self.device)
        return self._ws

    def forward_pooled(self, pooled: torch.Tensor, score, batch: int, seq: int, stream=None) -> None:
        assert pooled.dtype == torch.float16
        self._workspace(batch * seq)
        call("aic_critic_forward_pooled", self.h, _vp(pooled), _vp(score), int(batch), int(seq),
             C.c_void_p(self._ws.ptr), _stream(stream))

    def forward(self, x, x_s, score, batch: int, seq: int, stream=None) -> None:
        self._workspace(batch * seq)
        call("aic_critic_forward", self.h, _vp(x), _vp(x_s), _vp(score), int(batch), int(seq),
             C.c_void_p(self._ws.ptr), _stream(stream))

    def train_bind(self, learning_rate: float, penalty: float) -> None:
        """Training state (Critic::backward): gradients and SGD settings; W1, W2 and
        Wlambda are updated in place."""
        nb = _size_out()
        call("aic_critic_train_bytes", self.h, C.byref(nb))
        self.train_state = _Arena(nb.value, self.device)
        call("aic_critic_train_bind", self.h, C.c_void_p(self.train_state.ptr), float(learning_rate), float(penalty))

    def backward(self, pred_score: torch.Tensor, real_score: float, stream=None) -> None:
        """The step just run (batch 1, traces bound): pred_score the device score it wrote."""
        call("aic_critic_backward", self.h, _vp(pred_score), float(real_score), _stream(stream))

    def train_views(self):
        """(grad_w1, grad_w2, grad_lambda) fp32 device views."""
        n1 = 2 * self.desc.in_channels * self.desc.units
        return tuple(_train_views("aic_critic_train_views", self.h, self.train_state, (n1, 2 * self.desc.units, n1)))

    def weights(self):
        """(w1, w2, wlambda) fp32 device views of the bound parameters (laid out
        in order, each at a 256-byte boundary)."""
        n1, n2 = 2 * self.desc.in_channels * self.desc.units, 2 * self.desc.units

        def up(b):
            return (b + 255) // 256 * 256
        o2 = up(4 * n1)
        o3 = up(o2 + 4 * n2)
        base = self.params.ptr
        return (self.params.view(base, n1, torch.float32), self.params.view(base + o2, n2, torch.float32),
                self.params.view(base + o3, n1, torch.float32))


class Cortex(_Handle):
    """Full forward: stem -> conv blocks -> GAP -> Mamba units -> actor (+ critic)."""
    _destroy = "aic_cortex_destroy"

    def __init__(self, desc: _lib.CortexDesc, device="cuda"):
        self.desc = desc
        self.device = torch.device(device)
        h = C.c_void_p()
        call("aic_cortex_create", C.byref(self.desc), C.byref(h))
        super().__init__(h, True)
        nb = _size_out()
        call("aic_cortex_param_bytes", self.h, C.byref(nb))
        self.params = _Arena(nb.value, self.device)
        call("aic_cortex_bind", self.h, C.c_void_p(self.params.ptr))
        self.blocks = []
        for i in range(desc.n_blocks):
            bh = C.c_void_p()
            call("aic_cortex_block", self.h, i, C.byref(bh))
            b = desc.blocks[i]
            self.blocks.append(ConvBlock(b.in_channels, b.mid_channels, b.out_channels, b.stride, b.dim_in, b.dim_out,
                                         b.dw_kernel, b.survival_probability, b.residual_factor, device=device,
                                         _handle=bh, _arena=self.params))
        self.units = []
        for i in range(desc.n_units):
            uh = C.c_void_p()
            call("aic_cortex_unit", self.h, i, C.byref(uh))
            self.units.append(MambaLayer(desc.d_model, desc.d_state, desc.d_model, 1, device=device, _handle=uh,
                                         _arena=self.params))
        ah = C.c_void_p()
        call("aic_cortex_actor", self.h, C.byref(ah))
        self.actor = MambaLayer(desc.d_model, desc.d_state, desc.actor_out, desc.actor_activation, device=device,
                                _handle=ah, _arena=self.params)
        self.critic = None
        if desc.critic_units > 0:
            ch = C.c_void_p()
            call("aic_cortex_critic", self.h, C.byref(ch))
            self.critic = Critic(desc.d_model, desc.critic_units, 1, device=device, _handle=ch, _arena=self.params)
        self.state = None
        self.batch = None
        self._ws = None

    def bind_state(self, batch: int, stream=None) -> None:
        nb = _size_out()
        call("aic_cortex_state_bytes", self.h, int(batch), C.byref(nb))
        self.state = _Arena(nb.value, self.device)
        self.batch = int(batch)
        call("aic_cortex_bind_state", self.h, C.c_void_p(self.state.ptr), int(batch))
        self.reset(stream)

    def reset(self, stream=None) -> None:
        call("aic_cortex_reset_state", self.h, _stream(stream))

    def set_exact(self, exact: bool) -> None:
        """True: every quantized conv on CUDA cores with the reference kernels' structure
        (AIC_CONV_SIMT) and the reference-order Mamba out-projection (AIC_MAMBA_EXACT);
        False: the defaults AIC_CONV_ORDERED (bit-identical too) and AIC_MAMBA_TENSOR."""
        call("aic_cortex_set_exact", self.h, int(exact))

    def set_mamba_mode(self, mode: int) -> None:
        """AIC_MAMBA_TENSOR (default) or AIC_MAMBA_EXACT for every Mamba layer."""
        call("aic_cortex_set_mamba_mode", self.h, int(mode))

    def set_conv_mode(self, mode: int) -> None:
        """AIC_CONV_ORDERED (default), AIC_CONV_FAST or AIC_CONV_SIMT for every conv layer."""
        call("aic_cortex_set_conv_mode", self.h, int(mode))

    def workspace_bytes(self, batch: int, seq: int) -> int:
        nb = _size_out()
        call("aic_cortex_workspace_bytes", self.h, int(batch), int(seq), C.byref(nb))
        return nb.value

    def forward(self, planes: torch.Tensor, batch: int, seq: int, actor_out: torch.Tensor,
                critic_out: Optional[torch.Tensor] = None, features: Optional[Sequence[torch.Tensor]] = None,
                stream=None) -> int:
        """Runs the forward; returns the number of kernel launches issued."""
        assert planes.dtype == torch.float16 and planes.is_contiguous()
        nb = self.workspace_bytes(batch, seq)
        if self._ws is None or self._ws.nbytes < nb:
            self._ws = _Arena(nb, self.device)
        fw, fs = (features if features is not None else (None, None))
        call("aic_cortex_forward", self.h, _vp(planes), int(batch), int(seq), _vp(actor_out), _vp(critic_out),
             _vp(fw), _vp(fs), C.c_void_p(self._ws.ptr), _stream(stream))
        n = C.c_int64()
        call("aic_cortex_last_launches", self.h, C.byref(n))
        return n.value


def grad_clip_factor(grad: torch.Tensor, stream=None) -> torch.Tensor:
    """[clip factor, square sum] of a gradient (clip_op of the layer classes), on the device."""
    n = grad.numel()
    nf = C.c_int64()
    call("aic_grad_clip_partials", int(n), C.byref(nf))
    partial = torch.empty(nf.value, dtype=torch.float32, device=grad.device)
    factor = torch.empty(2, dtype=torch.float32, device=grad.device)
    call("aic_grad_clip_factor", _vp(grad), int(n), _vp(partial), _vp(factor), _stream(stream))
    return factor


def sgd_update(data: torch.Tensor, grad: torch.Tensor, factor: torch.Tensor, learning_rate: float, penalty: float,
               stream=None) -> None:
    """updateParamsKernel: data = grad * (-lr * factor[0]) + data * (1 - lr * penalty), in place."""
    call("aic_sgd_update", _vp(data), _vp(grad), int(data.numel()), _vp(factor), float(learning_rate), float(penalty),
         _stream(stream))


def residual_backward(grad_next: torch.Tensor, grad_res: torch.Tensor, survival_prob_inv: float,
                      residual_factor: float, stream=None) -> None:
    """residualAddBwdKernel: grad_res = grad_next; grad_next *= survival_prob_inv * residual_factor."""
    call("aic_residual_backward", _vp(grad_next), _vp(grad_res), int(grad_next.numel()), float(survival_prob_inv),
         float(residual_factor), _stream(stream))


def pack_f32(x: torch.Tensor, stochastic=False, add_idx=0, stream=None):
    """quantizeKernel on a float32 device tensor (numel % 32 == 0)."""
    assert x.dtype == torch.float32 and x.is_contiguous() and x.numel() % 32 == 0
    g = x.numel() // 32
    w = torch.empty(4 * g, dtype=torch.int32, device=x.device)
    s = torch.empty(g, dtype=torch.int8, device=x.device)
    call("aic_pack_f32", _vp(x), x.numel(), _vp(w), _vp(s), int(stochastic), int(add_idx), _stream(stream))
    return w, s


def stem_pack(planes: torch.Tensor, channels: int, stream=None):
    """quantizeNCHWtoNHWCKernel over frames: planes fp16 [frames, P, dim, dim]."""
    assert planes.dtype == torch.float16 and planes.is_contiguous() and planes.dim() == 4
    f, p, dim, _ = planes.shape
    w, s = empty_f(f * dim * dim, channels, planes.device)
    call("aic_stem_pack", _vp(planes), f, p, channels, dim, _vp(w), _vp(s), _stream(stream))
    return w, s


def residual_add(main_w, main_s, res_w, res_s, positions, channels, main_mult=1.0, skipped=False, stream=None):
    w, s = empty_f(positions, channels, res_w.device)
    call("aic_residual_add", _vp(main_w), _vp(main_s), _vp(res_w), _vp(res_s), _vp(w), _vp(s), int(positions),
         int(channels), float(main_mult), int(skipped), _stream(stream))
    return w, s


def gap(x_w, x_s, frames, hw, channels, quantize=True, stream=None):
    out = torch.empty(frames, channels, dtype=torch.float32, device=x_w.device)
    qw, qs = empty_f(frames, channels, x_w.device) if quantize else (None, None)
    call("aic_gap", _vp(x_w), _vp(x_s), int(frames), int(hw), int(channels), _vp(out), _vp(qw), _vp(qs),
         _stream(stream))
    return out, qw, qs


def gap_f16(x_w, x_s, frames, hw, channels, stream=None):
    out = torch.empty(frames, channels, dtype=torch.float16, device=x_w.device)
    call("aic_gap_f16", _vp(x_w), _vp(x_s), int(frames), int(hw), int(channels), _vp(out), _stream(stream))
    return out


def set_actions(probs: torch.Tensor, stream=None) -> torch.Tensor:
    assert probs.dtype == torch.float32 and probs.dim() == 2 and probs.is_contiguous()
    rows, count = probs.shape
    out = torch.empty(rows, (count + 63) // 64, dtype=torch.int64, device=probs.device)
    call("aic_set_actions", _vp(probs), rows, count, _vp(out), _stream(stream))
    return out


def screen_frontend(bgra: torch.Tensor, frame: torch.Tensor, first_channel: int = 0, train: bool = False,
                    frame_seed: int = 0, brightness: float = 0.0, contrast: float = 1.0, stream=None) -> None:
    """Screen front-end (cs.cu): uint8 BGRA [dim, dim, 4] -> fp16 planes B, G, R, A at
    frame[first_channel : first_channel + 4] (fp16 [C][dim][dim]); train adds the
    reference's pixel dropout (seeded by frame_seed) and brightness/contrast augmentation."""
    assert bgra.dtype == torch.uint8 and bgra.is_contiguous() and bgra.numel() == 4 * frame.shape[-1] ** 2
    assert frame.dtype == torch.float16 and frame.dim() == 3 and frame.is_contiguous()
    assert 0 <= first_channel and first_channel + 4 <= frame.shape[0] and frame.shape[1] == frame.shape[2]
    call("aic_screen_frontend", _vp(bgra), _vp(frame), int(frame.shape[-1]), int(first_channel), int(bool(train)),
         C.c_uint32(frame_seed & 0xFFFFFFFF), float(brightness), float(contrast), _stream(stream))


def audio_frontend(pcm: torch.Tensor, frame: torch.Tensor, first_channel: int = 4, stream=None) -> None:
    """Audio front-end (ca.cu): 2048 int16 PCM samples -> |FFT| and phase planes
    written to frame[first_channel] and frame[first_channel + 1] (fp16 [C][dim][dim])."""
    assert pcm.dtype == torch.int16 and pcm.numel() == 2048 and pcm.is_contiguous()
    assert frame.dtype == torch.float16 and frame.dim() == 3 and frame.is_contiguous()
    assert 0 <= first_channel and first_channel + 2 <= frame.shape[0] and frame.shape[1] == frame.shape[2]
    nb = _size_out()
    call("aic_audio_workspace_bytes", C.byref(nb))
    ws = _Arena(nb.value, frame.device)
    if stream is not None:
        ws.raw.record_stream(stream)  # the workspace is freed on return while the kernels may still run
    call("aic_audio_frontend", _vp(pcm), _vp(frame), int(frame.shape[-1]), int(first_channel), C.c_void_p(ws.ptr),
         _stream(stream))
