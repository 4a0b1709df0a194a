"""CPU oracle of the AICortex inference hot path -- TEST INFRASTRUCTURE ONLY.

numpy front-end over oracle/_build/liboracle.so (oracle/aic_oracle.c, a
plain-C restatement of the reference kernels) plus the layer/block
compositions of the reference headers. Only tests/, __graft_entry__.smoke()
and bench.py's CPU legs import this package; it is the checker, never the
thing measured as the product.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle.so"


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def _load() -> C.CDLL:
    if not LIB_PATH.exists():
        build()
    lib = C.CDLL(str(LIB_PATH))
    P, I64, I32, F = C.c_void_p, C.c_int64, C.c_int, C.c_float
    sigs = {
        "orc_unique_seed": ([C.c_uint32, C.c_int32], C.c_uint32),
        "orc_uniform": ([C.c_uint32, F], F),
        "orc_quantize_scale": ([F], C.c_int8),
        "orc_dequantize_scale": ([C.c_int8], F),
        "orc_pack_f32": ([P, I64, P, P, I32, C.c_int32], None),
        "orc_stem_pack": ([P, I64, I32, I32, I32, P, P], None),
        "orc_conv_pw": ([P, P, P, P, P, P, P, I64, I32, I32, I32], None),
        "orc_conv_dense": ([P, P, P, P, P, P, P, I64, I32, I32, I32, I32, I32, I32, I32], None),
        "orc_conv_dw": ([P, P, P, P, P, P, P, I64, I32, I32, I32, I32, I32], None),
        "orc_residual": ([P, P, P, P, P, P, I64, I32, F, I32], None),
        "orc_gap_f32": ([P, P, I64, I32, I32, P], None),
        "orc_gap_f16": ([P, P, I64, I32, I32, P], None),
        "orc_mamba_blob_elems": ([I32, I32, I32], I64),
        "orc_ssm_scan": ([P, P, P, P, I32, I32, I32, P, P, I32, I32], None),
        "orc_ssm_scan_traced": ([P, P, P, P, I32, I32, I32, P, P, P, I32, I32], None),
        "orc_outproj": ([P, P, P, P, I32, I32, I32, I32, I64, P], None),
        "orc_critic": ([P, P, P, P, I32, I32, P, P, I32, I32], None),
        "orc_critic_traced": ([P, P, P, P, I32, I32, P, P, P, P, I32, I32], None),
        "orc_set_actions": ([P, I64, I32, P], None),
        "orc_num_threads": ([], I32),
        "orc_audio_pcm_to_half": ([P, I32, P], None),
        "orc_resize_half": ([P, P, I32, I32, I32, I32], None),
        "orc_fft_rows": ([P, I32, P], None),
        "orc_fft_cols": ([P, I32, P], None),
        "orc_screen_frontend": ([P, I32, I32, C.c_uint32, C.c_float, C.c_float, P], None),
        "orc_sgd_update": ([P, P, I64, F, F, F], None),
        "orc_clip_factor": ([P, I64, I32, P], F),
        "orc_conv_backward": ([P, P, P, P, P, P, P, I32, I32, I32, I32, I32, I32, I32, P, P, P], None),
        "orc_mamba_backward": ([P, P, P, P, P, P, P, P, P, I32, I32, I32, I32, P, P, P], None),
        "orc_critic_backward": ([P, P, P, P, F, F, I32, I32, P, P, P], None),
    }
    for name, (args, res) in sigs.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    return lib


lib = _load()


def _p(a: np.ndarray) -> C.c_void_p:
    assert a.flags["C_CONTIGUOUS"]
    return C.c_void_p(a.ctypes.data)


def num_threads() -> int:
    return lib.orc_num_threads()


def pack_f32(x: np.ndarray, stochastic: bool = False, add_idx: int = 0):
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    g = x.size // 32
    w = np.zeros(4 * g, dtype=np.uint32)
    s = np.zeros(g, dtype=np.int8)
    lib.orc_pack_f32(_p(x), x.size, _p(w), _p(s), int(stochastic), int(add_idx))
    return w, s


def stem_pack(planes_f16: np.ndarray, channels: int = 32):
    planes = np.ascontiguousarray(planes_f16, dtype=np.float16)
    f, p, dim, _ = planes.shape
    w = np.zeros((f * dim * dim, channels // 8), dtype=np.uint32)
    s = np.zeros((f * dim * dim, channels // 32), dtype=np.int8)
    lib.orc_stem_pack(_p(planes.view(np.uint16)), f, p, channels, dim, _p(w), _p(s))
    return w, s


def conv(x_w, x_s, w_w, w_s, bias, frames, in_c, out_c, k, stride, d_in, d_out, act):
    """ConvLayer::forward dispatch (conv_layer.h:102-149)."""
    depthwise = k > 1 and k % 2 == 1
    out_w = np.zeros((frames * d_out * d_out, out_c // 8), dtype=np.uint32)
    out_s = np.zeros((frames * d_out * d_out, out_c // 32), dtype=np.int8)
    args = [_p(np.ascontiguousarray(x_w, np.uint32)), _p(np.ascontiguousarray(x_s, np.int8)),
            _p(np.ascontiguousarray(w_w, np.uint32)), _p(np.ascontiguousarray(w_s, np.int8)),
            _p(np.ascontiguousarray(bias, np.float32)), _p(out_w), _p(out_s)]
    if depthwise:
        lib.orc_conv_dw(*args, frames, in_c, k, stride, d_in, d_out)
    elif k == 1:
        lib.orc_conv_pw(*args, frames * d_out * d_out, in_c, out_c, int(act))
    else:
        lib.orc_conv_dense(*args, frames, in_c, out_c, k, stride, d_in, d_out, int(act))
    return out_w, out_s


def residual(main_w, main_s, res_w, res_s, positions, channels, main_mult=1.0, skipped=False):
    out_w = np.zeros((positions, channels // 8), dtype=np.uint32)
    out_s = np.zeros((positions, channels // 32), dtype=np.int8)
    lib.orc_residual(_p(np.ascontiguousarray(main_w, np.uint32)), _p(np.ascontiguousarray(main_s, np.int8)),
                     _p(np.ascontiguousarray(res_w, np.uint32)), _p(np.ascontiguousarray(res_s, np.int8)),
                     _p(out_w), _p(out_s), positions, channels, float(main_mult), int(skipped))
    return out_w, out_s


def gap_f32(x_w, x_s, frames, hw, channels):
    out = np.zeros((frames, channels), dtype=np.float32)
    lib.orc_gap_f32(_p(np.ascontiguousarray(x_w, np.uint32)), _p(np.ascontiguousarray(x_s, np.int8)), frames, hw,
                    channels, _p(out))
    return out


def gap_f16(x_w, x_s, frames, hw, channels):
    out = np.zeros((frames, channels), dtype=np.uint16)
    lib.orc_gap_f16(_p(np.ascontiguousarray(x_w, np.uint32)), _p(np.ascontiguousarray(x_s, np.int8)), frames, hw,
                    channels, _p(out))
    return out.view(np.float16)


def ssm_scan(x_w, x_s, blob_w, blob_s, d_model, d_state, out, h, B, T, traces=None):
    """Returns y [B*T][2*d_model]; h [B][E][d_state/32][2] is updated in place,
    and so are the training-mode traces [3][B][E][d_state/32][2] when given."""
    E = 2 * d_model
    y = np.zeros((B * T, E), dtype=np.float32)
    assert h.dtype == np.float32 and h.flags["C_CONTIGUOUS"]
    args = [_p(np.ascontiguousarray(x_w, np.uint32)), _p(np.ascontiguousarray(x_s, np.int8)),
            _p(np.ascontiguousarray(blob_w, np.uint32)), _p(np.ascontiguousarray(blob_s, np.int8)), d_model, d_state, out,
            _p(h)]
    if traces is None:
        lib.orc_ssm_scan(*args, _p(y), B, T)
    else:
        assert traces.dtype == np.float32 and traces.flags["C_CONTIGUOUS"] and traces.size == 3 * h.size
        lib.orc_ssm_scan_traced(*args, _p(traces), _p(y), B, T)
    return y


def outproj(y, blob_w, blob_s, bias, d_model, d_state, out, act):
    y = np.ascontiguousarray(y, np.float32)
    rows = y.shape[0]
    o = np.zeros((rows, out), dtype=np.float32)
    lib.orc_outproj(_p(y), _p(np.ascontiguousarray(blob_w, np.uint32)), _p(np.ascontiguousarray(blob_s, np.int8)),
                    _p(np.ascontiguousarray(bias, np.float32)), d_model, d_state, out, act, rows, _p(o))
    return o


def critic(x_f16, w1, wl, w2, in_c, units, h, B, T, traces=None):
    """Returns the scores [B*T]; h [B][units][2] is updated in place, and so are
    the traces (trace_w1 [B][in][units][2], trace_lambda [B][units][in][2]) when
    given as a pair of arrays."""
    score = np.zeros(B * T, dtype=np.float32)
    x = np.ascontiguousarray(x_f16, np.float16)
    args = [_p(x.view(np.uint16)), _p(np.ascontiguousarray(w1, np.float32)), _p(np.ascontiguousarray(wl, np.float32)),
            _p(np.ascontiguousarray(w2, np.float32)), in_c, units, _p(h)]
    if traces is None:
        lib.orc_critic(*args, _p(score), B, T)
    else:
        tw, tl = traces
        assert tw.dtype == np.float32 and tw.flags["C_CONTIGUOUS"] and tl.dtype == np.float32 and tl.flags["C_CONTIGUOUS"]
        lib.orc_critic_traced(*args, _p(tw), _p(tl), _p(score), B, T)
    return score


def set_actions(probs):
    probs = np.ascontiguousarray(probs, np.float32)
    rows, count = probs.shape
    out = np.zeros((rows, (count + 63) // 64), dtype=np.uint64)
    lib.orc_set_actions(_p(probs), rows, count, _p(out))
    return out


def screen_frontend(bgra: np.ndarray, train: bool = False, frame_seed: int = 0, brightness: float = 0.0,
                    contrast: float = 1.0) -> np.ndarray:
    """cs.cu:5-45: uint8 BGRA [H, W, 4] -> fp16 planes [4][H][W] (B, G, R, A)."""
    bgra = np.ascontiguousarray(bgra, np.uint8)
    h, w = bgra.shape[:2]
    out = np.zeros(4 * h * w, np.uint16)
    lib.orc_screen_frontend(_p(bgra), h * w, int(bool(train)), frame_seed & 0xFFFFFFFF, float(brightness),
                            float(contrast), _p(out))
    return out.view(np.float16).reshape(4, h, w)


def audio_frontend(pcm: np.ndarray, dim: int = 256, n: int = 1024):
    """ca.cu:106-113 with the row FFT's out-of-range rows reading zeros and the
    column FFT out of place. Returns (planes [2][n][n], out [2][dim][dim]) fp16."""
    pcm = np.ascontiguousarray(pcm, np.int16)
    h = np.zeros(pcm.size, np.uint16)
    lib.orc_audio_pcm_to_half(_p(pcm), pcm.size, _p(h))
    image = np.zeros(2 * n * n, np.uint16)
    lib.orc_resize_half(_p(h), _p(image), n, 1, n, 1)  # src_h: the 1024-sample buffer (ca.cu:107)
    rows = np.zeros(2 * n * n, np.uint16)
    lib.orc_fft_rows(_p(image), n, _p(rows))
    planes = np.zeros(2 * n * n, np.uint16)
    lib.orc_fft_cols(_p(rows), n, _p(planes))
    out = np.zeros(2 * dim * dim, np.uint16)
    lib.orc_resize_half(_p(planes), _p(out), n, n, dim, 2)
    return planes.view(np.float16).reshape(2, n, n), out.view(np.float16).reshape(2, dim, dim)


# ---- compositions ---------------------------------------------------------

class MambaLayerRef:
    """MambaLayer (mamba_layer.h) on the CPU: packed blob, compact state."""

    def __init__(self, d_model, d_state, out, act, blob_master, bias, batch):
        self.d_model, self.d_state, self.out, self.act = d_model, d_state, out, act
        self.w, self.s = pack_f32(blob_master, stochastic=True, add_idx=blob_master.size)
        self.bias = np.ascontiguousarray(bias, np.float32)
        self.h = np.zeros((batch, 2 * d_model, d_state // 32, 2), dtype=np.float32)

    def forward(self, x_w, x_s, B, T):
        y = ssm_scan(x_w, x_s, self.w, self.s, self.d_model, self.d_state, self.out, self.h, B, T)
        return outproj(y, self.w, self.s, self.bias, self.d_model, self.d_state, self.out, self.act)


def conv_block(x_w, x_s, layers, frames, geo, main_mult=1.0, skipped=False):
    """ConvBlock::forward (conv_block.h:74-82). layers: 4 x (words, exps, bias)."""
    cin, mid, cout, stride, d_in, d_out, k = geo
    s1 = stride if d_in != d_out else 1
    a = conv(x_w, x_s, *layers[0], frames, cin, cin, k, s1, d_in, d_out, 0)
    b = conv(*a, *layers[1], frames, cin, mid, 1, 1, d_out, d_out, 1)
    a = conv(*b, *layers[2], frames, mid, cout, 1, 1, d_out, d_out, 0)
    sc = conv(x_w, x_s, *layers[3], frames, cin, cout, s1, s1, d_in, d_out, 0)
    return residual(a[0], a[1], sc[0], sc[1], frames * d_out * d_out, cout, main_mult, skipped)


def pack_conv_layer(master, bias):
    w, s = pack_f32(master, stochastic=True, add_idx=master.size)
    return w, s, np.ascontiguousarray(bias, np.float32)


class CortexRef:
    """The cortex forward composition on the CPU: stem pack -> ConvBlocks ->
    GAP -> requant -> units (MambaLayer + requant + residual) -> actor, and the
    critic on the trunk output (cortex.h:281-303, conv_block.h:74-82,
    mamba_block.h:60-65, critic.h:106-116). Weights are packed once at
    construction, as the reference does at load time."""

    def __init__(self, weights: dict, blocks_geo, d_model: int, d_state: int, actor_out: int, critic_units: int,
                 stem_channels: int = 32):
        self.geo = list(blocks_geo)
        self.d_model, self.d_state, self.actor_out = d_model, d_state, actor_out
        self.critic_units, self.stem_channels = critic_units, stem_channels
        self.blocks = [[pack_conv_layer(m, b) for (m, b) in layers] for layers in weights["blocks"]]
        self.units = [(pack_f32(blob, True, blob.size), np.ascontiguousarray(bias, np.float32))
                      for blob, bias in weights["units"]]
        blob, bias = weights["actor"]
        self.actor = (pack_f32(blob, True, blob.size), np.ascontiguousarray(bias, np.float32))
        self.critic_w = weights["critic"]

    def _layer(self, packed, out, act, B):
        (w, s), bias = packed
        ref = MambaLayerRef.__new__(MambaLayerRef)
        ref.d_model, ref.d_state, ref.out, ref.act = self.d_model, self.d_state, out, act
        ref.w, ref.s, ref.bias = w, s, bias
        ref.h = np.zeros((B, 2 * self.d_model, self.d_state // 32, 2), dtype=np.float32)
        return ref

    def forward(self, planes_f16: np.ndarray, B: int, T: int):
        """Returns (actor [B*T][actor_out], critic [B*T] or None, features (words, exps))."""
        frames = B * T
        xw, xs = stem_pack(planes_f16, self.stem_channels)
        for geo, packed in zip(self.geo, self.blocks):
            xw, xs = conv_block(xw, xs, packed, frames, geo)
        fd = self.geo[-1][5]
        pooled = gap_f32(xw, xs, frames, fd * fd, self.d_model)
        fw, fs = pack_f32(pooled)
        cur = (fw.reshape(frames, -1), fs.reshape(frames, -1))
        feats = cur
        for packed in self.units:
            o = self._layer(packed, self.d_model, 1, B).forward(cur[0], cur[1], B, T)
            qw, qs = pack_f32(o)
            cur = residual(qw, qs, cur[0], cur[1], frames, self.d_model, 1.0, False)
        actor = self._layer(self.actor, self.actor_out, 0, B).forward(cur[0], cur[1], B, T)
        score = None
        if self.critic_units:
            w1, w2, wl = self.critic_w
            pooled_h = gap_f16(cur[0], cur[1], frames, 1, self.d_model)
            h = np.zeros((B, self.critic_units, 2), dtype=np.float32)
            score = critic(pooled_h, w1, wl, w2, self.d_model, self.critic_units, h, B, T)
        return actor, score, feats


def cortex_forward(weights: dict, planes_f16: np.ndarray, B: int, T: int, blocks_geo, d_model: int, d_state: int,
                   actor_out: int, critic_units: int, stem_channels: int = 32):
    """One-shot CortexRef(...).forward(...)."""
    return CortexRef(weights, blocks_geo, d_model, d_state, actor_out, critic_units, stem_channels).forward(
        planes_f16, B, T)


# ---------------------------------------------------------------- training path

def _f32(a):
    return np.ascontiguousarray(a, np.float32)


def sgd_update(data, grad, factor, lr, penalty):
    """updateParamsKernel on a copy of `data` with grad_norm_factor `factor`."""
    d = _f32(data).copy()
    lib.orc_sgd_update(_p(d), _p(_f32(grad)), d.size, float(factor), float(lr), float(penalty))
    return d


def clip_factor(grad, blocks):
    """(clip factor, square sum) over `blocks` 256-thread blocks, added in block order."""
    s = np.zeros(1, np.float32)
    f = lib.orc_clip_factor(_p(_f32(grad)), grad.size, int(blocks), _p(s))
    return float(f), float(s[0])


def conv_backward(x_w, x_s, w_w, w_s, bias, master, dy, in_c, out_c, k, stride, d_in, d_out, act):
    """ConvLayer::backward's gradients on one frame: (gw, gb, grad_in from zeros)."""
    dw = k > 1 and k % 2 == 1
    gw = np.zeros(master.size, np.float32)
    gb = np.zeros(out_c, np.float32)
    gi = np.zeros(d_in * d_in * in_c, np.float32)
    lib.orc_conv_backward(_p(np.ascontiguousarray(x_w, np.uint32)), _p(np.ascontiguousarray(x_s, np.int8)),
                          _p(np.ascontiguousarray(w_w, np.uint32)), _p(np.ascontiguousarray(w_s, np.int8)),
                          _p(_f32(bias)), _p(_f32(master)), _p(_f32(dy)), in_c, out_c, k, stride, d_in, d_out,
                          int(act and not dw), _p(gw), _p(gb), _p(gi))
    return gw, gb, gi


def mamba_backward(x_w, x_s, h, traces, blob, bias, dy, d_model, d_state, out_c, act):
    """MambaLayer::backward's gradients for one sequence after a step: h [E][P][2],
    traces [3][E][P][2] (this sequence). Returns (gw, gb, grad_in)."""
    gw = np.zeros(blob.size, np.float32)
    gb = np.zeros(out_c, np.float32)
    gi = np.zeros(d_model, np.float32)
    t = _f32(traces)
    lib.orc_mamba_backward(_p(np.ascontiguousarray(x_w, np.uint32)), _p(np.ascontiguousarray(x_s, np.int8)),
                           _p(_f32(h)), _p(np.ascontiguousarray(t[0])), _p(np.ascontiguousarray(t[1])),
                           _p(np.ascontiguousarray(t[2])), _p(_f32(blob)), _p(_f32(bias)), _p(_f32(dy)), d_model,
                           d_state, out_c, act, _p(gw), _p(gb), _p(gi))
    return gw, gb, gi


def critic_backward(w2, trace_w1, trace_l, hidden, pred, real, units, in_c):
    """Critic::backward's gradients (gw1, gl, gw2) for one sequence."""
    gw1 = np.zeros(2 * units * in_c, np.float32)
    gl = np.zeros(2 * units * in_c, np.float32)
    gw2 = np.zeros(2 * units, np.float32)
    lib.orc_critic_backward(_p(_f32(w2)), _p(_f32(trace_w1)), _p(_f32(trace_l)), _p(_f32(hidden)), float(pred),
                            float(real), units, in_c, _p(gw1), _p(gl), _p(gw2))
    return gw1, gl, gw2
