"""Generates the golden fixtures in tests/golden/ by running the REFERENCE's own
CUDA kernels (AICortex kernels.h, compiled for sm_100a by oracle/build_ref.sh
into oracle/_ref/libaicref_D<d_model>_N<d_state>.so) on seeded inputs.

Needs a GPU and the oracle/_ref libraries; run it on a B200 box:

    python tests/golden/make_golden.py [out_dir]

Each fixture is an .npz holding the inputs and the reference outputs of one
kernel (or one reference composition), small enough to commit. The reference
kernels are launched with the launch geometry of the reference layer classes
(see oracle/ref_harness.cu) on the legacy default stream.
"""
from __future__ import annotations

import ctypes as C
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
from aicortex_b200 import workloads as W  # noqa: E402

REF_DIR = ROOT / "oracle" / "_ref"
OUT = Path(sys.argv[1]) if len(sys.argv) > 1 else Path(__file__).resolve().parent
DEV = torch.device("cuda")

_libs: dict = {}


def ref(d_model: int = 256, d_state: int = 128) -> C.CDLL:
    key = (d_model, d_state)
    if key not in _libs:
        _libs[key] = C.CDLL(str(REF_DIR / f"libaicref_D{d_model}_N{d_state}.so"))
    return _libs[key]


def dev(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def zeros(n: int, dtype) -> torch.Tensor:
    return torch.zeros(n, dtype=dtype, device=DEV)


def vp(t: torch.Tensor) -> C.c_void_p:
    return C.c_void_p(t.data_ptr())


def host(t: torch.Tensor) -> np.ndarray:
    return t.cpu().numpy()


def run(lib, name, *args):
    fn = getattr(lib, name)
    fn.restype = C.c_int
    st = fn(*args)
    if st != 0:
        raise RuntimeError(f"{name} launch status {st}")
    lib.aicref_sync.restype = C.c_int
    st = lib.aicref_sync()
    if st != 0:
        raise RuntimeError(f"{name} sync status {st}")


def quantize(lib, x: np.ndarray, stochastic: bool, add_idx: int):
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    xi = dev(x)
    w = zeros(x.size // 8, torch.int32)
    s = zeros(x.size // 32, torch.int8)
    run(lib, "aicref_quantize_f32", vp(xi), vp(w), vp(s), C.c_int(x.size), C.c_int(int(stochastic)), C.c_int(add_idx))
    return host(w).view(np.uint32), host(s)


def pack_weights(lib, master: np.ndarray):
    return quantize(lib, master, True, master.size)


def act_f(lib, rng, rows: int, channels: int, scale: float = 1.0):
    x = (rng.standard_normal((rows, channels)) * scale).astype(np.float32)
    w, s = quantize(lib, x, False, 0)
    return w.reshape(rows, channels // 8), s.reshape(rows, channels // 32)


def save(name: str, **arrays):
    OUT.mkdir(parents=True, exist_ok=True)
    np.savez_compressed(OUT / f"{name}.npz", **arrays)
    print("wrote", name)


def f_out(rows, channels):
    return zeros(rows * channels // 8, torch.int32), zeros(rows * channels // 32, torch.int8)


def gen_pack(lib):
    rng = np.random.default_rng(100)
    master = W.conv_weights(rng, 64, 128, 1, False)
    w, s = pack_weights(lib, master)
    acts = (rng.standard_normal(4096) * 3).astype(np.float32)
    acts[:32] = 0.0            # an all-zero group (absmax < eps -> scale 1)
    acts[32:64] *= 1e-4        # a tiny group (clamped dequantisation)
    aw, as_ = quantize(lib, acts, False, 0)
    save("pack", master=master, w=w, s=s, acts=acts, acts_w=aw, acts_s=as_)


def gen_stem(lib):
    rng = np.random.default_rng(101)
    dim, ch = 64, 32
    planes = np.zeros((ch, dim, dim), dtype=np.float16)
    planes[:3] = rng.random((3, dim, dim), dtype=np.float32).astype(np.float16)
    w, s = f_out(dim * dim, ch)
    run(lib, "aicref_stem", vp(dev(planes)), vp(w), vp(s), C.c_int(dim), C.c_int(ch))
    save("stem", planes=planes[:3], channels=np.int32(ch), w=host(w).view(np.uint32), s=host(s))


def gen_conv(lib):
    rng = np.random.default_rng(102)
    cases = [  # (name, in, out, k, stride, din, dout, act)
        ("pw_64_128_silu", 64, 128, 1, 1, 16, 16, 1),
        ("pw_128_64", 128, 64, 1, 1, 16, 16, 0),
        ("pw_64_512_silu", 64, 512, 1, 1, 8, 8, 1),
        ("pw_96_96", 96, 96, 1, 1, 8, 8, 0),
        ("dense_k2_64_128", 64, 128, 2, 2, 16, 8, 0),
        ("dense_k4_32_64", 32, 64, 4, 4, 32, 8, 0),
        ("dense_k2_160_288", 160, 288, 2, 2, 8, 4, 0),
        ("dw_k3_s2_64", 64, 64, 3, 2, 16, 8, 0),
        ("dw_k5_s1_32", 32, 32, 5, 1, 8, 8, 0),
        ("dw_k7_s2_96", 96, 96, 7, 2, 16, 8, 0),
    ]
    for name, cin, cout, k, st, din, dout, act in cases:
        dw = k > 1 and k % 2 == 1
        master = W.conv_weights(rng, cin, cout, k, dw)
        bias = W.bias(rng, cout)
        ww, ws = pack_weights(lib, master)
        xw, xs = act_f(lib, rng, din * din, cin)
        ow, os_ = f_out(dout * dout, cout)
        args = [vp(dev(xw)), vp(dev(xs)), vp(dev(ww)), vp(dev(ws)), vp(dev(bias)), vp(ow), vp(os_)]
        if dw:
            run(lib, "aicref_conv_dw", *args, *map(C.c_int, (cin, k, st, din, dout)))
        elif k == 1:
            run(lib, "aicref_conv_pw", *args, *map(C.c_int, (din * din, cin, cout, act)))
        else:
            run(lib, "aicref_conv_dense", *args, *map(C.c_int, (cin, cout, k, st, din, dout, act)))
        save(f"conv_{name}", master=master, bias=bias, w=ww, s=ws, x_w=xw, x_s=xs,
             geo=np.array([cin, cout, k, st, din, dout, act], np.int32),
             out_w=host(ow).view(np.uint32), out_s=host(os_))


def gen_residual(lib):
    rng = np.random.default_rng(103)
    for name, pos, ch, dim, rf in (("res_160", 64, 160, 8, 0.625), ("res_mamba_256", 1, 256, 1, 1.0)):
        mw, ms = act_f(lib, rng, pos, ch)
        rw, rs = act_f(lib, rng, pos, ch, 0.5)
        ow, os_ = f_out(pos, ch)
        run(lib, "aicref_residual", vp(dev(mw)), vp(dev(ms)), vp(dev(rw)), vp(dev(rs)), vp(ow), vp(os_), C.c_int(ch),
            C.c_int(dim), C.c_float(1.0), C.c_int(0), C.c_float(rf))
        save(name, main_w=mw, main_s=ms, res_w=rw, res_s=rs, channels=np.int32(ch), rf=np.float32(rf),
             out_w=host(ow).view(np.uint32), out_s=host(os_))


def gen_gap(lib):
    rng = np.random.default_rng(104)
    xw, xs = act_f(lib, rng, 64, 256)
    pooled = zeros(256, torch.float32)
    run(lib, "aicref_gap_f32", vp(dev(xw)), vp(dev(xs)), vp(pooled), C.c_int(64), C.c_int(256))
    cw, cs = act_f(lib, rng, 16, 32)
    pooled_h = zeros(32, torch.float16)
    run(lib, "aicref_gap_f16", vp(dev(cw)), vp(dev(cs)), vp(pooled_h), C.c_int(16), C.c_int(32))
    save("gap", x_w=xw, x_s=xs, out=host(pooled), c_w=cw, c_s=cs, c_out=host(pooled_h))


def gen_ssm(d_state: int):
    lib = ref(256, d_state)
    rng = np.random.default_rng(105 + d_state)
    D, T = 256, 8
    E = 2 * D
    blob = W.mamba_blob(rng, D, d_state, D, a_im=None)
    bw, bs = pack_weights(lib, blob)
    bwd, bsd = dev(bw), dev(bs)
    h = zeros(E * d_state * 2, torch.float32)
    tr = [zeros(E * d_state * 2, torch.float32) for _ in range(3)]
    y = zeros(E, torch.float32)
    xw, xs = act_f(lib, rng, T, D)
    ys = []
    for t in range(T):
        run(lib, "aicref_ssm_step", vp(dev(xw[t])), vp(dev(xs[t])), vp(bwd), vp(bsd), vp(h), vp(tr[0]), vp(tr[1]),
            vp(tr[2]), vp(y))
        ys.append(host(y).copy())
    outs = {}
    bias = W.bias(rng, 512)
    yin = (rng.standard_normal(E) * 2).astype(np.float32)
    for out_c, act in ((256, 1), (64, 0), (256, 2)):
        blob_o = W.mamba_blob(rng, D, d_state, out_c, a_im=None)
        ow_, os__ = pack_weights(lib, blob_o)
        o = zeros(out_c, torch.float32)
        run(lib, "aicref_outproj", vp(dev(yin)), vp(dev(ow_)), vp(dev(os__)), vp(dev(bias[:out_c])), vp(o),
            C.c_int(out_c), C.c_int(act))
        outs[f"op{out_c}_{act}_blob"] = blob_o
        outs[f"op{out_c}_{act}_out"] = host(o)
    save(f"ssm_N{d_state}", blob=blob, blob_w=bw, blob_s=bs, x_w=xw, x_s=xs, y=np.stack(ys),
         h=host(h).reshape(E, d_state, 2), yin=yin, bias=bias, **outs)


def gen_mamba_block():
    """MambaBlock::forward (mamba_block.h:58-72, inference) for T steps, d_state 128."""
    lib = ref(256, 128)
    rng = np.random.default_rng(106)
    D, N, T, OUT = 256, 128, 6, 128
    E = 2 * D
    blobs = [W.mamba_blob(rng, D, N, D, a_im=None), W.mamba_blob(rng, D, N, D, a_im=None),
             W.mamba_blob(rng, D, N, OUT, a_im=None)]
    biases = [W.bias(rng, D), W.bias(rng, D), W.bias(rng, OUT)]
    packed = [tuple(dev(a) for a in pack_weights(lib, b)) for b in blobs]
    outs_c = (D, D, OUT)
    acts = (1, 1, 2)
    st = [[zeros(E * N * 2, torch.float32) for _ in range(4)] for _ in range(3)]
    y = zeros(E, torch.float32)
    o = [zeros(c, torch.float32) for c in outs_c]
    aw, as_ = f_out(1, D)
    bw, bs = f_out(1, D)
    xw, xs = act_f(lib, rng, T, D)
    res = []

    def layer(i, inw, ins):
        run(lib, "aicref_ssm_step", vp(inw), vp(ins), vp(packed[i][0]), vp(packed[i][1]), *[vp(t) for t in st[i]], vp(y))
        run(lib, "aicref_outproj", vp(y), vp(packed[i][0]), vp(packed[i][1]), vp(dev(biases[i])), vp(o[i]),
            C.c_int(outs_c[i]), C.c_int(acts[i]))

    for t in range(T):
        xin_w, xin_s = dev(xw[t]), dev(xs[t])
        layer(0, xin_w, xin_s)
        run(lib, "aicref_quantize_f32", vp(o[0]), vp(aw), vp(as_), C.c_int(D), C.c_int(0), C.c_int(0))
        run(lib, "aicref_residual", vp(aw), vp(as_), vp(xin_w), vp(xin_s), vp(bw), vp(bs), C.c_int(D), C.c_int(1),
            C.c_float(1.0), C.c_int(0), C.c_float(1.0))
        layer(1, bw, bs)
        run(lib, "aicref_quantize_f32", vp(o[1]), vp(aw), vp(as_), C.c_int(D), C.c_int(0), C.c_int(0))
        layer(2, aw, as_)
        res.append(host(o[2]).copy())
    save("mamba_block_N128", blob0=blobs[0], blob1=blobs[1], blob2=blobs[2], bias0=biases[0], bias1=biases[1],
         bias2=biases[2], x_w=xw, x_s=xs, out=np.stack(res))


def gen_conv_block(lib):
    """ConvBlock::forward (conv_block.h:74-82, inference) on one frame."""
    rng = np.random.default_rng(107)
    cin, mid, cout, st, din, dout, k = 64, 256, 128, 2, 32, 16, 3
    masters, biases, packed = [], [], []
    geo = [(cin, cin, k, True), (cin, mid, 1, False), (mid, cout, 1, False), (cin, cout, 2, False)]
    for (a, b, kk, dw) in geo:
        m = W.conv_weights(rng, a, b, kk, dw)
        bi = W.bias(rng, b)
        masters.append(m)
        biases.append(bi)
        packed.append(tuple(dev(x) for x in pack_weights(lib, m)) + (dev(bi),))
    xw, xs = act_f(lib, rng, din * din, cin)
    xwd, xsd = dev(xw), dev(xs)
    a_w, a_s = f_out(dout * dout, mid)
    b_w, b_s = f_out(dout * dout, mid)
    o_w, o_s = f_out(dout * dout, cout)
    run(lib, "aicref_conv_dw", vp(xwd), vp(xsd), *map(vp, packed[0]), vp(a_w), vp(a_s), *map(C.c_int, (cin, k, st, din, dout)))
    run(lib, "aicref_conv_pw", vp(a_w), vp(a_s), *map(vp, packed[1]), vp(b_w), vp(b_s), *map(C.c_int, (dout * dout, cin, mid, 1)))
    run(lib, "aicref_conv_pw", vp(b_w), vp(b_s), *map(vp, packed[2]), vp(a_w), vp(a_s), *map(C.c_int, (dout * dout, mid, cout, 0)))
    run(lib, "aicref_conv_dense", vp(xwd), vp(xsd), *map(vp, packed[3]), vp(b_w), vp(b_s), *map(C.c_int, (cin, cout, 2, 2, din, dout, 0)))
    run(lib, "aicref_residual", vp(a_w), vp(a_s), vp(b_w), vp(b_s), vp(o_w), vp(o_s), C.c_int(cout), C.c_int(dout),
        C.c_float(1.0), C.c_int(0), C.c_float(0.75))
    save("conv_block", **{f"m{i}": m for i, m in enumerate(masters)}, **{f"b{i}": b for i, b in enumerate(biases)},
         x_w=xw, x_s=xs, geo=np.array([cin, mid, cout, st, din, dout, k], np.int32), rf=np.float32(0.75),
         out_w=host(o_w).view(np.uint32), out_s=host(o_s))


def gen_critic(lib):
    rng = np.random.default_rng(108)
    cin, units, T = 32, 128, 5
    w1, w2, wl = W.critic_weights(rng, cin, units)
    h = zeros(2 * units, torch.float32)
    tw1 = zeros(cin * units * 2, torch.float32)
    tl = zeros(cin * units * 2, torch.float32)
    score = zeros(1, torch.float32)
    x = (rng.standard_normal((T, cin)) * 0.5).astype(np.float16)
    scores = []
    w1d, w2d, wld = dev(w1), dev(w2), dev(wl)
    for t in range(T):
        run(lib, "aicref_critic", vp(dev(x[t])), vp(w1d), vp(wld), vp(w2d), vp(h), vp(tw1), vp(tl), vp(score),
            C.c_int(units), C.c_int(cin))
        scores.append(float(host(score)[0]))
    save("critic", w1=w1, w2=w2, wl=wl, x=x, score=np.array(scores, np.float32), h=host(h))


def gen_actions(lib):
    rng = np.random.default_rng(109)
    probs = rng.random(98).astype(np.float32)
    probs[:8] = rng.random(8).astype(np.float32) * 0.06
    acts = torch.zeros(2, dtype=torch.int64, device=DEV)
    run(lib, "aicref_set_actions", vp(dev(probs)), vp(acts), C.c_int(98))
    save("actions", probs=probs, words=host(acts).view(np.uint64))


def main():
    lib = ref(256, 128)
    gen_pack(lib)
    gen_stem(lib)
    gen_conv(lib)
    gen_residual(lib)
    gen_gap(lib)
    for n in (32, 128, 512):
        gen_ssm(n)
    gen_mamba_block()
    gen_conv_block(lib)
    gen_critic(lib)
    gen_actions(lib)


if __name__ == "__main__":
    main()
