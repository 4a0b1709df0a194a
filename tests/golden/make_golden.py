"""Generates the golden fixtures in tests/golden/ by running the REFERENCE's own
CUDA kernels (AICortex kernels.h, compiled for sm_100a by oracle/build_ref.sh
into oracle/_ref/libaicref_D<d_model>_N<d_state>.so) on the seeded inputs of
golden_specs.py.

Needs a GPU and the oracle/_ref libraries; run it on a B200 box:

    python tests/golden/make_golden.py [out_dir]

A fixture (.npz) stores the packed activations fed to the reference kernels,
the reference outputs, and sha256 digests of the regenerated fp32 masters and
of the reference-packed weights (masters are regenerated from the specs by the
tests instead of being stored). Reference kernels are launched with the launch
geometry of the reference layer classes (oracle/ref_harness.cu) on the legacy
default stream; every device buffer stays referenced until its kernel ends.
"""
from __future__ import annotations

import ctypes as C
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(HERE))
import golden_specs as S  # noqa: E402

REF_DIR = ROOT / "oracle" / "_ref"
_NAMES = {"ssm", "critic", "train", "backward"}  # fixture groups that can be regenerated alone
_dirs = [a for a in sys.argv[1:] if a not in _NAMES]
OUT = Path(_dirs[0]) if _dirs else HERE
DEV = torch.device("cuda")
_libs: dict = {}


def ref(d_model: int = 256, d_state: int = 128) -> C.CDLL:
    key = (d_model, d_state)
    if key not in _libs:
        _libs[key] = C.CDLL(str(REF_DIR / f"libaicref_D{d_model}_N{d_state}.so"))
    return _libs[key]


class Dev:
    """Holds every device tensor it hands out, so none is freed (and its
    memory reused by the caching allocator) while a kernel may still use it."""

    def __init__(self):
        self.keep = []

    def put(self, a: np.ndarray) -> C.c_void_p:
        return self.put_t(a)[1]

    def put_t(self, a: np.ndarray) -> tuple[torch.Tensor, C.c_void_p]:
        t = torch.from_numpy(np.ascontiguousarray(a)).to(DEV)
        self.keep.append(t)
        return t, C.c_void_p(t.data_ptr())

    def zeros(self, n: int, dtype) -> tuple[torch.Tensor, C.c_void_p]:
        t = torch.zeros(n, dtype=dtype, device=DEV)
        self.keep.append(t)
        return t, C.c_void_p(t.data_ptr())


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


def u32(t: torch.Tensor) -> np.ndarray:
    return t.cpu().numpy().view(np.uint32)


def quantize(lib, x: np.ndarray, stochastic: bool, add_idx: int):
    d = Dev()
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    px = d.put(x)
    w, pw = d.zeros(x.size // 8, torch.int32)
    s, ps = d.zeros(x.size // 32, torch.int8)
    run(lib, "aicref_quantize_f32", px, pw, ps, C.c_int(x.size), C.c_int(int(stochastic)), C.c_int(add_idx))
    return u32(w), s.cpu().numpy()


def pack_weights(lib, master: np.ndarray):
    return quantize(lib, master, True, master.size)


def act_f(lib, x: np.ndarray):
    rows, ch = x.shape
    w, s = quantize(lib, x, False, 0)
    return w.reshape(rows, ch // 8), s.reshape(rows, ch // 32)


def save(name: str, **arrays):
    OUT.mkdir(parents=True, exist_ok=True)
    np.savez_compressed(OUT / f"{name}.npz", **arrays)
    print("wrote", name)


def gen_pack(lib):
    master, acts = S.pack_master()
    w, s = pack_weights(lib, master)
    aw, as_ = quantize(lib, acts, False, 0)
    save("pack", master_sha=S.sha(master), w=w, s=s, acts_sha=S.sha(acts), acts_w=aw, acts_s=as_)


def gen_stem(lib):
    d = Dev()
    planes3 = S.stem_case()
    dim, ch = planes3.shape[1], 32
    planes = np.zeros((ch, dim, dim), dtype=np.float16)
    planes[:3] = planes3
    w, pw = d.zeros(dim * dim * ch // 8, torch.int32)
    s, ps = d.zeros(dim * dim * ch // 32, torch.int8)
    run(lib, "aicref_stem", d.put(planes), pw, ps, C.c_int(dim), C.c_int(ch))
    save("stem", planes_sha=S.sha(planes3), w=u32(w), s=s.cpu().numpy())


def gen_conv(lib):
    for name, (cin, cout, k, st, din, dout, act) in S.CONV_CASES.items():
        d = Dev()
        master, bias, x = S.conv_case(name)
        dw = k > 1 and k % 2 == 1
        ww, ws = pack_weights(lib, master)
        xw, xs = act_f(lib, x)
        ow, pow_ = d.zeros(dout * dout * cout // 8, torch.int32)
        os_, pos = d.zeros(dout * dout * cout // 32, torch.int8)
        args = [d.put(xw), d.put(xs), d.put(ww), d.put(ws), d.put(bias), pow_, pos]
        if dw:
            run(lib, "aicref_conv_dw", *args, *map(C.c_int, (cin, k, st, din, dout)))
        elif k == 1:
            run(lib, "aicref_conv_pw", *args, *map(C.c_int, (din * din, cin, cout, act)))
        else:
            run(lib, "aicref_conv_dense", *args, *map(C.c_int, (cin, cout, k, st, din, dout, act)))
        save(f"conv_{name}", master_sha=S.sha(master), bias_sha=S.sha(bias), w_sha=S.sha(ww), s_sha=S.sha(ws),
             x_w=xw, x_s=xs, out_w=u32(ow), out_s=os_.cpu().numpy())


def gen_residual(lib):
    for name, (pos, ch, dim, rf) in S.RES_CASES.items():
        d = Dev()
        m, r = S.residual_case(name)
        mw, ms = act_f(lib, m)
        rw, rs = act_f(lib, r)
        ow, pow_ = d.zeros(pos * ch // 8, torch.int32)
        os_, pos_ = d.zeros(pos * ch // 32, torch.int8)
        run(lib, "aicref_residual", d.put(mw), d.put(ms), d.put(rw), d.put(rs), pow_, pos_, C.c_int(ch), C.c_int(dim),
            C.c_float(1.0), C.c_int(0), C.c_float(rf))
        save(name, main_w=mw, main_s=ms, res_w=rw, res_s=rs, out_w=u32(ow), out_s=os_.cpu().numpy())


def gen_gap(lib):
    d = Dev()
    x, c = S.gap_case()
    xw, xs = act_f(lib, x)
    cw, cs = act_f(lib, c)
    pooled, pp = d.zeros(256, torch.float32)
    run(lib, "aicref_gap_f32", d.put(xw), d.put(xs), pp, C.c_int(64), C.c_int(256))
    pooled_h, ph = d.zeros(32, torch.float16)
    run(lib, "aicref_gap_f16", d.put(cw), d.put(cs), ph, C.c_int(16), C.c_int(32))
    save("gap", x_w=xw, x_s=xs, out=pooled.cpu().numpy(), c_w=cw, c_s=cs, c_out=pooled_h.cpu().numpy())


def gen_ssm(d_state: int):
    lib = ref(S.SSM_D, d_state)
    d = Dev()
    blob, x = S.ssm_case(d_state)
    E = 2 * S.SSM_D
    bw, bs = pack_weights(lib, blob)
    pbw, pbs = d.put(bw), d.put(bs)
    h, ph = d.zeros(E * d_state * 2, torch.float32)
    trs_t = [d.zeros(E * d_state * 2, torch.float32) for _ in range(3)]  # trace_A, trace_B, trace_Delta
    trs = [pt for _, pt in trs_t]
    y, py = d.zeros(E, torch.float32)
    xw, xs = act_f(lib, x)
    ys = []
    for t in range(S.SSM_T):
        run(lib, "aicref_ssm_step", d.put(xw[t]), d.put(xs[t]), pbw, pbs, ph, *trs, py)
        ys.append(y.cpu().numpy().copy())
    lane = np.arange(E) % 32

    def active(buf):  # [E][N] complex -> the P states each channel updates, [E][P][2]
        v = buf.cpu().numpy().reshape(E, d_state, 2)
        return np.stack([v[np.arange(E), lane + 32 * c] for c in range(d_state // 32)], axis=1)

    h_active = active(h)
    tr_active = np.stack([active(tt) for tt, _ in trs_t])
    extra = {}
    for out_c, act in S.OUTPROJ_CASES:
        blob_o, bias_o, yin = S.outproj_case(d_state, out_c, act)
        ow_, os__ = pack_weights(lib, blob_o)
        o, po = d.zeros(out_c, torch.float32)
        run(lib, "aicref_outproj", d.put(yin), d.put(ow_), d.put(os__), d.put(bias_o), po, C.c_int(out_c), C.c_int(act))
        extra[f"op{out_c}_{act}_sha"] = S.sha(blob_o)
        extra[f"op{out_c}_{act}_out"] = o.cpu().numpy()
    save(f"ssm_N{d_state}", blob_sha=S.sha(blob), w_sha=S.sha(bw), s_sha=S.sha(bs), x_w=xw, x_s=xs, y=np.stack(ys),
         h=h_active, traces=tr_active, **extra)


def gen_mamba_block():
    """MambaBlock::forward (mamba_block.h:58-72, inference) for T steps."""
    lib = ref(S.MB_D, S.MB_N)
    d = Dev()
    blobs, biases, x = S.mamba_block_case()
    D, N, E = S.MB_D, S.MB_N, 2 * S.MB_D
    packed = [tuple(d.put(a) for a in pack_weights(lib, b)) for b in blobs]
    pbias = [d.put(b) for b in biases]
    outs_c = (D, D, S.MB_OUT)
    acts = (1, 1, 2)
    st = [[d.zeros(E * N * 2, torch.float32)[1] for _ in range(4)] for _ in range(3)]
    _, py = d.zeros(E, torch.float32)
    o = [d.zeros(c, torch.float32) for c in outs_c]
    _, paw = d.zeros(D // 8, torch.int32)
    _, pas = d.zeros(D // 32, torch.int8)
    _, pbw = d.zeros(D // 8, torch.int32)
    _, pbs = d.zeros(D // 32, torch.int8)
    xw, xs = act_f(lib, x)
    res = []

    def layer(i, inw, ins):
        run(lib, "aicref_ssm_step", inw, ins, packed[i][0], packed[i][1], *st[i], py)
        run(lib, "aicref_outproj", py, packed[i][0], packed[i][1], pbias[i], o[i][1], C.c_int(outs_c[i]),
            C.c_int(acts[i]))

    for t in range(S.MB_T):
        xin_w, xin_s = d.put(xw[t]), d.put(xs[t])
        layer(0, xin_w, xin_s)
        run(lib, "aicref_quantize_f32", o[0][1], paw, pas, C.c_int(D), C.c_int(0), C.c_int(0))
        run(lib, "aicref_residual", paw, pas, xin_w, xin_s, pbw, pbs, C.c_int(D), C.c_int(1), C.c_float(1.0),
            C.c_int(0), C.c_float(1.0))
        layer(1, pbw, pbs)
        run(lib, "aicref_quantize_f32", o[1][1], paw, pas, C.c_int(D), C.c_int(0), C.c_int(0))
        layer(2, paw, pas)
        res.append(o[2][0].cpu().numpy().copy())
    save("mamba_block_N128", blob_sha=np.array([S.sha(b) for b in blobs]), x_w=xw, x_s=xs, out=np.stack(res))


def gen_mamba_block_train():
    """MambaBlock::forward in training mode (mamba_block.h:58-72, on_training =
    true): both requants stochastic with add_seed (quantizeKernel<float,false>,
    :63,69) and the residual scaled by 1/p when the step survives, or the main
    branch dropped when it does not (:65). Same weights and inputs as the
    inference fixture; the skipped steps are MB_TRAIN_SKIPPED."""
    lib = ref(S.MB_D, S.MB_N)
    d = Dev()
    blobs, biases, x = S.mamba_block_case()
    D, N, E = S.MB_D, S.MB_N, 2 * S.MB_D
    packed = [tuple(d.put(a) for a in pack_weights(lib, b)) for b in blobs]
    pbias = [d.put(b) for b in biases]
    outs_c = (D, D, S.MB_OUT)
    acts = (1, 1, 2)
    st = [[d.zeros(E * N * 2, torch.float32)[1] for _ in range(4)] for _ in range(3)]
    _, py = d.zeros(E, torch.float32)
    o = [d.zeros(c, torch.float32) for c in outs_c]
    _, paw = d.zeros(D // 8, torch.int32)
    _, pas = d.zeros(D // 32, torch.int8)
    _, pbw = d.zeros(D // 8, torch.int32)
    _, pbs = d.zeros(D // 32, torch.int8)
    xw, xs = act_f(lib, x)
    res = []
    surv_inv = np.float32(1.0) / np.float32(S.MB_TRAIN_SURV)

    def layer(i, inw, ins):
        run(lib, "aicref_ssm_step", inw, ins, packed[i][0], packed[i][1], *st[i], py)
        run(lib, "aicref_outproj", py, packed[i][0], packed[i][1], pbias[i], o[i][1], C.c_int(outs_c[i]),
            C.c_int(acts[i]))

    seed = C.c_int(S.MB_TRAIN_SEED)
    for t in range(S.MB_T):
        survived = t not in S.MB_TRAIN_SKIPPED
        xin_w, xin_s = d.put(xw[t]), d.put(xs[t])
        layer(0, xin_w, xin_s)
        run(lib, "aicref_quantize_f32", o[0][1], paw, pas, C.c_int(D), C.c_int(1), seed)
        run(lib, "aicref_residual", paw, pas, xin_w, xin_s, pbw, pbs, C.c_int(D), C.c_int(1),
            C.c_float(surv_inv if survived else 1.0), C.c_int(0 if survived else 1), C.c_float(1.0))
        layer(1, pbw, pbs)
        run(lib, "aicref_quantize_f32", o[1][1], paw, pas, C.c_int(D), C.c_int(1), seed)
        layer(2, paw, pas)
        res.append(o[2][0].cpu().numpy().copy())
    save("mamba_block_train_N128", blob_sha=np.array([S.sha(b) for b in blobs]), x_w=xw, x_s=xs,
         out=np.stack(res))


def gen_conv_block_train(lib):
    """ConvBlock::forward in training mode (conv_block.h:74-82, train_mode =
    true): the residual scales the main branch by 1/p when the block survives
    and drops it when it does not (:81). One frame, both cases."""
    d = Dev()
    masters, biases, x = S.conv_block_case()
    cin, mid, cout, st, din, dout, k = S.CB_GEO
    packed = []
    for m, b in zip(masters, biases):
        w, s = pack_weights(lib, m)
        packed.append((d.put(w), d.put(s), d.put(b)))
    xw, xs = act_f(lib, x)
    pxw, pxs = d.put(xw), d.put(xs)
    _, paw = d.zeros(dout * dout * mid // 8, torch.int32)
    _, pas = d.zeros(dout * dout * mid // 32, torch.int8)
    _, pbw = d.zeros(dout * dout * mid // 8, torch.int32)
    _, pbs = d.zeros(dout * dout * mid // 32, torch.int8)
    out = {}
    surv_inv = np.float32(1.0) / np.float32(S.CB_TRAIN_SURV)
    for name, survived in (("survived", True), ("skipped", False)):
        ow, pow_ = d.zeros(dout * dout * cout // 8, torch.int32)
        os_, pos = d.zeros(dout * dout * cout // 32, torch.int8)
        run(lib, "aicref_conv_dw", pxw, pxs, *packed[0], paw, pas, *map(C.c_int, (cin, k, st, din, dout)))
        run(lib, "aicref_conv_pw", paw, pas, *packed[1], pbw, pbs, *map(C.c_int, (dout * dout, cin, mid, 1)))
        run(lib, "aicref_conv_pw", pbw, pbs, *packed[2], paw, pas, *map(C.c_int, (dout * dout, mid, cout, 0)))
        run(lib, "aicref_conv_dense", pxw, pxs, *packed[3], pbw, pbs, *map(C.c_int, (cin, cout, 2, 2, din, dout, 0)))
        run(lib, "aicref_residual", paw, pas, pbw, pbs, pow_, pos, C.c_int(cout), C.c_int(dout),
            C.c_float(surv_inv if survived else 1.0), C.c_int(0 if survived else 1), C.c_float(S.CB_RF))
        out[f"{name}_w"] = u32(ow)
        out[f"{name}_s"] = os_.cpu().numpy()
    save("conv_block_train", master_sha=np.array([S.sha(m) for m in masters]), x_w=xw, x_s=xs, **out)


def _clip(sum_sq: float) -> float:
    """clip_op (conv_layer.h:209-213) in fp32, as the host computes it."""
    norm = np.sqrt(np.float32(sum_sq) + np.float32(1.0 / 8192.0), dtype=np.float32)
    return float(np.float32(1.0) / norm) if norm > np.float32(1.0) else 1.0


def _sum_sq(lib, ptr, n):
    out = C.c_float(0.0)
    run(lib, "aicref_sum_sq", ptr, C.c_int(n), C.byref(out))
    return out.value


def _update(lib, data_ptr, grad_ptr, n, factor, penalty):
    run(lib, "aicref_update_params", data_ptr, grad_ptr, C.c_int(n), C.c_float(factor), C.c_float(S.TRAIN_LR),
        C.c_float(penalty))


def gen_backward_conv(lib):
    """ConvLayer::backward (conv_layer.h:150-219) on one frame per case: the
    reference's gradient kernels, its square-sum reduction, clip and update
    kernels, and the re-quantisation of the masters."""
    out = {}
    for (name, cin, cout, k, st, din, dout, act) in S.CONV_BWD_CASES:
        d = Dev()
        master, bias, x, gout = S.conv_bwd_case(name)
        w, s = pack_weights(lib, master)
        xw, xs = act_f(lib, x)
        (tm, pm), (tb, pb) = d.put_t(master), d.put_t(bias)
        gw, pgw = d.zeros(master.size, torch.float32)
        gb, pgb = d.zeros(cout, torch.float32)
        gi, pgi = d.zeros(din * din * cin, torch.float32)
        pw, ps = d.put(w), d.put(s)
        run(lib, "aicref_conv_bwd", d.put(xw), d.put(xs), pw, ps, pb, pm, d.put(gout), pgi, pgw, pgb,
            *map(C.c_int, (cin, cout, k, st, din, dout, act)))
        sw, sb = _sum_sq(lib, pgw, master.size), _sum_sq(lib, pgb, cout)
        out[f"{name}_gw"], out[f"{name}_gb"], out[f"{name}_gi"] = (gw.cpu().numpy(), gb.cpu().numpy(),
                                                                   gi.cpu().numpy())
        _update(lib, pm, pgw, master.size, _clip(sw), S.TRAIN_PENALTY)
        _update(lib, pb, pgb, cout, _clip(sb), 0.0)
        nw, ns = d.zeros(master.size // 8, torch.int32), d.zeros(master.size // 32, torch.int8)
        run(lib, "aicref_quantize_f32", pm, nw[1], ns[1], C.c_int(master.size), C.c_int(1), C.c_int(master.size))
        out[f"{name}_sums"] = np.array([sw, sb], np.float32)
        out[f"{name}_master"], out[f"{name}_bias"] = tm.cpu().numpy(), tb.cpu().numpy()
        out[f"{name}_w"], out[f"{name}_s"] = u32(nw[0]), ns[0].cpu().numpy()
        out[f"{name}_xw"], out[f"{name}_xs"] = xw, xs
    save("backward_conv", **out)


def gen_backward_mamba():
    """MambaLayer::backward (mamba_layer.h:146-167) after MB_BWD_T training
    forward steps from zero state (traces advancing), per case."""
    lib = ref(S.SSM_D, 128)
    D, N, E = S.SSM_D, 128, 2 * S.SSM_D
    out = {}
    for out_c, act in S.MB_BWD_CASES:
        d = Dev()
        blob, bias, x, gout = S.mamba_bwd_case(out_c, act)
        bw, bs = pack_weights(lib, blob)
        pbw, pbs = d.put(bw), d.put(bs)
        st = [d.zeros(E * N * 2, torch.float32)[1] for _ in range(4)]
        _, py = d.zeros(E, torch.float32)
        xw, xs = act_f(lib, x)
        ins = [(d.put(xw[t]), d.put(xs[t])) for t in range(S.MB_BWD_T)]
        for t in range(S.MB_BWD_T):
            run(lib, "aicref_ssm_step", ins[t][0], ins[t][1], pbw, pbs, *st, py)
        (tm, pm), (tb, pb) = d.put_t(blob), d.put_t(bias)
        _, praw = d.zeros(out_c, torch.float32)
        gw, pgw = d.zeros(blob.size, torch.float32)
        gb, pgb = d.zeros(out_c, torch.float32)
        gi, pgi = d.zeros(D, torch.float32)
        run(lib, "aicref_mamba_bwd", ins[-1][0], ins[-1][1], st[0], st[1], st[2], st[3], pm, pb, d.put(gout), praw, pgw,
            pgb, pgi, C.c_int(out_c), C.c_int(act))
        sw, sb = _sum_sq(lib, pgw, blob.size), _sum_sq(lib, pgb, out_c)
        tag = f"o{out_c}_a{act}"
        out[f"{tag}_gw"], out[f"{tag}_gb"], out[f"{tag}_gi"] = gw.cpu().numpy(), gb.cpu().numpy(), gi.cpu().numpy()
        _update(lib, pm, pgw, blob.size, _clip(sw), S.TRAIN_PENALTY)
        _update(lib, pb, pgb, out_c, _clip(sb), 0.0)
        out[f"{tag}_sums"] = np.array([sw, sb], np.float32)
        out[f"{tag}_master"], out[f"{tag}_bias"] = tm.cpu().numpy(), tb.cpu().numpy()
        out[f"{tag}_xw"], out[f"{tag}_xs"] = xw, xs
    save("backward_mamba_N128", **out)


def gen_backward_critic(lib):
    """Critic::backward (critic.h:117-131) after the critic fixture's steps."""
    d = Dev()
    w1, w2, wl, x = S.critic_case()
    T, cin, units = x.shape[0], 32, 128
    h, ph = d.zeros(2 * units, torch.float32)
    tw, ptw = d.zeros(cin * units * 2, torch.float32)
    tl, ptl = d.zeros(cin * units * 2, torch.float32)
    score, psc = d.zeros(1, torch.float32)
    (t1, pw1), (t2, pw2), (tlw, pwl) = d.put_t(w1), d.put_t(w2), d.put_t(wl)
    for t in range(T):
        run(lib, "aicref_critic", d.put(x[t]), pw1, pwl, pw2, ph, ptw, ptl, psc, C.c_int(units), C.c_int(cin))
    pred = float(score.cpu().numpy()[0])
    g1, pg1 = d.zeros(w1.size, torch.float32)
    gl, pgl = d.zeros(wl.size, torch.float32)
    g2, pg2 = d.zeros(w2.size, torch.float32)
    run(lib, "aicref_critic_bwd", pw2, ptw, ptl, ph, pg1, pgl, pg2, C.c_float(pred), C.c_float(S.CRITIC_BWD_REAL),
        C.c_int(units), C.c_int(cin))
    s1, s2, sl = _sum_sq(lib, pg1, w1.size), _sum_sq(lib, pg2, w2.size), _sum_sq(lib, pgl, wl.size)
    grads = dict(gw1=g1.cpu().numpy(), gw2=g2.cpu().numpy(), gl=gl.cpu().numpy())
    _update(lib, pw1, pg1, w1.size, _clip(s1), S.TRAIN_PENALTY)
    _update(lib, pw2, pg2, w2.size, _clip(s2), S.TRAIN_PENALTY)
    _update(lib, pwl, pgl, wl.size, _clip(sl), S.TRAIN_PENALTY)
    save("backward_critic", pred=np.array([pred], np.float32), sums=np.array([s1, s2, sl], np.float32), **grads,
         w1_after=t1.cpu().numpy(), w2_after=t2.cpu().numpy(), wl_after=tlw.cpu().numpy())


def gen_conv_block(lib):
    """ConvBlock::forward (conv_block.h:74-82, inference) on one frame."""
    d = Dev()
    masters, biases, x = S.conv_block_case()
    cin, mid, cout, st, din, dout, k = S.CB_GEO
    packed = []
    for m, b in zip(masters, biases):
        w, s = pack_weights(lib, m)
        packed.append((d.put(w), d.put(s), d.put(b)))
    xw, xs = act_f(lib, x)
    pxw, pxs = d.put(xw), d.put(xs)
    _, paw = d.zeros(dout * dout * mid // 8, torch.int32)
    _, pas = d.zeros(dout * dout * mid // 32, torch.int8)
    _, pbw = d.zeros(dout * dout * mid // 8, torch.int32)
    _, pbs = d.zeros(dout * dout * mid // 32, torch.int8)
    ow, pow_ = d.zeros(dout * dout * cout // 8, torch.int32)
    os_, pos = d.zeros(dout * dout * cout // 32, torch.int8)
    run(lib, "aicref_conv_dw", pxw, pxs, *packed[0], paw, pas, *map(C.c_int, (cin, k, st, din, dout)))
    run(lib, "aicref_conv_pw", paw, pas, *packed[1], pbw, pbs, *map(C.c_int, (dout * dout, cin, mid, 1)))
    run(lib, "aicref_conv_pw", pbw, pbs, *packed[2], paw, pas, *map(C.c_int, (dout * dout, mid, cout, 0)))
    run(lib, "aicref_conv_dense", pxw, pxs, *packed[3], pbw, pbs, *map(C.c_int, (cin, cout, 2, 2, din, dout, 0)))
    run(lib, "aicref_residual", paw, pas, pbw, pbs, pow_, pos, C.c_int(cout), C.c_int(dout), C.c_float(1.0),
        C.c_int(0), C.c_float(S.CB_RF))
    save("conv_block", master_sha=np.array([S.sha(m) for m in masters]), x_w=xw, x_s=xs, out_w=u32(ow),
         out_s=os_.cpu().numpy())


def gen_critic(lib):
    d = Dev()
    w1, w2, wl, x = S.critic_case()
    T, cin, units = x.shape[0], 32, 128
    h, ph = d.zeros(2 * units, torch.float32)
    tw, ptw = d.zeros(cin * units * 2, torch.float32)
    tl, ptl = d.zeros(cin * units * 2, torch.float32)
    score, psc = d.zeros(1, torch.float32)
    pw1, pw2, pwl = d.put(w1), d.put(w2), d.put(wl)
    scores = []
    for t in range(T):
        run(lib, "aicref_critic", d.put(x[t]), pw1, pwl, pw2, ph, ptw, ptl, psc, C.c_int(units), C.c_int(cin))
        scores.append(float(score.cpu().numpy()[0]))
    save("critic", w_sha=np.array([S.sha(w1), S.sha(w2), S.sha(wl), S.sha(x)]), score=np.array(scores, np.float32),
         h=h.cpu().numpy(), trace_w1=tw.cpu().numpy(), trace_lambda=tl.cpu().numpy())


def gen_actions(lib):
    d = Dev()
    probs = S.actions_case()
    acts, pa = d.zeros(2, torch.int64)
    run(lib, "aicref_set_actions", d.put(probs), pa, C.c_int(98))
    save("actions", probs_sha=S.sha(probs), words=acts.cpu().numpy().view(np.uint64))


def gen_audio(lib):
    """ca.cu:106-113 one hop window at a time: convert, resize 1024 x 1 -> 1024
    x 1024, row FFT over a 2 x 1024 x 1024 input with a zero upper half, column
    FFT into a separate planes buffer, resize both planes to 256 x 256."""
    n, dim = 1024, S.AUDIO_DIM
    pcm = S.audio_case()
    outs, plane_sha = [], []
    for win in pcm:
        d = Dev()
        h, ph = d.zeros(2048, torch.float16)
        run(lib, "aicref_audio_convert", d.put(win), ph)
        image, pimg = d.zeros(2 * n * n, torch.float16)
        run(lib, "aicref_resize", ph, pimg, C.c_int(1024), C.c_int(1), C.c_int(n), C.c_int(1))
        rows, prows = d.zeros(2 * n * n, torch.float16)
        run(lib, "aicref_fft_rows", pimg, prows)
        planes, ppl = d.zeros(2 * n * n, torch.float16)
        run(lib, "aicref_fft_cols", prows, ppl)
        out, pout = d.zeros(2 * dim * dim, torch.float16)
        run(lib, "aicref_resize", ppl, pout, C.c_int(n), C.c_int(n), C.c_int(dim), C.c_int(2))
        outs.append(out.cpu().numpy().reshape(2, dim, dim))
        plane_sha.append(S.sha(planes.cpu().numpy()))
    save("audio", pcm_sha=S.sha(pcm), out=np.stack(outs), planes_sha=np.array(plane_sha))


def gen_screen(lib):
    """cs.cu:116-122 on one frame: inference (conversion only) and training
    (pixel dropout from the frame seed, then the brightness/contrast
    augmentation over all four planes as half2 pairs)."""
    bgra = S.screen_case()
    px = bgra.shape[0] * bgra.shape[1]
    outs = []
    for train in (0, 1):
        d = Dev()
        out, po = d.zeros(4 * px, torch.float16)
        run(lib, "aicref_screen", d.put(bgra), po, C.c_int(px), C.c_uint(S.SCREEN_SEED), C.c_int(train))
        if train:
            run(lib, "aicref_augment", po, C.c_int(2 * px), C.c_float(S.SCREEN_AUG[0]), C.c_float(S.SCREEN_AUG[1]))
        outs.append(out.cpu().numpy().reshape(4, bgra.shape[0], bgra.shape[1]))
    save("screen", bgra_sha=S.sha(bgra), out=np.stack(outs))


def main():
    only = set(sys.argv[1:]) & _NAMES  # e.g. "ssm critic": regenerate those fixtures only
    if only:
        if "ssm" in only:
            for n in (32, 128, 512):
                gen_ssm(n)
        if "critic" in only:
            gen_critic(ref(256, 128))
        if "backward" in only:
            gen_backward_conv(ref(256, 128))
            gen_backward_mamba()
            gen_backward_critic(ref(256, 128))
        if "train" in only:
            gen_mamba_block_train()
            gen_conv_block_train(ref(256, 128))
        return
    lib = ref(256, 128)
    gen_screen(lib)
    gen_audio(lib)
    gen_pack(lib)
    gen_stem(lib)
    gen_conv(lib)
    gen_residual(lib)
    gen_gap(lib)
    for n in (32, 128, 512):
        gen_ssm(n)
    gen_mamba_block()
    gen_conv_block(lib)
    gen_mamba_block_train()
    gen_conv_block_train(lib)
    gen_critic(lib)
    gen_backward_conv(lib)
    gen_backward_mamba()
    gen_backward_critic(lib)
    gen_actions(lib)


if __name__ == "__main__":
    main()
