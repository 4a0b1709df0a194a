"""Times the REFERENCE's own CUDA kernels on this GPU, for comparison with the
product's kernels on the full-cortex workload.

Measurement infrastructure, not a test: it needs a GPU and the oracle/_ref
libraries that oracle/build_ref.sh compiles from the reference's kernels.h for
sm_100a (the reference build flags: -O3 --use_fast_math). Every kernel is
launched through oracle/ref_harness.cu with the launch geometry of the
reference layer classes, one frame (or one time step of one environment) per
launch, which is how the reference's single-environment forward runs
(cortex.h:294-372). Per kernel: 20 untimed launches, then CUDA events around
`--launches` back-to-back launches on the legacy default stream (the stream
the harness launches on); the result is the mean time per launch.

Architecture: the full-cortex workload (3x128x128 fp16 frame -> stem 32 ch ->
4 ConvBlocks dw3x3/s2 32-64-128-256-256, mid 2x -> GAP -> 4 Mamba units
D=256 with reference d_state 512 -> actor 64 -> critic 128 units). Weights are
seeded random masters packed by the reference's own quantizeKernel.

    python tests/reference_kernel_times.py [--launches 200] [--out FILE]

prints one JSON object per kernel site and a total per frame.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[1]
REF_LIB = ROOT / "oracle" / "_ref" / "libaicref_D256_N512.so"
DEV = torch.device("cuda")
DIM, STEM_C, D_MODEL, D_STATE, ACTOR, CRITIC = 128, 32, 256, 512, 64, 128
BLOCKS = [(32, 128, 64), (64, 256, 128), (128, 512, 256), (256, 512, 256)]  # (in, mid, out), stride 2


class Bufs:
    def __init__(self, rng):
        self.rng = rng
        self.keep = []

    def t(self, n, dtype=torch.float32, zero=False):
        x = torch.zeros(n, dtype=dtype, device=DEV) if zero else torch.empty(n, dtype=dtype, device=DEV)
        self.keep.append(x)
        return x

    def p(self, x):
        return C.c_void_p(x.data_ptr())

    def randn(self, n, scale=1.0):
        x = torch.from_numpy((self.rng.standard_normal(n) * scale).astype(np.float32)).to(DEV)
        self.keep.append(x)
        return x


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--launches", type=int, default=200)
    ap.add_argument("--out", default=None)
    args = ap.parse_args()
    lib = C.CDLL(str(REF_LIB))
    assert lib.aicref_d_model() == D_MODEL and lib.aicref_d_state() == D_STATE
    lib.aicref_residual.argtypes = [C.c_void_p] * 6 + [C.c_int, C.c_int, C.c_float, C.c_int, C.c_float]
    rng = np.random.default_rng(11)
    b = Bufs(rng)

    def pack(x, stochastic):
        n = x.numel()
        w, s = b.t(n // 8, torch.int32), b.t(n // 32, torch.int8)
        assert lib.aicref_quantize_f32(b.p(x), b.p(w), b.p(s), n, int(stochastic), n if stochastic else 0) == 0
        return w, s

    def weights(n, scale=0.01):
        return pack(b.randn(n, scale), True)

    def act(n):
        return pack(b.randn(n), False)

    rows = []

    def timed(site, fn, per_frame=1):
        for _ in range(20):
            assert fn() == 0, site
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.launches):
            fn()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / args.launches
        rows.append({"site": site, "us_per_launch": us, "launches_per_frame": per_frame, "us_per_frame": us * per_frame})
        print(json.dumps(rows[-1]), flush=True)

    # stem: one fp16 NCHW frame, 3 planes padded to 32 channels by the caller's zero planes (cortex.h:294-295)
    planes = b.t(STEM_C * DIM * DIM, torch.float16, zero=True)
    planes[: 3 * DIM * DIM] = torch.rand(3 * DIM * DIM, device=DEV).half()
    sw, ss = b.t(DIM * DIM * STEM_C // 8, torch.int32), b.t(DIM * DIM, torch.int8)
    timed("stem", lambda: lib.aicref_stem(b.p(planes), b.p(sw), b.p(ss), DIM, STEM_C))

    d = DIM
    for i, (cin, mid, cout) in enumerate(BLOCKS):
        do = d // 2
        x, xs = act(d * d * cin)
        dw_w, dw_s = weights(9 * cin)
        dw_b = b.randn(cin, 0.1)
        y1, y1s = b.t(do * do * cin // 8, torch.int32), b.t(do * do * cin // 32, torch.int8)
        timed(f"b{i}.dw", lambda: lib.aicref_conv_dw(b.p(x), b.p(xs), b.p(dw_w), b.p(dw_s), b.p(dw_b), b.p(y1),
                                                      b.p(y1s), cin, 3, 2, d, do))
        p1w, p1s = weights(mid * cin)
        p1b = b.randn(mid, 0.1)
        y2, y2s = b.t(do * do * mid // 8, torch.int32), b.t(do * do * mid // 32, torch.int8)
        timed(f"b{i}.pw1", lambda: lib.aicref_conv_pw(b.p(y1), b.p(y1s), b.p(p1w), b.p(p1s), b.p(p1b), b.p(y2),
                                                       b.p(y2s), do * do, cin, mid, 1))
        p2w, p2s = weights(cout * mid)
        p2b = b.randn(cout, 0.1)
        y3, y3s = b.t(do * do * cout // 8, torch.int32), b.t(do * do * cout // 32, torch.int8)
        timed(f"b{i}.pw2", lambda: lib.aicref_conv_pw(b.p(y2), b.p(y2s), b.p(p2w), b.p(p2s), b.p(p2b), b.p(y3),
                                                       b.p(y3s), do * do, mid, cout, 0))
        scw, scs = weights(cout * 4 * cin)
        scb = b.randn(cout, 0.1)
        y4, y4s = b.t(do * do * cout // 8, torch.int32), b.t(do * do * cout // 32, torch.int8)
        timed(f"b{i}.sc", lambda: lib.aicref_conv_dense(b.p(x), b.p(xs), b.p(scw), b.p(scs), b.p(scb), b.p(y4),
                                                         b.p(y4s), cin, cout, 2, 2, d, do, 0))
        o, os_ = b.t(do * do * cout // 8, torch.int32), b.t(do * do * cout // 32, torch.int8)
        timed(f"b{i}.res", lambda: lib.aicref_residual(b.p(y3), b.p(y3s), b.p(y4), b.p(y4s), b.p(o), b.p(os_), cout,
                                                        do, 1.0, 0, 1.0))
        d = do

    fx, fxs = act(d * d * D_MODEL)
    pooled = b.t(D_MODEL, zero=True)
    timed("gap", lambda: lib.aicref_gap_f32(b.p(fx), b.p(fxs), b.p(pooled), d * d, D_MODEL))

    E = 2 * D_MODEL
    blob_n = E * (34 + 4 * D_STATE)

    def mamba(site, out_c, act_kind):
        u, us = act(D_MODEL)
        mw, ms = weights(blob_n + E * out_c)
        mb = b.randn(out_c, 0.1)
        h = b.t(E * D_STATE * 2, zero=True)
        tra, trb, trd = (b.t(E * D_STATE * 2, zero=True) for _ in range(3))
        y = b.t(E, zero=True)
        out = b.t(out_c)
        timed(f"{site}.scan", lambda: lib.aicref_ssm_step(b.p(u), b.p(us), b.p(mw), b.p(ms), b.p(h), b.p(tra),
                                                           b.p(trb), b.p(trd), b.p(y)))
        # the kernel finds W_out inside the whole packed blob (kernels.h:1191-1192, mamba_layer.h:142-145)
        timed(f"{site}.outproj", lambda: lib.aicref_outproj(b.p(y), b.p(mw), b.p(ms), b.p(mb), b.p(out), out_c, act_kind))
        if site.startswith("u"):
            rq, rqs = b.t(D_MODEL // 8, torch.int32), b.t(D_MODEL // 32, torch.int8)
            timed(f"{site}.requant", lambda: lib.aicref_quantize_f32(b.p(out), b.p(rq), b.p(rqs), D_MODEL, 0, 0))
            ro, ros = b.t(D_MODEL // 8, torch.int32), b.t(D_MODEL // 32, torch.int8)
            timed(f"{site}.res", lambda: lib.aicref_residual(b.p(rq), b.p(rqs), b.p(u), b.p(us), b.p(ro), b.p(ros),
                                                               D_MODEL, 1, 1.0, 0, 1.0))

    for i in range(4):
        mamba(f"u{i}", D_MODEL, 0)
    mamba("actor", ACTOR, 0)

    pooled16 = torch.randn(D_MODEL, device=DEV).half()
    b.keep.append(pooled16)
    w1, wl = b.randn(D_MODEL * CRITIC * 2, 0.05), b.randn(CRITIC * D_MODEL * 2, 0.05)
    w2 = b.randn(CRITIC * 2, 0.05)
    hc = b.t(CRITIC * 2, zero=True)
    tw1, tl = b.t(D_MODEL * CRITIC * 2, zero=True), b.t(CRITIC * D_MODEL * 2, zero=True)
    score = b.t(1, zero=True)
    timed("critic", lambda: lib.aicref_critic(b.p(pooled16), b.p(w1), b.p(wl), b.p(w2), b.p(hc), b.p(tw1), b.p(tl),
                                               b.p(score), CRITIC, D_MODEL))
    total = sum(r["us_per_frame"] for r in rows)
    summary = {"total_us_per_frame": total, "frames_per_s": 1e6 / total, "launches": args.launches,
               "device": torch.cuda.get_device_name(0), "kernels_per_frame": len(rows)}
    print(json.dumps(summary), flush=True)
    if args.out:
        Path(args.out).write_text("\n".join(json.dumps(r) for r in rows + [summary]) + "\n")
    return 0


if __name__ == "__main__":
    sys.exit(main())
