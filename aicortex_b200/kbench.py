"""Per-kernel micro-benchmark: one layer of the inference path on one GPU.

    python -m aicortex_b200.kbench conv --cin 32 --cout 128 --k 1 --dim 64 --frames 2048 --act
    python -m aicortex_b200.kbench dw --cin 32 --k 3 --stride 2 --dim 128 --frames 2048
    python -m aicortex_b200.kbench layer --d-model 256 --d-state 512 --batch 256 --seq 128
    python -m aicortex_b200.kbench scan --d-model 1024 --d-state 512 --batch 32 --seq 8192
    python -m aicortex_b200.kbench outproj --d-model 1024 --d-state 512 --batch 32 --seq 8192 [--mode exact]
    python -m aicortex_b200.kbench sweep [--mode fast]

`sweep` runs the packed-operand GEMM sweep M in {4096, 65536, 1048576} x
K in {256, 1024} x N in {512, 2048, 4096} as pointwise convs (M pixel rows
= frames x 64 x 64, K input channels, N output channels, the fused RMSNorm,
bias and requant epilogue), one JSON line per case.

Times `--iters` launches with CUDA events after `--warmup` launches and prints
one JSON line with the mean time per launch and the algorithmic throughput
(the same work counts as the library's per-site tracer). Used for ncu
captures of a single kernel on a small case.
"""
from __future__ import annotations

import argparse
import json

import numpy as np
import torch

from . import layers as L
from . import workloads as W


def _time(fn, iters: int, warmup: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / max(iters, 1)


def _f_bytes(n: float) -> float:
    return n * (0.5 + 1.0 / 32.0)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("kind", choices=["conv", "dw", "layer", "scan", "outproj", "sweep"])
    ap.add_argument("--cin", type=int, default=32)
    ap.add_argument("--cout", type=int, default=128)
    ap.add_argument("--k", type=int, default=1)
    ap.add_argument("--stride", type=int, default=1)
    ap.add_argument("--dim", type=int, default=64, help="input H = W")
    ap.add_argument("--frames", type=int, default=2048)
    ap.add_argument("--act", action="store_true")
    ap.add_argument("--exact", action="store_true", help="reference-order CUDA-core kernel")
    ap.add_argument("--mode", choices=["ordered", "fast", "simt", "tensor", "exact"], default=None,
                    help="conv mode (ordered, fast, simt) or Mamba out-projection mode (tensor, exact)")
    ap.add_argument("--d-model", type=int, default=256)
    ap.add_argument("--d-state", type=int, default=512)
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--seq", type=int, default=128)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args(argv)
    dev = torch.device("cuda")
    rng = np.random.default_rng(0)

    def t(x):
        return torch.from_numpy(np.ascontiguousarray(x)).to(dev)

    def conv_case(kind, cin, cout, k, stride, dim, frames, act):
        depthwise = kind == "dw"
        cout = cin if depthwise else cout
        stride = stride if depthwise else k
        dout = (dim - 1) // stride + 1 if depthwise else dim // k
        layer = L.ConvLayer(cin, cout, k, stride, dim, dout, disable_activation=not act)
        layer.load_weights(t(W.conv_weights(rng, cin, cout, k, depthwise)), t(W.bias(rng, cout)))
        x = torch.randn(frames * dim * dim * cin, device=dev)
        xw, xs = L.pack_f32(x)
        del x
        ow, os_ = L.empty_f(frames * dout * dout, cout, dev)
        layer.set_mode({"ordered": 0, "fast": 1, "simt": 2}[a.mode or "ordered"])
        fwd = layer.forward_exact if a.exact else layer.forward
        ms = _time(lambda: fwd(xw, xs, ow, os_, frames), a.iters, a.warmup)
        rows = frames * dout * dout
        flops = 2.0 * rows * cout * k * k * cin if not depthwise else 2.0 * rows * cout * k * k
        nbytes = _f_bytes(frames * dim * dim * cin) + _f_bytes(rows * cout) + _f_bytes(layer.weight_elems)
        return ms, flops, nbytes

    if a.kind == "sweep":
        for m in (4096, 65536, 1048576):
            for kk in (256, 1024):
                for n in (512, 2048, 4096):
                    ms, flops, nbytes = conv_case("conv", kk, n, 1, 1, 64, m // 4096, False)
                    print(json.dumps({"kind": "sweep", "M": m, "K": kk, "N": n, "mode": a.mode or "ordered",
                                      "ms_per_launch": ms, "tflops": flops / ms / 1e9, "gbs": nbytes / ms / 1e6}),
                          flush=True)
                    torch.cuda.empty_cache()
        return
    if a.kind in ("conv", "dw"):
        ms, flops, nbytes = conv_case(a.kind, a.cin, a.cout, a.k, a.stride, a.dim, a.frames, a.act)
    else:
        E = 2 * a.d_model
        layer = L.MambaLayer(a.d_model, a.d_state, a.d_model, 1)
        layer.set_mode(1 if a.mode == "exact" else 0)
        blob = W.mamba_blob(rng, a.d_model, a.d_state, a.d_model)
        layer.load_weights(t(blob), t(W.bias(rng, a.d_model)))
        layer.bind_state(a.batch)
        rows = a.batch * a.seq
        xw, xs = L.pack_f32(torch.randn(rows * a.d_model, device=dev))
        out = torch.empty(rows, a.d_model, dtype=torch.float32, device=dev)
        P = a.d_state // 32
        scan_flops = rows * E * (31.0 * P + 15.0)
        gemm_flops = 2.0 * rows * E * a.d_model
        if a.kind == "layer":
            ms = _time(lambda: layer.forward(xw, xs, out, a.batch, a.seq), a.iters, a.warmup)
            flops = scan_flops + gemm_flops
            nbytes = _f_bytes(rows * a.d_model) + 8.0 * rows * E + 4.0 * rows * a.d_model
        else:
            y = torch.empty(rows * E, dtype=torch.float32, device=dev)
            split = a.mode != "exact"
            layer.scan(xw, xs, y, a.batch, a.seq, split=split)
            if a.kind == "scan":
                ms = _time(lambda: layer.scan(xw, xs, y, a.batch, a.seq, split=split), a.iters, a.warmup)
                flops = scan_flops
                nbytes = _f_bytes(rows * a.d_model) + 4.0 * rows * E
            else:
                fn = (lambda: layer.outproj(y, out, rows)) if a.mode == "exact" else \
                    (lambda: layer.outproj_split(y, out, rows))
                ms = _time(fn, a.iters, a.warmup)
                flops = gemm_flops
                nbytes = 4.0 * rows * E + (4.0 if a.mode == "exact" else 2.0) * E * a.d_model + 4.0 * rows * a.d_model
    print(json.dumps({"kind": a.kind, "ms_per_launch": ms, "tflops": flops / ms / 1e9, "gbs": nbytes / ms / 1e6,
                      "flops": flops, "bytes": nbytes, "args": vars(a)}))


if __name__ == "__main__":
    main()
