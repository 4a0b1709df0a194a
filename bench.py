"""Benchmark of the AICortex inference hot path on B200.

Metric: cortex forward steps/sec = environment steps (frames) processed per
second by the full forward: fp16 input planes -> stem pack -> 4 quantized
ConvBlocks -> global average pool -> 4 Mamba units -> actor layer + critic.
Workload: the full-cortex configuration (batch 256 environments x 128
sequential steps, 3x128x128 synthetic frames, 16 complex states per channel)
on every GPU; N GPUs run N independent batch shards (weak scaling, no
collective on the data path). A step is one forward over the whole B x T
batch from zero recurrent state.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

One process per GPU (torchrun for N > 1); rank 0 prints one JSON line.
`value` is timed with CUDA events on the compute stream with inputs already
in HBM (3.2 GB of fp16 planes per GPU, larger than L2), max over ranks. `e2e`
is the same metric through aic_cortex_forward_host with pinned host input and
output buffers (host<->device copies inside the timed region). `roofline`
describes the launch site that takes the most time, from the library's
per-site CUDA-event timers over the timed region. `--impl reference` times the
CPU restatement of the reference kernels (oracle/) on the host cores instead.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "cortex forward steps/sec"
UNIT = "steps/s"
WORKLOAD = "full cortex forward: 3x128x128 fp16 frames -> stem -> 4 ConvBlocks (dw3x3/s2, 32-64-128-256-256, " \
           "mid 2x) -> GAP -> 4 Mamba units (D=256, E=512, 16 states/channel) -> actor (64) + critic (128 units)"
SEED = 2


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="product", choices=["product", "reference"])
    p.add_argument("--batch", type=int, default=256, help="environments per GPU")
    p.add_argument("--seq", type=int, default=128)
    p.add_argument("--chunk", type=int, default=2048, help="frames per conv-stack pass")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu", action="store_true")
    return p.parse_args()


def load_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "tflops": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "tflops": 1400.0, "source": "fallback"}


def traffic_from_profiles(site: str):
    """DRAM bytes per launch of `site` from the committed ncu summary, if any."""
    path = ROOT / "profiles" / "traffic_per_launch.txt"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        parts = line.split()
        if len(parts) >= 2 and parts[0] == site:
            try:
                return float(parts[1])
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clock/throttle sampling during the timed region."""

    FIELDS = ("index,uuid,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str | None):
        self.uuid = uuid
        self.proc = None
        self.tmp = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=self.tmp, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait(timeout=10)
        self.tmp.flush()
        rows = []
        for line in Path(self.tmp.name).read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 10:
                continue
            if self.uuid and self.uuid not in f[1]:
                continue
            rows.append(f)
        os.unlink(self.tmp.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        smax = max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[6 + i].lower().startswith("active")})
        loaded = [v for v in sm if v > 0.5 * smax] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": smax, "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------------ reference arm

def cpu_sample(oracle, wts, B, T):
    """Times the oracle cortex forward on a B x T sample; returns (frames/s, seconds)."""
    from aicortex_b200 import workloads as W
    ref = oracle.CortexRef(wts, W.cfg2_blocks(128), 256, W.D_STATE, 64, 128)
    planes = W.planes_u01(np.random.default_rng(SEED), B * T)
    t0 = time.perf_counter()
    ref.forward(planes, B, T)
    dt = time.perf_counter() - t0
    return B * T / dt, dt


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    # every host core this process may run on (torchrun sets OMP_NUM_THREADS=1
    # for its workers); read by the OpenMP runtime when the oracle loads
    os.environ["OMP_NUM_THREADS"] = str(len(os.sched_getaffinity(0)))
    import oracle
    from aicortex_b200 import workloads as W
    wts = W.cortex_weights(SEED)
    B, T = 4, 8  # bounded sample of the same workload per step
    for _ in range(max(0, args.warmup)):
        cpu_sample(oracle, wts, B, T)
    times = [cpu_sample(oracle, wts, B, T)[1] for _ in range(max(1, args.steps))]
    sec = float(np.mean(times))
    value = B * T / sec
    cores = oracle.num_threads()
    sample = f"B={B} envs x T={T} steps per step of the same cfg3 workload, OpenMP over {cores} threads"
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "s4/f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "global_batch": B, "seq_len": T, "parallelism": "cpu"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


# ------------------------------------------------------------------ product arm

def build_cortex(A, W, torch, dev, B, chunk):
    desc = W.cortex_desc(batch_chunk=chunk)
    wts = W.cortex_weights(SEED)
    cx = A.Cortex(desc, device=dev)

    def t(a):
        return torch.from_numpy(np.ascontiguousarray(a)).to(dev)

    for blk, layers in zip(cx.blocks, wts["blocks"]):
        for lay, (m, b) in zip(blk.layers, layers):
            lay.load_weights(t(m), t(b))
    for u, (m, b) in zip(cx.units, wts["units"]):
        u.load_weights(t(m), t(b))
    cx.actor.load_weights(t(wts["actor"][0]), t(wts["actor"][1]))
    cx.critic.load_weights(*(t(a) for a in wts["critic"]))
    cx.bind_state(B)
    torch.cuda.synchronize(dev)
    return cx, wts


def make_planes(torch, dev, rank, B, T):
    """fp16 planes U(0,1) [B*T][3][128][128]; env g = rank*B + b has its own seed,
    so a shard equals the same rows of a single-GPU run."""
    planes = torch.empty(B * T, 3, 128, 128, dtype=torch.float16, device=dev)
    gen = torch.Generator(device=dev)
    for b in range(B):
        gen.manual_seed(SEED * 1_000_003 + rank * B + b)
        planes[b * T:(b + 1) * T].uniform_(0.0, 1.0, generator=gen)
    return planes


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    import ctypes as C

    import torch
    import torch.distributed as dist

    import aicortex_b200 as A
    from aicortex_b200 import workloads as W
    from aicortex_b200._lib import call

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=dev)

    B, T = args.batch, args.seq
    frames = B * T
    cx, wts = build_cortex(A, W, torch, dev, B, args.chunk)
    planes = make_planes(torch, dev, rank, B, T)
    actor = torch.empty(frames, 64, dtype=torch.float32, device=dev)
    critic = torch.empty(frames, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        cx.reset()
        return cx.forward(planes, B, T, actor, critic)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t_ = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t_, op=dist.ReduceOp.MAX)
        return float(t_.item())

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)

    # ---- timed region: inputs resident in HBM
    props = torch.cuda.get_device_properties(dev)
    uuid = str(getattr(props, "uuid", "")) or None
    clocks = ClockSampler(uuid)
    call("aic_cortex_profile_reset", cx.h)
    call("aic_cortex_profile_enable", cx.h, 1)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize(dev)
    clocks.start()
    e0.record(stream)
    launches = 0
    for _ in range(args.steps):
        launches += step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    clock_info = clocks.stop()
    call("aic_cortex_profile_enable", cx.h, 0)
    ms = max_over_ranks(e0.elapsed_time(e1)) / args.steps
    value = frames * world / (ms / 1e3)

    # per-site timing over the timed region
    n = C.c_int()
    call("aic_cortex_profile_count", cx.h, C.byref(n))
    sites = []
    for i in range(n.value):
        name = C.create_string_buffer(32)
        tms, nl, fl, by = C.c_double(), C.c_int64(), C.c_double(), C.c_double()
        call("aic_cortex_profile_get", cx.h, i, name, C.byref(tms), C.byref(nl), C.byref(fl), C.byref(by))
        sites.append({"site": name.value.decode(), "ms": tms.value, "launches": nl.value, "flops": fl.value,
                      "bytes": by.value})
    sites.sort(key=lambda s: -s["ms"])
    peaks = load_peaks()
    top = sites[0]
    per_launch_s = top["ms"] / 1e3 / max(1, top["launches"])
    intensity = top["flops"] / max(top["bytes"], 1.0)
    ridge = peaks["tflops"] * 1e12 / (peaks["hbm_gbs"] * 1e9)
    if intensity >= ridge:
        achieved, peak, unit, bound = top["flops"] / per_launch_s / 1e12, peaks["tflops"], "TFLOP/s", "tensor"
    else:
        achieved, peak, unit, bound = top["bytes"] / per_launch_s / 1e9, peaks["hbm_gbs"], "GB/s", "hbm"
    roofline = {"bound": bound, "achieved": achieved, "peak": peak, "unit": unit, "frac": achieved / peak,
                "traffic": traffic_from_profiles(top["site"]), "site": top["site"],
                "share_of_step": top["ms"] / (ms * args.steps), "peak_source": peaks["source"],
                "algorithmic_flops_per_launch": top["flops"], "algorithmic_bytes_per_launch": top["bytes"]}

    # ---- e2e through the host-buffer API
    e2e = None
    if not args.no_e2e:
        planes_h = torch.empty(planes.shape, dtype=torch.float16, pin_memory=True)
        planes_h.copy_(planes)
        actor_h = torch.empty(actor.shape, dtype=torch.float32, pin_memory=True)
        critic_h = torch.empty(critic.shape, dtype=torch.float32, pin_memory=True)
        wsb = C.c_size_t()
        call("aic_cortex_host_workspace_bytes", cx.h, B, T, C.byref(wsb))
        ws = torch.empty(wsb.value + 256, dtype=torch.uint8, device=dev)
        wsp = ws.data_ptr() + (-ws.data_ptr()) % 256
        sp = C.c_void_p(stream.cuda_stream)

        def host_step():
            cx.reset()
            call("aic_cortex_forward_host", cx.h, C.c_void_p(planes_h.data_ptr()), B, T, C.c_void_p(actor_h.data_ptr()),
                 C.c_void_p(critic_h.data_ptr()), C.c_void_p(wsp), sp)

        host_step()
        torch.cuda.synchronize(dev)
        barrier()
        torch.cuda.synchronize(dev)
        e0.record(stream)
        for _ in range(args.steps):
            host_step()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        ms_e2e = max_over_ranks(e0.elapsed_time(e1)) / args.steps
        e2e = {"value": frames * world / (ms_e2e / 1e3), "unit": UNIT, "ms_per_step": ms_e2e,
               "h2d_bytes_per_step": planes.numel() * 2, "d2h_bytes_per_step": actor.numel() * 4 + critic.numel() * 4}
        # the host path must produce what the device path produced
        torch.cuda.synchronize(dev)
        step()
        torch.cuda.synchronize(dev)
        da = (actor.cpu() - actor_h).abs()
        dc = (critic.cpu() - critic_h).abs()
        e2e["matches_device_path"] = bool(torch.equal(actor.cpu(), actor_h) and torch.equal(critic.cpu(), critic_h))
        e2e["max_abs_diff"] = [float(da.max()), float(dc.max())]
        e2e["rows_differing"] = int((da.amax(dim=1) > 0).sum())

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        import oracle
        Bs, Ts = 4, 8
        v, sec = cpu_sample(oracle, wts, Bs, Ts)
        cpu = {"value": v, "unit": UNIT, "cores": oracle.num_threads(), "kind": "port",
               "sample": f"B={Bs} x T={Ts} frames of the same workload ({sec:.1f} s), CPU restatement, "
                         f"OpenMP over {oracle.num_threads()} threads"}

    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "s4/f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "global_batch": B * world, "batch_per_gpu": B, "seq_len": T,
                       "frames_per_step": frames * world, "parallelism": f"batch-shard x{world}, no collectives",
                       "l2": "inputs larger than L2: 3.2 GB fp16 planes per GPU", "chunk_frames": args.chunk},
            "roofline": roofline, "cpu_baseline": cpu, "clocks": clock_info, "e2e": e2e,
            "gpu_launches": launches, "sites": sites[:12],
        }), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
