"""Benchmark of the AICortex inference hot path on B200.

Metric: cortex forward steps/sec = environment steps (frames) processed per
second by the full forward: fp16 input planes -> stem pack -> 4 quantized
ConvBlocks -> global average pool -> 4 Mamba units -> actor layer + critic.

Default workload: the batch-sharded sweep, a full cortex forward over a global
batch of 4096 environments x 256 sequential steps (1,048,576 frames of
3x128x128, 16 complex states per channel), split into contiguous batch shards
over N GPUs (strong scaling, no collective on the data path). A step is one
forward over the whole batch from zero recurrent state. `--workload b256_t128`
runs the 256 x 128 full-cortex case per GPU instead (weak scaling).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

One process per GPU (torchrun for N > 1); rank 0 prints one JSON line.
`value` is timed with CUDA events on the compute stream with inputs already
in HBM (103 GB of fp16 planes for the whole sweep, far larger than L2), max
over ranks. `e2e` is the same metric through aic_cortex_forward_host with the
planes in pinned host memory (host<->device copies inside the timed region).
`roofline` describes the launch site that takes the most time, from the
library's per-site CUDA-event timers over the timed region. `parity` compares
the timed forward's outputs for the first 4 environments x 8 steps with the
CPU oracle run on the same planes. `--impl reference` times the CPU
restatement of the reference kernels (oracle/) on the host cores instead.
"""
from __future__ import annotations

import argparse
import importlib.util
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
ARCH = "3x128x128 fp16 frames -> stem -> 4 ConvBlocks (dw3x3/s2, 32-64-128-256-256, mid 2x) -> GAP -> " \
       "4 Mamba units (D=256, E=512, 16 states/channel) -> actor (64) + critic (128 units)"
WORKLOADS = {
    # name: (batch, seq, seed, scaling); strong: batch is global, weak: per GPU
    "b4096_t256": (4096, 256, 4, "strong"),
    "b256_t128": (256, 128, 2, "weak"),
}
PARITY_B, PARITY_T = 4, 8  # oracle sample: first environments x first steps of the timed forward


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=3)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="product", choices=["product", "reference"])
    p.add_argument("--workload", default="b4096_t256", choices=sorted(WORKLOADS))
    p.add_argument("--chunk", type=int, default=8192, help="frames per conv-stack pass")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu", action="store_true")
    p.add_argument("--no-parity", action="store_true")
    return p.parse_args()


def load_workloads():
    """aicortex_b200/workloads.py (numpy only) loaded from its file, so the CPU
    legs never load the product library through the package's __init__."""
    spec = importlib.util.spec_from_file_location("aic_bench_workloads", ROOT / "aicortex_b200" / "workloads.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def shard(args, world: int, rank: int):
    """(global batch, seq, seed, scaling, [start, stop) envs of this rank)."""
    batch, seq, seed, scaling = WORKLOADS[args.workload]
    gb = batch if scaling == "strong" else batch * world
    base, extra = divmod(gb, world)
    start = rank * base + min(rank, extra)
    return gb, seq, seed, scaling, (start, start + base + (1 if rank < extra else 0))


def config(args, world: int) -> dict:
    gb, seq, seed, scaling, _ = shard(args, world, 0)
    planes_gb = gb * seq * 3 * 128 * 128 * 2 / 1e9
    return {"workload": f"full cortex forward, batch {gb} x seq {seq}: {ARCH}", "name": args.workload,
            "global_batch": gb, "batch_per_gpu": gb // world, "seq_len": seq, "frames_per_step": gb * seq,
            "seed": seed, "parallelism": f"batch-shard x{world}, no collectives",
            "l2": f"inputs larger than L2: {planes_gb:.1f} GB fp16 planes in total", "chunk_frames": args.chunk}


def load_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "tflops": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "tflops": 1400.0, "source": "fallback"}


TRAFFIC_FRAMES = 2048  # frames per launch of the committed traffic measurements


def traffic_from_profiles(site: str):
    """(DRAM bytes per launch of `site`, note) from the committed ncu summary, if any."""
    path = ROOT / "profiles" / "traffic_per_launch.txt"
    if not path.exists():
        return None, None
    for line in path.read_text().splitlines():
        parts = line.split()
        if len(parts) >= 2 and parts[0] == site:
            try:
                return float(parts[1]), " ".join(parts[2:]) or None
            except ValueError:
                return None, None
    return None, None


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


# ------------------------------------------------------------------ CPU legs (oracle)

def cpu_forward_timer(oracle, W, wts):
    ref = oracle.CortexRef(wts, W.cfg2_blocks(128), 256, W.D_STATE, 64, 128)
    planes = W.planes_u01(np.random.default_rng(0), PARITY_B * PARITY_T)

    def once() -> float:
        t0 = time.perf_counter()
        ref.forward(planes, PARITY_B, PARITY_T)
        return time.perf_counter() - t0

    return once


def cpu_baseline_measure(oracle, W, wts, warmup: int, calls: int | None, min_seconds: float):
    """Mean seconds per call of the oracle forward on a B=4 x T=8 sample after
    `warmup` untimed calls; `calls` calls, or as many as fill `min_seconds`."""
    once = cpu_forward_timer(oracle, W, wts)
    for _ in range(warmup):
        once()
    times = []
    while (calls is not None and len(times) < calls) or (calls is None and sum(times) < min_seconds):
        times.append(once())
    return float(np.mean(times)), len(times)


def cpu_sample_text(n_calls: int, cores: int, sec: float) -> str:
    return (f"B={PARITY_B} envs x T={PARITY_T} steps of the same architecture and weights per call, mean of "
            f"{n_calls} calls after warm-up ({sec:.2f} s per call), CPU restatement of the reference kernels, "
            f"OpenMP over {cores} threads")


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    # every host core this process may run on (torchrun sets OMP_NUM_THREADS=1
    # for its workers); read by the OpenMP runtime when the oracle loads
    os.environ["OMP_NUM_THREADS"] = str(len(os.sched_getaffinity(0)))
    import oracle
    W = load_workloads()
    wts = W.cortex_weights(shard(args, world, 0)[2])
    sec, n = cpu_baseline_measure(oracle, W, wts, max(0, args.warmup), max(1, args.steps), 0.0)
    value = PARITY_B * PARITY_T / sec
    cores = oracle.num_threads()
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
        "scaling": WORKLOADS[args.workload][3], "vs_baseline": None, "dtype": "s4/f32", "data": "synthetic",
        "config": config(args, world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": cpu_sample_text(n, cores, sec)},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ------------------------------------------------------------------ product arm

def build_cortex(A, W, torch, dev, B, chunk, seed):
    desc = W.cortex_desc(batch_chunk=chunk)
    wts = W.cortex_weights(seed)
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


def make_planes(torch, dev, seed, env0, B, T):
    """fp16 planes U(0,1) [B*T][3][128][128]; environment g has its own generator
    seed, so a shard equals the same rows of a single-GPU run."""
    planes = torch.empty(B * T, 3, 128, 128, dtype=torch.float16, device=dev)
    gen = torch.Generator(device=dev)
    for b in range(B):
        gen.manual_seed(seed * 1_000_003 + env0 + b)
        planes[b * T:(b + 1) * T].uniform_(0.0, 1.0, generator=gen)
    return planes


def parity_block(oracle, W, wts, planes, actor, critic, feats, T, fmt):
    """Oracle forward over the first PARITY_B environments x PARITY_T steps of
    the planes the GPU consumed, against the GPU rows b*T + t of the same
    timed forward (a step depends only on earlier steps of its environment)."""
    import torch
    rows = np.array([b * T + t for b in range(PARITY_B) for t in range(PARITY_T)])
    idx = torch.as_tensor(rows, device=planes.device)
    p = planes.index_select(0, idx).cpu().numpy()
    ref = oracle.CortexRef(wts, W.cfg2_blocks(128), 256, W.D_STATE, 64, 128)
    a_ref, c_ref, (frw, frs) = ref.forward(np.ascontiguousarray(p), PARITY_B, PARITY_T)
    a = actor.index_select(0, idx).cpu().numpy()
    c = critic.index_select(0, idx).cpu().numpy()
    fw = feats[0].index_select(0, idx).cpu().numpy().view(np.uint32)
    fs = feats[1].index_select(0, idx).cpu().numpy()
    a_ref, c_ref = a_ref.reshape(a.shape), c_ref.reshape(c.shape)
    codes_gpu, codes_ref = fmt.codes(fw.reshape(-1)), fmt.codes(np.asarray(frw).reshape(-1))
    exp_gpu, exp_ref = fs.reshape(-1), np.asarray(frs).reshape(-1)
    return {
        "sample": f"first {PARITY_B} environments x {PARITY_T} steps of the timed forward vs the CPU oracle",
        "actor_max_abs_rel": float(np.abs(a - a_ref).max() / max(np.abs(a_ref).max(), 1e-30)),
        "critic_max_abs_rel": float(np.abs(c - c_ref).max() / max(np.abs(c_ref).max(), 1e-30)),
        "tolerance": 1e-3,
        "features_bit_identical": bool(np.array_equal(codes_gpu, codes_ref) and np.array_equal(exp_gpu, exp_ref)),
        "feature_code_flip_rate": float(np.mean(codes_gpu != codes_ref)),
        "feature_exponent_mismatch_rate": float(np.mean(exp_gpu != exp_ref)),
    }


class HostPinned:
    """A page-locked host array: numpy memory registered with the CUDA runtime
    (exact size; torch's pinned allocator rounds sizes up to a power of two,
    which would pin up to twice the input planes)."""

    def __init__(self, torch, shape, dtype):
        self.torch = torch
        self.a = np.empty(shape, dtype=dtype)
        self.ptr = self.a.ctypes.data
        torch.cuda.check_error(torch.cuda.cudart().cudaHostRegister(self.ptr, self.a.nbytes, 0))
        self.t = torch.from_numpy(self.a)

    def release(self):
        if self.a is not None:
            self.torch.cuda.check_error(self.torch.cuda.cudart().cudaHostUnregister(self.ptr))
            self.a = self.t = None


def pinned_budget_ok(nbytes: int, local_world: int) -> bool:
    """Pinned host input buffers stay within 60% of the host's available memory."""
    try:
        for line in Path("/proc/meminfo").read_text().splitlines():
            if line.startswith("MemAvailable:"):
                avail = int(line.split()[1]) * 1024
                return nbytes * local_world <= 0.6 * avail
    except OSError:
        pass
    return True


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    import ctypes as C

    import torch
    import torch.distributed as dist

    import aicortex_b200 as A
    from aicortex_b200 import fmt, workloads as W
    from aicortex_b200._lib import call

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
    dev = torch.device(f"cuda:{local}")
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=900), device_id=dev)

    gb, T, seed, scaling, (e0_env, e1_env) = shard(args, world, rank)
    B = e1_env - e0_env
    frames = B * T
    cx, wts = build_cortex(A, W, torch, dev, B, args.chunk, seed)
    planes = make_planes(torch, dev, seed, e0_env, B, T)
    actor = torch.empty(frames, 64, dtype=torch.float32, device=dev)
    critic = torch.empty(frames, dtype=torch.float32, device=dev)
    feats = A.empty_f(frames, 256, dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        cx.reset()
        return cx.forward(planes, B, T, actor, critic, features=feats)

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
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize(dev)
    clocks.start()
    ev0.record(stream)
    launches = 0
    for _ in range(args.steps):
        launches += step()
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    clock_info = clocks.stop()
    call("aic_cortex_profile_enable", cx.h, 0)
    ms = max_over_ranks(ev0.elapsed_time(ev1)) / args.steps
    value = gb * T / (ms / 1e3)

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
    traffic, traffic_note = traffic_from_profiles(top["site"])
    if traffic is not None:  # measured per 2048-frame launch; a conv site's traffic grows with its frames
        traffic *= args.chunk / TRAFFIC_FRAMES
        traffic_note = f"ncu DRAM read+write of a {TRAFFIC_FRAMES}-frame launch x {args.chunk / TRAFFIC_FRAMES:g} " \
                       f"(read, write, algorithmic bytes at {TRAFFIC_FRAMES} frames: {traffic_note})"
    roofline = {"bound": bound, "achieved": achieved, "peak": peak, "unit": unit, "frac": achieved / peak,
                "traffic": traffic, "traffic_source": traffic_note, "site": top["site"],
                "share_of_step": top["ms"] / (ms * args.steps), "peak_source": peaks["source"],
                "launch_ms": per_launch_s * 1e3,
                "algorithmic_flops_per_launch": top["flops"], "algorithmic_bytes_per_launch": top["bytes"]}

    # ---- parity of the timed forward against the oracle (first environments of rank 0)
    parity = None
    if rank == 0 and not args.no_parity:
        import oracle
        parity = parity_block(oracle, W, wts, planes, actor, critic, feats, T, fmt)

    # ---- e2e through the host-buffer API
    e2e = None
    if not args.no_e2e:
        fits = pinned_budget_ok(planes.numel() * 2, local_world)
        fits = max_over_ranks(0.0 if fits else 1.0) == 0.0
        if not fits:
            e2e = {"value": None, "unit": UNIT, "skipped": "pinned host planes would exceed 60% of host memory"}
        else:
            planes_h = HostPinned(torch, planes.shape, np.float16)
            planes_h.t.copy_(planes)
            actor_h = HostPinned(torch, actor.shape, np.float32)
            critic_h = HostPinned(torch, critic.shape, np.float32)
            wsb = C.c_size_t()
            call("aic_cortex_host_workspace_bytes", cx.h, B, T, C.byref(wsb))
            ws = torch.empty(wsb.value + 256, dtype=torch.uint8, device=dev)
            wsp = ws.data_ptr() + (-ws.data_ptr()) % 256
            sp = C.c_void_p(stream.cuda_stream)

            def host_step():
                cx.reset()
                call("aic_cortex_forward_host", cx.h, C.c_void_p(planes_h.ptr), B, T, C.c_void_p(actor_h.ptr),
                     C.c_void_p(critic_h.ptr), C.c_void_p(wsp), sp)

            host_step()
            torch.cuda.synchronize(dev)
            barrier()
            torch.cuda.synchronize(dev)
            ev0.record(stream)
            for _ in range(args.steps):
                host_step()
            ev1.record(stream)
            torch.cuda.synchronize(dev)
            barrier()
            ms_e2e = max_over_ranks(ev0.elapsed_time(ev1)) / args.steps
            e2e = {"value": gb * T / (ms_e2e / 1e3), "unit": UNIT, "ms_per_step": ms_e2e,
                   "h2d_bytes_per_step": planes.numel() * 2 * world,
                   "d2h_bytes_per_step": (actor.numel() * 4 + critic.numel() * 4) * world}
            # the host path must produce what the device path produced (the last timed step)
            e2e["matches_device_path"] = bool(torch.equal(actor.cpu(), actor_h.t) and torch.equal(critic.cpu(), critic_h.t))
            for buf in (planes_h, actor_h, critic_h):
                buf.release()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        import oracle
        sec, ncalls = cpu_baseline_measure(oracle, W, wts, 1, None, 10.0)
        cpu = {"value": PARITY_B * PARITY_T / sec, "unit": UNIT, "cores": oracle.num_threads(), "kind": "port",
               "sample": cpu_sample_text(ncalls, oracle.num_threads(), sec)}

    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": scaling,
            "vs_baseline": None, "dtype": "s4/f32", "data": "synthetic", "config": config(args, world),
            "roofline": roofline, "parity": parity, "cpu_baseline": cpu, "clocks": clock_info, "e2e": e2e,
            "gpu_launches": launches, "sites": sites,
        }), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
