"""The N > 1 path on CPU: two gloo ranks each run their batch shard (the CPU
oracle stands in for the GPU forward), rank 0 gathers, and the result must be
byte-identical to one process running the whole batch. Also the failure path:
a rank that raises before the barrier makes the other rank's collective fail
within the process-group timeout instead of hanging."""
import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from aicortex_b200.shard import shard_planes, shard_range

B, T, DIM, SEED = 3, 2, 16, 9


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _forward(planes, B_local):
    import oracle as O
    from aicortex_b200 import workloads as W
    wts = W.cortex_weights(4, d_state=32, critic_units=32, dim=DIM, n_units=2)
    ref = O.CortexRef(wts, W.cfg2_blocks(DIM), 256, 32, 64, 32)
    actor, critic, _ = ref.forward(planes, B_local, T)
    return actor, critic


def _worker(rank, world, port, out_dir, fail_rank):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    try:
        if rank == fail_rank:
            raise RuntimeError("injected rank failure")
        start, stop = shard_range(B, world, rank)
        actor, critic = _forward(shard_planes(SEED, start, stop, T, 3, DIM), stop - start)
        gathered = [None] * world
        dist.all_gather_object(gathered, (start, actor, critic))
        if rank == 0:
            gathered.sort(key=lambda g: g[0])
            np.save(os.path.join(out_dir, "actor.npy"), np.concatenate([g[1] for g in gathered]))
            np.save(os.path.join(out_dir, "critic.npy"), np.concatenate([g[2] for g in gathered]))
    except RuntimeError as e:
        with open(os.path.join(out_dir, f"err{rank}.txt"), "w") as f:
            f.write(str(e))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_shard_range_partitions():
    for n, w in [(256, 1), (256, 8), (7, 3), (2, 4)]:
        spans = [shard_range(n, w, r) for r in range(w)]
        assert spans[0][0] == 0 and spans[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def test_two_rank_shards_equal_single_process(tmp_path):
    port = _free_port()
    mp.start_processes(_worker, args=(2, port, str(tmp_path), -1), nprocs=2, join=True, start_method="spawn")
    actor, critic = _forward(shard_planes(SEED, 0, B, T, 3, DIM), B)
    np.testing.assert_array_equal(np.load(tmp_path / "actor.npy"), actor)
    np.testing.assert_array_equal(np.load(tmp_path / "critic.npy"), critic)


def test_failed_rank_surfaces_as_error(tmp_path):
    port = _free_port()
    mp.start_processes(_worker, args=(2, port, str(tmp_path), 1), nprocs=2, join=True, start_method="spawn")
    assert (tmp_path / "err1.txt").read_text() == "injected rank failure"
    # rank 0 is left alone in the all_gather; gloo ends it with an error at the timeout
    assert (tmp_path / "err0.txt").exists()
