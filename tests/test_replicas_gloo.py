"""Multi-GPU plumbing of bench.py on CPU: world_size-2 gloo ranks.

The decode path does not shard, so N GPUs run N independent replicas; the
only cross-rank steps are the start barrier and the max-over-ranks timing
reduction. Both, the per-rank seed/id partition and the reference arm's
rank>0 early exit, are exercised here with gloo on CPU."""
from __future__ import annotations

import os
import socket
import sys

import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank: int, world: int, port: int, q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "magenta-realtime-mlx-cpp_b200"))
    import bench
    import mrtdf

    r, w, l = bench.dist_env()
    dist = bench.init_dist(w, l, backend="gloo")
    bench.barrier(dist)
    mx = bench.max_over_ranks(dist, 10.0 + rank)
    cfg = mrtdf.preset("hybrid")
    ids = bench._initial_ids(mrtdf.build_encoder_inputs, r)
    # the reference arm prints from rank 0 only and returns 0 elsewhere
    rc = bench.run_reference(type("A", (), {"warmup": 0, "steps": 0})()) if r != 0 else 0
    q.put((r, mx, ids[0, -6:].tolist(), rc))
    dist.destroy_process_group()


def test_two_rank_barrier_and_max():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    out.sort()
    assert [o[1] for o in out] == [11.0, 11.0]  # max over ranks seen by every rank
    assert out[0][2] != out[1][2]  # replicas get different style ids / seeds
    assert out[1][3] == 0  # reference arm: rank 1 exits without work


def test_launch_count_matches_graph_structure():
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "magenta-realtime-mlx-cpp_b200"))
    import bench
    import mrtdf

    cfg = mrtdf.preset("hybrid")
    # encoder: embed + 12 x 7 + final norm + cross-K/V GEMM; PAD embedding;
    # fused phases: 50 x (20 x 3 temporal + 16 x (4 x 2 depth + lm_head + sampler))
    assert bench.st_launch_count(cfg) == (1 + 12 * 7 + 2) + 1 + 50 * (20 * 3 + 16 * 10)
    # per projection (the self-attention inside the q/k/v cluster launch):
    # 50 x (20 x 7 temporal + 16 x (4 x 4 depth + lm_head + sampler))
    assert bench.st_launch_count(cfg, fused=False) == (1 + 12 * 7 + 2) + 1 + 50 * (20 * 7 + 16 * 18)
