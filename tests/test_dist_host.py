"""Host side of the N > 1 bench path on CPU: two gloo ranks launched the way
torchrun launches bench.py (RANK / WORLD_SIZE / MASTER_* in the environment,
127.0.0.1 rendezvous).  Checks the rank plumbing (barrier, max / sum of
per-rank scalars), the weak-scaling aggregate (all ranks' tokens over the
slowest rank's time), the per-rank workloads (own seeded batch per rank) and
that the reference arm does its work on rank 0 only."""

import os
import socket
import sys

import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, q):
    os.environ.update({"RANK": str(rank), "LOCAL_RANK": str(rank), "WORLD_SIZE": str(world),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    sys.path.insert(0, ROOT)
    try:
        import torch
        import bench

        d = bench.Dist("gloo")
        d.init(torch)
        assert d.pg and d.world == world and d.rank == rank
        d.barrier(torch)
        d.cpu_barrier()  # the host-side wait of the sharder leg
        # rank r encodes 1000 (r + 1) tokens per step in 0.5 + r seconds over 3 steps
        rate, max_s, total = bench.whole_job_rate(d, torch, 1000 * (rank + 1), 3, 0.5 + rank)
        spec, seqs = bench.workload(rank)
        lens = [len(s) for s in seqs]
        other = bench.workload(1 - rank)[1]
        # reference arm: ranks other than 0 exit at once without work
        rc_ref = bench.run_reference(None, d) if rank != 0 else None
        d.barrier(torch)
        d.close()
        q.put((rank, rate, max_s, total, len(seqs), min(lens), max(lens),
               any(len(a) != len(b) or (a != b).any() for a, b in zip(seqs, other)), rc_ref))
    except Exception as e:  # report instead of hanging the other rank's test
        q.put((rank, "error", repr(e)))


def test_two_gloo_ranks():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r = q.get(timeout=180)
        res[r[0]] = r
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world):
        assert res[r][1] != "error", res[r]
        _, rate, max_s, total, n, lo, hi, differs, rc_ref = res[r]
        assert max_s == pytest.approx(1.5)         # slowest rank
        assert total == pytest.approx(3000.0)      # 1000 + 2000 tokens per step
        assert rate == pytest.approx(3000.0 * 3 / 1.5)
        assert n == 128 and lo >= 33 and hi <= 2049  # U[32, 2048] + EOS per rank
        assert differs                             # each rank its own seeded batch
    assert res[1][8] == 0
