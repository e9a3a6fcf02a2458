"""The multi-rank host logic of bench.py on two CPU ranks (gloo).

On a GPU node `bench.py --gpus N` runs one replica per GPU under torchrun: the
recordings do not shard, so the only cross-rank steps are the barriers around
the timed region and the max over ranks of the measured times.  These tests
run that plumbing with the gloo backend (MTB_DIST_BACKEND=gloo) in two spawned
processes that rendezvous on 127.0.0.1: the max over ranks, the whole-job
throughput, and the reference arm running on rank 0 only.
"""
import contextlib
import io
import multiprocessing as mp
import os
import socket
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, mode: str, q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port), MTB_DIST_BACKEND="gloo")
    sys.path.insert(0, ROOT)
    try:
        import bench
        if mode == "reduce":
            r, local, w, dist, torch = bench.dist_setup()
            worst = bench.max_over_ranks(1.5 + r, dist, torch, local)
            rate = bench.job_throughput(w, 400.0, worst)
            dist.barrier()
            dist.destroy_process_group()
            q.put((r, w, worst, rate, ""))
        elif mode == "partition":  # configs[4]: each rank's round-robin share of the 64 recordings
            r, local, w, dist, torch = bench.dist_setup()
            sys.path.insert(0, os.path.join(ROOT, "moss-transcribe.cpp_b200"))
            from mtb import recordings
            mine = recordings.partition(bench.MS_RECORDINGS, w, r)
            shares = [None] * w
            dist.all_gather_object(shares, mine)
            t_rank = 1.0 + r  # a rank's own seconds; the job's time is the slowest rank's
            worst = bench.max_over_ranks(t_rank, dist, torch, local)
            tokens = bench.MS_NEW * len(mine)
            total = bench.sum_over_ranks(float(tokens), dist, torch, local)
            dist.barrier()
            dist.destroy_process_group()
            q.put((r, w, worst, total, repr(shares)))
        else:  # the reference arm: rank 0 would time the CPU path, the others leave at once
            out = io.StringIO()
            if rank == 0:
                r, local, w, dist, torch = bench.dist_setup()
            else:
                with contextlib.redirect_stdout(out):
                    bench.main(["--impl", "reference"])
                import torch.distributed as dist
                w = dist.get_world_size()
            dist.destroy_process_group()
            q.put((rank, w, None, None, out.getvalue()))
    except Exception as e:  # reported to the test, which fails on it
        q.put((rank, -1, None, None, repr(e)))


def _run(mode: str, world: int = 2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        results = [q.get(timeout=180) for _ in range(world)]
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return sorted(results)


def test_max_over_ranks_and_job_throughput_on_two_gloo_ranks():
    res = _run("reduce")
    assert [r[0] for r in res] == [0, 1]
    for rank, world, worst, rate, err in res:
        assert err == "" and world == 2
        assert worst == pytest.approx(2.5)                # the slower rank's time
        assert rate == pytest.approx(2 * 400.0 / 2.5)     # both ranks' units over that time


def test_reference_arm_runs_on_rank_zero_only():
    res = _run("reference")
    assert [r[0] for r in res] == [0, 1]
    for rank, world, _, _, out in res:
        assert world == 2, out
    assert res[1][4] == ""  # rank 1 printed nothing and did no work


def test_recordings_partition_over_two_gloo_ranks():
    """configs[4]'s 64 recordings round robin over the ranks: together the
    shares cover every recording once; the job's tokens are summed over the
    ranks and its time is the slowest rank's."""
    import ast
    res = _run("partition")
    assert [r[0] for r in res] == [0, 1]
    for rank, world, worst, total, shares in res:
        assert world == 2 and worst == pytest.approx(2.0)
        parts = ast.literal_eval(shares)
        assert sorted(i for p in parts for i in p) == list(range(64))
        assert parts[rank] == list(range(rank, 64, 2))
        assert total == pytest.approx(64 * 768)
