"""Session sharding over ranks, on CPU (no GPU): the partition `bench.py`
uses for `--gpus N`, the job-wide EOS schedule every rank derives alike, and
a world-size-2 gloo run of the rank plumbing.  The path shards by session:
each rank's sessions are computed from its own shard alone (no data-path
collective), so a rank's frame must equal the single-process frame of the
same sessions; the only collectives are the bench's barrier and the max / sum
of its timing scalars."""
import multiprocessing as mp
import os
import socket
import sys

import numpy as np
import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

import bench  # noqa: E402
from magpie_tts_rt_b200.model import EMBED, SHAPE_BASELINE, make_weights  # noqa: E402
from oracle import lt_oracle  # noqa: E402


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_config4_shards_partition_the_sessions(world):
    cfg = bench.WORKLOADS["config4"]
    seen = np.zeros(cfg["total_streams"], np.int64)
    sizes = set()
    for rank in range(world):
        n, first, total = bench.rank_streams(cfg, world, rank)
        assert total == cfg["total_streams"]
        seen[first:first + n] += 1
        sizes.add(n)
    assert (seen == 1).all() and sizes == {cfg["total_streams"] // world}


def test_config3_is_per_gpu():
    cfg = bench.WORKLOADS["config3"]
    for rank in range(4):
        n, first, total = bench.rank_streams(cfg, 4, rank)
        assert n == 64 and first == 64 * rank and total == 256


def test_eos_schedule_is_job_wide():
    cfg = bench.WORKLOADS["config4"]
    a = bench.eos_schedule(cfg, 1024, cfg["frames"])
    b = bench.eos_schedule(cfg, 1024, cfg["frames"])
    np.testing.assert_array_equal(a, b)  # every rank derives the same schedule
    early = a <= cfg["frames"]
    assert early.sum() == round(cfg["eos_frac"] * 1024)
    assert (a[early] >= cfg["eos_lo"]).all() and (a[early] <= cfg["eos_hi"]).all()
    act, unf, fin, forb = bench.flag_tables(a, 60)
    s = int(np.flatnonzero(early & (a < 60))[0]) if (early & (a < 60)).any() else None
    if s is not None:  # active through its EOS frame, finished exactly there
        assert act[: a[s] + 1, s].all() and not act[a[s] + 1:, s].any()
        assert fin[a[s], s] and not unf[a[s], s]
    assert forb[:2].all() and not forb[2:].any()


def _shard_frame(w, first, n, seed0):
    """The CPU oracle frame of sessions [first, first + n) with per-session
    seeds and hidden states derived from the global session index."""
    hidden = torch.stack([torch.randn(2, EMBED, generator=torch.Generator().manual_seed(seed0 + s))
                          for s in range(first, first + n)]).to(torch.bfloat16)
    seeds = np.arange(first, first + n)
    r = lt_oracle.run_frame(w, hidden, np.ones(n, bool), np.zeros(n, bool), np.zeros(n, bool), seeds,
                            np.zeros(n, np.int64), eos=False)
    return np.asarray(r.tokens), np.asarray(r.counter)


def _worker(rank, world, port, q):
    os.environ.update(WORLD_SIZE=str(world), RANK=str(rank), LOCAL_RANK=str(rank),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.set_num_threads(1)
    try:
        w_, r_, l_ = bench.dist_init()
        assert (w_, r_, l_) == (world, rank, rank)
        cfg = dict(bench.WORKLOADS["config4"], total_streams=4)  # 2 sessions per rank
        n, first, total = bench.rank_streams(cfg, world, rank)
        bench.barrier(world)
        frames_total = bench.sum_over_ranks(float(n), world)
        slowest = bench.max_over_ranks(float(rank + 1), world)
        w = make_weights(SHAPE_BASELINE, seed=5, dtype=torch.bfloat16, profile="parity", with_final=False)
        tokens, counter = _shard_frame(w, first, n, 900)
        q.put((rank, n, first, total, frames_total, slowest, tokens, counter))
        import torch.distributed as dist
        dist.destroy_process_group()
    except Exception as e:  # report, the parent fails the test
        q.put((rank, "error", repr(e)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_compute_their_shards_independently():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        item = q.get(timeout=300)
        assert item[1] != "error", item
        results[item[0]] = item
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # the shards cover the job once; the timing reductions see every rank
    assert sorted((results[r][2], results[r][1]) for r in range(world)) == [(0, 2), (2, 2)]
    for r in range(world):
        assert results[r][4] == 4.0 and results[r][5] == 2.0
    # each rank's frame equals the single-process frame of the same sessions
    w = make_weights(SHAPE_BASELINE, seed=5, dtype=torch.bfloat16, profile="parity", with_final=False)
    tokens, counter = _shard_frame(w, 0, 4, 900)
    for r in range(world):
        first = results[r][2]
        np.testing.assert_array_equal(results[r][6], tokens[first:first + 2])
        np.testing.assert_array_equal(results[r][7], counter[first:first + 2])
