"""The multi-GPU host logic of bench.py on CPU: two gloo ranks shard the sessions by index and take
the slowest rank's time. Sessions never interact, so the only cross-rank step is that one scalar
reduction; this checks that the ranks' session ranges and prompts tile the global workload
exactly, that the Philox prompt rows are the global session ids whatever the world size, and
that every rank ends up with the maximum time."""
import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, sessions, out_dir):
    import datetime

    import torch
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    first, end = bench.session_range(rank, sessions)
    prompts = bench.prompts_for(rank, sessions)
    ms = bench.max_over_ranks(10.0 + 5.0 * rank, dist, torch.device("cpu"))
    ranges = [None] * world
    dist.all_gather_object(ranges, (first, end))
    # the strong-scaling workloads (config 3 sample, config 4 score): 50 sessions split over the ranks
    sf, se = bench.strong_range(rank, world, 50)
    sp, sl, slim, _ = bench.sample_inputs(sf, se, 50)
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), prompts=prompts, ms=ms, ranges=np.array(ranges),
             sp=sp, sl=sl, slim=slim, srange=np.array([sf, se]))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_two_gloo_ranks_shard_sessions_and_take_the_max_time(tmp_path):
    import torch.multiprocessing as mp
    sys.path.insert(0, ROOT)
    import bench
    from mignon_ai_b200 import synth
    world, sessions = 2, 24
    mp.start_processes(_rank_main, args=(world, _free_port(), sessions, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    res = [np.load(tmp_path / f"rank{r}.npz") for r in range(world)]
    for r in res:
        assert float(r["ms"]) == 15.0  # the slower rank's time, on every rank
        assert [tuple(x) for x in r["ranges"]] == [(0, 24), (24, 48)]
    whole = synth.prompts_uniform_fast(world * sessions, bench.PROMPT, synth.CONFIGS[bench.CONFIG].vocab,
                                       bench.PROMPT_SEED)
    assert np.array_equal(np.concatenate([r["prompts"] for r in res]), whole)
    # a one-rank run of the same global sessions sees the same prompt rows
    assert np.array_equal(bench.prompts_for(0, world * sessions), whole)
    # strong scaling: the ranks' shards tile the one-rank workload exactly
    assert [tuple(r["srange"]) for r in res] == [(0, 25), (25, 50)]
    p1, l1, lim1, _ = bench.sample_inputs(0, 50, 50)
    assert np.array_equal(np.concatenate([r["sp"] for r in res]), p1)
    assert np.array_equal(np.concatenate([r["sl"] for r in res]), l1)
    assert np.array_equal(np.concatenate([r["slim"] for r in res]), lim1)
    assert np.all(lim1 == 128 - l1) and l1.min() >= 16 and l1.max() <= 64
