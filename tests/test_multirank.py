"""CPU, 2 gloo ranks: the host side of the multi-GPU design.

Utterances are independent: each rank owns a shard (bench.shard) and needs no
exchange on the data path; the only collective is the max over ranks of the
timings (bench.max_over_ranks). Checked here with the CPU restatement standing
in for the device work:
  * the shards partition the global set and each rank's results equal a
    single-process run over the same utterances;
  * the max-over-ranks reduction;
  * a rank that fails before the collective makes the other rank end with an
    error within the process-group timeout instead of waiting forever.
"""
import datetime as dt
import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _utterance(idx, T=5):
    """Deterministic inputs of global utterance idx (x, stand-ins, params)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import pyoracle as po
    r = np.random.default_rng(1000 + idx)
    ps, si, x = po.random_block_inputs(r, T)
    return ps, si, x


def _worker(rank, world, port, per_rank, out_dir, fail_rank):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import torch
    import torch.distributed as dist
    import bench
    import pyoracle as po
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=dt.timedelta(seconds=20))
    try:
        if rank == fail_rank:
            raise RuntimeError("injected failure on the host before the collective")
        oracle = po.Oracle()
        outs = {}
        for idx in bench.shard(rank, world, per_rank):
            ps, si, x = _utterance(idx)
            xo, _ = oracle.conformer_block(x, ps, si)
            outs[idx] = xo
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **{str(k): v for k, v in outs.items()})
        slowest = bench.max_over_ranks(10.0 * (rank + 1), world)
        with open(os.path.join(out_dir, f"max{rank}.txt"), "w") as f:
            f.write(repr(slowest))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass
    del torch


def _spawn(world, per_rank, tmp_path, fail_rank=-1):
    port = _free_port()
    return mp.start_processes(_worker, args=(world, port, per_rank, str(tmp_path), fail_rank),
                              nprocs=world, join=False, start_method="spawn")


def test_two_ranks_shard_and_reduce(tmp_path, oracle):
    ctx = _spawn(2, 3, tmp_path)
    while not ctx.join(timeout=120):
        pass
    got = {}
    for r in range(2):
        got.update({int(k): v for k, v in np.load(tmp_path / f"rank{r}.npz").items()})
        assert float((tmp_path / f"max{r}.txt").read_text()) == 20.0
    assert sorted(got) == list(range(6))          # the shards partition the set
    for idx, xo in got.items():                   # independent items: same as one process
        ps, si, x = _utterance(idx)
        want, _ = oracle.conformer_block(x, ps, si)
        assert np.array_equal(xo, want)


def test_failed_rank_does_not_hang_the_other(tmp_path):
    ctx = _spawn(2, 1, tmp_path, fail_rank=1)
    with pytest.raises(Exception):
        while not ctx.join(timeout=120):
            pass
    assert not (tmp_path / "max0.txt").exists()   # rank 0 did not complete its collective


def test_shard_ranges():
    sys.path.insert(0, ROOT)
    import bench
    assert list(bench.shard(0, 1, 4)) == [0, 1, 2, 3]
    assert [list(bench.shard(r, 4, 2)) for r in range(4)] == [[0, 1], [2, 3], [4, 5], [6, 7]]
    assert bench.max_over_ranks(3.5, 1) == 3.5
