"""Multi-rank host logic of the batch-sharded replicas, as world_size-2 gloo ranks on the CPU:
slices partition the batch, the max over ranks is taken, and per-rank results of a small plan
(run by the oracle, no GPU) gathered in rank order equal the single-process result."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from simdonnx_b200.replicas import shard_range


def test_shard_ranges_partition():
    for gb in (1, 7, 8, 256, 257):
        for world in (1, 2, 3, 8):
            spans = [shard_range(gb, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == gb
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    import torch.distributed as dist
    from oracle.runner import OracleSession
    from simdonnx_b200 import configs
    from simdonnx_b200.replicas import gather_outputs, max_over_ranks
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        gb = 5
        full = configs.build_c1(batch=gb, hw=16, c=16)
        feeds = {k: f() for k, f in full.feeds.items()}
        b, e = shard_range(gb, world, rank)
        part = configs.build_c1(batch=e - b, hw=16, c=16)
        local = OracleSession(part).run({k: v[b:e] for k, v in feeds.items()})[part.output]
        t = max_over_ranks(1.0 + rank, dist)
        got = gather_outputs(local, dist)
        if rank == 0:
            np.save(os.path.join(out_dir, "gathered.npy"), got)
            np.save(os.path.join(out_dir, "tmax.npy"), np.array([t]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_rank_sharded_run_matches_single_process(tmp_path):
    from oracle.runner import OracleSession
    from simdonnx_b200 import configs
    mp.start_processes(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    full = configs.build_c1(batch=5, hw=16, c=16)
    feeds = {k: f() for k, f in full.feeds.items()}
    want = OracleSession(full).run(feeds)[full.output]
    got = np.load(tmp_path / "gathered.npy")
    assert np.array_equal(got, want)
    assert float(np.load(tmp_path / "tmax.npy")[0]) == 2.0


def _failing_worker(rank, world, port, out_dir):
    """Rank 1's shard fails on the host (an injected allocation fault in the C ABI, no GPU work);
    rank 0's shard runs. Every rank takes the same gather; rank 0 sees the failure and rank 0's own
    result is intact."""
    import torch.distributed as dist
    from datetime import timedelta
    from oracle.runner import OracleSession
    from simdonnx_b200 import _native as N, configs
    from simdonnx_b200.replicas import ShardFailure, run_shards
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    try:
        gb = 4
        full = configs.build_c1(batch=gb, hw=16, c=16)
        feeds = {k: f() for k, f in full.feeds.items()}
        b, e = shard_range(gb, world, rank)

        def local():
            import ctypes
            if rank == 1:
                N.call("sdx_fault_inject", N.FAULT_MALLOC, 1)
                p = ctypes.c_void_p()
                N.call("sdx_host_alloc_pinned", 1 << 20, ctypes.byref(p))  # the shard's staging: fails
            part = configs.build_c1(batch=e - b, hw=16, c=16)
            return OracleSession(part).run({k: v[b:e] for k, v in feeds.items()})[part.output]

        try:
            got = run_shards(local, dist)
            result = ("ok", got)
        except ShardFailure as f:
            result = ("failed", f)
        if rank == 0:
            kind, val = result
            np.save(os.path.join(out_dir, "kind.npy"), np.array([kind == "failed"]))
            if kind == "failed":
                np.save(os.path.join(out_dir, "failed_ranks.npy"), np.array(sorted(val.failed)))
                np.save(os.path.join(out_dir, "rank0.npy"), val.partial[0])
                with open(os.path.join(out_dir, "msg.txt"), "w") as fh:
                    fh.write(str(val))
        else:
            assert result == ("ok", None)
        dist.barrier()
    finally:
        N.call("sdx_fault_inject", 0, 0)
        dist.destroy_process_group()


def test_one_shard_failing_reports_batch_failure(tmp_path):
    """SURVEY's replica failure rule: one shard errors -> the whole batch reports a failure, the other
    shards are unaffected (rank 0's slice equals its single-process result)."""
    from oracle.runner import OracleSession
    from simdonnx_b200 import configs
    mp.start_processes(_failing_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    assert bool(np.load(tmp_path / "kind.npy")[0])
    assert list(np.load(tmp_path / "failed_ranks.npy")) == [1]
    assert "INJECTED" in (tmp_path / "msg.txt").read_text()
    full = configs.build_c1(batch=4, hw=16, c=16)
    feeds = {k: f() for k, f in full.feeds.items()}
    b, e = shard_range(4, 2, 0)
    want = OracleSession(full).run(feeds)[full.output][b:e]
    assert np.array_equal(np.load(tmp_path / "rank0.npy"), want)


def _dying_worker(rank, world, port, out_dir):
    """Rank 1 exits before the gather (a rank that never reports); rank 0's gather must end with an
    error instead of waiting forever."""
    import time
    import torch.distributed as dist
    from datetime import timedelta
    from simdonnx_b200.replicas import run_shards
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        os._exit(0)  # leaves without a collective step
    t0 = time.time()
    try:
        run_shards(lambda: np.zeros((1, 2), np.float32), dist)
        outcome = "returned"
    except Exception as e:  # the process group's error
        outcome = type(e).__name__
    with open(os.path.join(out_dir, "outcome.txt"), "w") as fh:
        fh.write(f"{outcome} {time.time() - t0:.1f}")
    os._exit(0)


def test_rank_that_dies_ends_the_gather_with_an_error(tmp_path):
    ctx = mp.start_processes(_dying_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=False,
                             start_method="spawn")
    import time
    deadline = time.time() + 60
    while not ctx.join(timeout=1):
        assert time.time() < deadline, "rank 0 did not finish"
    outcome, secs = (tmp_path / "outcome.txt").read_text().split()
    assert outcome != "returned"
    assert float(secs) < 30
