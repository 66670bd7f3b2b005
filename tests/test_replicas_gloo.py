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
