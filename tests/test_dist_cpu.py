"""Multi-rank host logic on CPU (gloo, world sizes 2 and 3): the surfel-range
sharding of the RVQ decode, the all-gather of decoded rows, and the camera
partition. The GPU path uses the same code with NCCL."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from nest_b200 import synth
from nest_b200.views import DecodeRing, DecodeShard, camera_share, shard_range


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _decode_cpu(idx, cb, out):
    from oracle import oracle
    out.copy_(oracle.rvq_decode_torch(idx, cb))
    return out


def _worker(rank, world, port, n, result_dir):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    for p in (os.path.join(here, "..", "nest-splatting_b200"), os.path.join(here, "..")):
        sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        cb, idx = synth.config0(n=n, seed=7)
        sh = DecodeShard.create(idx, cb.shape[2], world, rank)
        full = sh.decode_and_gather(cb, _decode_cpu).clone()
        sh.dec_full.zero_()
        alt = sh.gather_indices_and_decode(cb, _decode_cpu)
        # DecodeRing (CPU: in order): frames alternate between two buffers.
        ring = DecodeRing(idx, cb.shape[2], world, rank)
        for i in range(3):
            ring.prefetch(i, cb, _decode_cpu)
            got = ring.acquire(i)
            assert got.data_ptr() == ring.shards[i % 2].decoded.data_ptr()
            assert torch.equal(got, full)
            ring.release(i)
        # The frame's exchange: every column decoded, the 10 geometric ones gathered.
        sh10 = DecodeShard.create(idx, cb.shape[2], world, rank, columns=synth.BASE_DIMS)
        part = sh10.decode_and_gather(cb, _decode_cpu).clone()
        assert part.shape == (n, synth.BASE_DIMS) and sh10.dec_shard.shape[1] == cb.shape[2]
        sh10.dec_full.zero_()
        part_alt = sh10.gather_indices_and_decode(cb, _decode_cpu).clone()
        ring10 = DecodeRing(idx, cb.shape[2], world, rank, columns=synth.BASE_DIMS)
        for i in range(2):
            ring10.prefetch(i, cb, _decode_cpu)
            assert torch.equal(ring10.acquire(i), part)
            ring10.release(i)
        torch.save({"full": full, "alt": alt.clone(), "part": part, "part_alt": part_alt,
                    "views": camera_share(64, world, rank)}, os.path.join(result_dir, f"rank{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n", [(2, 10_001), (3, 7_000)])
def test_sharded_decode_all_gather_matches_full_decode(tmp_path, world, n):
    port = _free_port()
    mp.start_processes(_worker, args=(world, port, n, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    from oracle import oracle
    cb, idx = synth.config0(n=n, seed=7)
    ref = oracle.rvq_decode_np(idx.numpy(), cb.numpy())
    views = []
    for r in range(world):
        d = torch.load(tmp_path / f"rank{r}.pt")
        assert np.array_equal(d["full"].numpy().view(np.uint32), ref.view(np.uint32))
        assert np.array_equal(d["alt"].numpy().view(np.uint32), ref.view(np.uint32))
        sub = np.ascontiguousarray(ref[:, : synth.BASE_DIMS])
        assert np.array_equal(d["part"].numpy().view(np.uint32), sub.view(np.uint32))
        assert np.array_equal(d["part_alt"].numpy().view(np.uint32), sub.view(np.uint32))
        views += d["views"]
    assert sorted(views) == list(range(64))


def test_shard_ranges_partition_surfels():
    for P in (1, 7, 1000, 1_000_000):
        for world in (1, 2, 3, 4, 8):
            covered = []
            for r in range(world):
                lo, hi = shard_range(P, world, r)
                assert 0 <= lo <= hi <= P
                covered += list(range(lo, hi)) if P < 2000 else [lo, hi]
            if P < 2000:
                assert covered == list(range(P))


def test_camera_share_balanced():
    for n in (1, 5, 64):
        for world in (1, 2, 4, 8):
            sizes = [len(camera_share(n, world, r)) for r in range(world)]
            assert sum(sizes) == n and max(sizes) - min(sizes) <= 1
