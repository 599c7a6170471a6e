"""Per-read sharding: the reference partition (golden cases generated from
sigcomp/read_assignment.py by tests/golden/make_golden.py) and the byte-count
exchange of a sharded compression, run as gloo ranks on the CPU."""

import json
import os
import struct

import numpy as np
import pytest

from sigcomp_b200.sharding import compress_shard, sample_balanced_ranges, shard_offsets


def test_partition_matches_reference_golden(golden):
    d = json.loads((golden / "sharding.json").read_text())
    assert len(d["cases"]) > 20
    for case in d["cases"]:
        got = sample_balanced_ranges(case["counts"], case["workers"])
        assert [[r.start, r.stop, r.num_samples] for r in got] == case["ranges"], case["counts"][:8]


def test_partition_errors_match_reference(golden):
    d = json.loads((golden / "sharding.json").read_text())
    for case in d["errors"]:
        with pytest.raises(ValueError, match=case["error"]):
            sample_balanced_ranges(case["counts"], case["workers"])


def test_partition_properties():
    rng = np.random.default_rng(3)
    for workers in (1, 2, 5, 8, 64):
        counts = rng.integers(2000, 10 ** 6, size=int(rng.integers(1, 300)))
        ranges = sample_balanced_ranges(counts.tolist(), workers)
        assert len(ranges) == min(workers, len(counts))
        assert ranges[0].start == 0 and ranges[-1].stop == len(counts)
        assert all(a.stop == b.start and a.stop > a.start for a, b in zip(ranges, ranges[1:]))
        assert sum(r.num_samples for r in ranges) == int(counts.sum())


def test_shard_offsets():
    assert shard_offsets([]) == ([], 0)
    assert shard_offsets([5, 0, 7], base=10) == ([10, 15, 15], 22)


class _FakeCodec:
    """Stands in for the device codec: a deterministic record per read."""

    def batch_inference_reads(self, list_of_reads=None, batch_size=64):
        return [struct.pack("<I", len(r)) + np.asarray(r, np.uint8)[::3].tobytes() for r in list_of_reads]


def _reads(n=23, seed=5):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, 256, size=int(k)).astype(np.uint8) for k in rng.integers(1, 5000, size=n)]


def _rank_main(rank, world, port, out_dir, n_reads):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        shard = compress_shard(_FakeCodec(), _reads(n_reads), rank=rank, world=world)
        with open(os.path.join(out_dir, f"rank{rank}.json"), "w") as f:
            json.dump({"start": shard.reads.start, "stop": shard.reads.stop, "offset": shard.byte_offset,
                       "total": shard.total_bytes, "sizes": shard.rank_bytes,
                       "data": b"".join(shard.records).hex()}, f)
    finally:
        dist.destroy_process_group()


def _free_port():
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world,n_reads", [(2, 23), (3, 2)])
def test_sharded_compress_reassembles_single_process_output(tmp_path, world, n_reads):
    import torch.multiprocessing as mp
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path), n_reads), nprocs=world,
                       start_method="spawn", join=True)
    whole = b"".join(_FakeCodec().batch_inference_reads(_reads(n_reads)))
    region = bytearray(len(whole))
    seen = []
    for r in range(world):
        d = json.loads((tmp_path / f"rank{r}.json").read_text())
        data = bytes.fromhex(d["data"])
        assert d["total"] == len(whole) and len(d["sizes"]) == world and d["sizes"][r] == len(data)
        region[d["offset"]:d["offset"] + len(data)] = data
        seen.append((d["start"], d["stop"]))
    assert bytes(region) == whole
    assert seen[0][0] == 0 and max(s[1] for s in seen) == n_reads
    if n_reads < world:   # ranks without reads still join the exchange, with an empty shard
        assert seen[-1][0] == seen[-1][1] == n_reads


def _rank_dies_main(rank, world, port, out_dir):
    """Rank 1 leaves before the byte-count exchange; rank 0 must get an error, not hang."""
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    if rank == 1:
        os._exit(0)                       # dies without taking part in the collective
    try:
        compress_shard(_FakeCodec(), _reads(7), rank=rank, world=world)
        outcome = "completed"
    except Exception as e:                # gloo reports the lost peer or the timeout
        outcome = "error: " + type(e).__name__
    with open(os.path.join(out_dir, "rank0.txt"), "w") as f:
        f.write(outcome)
    os._exit(0)


def test_lost_rank_is_reported_to_the_others(tmp_path):
    import torch.multiprocessing as mp
    ctx = mp.start_processes(_rank_dies_main, args=(2, _free_port(), str(tmp_path)), nprocs=2,
                             start_method="spawn", join=False)
    import time
    deadline = time.time() + 120
    while not ctx.join(timeout=5) and time.time() < deadline:
        pass
    for p in ctx.processes:
        if p.is_alive():
            p.kill()
    outcome = (tmp_path / "rank0.txt").read_text()
    assert outcome.startswith("error"), outcome
