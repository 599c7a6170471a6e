"""Read-record serialisation against the reference writer / reader / index
format (golden vectors from sigcomp/main.py:549-590 and archive_shards.py:22,
see tests/golden/make_golden.py), and the offset-scan merge: gloo ranks write
their record regions at their offsets into one file."""

import json
import os

import numpy as np
import pytest

from sigcomp_b200.records import REC_FMT, index_bytes, pack_records, parse_records, write_region_at


def _golden(golden):
    z = np.load(golden / "records.npz")

    def split(flat, off):
        return [flat[off[i]:off[i + 1]].tobytes() for i in range(len(off) - 1)]

    recs = split(z["rec"], z["rec_off"])
    s, l, p = split(z["s"], z["s_off"]), split(z["l"], z["l_off"]), split(z["p"], z["p_off"])
    meta = z["meta"]
    return z, recs, meta, s, l, p


def test_pack_matches_reference_writer(golden):
    z, recs, meta, s, l, p = _golden(golden)
    region, offsets = pack_records(recs, meta[:, 0], meta[:, 1], meta[:, 2], s, l, p)
    assert region == z["region"].tobytes()
    assert offsets[-1] == len(region)


def test_parse_matches_reference_reader(golden):
    z, recs, meta, s, l, p = _golden(golden)
    parsed = parse_records(z["region"].tobytes())
    assert [(r["sig0"], r["N"], r["c_small"], r["c_large"]) for r in parsed] == [tuple(x) for x in z["parsed"]]
    assert [r["s_bytes"] for r in parsed] == s and [r["p_bytes"] for r in parsed] == p
    with pytest.raises(ValueError):
        parse_records(z["region"].tobytes()[:-1])


def test_index_matches_reference_format(golden):
    z, recs, meta, s, l, p = _golden(golden)
    _, offsets = pack_records(recs, meta[:, 0], meta[:, 1], meta[:, 2], s, l, p)
    got = index_bytes([r[:16] for r in recs], offsets[:-1], data_start=int(z["index_base"][0]))
    assert got == z["index"].tobytes()


def _merge_main(rank, world, port, path, sizes_file):
    import torch.distributed as dist
    from sigcomp_b200.sharding import exchange_shard_bytes, sample_balanced_ranges, shard_offsets
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(2)
        n_reads = 29
        blobs = [rng.bytes(int(k)) for k in rng.integers(0, 700, size=n_reads)]
        ranges = sample_balanced_ranges([len(b) + 1 for b in blobs], world)
        mine = ranges[rank]
        recs = [bytes([i]) * 16 + bytes(REC_FMT.size - 16) for i in range(mine.start, mine.stop)]
        k = mine.stop - mine.start
        region, _ = pack_records(recs, [i for i in range(k)], [1000 + i for i in range(k)], [i for i in range(k)],
                                 blobs[mine.start:mine.stop], [b""] * k, [b"x"] * k)
        sizes = exchange_shard_bytes(len(region))
        starts, total = shard_offsets(sizes, base=8)           # after an 8-byte stand-in header
        write_region_at(path, starts[rank], region)
        if rank == 0:
            write_region_at(path, 0, b"HEADER00")
            with open(sizes_file, "w") as f:
                json.dump({"total": total}, f)
    finally:
        dist.destroy_process_group()


def _free_port():
    import socket
    with socket.socket() as s_:
        s_.bind(("127.0.0.1", 0))
        return s_.getsockname()[1]


def test_ranks_write_their_regions_into_one_archive(tmp_path):
    import torch.multiprocessing as mp
    path = str(tmp_path / "archive.bin")
    mp.start_processes(_merge_main, args=(3, _free_port(), path, str(tmp_path / "total.json")), nprocs=3,
                       start_method="spawn", join=True)
    # single-process region of the same reads
    rng = np.random.default_rng(2)
    blobs = [rng.bytes(int(k)) for k in rng.integers(0, 700, size=29)]
    from sigcomp_b200.sharding import sample_balanced_ranges
    parts = []
    for r in sample_balanced_ranges([len(b) + 1 for b in blobs], 3):
        k = r.stop - r.start
        recs = [bytes([i]) * 16 + bytes(REC_FMT.size - 16) for i in range(r.start, r.stop)]
        parts.append(pack_records(recs, list(range(k)), [1000 + i for i in range(k)], list(range(k)),
                                  blobs[r.start:r.stop], [b""] * k, [b"x"] * k)[0])
    data = open(path, "rb").read()
    assert data == b"HEADER00" + b"".join(parts)
    assert json.loads((tmp_path / "total.json").read_text())["total"] == len(data)
